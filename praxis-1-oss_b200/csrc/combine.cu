// Weighted combine of the routed rows back to tokens (+ shared expert).
//
// Replaces praxis/kernels/nvfp4_moe.py:206-311 (_rescale_combine), the same
// arithmetic in the same order, without FMA contraction:
//   per token t and slot s: i = inverse[t*k+s], e = top[t,s],
//   src = pcsr[e] + i - csr[e]
//   v = bf16(raw[src] * bf16(g_h[e] * g_w[e]))   (skipped when the down GEMM
//                                                  epilogue already did it)
//   acc[s % 4] += v * (f32(gate[t,s]) * f32(scaling))
//   y = bf16(((acc0 + acc1) + acc2) + acc3);  y = bf16(y + shared)
// One warp per token, 16-byte gathers of the routed rows.
#include "common.cuh"
#include "kernels.h"

namespace praxis {

// KMAX: slots held per lane (top_k <= KMAX); U: 8-column chunks per lane per
// pass, so that KMAX * U 16-byte loads are in flight per lane.
template <int KMAX, int U>
__global__ void __launch_bounds__(256) combine_kernel(
    const uint16_t* __restrict__ rows, int cols, const int64_t* __restrict__ inverse,
    const int64_t* __restrict__ top_idx, const uint16_t* __restrict__ gate, const int32_t* __restrict__ csr,
    const int32_t* __restrict__ pcsr, const float* __restrict__ h_global, const uint32_t* __restrict__ h_amax,
    const float* __restrict__ w_global, int rows_rescaled, float scaling, const uint16_t* __restrict__ shared,
    uint16_t* __restrict__ out, int64_t tokens, int top_k, int experts, Passes passes) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  __shared__ int64_t s_src[8][8];
  __shared__ float s_scale[8][8], s_mult[8][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 8 + warp;
  if (t >= tokens) return;
  if (lane < top_k) {
    const int64_t p = t * top_k + lane;
    const int e = checked_expert(top_idx[p], experts), g = route_group(e, t, passes);
    s_src[warp][lane] = (int64_t)pcsr[g] + inverse[p] - csr[g];
    s_scale[warp][lane] = mul_rn(bf16_to_f32(gate[p]), scaling);
    float mult = 1.0f;
    if (!rows_rescaled) {
      const float gh = h_global != nullptr ? h_global[g] : global_from_amax_bits(h_amax[g]);
      mult = bf16_round(mul_rn(gh, w_global[e]));
    }
    s_mult[warp][lane] = mult;
  }
  __syncwarp();
  // U 8-column chunks per lane per pass: every routed-row load of the pass
  // is issued before any arithmetic (U * top_k 16-byte loads in flight).
  for (int c0 = lane * 8; c0 < cols; c0 += 256 * U) {
    uint4 v[U][KMAX];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * 256;
#pragma unroll
      for (int s = 0; s < KMAX; ++s)
        if (s < top_k && c < cols) v[u][s] = ldg_stream(reinterpret_cast<const uint4*>(rows + s_src[warp][s] * cols + c));
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * 256;
      if (c >= cols) break;
      // column pairs (2j, 2j+1) in paired fp32 arithmetic, same operations
      // and order per element as the scalar form
      float2 acc[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[a][j] = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int s = 0; s < KMAX; ++s) {
        if (s < top_k) {
          const uint32_t wv[4] = {v[u][s].x, v[u][s].y, v[u][s].z, v[u][s].w};
          const float2 sc = make_float2(s_scale[warp][s], s_scale[warp][s]);
          const float mult = s_mult[warp][s];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 val = rows_rescaled ? unpack_bf16x2(wv[j]) : unpack_bf16x2(rescale_pair(
                                                                          __uint_as_float(wv[j] << 16),
                                                                          __uint_as_float(wv[j] & 0xFFFF0000u), mult));
            acc[s & 3][j] = add2_rn(acc[s & 3][j], mul2_rn(val, sc));
          }
        }
      }
      uint4 sh = make_uint4(0, 0, 0, 0);
      if (shared != nullptr) sh = ldg_stream(reinterpret_cast<const uint4*>(shared + t * cols + c));
      const uint32_t shv[4] = {sh.x, sh.y, sh.z, sh.w};
      uint32_t packed[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 sum = add2_rn(add2_rn(add2_rn(acc[0][j], acc[1][j]), acc[2][j]), acc[3][j]);
        packed[j] = cvt_bf16x2(sum.x, sum.y);
        if (shared != nullptr) {
          const float2 y = add2_rn(unpack_bf16x2(packed[j]), unpack_bf16x2(shv[j]));
          packed[j] = cvt_bf16x2(y.x, y.y);
        }
      }
      *reinterpret_cast<uint4*>(out + t * cols + c) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
  }
}

int run_combine(const uint16_t* rows, int cols, const int64_t* inverse, const int64_t* top_idx, const uint16_t* gate,
                const int32_t* csr, const int32_t* pcsr, const float* h_global, const uint32_t* h_amax,
                const float* w_global, int rows_rescaled, float scaling, const uint16_t* shared, uint16_t* out,
                int64_t tokens, int top_k, int experts, cudaStream_t stream, Passes passes) {
  if (cols % 8 != 0) return set_error(PRAXIS_B200_EINVAL, "combine needs C %% 8 == 0");
  if (top_k < 1 || top_k > 8) return set_error(PRAXIS_B200_EINVAL, "top_k must be 1..8");
  if (!rows_rescaled && (w_global == nullptr || (h_global == nullptr && h_amax == nullptr)))
    return set_error(PRAXIS_B200_EINVAL, "combine needs global scales to rescale raw rows");
  if (tokens == 0) return PRAXIS_B200_OK;
  const int64_t blocks = (tokens + 7) / 8;
  // eight 16-byte loads in flight per lane for every top_k
#define PRAXIS_COMBINE(KMAX, U)                                                                                    \
  launch_pdl(combine_kernel<KMAX, U>, dim3((unsigned)blocks), dim3(256), 0, stream, rows, cols, inverse, top_idx, gate, \
             csr, pcsr, h_global, h_amax, w_global, rows_rescaled, scaling, shared, out, tokens, top_k, experts,  \
             passes)
  if (top_k == 1) PRAXIS_COMBINE(1, 8);
  else if (top_k == 2) PRAXIS_COMBINE(2, 4);
  else if (top_k <= 4) PRAXIS_COMBINE(4, 2);
  else PRAXIS_COMBINE(8, 1);
#undef PRAXIS_COMBINE
  return check_launch("combine");
}

}  // namespace praxis
