// The MoE tail fused into what follows it: the next block's residual add +
// RMSNorm (optionally with its modulation), or the residual add alone.
//
// Replaces praxis/kernels/moe_tail_triton.py:99-194 (_tail_add_norm_scale),
// :196-307 (_tail_add_mod_norm_scale) and :401-445 (_tail_residual_add), NVFP4
// one-chunk mode, with their contract (praxis/kernels/norm_triton.py:1-32,
// praxis/layers.py:429-441): the routed combine of rescale_combine and the
// shared add give y (bf16, never stored), then
//   xo = bf16(f32(x) + f32(y))                          (the residual add)
//   MOD: xo = bf16(fma(f32(xo), bf16(f32(scl) + 1), f32(shf)))
//        (without mod_fma: the product rounded to fp32 first)
//   ss = sum of f32(xo)^2 in the order of torch's vectorized RMSNorm kernel:
//        one 128-thread row, thread t = 32 w + l adds the squares of the four
//        elements of float4 vectors t, t + 128, ... to its own sum in order,
//        a shuffle-down tree (16, 8, 4, 2, 1) per warp, then
//        (w0 + w2) + (w1 + w3)
//   r  = rsqrt(ss / N + eps)   (IEEE division; the hardware reciprocal
//                                square root, as torch's and Triton's rsqrt)
//   h  = bf16(bf16(w1 * (r * f32(xo))) * s)            (w1 = 1 + weight, fp32)
// with no FMA contraction outside the modulation. One warp per token emulates
// the four warps of the row: lane l keeps one sum per emulated warp w for the
// elements 512 i + 128 w + 4 l + e.
#include "common.cuh"
#include "kernels.h"

namespace praxis {

__device__ __forceinline__ float rsqrt_hw(float v) {
  float r;
  asm("rsqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

// Four consecutive bf16 (8 bytes) of a row, read once.
__device__ __forceinline__ uint2 ldg_stream8(const uint16_t* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

// The modulation row of token row `row` (praxis/kernels/norm_triton.py:417-431):
// batch row / RF holds RF token rows [NREG | (f, y, i, x, j)] and RC modulation
// rows [NREG | (f, y, x)] (i < PH, j < PW, x < WD); {1, 1, 0, 1, 1, 1} maps
// every row to itself.
__device__ __forceinline__ int64_t mod_row(int64_t row, const int64_t* g) {
  const int64_t rf = g[0], rc = g[1], nreg = g[2], pw = g[3], wd = g[4], ph = g[5];
  const int64_t b = row / rf, t = row - b * rf;
  const int64_t u = t - nreg > 0 ? t - nreg : 0;
  const int64_t q = u / pw;
  const int64_t xx = q % wd, fy = (q / wd) / ph;
  return b * rc + (t < nreg ? t : nreg + fy * wd + xx);
}

// NORM: residual add + RMSNorm (else the residual add alone); MOD: the
// modulation between them.
template <int KMAX, bool NORM, bool MOD>
__global__ void __launch_bounds__(256) combine_tail_kernel(
    const uint16_t* __restrict__ rows, int cols, const int64_t* __restrict__ inverse,
    const int64_t* __restrict__ top_idx, const uint16_t* __restrict__ gate, const int32_t* __restrict__ csr,
    const int32_t* __restrict__ pcsr, const float* __restrict__ h_global, const uint32_t* __restrict__ h_amax,
    const float* __restrict__ w_global, int rows_rescaled, float scaling, const uint16_t* __restrict__ shared,
    TailArgs tail, int64_t tokens, int top_k, int experts, Passes passes) {
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
  const uint16_t* xr = tail.x + t * cols;
  uint16_t* xor_ = tail.x_out + t * cols;
  const uint16_t* mr = nullptr;
  if constexpr (MOD) mr = tail.mod + mod_row(t + tail.mod_row0, tail.mod_geom) * 2 * cols;
  float acc_sq[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // the sums of emulated warps 0..3 at lane `lane`
  for (int c0 = 0; c0 < cols; c0 += 512) {
    // every load of the 512-column chunk first: 4 vectors per slot per lane,
    // and the residual, shared and modulation vectors of the same columns
    uint2 v[KMAX][4];
    uint2 xq[4], shq[4], mshq[4], mscq[4];
#pragma unroll
    for (int s = 0; s < KMAX; ++s)
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const int c = c0 + 128 * w + 4 * lane;
        if (s < top_k && c < cols) v[s][w] = ldg_stream8(rows + s_src[warp][s] * cols + c);
      }
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int c = c0 + 128 * w + 4 * lane;
      xq[w] = shq[w] = mshq[w] = mscq[w] = make_uint2(0, 0);
      if (c < cols) {
        xq[w] = ldg_stream8(xr + c);
        if (shared != nullptr) shq[w] = ldg_stream8(shared + t * cols + c);
        if constexpr (MOD) {
          mshq[w] = *reinterpret_cast<const uint2*>(mr + c);
          mscq[w] = *reinterpret_cast<const uint2*>(mr + cols + c);
        }
      }
    }
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int c = c0 + 128 * w + 4 * lane;
      if (c >= cols) continue;
      // the combine (rescale_combine's arithmetic and order) on columns c..c+3
      float2 acc[4][2];
#pragma unroll
      for (int a = 0; a < 4; ++a) acc[a][0] = acc[a][1] = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int s = 0; s < KMAX; ++s) {
        if (s < top_k) {
          const uint32_t wv[2] = {v[s][w].x, v[s][w].y};
          const float2 sc = make_float2(s_scale[warp][s], s_scale[warp][s]);
          const float mult = s_mult[warp][s];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const float2 val = rows_rescaled ? unpack_bf16x2(wv[j]) : unpack_bf16x2(rescale_pair(
                                                                          __uint_as_float(wv[j] << 16),
                                                                          __uint_as_float(wv[j] & 0xFFFF0000u), mult));
            acc[s & 3][j] = add2_rn(acc[s & 3][j], mul2_rn(val, sc));
          }
        }
      }
      const uint32_t xw[2] = {xq[w].x, xq[w].y}, shw[2] = {shq[w].x, shq[w].y};
      const uint32_t mshw[2] = {mshq[w].x, mshq[w].y}, mscw[2] = {mscq[w].x, mscq[w].y};
      uint32_t xo[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float2 sum = add2_rn(add2_rn(add2_rn(acc[0][j], acc[1][j]), acc[2][j]), acc[3][j]);
        uint32_t y = cvt_bf16x2(sum.x, sum.y);
        if (shared != nullptr) {
          const float2 ys = add2_rn(unpack_bf16x2(y), unpack_bf16x2(shw[j]));
          y = cvt_bf16x2(ys.x, ys.y);
        }
        const float2 r = add2_rn(unpack_bf16x2(xw[j]), unpack_bf16x2(y));
        xo[j] = cvt_bf16x2(r.x, r.y);
        if constexpr (MOD) {
          const float2 xf = unpack_bf16x2(xo[j]), shf = unpack_bf16x2(mshw[j]), scf = unpack_bf16x2(mscw[j]);
          const float s1x = bf16_round(add_rn(scf.x, 1.0f)), s1y = bf16_round(add_rn(scf.y, 1.0f));
          float mx, my;
          if (tail.mod_fma) {
            mx = __fmaf_rn(xf.x, s1x, shf.x);
            my = __fmaf_rn(xf.y, s1y, shf.y);
          } else {
            mx = add_rn(mul_rn(xf.x, s1x), shf.x);
            my = add_rn(mul_rn(xf.y, s1y), shf.y);
          }
          xo[j] = cvt_bf16x2(mx, my);
        }
      }
      *reinterpret_cast<uint2*>(xor_ + c) = make_uint2(xo[0], xo[1]);
      if constexpr (NORM) {
        // squares of the four elements in order (exact in fp32 for bf16 values)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float2 f = unpack_bf16x2(xo[j]);
          acc_sq[w] = add_rn(acc_sq[w], mul_rn(f.x, f.x));
          acc_sq[w] = add_rn(acc_sq[w], mul_rn(f.y, f.y));
        }
      }
    }
  }
  if constexpr (NORM) {
    // per emulated warp: the shuffle-down tree; then (w0 + w2) + (w1 + w3)
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc_sq[w] = add_rn(acc_sq[w], __shfl_down_sync(0xffffffffu, acc_sq[w], o));
    float ss = add_rn(add_rn(acc_sq[0], acc_sq[2]), add_rn(acc_sq[1], acc_sq[3]));
    ss = __shfl_sync(0xffffffffu, ss, 0);
    const float r = rsqrt_hw(add_rn(div_rn(ss, (float)cols), tail.eps));
    __syncwarp();  // this warp's residual stores above are read back below
    const float s = tail.norm_scale;
    uint16_t* hr = tail.h_out + t * cols;
    for (int c0 = 0; c0 < cols; c0 += 512) {
      // the chunk's residual (this warp's own stores above) and weight loads first
      uint2 xq[4];
      float4 wq[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const int c = c0 + 128 * w + 4 * lane;
        if (c < cols) {
          xq[w] = *reinterpret_cast<const uint2*>(xor_ + c);
          wq[w] = *reinterpret_cast<const float4*>(tail.w1 + c);
        }
      }
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const int c = c0 + 128 * w + 4 * lane;
        if (c >= cols) continue;
        const float2 x01 = unpack_bf16x2(xq[w].x), x23 = unpack_bf16x2(xq[w].y);
        const float o0 = bf16_round(mul_rn(wq[w].x, mul_rn(r, x01.x)));
        const float o1 = bf16_round(mul_rn(wq[w].y, mul_rn(r, x01.y)));
        const float o2 = bf16_round(mul_rn(wq[w].z, mul_rn(r, x23.x)));
        const float o3 = bf16_round(mul_rn(wq[w].w, mul_rn(r, x23.y)));
        *reinterpret_cast<uint2*>(hr + c) =
            make_uint2(cvt_bf16x2(mul_rn(o0, s), mul_rn(o1, s)), cvt_bf16x2(mul_rn(o2, s), mul_rn(o3, s)));
      }
    }
  }
}

int run_combine_tail(const uint16_t* rows, int cols, const int64_t* inverse, const int64_t* top_idx,
                     const uint16_t* gate, const int32_t* csr, const int32_t* pcsr, const float* h_global,
                     const uint32_t* h_amax, const float* w_global, int rows_rescaled, float scaling,
                     const uint16_t* shared, const TailArgs& tail, int64_t tokens, int top_k, int experts,
                     cudaStream_t stream, Passes passes) {
  if (cols % 4 != 0 || cols <= 0) return set_error(PRAXIS_B200_EINVAL, "combine_tail needs C %% 4 == 0");
  if (top_k < 1 || top_k > 8) return set_error(PRAXIS_B200_EINVAL, "top_k must be 1..8");
  if (!rows_rescaled && (w_global == nullptr || (h_global == nullptr && h_amax == nullptr)))
    return set_error(PRAXIS_B200_EINVAL, "combine_tail needs global scales to rescale raw rows");
  if (tail.x == nullptr || tail.x_out == nullptr)
    return set_error(PRAXIS_B200_EINVAL, "combine_tail needs the residual and its output");
  const bool norm = tail.w1 != nullptr, mod = tail.mod != nullptr;
  if (norm && tail.h_out == nullptr) return set_error(PRAXIS_B200_EINVAL, "combine_tail: the norm needs normed_out");
  if (mod && !norm) return set_error(PRAXIS_B200_EINVAL, "combine_tail: the modulation needs the norm");
  if (mod) {
    const int64_t* g = tail.mod_geom;
    if (g[0] <= 0 || g[1] <= 0 || g[2] < 0 || g[3] <= 0 || g[4] <= 0 || g[5] <= 0 || tail.mod_row0 < 0)
      return set_error(PRAXIS_B200_EINVAL, "combine_tail: bad modulation geometry");
  }
  if ((((uintptr_t)rows | (uintptr_t)tail.x | (uintptr_t)tail.x_out | (uintptr_t)tail.h_out | (uintptr_t)shared |
        (uintptr_t)tail.mod) & 7) ||
      ((uintptr_t)tail.w1 & 15))
    return set_error(PRAXIS_B200_EINVAL, "combine_tail: bf16 buffers 8-byte, the norm weight 16-byte aligned");
  if (tokens == 0) return PRAXIS_B200_OK;
  const int64_t blocks = (tokens + 7) / 8;
#define PRAXIS_TAIL(KMAX, NORM, MOD)                                                                               \
  launch_pdl(combine_tail_kernel<KMAX, NORM, MOD>, dim3((unsigned)blocks), dim3(256), 0, stream, rows, cols,       \
             inverse, top_idx, gate, csr, pcsr, h_global, h_amax, w_global, rows_rescaled, scaling, shared, tail,  \
             tokens, top_k, experts, passes)
#define PRAXIS_TAIL_K(NORM, MOD)          \
  if (top_k <= 2) PRAXIS_TAIL(2, NORM, MOD);      \
  else if (top_k <= 4) PRAXIS_TAIL(4, NORM, MOD); \
  else PRAXIS_TAIL(8, NORM, MOD);
  if (mod) {
    PRAXIS_TAIL_K(true, true)
  } else if (norm) {
    PRAXIS_TAIL_K(true, false)
  } else {
    PRAXIS_TAIL_K(false, false)
  }
#undef PRAXIS_TAIL_K
#undef PRAXIS_TAIL
  return check_launch("combine_tail");
}

}  // namespace praxis
