// Stand-alone rescale + SwiGLU + row max over a padded gate/up GEMM output.
//
// Replaces praxis/kernels/nvfp4_moe.py:102-158 (rescale_swiglu_maximum): row r
// of the padded rows belongs to expert e (the pcsr segment holding it, rows
// past the end to the last expert); m = bf16(g_a[e] * g_w[e]);
// gate = bf16(raw[r, :F] * m), up = bf16(raw[r, F:] * m),
// h = bf16(bf16(gate * sigmoid(gate)) * up), rowmax[r] = bf16(max |h|).
// The fused GEMM epilogue computes the same element two columns at a time
// with swiglu_pair (paired fp32 arithmetic, refined reciprocal); `alu`
// selects that implementation (1) or the scalar IEEE-division one (0), so the
// two can be compared on every input.
#include "common.cuh"
#include "kernels.h"

namespace praxis {

__device__ __forceinline__ int expert_of_row(const int32_t* __restrict__ csr, int experts, int64_t row) {
  int lo = 0, hi = experts;  // number of experts whose end <= row
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if ((int64_t)csr[mid + 1] <= row) lo = mid + 1;
    else hi = mid;
  }
  return lo < experts ? lo : experts - 1;
}

template <bool kAlu>
__global__ void __launch_bounds__(256) rescale_swiglu_kernel(
    const uint16_t* __restrict__ raw, int64_t rows, int hidden, const int32_t* __restrict__ pcsr, int experts,
    const float* __restrict__ act_global, const float* __restrict__ w_global, uint16_t* __restrict__ out,
    uint16_t* __restrict__ rowmax) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= rows) return;
  const int e = expert_of_row(pcsr, experts, r);
  const float mult = bf16_round(mul_rn(act_global[e], w_global[e]));
  const uint16_t* gr = raw + r * 2 * hidden;
  float m = 0.0f;
  if constexpr (kAlu) {
    for (int c = 2 * lane; c < hidden; c += 64) {  // hidden is even
      const uint32_t h = swiglu_pair(bf16_to_f32(gr[c]), bf16_to_f32(gr[c + 1]), bf16_to_f32(gr[hidden + c]),
                                     bf16_to_f32(gr[hidden + c + 1]), mult);
      *reinterpret_cast<uint32_t*>(out + r * hidden + c) = h;
      m = fmaxf(m, fmaxf(fabsf(__uint_as_float(h << 16)), fabsf(__uint_as_float(h & 0xFFFF0000u))));
    }
  } else {
    for (int c = lane; c < hidden; c += 32) {
      const float g = bf16_to_f32(gr[c]);
      const float u = bf16_to_f32(gr[hidden + c]);
      const float h = swiglu_element<false>(g, u, mult);
      out[r * hidden + c] = (uint16_t)(__float_as_uint(h) >> 16);
      m = fmaxf(m, fabsf(h));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0 && rowmax != nullptr) rowmax[r] = (uint16_t)(__float_as_uint(m) >> 16);
}

int run_rescale_swiglu(const uint16_t* raw, int64_t rows, int hidden, const int32_t* pcsr, int experts,
                       const float* act_global, const float* w_global, uint16_t* out, uint16_t* rowmax, int alu,
                       cudaStream_t stream) {
  if (hidden <= 0 || hidden % 2 || experts <= 0) return set_error(PRAXIS_B200_EINVAL, "rescale_swiglu: bad sizes");
  if (rows == 0) return PRAXIS_B200_OK;
  const int64_t blocks = (rows + 7) / 8;
  if (alu)
    rescale_swiglu_kernel<true><<<(unsigned)blocks, 256, 0, stream>>>(raw, rows, hidden, pcsr, experts, act_global,
                                                                       w_global, out, rowmax);
  else
    rescale_swiglu_kernel<false><<<(unsigned)blocks, 256, 0, stream>>>(raw, rows, hidden, pcsr, experts,
                                                                        act_global, w_global, out, rowmax);
  return check_launch("rescale_swiglu");
}

}  // namespace praxis
