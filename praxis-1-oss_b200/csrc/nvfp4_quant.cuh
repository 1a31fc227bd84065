// NVFP4 quantization helpers shared by the quantize kernels and the FP4
// epilogue of the gate/up GEMM: the reference recipe
// (praxis/kernels/nvfp4.py:44-124) per 16 values, with the division-free
// scale path (bit-identical) and the compact 128x4 scale-atom layout
// (praxis/kernels/nvfp4.py:114-119).
#pragma once

#include "common.cuh"

namespace praxis {

constexpr float kOneSixth = 0.16666667163372040f;  // f32(1/6)

__device__ __forceinline__ uint32_t sf_offset(int64_t row, int col, int kb) {
  return (uint32_t)(((row >> 7) * (kb >> 2) + (col >> 2)) * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4 +
                    (col & 3));
}

__device__ __forceinline__ float clamp6(float x) { return fminf(fmaxf(x, -6.0f), 6.0f); }

// Eight floats -> eight E2M1 codes in one word (element 0 in the low nibble).
__device__ __forceinline__ uint32_t e2m1x8(float2 a, float2 b, float2 c, float2 d) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y), "f"(d.x), "f"(d.y));
  return out;
}

// The scale and reciprocal of one 16-block without the two IEEE divisions
// of the recipe (bit-identical results):
//  * sf = e4m3(clamp(div_rn(bs, g), 2^-6, 448)). q = bs * inv_g (inv_g =
//    div_rn(1, g)) is within 3 f32 ulps of div_rn(bs, g); both round to the
//    same e4m3 byte unless an e4m3 rounding midpoint (the 20 bits e4m3 drops
//    = 0x80000) lies between them, so q is used unless its dropped bits are
//    within 16 ulps of a midpoint, where the division decides. Outside the
//    normal range both sides clamp alike (2^-6 and 448 are e4m3 values far
//    from any midpoint; a tiny or overflowing q clamps to the same bound).
//  * rc = div_rn(inv_g, sf). sf = 2^(E-7) * (1 + m/8) (E = byte >> 3 >= 1
//    after the clamp, m = byte & 7), so rc = 2^(7-E) * div_rn(inv_g, 1 + m/8)
//    exactly while the result stays normal, which it does for every global
//    scale the recipe produces (inv_g in [7.9e-36, 2.7e15], 2^(7-E) in
//    [2^-8, 2^6]). recip8[m] = div_rn(inv_g, 1 + m/8) is computed once per
//    global scale.
__device__ __forceinline__ float recip8_entry(float inv_g, int m) { return div_rn(inv_g, 1.0f + 0.125f * (float)m); }

// bs = mul_rn(amax, f32(1/6)), the block's scale before the global one (the
// same for every global scale a block is quantized with).
__device__ __forceinline__ void quantize16_bs(const float (&v)[16], float bs, float g, float inv_g,
                                              const float* recip8, bool has_nan, uint32_t& lo, uint32_t& hi,
                                              uint32_t& sf) {
  float qv = mul_rn(bs, inv_g);
  const uint32_t dropped = __float_as_uint(qv) & 0xFFFFFu;
  if (has_nan || dropped - (0x80000u - 16u) <= 32u) qv = div_rn(bs, g);
  sf = f32_to_e4m3_byte(fminf(fmaxf(qv, 0.015625f), 448.0f));
  const float rc = __int_as_float(__float_as_int(recip8[sf & 7u]) - ((int)(sf >> 3) - 7) * (1 << 23));
  const float2 rc2 = make_float2(rc, rc);
  float2 n[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) n[i] = mul2_rn(make_float2(v[2 * i], v[2 * i + 1]), rc2);
  if (has_nan) {
#pragma unroll
    for (int i = 0; i < 8; ++i) n[i] = make_float2(clamp6(n[i].x), clamp6(n[i].y));
  }
  lo = e2m1x8(n[0], n[1], n[2], n[3]);
  hi = e2m1x8(n[4], n[5], n[6], n[7]);
}

__device__ __forceinline__ void quantize16_fast(const float (&v)[16], float amax, float g, float inv_g,
                                                const float* recip8, bool has_nan, uint32_t& lo, uint32_t& hi,
                                                uint32_t& sf) {
  quantize16_bs(v, mul_rn(amax, kOneSixth), g, inv_g, recip8, has_nan, lo, hi, sf);
}

// Byte offset of row `row`'s scale of k-block 0 in the compact layout; the
// scale of 16-block j then sits at + (j >> 2) * 512 + (j & 3).
__device__ __forceinline__ int64_t sf_row_base(int64_t row, int kb) {
  return ((row >> 7) * (kb >> 2)) * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4;
}

// 16 bf16 values held as 8 words -> floats, their max |v| and whether any
// is not finite, the maximum taken on the magnitude bits (for finite bf16
// values the unsigned order of the magnitude bits is the order of |v|;
// blocks holding an infinity or NaN recompute it NaN-ignoring, as the
// reference's max).
__device__ __forceinline__ void unpack16_bf16(const uint32_t (&w)[8], float (&v)[16], float& amax, bool& has_nan) {
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    uint32_t r;
    asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(m), "r"(w[i] & 0x7FFF7FFFu));
    m = r;
  }
  const uint32_t hi = m >> 16, lo = m & 0xFFFFu;
  has_nan = hi >= 0x7F80u || lo >= 0x7F80u;
  amax = __uint_as_float((hi > lo ? hi : lo) << 16);
  if (has_nan) {
    amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
}

// The same for 16 bf16 values read from global memory (32 bytes, aligned).
__device__ __forceinline__ void load16_bf16_fast(const uint16_t* src, float (&v)[16], float& amax, bool& has_nan) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  const uint4 a = __ldg(s), b = __ldg(s + 1);
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  unpack16_bf16(w, v, amax, has_nan);
}

}  // namespace praxis
