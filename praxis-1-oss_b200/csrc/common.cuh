// Shared device helpers for the sm_100a MoE kernels: bf16/fp8/fp4 element
// conversions, mbarriers with bounded waits, TMA and tcgen05 wrappers.
//
// Every wait on an mbarrier is bounded (wall-clock limit from %globaltimer):
// on expiry the waiting thread records a code in the device error word and
// returns false, so a kernel never hangs the GPU; the host reads the word at
// a sync point (praxis_b200_device_error).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/praxis_b200_moe.h"

namespace praxis {

// ---------------------------------------------------------------------------
// Device error word (one per device, cleared by the host after reading)
// ---------------------------------------------------------------------------
// Defined here: the library is one translation unit (praxis_b200_moe.cu).
__device__ unsigned int g_device_error = 0;

enum DeviceError : unsigned int {
  kErrNone = 0,
  kErrTimeoutProducer = 1,
  kErrTimeoutMma = 2,
  kErrTimeoutEpilogue = 3,
  kErrIndexRange = 4,
  kErrTimeoutPeer = 5,
};

__device__ __forceinline__ void record_error(unsigned int code) {
  atomicCAS(&g_device_error, 0u, code);
}

// Programmatic dependent launch. The hot-path kernels are launched with
// launch_pdl (kernels.h): a kernel's CTAs may be scheduled while the previous
// kernel of the stream is finishing, so its launch latency overlaps that
// kernel's tail. pdl_wait(), the first statement of each such kernel, blocks
// until the previous kernel has completed and its writes are visible (a no-op
// for a kernel launched without the attribute); pdl_trigger() lets the next
// kernel be scheduled once every CTA of this one has started.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ bool error_raised() {
  return *((volatile unsigned int*)&g_device_error) != 0u;
}

// ---------------------------------------------------------------------------
// Numeric helpers (explicit roundings; nothing here may be contracted)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
  return __uint_as_float(((uint32_t)b) << 16);
}

__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

__device__ __forceinline__ float bf16_round(float f) { return bf16_to_f32(f32_to_bf16(f)); }

// float -> e4m3 (RNE, satfinite) as a byte; input already clamped to [2^-6, 448].
__device__ __forceinline__ uint32_t f32_to_e4m3_byte(float f) {
  uint16_t pair;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(pair) : "f"(0.0f), "f"(f));
  return (uint32_t)(pair & 0xFFu);
}

// e4m3 byte -> float (exact).
__device__ __forceinline__ float e4m3_byte_to_f32(uint32_t b) {
  uint32_t h2;
  uint16_t in = (uint16_t)(b & 0xFFu);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(in));
  __half h = __ushort_as_half((unsigned short)(h2 & 0xFFFFu));
  return __half2float(h);
}

// Two floats -> one byte of two E2M1 codes: `lo` in bits 0-3, `hi` in 4-7
// (round to nearest even, satfinite).
__device__ __forceinline__ uint32_t f32x2_to_e2m1_byte(float lo, float hi) {
  uint32_t out;
  asm("{\n\t.reg .b8 b;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b, %1, %2;\n\t"
      "cvt.u32.u8 %0, b;\n\t}"
      : "=r"(out)
      : "f"(hi), "f"(lo));
  return out;
}

// 16-byte streaming load through the non-coherent path (read-once data).
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// IEEE round-to-nearest division and product/sum with no contraction.
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

// Triton's fp32 sigmoid as the reference's SwiGLU kernels compile it:
// 1 / (1 + ex2.approx(-x * log2 e)) with an IEEE division.
__device__ __forceinline__ float sigmoid_triton(float x) {
  float t = mul_rn(-x, 1.4426950408889634f);
  float e;
  asm("ex2.approx.f32 %0, %1;" : "=f"(e) : "f"(t));
  return div_rn(1.0f, add_rn(1.0f, e));
}

// e^x for x <= 0, the softmax router's exponential (x = logit - row max).
// Cody and Waite's range reduction (W. J. Cody, W. Waite, "Software Manual
// for the Elementary Functions", 1980): x = n ln2 + r with n = rint(x log2 e)
// and ln2 split as C1 + C2 (C1 = 355/512 has 9 significant bits, so n * C1 is
// exact for |n| <= 127), then e^r (|r| <= ln2 / 2) by its Taylor polynomial
// to degree 7 in Horner form (truncation below 2^-27 relative), then 2^n by
// exponent arithmetic. Every step is one IEEE-rounded float32 multiply or add
// with no contraction, so a float32 restatement on the CPU gives the same
// bits (the oracle's route(activation="softmax") does). Within 2 ulp of e^x;
// x < -87 gives 0 (below every softmax probability that can reach a top-k
// slot), NaN stays NaN.
__device__ __forceinline__ float exp_softmax(float x) {
  if (x != x) return x;
  if (x < -87.0f) return 0.0f;
  // float32 constants as exact hex literals: log2 e, C1, C2, 1/5040 .. 1/6
  const float n = rintf(__fmul_rn(x, 0x1.715476p+0f));
  float r = __fadd_rn(x, __fmul_rn(-n, 0x1.63p-1f));
  r = __fadd_rn(r, __fmul_rn(-n, -0x1.bd0106p-13f));
  float q = 0x1.a01a02p-13f;
  q = __fadd_rn(__fmul_rn(q, r), 0x1.6c16c2p-10f);
  q = __fadd_rn(__fmul_rn(q, r), 0x1.111112p-7f);
  q = __fadd_rn(__fmul_rn(q, r), 0x1.555556p-5f);
  q = __fadd_rn(__fmul_rn(q, r), 0x1.555556p-3f);
  q = __fadd_rn(__fmul_rn(q, r), 0.5f);
  q = __fadd_rn(__fmul_rn(q, r), 1.0f);
  q = __fadd_rn(__fmul_rn(q, r), 1.0f);
  return __fmul_rn(q, __int_as_float(((int)n + 127) << 23));
}

// ---------------------------------------------------------------------------
// ALU-only variants for the GEMM epilogues. The conversion/transcendental
// (XU) pipe is the epilogue's bottleneck, so roundings use integer ops and
// the sigmoid's division uses one reciprocal estimate refined on the FMA
// pipe. Both produce the same bits as the variants above; the division's
// equality is checked on every bf16 gate value (tests/test_gpu_parity.py).
// ---------------------------------------------------------------------------
// float -> bf16 (round to nearest even) in the high 16 bits; NaN -> qNaN.
__device__ __forceinline__ uint32_t bf16_hi_bits(float x) {
  const uint32_t u = __float_as_uint(x);
  const uint32_t r = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  return ((u & 0x7FFFFFFFu) > 0x7F800000u) ? 0x7FC00000u : r;
}
__device__ __forceinline__ float bf16_round_alu(float x) { return __uint_as_float(bf16_hi_bits(x)); }
// Two floats -> packed bf16x2 (lo in bits 0-15).
__device__ __forceinline__ uint32_t pack_bf16x2_alu(float lo, float hi) {
  return __byte_perm(bf16_hi_bits(lo), bf16_hi_bits(hi), 0x7632);
}

// 1 / d rounded to nearest for d >= 1 (d = 1 + 2^t in the sigmoid).
// Newton-Raphson refinement of the hardware reciprocal estimate, then one
// residual correction of the quotient (Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. R&D 34(1), 1990):
//   y1 = y0 + y0 (1 - d y0);  q0 = n y1;  q = q0 + (n - d q0) y1.
// d > 2^64 is scaled by 2^-64 together with the numerator (exact), so the
// estimate stays normal and a subnormal quotient is still rounded correctly.
__device__ __forceinline__ float recip_rn_ge1(float d) {
  const bool big = d > 1.8446744073709552e19f;
  const float ds = big ? __fmul_rn(d, 5.421010862427522e-20f) : d;
  const float n = big ? 5.421010862427522e-20f : 1.0f;
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(ds));
  y = __fmaf_rn(y, __fmaf_rn(-ds, y, 1.0f), y);
  const float q0 = __fmul_rn(n, y);
  const float q = __fmaf_rn(__fmaf_rn(-ds, q0, n), y, q0);
  return isinf(d) ? 0.0f : q;
}

__device__ __forceinline__ float sigmoid_triton_alu(float x) {
  const float t = __fmul_rn(-x, 1.4426950408889634f);
  float e;
  asm("ex2.approx.f32 %0, %1;" : "=f"(e) : "f"(t));
  return recip_rn_ge1(__fadd_rn(1.0f, e));
}

// The reference's SwiGLU element (praxis/kernels/nvfp4_moe.py:125-128) on the
// raw fp32 accumulators of gate and up: gemm output bf16(acc), rescale
// bf16(. * mult), silu = bf16(gate * sigmoid(gate)), h = bf16(silu * up).
// Returns h as a float (a bf16 value).
template <bool kAlu>
__device__ __forceinline__ float swiglu_element(float gate_acc, float up_acc, float mult) {
  if constexpr (kAlu) {
    const float g = bf16_round_alu(__fmul_rn(bf16_round_alu(gate_acc), mult));
    const float u = bf16_round_alu(__fmul_rn(bf16_round_alu(up_acc), mult));
    const float silu = bf16_round_alu(__fmul_rn(g, sigmoid_triton_alu(g)));
    return bf16_round_alu(__fmul_rn(silu, u));
  } else {
    const float g = bf16_round(mul_rn(bf16_round(gate_acc), mult));
    const float u = bf16_round(mul_rn(bf16_round(up_acc), mult));
    const float silu = bf16_round(mul_rn(g, sigmoid_triton(g)));
    return bf16_round(mul_rn(silu, u));
  }
}

// ---------------------------------------------------------------------------
// Paired epilogue arithmetic: sm_100 f32x2 instructions (two IEEE fp32
// operations, each rounded to nearest like its scalar form) and one
// conversion for two bf16 roundings. Same bits as the scalar forms above.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
// a * b + c with one rounding per lane
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
// (lo, hi) -> packed bf16x2 (lo in bits 0-15), round to nearest even
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
}
// bf16(bf16(acc) * mult) for two accumulators of one row (packed)
__device__ __forceinline__ uint32_t rescale_pair(float a0, float a1, float mult) {
  const float2 v = mul2_rn(unpack_bf16x2(cvt_bf16x2(a0, a1)), make_float2(mult, mult));
  return cvt_bf16x2(v.x, v.y);
}

// a * b per bf16 lane, rounded once to bf16 (round to nearest even). For
// bf16 operands the f32 product is exact wherever it is normal, so this is
// bf16(f32(a) * f32(b)) for every product of at least 2^-126 in magnitude
// (and for overflow, which gives infinity both ways).
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// rescale_pair with the multiplier given as a packed bf16x2 pair (mult_bf2 =
// cvt_bf16x2(mult, mult), mult a bf16 value): one conversion and one bf16x2
// multiply. It equals rescale_pair whenever the products are normal, which
// the GEMM epilogues' accumulators times a bf16(g_a * g_w) multiplier are
// (|acc| is 0 or at least the FP4 product quantum, the global scales at least
// 1e-12 / 2688 each).
__device__ __forceinline__ uint32_t rescale_pair_bf2(float a0, float a1, uint32_t mult_bf2) {
  return mul_bf16x2(cvt_bf16x2(a0, a1), mult_bf2);
}

// The SwiGLU element of swiglu_element<> for two adjacent columns of one row
// (gate accumulators g0, g1; up accumulators u0, u1); returns h packed as
// bf16x2. The sigmoid's division 1 / d (d = 1 + 2^t >= 1) is recip_rn_ge1
// unrolled: for d <= 2^64 its scale is 1, so
//   y1 = y0 + y0 (1 - d y0);  q = y1 + (1 - d y1) y1
// on both lanes at once; larger (or infinite) d take the scalar form.
template <bool kBf2>
__device__ __forceinline__ uint32_t swiglu_pair_impl(float g0, float g1, float u0, float u1, float mult,
                                                     uint32_t mult_bf2) {
  const uint32_t gp = kBf2 ? rescale_pair_bf2(g0, g1, mult_bf2) : rescale_pair(g0, g1, mult);
  const uint32_t up = kBf2 ? rescale_pair_bf2(u0, u1, mult_bf2) : rescale_pair(u0, u1, mult);
  const float2 g = unpack_bf16x2(gp);
  const float2 t = mul2_rn(g, make_float2(-1.4426950408889634f, -1.4426950408889634f));
  // The flush-to-zero form gives the same d = 1 + 2^t as the reference's
  // ex2.approx.f32: a subnormal t gives 2^t = 1 either way, and a subnormal
  // 2^t (t < -126) vanishes in 1 + 2^t either way.
  float e0, e1;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(t.x));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(t.y));
  const float2 one = make_float2(1.0f, 1.0f);
  const float2 d = add2_rn(one, make_float2(e0, e1));
  float2 s;
  if (fmaxf(d.x, d.y) > 1.8446744073709552e19f) {  // d >= 1: never NaN
    s = make_float2(recip_rn_ge1(d.x), recip_rn_ge1(d.y));
  } else {
    float2 y0;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0.x) : "f"(d.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0.y) : "f"(d.y));
    // one residual correction of the estimate; d = 1 + 2^t takes one value
    // per bf16 gate value, and every one of them is checked against the IEEE
    // division (the exhaustive SwiGLU test)
    const float2 nd = make_float2(-d.x, -d.y);
    s = fma2_rn(fma2_rn(nd, y0, one), y0, y0);
  }
  const float2 gs = mul2_rn(g, s);
  if constexpr (kBf2) {
    return mul_bf16x2(cvt_bf16x2(gs.x, gs.y), up);
  } else {
    const float2 silu = unpack_bf16x2(cvt_bf16x2(gs.x, gs.y));
    const float2 h = mul2_rn(silu, unpack_bf16x2(up));
    return cvt_bf16x2(h.x, h.y);
  }
}

__device__ __forceinline__ uint32_t swiglu_pair(float g0, float g1, float u0, float u1, float mult) {
  return swiglu_pair_impl<false>(g0, g1, u0, u1, mult, 0u);
}

// The same with the bf16x2 multiplies of rescale_pair_bf2 (and h = silu * u
// as one bf16x2 multiply of two bf16 pairs): the GEMM epilogue's form.
__device__ __forceinline__ uint32_t swiglu_pair_bf2(float g0, float g1, float u0, float u1, uint32_t mult_bf2) {
  return swiglu_pair_impl<true>(g0, g1, u0, u1, 0.0f, mult_bf2);
}

// ---------------------------------------------------------------------------
// Shared-memory addresses and mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Named (hardware) barriers between warps of one CTA: `named_sync` blocks the
// warp until `threads` threads (whole warps) have arrived at barrier `id`
// (1..15; 0 is __syncthreads); `named_arrive` counts the warp without
// waiting. Unlike an mbarrier wait, a named-barrier wait does not stall the
// MMA issue of the thread that runs it. They have no time limit: every user
// here runs the same number of arrivals and syncs on every path, errors
// included (all other waits of the kernels are bounded).
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_arrive(uint32_t id, uint32_t threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Wait for the phase with the given parity to complete. Bounded: gives up
// after `limit_ns` of wall time (or, with `stop_on_error`, as soon as another
// thread raised an error), records `code` and returns false. Waits that keep
// a lock-step protocol going after an error (a phase that is completed on
// every path) pass stop_on_error = false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int code,
                                          uint64_t limit_ns = 2000000000ull, bool stop_on_error = true) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t start = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0u) {
      if (stop_on_error && error_raised()) return false;
      if (globaltimer_ns() - start > limit_ns) {
        record_error(code);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA loads: every copy lands in the issuing CTA's own shared memory
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}

// 2-D tiled load; c0 is the innermost coordinate in elements (bytes here),
// always a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* desc, uint64_t* bar, int32_t c0,
                                            int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 1-D bulk copy global -> shared; both addresses 16-byte aligned, size a
// multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core, accumulators in tensor memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive on an mbarrier once every tcgen05 operation issued so far by this
// thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Block-scaled FP4 x FP4 -> FP32 MMA, 16-element blocks with UE4M3 scales,
// both operands K-major in shared memory, scales in tensor memory.
__device__ __forceinline__ void tc_mma_nvf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// bf16 x bf16 -> fp32 MMA (kind::f16), both operands K-major in shared memory.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Copy 32 rows x 128 bits from shared memory into tensor memory, replicated
// into all four 32-lane sub-partitions (the scale-factor layout the
// block-scaled MMA reads).
__device__ __forceinline__ void tc_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread.
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns -> 16 registers per thread.
__device__ __forceinline__ void tc_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16 (32) registers per thread -> 32 lanes x 16 (32) consecutive 32-bit
// columns of tensor memory (the warp's own lane quadrant). Completion:
// tc_wait_st().
__device__ __forceinline__ void tc_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
               : "memory");
}
__device__ __forceinline__ void tc_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
               : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// CTA pairs (cluster of 2) for cta_group::2 MMAs. No multicast loads: each
// CTA's TMA copies land in its own shared memory; only completion signals
// and tcgen05.commit arrivals cross to the peer.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
  return out;
}

// Arrive on the peer CTA's mbarrier (`cluster_addr`, a shared::cluster
// address). Relaxed: the kernels here use it only to say that tensor-memory
// accesses completed (after tcgen05.wait::ld / wait::st and
// tcgen05.fence::before_thread_sync, which order them), never to publish
// generic-memory data; an arrive with release semantics at cluster scope cost
// about a microsecond per call, a tensor-pipe drain at every k-tile.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion is counted
// on the pair leader's mbarrier (`bar_cluster`, a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* desc, uint32_t bar_cluster, int32_t c0,
                                                 int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

// 2-D tiled store shared -> global (bulk group of the issuing thread).
__device__ __forceinline__ void tma_store_2d(const void* desc, const void* src, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(desc)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the shared-memory sources of this thread's bulk stores can be reused.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until this thread's bulk stores completed.
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Arrive on the mbarrier at the same offset in every CTA of `mask` once all
// prior tcgen05 operations of this thread completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

__device__ __forceinline__ void tc_mma_nvf4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

__device__ __forceinline__ void tc_cp_128x256b_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void tc_cp_32x128b_warpx4_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Shared-memory matrix descriptor (sm_100 format): start address, leading
// and stride byte offsets (16-byte units), version 1, layout type.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout_type) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // descriptor version for sm_100
  d |= (uint64_t)(layout_type & 7u) << 61;
  return d;
}

constexpr uint32_t kLayoutSwizzleNone = 0;
constexpr uint32_t kLayoutSwizzle128B = 2;

// Instruction descriptor of kind::mxf4nvf4 (E2M1 x E2M1, UE4M3 scales,
// K-major A and B, dense K = 64, F32 accumulate).
__host__ __device__ constexpr uint32_t idesc_nvf4(uint32_t m, uint32_t n) {
  return (1u << 7)                 // A format: E2M1
         | (1u << 10)              // B format: E2M1
         | ((n >> 3) << 17)        // N / 8
         | (0u << 23)              // scale format: UE4M3
         | ((m >> 4) << 24);       // M / 16
}

// Instruction descriptor of kind::f16 with bf16 A and B (K-major), F32
// accumulate.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t m, uint32_t n) {
  return (1u << 4)                 // D format: F32
         | (1u << 7)               // A format: BF16
         | (1u << 10)              // B format: BF16
         | ((n >> 3) << 17)        // N / 8
         | ((m >> 4) << 24);       // M / 16
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// Tile table entry written by the dispatch kernel, read by GEMMs/quantize
// ---------------------------------------------------------------------------
struct TileEntry {
  int32_t expert;  // expert of the 128-row tile
  int32_t row0;    // first padded row of the tile
  int32_t valid;   // rows of the tile that hold routed rows (1..128)
  int32_t pad;
};

constexpr int kTileRows = 128;

// Lockstep passes (the two inputs of a classifier-free-guidance pair, tokens
// back to back, pass 1 from token t0): the routed rows of token t sent to
// expert e form group e * n + pass, each group with its own activation and
// hidden global scales and its own padded rows, so every row keeps the bits
// of its pass run alone (praxis/kernels/nvfp4_pair.py:1-20; segment order of
// praxis/kernels/router_fused.py:820-839). n = 1: group e.
struct Passes {
  int32_t n;
  int64_t t0;
};

__device__ __forceinline__ int route_group(int e, int64_t token, Passes ps) {
  return ps.n == 2 ? 2 * e + (token >= ps.t0 ? 1 : 0) : e;
}

// The expert index of a routed slot, clamped (with an index-range error
// recorded) when out of range.
__device__ __forceinline__ int checked_expert(int64_t e, int experts) {
  if (e < 0 || e >= experts) {
    record_error(kErrIndexRange);
    return e < 0 ? 0 : experts - 1;
  }
  return (int)e;
}

}  // namespace praxis
