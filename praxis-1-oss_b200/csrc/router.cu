// Router: float32 logits of bf16 tokens, gating, top-k and renormalised gates.
//
// Replaces praxis/layers.py:1104-1122 (fp32 router GEMM) and the stock routing
// ops of praxis/layers.py:1647-1653 / :2167-2173 (as router_fused does for
// E=128/k=8, praxis/kernels/router_fused.py:465-573, here for any E <= 256,
// k <= 8):
//   s = sigmoid(l)              ATen CUDA: 1 / (1 + expf(-l)), IEEE division
//   b = s + bias
//   top = topk(b, k)            the set, and ATen's CUDA slot order on ties
//                               (k-th-value ties: lowest index; elements above
//                               the k-th value then equal to it, each in index
//                               order, through the 32-wide bitonic sort)
//   gate = bf16(s[top] / sum)   ATen's CUDA reduction order of a k-wide row
// softmax gating (this build's extension) uses the same selection and gates.
//
// logits: one CTA per 64 tokens, bf16 mma.sync (m16n8k16, fp32 accumulate) on
// the exact bf16 inputs; an fp32 router weight is passed as 3 bf16 terms
// (hi + mid + lo == the fp32 value), so every product is exact and only the
// fp32 summation order differs from cuBLAS SGEMM. The same pass computes the
// per-token max |x| used by the activation global scale.
// routing: one warp per token.
#include "common.cuh"
#include "kernels.h"

namespace praxis {

constexpr int kRouterBM = 64;
constexpr int kRouterBK = 32;
constexpr int kRouterPad = 40;  // bf16 per smem row (80 B: conflict-free ldmatrix)

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  const uint32_t d = smem_u32(dst);
  const int size = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(size) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldmatrix_x2(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// NT = experts/8 rounded up to a power of two; SPLITS = 1 (bf16 weight) or 3.
template <int NT, int SPLITS>
__global__ void __launch_bounds__(128) router_logits_kernel(const uint16_t* __restrict__ x,
                                                            const uint16_t* __restrict__ w, int64_t tokens,
                                                            int dim, int experts, float* __restrict__ logits,
                                                            uint16_t* __restrict__ row_amax) {
  constexpr int EP = NT * 8;
  extern __shared__ __align__(16) uint16_t s_router[];
  uint16_t* sx = s_router;                                // [2][64][40]
  uint16_t* sw = s_router + 2 * kRouterBM * kRouterPad;  // [2][SPLITS*EP][40]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row0 = (int64_t)blockIdx.x * kRouterBM;
  const int ktiles = dim / kRouterBK;

  auto load_stage = [&](int stage, int kt) {
    const int k0 = kt * kRouterBK;
    for (int c = tid; c < kRouterBM * 4; c += 128) {
      const int r = c >> 2, ch = c & 3;
      const int64_t gr = row0 + r;
      const bool ok = gr < tokens;
      cp_async16(sx + (stage * kRouterBM + r) * kRouterPad + ch * 8, x + (ok ? gr : 0) * dim + k0 + ch * 8, ok);
    }
    for (int c = tid; c < SPLITS * EP * 4; c += 128) {
      const int r = c >> 2, ch = c & 3;
      const int s = r / EP, e = r % EP;
      const bool ok = e < experts;
      cp_async16(sw + (stage * SPLITS * EP + r) * kRouterPad + ch * 8,
                 w + ((int64_t)s * experts + (ok ? e : 0)) * dim + k0 + ch * 8, ok);
    }
    cp_async_commit();
  };

  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
  float rmax = 0.0f;

  load_stage(0, 0);
  for (int kt = 0; kt < ktiles; ++kt) {
    const int stage = kt & 1;
    if (kt + 1 < ktiles) {
      load_stage(stage ^ 1, kt + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint16_t* xs = sx + stage * kRouterBM * kRouterPad;
    const uint16_t* ws = sw + stage * SPLITS * EP * kRouterPad;
    {  // per-token max |x| (thread -> row tid/2, 16 columns)
      const uint4* p = reinterpret_cast<const uint4*>(xs + (tid >> 1) * kRouterPad + (tid & 1) * 16);
      uint4 a = p[0], b = p[1];
      const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
        rmax = fmaxf(rmax, fmaxf(fabsf(bf16_to_f32((uint16_t)(v[i] & 0xFFFFu))), fabsf(bf16_to_f32((uint16_t)(v[i] >> 16)))));
    }
#pragma unroll
    for (int ks = 0; ks < kRouterBK / 16; ++ks) {
      uint32_t a[4];
      ldmatrix_x4(a, xs + (warp * 16 + (lane & 15)) * kRouterPad + ks * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int s = 0; s < SPLITS; ++s) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          uint32_t b[2];
          ldmatrix_x2(b, ws + (s * EP + nt * 8 + (lane & 7)) * kRouterPad + ks * 16 + ((lane >> 3) & 1) * 8);
          mma_bf16(acc[nt], a, b);
        }
      }
    }
    __syncthreads();
  }
  rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 1));
  if (row_amax != nullptr && (tid & 1) == 0 && row0 + (tid >> 1) < tokens) row_amax[row0 + (tid >> 1)] = f32_to_bf16(rmax);
  const int r_lo = warp * 16 + (lane >> 2);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int col = nt * 8 + (lane & 3) * 2;
    if (col < experts) {
      if (row0 + r_lo < tokens)
        *reinterpret_cast<float2*>(logits + (row0 + r_lo) * experts + col) = make_float2(acc[nt][0], acc[nt][1]);
      if (row0 + r_lo + 8 < tokens)
        *reinterpret_cast<float2*>(logits + (row0 + r_lo + 8) * experts + col) = make_float2(acc[nt][2], acc[nt][3]);
    }
  }
}

// ---------------------------------------------------------------------------
// Routing (one warp per token; experts <= 256, top_k <= 8)
// ---------------------------------------------------------------------------
constexpr int kMaxPerLane = 8;

__device__ __forceinline__ uint32_t ordered_u32(float v) {
  // float order -> unsigned integer order (-0.0 < +0.0), ATen TopKTypeConfig
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int o) {
  uint32_t lo = (uint32_t)v, hi = (uint32_t)(v >> 32);
  lo = __shfl_xor_sync(0xffffffffu, lo, o);
  hi = __shfl_xor_sync(0xffffffffu, hi, o);
  return ((uint64_t)hi << 32) | lo;
}

__global__ void __launch_bounds__(256) route_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                                    int64_t tokens, int experts, int top_k, int activation,
                                                    int64_t* __restrict__ top_idx, uint16_t* __restrict__ gate) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const float* lr = logits + t * experts;
  float score[kMaxPerLane], biased[kMaxPerLane];
  float lmax = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    score[i] = e < experts ? lr[e] : -INFINITY;
    lmax = fmaxf(lmax, score[i]);
  }
  if (activation == PRAXIS_B200_SOFTMAX) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      score[i] = e < experts ? expf(__fsub_rn(score[i], lmax)) : 0.0f;
      sum = add_rn(sum, score[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = add_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) score[i] = div_rn(score[i], sum);
  } else {
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) score[i] = div_rn(1.0f, add_rn(1.0f, expf(-score[i])));
  }
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    biased[i] = (bias != nullptr && e < experts) ? add_rn(score[i], bias[e]) : score[i];
  }

  // -- the top-k set: k rounds of a warp arg-max over 64-bit keys
  //    (value order, then the lower expert index)
  uint32_t taken = 0;
  int sel_idx[8];
  uint32_t sel_hi[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    sel_idx[j] = 0;
    sel_hi[j] = 0;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j < top_k) {
      uint64_t best = 0;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) {
        const int e = lane + 32 * i;
        if (e < experts && !(taken & (1u << i))) {
          const uint64_t key = ((uint64_t)ordered_u32(biased[i]) << 32) | (uint32_t)(experts - 1 - e);
          best = key > best ? key : best;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const uint64_t other = shfl_xor_u64(best, o);
        best = other > best ? other : best;
      }
      const int e = experts - 1 - (int)(uint32_t)best;
      sel_idx[j] = e;
      sel_hi[j] = (uint32_t)(best >> 32);
      if ((e & 31) == lane) taken |= 1u << (e >> 5);
    }
  }

  // -- gather order: entries above the k-th value, then the ties, each by index
  const uint32_t kth = sel_hi[top_k - 1];
  int my_idx = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j < top_k) {
      const int tj = sel_hi[j] == kth;
      int rank = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < top_k) {
          const int ti = sel_hi[i] == kth;
          rank += (ti < tj) || (ti == tj && sel_idx[i] < sel_idx[j]);
        }
      }
      if (rank == lane) my_idx = sel_idx[j];
    }
  }
  bool valid = lane < top_k;
  // value of my entry (biased) and its unbiased score
  float my_val = 0.0f, my_score = 0.0f;
  {
    const int src_lane = my_idx & 31, src_i = my_idx >> 5;
    float bv = 0.0f, sv = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const float b_i = __shfl_sync(0xffffffffu, biased[i], src_lane);
      const float s_i = __shfl_sync(0xffffffffu, score[i], src_lane);
      if (i == src_i) {
        bv = b_i;
        sv = s_i;
      }
    }
    my_val = bv;
    my_score = sv;
  }

  // -- ATen's 32-wide bitonic key/value sort (16 threads x 2 items; invalid
  //    entries sort last), one item per lane: positions p and p^stride.
  for (int size = 2; size <= 32; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const float o_val = __shfl_xor_sync(0xffffffffu, my_val, stride);
      const float o_score = __shfl_xor_sync(0xffffffffu, my_score, stride);
      const int o_idx = __shfl_xor_sync(0xffffffffu, my_idx, stride);
      const bool o_valid = __shfl_xor_sync(0xffffffffu, valid ? 1 : 0, stride) != 0;
      const int lo = lane & ~stride;
      const bool is_a = lane == lo;
      const float va = is_a ? my_val : o_val, vb = is_a ? o_val : my_val;
      const bool ok_a = is_a ? valid : o_valid, ok_b = is_a ? o_valid : valid;
      bool flag = false;
      if (size < 32) {
        const int tid = (lo / (2 * stride)) * stride + (lo % stride);
        flag = (tid & (size >> 1)) != 0;
      }
      const bool swap = ((va > vb) && ok_a) || !ok_b;
      if (swap == flag) {
        my_val = o_val;
        my_score = o_score;
        my_idx = o_idx;
        valid = o_valid;
      }
    }
  }

  // -- gates: s / sum(s) in ATen's reduction order, rounded to bf16
  const int w = 1 << (31 - __clz(top_k));
  float acc = my_score;
#pragma unroll
  for (int m = 1; m < 8; ++m) {
    const int src = lane + m * w;
    const float v = __shfl_sync(0xffffffffu, my_score, src & 31);
    if (src < top_k && m * w < 8) acc = add_rn(acc, v);
  }
  for (int off = w >> 1; off > 0; off >>= 1) {
    const float v = __shfl_down_sync(0xffffffffu, acc, off);
    if (lane + off < w) acc = add_rn(acc, v);
  }
  const float total = __shfl_sync(0xffffffffu, acc, 0);
  if (lane < top_k) {
    top_idx[t * top_k + lane] = my_idx;
    gate[t * top_k + lane] = f32_to_bf16(div_rn(my_score, total));
  }
}

// ---------------------------------------------------------------------------
// Host entries
// ---------------------------------------------------------------------------
template <int NT, int SPLITS>
static int launch_router_logits(const uint16_t* x, const uint16_t* w, int64_t tokens, int dim, int experts,
                                float* logits, uint16_t* row_amax, cudaStream_t stream) {
  const size_t smem = (size_t)2 * (kRouterBM + SPLITS * NT * 8) * kRouterPad * 2;
  auto kern = router_logits_kernel<NT, SPLITS>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  const int64_t blocks = (tokens + kRouterBM - 1) / kRouterBM;
  kern<<<(unsigned)blocks, 128, smem, stream>>>(x, w, tokens, dim, experts, logits, row_amax);
  return check_launch("router_logits");
}

template <int SPLITS>
static int dispatch_router_nt(int nt, const uint16_t* x, const uint16_t* w, int64_t tokens, int dim, int experts,
                              float* logits, uint16_t* row_amax, cudaStream_t stream) {
  switch (nt) {
    case 1: return launch_router_logits<1, SPLITS>(x, w, tokens, dim, experts, logits, row_amax, stream);
    case 2: return launch_router_logits<2, SPLITS>(x, w, tokens, dim, experts, logits, row_amax, stream);
    case 4: return launch_router_logits<4, SPLITS>(x, w, tokens, dim, experts, logits, row_amax, stream);
    case 8: return launch_router_logits<8, SPLITS>(x, w, tokens, dim, experts, logits, row_amax, stream);
    case 16: return launch_router_logits<16, SPLITS>(x, w, tokens, dim, experts, logits, row_amax, stream);
    case 32: return launch_router_logits<32, SPLITS>(x, w, tokens, dim, experts, logits, row_amax, stream);
    default: return set_error(PRAXIS_B200_EINVAL, "unsupported expert count");
  }
}

int run_router_logits(const uint16_t* x, const uint16_t* w, int splits, int64_t tokens, int dim, int experts,
                      float* logits, uint16_t* row_amax, cudaStream_t stream) {
  if (experts < 1 || experts > 256) return set_error(PRAXIS_B200_EINVAL, "router supports 1..256 experts");
  if (dim % kRouterBK != 0) return set_error(PRAXIS_B200_EINVAL, "router needs dim %% 32 == 0");
  if (splits != 1 && splits != 3) return set_error(PRAXIS_B200_EINVAL, "router weight splits must be 1 or 3");
  if (tokens == 0) return PRAXIS_B200_OK;
  int nt = 1;
  while (nt * 8 < experts) nt <<= 1;
  if (nt > 16 && splits == 3) return set_error(PRAXIS_B200_EINVAL, "fp32 router weight supports <= 128 experts");
  return splits == 1 ? dispatch_router_nt<1>(nt, x, w, tokens, dim, experts, logits, row_amax, stream)
                     : dispatch_router_nt<3>(nt, x, w, tokens, dim, experts, logits, row_amax, stream);
}

int run_route(const float* logits, const float* bias, int64_t tokens, int experts, int top_k, int activation,
              int64_t* top_idx, uint16_t* gate, cudaStream_t stream) {
  if (experts < 1 || experts > 256) return set_error(PRAXIS_B200_EINVAL, "routing supports 1..256 experts");
  if (top_k < 1 || top_k > 8 || top_k > experts) return set_error(PRAXIS_B200_EINVAL, "top_k must be 1..min(8, E)");
  if (activation != PRAXIS_B200_SIGMOID && activation != PRAXIS_B200_SOFTMAX)
    return set_error(PRAXIS_B200_EINVAL, "unknown router activation");
  if (tokens == 0) return PRAXIS_B200_OK;
  const int64_t blocks = (tokens + 7) / 8;
  route_kernel<<<(unsigned)blocks, 256, 0, stream>>>(logits, bias, tokens, experts, top_k, activation, top_idx, gate);
  return check_launch("route");
}

}  // namespace praxis
