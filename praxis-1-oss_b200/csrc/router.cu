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
// logits: tcgen05 kind::f16 MMA over 128-row tiles, one CTA per `rows`
// tokens (rows <= 128, chosen so that the grid fills the SMs; the rows of a
// tile past the CTA's own are computed and dropped). x and the weight
// terms are staged by TMA in 64-column (128-byte swizzled) slabs; an fp32
// router weight is passed as 3 bf16 terms (hi + mid + lo == the fp32 value),
// each term's products accumulate in its own tensor-memory columns and the
// epilogue adds the three (every product is exact; only the fp32 summation
// order differs from cuBLAS SGEMM). While the MMAs run, the epilogue warps
// take the per-token max |x| (activation global scale) from the staged slabs.
// routing: one warp per token.
#include "common.cuh"
#include "kernels.h"

namespace praxis {

constexpr int kRouterBM = 128;
constexpr int kRouterBK = 64;          // bf16 columns per 128-byte swizzled slab
constexpr int kRouterABytes = kRouterBM * 128;
constexpr int kRouterSmemBudget = 200 * 1024;

// Warp 0: TMA producer; warp 1: tensor-memory owner and MMA issuer; warps
// 2..5: row max |x| during the main loop, then the logits epilogue (warp w
// reads tensor-memory lanes 32 * (w % 4) .. + 31 = tokens of those rows).
__global__ void __launch_bounds__(192, 1) router_logits_kernel(
    const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w, int64_t tokens, int dim,
    int experts, int splits, int e_pad, int stages, uint32_t tmem_cols, int rows, float* __restrict__ logits,
    uint16_t* __restrict__ row_amax) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int b_bytes = splits * e_pad * 128;
  const int stage_bytes = kRouterABytes + b_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)stages * stage_bytes);
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t)blockIdx.x * rows;
  const int ktiles = (dim + kRouterBK - 1) / kRouterBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + 4);  // MMA commit + 4 row-max warps
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      for (int kt = 0; kt < ktiles; ++kt) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, kErrTimeoutProducer)) break;
        uint8_t* st = smem + (size_t)stage * stage_bytes;
        mbar_arrive_expect_tx(&full[stage], (uint32_t)stage_bytes);
        // every CTA walks the columns in the same order, so a token's logits
        // do not depend on where its row sits in the call (a lockstep pair,
        // a router_rows slice and a lone call give the same bits)
        tma_load_2d(st, &tmap_x, &full[stage], kt * kRouterBK, (int32_t)row0);
        for (int s = 0; s < splits; ++s)
          tma_load_2d(st + kRouterABytes + s * e_pad * 128, &tmap_w, &full[stage], kt * kRouterBK, s * experts);
        if (++stage == (uint32_t)stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // the terms' weight rows are contiguous in shared memory: one MMA per
      // chunk of up to 256 columns covers several terms at once
      const int n_total = splits * e_pad;
      const int n0 = n_total > 256 ? 256 : n_total;
      const uint32_t idesc0 = idesc_bf16(128, (uint32_t)n0);
      const uint32_t idesc1 = idesc_bf16(128, (uint32_t)(n_total > 256 ? n_total - 256 : 16));
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int kt = 0; kt < ktiles; ++kt) {
        if (!mbar_wait(&full[stage], phase, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + (size_t)stage * stage_bytes);
#pragma unroll
        for (int ks = 0; ks < kRouterBK / 16; ++ks) {
          const uint64_t ad = smem_desc(a_base + ks * 32, 16, 1024, kLayoutSwizzle128B);
          const uint32_t acc = (kt | ks) != 0 ? 1u : 0u;
          tc_mma_bf16(tmem, ad, smem_desc(a_base + kRouterABytes + ks * 32, 16, 1024, kLayoutSwizzle128B), idesc0,
                      acc);
          if (n_total > 256)
            tc_mma_bf16(tmem + 256, ad,
                        smem_desc(a_base + kRouterABytes + 256 * 128 + ks * 32, 16, 1024, kLayoutSwizzle128B),
                        idesc1, acc);
        }
        tc_commit(&empty[stage]);
        if (++stage == (uint32_t)stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) tc_commit(acc_full);
    }
  } else {
    const uint32_t quad = (uint32_t)(warp & 3);
    const int row = (int)(quad * 32 + lane);
    // partial max |x| of rows quad*32 + 4i + lane/8, 16-byte chunk lane%8:
    // each load instruction reads 4 whole slab rows (512 contiguous bytes)
    float part[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    for (int kt = 0; kt < ktiles; ++kt) {
      if (!mbar_wait(&full[stage], phase, kErrTimeoutEpilogue)) {
        ok = false;
        break;
      }
      // (the swizzle permutes 16-byte chunks within a row; the max does not care)
      const uint8_t* src = smem + (size_t)stage * stage_bytes + quad * 32 * 128 + lane * 16;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 v = *reinterpret_cast<const uint4*>(src + i * 512);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          part[i] = fmaxf(part[i], fmaxf(fabsf(__uint_as_float(w[j] << 16)), fabsf(__uint_as_float(w[j] & 0xFFFF0000u))));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == (uint32_t)stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    // reduce each row's 8 chunk maxima; lane L keeps row quad*32 + L
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float v = part[i];
      v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
      v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
      v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
      const float r = __shfl_sync(0xffffffffu, v, (lane & 3) * 8);
      if ((int)(lane >> 2) == i) m = r;
    }
    const int64_t grow = row0 + row;
    const bool mine = row < rows && grow < tokens;
    if (row_amax != nullptr && mine) row_amax[grow] = f32_to_bf16(m);
    if (ok && mbar_wait(acc_full, 0, kErrTimeoutEpilogue)) {
      tc_fence_after();
      const uint32_t lane_base = tmem + ((quad * 32u) << 16);
      float* out = logits + grow * experts;
      for (int e0 = 0; e0 < e_pad; e0 += 16) {
        float acc[16];
        for (int s = 0; s < splits; ++s) {
          uint32_t r[16];
          tc_ld_32x32b_x16(lane_base + s * e_pad + e0, r);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] = s == 0 ? __uint_as_float(r[j]) : add_rn(acc[j], __uint_as_float(r[j]));
        }
        if (mine) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (e0 + j < experts) out[e0 + j] = acc[j];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// Routing (one warp per token; experts <= 256, top_k <= 8)
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t ordered_u32(float v) {
  // float order -> unsigned integer order (-0.0 < +0.0), ATen TopKTypeConfig
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// inverse of ordered_u32
__device__ __forceinline__ float from_ordered_u32(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}

__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int o) {
  uint32_t lo = (uint32_t)v, hi = (uint32_t)(v >> 32);
  lo = __shfl_xor_sync(0xffffffffu, lo, o);
  hi = __shfl_xor_sync(0xffffffffu, hi, o);
  return ((uint64_t)hi << 32) | lo;
}

// P = experts per lane (experts <= 32 * P), K = top_k (the selection, tie
// and order loops unroll to K entries).
template <int P, int K>
__global__ void __launch_bounds__(256) route_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                                    int64_t tokens, int experts, int activation,
                                                    int64_t* __restrict__ top_idx, uint16_t* __restrict__ gate) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  constexpr int top_k = K;
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const float* lr = logits + t * experts;
  float score[P], biased[P];
  float lmax = -INFINITY;
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const int e = lane + 32 * i;
    score[i] = e < experts ? lr[e] : -INFINITY;
    lmax = fmaxf(lmax, score[i]);
  }
  if (activation == PRAXIS_B200_SOFTMAX) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const int e = lane + 32 * i;
      score[i] = e < experts ? exp_softmax(__fsub_rn(score[i], lmax)) : 0.0f;
      sum = add_rn(sum, score[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = add_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
#pragma unroll
    for (int i = 0; i < P; ++i) score[i] = div_rn(score[i], sum);
  } else {
#pragma unroll
    for (int i = 0; i < P; ++i) score[i] = div_rn(1.0f, add_rn(1.0f, expf(-score[i])));
  }
#pragma unroll
  for (int i = 0; i < P; ++i) {
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
      for (int i = 0; i < P; ++i) {
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

  // -- distinct selected values (the usual case): the sort below yields them
  //    in descending order, which is the selection order; otherwise (ties,
  //    +0/-0, NaN) the sort's tie order is emulated step by step
  bool distinct = true;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
#pragma unroll
    for (int i = 0; i < j; ++i)
      if (j < top_k) {
        const float vi = from_ordered_u32(sel_hi[i]), vj = from_ordered_u32(sel_hi[j]);
        distinct = distinct && vi != vj && vi == vi && vj == vj;
      }
  }

  // -- gather order: entries above the k-th value, then the ties, each by index
  uint32_t kth = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (j == top_k - 1) kth = sel_hi[j];
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
      if (distinct ? j == (int)lane : rank == (int)lane) my_idx = sel_idx[j];
    }
  }
  bool valid = lane < top_k;
  // value of my entry (biased) and its unbiased score
  float my_val = 0.0f, my_score = 0.0f;
  {
    const int src_lane = my_idx & 31, src_i = my_idx >> 5;
    float bv = 0.0f, sv = 0.0f;
#pragma unroll
    for (int i = 0; i < P; ++i) {
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
  for (int size = distinct ? 64 : 2; size <= 32; size <<= 1) {
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
static int make_bf16_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(PRAXIS_B200_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)kRouterBK, (cuuint32_t)box_rows};
  cuuint32_t estride[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(PRAXIS_B200_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return PRAXIS_B200_OK;
}

int run_router_logits(const uint16_t* x, const uint16_t* w, int splits, int64_t tokens, int dim, int experts,
                      float* logits, uint16_t* row_amax, cudaStream_t stream) {
  if (experts < 1 || experts > 256) return set_error(PRAXIS_B200_EINVAL, "router supports 1..256 experts");
  if (dim % 32 != 0) return set_error(PRAXIS_B200_EINVAL, "router needs dim %% 32 == 0");
  if (splits != 1 && splits != 3) return set_error(PRAXIS_B200_EINVAL, "router weight splits must be 1 or 3");
  if (splits == 3 && experts > 128) return set_error(PRAXIS_B200_EINVAL, "fp32 router weight supports <= 128 experts");
  if (((uintptr_t)x | (uintptr_t)w) & 15) return set_error(PRAXIS_B200_EINVAL, "router inputs must be 16-byte aligned");
  if (tokens == 0) return PRAXIS_B200_OK;
  const int e_pad = (experts + 15) / 16 * 16;
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)(splits * e_pad)) tmem_cols <<= 1;
  const int stage_bytes = kRouterABytes + splits * e_pad * 128;
  int stages = kRouterSmemBudget / stage_bytes;
  stages = stages < 2 ? 2 : stages > 6 ? 6 : stages;
  const size_t smem = 1024 + (size_t)stages * stage_bytes + (2 * stages + 2) * 8;
  static DeviceOnce attr;
  int rc = device_once(attr, [](int dev) {
    const cudaError_t e =
        cudaFuncSetAttribute(router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    if (e != cudaSuccess)
      return set_error(PRAXIS_B200_ECUDA, "router smem attribute (device %d): %s", dev, cudaGetErrorString(e));
    return (int)PRAXIS_B200_OK;
  });
  if (rc) return rc;
  CUtensorMap mx, mw;
  rc = make_bf16_map(&mx, x, tokens, dim, kRouterBM);
  if (rc) return rc;
  rc = make_bf16_map(&mw, w, (int64_t)splits * experts, dim, e_pad);
  if (rc) return rc;
  // rows per CTA: a multiple of 16, at most one tile, so that the CTAs cover
  // the SMs once when the tokens allow it (one CTA per SM: shared memory)
  const int64_t sms = sm_count();
  int64_t rows = (tokens + sms - 1) / sms;
  rows = (rows + 15) / 16 * 16;
  rows = rows < 16 ? 16 : rows > kRouterBM ? kRouterBM : rows;
  const int64_t blocks = (tokens + rows - 1) / rows;
  launch_pdl(router_logits_kernel, dim3((unsigned)blocks), dim3(192), smem, stream, mx, mw, tokens, dim, experts,
             splits, e_pad, stages, tmem_cols, (int)rows, logits, row_amax);
  return check_launch("router_logits");
}

int run_route(const float* logits, const float* bias, int64_t tokens, int experts, int top_k, int activation,
              int64_t* top_idx, uint16_t* gate, cudaStream_t stream) {
  if (experts < 1 || experts > 256) return set_error(PRAXIS_B200_EINVAL, "routing supports 1..256 experts");
  if (top_k < 1 || top_k > 8 || top_k > experts) return set_error(PRAXIS_B200_EINVAL, "top_k must be 1..min(8, E)");
  if (activation != PRAXIS_B200_SIGMOID && activation != PRAXIS_B200_SOFTMAX)
    return set_error(PRAXIS_B200_EINVAL, "unknown router activation");
  if (tokens == 0) return PRAXIS_B200_OK;
  const unsigned blocks = (unsigned)((tokens + 7) / 8);
  using Kernel = decltype(&route_kernel<1, 1>);
#define PRAXIS_ROUTE_ROW(P)                                                                                     \
  {route_kernel<P, 1>, route_kernel<P, 2>, route_kernel<P, 3>, route_kernel<P, 4>, route_kernel<P, 5>,         \
   route_kernel<P, 6>, route_kernel<P, 7>, route_kernel<P, 8>}
  static const Kernel kernels[4][8] = {PRAXIS_ROUTE_ROW(1), PRAXIS_ROUTE_ROW(2), PRAXIS_ROUTE_ROW(4),
                                       PRAXIS_ROUTE_ROW(8)};
#undef PRAXIS_ROUTE_ROW
  const int pi = experts <= 32 ? 0 : experts <= 64 ? 1 : experts <= 128 ? 2 : 3;
  launch_pdl(kernels[pi][top_k - 1], dim3(blocks), dim3(256), 0, stream, logits, bias, tokens, experts, activation,
             top_idx, gate);
  return check_launch("route");
}

}  // namespace praxis
