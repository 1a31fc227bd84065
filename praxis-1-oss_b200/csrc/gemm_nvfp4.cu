// Grouped NVFP4 x NVFP4 GEMM for routed experts on sm_100a (tcgen05).
//
// Replaces praxis/kernels/nvfp4.py:355-419 (grouped_nvfp4_mm -> FlashInfer's
// CuTe-DSL block-scaled contiguous grouped GEMM, alpha = 1, 128-row expert
// tiles) and fuses the element-wise stage that follows it:
//   EPI_PLAIN   out = bf16(acc)
//   EPI_SWIGLU  praxis/kernels/nvfp4_moe.py:102-133 (rescale, SwiGLU with
//               Triton's sigmoid, every bf16 rounding kept) + the per-expert
//               max |hidden| that praxis/kernels/nvfp4_moe.py:60-81 reduces
//   EPI_RESCALE bf16(bf16(acc) * bf16(g_a * g_w)), the first step of
//               praxis/kernels/nvfp4_moe.py:236-247 (rescale_combine)
//
// Design (one CTA per SM, persistent over (m-tile, n-tile) units):
//   warp 0      TMA producer: A and B tiles (2-D, 128B swizzle) and the
//               pre-swizzled scale atoms (1-D bulk copies) into a 5-stage ring
//   warp 1      tcgen05 issuer: scale atoms smem -> TMEM (tcgen05.cp), then
//               kind::mxf4nvf4 block16 MMAs (M=128, N=BLOCK_N, K=64) into a
//               double-buffered TMEM accumulator
//   warps 2..5  epilogue: TMEM -> registers (tcgen05.ld), fused math, stores
// Every mbarrier wait is bounded (see common.cuh).
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"
#include "nvfp4_quant.cuh"

namespace praxis {

template <int BLOCK_N>
struct GemmShape {
  static constexpr int BM = kTileRows;          // rows per tile
  static constexpr int BK_BYTES = 128;          // 256 FP4 values per k-tile
  static constexpr int STAGES = 5;
  static constexpr int A_BYTES = BM * BK_BYTES;  // 16 KB
  static constexpr int B_BYTES = BLOCK_N * BK_BYTES;
  static constexpr int SF_ATOM = 512;           // 128 rows x 4 scales
  static constexpr int SFA_BYTES = 4 * SF_ATOM;
  static constexpr int SFB_BYTES = (BLOCK_N / 128) * 4 * SF_ATOM;
  static constexpr int ACC_BUFS = 2;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SFA_COL = ACC_BUFS * BLOCK_N;  // 4 columns per k-block
  static constexpr int SFB_COL = SFA_COL + 16;        // (BLOCK_N/128)*4 per k-block
  static constexpr size_t SMEM_BYTES =
      1024 + (size_t)STAGES * (A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES) + 256;
  static_assert(SFB_COL + 4 * (BLOCK_N / 128) * 4 <= TMEM_COLS, "tensor memory budget");
};

__device__ __forceinline__ void store_row_chunk(uint16_t* dst, const uint32_t (&packed)[16]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    d[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
}

// Tile expert e reads weights (e / groups_per_weight) % weight_experts: one
// expert per tile on a single GPU; with lockstep passes a tile's "expert" is
// a group (expert, pass) = expert * passes + pass; with expert parallelism a
// segment (source rank, local expert) = rank * local experts + expert. Either
// way the group has activation scales of its own.
__device__ __forceinline__ int weight_expert(const GemmParams& p, int e) {
  const int w = p.groups_per_weight > 1 ? e / p.groups_per_weight : e;
  return w < p.weight_experts ? w : w % p.weight_experts;
}

__device__ __forceinline__ float expert_multiplier(const GemmParams& p, int e) {
  // bf16(g_a * g_w) in float32 (praxis/kernels/nvfp4_moe.py:117-121, :237-241)
  float ga;
  if (p.act_global_scalar > 0.0f) {
    ga = p.act_global_scalar;
  } else if (p.act_global != nullptr) {
    ga = p.act_global[e];
  } else {
    ga = global_from_amax_bits(p.act_amax[e]);
  }
  return bf16_round(mul_rn(ga, p.w_global[weight_expert(p, e)]));
}

// Hidden 32-column chunk computed by 64-row gate/up block `blk` of the
// interleaved weights: blocks 1 and 2 of every group of four trade places
// (see interleave_gate_up_kernel).
__host__ __device__ __forceinline__ int hidden_chunk(int blk) {
  const int b = blk & 3;
  return (blk & ~3) | ((b & 1) << 1) | (b >> 1);
}

template <int BLOCK_N, int EPI>
__global__ void __launch_bounds__(192, 1) gemm_nvfp4_kernel(const __grid_constant__ GemmParams p) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  using S = GemmShape<BLOCK_N>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + S::STAGES * S::A_BYTES;
  uint8_t* sSFA = sB + S::STAGES * S::B_BYTES;
  uint8_t* sSFB = sSFA + S::STAGES * S::SFA_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSFB + S::STAGES * S::SFB_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + S::STAGES;
  uint64_t* acc_full = bars + 2 * S::STAGES;
  uint64_t* acc_empty = acc_full + S::ACC_BUFS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + S::ACC_BUFS);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < S::ACC_BUFS; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmap_a);
    tma_prefetch_desc(&p.tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int n_tiles = p.N / BLOCK_N;
  const int num_m = *p.num_tiles;
  const int total = num_m * n_tiles;
  const int k_tiles = (p.K + 255) / 256;
  const int kb_total = p.K / 64;  // scale atoms per 128-row tile

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const int m = u / n_tiles, n = u - (u / n_tiles) * n_tiles;
        const TileEntry t = p.tiles[m];
        const int we = weight_expert(p, t.expert);
        const int brow = we * p.N + n * BLOCK_N;
        const uint8_t* sfa = p.sfa + (size_t)(t.row0 / 128) * kb_total * S::SF_ATOM;
        const uint8_t* sfb =
            p.sfb + ((size_t)we * (p.N / 128) + (size_t)n * (BLOCK_N / 128)) * kb_total * S::SF_ATOM;
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          const int kb = min(4, kb_total - kt * 4);
          const uint32_t sf_bytes = (uint32_t)kb * S::SF_ATOM;
          mbar_arrive_expect_tx(&full[stage],
                                S::A_BYTES + S::B_BYTES + sf_bytes * (1 + BLOCK_N / 128));
          tma_load_2d(sA + stage * S::A_BYTES, &p.tmap_a, &full[stage], kt * S::BK_BYTES, t.row0);
          tma_load_2d(sB + stage * S::B_BYTES, &p.tmap_b, &full[stage], kt * S::BK_BYTES, brow);
          bulk_load(sSFA + stage * S::SFA_BYTES, sfa + (size_t)kt * 4 * S::SF_ATOM, sf_bytes, &full[stage]);
#pragma unroll
          for (int h = 0; h < BLOCK_N / 128; ++h)
            bulk_load(sSFB + stage * S::SFB_BYTES + h * S::SFA_BYTES,
                      sfb + ((size_t)h * kb_total + (size_t)kt * 4) * S::SF_ATOM, sf_bytes, &full[stage]);
          if (++stage == S::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- tcgen05 issuer ----------------
      constexpr uint32_t idesc = idesc_nvf4(128, BLOCK_N);
      const uint32_t sfa_t = tmem + S::SFA_COL;
      const uint32_t sfb_t = tmem + S::SFB_COL;
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * BLOCK_N;
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&full[stage], phase, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int kb_n = min(4, kb_total - kt * 4);
          const uint32_t a_base = smem_u32(sA + stage * S::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * S::B_BYTES);
          const uint32_t sfa_s = smem_u32(sSFA + stage * S::SFA_BYTES);
          const uint32_t sfb_s = smem_u32(sSFB + stage * S::SFB_BYTES);
          for (int kb = 0; kb < kb_n; ++kb) {
            tc_cp_32x128b_warpx4(sfa_t + kb * 4, smem_desc(sfa_s + kb * S::SF_ATOM, 0, 128, kLayoutSwizzleNone));
#pragma unroll
            for (int h = 0; h < BLOCK_N / 128; ++h)
              tc_cp_32x128b_warpx4(sfb_t + (kb * (BLOCK_N / 128) + h) * 4,
                                   smem_desc(sfb_s + h * S::SFA_BYTES + kb * S::SF_ATOM, 0, 128, kLayoutSwizzleNone));
          }
          for (int kb = 0; kb < kb_n; ++kb) {
            const uint64_t ad = smem_desc(a_base + kb * 32, 16, 1024, kLayoutSwizzle128B);
            const uint64_t bd = smem_desc(b_base + kb * 32, 16, 1024, kLayoutSwizzle128B);
            tc_mma_nvf4(d_tmem, ad, bd, idesc, sfa_t + kb * 4, sfb_t + kb * (BLOCK_N / 128) * 4,
                        (kt | kb) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == S::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[acc]);
        acc ^= 1u;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const uint32_t quad = (uint32_t)(warp & 3);  // TMEM lanes 32*quad .. +31
    const int row_in_tile = (int)(quad * 32 + lane);
    uint32_t acc = 0, acc_phase = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      const int m = u / n_tiles, n = u - (u / n_tiles) * n_tiles;
      const TileEntry t = p.tiles[m];
      if (!mbar_wait(&acc_full[acc], acc_phase, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const bool valid = row_in_tile < t.valid;
      const size_t grow = (size_t)t.row0 + row_in_tile;
      const uint32_t taddr = tmem + ((quad * 32u) << 16) + acc * BLOCK_N;
      if constexpr (EPI == EPI_SWIGLU) {
        // B rows come in 64-row blocks of 32 gate rows then the matching 32
        // up rows (praxis_b200_interleave_gate_up): tile columns [64c, 64c+32)
        // are gate and [64c+32, 64c+64) up for hidden columns 32c.. of the tile.
        const float mult = expert_multiplier(p, t.expert);
        __nv_bfloat162 hmax = __floats2bfloat162_rn(0.0f, 0.0f);
        constexpr int HALF = BLOCK_N / 2;
#pragma unroll 1
        for (int c = 0; c < HALF / 32; ++c) {
          uint32_t g[32], up[32];
          tc_ld_32x32b_x32(taddr + c * 64, g);
          tc_ld_32x32b_x32(taddr + c * 64 + 32, up);
          tc_wait_ld();
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            uint32_t h = swiglu_pair(__uint_as_float(g[j]), __uint_as_float(g[j + 1]), __uint_as_float(up[j]),
                                     __uint_as_float(up[j + 1]), mult);
            if (!valid) h = 0u;
            hmax = __hmax2(hmax, __habs2(*reinterpret_cast<__nv_bfloat162*>(&h)));
            packed[j / 2] = h;
          }
          store_row_chunk(p.out + grow * p.out_cols + (size_t)32 * hidden_chunk(n * (BLOCK_N / 64) + c), packed);
        }
        const uint32_t hm = *reinterpret_cast<uint32_t*>(&hmax);
        float rmax = fmaxf(__uint_as_float(hm << 16), __uint_as_float(hm & 0xFFFF0000u));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, o));
        if (lane == 0) atomicMax(p.amax_out + t.expert, __float_as_uint(rmax));
      } else {
        const float mult = (EPI == EPI_RESCALE) ? expert_multiplier(p, t.expert) : 1.0f;
#pragma unroll 1
        for (int c = 0; c < BLOCK_N / 32; ++c) {
          uint32_t r[32];
          tc_ld_32x32b_x32(taddr + c * 32, r);
          tc_wait_ld();
          if (valid) {
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float v0 = __uint_as_float(r[j]), v1 = __uint_as_float(r[j + 1]);
              packed[j / 2] = EPI == EPI_RESCALE ? rescale_pair(v0, v1, mult) : cvt_bf16x2(v0, v1);
            }
            store_row_chunk(p.out + grow * p.out_cols + (size_t)n * BLOCK_N + c * 32, packed);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair kernel: M = 256 (128 rows per CTA), N = 256, cta_group::2.
//
// Each CTA loads its own 128 A rows and its own half (128 rows) of the B
// tile; the pair's MMA reads B from both CTAs' shared memory, so per SM the
// operand traffic per FLOP is half that of the 1-CTA 128x128 tile. Each CTA
// also holds the scales of its A rows and of all 256 B rows (the MMA reads
// SFB of every N column in each CTA's tensor memory).
//
// Tensor memory (512 columns per CTA): the accumulator of tile i starts at
// column 0 for even i and 128 for odd i; the two overlap in 128 columns
// (columns 128..255). Each epilogue warp drains the 64-column block it owns
// inside the overlap first and then releases, so the next tile's MMAs start
// after one tensor-memory load per warp. Scales live in columns 384..479: two
// slots of 48 columns (A scales at +0, B scales at +16) used by alternate
// k-tiles.
//
// Roles: warp 0 TMA (both CTAs; completion counted on the leader's barrier),
// warp 1 MMA issuer and scale copier (leader CTA only), warps 2..9 epilogue
// (both CTAs, two warps per TMEM lane quadrant; the warps of half h take
// 64-column blocks h and h + 2). The scale copies run in the tensor pipe in
// order with the MMAs; the MMA thread issues each k-tile's copies just
// before its MMAs, so nothing waits on a copy's completion.
//
// Scale factors reach tensor memory in one of two ways:
//  REP = false  the reference's compact layout (512-byte atom = 128 rows x 4
//               scales); one tcgen05.cp 32x128b.warpx4 per atom replicates it
//               into the four lane quadrants (12 copies per k-tile).
//  REP = true   atoms stored four times in a row in global memory ("replicated
//               layout", produced by this library's quantize kernels and
//               praxis_b200_replicate_scales); one tcgen05.cp 128x256b moves
//               two replicated atoms (6 copies per k-tile; the MMAs and copies
//               of GEMM1 of config 2 take 293 us against 385 us with the
//               compact copies, 251 us for the MMAs alone).
//
// Output stores:
//  DIRECT       the SwiGLU epilogue (128 hidden columns per tile) stores its
//               rows straight from registers (32-byte stores, 64 contiguous
//               bytes per row and block); the freed staging memory holds a
//               fourth k-tile stage, which the TMA loads need to stay ahead
//               of the MMAs (3 stages: 441 us, 4 stages: 408 us for GEMM1 of
//               config 2). The rescale epilogue (256 columns) keeps the
//               staged TMA stores, which write full lines.
// ---------------------------------------------------------------------------
// Named barriers of the scale slots (ids 1, 2): the leader's MMA warp and
// its four scale-loader warps.
constexpr uint32_t kSfBarrier0 = 1;
constexpr uint32_t kSfBarrierThreads = 32 * 5;

template <bool REP, bool DIRECT>
struct PairShape {
  static constexpr int BN = 256;
  static constexpr int BK_BYTES = 128;
  static constexpr int A_BYTES = 128 * BK_BYTES;
  static constexpr int B_BYTES = 128 * BK_BYTES;
  static constexpr int SF_COPIES = REP ? 4 : 1;
  static constexpr int SFA_BYTES = 4 * 512 * SF_COPIES;      // 4 k-blocks
  static constexpr int SFB_BYTES = 2 * 4 * 512 * SF_COPIES;  // 2 row-tiles x 4 k-blocks
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
  // Output staging per epilogue warp: one 32 x 64 bf16 box (4 KB) in the TMA
  // 128-byte swizzle (none for direct stores).
  static constexpr int OUT_STAGE_BYTES = DIRECT ? 0 : 4096;
  static constexpr int EPI_WARPS = 8;
  // As many k-tile stages as fit beside the output staging (5 with compact
  // scales, 3 or 4 with replicated ones).
  static constexpr int STAGES_FIT = (232448 - 1024 - 256 - EPI_WARPS * OUT_STAGE_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 5 ? 5 : STAGES_FIT;
  static constexpr int ACC_ALT_COL = 128;  // start of every other accumulator
  // Scale slots: one per k-tile, A scales at +0 (16 columns), B scales at +16
  // (32 columns); two slots in the columns 384..479 the accumulators leave
  // free, used in turn.
  static constexpr int SF_COL = 384;
  static constexpr int SF_SLOT_COLS = 48;
  static constexpr int SF_SLOTS = 2;
  static constexpr int TMEM_COLS = 512;
  static_assert(SF_COL + SF_SLOTS * SF_SLOT_COLS <= TMEM_COLS, "tensor memory budget");
  static constexpr int SF_WARP0 = 2 + EPI_WARPS;  // scale loaders: one warp per lane quadrant
  static constexpr int SF_WARPS = 4;
  static constexpr int THREADS = 32 * (SF_WARP0 + SF_WARPS);
  static constexpr size_t SMEM_BYTES =
      1024 + (size_t)STAGES * STAGE_BYTES + (size_t)EPI_WARPS * OUT_STAGE_BYTES + 256;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(STAGES >= 3, "pipeline depth");
};

// Writes 8 bf16 (16 bytes) of row `row` (0..31), 16-byte chunk `chunk` (0..7)
// of a 32 x 64 box staged in the TMA 128-byte swizzle (chunk ^ row % 8).
__device__ __forceinline__ void stage_chunk(uint8_t* box, int row, int chunk, uint4 v) {
  *reinterpret_cast<uint4*>(box + row * 128 + ((chunk ^ (row & 7)) << 4)) = v;
}

// Writes 32 bytes (16 bf16) to global memory; ptr is 32-byte aligned.
__device__ __forceinline__ void st_global_v8(uint16_t* ptr, uint4 a, uint4 b) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(ptr), "r"(a.x), "r"(a.y), "r"(a.z),
               "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}

// Whether an epilogue stores its rows straight from registers (else through
// the staged TMA stores). The rescale epilogue's 256 columns per tile take the
// staged stores: from registers, 32 bytes per row per instruction, GEMM2 of
// config 2 took 224 us instead of 186 us.
template <int EPI>
__host__ __device__ constexpr bool pair_direct() {
  return EPI == EPI_SWIGLU || EPI == EPI_SWIGLU_FP4;
}

template <int EPI, bool REP>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairShape<REP, pair_direct<EPI>()>::THREADS, 1)
    gemm_nvfp4_pair_kernel(const __grid_constant__ GemmParams p) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  constexpr bool DIRECT = pair_direct<EPI>();
  using S = PairShape<REP, DIRECT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + S::STAGES * S::A_BYTES;
  uint8_t* sSFA = sB + S::STAGES * S::B_BYTES;
  uint8_t* sSFB = sSFA + S::STAGES * S::SFA_BYTES;
  uint8_t* sOut = sSFB + S::STAGES * S::SFB_BYTES;  // 1 KB aligned (stage sizes are multiples of 1 KB)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + S::EPI_WARPS * S::OUT_STAGE_BYTES);
  uint64_t* full = bars;                    // leader: both CTAs' A/B loads of a stage
  uint64_t* empty = bars + S::STAGES;       // each CTA: stage free again
  uint64_t* sf_full = bars + 2 * S::STAGES;  // each CTA: its scale loads of a stage
  uint64_t* acc_full = bars + 3 * S::STAGES;
  uint64_t* acc_empty = acc_full + 1;       // leader: 16 epilogue warps of the pair
  uint64_t* sf_ready = acc_empty + 1;       // leader: the peer's 4 loader warps wrote a scale slot
  uint64_t* sf_free = sf_ready + S::SF_SLOTS;  // each CTA: the MMAs reading a scale slot are done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sf_free + S::SF_SLOTS);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader, 1 = peer
  // EPI_SWIGLU_FP4: div_rn(1/g, 1 + m/8) of the frozen hidden global g
  __shared__ float s_r8[8];
  if constexpr (EPI == EPI_SWIGLU_FP4) {
    if (threadIdx.x < 8) s_r8[threadIdx.x] = recip8_entry(div_rn(1.0f, p.fixed_global), (int)threadIdx.x);
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&sf_full[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * S::EPI_WARPS);
    for (int s = 0; s < S::SF_SLOTS; ++s) {
      mbar_init(&sf_ready[s], S::SF_WARPS);
      mbar_init(&sf_free[s], 1);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmap_a);
    tma_prefetch_desc(&p.tmap_b);
    tma_prefetch_desc(&p.tmap_sfa);
    tma_prefetch_desc(&p.tmap_sfb);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    tmem_relinquish_pair();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const TileEntry* pairs = p.tiles + p.max_tiles;
  const int n_tiles = p.N / S::BN;
  const int num_pairs = p.num_tiles[1];
  const int total = num_pairs * n_tiles;
  const int k_tiles = (p.K + 255) / 256;
  const int kb_total = p.K / 64;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int u = cluster; u < total && ok; u += nclusters) {
        const int m = u / n_tiles, n = u - (u / n_tiles) * n_tiles;
        const TileEntry t = pairs[m];
        const int a_row = t.row0 + 128 * (int)rank;
        const int we = weight_expert(p, t.expert);
        const int b_row = we * p.N + n * S::BN + 128 * (int)rank;
        // scale atoms as 256-byte rows (2 per 512-byte atom)
        const int sfa_row = ((t.row0 / 128 + (int)rank) * kb_total) * 2 * S::SF_COPIES;
        const int sfb_row0 =
            REP ? ((we * (p.N / 256) + n) * kb_total) * 16 : ((we * (p.N / 128) + n * 2) * kb_total) * 2;
        const int sfb_row1 = sfb_row0 + kb_total * 2;
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_leader + stage * 8;
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (S::A_BYTES + S::B_BYTES));
          mbar_arrive_expect_tx(&sf_full[stage], S::SFA_BYTES + S::SFB_BYTES);
          tma_load_2d_pair(sA + stage * S::A_BYTES, &p.tmap_a, fb, kt * S::BK_BYTES, a_row);
          tma_load_2d_pair(sB + stage * S::B_BYTES, &p.tmap_b, fb, kt * S::BK_BYTES, b_row);
          // the scales go to this CTA's loader warps (its own barrier)
          if constexpr (REP) {
            // [k-block][4 copies][512 B] for A; [k-block][row-tile][4 copies][512 B] for B
            tma_load_2d(sSFA + stage * S::SFA_BYTES, &p.tmap_sfa, &sf_full[stage], 0, sfa_row + kt * 32);
            tma_load_2d(sSFB + stage * S::SFB_BYTES, &p.tmap_sfb, &sf_full[stage], 0, sfb_row0 + kt * 64);
          } else {
            // [k-block][512 B] for A; [row-tile][k-block][512 B] for B
            tma_load_2d(sSFA + stage * S::SFA_BYTES, &p.tmap_sfa, &sf_full[stage], 0, sfa_row + kt * 8);
            tma_load_2d(sSFB + stage * S::SFB_BYTES, &p.tmap_sfb, &sf_full[stage], 0, sfb_row0 + kt * 8);
            tma_load_2d(sSFB + stage * S::SFB_BYTES + 2048, &p.tmap_sfb, &sf_full[stage], 0, sfb_row1 + kt * 8);
          }
          if (++stage == S::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------- MMA issuer (leader; the whole warp, lane 0 issues) ----------------
      // Per k-tile the warp meets the leader's four loader warps at the named
      // barrier of the scale slot: they arrive once both CTAs' scales are in
      // tensor memory and the stage's A/B tiles of both CTAs have landed. An
      // mbarrier wait here stalls the MMA issue for hundreds of cycles (the
      // tensor pipe ran at half rate with one per k-tile); a named barrier
      // does not. The warp never waits on a tcgen05 operation of another
      // thread either (it would queue behind the MMAs already issued). After
      // an error the loop keeps meeting the loaders at every k-tile and keeps
      // committing (with no MMAs), so every barrier keeps its phases and no
      // warp waits for a signal that never comes.
      constexpr uint32_t idesc = idesc_nvf4(256, S::BN);
      uint32_t stage = 0, it = 0, slot = 0;
      bool ok = true;
      for (int u = cluster; u < total; u += nclusters, ++it) {
        ok = ok && mbar_wait(acc_empty, (it & 1u) ^ 1u, kErrTimeoutMma);
        tc_fence_after();
        const uint32_t d_tmem = tmem + ((it & 1u) ? S::ACC_ALT_COL : 0u);
        for (int kt = 0; kt < k_tiles; ++kt) {
          named_sync(kSfBarrier0 + slot, kSfBarrierThreads);
          tc_fence_after();
          if (lane == 0) {
            if (ok) {
              const int kb_n = min(4, kb_total - kt * 4);  // 2 or 4 (K % 128 == 0)
              const uint32_t a_base = smem_u32(sA + stage * S::A_BYTES);
              const uint32_t b_base = smem_u32(sB + stage * S::B_BYTES);
              const uint32_t sfa_t = tmem + S::SF_COL + S::SF_SLOT_COLS * slot, sfb_t = sfa_t + 16;
              for (int kb = 0; kb < kb_n; ++kb) {
                const uint64_t ad = smem_desc(a_base + kb * 32, 16, 1024, kLayoutSwizzle128B);
                const uint64_t bd = smem_desc(b_base + kb * 32, 16, 1024, kLayoutSwizzle128B);
                tc_mma_nvf4_pair(d_tmem, ad, bd, idesc, sfa_t + kb * 4, sfb_t + kb * 8, (kt | kb) != 0 ? 1u : 0u);
              }
            }
            tc_commit_pair(&sf_free[slot], 0x3);
            tc_commit_pair(&empty[stage], 0x3);
          }
          __syncwarp();
          if (++slot == S::SF_SLOTS) slot = 0;
          if (++stage == S::STAGES) stage = 0;
        }
        if (lane == 0) tc_commit_pair(acc_full, 0x3);
        __syncwarp();
      }
    }
  } else if (warp >= S::SF_WARP0) {
    // ---------------- scale loaders (warps 10..13, both CTAs) ----------------
    // Each warp writes its lane quadrant of the next scale slot of its CTA's
    // tensor memory from the stage's scale bytes in shared memory: lane l
    // takes the 16 bytes at l * 16 of every 512-byte atom (scales of rows l,
    // l + 32, l + 64, l + 96), the layout tcgen05.cp 32x128b.warpx4 writes,
    // with one tcgen05.st of 16 columns (A: 4 k-blocks x 4) and one of 32
    // (B: 4 k-blocks x 2 row-tiles x 4). tcgen05.st runs beside the MMAs,
    // where tcgen05.cp would queue behind them.
    const uint32_t lane_base = ((uint32_t)(warp & 3) * 32u) << 16;
    const uint32_t sf_ready_leader = mapa_shared(smem_u32(sf_ready), 0);
    uint32_t stage = 0, phase = 0, slot = 0, slot_phase = 0;
    bool ok = true;
    for (int u = cluster; u < total; u += nclusters) {
      for (int kt = 0; kt < k_tiles; ++kt) {
        // The leader's loaders also wait for the stage's A/B tiles, so the
        // MMA warp needs no other signal. The sf_free wait runs on every path:
        // the MMA warp commits every slot, errors included, and the wait keeps
        // the loaders from running more than two k-tiles ahead of the named
        // barriers.
        ok = ok && mbar_wait(&sf_full[stage], phase, kErrTimeoutProducer) &&
             (rank != 0 || mbar_wait(&full[stage], phase, kErrTimeoutProducer));
        ok = mbar_wait(&sf_free[slot], slot_phase ^ 1u, kErrTimeoutProducer, 2000000000ull, false) && ok;
        if (ok) {
          tc_fence_after();
          const uint8_t* sa = sSFA + stage * S::SFA_BYTES + lane * 16;
          const uint8_t* sb = sSFB + stage * S::SFB_BYTES + lane * 16;
          uint32_t ra[16], rb[32];
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            const uint4 v = *reinterpret_cast<const uint4*>(sa + kb * 512 * S::SF_COPIES);
            ra[4 * kb] = v.x;
            ra[4 * kb + 1] = v.y;
            ra[4 * kb + 2] = v.z;
            ra[4 * kb + 3] = v.w;
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const uint4 w = *reinterpret_cast<const uint4*>(sb + (REP ? kb * 4096 + t * 2048 : t * 2048 + kb * 512));
              rb[8 * kb + 4 * t] = w.x;
              rb[8 * kb + 4 * t + 1] = w.y;
              rb[8 * kb + 4 * t + 2] = w.z;
              rb[8 * kb + 4 * t + 3] = w.w;
            }
          }
          const uint32_t sfa_t = tmem + lane_base + S::SF_COL + S::SF_SLOT_COLS * slot;
          tc_st_32x32b_x16(sfa_t, ra);
          tc_st_32x32b_x32(sfa_t + 16, rb);
          tc_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (rank == 0) {
          // the peer's loaders are done with the slot too, then the MMA warp may go
          ok = mbar_wait(&sf_ready[slot], slot_phase, kErrTimeoutProducer, 2000000000ull, false) && ok;
          named_arrive(kSfBarrier0 + slot, kSfBarrierThreads);
        } else if (lane == 0) {
          mbar_arrive_cluster(sf_ready_leader + slot * 8);
        }
        if (++slot == S::SF_SLOTS) {
          slot = 0;
          slot_phase ^= 1u;
        }
        if (++stage == S::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9, both CTAs) ----------------
    const uint32_t quad = (uint32_t)(warp & 3);
    const int half = (warp - 2) >> 2;  // columns [128*half, 128*half + 128)
    const int row_in_tile = (int)(quad * 32 + lane);
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(acc_empty), 0);
    uint8_t* stg = sOut + (warp - 2) * S::OUT_STAGE_BYTES;
    uint32_t it = 0;
    for (int u = cluster; u < total; u += nclusters, ++it) {
      const int m = u / n_tiles, n = u - (u / n_tiles) * n_tiles;
      const TileEntry t = pairs[m];
      if (!mbar_wait(acc_full, it & 1u, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const bool odd = (it & 1u) != 0;
      // This warp's blocks are half and half + 2; the next accumulator covers
      // blocks 2, 3 of an even tile and blocks 0, 1 of an odd one, so the
      // warp's block inside it goes first and is released once it is read.
      const int first_blk = odd ? half : half + 2;
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) mbar_arrive(acc_empty);
          else mbar_arrive_cluster(acc_empty_leader);
        }
      };
      const int here_valid = min(max(t.valid - 128 * (int)rank, 0), 128);
      const bool live = t.pad - 128 * (int)rank > 0;  // this CTA's 128 rows are in live tiles
      const bool valid = row_in_tile < here_valid;
      const int64_t grow = (int64_t)t.row0 + 128 * (int)rank + row_in_tile;
      uint16_t* const orow = p.out + grow * p.out_cols;  // used by direct stores of live rows only
      const bool store_row = live && grow < p.out_rows;
      const uint32_t tbase = tmem + ((quad * 32u) << 16) + (odd ? S::ACC_ALT_COL : 0u);
      const float mult = (EPI == EPI_PLAIN) ? 1.0f : expert_multiplier(p, t.expert);
      const uint32_t mult_bf2 = cvt_bf16x2(mult, mult);  // exact: mult is a bf16 value
      const float fp4_inv_g = (EPI == EPI_SWIGLU_FP4) ? div_rn(1.0f, p.fixed_global) : 0.0f;
      __nv_bfloat162 hmax = __floats2bfloat162_rn(0.0f, 0.0f);  // max |h| per column parity
      if constexpr (!DIRECT) {
        // the staging boxes are free once this warp's previous stores read them
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
      }
#pragma unroll 1
      for (int i = 0; i < 2; ++i) {
        const int blk = i == 0 ? first_blk : first_blk ^ 2;
        const int bl = blk >> 1;  // 0 for block half, 1 for block half + 2
        uint32_t r0[32], r1[32];
        tc_ld_32x32b_x32(tbase + blk * 64, r0);
        tc_ld_32x32b_x32(tbase + blk * 64 + 32, r1);
        tc_wait_ld();
        if (i == 0) release();
        if constexpr (EPI == EPI_SWIGLU) {
          // block = 32 gate columns then the matching 32 up columns -> 32
          // hidden columns. The gate/up interleave maps blocks (0, 2) to
          // hidden chunks (0, 1) and (1, 3) to (2, 3) of the tile, so the two
          // blocks of a warp fill its 64 hidden columns 64*half .. 64*half+63
          // of the tile: 8-column chunks 4*bl .. 4*bl+3.
          uint4 prev = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int e0 = c * 8 + 2 * j;
              uint32_t h = swiglu_pair_bf2(__uint_as_float(r0[e0]), __uint_as_float(r0[e0 + 1]),
                                           __uint_as_float(r1[e0]), __uint_as_float(r1[e0 + 1]), mult_bf2);
              if (!valid) h = 0u;
              hmax = __hmax2(hmax, __habs2(*reinterpret_cast<__nv_bfloat162*>(&h)));
              w[j] = h;
            }
            // two chunks (32 bytes, one sector) per store
            if (c & 1) {
              if (store_row)
                st_global_v8(orow + n * (S::BN / 2) + 64 * half + 8 * (4 * bl + c - 1), prev,
                             make_uint4(w[0], w[1], w[2], w[3]));
            } else {
              prev = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        } else if constexpr (EPI == EPI_SWIGLU_FP4) {
          // the same 32 hidden values (columns 64*half + 32*bl .. + 31 of the
          // tile: two 16-blocks), quantized with the frozen global as the
          // hidden quantize would (codes 16 bytes, two scale bytes)
          uint32_t codes[4];
          uint32_t sf2 = 0;
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            uint32_t w[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int e0 = b * 16 + 2 * j;
              const uint32_t h = swiglu_pair_bf2(__uint_as_float(r0[e0]), __uint_as_float(r0[e0 + 1]),
                                                 __uint_as_float(r1[e0]), __uint_as_float(r1[e0 + 1]), mult_bf2);
              w[j] = valid ? h : 0u;
            }
            float v[16];
            float amax;
            bool has_nan;
            unpack16_bf16(w, v, amax, has_nan);
            uint32_t sfb;
            quantize16_fast(v, amax, p.fixed_global, fp4_inv_g, s_r8, has_nan, codes[2 * b], codes[2 * b + 1], sfb);
            sf2 |= sfb << (8 * b);
          }
          if (store_row) {
            const int hcol = n * (S::BN / 2) + 64 * half + 32 * bl;  // first hidden column
            const int j16 = hcol >> 4;
            *reinterpret_cast<uint4*>(p.q_out + grow * (p.out_cols / 2) + (hcol >> 1)) =
                make_uint4(codes[0], codes[1], codes[2], codes[3]);
            *reinterpret_cast<uint16_t*>(p.sf_out + sf_row_base(grow, p.out_cols / 16) + (j16 >> 2) * 512 +
                                         (j16 & 3)) = (uint16_t)sf2;
          }
        } else {
          // one 32 x 64 box per block: reuse the staging box once the
          // previous block's store has read it
          if (i == 1) {
            if (lane == 0) bulk_wait_group_read0();
            __syncwarp();
          }
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t* r = c < 4 ? r0 : r1;
            const int b0 = (c & 3) * 8;
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float v0 = __uint_as_float(r[b0 + 2 * j]), v1 = __uint_as_float(r[b0 + 2 * j + 1]);
              w[j] = EPI == EPI_RESCALE ? rescale_pair_bf2(v0, v1, mult_bf2) : cvt_bf16x2(v0, v1);
            }
            stage_chunk(stg, (int)lane, c, make_uint4(w[0], w[1], w[2], w[3]));
          }
          fence_proxy_async_shared();
          __syncwarp();
          if (lane == 0 && live) {
            tma_store_2d(&p.tmap_out, stg, n * S::BN + 64 * blk, t.row0 + 128 * (int)rank + (int)quad * 32);
            bulk_commit_group();
          }
        }
      }
      if constexpr (EPI == EPI_SWIGLU) {
        const uint32_t hm = *reinterpret_cast<uint32_t*>(&hmax);
        float rmax = fmaxf(__uint_as_float(hm << 16), __uint_as_float(hm & 0xFFFF0000u));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, o));
        if (lane == 0) atomicMax(p.amax_out + t.expert, __float_as_uint(rmax));
      }
    }
    if (lane == 0) bulk_wait_group0();
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();  // all tensor-memory reads and cross-CTA signals of the pair done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, S::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Packed FP4 rows viewed as bytes: dims {K/2, rows}, box {128 B, box_rows}.
static int make_fp4_map(CUtensorMap* map, const void* base, int64_t rows, int64_t k, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(PRAXIS_B200_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t gdim[2] = {(cuuint64_t)(k / 2), (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)(k / 2)};
  cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  cuuint32_t estride[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(PRAXIS_B200_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return PRAXIS_B200_OK;
}

template <int BLOCK_N, int EPI>
static int launch_gemm(const GemmParams& p, int max_tiles, cudaStream_t stream) {
  using S = GemmShape<BLOCK_N>;
  auto kernel = gemm_nvfp4_kernel<BLOCK_N, EPI>;
  static DeviceOnce attr;
  const int rc = device_once(attr, [&](int dev) {
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::SMEM_BYTES);
    if (e != cudaSuccess)
      return set_error(PRAXIS_B200_ECUDA, "gemm smem attribute (device %d): %s", dev, cudaGetErrorString(e));
    return (int)PRAXIS_B200_OK;
  });
  if (rc) return rc;
  const int units = max_tiles * (p.N / BLOCK_N);
  if (units <= 0) return PRAXIS_B200_OK;
  int grid = units < sm_count() ? units : sm_count();
  if (p.sm_limit > 0 && grid > p.sm_limit) grid = p.sm_limit;
  launch_pdl(kernel, dim3(grid), dim3(192), S::SMEM_BYTES, stream, p);
  return check_launch("gemm_nvfp4");
}

// Scale-factor atoms viewed as rows of 256 bytes, box {256 B, box_rows},
// no swizzle (8 rows = the 4 compact atoms of one k-tile of a 128-row tile).
static int make_bytes_map(CUtensorMap* map, const void* base, size_t bytes, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(PRAXIS_B200_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  if (bytes % 256 != 0 || bytes == 0) return set_error(PRAXIS_B200_EINVAL, "scale buffer size %zu", bytes);
  cuuint64_t gdim[2] = {256u, (cuuint64_t)(bytes / 256)};
  cuuint64_t gstride[1] = {256u};
  cuuint32_t box[2] = {256u, (cuuint32_t)box_rows};
  cuuint32_t estride[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(PRAXIS_B200_ECUDA, "cuTensorMapEncodeTiled (scales) failed (%d)", (int)r);
  return PRAXIS_B200_OK;
}

// bf16 output rows [rows, cols]: box {64 columns (128 B), 32 rows}, the TMA
// 128-byte swizzle (the epilogue stages each 32-row slab in that layout).
static int make_out_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(PRAXIS_B200_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64u, 32u};
  cuuint32_t estride[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(PRAXIS_B200_ECUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
  return PRAXIS_B200_OK;
}

// Compact scale layout: 0 = CTA-pair kernel where N % 256 == 0 (default),
// 1 = the 1-CTA kernel (PRAXIS_B200_GEMM=single).
static int gemm_variant() {
  const char* s = getenv("PRAXIS_B200_GEMM");
  return (s != nullptr && strcmp(s, "single") == 0) ? 1 : 0;
}

template <int EPI, bool REP>
static int launch_gemm_pair(const GemmParams& p, int max_tiles, cudaStream_t stream) {
  using S = PairShape<REP, pair_direct<EPI>()>;
  auto kernel = gemm_nvfp4_pair_kernel<EPI, REP>;
  static DeviceOnce attr;
  static int max_clusters[kMaxDevices] = {0};
  const int rc = device_once(attr, [&](int dev) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::SMEM_BYTES);
    if (e != cudaSuccess)
      return set_error(PRAXIS_B200_ECUDA, "pair gemm smem attribute (device %d): %s", dev, cudaGetErrorString(e));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sm_count() / 2));
    cfg.blockDim = dim3(S::THREADS);
    cfg.dynamicSmemBytes = S::SMEM_BYTES;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
    if (e != cudaSuccess || n <= 0) n = sm_count() / 2;
    max_clusters[dev] = n;
    return (int)PRAXIS_B200_OK;
  });
  if (rc) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  const int units = max_tiles * (p.N / S::BN);
  if (units <= 0) return PRAXIS_B200_OK;
  int clusters = units < max_clusters[dev] ? units : max_clusters[dev];
  if (p.sm_limit > 0 && clusters > p.sm_limit / 2) clusters = p.sm_limit / 2 > 0 ? p.sm_limit / 2 : 1;
  launch_pdl(kernel, dim3(2 * clusters), dim3(S::THREADS), S::SMEM_BYTES, stream, p);
  return check_launch("gemm_nvfp4_pair");
}

template <bool REP>
static int launch_pair_epi(const GemmParams& p, int epilogue, int max_tiles, cudaStream_t stream) {
  switch (epilogue) {
    case EPI_SWIGLU:
      return launch_gemm_pair<EPI_SWIGLU, REP>(p, max_tiles, stream);
    case EPI_SWIGLU_FP4:
      return launch_gemm_pair<EPI_SWIGLU_FP4, REP>(p, max_tiles, stream);
    case EPI_RESCALE:
      return launch_gemm_pair<EPI_RESCALE, REP>(p, max_tiles, stream);
    default:
      return launch_gemm_pair<EPI_PLAIN, REP>(p, max_tiles, stream);
  }
}

int run_grouped_gemm(const void* a_q, const void* a_sf, const void* b_q, const void* b_sf, const TileEntry* tiles,
                     const int32_t* num_tiles, int max_tiles, int64_t rows_padded, int32_t n, int32_t k,
                     int32_t experts, int epilogue, uint16_t* out, int32_t out_cols, const float* act_global,
                     const uint32_t* act_amax, const float* w_global, uint32_t* amax_out, int sf_layout,
                     cudaStream_t stream, int sm_limit, int groups_per_weight, uint8_t* q_out, uint8_t* sf_out,
                     float fixed_global, float act_global_scalar) {
  if (n % 128 != 0 || k % 128 != 0 || n <= 0 || k <= 0)
    return set_error(PRAXIS_B200_EINVAL, "grouped GEMM needs N and K multiples of 128 (N=%d K=%d)", n, k);
  if (experts < 1) return set_error(PRAXIS_B200_EINVAL, "grouped GEMM needs at least one expert");
  if (max_tiles < 0 || rows_padded < (int64_t)max_tiles * 128)
    return set_error(PRAXIS_B200_EINVAL, "tile table larger than the padded rows");
  if (epilogue == EPI_SWIGLU && (out_cols * 2 != n || amax_out == nullptr || w_global == nullptr))
    return set_error(PRAXIS_B200_EINVAL, "SwiGLU epilogue needs out_cols = N/2, amax_out and w_global");
  if (epilogue == EPI_PLAIN && out_cols != n)
    return set_error(PRAXIS_B200_EINVAL, "plain epilogue needs out_cols = N");
  const bool have_act_global = act_global != nullptr || act_amax != nullptr || act_global_scalar > 0.0f;
  if (epilogue == EPI_RESCALE && (out_cols != n || w_global == nullptr || !have_act_global))
    return set_error(PRAXIS_B200_EINVAL, "rescale epilogue needs global scales");
  if (epilogue != EPI_PLAIN && epilogue != EPI_SWIGLU && epilogue != EPI_RESCALE && epilogue != EPI_SWIGLU_FP4)
    return set_error(PRAXIS_B200_EINVAL, "unknown epilogue %d", epilogue);
  if (epilogue == EPI_SWIGLU_FP4) {
    if (out_cols * 2 != n || w_global == nullptr || !have_act_global || q_out == nullptr || sf_out == nullptr ||
        !(fixed_global > 0.0f && fixed_global < 3.4e38f))
      return set_error(PRAXIS_B200_EINVAL,
                       "FP4 SwiGLU epilogue needs out_cols = N/2, w_global, FP4 outputs and a positive global");
    if (n % 256 != 0 || out_cols % 64 != 0 || sf_layout != PRAXIS_B200_SF_COMPACT || gemm_variant() != 0)
      return set_error(PRAXIS_B200_EINVAL, "FP4 SwiGLU epilogue needs the CTA-pair kernel (N %% 256 == 0) "
                                           "with compact scales");
    if (((uintptr_t)q_out & 15) || ((uintptr_t)sf_out & 15))
      return set_error(PRAXIS_B200_EINVAL, "FP4 outputs must be 16-byte aligned");
  }
  if (act_global_scalar < 0.0f || !(act_global_scalar < 3.4e38f))
    return set_error(PRAXIS_B200_EINVAL, "bad activation global scale");
  if (sf_layout != PRAXIS_B200_SF_COMPACT && sf_layout != PRAXIS_B200_SF_REPLICATED)
    return set_error(PRAXIS_B200_EINVAL, "unknown scale layout %d", sf_layout);
  if (sf_layout == PRAXIS_B200_SF_REPLICATED && n % 256 != 0)
    return set_error(PRAXIS_B200_EINVAL, "the replicated scale layout needs N %% 256 == 0");
  if (((uintptr_t)a_sf | (uintptr_t)b_sf | (uintptr_t)out) & 15)
    return set_error(PRAXIS_B200_EINVAL, "scale and output buffers must be 16-byte aligned");
  if (epilogue == EPI_SWIGLU && ((uintptr_t)out & 31))
    return set_error(PRAXIS_B200_EINVAL, "the SwiGLU output must be 32-byte aligned");
  if (rows_padded == 0 || max_tiles == 0) return PRAXIS_B200_OK;
  GemmParams p;
  memset(&p, 0, sizeof(p));
  int rc = make_fp4_map(&p.tmap_a, a_q, rows_padded, k, 128);
  if (rc) return rc;
  rc = make_fp4_map(&p.tmap_b, b_q, (int64_t)experts * n, k, 128);
  if (rc) return rc;
  p.sfa = static_cast<const uint8_t*>(a_sf);
  p.sfb = static_cast<const uint8_t*>(b_sf);
  p.tiles = tiles;
  p.num_tiles = num_tiles;
  p.N = n;
  p.K = k;
  p.out = out;
  p.out_cols = out_cols;
  p.out_rows = rows_padded;
  p.act_global = act_global;
  p.act_amax = act_amax;
  p.w_global = w_global;
  p.amax_out = amax_out;
  p.max_tiles = max_tiles;
  p.weight_experts = experts;
  p.groups_per_weight = groups_per_weight;
  p.q_out = q_out;
  p.sf_out = sf_out;
  p.fixed_global = fixed_global;
  p.act_global_scalar = act_global_scalar;
  p.sm_limit = sm_limit;
  const bool rep = sf_layout == PRAXIS_B200_SF_REPLICATED;
  if (n % 256 == 0 && (rep || gemm_variant() == 0)) {
    const size_t copies = rep ? 4 : 1;
    rc = make_bytes_map(&p.tmap_sfa, a_sf, (size_t)rows_padded * (k / 16) * copies, rep ? 32 : 8);
    if (rc) return rc;
    rc = make_bytes_map(&p.tmap_sfb, b_sf, (size_t)experts * n * (k / 16) * copies, rep ? 64 : 8);
    if (rc) return rc;
    if (epilogue != EPI_SWIGLU_FP4) {  // the FP4 epilogue writes codes and scales with plain stores
      rc = make_out_map(&p.tmap_out, out, rows_padded, out_cols);
      if (rc) return rc;
    }
    return rep ? launch_pair_epi<true>(p, epilogue, max_tiles, stream)
               : launch_pair_epi<false>(p, epilogue, max_tiles, stream);
  }
  switch (epilogue) {
    case EPI_SWIGLU:
      return launch_gemm<128, EPI_SWIGLU>(p, max_tiles, stream);
    case EPI_RESCALE:
      return launch_gemm<128, EPI_RESCALE>(p, max_tiles, stream);
    default:
      return launch_gemm<128, EPI_PLAIN>(p, max_tiles, stream);
  }
}

}  // namespace praxis
