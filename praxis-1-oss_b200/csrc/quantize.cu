// NVFP4 quantization kernels (E2M1 codes + UE4M3 scale per 16 elements +
// FP32 per-expert global scale), bit-identical to the reference recipe:
//
//   praxis/kernels/nvfp4.py:44-124   _quantize: bs = max|v| * f32(1/6);
//                                    sf = e4m3(clamp(div_rn(bs, g), 2^-6, 448));
//                                    rc = div_rn(div_rn(1, g), sf);
//                                    code = e2m1_rn(clamp(v * rc, -6, 6));
//                                    even element in the low nibble; scales in
//                                    128x4 swizzled atoms (:114-119)
//   praxis/quantization/nvfp4.py:67-146  the same recipe for weights, one
//                                    global per expert matrix, rows = output
//                                    features of W^T
//
// quantize_gather  token-major: each token row is read once and quantized for
//                  each of its top-k experts with that expert's global scale;
//                  extra CTAs zero the padding rows of partly filled tiles
// quantize_rows    the hidden rows of every tile that holds routed rows
// pack_weights     GPU packing of expert-first bf16 banks (replaces the
//                  ~18 min CPU packing of praxis/quantization/loading.py)
// interleave       gate/up row blocks of 64 for the fused SwiGLU GEMM
#include "common.cuh"
#include "kernels.h"
#include "nvfp4_quant.cuh"

namespace praxis {

// Replicated layout (PRAXIS_B200_SF_REPLICATED): the atom of (row group,
// k-block) is stored four times in a row; a group is 128 rows (activations)
// or 256 rows = two atoms (weights, [group][k-block][half][copy][512 B]).
__device__ __forceinline__ uint32_t sf_offset_rep(int64_t row, int col, int kb, int group_rows, int copy) {
  const int64_t g = group_rows == 256 ? row >> 8 : row >> 7;
  const int half = group_rows == 256 ? (int)((row >> 7) & 1) : 0;
  return (uint32_t)((g * (kb >> 2) + (col >> 2)) * (group_rows * 16) + half * 2048 + copy * 512 + (row & 31) * 16 +
                    ((row & 127) >> 5) * 4 + (col & 3));
}

// Quantize 16 values with global g (inv_g = div_rn(1, g)) with the recipe's
// two IEEE divisions; returns the 8 code bytes in (lo, hi) and the scale
// byte. The reference clamps v * rc to [-6, 6] (NaN-ignoring min/max, so NaN
// -> -6) before the saturating conversion. For finite inputs v * rc stays
// finite (|v| <= amax, the scale is at least 2^-6), where the saturating
// conversion alone gives the same codes; blocks holding an infinity or NaN
// (has_nan) take the clamp.
__device__ __forceinline__ void quantize16(const float (&v)[16], float amax, float g, float inv_g, bool has_nan,
                                           uint32_t& lo, uint32_t& hi, uint32_t& sf) {
  const float bs = mul_rn(amax, kOneSixth);
  const float sfv = fminf(fmaxf(div_rn(bs, g), 0.015625f), 448.0f);
  sf = f32_to_e4m3_byte(sfv);
  const float rc = div_rn(inv_g, e4m3_byte_to_f32(sf));
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

// Gather the four scale bytes of lanes 4i..4i+3 into one word (the 4 scales
// of a 64-element group are adjacent in the atom) and store it: lane 4i in
// the compact layout; lane 4i+c writes copy c in the replicated one.
__device__ __forceinline__ void store_sf_group(uint8_t* sf_base, int64_t row, int col, int kb, uint32_t byte,
                                               bool active, bool rep) {
  const uint32_t lane = threadIdx.x & 31;
  uint32_t b1 = __shfl_down_sync(0xffffffffu, byte, 1);
  uint32_t b2 = __shfl_down_sync(0xffffffffu, byte, 2);
  uint32_t b3 = __shfl_down_sync(0xffffffffu, byte, 3);
  uint32_t word = byte | (b1 << 8) | (b2 << 16) | (b3 << 24);
  if (rep) {
    word = __shfl_sync(0xffffffffu, word, lane & ~3u);
    if (active)
      *reinterpret_cast<uint32_t*>(sf_base + sf_offset_rep(row, col & ~3, kb, 128, (int)(lane & 3))) = word;
  } else if (active && (lane & 3) == 0) {
    *reinterpret_cast<uint32_t*>(sf_base + sf_offset(row, col, kb)) = word;
  }
}

__device__ __forceinline__ float expert_global(const float* g, const uint32_t* amax, int e) {
  return g != nullptr ? g[e] : global_from_amax_bits(amax[e]);
}

// ---------------------------------------------------------------------------
// Gather quantize of the GEMM1 input (one warp per token)
// ---------------------------------------------------------------------------
constexpr int kGatherWarps = 8;

// Zero the padding rows of partly filled tiles (the reference allocates
// these buffers with zeros, praxis/kernels/nvfp4.py:227-231); one CTA per tile.
__device__ __forceinline__ void gather_zero_padding(int m, int k_dim, const TileEntry* __restrict__ tiles,
                                                    const int32_t* __restrict__ num_tiles, uint8_t* __restrict__ q,
                                                    uint8_t* __restrict__ sf, bool rep) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb = k_dim / 16;
  if (m >= *num_tiles) return;
  const TileEntry t = tiles[m];
  for (int r = t.valid + warp; r < kTileRows; r += kGatherWarps) {
    const int64_t row = (int64_t)t.row0 + r;
    uint4* qr = reinterpret_cast<uint4*>(q + row * (k_dim / 2));
    for (int i = lane; i < k_dim / 32; i += 32) qr[i] = make_uint4(0, 0, 0, 0);
    for (int g4 = lane; g4 < kb / 4; g4 += 32) {
      if (rep) {
#pragma unroll
        for (int c = 0; c < 4; ++c) *reinterpret_cast<uint32_t*>(sf + sf_offset_rep(row, g4 * 4, kb, 128, c)) = 0u;
      } else {
        *reinterpret_cast<uint32_t*>(sf + sf_offset(row, g4 * 4, kb)) = 0u;
      }
    }
  }
}

// Token-major gather: each token row is read once and quantized for each of
// its K routed rows with that row's global scale. One warp per token, lane
// j0 + l owning 16-block j0 + l of each 512-element chunk. The first chunk's
// loads go out before the routed rows are resolved (top-k -> group ->
// csr / pcsr / global: two dependent loads), and each chunk's loads before
// the previous chunk is quantized. Lane s resolves routed row s; the rows'
// code and scale pointers and global scales then sit in every lane's
// registers (K is a template argument), the per-row tables of the second
// division (recip8) in shared memory. CTAs token_blocks.. zero the padding
// rows of partly filled tiles, one tile each.
template <int K>
__global__ void __launch_bounds__(256) quantize_gather_kernel(
    const uint16_t* __restrict__ x, int64_t tokens, int k_dim, const int64_t* __restrict__ top_idx,
    const int64_t* __restrict__ inverse, const int32_t* __restrict__ csr, const int32_t* __restrict__ pcsr,
    const float* __restrict__ globals, const uint32_t* __restrict__ amax_bits, int experts, Passes passes,
    const TileEntry* __restrict__ tiles, const int32_t* __restrict__ num_tiles, int token_blocks,
    uint8_t* __restrict__ q, uint8_t* __restrict__ sf, bool rep) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  __shared__ float s_r8[kGatherWarps][K][8];  // [warp][routed row][m]: div_rn(1/g, 1 + m/8)
  if ((int)blockIdx.x >= token_blocks) {
    gather_zero_padding(blockIdx.x - token_blocks, k_dim, tiles, num_tiles, q, sf, rep);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kGatherWarps + warp;
  if (t >= tokens) return;
  const int kb = k_dim / 16;
  const uint4* xr = reinterpret_cast<const uint4*>(x + t * k_dim);
  uint4 na = make_uint4(0, 0, 0, 0), nb = na;
  if (lane < kb) {
    na = __ldg(xr + 2 * lane);
    nb = __ldg(xr + 2 * lane + 1);
  }
  int64_t my_dest = 0;
  float my_g = 1.0f;
  if (lane < K) {
    const int e = route_group(checked_expert(top_idx[t * K + lane], experts), t, passes);
    my_g = expert_global(globals, amax_bits, e);
    my_dest = (int64_t)pcsr[e] + inverse[t * K + lane] - csr[e];
  }
  const float my_ig = div_rn(1.0f, my_g);
#pragma unroll
  for (int i0 = 0; i0 < K * 8; i0 += 32) {
    const int i = i0 + lane;
    const float ig_i = __shfl_sync(0xffffffffu, my_ig, (i >> 3) & 31);
    if (i < K * 8) s_r8[warp][i >> 3][i & 7] = recip8_entry(ig_i, i & 7);
  }
  __syncwarp();
  uint8_t* qrow[K];
  int64_t sfrow[K], dest[K];
  float g[K], ig[K];
#pragma unroll
  for (int s = 0; s < K; ++s) {
    dest[s] = (int64_t)__shfl_sync(0xffffffffu, (unsigned long long)my_dest, s);
    qrow[s] = q + dest[s] * (k_dim / 2);
    sfrow[s] = sf_row_base(dest[s], kb);
    g[s] = __shfl_sync(0xffffffffu, my_g, s);
    ig[s] = __shfl_sync(0xffffffffu, my_ig, s);
  }
  for (int j0 = 0; j0 < kb; j0 += 32) {
    const uint32_t w[8] = {na.x, na.y, na.z, na.w, nb.x, nb.y, nb.z, nb.w};
    const int jn = j0 + 32 + lane;
    if (jn < kb) {
      na = __ldg(xr + 2 * jn);
      nb = __ldg(xr + 2 * jn + 1);
    }
    const int j = j0 + lane;
    const bool active = j < kb;
    float v[16];
    float amax;
    bool has_nan;
    unpack16_bf16(w, v, amax, has_nan);
    const float bs = mul_rn(amax, kOneSixth);
    const int64_t sf_col = (int64_t)(j >> 2) * 512 + (j & 3);
#pragma unroll
    for (int s = 0; s < K; ++s) {
      uint32_t lo = 0, hi = 0, sfb = 0;
      if (active) {
        quantize16_bs(v, bs, g[s], ig[s], s_r8[warp][s], has_nan, lo, hi, sfb);
        *reinterpret_cast<uint2*>(qrow[s] + (int64_t)j * 8) = make_uint2(lo, hi);
        if (!rep) sf[sfrow[s] + sf_col] = (uint8_t)sfb;
      }
      if (rep) store_sf_group(sf, dest[s], j, kb, sfb, active, true);
    }
  }
}

// ---------------------------------------------------------------------------
// Row quantize of the hidden activations (one warp per padded row of a tile)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) quantize_rows_kernel(
    const uint16_t* __restrict__ x, int k_dim, const TileEntry* __restrict__ tiles,
    const int32_t* __restrict__ num_tiles, const float* __restrict__ globals, const uint32_t* __restrict__ amax_bits,
    uint8_t* __restrict__ q, uint8_t* __restrict__ sf, bool rep) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * 8 + warp;  // tile * 128 + row
  const int m = (int)(item / kTileRows);
  if (m >= *num_tiles) return;
  const TileEntry t = tiles[m];
  const int64_t row = (int64_t)t.row0 + (item % kTileRows);
  const float g = expert_global(globals, amax_bits, t.expert);
  const float ig = div_rn(1.0f, g);
  // the block's 8 rows share one group (tiles are 128 rows): one table of
  // the second division for all of them
  __shared__ float s_r8[8];
  if (threadIdx.x < 8) s_r8[threadIdx.x] = recip8_entry(ig, threadIdx.x);
  __syncthreads();
  const int kb = k_dim / 16;
  const uint16_t* xr = x + row * k_dim;
  uint8_t* qr = q + row * (k_dim / 2);
  const int64_t sf_row = sf_row_base(row, kb);
  for (int j0 = 0; j0 < kb; j0 += 32) {
    const int j = j0 + lane;
    const bool active = j < kb;
    uint32_t lo = 0, hi = 0, sfb = 0;
    if (active) {
      float v[16];
      float amax;
      bool has_nan;
      load16_bf16_fast(xr + j * 16, v, amax, has_nan);
      quantize16_fast(v, amax, g, ig, s_r8, has_nan, lo, hi, sfb);
      *reinterpret_cast<uint2*>(qr + (int64_t)j * 8) = make_uint2(lo, hi);
      if (!rep) sf[sf_row + (int64_t)(j >> 2) * 512 + (j & 3)] = (uint8_t)sfb;
    }
    if (rep) store_sf_group(sf, row, j, kb, sfb, active, true);
  }
}

// ---------------------------------------------------------------------------
// Weight packing (expert-first bf16 [E, K, N] -> W^T rows of N outputs)
// ---------------------------------------------------------------------------
__global__ void pack_amax_kernel(const uint16_t* __restrict__ w, int64_t per_expert, uint32_t* __restrict__ amax) {
  const int e = blockIdx.y;
  const uint16_t* src = w + (int64_t)e * per_expert;
  float m = 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per_expert; i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(bf16_to_f32(src[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(amax + e, __float_as_uint(m));
}

__global__ void pack_quant_kernel(const uint16_t* __restrict__ w, int k_dim, int n_dim,
                                  const uint32_t* __restrict__ amax, uint8_t* __restrict__ q,
                                  uint8_t* __restrict__ sf, float* __restrict__ global_out) {
  const int e = blockIdx.z;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int j = blockIdx.y;  // 16-element block along K
  const float g = global_from_amax_bits(amax[e]);
  if (n == 0 && j == 0) global_out[e] = g;
  if (n >= n_dim) return;
  const uint16_t* src = w + (int64_t)e * k_dim * n_dim + (int64_t)j * 16 * n_dim + n;
  float v[16];
  float m = 0.0f;
  bool has_nan = false;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = bf16_to_f32(src[(int64_t)i * n_dim]);
    m = fmaxf(m, fabsf(v[i]));
    has_nan |= !isfinite(v[i]);
  }
  uint32_t lo, hi, sfb;
  quantize16(v, m, g, div_rn(1.0f, g), has_nan, lo, hi, sfb);
  const int kb = k_dim / 16;
  *reinterpret_cast<uint2*>(q + ((int64_t)e * n_dim + n) * (k_dim / 2) + (int64_t)j * 8) = make_uint2(lo, hi);
  sf[(int64_t)e * n_dim * kb + sf_offset(n, j, kb)] = (uint8_t)sfb;
}

// ---------------------------------------------------------------------------
// Gate/up interleave: kernel-layout row r of an expert's [2F, C] gate_up
// matrix, in 64-row block b = r / 64 serving hidden chunk h = hidden_chunk(b)
// (blocks 1 and 2 of each group of four swapped, so that each GEMM epilogue
// warp's two blocks give adjacent hidden columns), is gate row 32*h + r%64
// for r%64 < 32, else up row F + 32*h + r%64 - 32. One CTA per (row, expert).
// ---------------------------------------------------------------------------
__global__ void interleave_gate_up_kernel(const uint8_t* __restrict__ q, const uint8_t* __restrict__ sf, int f_dim,
                                          int c_dim, uint8_t* __restrict__ q_out, uint8_t* __restrict__ sf_out) {
  const int r = blockIdx.x, e = blockIdx.y;
  const int blk = r / 64, w = r % 64;
  const int h = (blk & ~3) | ((blk & 1) << 1) | ((blk & 3) >> 1);
  const int src = w < 32 ? 32 * h + w : f_dim + 32 * h + (w - 32);
  const int64_t rows = 2 * (int64_t)f_dim;
  const uint4* qs = reinterpret_cast<const uint4*>(q + ((int64_t)e * rows + src) * (c_dim / 2));
  uint4* qd = reinterpret_cast<uint4*>(q_out + ((int64_t)e * rows + r) * (c_dim / 2));
  for (int i = threadIdx.x; i < c_dim / 32; i += blockDim.x) qd[i] = qs[i];
  const int kb = c_dim / 16;
  const uint8_t* ss = sf + (int64_t)e * rows * kb;
  uint8_t* sd = sf_out + (int64_t)e * rows * kb;
  for (int j = threadIdx.x; j < kb; j += blockDim.x) sd[sf_offset(r, j, kb)] = ss[sf_offset(src, j, kb)];
}

// ---------------------------------------------------------------------------
// Compact -> replicated scales: one thread per 16-byte chunk (one row of 32
// within the atom: 4 quadrants x 4 scales), written to the four copies.
// ---------------------------------------------------------------------------
__global__ void replicate_scales_kernel(const uint4* __restrict__ sf, int64_t chunks, int kb, int group_rows,
                                        uint4* __restrict__ out) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= chunks) return;
  const int64_t atom = i >> 5;
  const int r32 = (int)(i & 31);
  const int kblocks = kb >> 2;
  const int64_t tile = atom / kblocks;  // 128-row tile
  const int col = (int)(atom % kblocks) * 4;
  const uint4 v = ldg_stream(sf + i);
  const int64_t row = tile * 128 + r32;
#pragma unroll
  for (int c = 0; c < 4; ++c) out[sf_offset_rep(row, col, kb, group_rows, c) >> 4] = v;
}

// ---------------------------------------------------------------------------
// Host entries
// ---------------------------------------------------------------------------
int run_quantize_gather(const uint16_t* x, int64_t tokens, int k_dim, const int64_t* top_idx, const int64_t* inverse,
                        const int32_t* csr, const int32_t* pcsr, const float* globals, const uint32_t* amax_bits,
                        int top_k, int experts, const TileEntry* tiles, const int32_t* num_tiles, int max_tiles,
                        uint8_t* q, uint8_t* sf, int sf_layout, cudaStream_t stream, Passes passes) {
  if (k_dim % 64 != 0) return set_error(PRAXIS_B200_EINVAL, "quantize needs K % 64 == 0");
  if (top_k < 1 || top_k > 8) return set_error(PRAXIS_B200_EINVAL, "top_k must be 1..8");
  if (globals == nullptr && amax_bits == nullptr) return set_error(PRAXIS_B200_EINVAL, "no global scales");
  if (sf_layout != PRAXIS_B200_SF_COMPACT && sf_layout != PRAXIS_B200_SF_REPLICATED)
    return set_error(PRAXIS_B200_EINVAL, "unknown scale layout %d", sf_layout);
  if (((uintptr_t)x | (uintptr_t)q) & 15)
    return set_error(PRAXIS_B200_EINVAL, "quantize_gather: x and q must be 16-byte aligned");
  const int64_t token_blocks = (tokens + kGatherWarps - 1) / kGatherWarps;
  const int64_t grid = token_blocks + max_tiles;
  if (grid == 0) return PRAXIS_B200_OK;
  using Kernel = decltype(&quantize_gather_kernel<1>);
  static const Kernel kernels[8] = {quantize_gather_kernel<1>, quantize_gather_kernel<2>, quantize_gather_kernel<3>,
                                    quantize_gather_kernel<4>, quantize_gather_kernel<5>, quantize_gather_kernel<6>,
                                    quantize_gather_kernel<7>, quantize_gather_kernel<8>};
  launch_pdl(kernels[top_k - 1], dim3((unsigned)grid), dim3(256), 0, stream, x, tokens, k_dim, top_idx, inverse, csr,
             pcsr, globals, amax_bits, experts, passes, tiles, num_tiles, (int)token_blocks, q, sf,
             sf_layout == PRAXIS_B200_SF_REPLICATED);
  return check_launch("quantize_gather");
}

int run_quantize_rows(const uint16_t* x, int k_dim, const TileEntry* tiles, const int32_t* num_tiles, int max_tiles,
                      const float* globals, const uint32_t* amax_bits, uint8_t* q, uint8_t* sf, int sf_layout,
                      cudaStream_t stream) {
  if (k_dim % 64 != 0) return set_error(PRAXIS_B200_EINVAL, "quantize needs K % 64 == 0");
  if (globals == nullptr && amax_bits == nullptr) return set_error(PRAXIS_B200_EINVAL, "no global scales");
  if (sf_layout != PRAXIS_B200_SF_COMPACT && sf_layout != PRAXIS_B200_SF_REPLICATED)
    return set_error(PRAXIS_B200_EINVAL, "unknown scale layout %d", sf_layout);
  if (((uintptr_t)x | (uintptr_t)q) & 15)
    return set_error(PRAXIS_B200_EINVAL, "quantize_rows: x and q must be 16-byte aligned");
  const int64_t blocks = (int64_t)max_tiles * kTileRows / 8;
  if (blocks == 0) return PRAXIS_B200_OK;
  launch_pdl(quantize_rows_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, x, k_dim, tiles, num_tiles, globals,
             amax_bits, q, sf, sf_layout == PRAXIS_B200_SF_REPLICATED);
  return check_launch("quantize_rows");
}

int run_pack_weights(const uint16_t* w, int experts, int k_dim, int n_dim, uint8_t* q, uint8_t* sf, float* global_out,
                     uint32_t* amax_scratch, cudaStream_t stream) {
  if (k_dim % 64 != 0 || n_dim % 128 != 0) return set_error(PRAXIS_B200_EINVAL, "pack needs K%64==0, N%128==0");
  if (experts <= 0) return PRAXIS_B200_OK;
  cudaError_t err = cudaMemsetAsync(amax_scratch, 0, sizeof(uint32_t) * experts, stream);
  if (err != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "memset: %s", cudaGetErrorString(err));
  const int64_t per = (int64_t)k_dim * n_dim;
  dim3 g1((unsigned)((per + 256 * 16 - 1) / (256 * 16)), (unsigned)experts);
  pack_amax_kernel<<<g1, 256, 0, stream>>>(w, per, amax_scratch);
  int rc = check_launch("pack_amax");
  if (rc) return rc;
  dim3 g2((unsigned)((n_dim + 127) / 128), (unsigned)(k_dim / 16), (unsigned)experts);
  pack_quant_kernel<<<g2, 128, 0, stream>>>(w, k_dim, n_dim, amax_scratch, q, sf, global_out);
  return check_launch("pack_quant");
}

int run_interleave_gate_up(const uint8_t* q, const uint8_t* sf, int experts, int f_dim, int c_dim, uint8_t* q_out,
                           uint8_t* sf_out, cudaStream_t stream) {
  if (f_dim % 128 != 0 || c_dim % 64 != 0) return set_error(PRAXIS_B200_EINVAL, "interleave needs F % 128, C % 64 == 0");
  if (experts <= 0) return PRAXIS_B200_OK;
  dim3 grid((unsigned)(2 * f_dim), (unsigned)experts);
  interleave_gate_up_kernel<<<grid, 128, 0, stream>>>(q, sf, f_dim, c_dim, q_out, sf_out);
  return check_launch("interleave_gate_up");
}

int run_replicate_scales(const uint8_t* sf, int64_t rows, int k_dim, int group_rows, uint8_t* out,
                         cudaStream_t stream) {
  if (k_dim % 64 != 0) return set_error(PRAXIS_B200_EINVAL, "replicate_scales needs K % 64 == 0");
  if (group_rows != 128 && group_rows != 256) return set_error(PRAXIS_B200_EINVAL, "group_rows must be 128 or 256");
  if (rows < 0 || rows % group_rows != 0)
    return set_error(PRAXIS_B200_EINVAL, "replicate_scales: rows (%lld) must be a multiple of %d", (long long)rows,
                     group_rows);
  const int64_t chunks = rows * (k_dim / 16) / 16;
  if (chunks == 0) return PRAXIS_B200_OK;
  launch_pdl(replicate_scales_kernel, dim3((unsigned)((chunks + 255) / 256)), dim3(256), 0, stream,
             reinterpret_cast<const uint4*>(sf), chunks, k_dim / 16, group_rows, reinterpret_cast<uint4*>(out));
  return check_launch("replicate_scales");
}

}  // namespace praxis
