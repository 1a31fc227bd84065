// Token dispatch: stable expert-major permutation, CSR offsets, padded CSR,
// 128-row tile table and per-expert activation global scales.
//
// Replaces, with identical values:
//   praxis/layers.py:1330-1346            _dispatch_rows (stable sort by expert,
//                                         tokens, sorted gates, int32 end offsets)
//   praxis/quantization/nvfp4.py:705-708  inverse[order] = arange(R)
//   praxis/kernels/nvfp4.py:37-41         _pad_csr (alignment 128)
//   praxis/kernels/nvfp4.py:344-352       per-tile expert metadata (here: only
//                                         tiles that hold routed rows)
//   praxis/kernels/nvfp4_moe.py:15-57     row max |x| and per-expert global scale
//
// Three launches (one, of all three passes in one CTA, when the routed rows
// fit 32 segments), no host synchronisation and no atomics on the data path:
//   1. count   one warp per segment of positions: per-segment expert
//              histogram and max row-amax (warp-aggregated shared atomics)
//   2. scan    one CTA: per-expert exclusive scan over segments, block scan
//              over experts -> csr, pcsr, offsets, tiles, global scales
//   3. scatter one warp per segment, positions in order; rank among equal
//              experts by __match_any_sync -> bit-exact stable order
#include "common.cuh"
#include "kernels.h"

namespace praxis {

constexpr int kDispatchWarps = 8;
constexpr int kDispatchUnroll = 8;  // 32-position passes whose loads are issued together
constexpr int kMaxExperts = 1024;

// ---------------------------------------------------------------------------
// Row max |x| (bf16), praxis/kernels/nvfp4_moe.py:15-21
// ---------------------------------------------------------------------------
__global__ void row_amax_kernel(const uint16_t* __restrict__ x, int64_t rows, int cols, uint16_t* __restrict__ out) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  const int warps = blockDim.x >> 5;
  const int64_t row = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* src = reinterpret_cast<const uint4*>(x + row * cols);
  float m = 0.0f;
  for (int i = lane; i < cols / 8; i += 32) {
    uint4 v = __ldg(src + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      m = fmaxf(m, fabsf(bf16_to_f32((uint16_t)(w[j] & 0xFFFFu))));
      m = fmaxf(m, fabsf(bf16_to_f32((uint16_t)(w[j] >> 16))));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) out[row] = f32_to_bf16(m);
}

// Token of routed position p (positions < 2^31, checked on the host: a
// 32-bit division).
__device__ __forceinline__ int64_t token_of(int64_t p, int top_k) {
  return (int64_t)((uint32_t)p / (uint32_t)top_k);
}

// ---------------------------------------------------------------------------
// 1. count
// ---------------------------------------------------------------------------
// `experts` counts the routed experts, `groups` = experts * passes.n the
// histogram bins (route_group).
// One warp's segment: its per-group histogram h and max row-amax hm (this
// warp's zeroed shared rows), then written to seg_count / seg_max.
__device__ __forceinline__ void count_segment(const int64_t* __restrict__ top_idx,
                                              const uint16_t* __restrict__ row_amax, int64_t positions, int top_k,
                                              int experts, Passes passes, int groups, int seg_len, int seg,
                                              uint32_t* h, uint32_t* hm, int32_t* __restrict__ seg_count,
                                              uint32_t* __restrict__ seg_max) {
  const int lane = threadIdx.x & 31;
  const int64_t begin = (int64_t)seg * seg_len;
  const int64_t end = min(positions, begin + seg_len);
  // the loads of 8 passes of 32 positions go out before the histogram work
  for (int64_t base = begin; base < end; base += 32 * kDispatchUnroll) {
    int ev[kDispatchUnroll];
    uint32_t mv[kDispatchUnroll];
#pragma unroll
    for (int u = 0; u < kDispatchUnroll; ++u) {
      const int64_t p = base + 32 * u + lane;
      const bool live = p < end;
      ev[u] = live ? route_group(checked_expert(top_idx[p], experts), token_of(p, top_k), passes) : -1;
      mv[u] = (live && row_amax != nullptr) ? __float_as_uint(bf16_to_f32(row_amax[token_of(p, top_k)])) : 0u;
    }
#pragma unroll
    for (int u = 0; u < kDispatchUnroll; ++u) {
      if (base + 32 * u >= end) break;
      const int e = ev[u];
      const bool live = e >= 0;
      const uint32_t peers = __match_any_sync(0xffffffffu, e);
      const int leader = __ffs(peers) - 1;
      if (live && lane == leader) atomicAdd(&h[e], (uint32_t)__popc(peers));
      if (live && row_amax != nullptr) atomicMax(&hm[e], mv[u]);
    }
  }
  __syncwarp();
  for (int e = lane; e < groups; e += 32) {
    seg_count[(int64_t)seg * groups + e] = (int32_t)h[e];
    seg_max[(int64_t)seg * groups + e] = hm[e];
  }
}

__global__ void dispatch_count_kernel(const int64_t* __restrict__ top_idx, const uint16_t* __restrict__ row_amax,
                                      int64_t positions, int top_k, int experts, Passes passes, int groups,
                                      int seg_len, int segments, int32_t* __restrict__ seg_count,
                                      uint32_t* __restrict__ seg_max) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  extern __shared__ uint32_t s_dc[];
  uint32_t* hist = s_dc;                                 // [warps][groups]
  uint32_t* hmax = s_dc + kDispatchWarps * groups;       // [warps][groups]
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kDispatchWarps * groups; i += blockDim.x) {
    hist[i] = 0;
    hmax[i] = 0;
  }
  __syncthreads();
  const int seg = blockIdx.x * kDispatchWarps + warp;
  if (seg < segments)
    count_segment(top_idx, row_amax, positions, top_k, experts, passes, groups, seg_len, seg, hist + warp * groups,
                  hmax + warp * groups, seg_count, seg_max);
}

// Block-wide exclusive scan of one value per thread (blockDim.x <= 1024).
__device__ int block_exclusive_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nwarps) s_warp[lane] = w;
  }
  __syncthreads();
  const int before = (warp > 0 ? s_warp[warp - 1] : 0) + x - v;
  if (total) *total = s_warp[nwarps - 1];
  __syncthreads();
  return before;
}

// ---------------------------------------------------------------------------
// 2. scan (single CTA of 1024 threads; experts <= 1024)
// ---------------------------------------------------------------------------
__device__ void scan_segments(
    int32_t* __restrict__ seg_count, const uint32_t* __restrict__ seg_max, int segments, int experts,
    int64_t positions, int align, int32_t* __restrict__ offsets, int32_t* __restrict__ csr,
    int32_t* __restrict__ pcsr, TileEntry* __restrict__ tiles, int max_tiles, int32_t* __restrict__ num_tiles,
    float* __restrict__ act_global, uint32_t* __restrict__ act_amax_bits) {
  __shared__ int s_warp[32];
  __shared__ int s_part[1024];
  __shared__ uint32_t s_pmax[1024];
  // Exclusive scan over segments per expert, in place (seg_count becomes the
  // offset of the segment's first row inside its expert). Thread t handles
  // expert t % E over one contiguous range of segments (consecutive threads
  // read consecutive experts of a segment row).
  const int parts = max(1, (int)blockDim.x / experts);
  const int t = threadIdx.x;
  const int te = t % experts, tp = t / experts;
  const int span = (segments + parts - 1) / parts;
  const int s0 = tp * span, s1 = min(segments, s0 + span);
  // (the loads of kScanBatch segments go out together: a thread's range is
  // read in a few memory latencies instead of one per segment)
  constexpr int kScanBatch = 8;
  int local = 0;
  uint32_t lmax = 0;
  if (tp < parts) {
    for (int s = s0; s < s1; s += kScanBatch) {
      int c[kScanBatch];
      uint32_t mx[kScanBatch];
#pragma unroll
      for (int u = 0; u < kScanBatch; ++u) {
        const int64_t i = (int64_t)(s + u) * experts + te;
        c[u] = s + u < s1 ? seg_count[i] : 0;
        mx[u] = s + u < s1 ? seg_max[i] : 0u;
      }
#pragma unroll
      for (int u = 0; u < kScanBatch; ++u) {
        local += c[u];
        lmax = max(lmax, mx[u]);
      }
    }
    s_part[t] = local;
    s_pmax[t] = lmax;
  }
  __syncthreads();
  if (tp < parts) {
    int before = 0;
    for (int q = 0; q < tp; ++q) before += s_part[q * experts + te];
    int run = before;
    for (int s = s0; s < s1; s += kScanBatch) {
      int c[kScanBatch];
#pragma unroll
      for (int u = 0; u < kScanBatch; ++u) c[u] = s + u < s1 ? seg_count[(int64_t)(s + u) * experts + te] : 0;
#pragma unroll
      for (int u = 0; u < kScanBatch; ++u) {
        if (s + u < s1) seg_count[(int64_t)(s + u) * experts + te] = run;
        run += c[u];
      }
    }
  }
  const int e = threadIdx.x;
  int count = 0;
  uint32_t m = 0;
  if (e < experts) {
    for (int q = 0; q < parts; ++q) {
      count += s_part[q * experts + e];
      m = max(m, s_pmax[q * experts + e]);
    }
  }
  __syncthreads();
  int total = 0;
  const int start = block_exclusive_scan(e < experts ? count : 0, s_warp, &total);
  if (e < experts) {
    csr[e] = start;
    offsets[e] = start + count;
    if (e == experts - 1) csr[experts] = start + count;
    const int64_t pstart = ((int64_t)start + (int64_t)(align - 1) * e) / align * align;
    pcsr[e] = (int32_t)pstart;
    if (e == experts - 1)
      pcsr[experts] = (int32_t)(((int64_t)start + count + (int64_t)(align - 1) * experts) / align * align);
    if (act_amax_bits) act_amax_bits[e] = m;
    if (act_global) act_global[e] = global_from_amax_bits(m);
  }
  // Tile table: ceil(count / 128) tiles per expert, in expert order.
  const int ntile = e < experts ? (count + kTileRows - 1) / kTileRows : 0;
  int tiles_total = 0;
  const int tstart = block_exclusive_scan(ntile, s_warp, &tiles_total);
  if (e < experts) {
    const int64_t pstart = ((int64_t)start + (int64_t)(align - 1) * e) / align * align;
    for (int j = 0; j < ntile; ++j) {
      if (tstart + j < max_tiles) {
        TileEntry t;
        t.expert = e;
        t.row0 = (int32_t)(pstart + (int64_t)j * kTileRows);
        t.valid = min(kTileRows, count - j * kTileRows);
        t.pad = 0;
        tiles[tstart + j] = t;
      } else {
        record_error(kErrIndexRange);
      }
    }
  }
  // Pair table (256-row units of the 2-CTA GEMM) after the tile table:
  // {expert, first padded row, routed rows of the 256 (1..256), live rows
  // (rows of the expert's 128-row tiles inside the 256)}.
  const int npair = e < experts ? (count + 2 * kTileRows - 1) / (2 * kTileRows) : 0;
  int pairs_total = 0;
  const int pstart_idx = block_exclusive_scan(npair, s_warp, &pairs_total);
  if (e < experts) {
    const int64_t pstart = ((int64_t)start + (int64_t)(align - 1) * e) / align * align;
    const int live_total = ntile * kTileRows;
    for (int j = 0; j < npair; ++j) {
      if (pstart_idx + j < max_tiles) {
        TileEntry t;
        t.expert = e;
        t.row0 = (int32_t)(pstart + (int64_t)j * 2 * kTileRows);
        t.valid = min(2 * kTileRows, count - j * 2 * kTileRows);
        t.pad = min(2 * kTileRows, live_total - j * 2 * kTileRows);
        tiles[max_tiles + pstart_idx + j] = t;
      }
    }
  }
  if (threadIdx.x == 0) {
    num_tiles[0] = min(tiles_total, max_tiles);
    num_tiles[1] = min(pairs_total, max_tiles);
  }
}

__global__ void __launch_bounds__(1024) dispatch_scan_kernel(
    int32_t* __restrict__ seg_count, const uint32_t* __restrict__ seg_max, int segments, int experts,
    int64_t positions, int align, int32_t* __restrict__ offsets, int32_t* __restrict__ csr,
    int32_t* __restrict__ pcsr, TileEntry* __restrict__ tiles, int max_tiles, int32_t* __restrict__ num_tiles,
    float* __restrict__ act_global, uint32_t* __restrict__ act_amax_bits) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  scan_segments(seg_count, seg_max, segments, experts, positions, align, offsets, csr, pcsr, tiles, max_tiles,
                num_tiles, act_global, act_amax_bits);
}


// ---------------------------------------------------------------------------
// Tile tables of received segments (expert parallelism): segment v holds
// counts[v] routed rows from padded row starts[v] (128-aligned); the 128-row
// tiles and 256-row pairs are laid out as by the dispatch, with v as the
// tile's expert. One CTA of 1024 threads, segments <= 1024.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) segment_tiles_kernel(const int32_t* __restrict__ counts,
                                                             const int32_t* __restrict__ starts, int segments,
                                                             TileEntry* __restrict__ tiles, int max_tiles,
                                                             int32_t* __restrict__ num_tiles) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  __shared__ int s_warp[32];
  const int v = threadIdx.x;
  const int count = v < segments ? max(counts[v], 0) : 0;
  const int64_t row0 = v < segments ? starts[v] : 0;
  const int ntile = (count + kTileRows - 1) / kTileRows;
  int tiles_total = 0;
  const int tstart = block_exclusive_scan(ntile, s_warp, &tiles_total);
  for (int j = 0; j < ntile; ++j) {
    if (tstart + j < max_tiles) {
      TileEntry t;
      t.expert = v;
      t.row0 = (int32_t)(row0 + (int64_t)j * kTileRows);
      t.valid = min(kTileRows, count - j * kTileRows);
      t.pad = 0;
      tiles[tstart + j] = t;
    } else {
      record_error(kErrIndexRange);
    }
  }
  const int npair = (count + 2 * kTileRows - 1) / (2 * kTileRows);
  int pairs_total = 0;
  const int pstart = block_exclusive_scan(npair, s_warp, &pairs_total);
  for (int j = 0; j < npair; ++j) {
    if (pstart + j < max_tiles) {
      TileEntry t;
      t.expert = v;
      t.row0 = (int32_t)(row0 + (int64_t)j * 2 * kTileRows);
      t.valid = min(2 * kTileRows, count - j * 2 * kTileRows);
      t.pad = min(2 * kTileRows, ntile * kTileRows - j * 2 * kTileRows);
      tiles[max_tiles + pstart + j] = t;
    }
  }
  if (threadIdx.x == 0) {
    num_tiles[0] = min(tiles_total, max_tiles);
    num_tiles[1] = min(pairs_total, max_tiles);
  }
}

int run_segment_tiles(const int32_t* counts, const int32_t* starts, int segments, TileEntry* tiles, int max_tiles,
                      int32_t* num_tiles, cudaStream_t stream) {
  if (segments < 1 || segments > 1024) return set_error(PRAXIS_B200_EINVAL, "segments must be 1..1024");
  launch_pdl(segment_tiles_kernel, dim3(1), dim3(1024), 0, stream, counts, starts, segments, tiles, max_tiles,
             num_tiles);
  return check_launch("segment_tiles");
}

// ---------------------------------------------------------------------------
// 3. scatter
// ---------------------------------------------------------------------------
// One warp's segment: its routed positions in order into their rows, from
// the warp's cursor row (cur[g] = csr[g] + the segment's start in group g).
__device__ __forceinline__ void scatter_segment(const int64_t* __restrict__ top_idx,
                                                const uint16_t* __restrict__ gate, int64_t positions, int top_k,
                                                int experts, Passes passes, int seg_len, int seg, int32_t* cur,
                                                int64_t* __restrict__ order, int64_t* __restrict__ inverse,
                                                int64_t* __restrict__ tokens, int32_t* __restrict__ tokens32,
                                                uint16_t* __restrict__ sorted_gate) {
  const int lane = threadIdx.x & 31;
  const int64_t begin = (int64_t)seg * seg_len;
  const int64_t end = min(positions, begin + seg_len);
  const uint32_t lt = (1u << lane) - 1u;
  for (int64_t base = begin; base < end; base += 32 * kDispatchUnroll) {
    int ev[kDispatchUnroll];
    uint16_t gv[kDispatchUnroll];
#pragma unroll
    for (int u = 0; u < kDispatchUnroll; ++u) {
      const int64_t p = base + 32 * u + lane;
      const bool live = p < end;
      ev[u] = live ? route_group(checked_expert(top_idx[p], experts), token_of(p, top_k), passes) : -1;
      gv[u] = (live && sorted_gate) ? gate[p] : (uint16_t)0;
    }
#pragma unroll
    for (int u = 0; u < kDispatchUnroll; ++u) {
      if (base + 32 * u >= end) break;
      const int64_t p = base + 32 * u + lane;
      const int e = ev[u];
      const bool live = e >= 0;
      const uint32_t peers = __match_any_sync(0xffffffffu, e);
      int dest = 0;
      if (live) dest = cur[e] + __popc(peers & lt);
      __syncwarp();
      if (live && lane == __ffs(peers) - 1) cur[e] += __popc(peers);
      __syncwarp();
      if (live) {
        if (order) order[dest] = p;
        if (inverse) inverse[p] = dest;
        const int32_t tok = (int32_t)token_of(p, top_k);
        if (tokens) tokens[dest] = tok;
        if (tokens32) tokens32[dest] = tok;
        if (sorted_gate) sorted_gate[dest] = gv[u];
      }
    }
  }
}

__global__ void dispatch_scatter_kernel(const int64_t* __restrict__ top_idx, const uint16_t* __restrict__ gate,
                                        int64_t positions, int top_k, int experts, Passes passes, int groups,
                                        int seg_len, int segments,
                                        const int32_t* __restrict__ seg_start, const int32_t* __restrict__ csr,
                                        int64_t* __restrict__ order, int64_t* __restrict__ inverse,
                                        int64_t* __restrict__ tokens, int32_t* __restrict__ tokens32,
                                        uint16_t* __restrict__ sorted_gate) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  extern __shared__ int32_t s_cursor[];  // [warps][groups]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seg = blockIdx.x * kDispatchWarps + warp;
  if (seg >= segments) return;
  int32_t* cur = s_cursor + warp * groups;
  for (int e = lane; e < groups; e += 32) cur[e] = csr[e] + seg_start[(int64_t)seg * groups + e];
  __syncwarp();
  scatter_segment(top_idx, gate, positions, top_k, experts, passes, seg_len, seg, cur, order, inverse, tokens,
                  tokens32, sorted_gate);
}

// ---------------------------------------------------------------------------
// Small batches: the three passes in one CTA of 32 warps (one per segment,
// segments <= 32), with the same arithmetic and results; the passes meet at
// __syncthreads (the scan's and the scatter's reads of seg_count / csr in
// global memory follow the writes of the same CTA).
// ---------------------------------------------------------------------------
constexpr int kFusedWarps = 32;
constexpr int kFusedMaxGroups = 256;

__global__ void __launch_bounds__(1024) dispatch_fused_kernel(
    const int64_t* __restrict__ top_idx, const uint16_t* __restrict__ gate, const uint16_t* __restrict__ row_amax,
    int64_t positions, int top_k, int experts, Passes passes, int groups, int seg_len, int segments,
    int32_t* __restrict__ seg_count, uint32_t* __restrict__ seg_max, int32_t* __restrict__ offsets,
    int32_t* __restrict__ csr, int32_t* __restrict__ pcsr, TileEntry* __restrict__ tiles, int max_tiles,
    int32_t* __restrict__ num_tiles, float* __restrict__ act_global, uint32_t* __restrict__ act_amax_bits,
    int64_t* __restrict__ order, int64_t* __restrict__ inverse, int64_t* __restrict__ tokens,
    int32_t* __restrict__ tokens32, uint16_t* __restrict__ sorted_gate) {
  pdl_wait();  // the previous kernel of the stream has completed
  pdl_trigger();
  extern __shared__ uint32_t s_df[];
  uint32_t* hist = s_df;                        // [warps][groups], then the scatter cursors
  uint32_t* hmax = s_df + kFusedWarps * groups;  // [warps][groups]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kFusedWarps * groups; i += blockDim.x) {
    hist[i] = 0;
    hmax[i] = 0;
  }
  __syncthreads();
  if (warp < segments)
    count_segment(top_idx, row_amax, positions, top_k, experts, passes, groups, seg_len, warp, hist + warp * groups,
                  hmax + warp * groups, seg_count, seg_max);
  __syncthreads();
  scan_segments(seg_count, seg_max, segments, groups, positions, (int)kTileRows, offsets, csr, pcsr, tiles, max_tiles,
                num_tiles, act_global, act_amax_bits);
  __syncthreads();
  if (positions > 0 && warp < segments) {
    int32_t* cur = reinterpret_cast<int32_t*>(hist) + warp * groups;
    for (int e = lane; e < groups; e += 32) cur[e] = csr[e] + seg_count[(int64_t)warp * groups + e];
    __syncwarp();
    scatter_segment(top_idx, gate, positions, top_k, experts, passes, seg_len, warp, cur, order, inverse, tokens,
                    tokens32, sorted_gate);
  }
}

// ---------------------------------------------------------------------------
// Host entry
// ---------------------------------------------------------------------------
static void dispatch_geometry(int64_t positions, int* seg_len, int* segments) {
  // Segments of >= 128 positions (one warp each: enough warps to cover the
  // memory latency of the count and scatter passes, few enough segments for
  // the single-CTA scan; config 2: 27.5 us for the three passes against 29.7
  // with 64 or 256), at most 2048 of them.
  int64_t len = 128;
  while ((positions + len - 1) / len > 2048) len *= 2;
  *seg_len = (int)len;
  *segments = (int)((positions + len - 1) / len);
  if (*segments == 0) *segments = 1;
}

// `groups`: routed experts x passes.
size_t dispatch_workspace_bytes(int64_t tokens, int top_k, int groups) {
  int seg_len, segments;
  dispatch_geometry(tokens * top_k, &seg_len, &segments);
  return (size_t)segments * groups * 8 + 256;
}

// With passes.n == 2 every per-expert output (offsets, csr, pcsr, the tile
// tables, the global scales) is per group (route_group), 2 * experts of them.
int run_dispatch(const int64_t* top_idx, const uint16_t* gate, const uint16_t* row_amax, int64_t tokens, int top_k,
                 int experts, Passes passes, void* workspace, size_t workspace_bytes, int64_t* order, int64_t* inverse,
                 int64_t* tokens_out, int32_t* tokens32, uint16_t* sorted_gate, int32_t* offsets, int32_t* csr,
                 int32_t* pcsr, TileEntry* tiles, int max_tiles, int32_t* num_tiles, float* act_global,
                 uint32_t* act_amax_bits, cudaStream_t stream) {
  if (passes.n != 1 && passes.n != 2) return set_error(PRAXIS_B200_EINVAL, "passes must be 1 or 2");
  if (passes.n == 2 && (passes.t0 < 0 || passes.t0 > tokens))
    return set_error(PRAXIS_B200_EINVAL, "pass 0 tokens %lld outside 0..%lld", (long long)passes.t0, (long long)tokens);
  const int groups = experts * passes.n;
  if (experts <= 0 || groups > kMaxExperts)
    return set_error(PRAXIS_B200_EINVAL, "experts x passes must be 1..%d", kMaxExperts);
  if (top_k <= 0 || tokens < 0) return set_error(PRAXIS_B200_EINVAL, "bad tokens/top_k");
  if (tokens * top_k >= (int64_t)1 << 31) return set_error(PRAXIS_B200_EINVAL, "too many routed rows");
  if (workspace_bytes < dispatch_workspace_bytes(tokens, top_k, groups))
    return set_error(PRAXIS_B200_EINVAL, "dispatch workspace too small");
  const int64_t positions = tokens * top_k;
  int seg_len, segments;
  dispatch_geometry(positions, &seg_len, &segments);
  int32_t* seg_count = static_cast<int32_t*>(workspace);
  uint32_t* seg_max = reinterpret_cast<uint32_t*>(seg_count + (size_t)segments * groups);
  const int blocks = (segments + kDispatchWarps - 1) / kDispatchWarps;
  const size_t smem_count = (size_t)2 * kDispatchWarps * groups * 4;
  const size_t smem_scatter = (size_t)kDispatchWarps * groups * 4;
  static DeviceOnce attr;
  int rc = device_once(attr, [](int dev) {
    cudaError_t e = cudaFuncSetAttribute(dispatch_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         2 * kDispatchWarps * kMaxExperts * 4);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(dispatch_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kDispatchWarps * kMaxExperts * 4);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(dispatch_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               2 * kFusedWarps * kFusedMaxGroups * 4);
    if (e != cudaSuccess)
      return set_error(PRAXIS_B200_ECUDA, "dispatch smem attribute (device %d): %s", dev, cudaGetErrorString(e));
    return (int)PRAXIS_B200_OK;
  });
  if (rc) return rc;
  if (segments <= kFusedWarps && groups <= kFusedMaxGroups) {
    // small batch (<= 32 segments): one launch instead of three
    launch_pdl(dispatch_fused_kernel, dim3(1), dim3(32 * kFusedWarps), (size_t)2 * kFusedWarps * groups * 4, stream,
               top_idx, gate, row_amax, positions, top_k, experts, passes, groups, seg_len, segments, seg_count,
               seg_max, offsets, csr, pcsr, tiles, max_tiles, num_tiles, row_amax ? act_global : nullptr,
               row_amax ? act_amax_bits : nullptr, order, inverse, tokens_out, tokens32, sorted_gate);
    return check_launch("dispatch_fused");
  }
  launch_pdl(dispatch_count_kernel, dim3(blocks), dim3(32 * kDispatchWarps), smem_count, stream, top_idx, row_amax,
             positions, top_k, experts, passes, groups, seg_len, segments, seg_count, seg_max);
  rc = check_launch("dispatch_count");
  if (rc) return rc;
  launch_pdl(dispatch_scan_kernel, dim3(1), dim3(1024), 0, stream, seg_count, seg_max, segments, groups, positions,
             (int)kTileRows, offsets, csr, pcsr, tiles, max_tiles, num_tiles, row_amax ? act_global : nullptr,
             row_amax ? act_amax_bits : nullptr);
  rc = check_launch("dispatch_scan");
  if (rc) return rc;
  if (positions > 0) {
    launch_pdl(dispatch_scatter_kernel, dim3(blocks), dim3(32 * kDispatchWarps), smem_scatter, stream, top_idx, gate,
               positions, top_k, experts, passes, groups, seg_len, segments, seg_count, csr, order, inverse, tokens_out,
               tokens32, sorted_gate);
    rc = check_launch("dispatch_scatter");
  }
  return rc;
}

int run_row_amax(const uint16_t* x, int64_t rows, int cols, uint16_t* out, cudaStream_t stream) {
  if (cols % 8 != 0) return set_error(PRAXIS_B200_EINVAL, "row_amax needs cols % 8 == 0");
  if (rows == 0) return PRAXIS_B200_OK;
  const int warps = 8;
  const int64_t blocks = (rows + warps - 1) / warps;
  launch_pdl(row_amax_kernel, dim3((unsigned)blocks), dim3(32 * warps), 0, stream, x, rows, cols, out);
  return check_launch("row_amax");
}

}  // namespace praxis
