/*
 * praxis_b200_moe.h - C ABI of the B200 (sm_100a) routed-expert NVFP4 MoE
 * library (libpraxis_b200_moe.so).
 *
 * The reference (runwayml/praxis-1-oss) is Python; its hot path is the MoE
 * module -> routed NVFP4 bank -> Triton/CuTe/FlashInfer kernel chain. Each
 * entry point below replaces one function of that chain and says which
 * (file:line in the reference). A Python binding is a ctypes stub over these
 * declarations (praxis-1-oss_b200/capi.py is that binding).
 *
 * Conventions
 *  - Every pointer is a device pointer unless stated otherwise. The caller
 *    allocates every buffer (outputs and workspaces); no entry point
 *    allocates device memory.
 *  - bf16 tensors are passed as `void*` / `const void*` (raw 16-bit values).
 *  - `stream` is a cudaStream_t; `device` the CUDA ordinal the buffers live
 *    on (made current for the call). Work is enqueued on `stream` only;
 *    nothing synchronizes the host, so every call can be captured in a CUDA
 *    graph. Offsets and counts stay on the device.
 *  - The return value is PRAXIS_B200_OK or an error code;
 *    praxis_b200_last_error() gives a message (per host thread). Argument
 *    errors are reported before any launch.
 *  - Device-side faults never trap: waits are bounded and out-of-range
 *    indices are clamped; either records a code in a per-device error word
 *    that praxis_b200_device_error() reads (and clears) at a sync point.
 */
#ifndef PRAXIS_B200_MOE_H
#define PRAXIS_B200_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PRAXIS_B200_ABI_VERSION 4

enum {
  PRAXIS_B200_OK = 0,
  PRAXIS_B200_EINVAL = 1,      /* argument check failed (nothing launched) */
  PRAXIS_B200_ECUDA = 2,       /* a CUDA call failed */
  PRAXIS_B200_EUNSUPPORTED = 3 /* device is not sm_100 */
};

enum { PRAXIS_B200_SIGMOID = 0, PRAXIS_B200_SOFTMAX = 1 };

/* Grouped-GEMM epilogues (praxis_b200_grouped_gemm). */
enum {
  PRAXIS_B200_EPI_PLAIN = 0,   /* out = bf16(acc) */
  PRAXIS_B200_EPI_SWIGLU = 1,  /* rescale + SwiGLU + per-expert max |hidden| */
  PRAXIS_B200_EPI_RESCALE = 2  /* out = bf16(bf16(acc) * bf16(g_act * g_w)) */
};

/* Layouts of the UE4M3 block-scale ("sf") buffers.
 * COMPACT     the reference's layout (praxis/kernels/nvfp4.py:114-119):
 *             per 128-row tile and 64-element k-block one 512-byte atom,
 *             byte (r%32)*16 + ((r%128)/32)*4 + j%4 for row r, scale j.
 * REPLICATED  this library's GEMM layout: every atom stored 4 times in a row
 *             (the four tensor-memory lane quadrants each get a copy with one
 *             128x256b tcgen05 copy). Activations: [tile][k-block][4][512 B];
 *             weights: [expert][256-row tile][k-block][2 x 128-row][4][512 B].
 *             Produced by the quantize entry points and
 *             praxis_b200_replicate_scales. */
enum { PRAXIS_B200_SF_COMPACT = 0, PRAXIS_B200_SF_REPLICATED = 1 };

int praxis_b200_abi_version(void);
const char* praxis_b200_last_error(void);
/* Number of SMs of `device`; 0 if it is not an sm_100 device. */
int praxis_b200_device_check(int device);
/* Reads and clears the device error word (synchronizes `device`). */
int praxis_b200_device_error(int device, uint32_t* code);

/* Padded rows of the expert-grouped layout: ((rows + 127 * experts) / 128) * 128.
 * Replaces praxis/kernels/nvfp4.py:212-213. Host function. */
int64_t praxis_b200_padded_rows(int64_t routed_rows, int32_t experts);

/* Router logits: logits[t, e] = sum_c f32(x[t, c]) * f32(W[e, c]) for bf16 x
 * [T, C], and row_amax[t] = bf16(max_c |x[t, c]|) when row_amax != NULL.
 * `weight` is [splits, E, C] bf16: splits = 1 for a bf16 router weight, 3 for
 * an fp32 weight given as hi + mid + lo bf16 terms (exact).
 * Replaces praxis/layers.py:1104-1122 (_router_logits_forward) and
 * praxis/kernels/nvfp4_moe.py:15-21 (_row_absmax). E <= 256, C % 32 == 0. */
int praxis_b200_router_logits(const void* x, const void* weight, int32_t weight_splits, int64_t tokens,
                              int32_t dim, int32_t experts, float* logits, void* row_amax, int device,
                              void* stream);

/* Routing of fp32 logits [T, E]: sigmoid (or softmax) scores, + bias (fp32
 * [E] or NULL), top-k (int64 [T, k], torch.topk's CUDA slot order incl.
 * ties), gates bf16(score / sum) [T, k].
 * Replaces praxis/layers.py:1647-1653 (== :2167-2173) and the routing half of
 * praxis/kernels/router_fused.py:738-804 (route_dispatch). E <= 256, k <= 8. */
int praxis_b200_route(const float* logits, const float* bias, int64_t tokens, int32_t experts, int32_t top_k,
                      int32_t activation, int64_t* top_idx, void* gate, int device, void* stream);

/* row_amax[r] = bf16(max |x[r, :]|) for bf16 x [rows, cols].
 * Replaces praxis/kernels/nvfp4_moe.py:15-21. */
int praxis_b200_row_amax(const void* x, int64_t rows, int32_t cols, void* out, int device, void* stream);

/* Dispatch of top_idx [T, k] (int64) and gate [T, k] (bf16):
 *   order[r], tokens[r] (int64), tokens32[r] (int32), sorted_gate[r] (bf16):
 *      the stable expert-major order of the T*k (token, slot) rows;
 *   inverse[p]: position of flat row p in that order;
 *   offsets[e]: int32 end offsets; csr[E+1]; pcsr[E+1] (128-aligned starts);
 *   tiles [2 * max_tiles, 4] int32: entries 0.. are the 128-row tiles that
 *      hold routed rows {expert, first padded row, routed rows, 0} in expert
 *      order; entries max_tiles.. are the 256-row pairs of the 2-CTA GEMM
 *      {expert, first padded row, routed rows, rows of live 128-row tiles};
 *      num_tiles[2] = {tiles, pairs};
 *   act_global[e] (fp32) and act_amax[e] (fp32 bits) from row_amax [T] (bf16)
 *      when row_amax != NULL: f32(bf16(max(amax, 1e-12))) * f32(1/2688).
 * Any output pointer except csr, pcsr, tiles, num_tiles may be NULL.
 * max_tiles = praxis_b200_padded_rows(T*k, E) / 128.
 * Replaces praxis/layers.py:1330-1346 (_dispatch_rows),
 * praxis/quantization/nvfp4.py:705-708 (inverse), praxis/kernels/nvfp4.py:37-41
 * (_pad_csr), :344-352 (tile metadata), praxis/kernels/nvfp4_moe.py:24-57
 * (segment global scales), and the dispatch half of
 * praxis/kernels/router_fused.py:738-804. */
size_t praxis_b200_dispatch_workspace_size(int64_t tokens, int32_t top_k, int32_t experts);
int praxis_b200_dispatch(const int64_t* top_idx, const void* gate, const void* row_amax, int64_t tokens,
                         int32_t top_k, int32_t experts, void* workspace, size_t workspace_size, int64_t* order,
                         int64_t* inverse, int64_t* tokens_out, int32_t* tokens32, void* sorted_gate,
                         int32_t* offsets, int32_t* csr, int32_t* pcsr, int32_t* tiles, int32_t max_tiles,
                         int32_t* num_tiles, float* act_global, uint32_t* act_amax, int device, void* stream);

/* praxis_b200_dispatch of `passes` (1 or 2) lockstep inputs, tokens back to
 * back (a classifier-free-guidance pair: pass 1 from token pass0_tokens).
 * With passes == 2 the routed rows of expert e and pass s form group
 * g = 2 e + s, and the per-expert outputs become per group: order / inverse
 * sort by (g, position), csr [2E + 1] is the reference's seg_csr, offsets
 * [2E] the group end offsets (the reference's per-expert offsets are
 * offsets[1::2]), pcsr / tiles / act_global / act_amax per group, each group
 * padded to 128 rows on its own. The same values as the reference's P = 2
 * route_dispatch / dispatch_ref (praxis/kernels/router_fused.py:738-804,
 * :820-852), the per-(expert, pass) segments of
 * praxis/kernels/nvfp4_pair.py:1-20. max_tiles =
 * praxis_b200_padded_rows(T*k, E*passes) / 128. */
size_t praxis_b200_dispatch_passes_workspace_size(int64_t tokens, int32_t top_k, int32_t experts, int32_t passes);
int praxis_b200_dispatch_passes(const int64_t* top_idx, const void* gate, const void* row_amax, int64_t tokens,
                                int32_t top_k, int32_t experts, int32_t passes, int64_t pass0_tokens, void* workspace,
                                size_t workspace_size, int64_t* order, int64_t* inverse, int64_t* tokens_out,
                                int32_t* tokens32, void* sorted_gate, int32_t* offsets, int32_t* csr, int32_t* pcsr,
                                int32_t* tiles, int32_t max_tiles, int32_t* num_tiles, float* act_global,
                                uint32_t* act_amax, int device, void* stream);

/* NVFP4 quantization of the routed rows (gathered from x [T, C] bf16 through
 * inverse/top_idx) into the padded expert-grouped layout: q [Rp, C/2] (two
 * E2M1 codes per byte, even element low), sf [Rp, C/16] (UE4M3, 128x4
 * swizzled atoms; 4x that size for sf_layout PRAXIS_B200_SF_REPLICATED);
 * padding rows of the listed tiles are zeroed. Global scale
 * per expert from act_global, or from act_amax when act_global is NULL.
 * Replaces praxis/kernels/nvfp4.py:197-254 + :44-124 (quantize_activations
 * with row_indices, alignment=128, grouped_scales=False). C % 64 == 0. */
int praxis_b200_quantize_gather(const void* x, int64_t tokens, int32_t dim, const int64_t* top_idx,
                                const int64_t* inverse, const int32_t* csr, const int32_t* pcsr,
                                const float* act_global, const uint32_t* act_amax, int32_t top_k,
                                int32_t experts, const int32_t* tiles, const int32_t* num_tiles,
                                int32_t max_tiles, void* q, void* sf, int32_t sf_layout, int device,
                                void* stream);

/* NVFP4 quantization of every row of the listed tiles of x [Rp, K] (bf16),
 * global per expert from globals, or from amax (fp32 bits) when NULL;
 * sf in sf_layout (as praxis_b200_quantize_gather).
 * Replaces praxis/kernels/nvfp4.py:197-254 for the hidden activations
 * (praxis/quantization/nvfp4.py:365-372). K % 64 == 0. */
int praxis_b200_quantize_rows(const void* x, int32_t k, const int32_t* tiles, const int32_t* num_tiles,
                              int32_t max_tiles, const float* globals, const uint32_t* amax, void* q, void* sf,
                              int32_t sf_layout, int device, void* stream);

/* Grouped NVFP4 GEMM on tcgen05: for each listed tile (expert e, rows r),
 * acc[r, n] = sum_k dq(a[r, k]) * dq(b[e, n, k]) (alpha = 1), then the
 * epilogue. a_q [Rp, K/2], a_sf [Rp, K/16], b_q [E, N, K/2], b_sf [E, N, K/16]
 * (swizzled). EPI_PLAIN: out [Rp, N]. EPI_SWIGLU: b rows in 64-row gate/up
 * blocks (praxis_b200_interleave_gate_up), out = hidden [Rp, N/2], amax_out[e]
 * atomically maxed with the bits of max |hidden|. EPI_RESCALE: out [Rp, N].
 * act_global (or act_amax) and w_global give bf16(g_act * g_w).
 * sf_layout PRAXIS_B200_SF_COMPACT: both scale buffers in the reference's
 * layout; PRAXIS_B200_SF_REPLICATED: a_sf replicated in 128-row groups and
 * b_sf in 256-row groups (praxis_b200_replicate_scales), N % 256 == 0.
 * Rows of a tile past its valid count hold the products of the padding rows
 * (zero for padding written by the quantize entry points; EPI_SWIGLU stores 0).
 * Replaces praxis/kernels/nvfp4.py:355-419 (grouped_nvfp4_mm) with
 * praxis/kernels/nvfp4_moe.py:102-158 (EPI_SWIGLU) or the rescale of
 * praxis/kernels/nvfp4_moe.py:236-247 (EPI_RESCALE) fused. N, K % 128 == 0.
 * Scale buffers and out are 16-byte aligned; the EPI_SWIGLU out 32-byte. */
/* (A tile whose expert index is >= experts uses weights index % experts.) */
int praxis_b200_grouped_gemm(const void* a_q, const void* a_sf, const void* b_q, const void* b_sf,
                             const int32_t* tiles, const int32_t* num_tiles, int32_t max_tiles,
                             int64_t rows_padded, int32_t n, int32_t k, int32_t experts, int32_t epilogue,
                             void* out, const float* act_global, const uint32_t* act_amax, const float* w_global,
                             uint32_t* amax_out, int32_t sf_layout, int device, void* stream);

/* The gate/up GEMM with SwiGLU and NVFP4 output at a calibrated hidden
 * global scale (SetFusedSwiglu / FC1 FP4 output): the hidden values of
 * EPI_SWIGLU (the same bits) are quantized in the epilogue with the frozen
 * global `hidden_global` by the reference's recipe (E2M1 codes, UE4M3 scale
 * per 16, compact 128x4 scale atoms) into q_out [Rp, N/4] and sf_out
 * [Rp, N/32]; the bf16 hidden rows, their per-expert maxima and the hidden
 * quantize pass are not needed. Replaces praxis/kernels/nvfp4_swiglu.py:40-74
 * (gate_up_fp4, a FlashInfer act-fusion kernel whose bits are not
 * available here: this entry computes the hidden quantize recipe of
 * praxis/kernels/nvfp4.py:197-254 at the frozen global on the EPI_SWIGLU
 * hidden values). N % 256 == 0, compact scales; outputs 16-byte aligned. */
int praxis_b200_gemm_swiglu_fp4(const void* a_q, const void* a_sf, const void* b_q, const void* b_sf,
                                const int32_t* tiles, const int32_t* num_tiles, int32_t max_tiles,
                                int64_t rows_padded, int32_t n, int32_t k, int32_t experts, const float* act_global,
                                const uint32_t* act_amax, const float* w_global, float hidden_global, void* q_out,
                                void* sf_out, int device, void* stream);

/* Copies compact scales sf [rows, k/16] (the reference's swizzled layout)
 * into the replicated GEMM layout out [4 * rows * k/16]: group_rows = 128 for
 * activations, 256 for weights (rows = E * N, N % 256 == 0). rows % group_rows
 * == 0, k % 64 == 0. Kernel-side layout only: no reference counterpart. */
int praxis_b200_replicate_scales(const void* sf, int64_t rows, int32_t k, int32_t group_rows, void* out,
                                 int device, void* stream);

/* Rescale + SwiGLU + row max over the padded gate/up GEMM output raw
 * [rows, 2F] (bf16, gate columns first): m = bf16(act_global[e] * w_global[e])
 * for the expert e whose pcsr segment holds the row; hidden [rows, F] and
 * rowmax [rows] (bf16, may be NULL). alu = 1: the arithmetic of the fused GEMM
 * epilogue (integer roundings, refined reciprocal); alu = 0: conversion-unit
 * roundings and IEEE division. Both give the same bits.
 * Replaces praxis/kernels/nvfp4_moe.py:102-158 (rescale_swiglu_maximum). */
int praxis_b200_rescale_swiglu(const void* raw, int64_t rows, int32_t hidden, const int32_t* pcsr,
                               int32_t experts, const float* act_global, const float* w_global, void* out,
                               void* rowmax, int32_t alu, int device, void* stream);

/* Weighted combine: out[t] = bf16(((a0 + a1) + a2) + a3) with
 * a_{s%4} += v_s * (f32(gate[t, s]) * f32(scaling)), v_s the routed row
 * pcsr[e] + inverse[t*k+s] - csr[e] of rows [Rp, C] (bf16), rescaled by
 * bf16(g_h[e] * g_w[e]) unless rows_rescaled; then out = bf16(out + shared)
 * when shared != NULL. Replaces praxis/kernels/nvfp4_moe.py:206-311. */
int praxis_b200_combine(const void* rows, int32_t cols, const int64_t* inverse, const int64_t* top_idx,
                        const void* gate, const int32_t* csr, const int32_t* pcsr, const float* h_global,
                        const uint32_t* h_amax, const float* w_global, int32_t rows_rescaled, float scaling,
                        const void* shared, void* out, int64_t tokens, int32_t top_k, int32_t experts, int device,
                        void* stream);

/* The MoE tail fused into what follows it (praxis.layers.MOE_TAIL_NORM):
 * the combine of praxis_b200_combine (its arithmetic, shared add included)
 * gives y, never stored; then, per token,
 *   x  = bf16(f32(residual) + f32(y))                  (the residual add)
 *   with mod: x = bf16(fma(f32(x), bf16(f32(scl) + 1), f32(shf)))
 *             (mod_fma == 0: the product rounded before the add)
 *   residual_out = x
 *   with norm_weight: normed_out = bf16(bf16(norm_weight * (r * f32(x))) * norm_scale),
 *             r = rsqrt(sum(f32(x)^2) / C + eps)
 * the sum in the order of torch's vectorized RMSNorm kernel (128 threads per
 * row, float4 vectors, shuffle-down tree, (w0 + w2) + (w1 + w3)), the IEEE
 * division and the hardware reciprocal square root. norm_weight is fp32 [C]
 * and already 1 + weight (RMSNorm's zero-centred scale), norm_scale the
 * block's scalar. mod rows are [R, 2C] bf16, shift then scale; the row of
 * token t follows praxis/kernels/norm_triton.py:417-431 with
 * mod_geom = {RF, RC, NREG, PW, WD, PH} ({1, 1, 0, 1, 1, 1}: row t) applied
 * to t + mod_row0 (the global row of a chunk's first token).
 * The three forms replace praxis/kernels/moe_tail_triton.py:329-352
 * (tail_add_norm_scale: norm_weight set, mod NULL), :355-385
 * (tail_add_mod_norm_scale: both set) and :431-445 (tail_residual_add:
 * norm_weight NULL, mod NULL), NVFP4 one-chunk mode. */
typedef struct praxis_b200_tail {
  const void* residual;      /* [T, C] bf16 */
  void* residual_out;        /* [T, C] bf16 */
  const float* norm_weight;  /* [C] fp32, 1 + weight; NULL: residual add only */
  void* normed_out;          /* [T, C] bf16 (with norm_weight) */
  float eps;
  float norm_scale;
  const void* mod;           /* [R, 2C] bf16 or NULL (needs norm_weight) */
  int32_t mod_fma;
  int64_t mod_geom[6];
  int64_t mod_row0;
} praxis_b200_tail;

/* C % 4 == 0; bf16 buffers 8-byte aligned, norm_weight 16-byte aligned. */
int praxis_b200_combine_tail(const void* rows, int32_t cols, const int64_t* inverse, const int64_t* top_idx,
                             const void* gate, const int32_t* csr, const int32_t* pcsr, const float* h_global,
                             const uint32_t* h_amax, const float* w_global, int32_t rows_rescaled, float scaling,
                             const void* shared, const praxis_b200_tail* tail, int64_t tokens, int32_t top_k,
                             int32_t experts, int device, void* stream);

/* Packs expert-first bf16 weights w [E, K, N] (RoutedExperts layout: input
 * features first) as W^T per expert: q [E, N, K/2], sf [E, N, K/16]
 * (swizzled), global [E]. scratch: E uint32.
 * Replaces praxis/quantization/nvfp4.py:67-146 (pack_routed_experts /
 * _pack_matrix_cpu), same bytes. K % 64 == 0, N % 128 == 0. */
int praxis_b200_pack_weights(const void* w, int32_t experts, int32_t k, int32_t n, void* q, void* sf,
                             float* global_out, uint32_t* scratch, int device, void* stream);

/* Copies gate_up q [E, 2F, C/2] / sf [E, 2F, C/16] into the fused-SwiGLU
 * GEMM layout: 64-row blocks of 32 gate rows then the matching 32 up rows;
 * block b serves hidden columns 32*h .. 32*h+31 with h = b except that blocks
 * 1 and 2 of every group of four trade places. F % 128 == 0.
 * Kernel-side layout only (the reference keeps gate rows 0..F-1, up rows
 * F..2F-1: praxis/quantization/nvfp4.py:132-144). */
int praxis_b200_interleave_gate_up(const void* q, const void* sf, int32_t experts, int32_t hidden, int32_t dim,
                                   void* q_out, void* sf_out, int device, void* stream);

/* One dispatch chunk of the routed bank (and optionally the router):
 * NVFP4RoutedExperts.routed_forward[_with_shared] on SM100,
 * praxis/quantization/nvfp4.py:490-544 and :616-747 for one chunk. */
typedef struct praxis_b200_moe_args {
  const void* x;             /* [T, C] bf16 */
  const void* router_weight; /* [splits, E, C] bf16, or NULL: top_idx/gate are inputs */
  int32_t router_splits;
  int32_t activation;        /* PRAXIS_B200_SIGMOID / SOFTMAX */
  const float* router_bias;  /* [E] or NULL */
  int64_t* top_idx;          /* [T, k]: input, or output when router_weight != NULL */
  void* gate;                /* [T, k] bf16: same */
  const void* shared;        /* [T, C] bf16 or NULL */
  void* out;                 /* [T, C] bf16 */
  const void* gate_up_q;     /* interleaved layout (praxis_b200_interleave_gate_up) */
  const void* gate_up_sf;
  const float* gate_up_global;
  const void* down_q;        /* [E, C, F/2] */
  const void* down_sf;       /* [E, C, F/16] */
  const float* down_global;
  int32_t gate_up_sf_layout; /* PRAXIS_B200_SF_* of gate_up_sf */
  int32_t down_sf_layout;    /* PRAXIS_B200_SF_* of down_sf (replicated needs C % 256 == 0) */
  int64_t tokens;
  int32_t dim;               /* C */
  int32_t hidden;            /* F */
  int32_t experts;           /* E */
  int32_t top_k;
  float scaling;
  void* workspace;
  size_t workspace_size;
  int device;
  void* stream;
  /* Optional MoE tail fused into what follows it (praxis_b200_combine_tail):
   * when set, its outputs replace `out`, which may be NULL. */
  const praxis_b200_tail* tail;
  /* Lockstep passes (0 or 1: one input; 2: a classifier-free-guidance pair
   * whose second input starts at token pass0_tokens): the routed rows of
   * both inputs go through one pass of the expert GEMMs, grouped per
   * (expert, input) as praxis_b200_dispatch_passes groups them, and every
   * output row has the bits of its input run alone
   * (MoEFeedForward.forward_pair, praxis/layers.py:1779-1853). */
  int32_t passes;
  int64_t pass0_tokens;
  /* > 0: the calibrated FC1 output scale (praxis_b200_gemm_swiglu_fp4): the
   * gate/up GEMM writes FP4 hidden rows at this frozen global, which is also
   * the down GEMM's activation global (NVFP4RoutedExperts.set_fused_swiglu_scale,
   * praxis/quantization/nvfp4.py:235-260, :327-339). 0: dynamic globals. */
  float fc1_output_scale;
} praxis_b200_moe_args;

size_t praxis_b200_moe_workspace_size(int64_t tokens, int32_t top_k, int32_t experts, int32_t dim, int32_t hidden,
                                      int32_t with_router, int32_t passes);
int praxis_b200_moe_forward(const praxis_b200_moe_args* args);

/* Expert-rank half of an expert-parallel layer (no reference counterpart:
 * the reference runs every expert on every GPU). Input: rows received from
 * the source ranks, already NVFP4-quantized by each source with its own
 * per-expert activation global scale, in padded segments: segment v
 * (= source * experts + local expert; local expert v % experts) holds
 * counts[v] rows from padded row starts[v] (multiples of 128, ascending,
 * starts[segments] = rows). Runs gate/up GEMM + SwiGLU, hidden quantize with
 * one global scale per segment (the reference's per-expert, per-dispatch-chunk
 * scale when each source's batch is one chunk), down GEMM + rescale, and
 * writes rows_out [rows, C] bf16 in the same layout for the return exchange.
 * Weights are the rank's local experts in the kernel layouts of
 * praxis_b200_moe_forward. */
typedef struct praxis_b200_expert_args {
  const void* q;              /* [rows, C/2] E2M1 */
  const void* sf;             /* [rows, C/16] UE4M3, compact swizzled */
  int64_t rows;
  const int32_t* counts;      /* [segments] */
  const int32_t* starts;      /* [segments + 1] */
  const float* act_global;    /* [segments] */
  int32_t segments;           /* <= 1024 */
  const void* gate_up_q;
  const void* gate_up_sf;
  const float* gate_up_global;
  const void* down_q;
  const void* down_sf;
  const float* down_global;
  int32_t gate_up_sf_layout;  /* PRAXIS_B200_SF_* of gate_up_sf */
  int32_t down_sf_layout;     /* PRAXIS_B200_SF_* of down_sf */
  int32_t dim;                /* C */
  int32_t hidden;             /* F */
  int32_t experts;            /* local experts */
  int32_t sm_limit;           /* GEMMs on at most this many SMs (0: all), leaving the rest to
                                 concurrent transfer kernels */
  void* rows_out;             /* [rows, C] bf16 */
  void* workspace;
  size_t workspace_size;
  int device;
  void* stream;
  /* Hidden-output mode (the down GEMM runs on the source rank): with
   * hidden_q != NULL the forward stops after the hidden quantize and writes
   * the FP4 hidden rows [rows, F/2], their compact scales [rows, F/16] and
   * each segment's max |hidden| (fp32 bits, [segments]); rows_out and the
   * down weights are not used. */
  void* hidden_q;
  void* hidden_sf;
  uint32_t* hidden_amax;
} praxis_b200_expert_args;

size_t praxis_b200_expert_workspace_size(int64_t rows, int32_t segments, int32_t dim, int32_t hidden);
int praxis_b200_expert_forward(const praxis_b200_expert_args* args);

/* Dispatch without a caller workspace: praxis_b200_dispatch with the same
 * arguments (minus workspace / workspace_size) and the same outputs, its
 * scratch taken from a static device array of this library instead.
 * No counterpart in the reference (its dispatch allocates with torch).
 *
 * For callers that cannot allocate device memory: a plugin host that hands
 * out only its own input/output buffers and no workspace, a runtime whose
 * memory budget is fixed up front, or a serving loop that must not call
 * cudaMalloc/cudaFree (they synchronize the device). This entry point
 * allocates nothing, torch included.
 *  - Limit: the scratch is PRAXIS_B200_DISPATCH_NOALLOC_SCRATCH bytes
 *    (4 MiB + 256, per device): enough for every token count with up to 256
 *    experts. A call needing more (praxis_b200_dispatch_workspace_size above
 *    the limit) returns PRAXIS_B200_EINVAL before any launch; use
 *    praxis_b200_dispatch with a workspace for it.
 *  - Set-up: the first call on each device looks up the scratch address
 *    (with that device current) and keeps it; make that first call before
 *    any stream capture starts.
 *  - Zeroing: no part of the scratch needs to start at zero; every call
 *    writes each scratch word before reading it.
 *  - Races: all calls on one device share the one scratch. Calls whose work
 *    can overlap (unordered streams, other host threads) corrupt each
 *    other's results; order them (one stream, or events).
 * The outputs, output sizes and errors are those of praxis_b200_dispatch. */
#define PRAXIS_B200_DISPATCH_NOALLOC_SCRATCH (((size_t)4 << 20) + 256)
int praxis_b200_dispatch_noalloc(const int64_t* top_idx, const void* gate, const void* row_amax, int64_t tokens,
                                 int32_t top_k, int32_t experts, int64_t* order, int64_t* inverse,
                                 int64_t* tokens_out, int32_t* tokens32, void* sorted_gate, int32_t* offsets,
                                 int32_t* csr, int32_t* pcsr, int32_t* tiles, int32_t max_tiles, int32_t* num_tiles,
                                 float* act_global, uint32_t* act_amax, int device, void* stream);

/* Peer buffers for the expert-parallel exchange (one process per GPU on one
 * node). No counterpart in the reference (it has no expert parallelism).
 * A rank allocates a buffer with praxis_b200_ipc_alloc, exports it with
 * praxis_b200_ipc_handle, and every other rank maps it with
 * praxis_b200_ipc_open (CUDA IPC, peer access enabled on first use); the
 * mapped pointer is valid on the opening rank's device until
 * praxis_b200_ipc_close. praxis_b200_copy_async copies device bytes on a
 * stream (a copy engine moves them; either side may be a mapped peer
 * buffer). The exporting rank must keep its buffer until every peer has
 * closed its mapping. */
#define PRAXIS_B200_IPC_HANDLE_BYTES 64
int praxis_b200_ipc_alloc(size_t bytes, int device, void** ptr);
int praxis_b200_ipc_free(void* ptr, int device);
int praxis_b200_ipc_handle(const void* ptr, int device, void* handle);
int praxis_b200_ipc_open(const void* handle, int device, void** ptr);
int praxis_b200_ipc_close(void* ptr, int device);
int praxis_b200_copy_async(void* dst, const void* src, size_t bytes, int device, void* stream);
/* The same copy done by `ctas` CTAs of SMs (16-byte loads here, stores to dst,
 * e.g. a mapped peer buffer over NVLink): runs beside the copy engines.
 * dst, src and bytes multiples of 16. */
int praxis_b200_sm_copy(void* dst, const void* src, size_t bytes, int ctas, int device, void* stream);
/* Stream-ordered wait until the int32 at flag (this device's memory, written
 * by a peer's copy engine after the data it guards) equals value: one
 * thread polls with system-scope acquire loads; after timeout_ns it records
 * error code 5 (peer timeout, praxis_b200_device_error) and returns, so the
 * stream never hangs. */
int praxis_b200_wait_value(const int32_t* flag, int32_t value, int64_t timeout_ns, int device, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PRAXIS_B200_MOE_H */
