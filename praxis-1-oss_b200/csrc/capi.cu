// extern "C" entry points (include/praxis_b200_moe.h): argument checks,
// device selection, workspace layout of the whole routed forward, and the
// launch sequence of one dispatch chunk.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace praxis {

// Internal entry points of the other .cu files.
size_t dispatch_workspace_bytes(int64_t tokens, int top_k, int groups);
int run_dispatch(const int64_t* top_idx, const uint16_t* gate, const uint16_t* row_amax, int64_t tokens, int top_k,
                 int experts, Passes passes, void* workspace, size_t workspace_bytes, int64_t* order, int64_t* inverse,
                 int64_t* tokens_out, int32_t* tokens32, uint16_t* sorted_gate, int32_t* offsets, int32_t* csr,
                 int32_t* pcsr, TileEntry* tiles, int max_tiles, int32_t* num_tiles, float* act_global,
                 uint32_t* act_amax_bits, cudaStream_t stream);
int run_row_amax(const uint16_t* x, int64_t rows, int cols, uint16_t* out, cudaStream_t stream);
int run_quantize_gather(const uint16_t* x, int64_t tokens, int k_dim, const int64_t* top_idx, const int64_t* inverse,
                        const int32_t* csr, const int32_t* pcsr, const float* globals, const uint32_t* amax_bits,
                        int top_k, int experts, const TileEntry* tiles, const int32_t* num_tiles, int max_tiles,
                        uint8_t* q, uint8_t* sf, int sf_layout, cudaStream_t stream, Passes passes = Passes{1, 0});
int run_quantize_rows(const uint16_t* x, int k_dim, const TileEntry* tiles, const int32_t* num_tiles, int max_tiles,
                      const float* globals, const uint32_t* amax_bits, uint8_t* q, uint8_t* sf, int sf_layout,
                      cudaStream_t stream);
int run_replicate_scales(const uint8_t* sf, int64_t rows, int k_dim, int group_rows, uint8_t* out, cudaStream_t stream);
int run_segment_tiles(const int32_t* counts, const int32_t* starts, int segments, TileEntry* tiles, int max_tiles,
                      int32_t* num_tiles, cudaStream_t stream);
int run_pack_weights(const uint16_t* w, int experts, int k_dim, int n_dim, uint8_t* q, uint8_t* sf, float* global_out,
                     uint32_t* amax_scratch, cudaStream_t stream);
int run_interleave_gate_up(const uint8_t* q, const uint8_t* sf, int experts, int f_dim, int c_dim, uint8_t* q_out,
                           uint8_t* sf_out, cudaStream_t stream);
int run_router_logits(const uint16_t* x, const uint16_t* w, int splits, int64_t tokens, int dim, int experts,
                      float* logits, uint16_t* row_amax, cudaStream_t stream);
int run_route(const float* logits, const float* bias, int64_t tokens, int experts, int top_k, int activation,
              int64_t* top_idx, uint16_t* gate, cudaStream_t stream);
int run_rescale_swiglu(const uint16_t* raw, int64_t rows, int hidden, const int32_t* pcsr, int experts,
                       const float* act_global, const float* w_global, uint16_t* out, uint16_t* rowmax, int alu,
                       cudaStream_t stream);
int run_combine(const uint16_t* rows, int cols, const int64_t* inverse, const int64_t* top_idx, const uint16_t* gate,
                const int32_t* csr, const int32_t* pcsr, const float* h_global, const uint32_t* h_amax,
                const float* w_global, int rows_rescaled, float scaling, const uint16_t* shared, uint16_t* out,
                int64_t tokens, int top_k, int experts, cudaStream_t stream, Passes passes = Passes{1, 0});
int run_combine_tail(const uint16_t* rows, int cols, const int64_t* inverse, const int64_t* top_idx,
                     const uint16_t* gate, const int32_t* csr, const int32_t* pcsr, const float* h_global,
                     const uint32_t* h_amax, const float* w_global, int rows_rescaled, float scaling,
                     const uint16_t* shared, const TailArgs& tail, int64_t tokens, int top_k, int experts,
                     cudaStream_t stream, Passes passes = Passes{1, 0});

// The ABI's tail descriptor as the kernel's arguments.
static TailArgs tail_args(const praxis_b200_tail& t) {
  TailArgs a;
  a.x = static_cast<const uint16_t*>(t.residual);
  a.x_out = static_cast<uint16_t*>(t.residual_out);
  a.w1 = t.norm_weight;
  a.h_out = static_cast<uint16_t*>(t.normed_out);
  a.eps = t.eps;
  a.norm_scale = t.norm_scale;
  a.mod = static_cast<const uint16_t*>(t.mod);
  a.mod_fma = t.mod_fma;
  for (int i = 0; i < 6; ++i) a.mod_geom[i] = t.mod_geom[i];
  a.mod_row0 = t.mod_row0;
  return a;
}

static thread_local char g_message[1024] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_message, sizeof(g_message), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return PRAXIS_B200_OK;
}

int sm_count() {
  static int cache[kMaxDevices] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxDevices && cache[dev]) return cache[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < kMaxDevices) cache[dev] = n;
  return n;
}

// Makes `device` current for this host thread and checks it is sm_100.
// Scratch of praxis_b200_dispatch_noalloc: one static array per device
// (module storage, no allocation call), its address looked up once per
// device with that device current.
static __device__ __align__(256) unsigned char g_dispatch_noalloc_scratch[PRAXIS_B200_DISPATCH_NOALLOC_SCRATCH];

static int dispatch_noalloc_scratch(int device, void** out) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {nullptr};
  std::lock_guard<std::mutex> lock(mu);
  if (addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_dispatch_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(PRAXIS_B200_ECUDA, "dispatch_noalloc: scratch address on device %d: %s", device,
                       cudaGetErrorString(e));
    addr[device] = p;
  }
  *out = addr[device];
  return PRAXIS_B200_OK;
}

static int use_device(int device) {
  static int arch_ok[kMaxDevices] = {0};
  if (device < 0 || device >= kMaxDevices) return set_error(PRAXIS_B200_EINVAL, "bad device %d", device);
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != device) {
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  }
  if (arch_ok[device] == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    arch_ok[device] = (major == 10 && minor == 0) ? 1 : -1;
  }
  if (arch_ok[device] < 0)
    return set_error(PRAXIS_B200_EUNSUPPORTED, "device %d is not sm_100 (this library is built for sm_100a)", device);
  return PRAXIS_B200_OK;
}

static int64_t padded_rows(int64_t rows, int64_t experts) { return (rows + 127 * experts) / 128 * 128; }

// Workspace of one routed forward, 256-byte aligned pieces.
struct MoeLayout {
  size_t dispatch, row_amax, logits, inverse, csr, pcsr, offsets, tiles, num_tiles, act_amax, act_global, h_amax,
      aq, asf, asf_compact, hidden, hq, hsf, hsf_compact, rows, total;
  int64_t rp;
  int max_tiles;
};

// `passes` lockstep passes: per-group buffers for experts * passes groups.
static MoeLayout moe_layout(int64_t tokens, int top_k, int experts, int passes, int dim, int hidden,
                            bool with_router) {
  MoeLayout L;
  const int groups = experts * passes;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) & ~(size_t)255;
    return o;
  };
  const int64_t r = tokens * top_k;
  L.rp = padded_rows(r, groups);
  L.max_tiles = (int)(L.rp / 128);
  L.dispatch = take(dispatch_workspace_bytes(tokens, top_k, groups));
  L.row_amax = take((size_t)tokens * 2);
  L.logits = take(with_router ? (size_t)tokens * experts * 4 : 0);
  L.inverse = take((size_t)r * 8);
  L.csr = take((size_t)(groups + 1) * 4);
  L.pcsr = take((size_t)(groups + 1) * 4);
  L.offsets = take((size_t)groups * 4);
  L.tiles = take((size_t)(2 * L.max_tiles + 1) * sizeof(TileEntry));
  L.num_tiles = take(8);
  L.act_amax = take((size_t)groups * 4);
  L.act_global = take((size_t)groups * 4);
  L.h_amax = take((size_t)groups * 4);
  L.aq = take((size_t)L.rp * dim / 2);
  L.asf = take((size_t)L.rp * dim / 16 * 4);  // room for the replicated layout
  L.asf_compact = take((size_t)L.rp * dim / 16);
  L.hidden = take((size_t)L.rp * hidden * 2);
  L.hq = take((size_t)L.rp * hidden / 2);
  L.hsf = take((size_t)L.rp * hidden / 16 * 4);
  L.hsf_compact = take((size_t)L.rp * hidden / 16);
  L.rows = take((size_t)L.rp * dim * 2);
  L.total = off;
  return L;
}

// Workspace of the expert-rank forward (expert parallelism).
struct ExpertLayout {
  size_t tiles, num_tiles, h_amax, asf, hidden, hq, hsf_compact, hsf, total;
  int max_tiles;
};

static ExpertLayout expert_layout(int64_t rows, int segments, int dim, int hidden) {
  ExpertLayout L;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) & ~(size_t)255;
    return o;
  };
  L.max_tiles = (int)(rows / 128);
  L.tiles = take((size_t)(2 * L.max_tiles + 1) * sizeof(TileEntry));
  L.num_tiles = take(8);
  L.h_amax = take((size_t)segments * 4);
  L.asf = take((size_t)rows * dim / 16 * 4);
  L.hidden = take((size_t)rows * hidden * 2);
  L.hq = take((size_t)rows * hidden / 2);
  L.hsf_compact = take((size_t)rows * hidden / 16);
  L.hsf = take((size_t)rows * hidden / 16 * 4);
  L.total = off;
  return L;
}

}  // namespace praxis

using namespace praxis;

#define PRAXIS_STREAM(s) static_cast<cudaStream_t>(s)
#define PRAXIS_DEVICE_OR_RETURN(d) \
  do {                             \
    int _rc = use_device(d);       \
    if (_rc) return _rc;           \
  } while (0)

extern "C" {

int praxis_b200_abi_version(void) { return PRAXIS_B200_ABI_VERSION; }

const char* praxis_b200_last_error(void) { return g_message; }

int praxis_b200_device_check(int device) {
  if (use_device(device) != PRAXIS_B200_OK) return 0;
  return sm_count();
}

int praxis_b200_device_error(int device, uint32_t* code) {
  PRAXIS_DEVICE_OR_RETURN(device);
  unsigned int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "device error word: %s", cudaGetErrorString(e));
  if (code) *code = v;
  return PRAXIS_B200_OK;
}

int64_t praxis_b200_padded_rows(int64_t routed_rows, int32_t experts) { return padded_rows(routed_rows, experts); }

int praxis_b200_router_logits(const void* x, const void* weight, int32_t weight_splits, int64_t tokens, int32_t dim,
                              int32_t experts, float* logits, void* row_amax, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (!weight || (tokens > 0 && (!x || !logits))) return set_error(PRAXIS_B200_EINVAL, "router_logits: null pointer");
  return run_router_logits(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(weight), weight_splits,
                           tokens, dim, experts, logits, static_cast<uint16_t*>(row_amax), PRAXIS_STREAM(stream));
}

int praxis_b200_route(const float* logits, const float* bias, int64_t tokens, int32_t experts, int32_t top_k,
                      int32_t activation, int64_t* top_idx, void* gate, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (tokens > 0 && (!logits || !top_idx || !gate)) return set_error(PRAXIS_B200_EINVAL, "route: null pointer");
  return run_route(logits, bias, tokens, experts, top_k, activation, top_idx, static_cast<uint16_t*>(gate),
                   PRAXIS_STREAM(stream));
}

int praxis_b200_row_amax(const void* x, int64_t rows, int32_t cols, void* out, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (rows > 0 && (!x || !out)) return set_error(PRAXIS_B200_EINVAL, "row_amax: null pointer");
  return run_row_amax(static_cast<const uint16_t*>(x), rows, cols, static_cast<uint16_t*>(out), PRAXIS_STREAM(stream));
}

size_t praxis_b200_dispatch_workspace_size(int64_t tokens, int32_t top_k, int32_t experts) {
  return dispatch_workspace_bytes(tokens, top_k, experts);
}

size_t praxis_b200_dispatch_passes_workspace_size(int64_t tokens, int32_t top_k, int32_t experts, int32_t passes) {
  return dispatch_workspace_bytes(tokens, top_k, experts * (passes == 2 ? 2 : 1));
}

int praxis_b200_dispatch_passes(const int64_t* top_idx, const void* gate, const void* row_amax, int64_t tokens,
                                int32_t top_k, int32_t experts, int32_t passes, int64_t pass0_tokens, void* workspace,
                                size_t workspace_size, int64_t* order, int64_t* inverse, int64_t* tokens_out,
                                int32_t* tokens32, void* sorted_gate, int32_t* offsets, int32_t* csr, int32_t* pcsr,
                                int32_t* tiles, int32_t max_tiles, int32_t* num_tiles, float* act_global,
                                uint32_t* act_amax, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if ((tokens > 0 && !top_idx) || !csr || !pcsr || !tiles || !num_tiles || !workspace)
    return set_error(PRAXIS_B200_EINVAL, "dispatch: null pointer");
  if (tokens > 0 && sorted_gate && !gate) return set_error(PRAXIS_B200_EINVAL, "dispatch: sorted_gate needs gate");
  if (passes != 1 && passes != 2) return set_error(PRAXIS_B200_EINVAL, "dispatch: passes must be 1 or 2");
  if (max_tiles < padded_rows(tokens * top_k, (int64_t)experts * passes) / 128)
    return set_error(PRAXIS_B200_EINVAL, "dispatch: max_tiles below padded_rows/128");
  int32_t* off = offsets;
  return run_dispatch(top_idx, static_cast<const uint16_t*>(gate), static_cast<const uint16_t*>(row_amax), tokens,
                      top_k, experts, Passes{passes, passes == 2 ? pass0_tokens : 0}, workspace, workspace_size, order,
                      inverse, tokens_out, tokens32, static_cast<uint16_t*>(sorted_gate), off ? off : csr + 1, csr,
                      pcsr, reinterpret_cast<TileEntry*>(tiles), max_tiles, num_tiles, act_global, act_amax,
                      PRAXIS_STREAM(stream));
}

int praxis_b200_dispatch(const int64_t* top_idx, const void* gate, const void* row_amax, int64_t tokens,
                         int32_t top_k, int32_t experts, void* workspace, size_t workspace_size, int64_t* order,
                         int64_t* inverse, int64_t* tokens_out, int32_t* tokens32, void* sorted_gate,
                         int32_t* offsets, int32_t* csr, int32_t* pcsr, int32_t* tiles, int32_t max_tiles,
                         int32_t* num_tiles, float* act_global, uint32_t* act_amax, int device, void* stream) {
  return praxis_b200_dispatch_passes(top_idx, gate, row_amax, tokens, top_k, experts, 1, 0, workspace,
                                     workspace_size, order, inverse, tokens_out, tokens32, sorted_gate, offsets, csr,
                                     pcsr, tiles, max_tiles, num_tiles, act_global, act_amax, device, stream);
}

int praxis_b200_dispatch_noalloc(const int64_t* top_idx, const void* gate, const void* row_amax, int64_t tokens,
                                 int32_t top_k, int32_t experts, int64_t* order, int64_t* inverse,
                                 int64_t* tokens_out, int32_t* tokens32, void* sorted_gate, int32_t* offsets,
                                 int32_t* csr, int32_t* pcsr, int32_t* tiles, int32_t max_tiles, int32_t* num_tiles,
                                 float* act_global, uint32_t* act_amax, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (tokens < 0 || top_k <= 0 || experts <= 0) return set_error(PRAXIS_B200_EINVAL, "dispatch_noalloc: bad sizes");
  const size_t need = dispatch_workspace_bytes(tokens, top_k, experts);
  if (need > PRAXIS_B200_DISPATCH_NOALLOC_SCRATCH)
    return set_error(PRAXIS_B200_EINVAL,
                     "dispatch_noalloc: %lld rows x %d experts need %zu bytes of scratch, the static scratch holds "
                     "%zu; use praxis_b200_dispatch with a workspace",
                     (long long)(tokens * top_k), experts, need, (size_t)PRAXIS_B200_DISPATCH_NOALLOC_SCRATCH);
  void* scratch = nullptr;
  const int rc = dispatch_noalloc_scratch(device, &scratch);
  if (rc) return rc;
  return praxis_b200_dispatch(top_idx, gate, row_amax, tokens, top_k, experts, scratch,
                              PRAXIS_B200_DISPATCH_NOALLOC_SCRATCH, order, inverse, tokens_out, tokens32, sorted_gate,
                              offsets, csr, pcsr, tiles, max_tiles, num_tiles, act_global, act_amax, device, stream);
}

int praxis_b200_quantize_gather(const void* x, int64_t tokens, int32_t dim, const int64_t* top_idx,
                                const int64_t* inverse, const int32_t* csr, const int32_t* pcsr,
                                const float* act_global, const uint32_t* act_amax, int32_t top_k, int32_t experts,
                                const int32_t* tiles, const int32_t* num_tiles, int32_t max_tiles, void* q, void* sf,
                                int32_t sf_layout, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if ((tokens > 0 && (!x || !top_idx || !inverse)) || !csr || !pcsr || !tiles || !num_tiles || !q || !sf)
    return set_error(PRAXIS_B200_EINVAL, "quantize_gather: null pointer");
  return run_quantize_gather(static_cast<const uint16_t*>(x), tokens, dim, top_idx, inverse, csr, pcsr, act_global,
                             act_amax, top_k, experts, reinterpret_cast<const TileEntry*>(tiles), num_tiles,
                             max_tiles, static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf), sf_layout,
                             PRAXIS_STREAM(stream));
}

int praxis_b200_quantize_rows(const void* x, int32_t k, const int32_t* tiles, const int32_t* num_tiles,
                              int32_t max_tiles, const float* globals, const uint32_t* amax, void* q, void* sf,
                              int32_t sf_layout, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (!x || !tiles || !num_tiles || !q || !sf) return set_error(PRAXIS_B200_EINVAL, "quantize_rows: null pointer");
  return run_quantize_rows(static_cast<const uint16_t*>(x), k, reinterpret_cast<const TileEntry*>(tiles), num_tiles,
                           max_tiles, globals, amax, static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf), sf_layout,
                           PRAXIS_STREAM(stream));
}

int praxis_b200_grouped_gemm(const void* a_q, const void* a_sf, const void* b_q, const void* b_sf,
                             const int32_t* tiles, const int32_t* num_tiles, int32_t max_tiles, int64_t rows_padded,
                             int32_t n, int32_t k, int32_t experts, int32_t epilogue, void* out,
                             const float* act_global, const uint32_t* act_amax, const float* w_global,
                             uint32_t* amax_out, int32_t sf_layout, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (!a_q || !a_sf || !b_q || !b_sf || !tiles || !num_tiles || !out)
    return set_error(PRAXIS_B200_EINVAL, "grouped_gemm: null pointer");
  const int out_cols = epilogue == PRAXIS_B200_EPI_SWIGLU ? n / 2 : n;
  return run_grouped_gemm(a_q, a_sf, b_q, b_sf, reinterpret_cast<const TileEntry*>(tiles), num_tiles, max_tiles,
                          rows_padded, n, k, experts, epilogue, static_cast<uint16_t*>(out), out_cols, act_global,
                          act_amax, w_global, amax_out, sf_layout, PRAXIS_STREAM(stream));
}

int praxis_b200_gemm_swiglu_fp4(const void* a_q, const void* a_sf, const void* b_q, const void* b_sf,
                                const int32_t* tiles, const int32_t* num_tiles, int32_t max_tiles,
                                int64_t rows_padded, int32_t n, int32_t k, int32_t experts, const float* act_global,
                                const uint32_t* act_amax, const float* w_global, float hidden_global, void* q_out,
                                void* sf_out, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (!a_q || !a_sf || !b_q || !b_sf || !tiles || !num_tiles || !q_out || !sf_out)
    return set_error(PRAXIS_B200_EINVAL, "gemm_swiglu_fp4: null pointer");
  return run_grouped_gemm(a_q, a_sf, b_q, b_sf, reinterpret_cast<const TileEntry*>(tiles), num_tiles, max_tiles,
                          rows_padded, n, k, experts, EPI_SWIGLU_FP4, nullptr, n / 2, act_global, act_amax, w_global,
                          nullptr, PRAXIS_B200_SF_COMPACT, PRAXIS_STREAM(stream), 0, 1, static_cast<uint8_t*>(q_out),
                          static_cast<uint8_t*>(sf_out), hidden_global, 0.0f);
}

int praxis_b200_replicate_scales(const void* sf, int64_t rows, int32_t k, int32_t group_rows, void* out, int device,
                                 void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (!sf || !out) return set_error(PRAXIS_B200_EINVAL, "replicate_scales: null pointer");
  return run_replicate_scales(static_cast<const uint8_t*>(sf), rows, k, group_rows, static_cast<uint8_t*>(out),
                              PRAXIS_STREAM(stream));
}

int praxis_b200_rescale_swiglu(const void* raw, int64_t rows, int32_t hidden, const int32_t* pcsr,
                               int32_t experts, const float* act_global, const float* w_global, void* out,
                               void* rowmax, int32_t alu, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (!raw || !pcsr || !act_global || !w_global || !out)
    return set_error(PRAXIS_B200_EINVAL, "rescale_swiglu: null pointer");
  return run_rescale_swiglu(static_cast<const uint16_t*>(raw), rows, hidden, pcsr, experts, act_global, w_global,
                            static_cast<uint16_t*>(out), static_cast<uint16_t*>(rowmax), alu, PRAXIS_STREAM(stream));
}

int praxis_b200_combine(const void* rows, int32_t cols, const int64_t* inverse, const int64_t* top_idx,
                        const void* gate, const int32_t* csr, const int32_t* pcsr, const float* h_global,
                        const uint32_t* h_amax, const float* w_global, int32_t rows_rescaled, float scaling,
                        const void* shared, void* out, int64_t tokens, int32_t top_k, int32_t experts, int device,
                        void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (tokens == 0) return PRAXIS_B200_OK;
  if (!rows || !inverse || !top_idx || !gate || !csr || !pcsr || !out)
    return set_error(PRAXIS_B200_EINVAL, "combine: null pointer");
  return run_combine(static_cast<const uint16_t*>(rows), cols, inverse, top_idx, static_cast<const uint16_t*>(gate),
                     csr, pcsr, h_global, h_amax, w_global, rows_rescaled, scaling,
                     static_cast<const uint16_t*>(shared), static_cast<uint16_t*>(out), tokens, top_k, experts,
                     PRAXIS_STREAM(stream));
}

int praxis_b200_combine_tail(const void* rows, int32_t cols, const int64_t* inverse, const int64_t* top_idx,
                             const void* gate, const int32_t* csr, const int32_t* pcsr, const float* h_global,
                             const uint32_t* h_amax, const float* w_global, int32_t rows_rescaled, float scaling,
                             const void* shared, const praxis_b200_tail* tail, int64_t tokens, int32_t top_k,
                             int32_t experts, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (tail == nullptr) return set_error(PRAXIS_B200_EINVAL, "combine_tail: null tail descriptor");
  if (tokens == 0) return PRAXIS_B200_OK;
  if (!rows || !inverse || !top_idx || !gate || !csr || !pcsr)
    return set_error(PRAXIS_B200_EINVAL, "combine_tail: null pointer");
  return run_combine_tail(static_cast<const uint16_t*>(rows), cols, inverse, top_idx,
                          static_cast<const uint16_t*>(gate), csr, pcsr, h_global, h_amax, w_global, rows_rescaled,
                          scaling, static_cast<const uint16_t*>(shared), tail_args(*tail), tokens, top_k, experts,
                          PRAXIS_STREAM(stream));
}

int praxis_b200_pack_weights(const void* w, int32_t experts, int32_t k, int32_t n, void* q, void* sf,
                             float* global_out, uint32_t* scratch, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (!w || !q || !sf || !global_out || !scratch) return set_error(PRAXIS_B200_EINVAL, "pack_weights: null pointer");
  return run_pack_weights(static_cast<const uint16_t*>(w), experts, k, n, static_cast<uint8_t*>(q),
                          static_cast<uint8_t*>(sf), global_out, scratch, PRAXIS_STREAM(stream));
}

int praxis_b200_interleave_gate_up(const void* q, const void* sf, int32_t experts, int32_t hidden, int32_t dim,
                                   void* q_out, void* sf_out, int device, void* stream) {
  PRAXIS_DEVICE_OR_RETURN(device);
  if (!q || !sf || !q_out || !sf_out) return set_error(PRAXIS_B200_EINVAL, "interleave: null pointer");
  return run_interleave_gate_up(static_cast<const uint8_t*>(q), static_cast<const uint8_t*>(sf), experts, hidden, dim,
                                static_cast<uint8_t*>(q_out), static_cast<uint8_t*>(sf_out), PRAXIS_STREAM(stream));
}

size_t praxis_b200_expert_workspace_size(int64_t rows, int32_t segments, int32_t dim, int32_t hidden) {
  return expert_layout(rows, segments, dim, hidden).total;
}

int praxis_b200_expert_forward(const praxis_b200_expert_args* a) {
  if (!a) return set_error(PRAXIS_B200_EINVAL, "expert_forward: null args");
  PRAXIS_DEVICE_OR_RETURN(a->device);
  const bool hidden_mode = a->hidden_q != nullptr;
  if (!a->counts || !a->starts || !a->act_global || !a->gate_up_q || !a->gate_up_sf || !a->gate_up_global ||
      !a->workspace)
    return set_error(PRAXIS_B200_EINVAL, "expert_forward: null pointer");
  if (hidden_mode ? (!a->hidden_sf || !a->hidden_amax)
                  : (!a->down_q || !a->down_sf || !a->down_global || !a->rows_out))
    return set_error(PRAXIS_B200_EINVAL, "expert_forward: null output or down weight");
  if (a->rows < 0 || a->rows % 128 || a->segments < 1 || a->segments > 1024 || a->experts < 1 || a->dim <= 0 ||
      a->hidden <= 0 || a->sm_limit < 0)
    return set_error(PRAXIS_B200_EINVAL, "expert_forward: bad sizes");
  if (a->dim % 128 || a->hidden % 128)
    return set_error(PRAXIS_B200_EINVAL, "expert_forward: C and F must be multiples of 128");
  const int gl = a->gate_up_sf_layout, dl = a->down_sf_layout;
  if ((gl != PRAXIS_B200_SF_COMPACT && gl != PRAXIS_B200_SF_REPLICATED) ||
      (dl != PRAXIS_B200_SF_COMPACT && dl != PRAXIS_B200_SF_REPLICATED))
    return set_error(PRAXIS_B200_EINVAL, "expert_forward: unknown weight scale layout (%d, %d)", gl, dl);
  if (dl == PRAXIS_B200_SF_REPLICATED && a->dim % 256 != 0)
    return set_error(PRAXIS_B200_EINVAL, "expert_forward: replicated down scales need C % 256 == 0");
  if (a->rows * (int64_t)(a->dim > 2 * a->hidden ? a->dim : 2 * a->hidden) >= ((int64_t)1 << 31) * 8)
    return set_error(PRAXIS_B200_EINVAL, "expert_forward: rows exceed the kernels' indexing range");
  const ExpertLayout L = expert_layout(a->rows, a->segments, a->dim, a->hidden);
  if (a->workspace_size < L.total)
    return set_error(PRAXIS_B200_EINVAL, "expert_forward: workspace %zu < %zu bytes", a->workspace_size, L.total);
  if (a->rows == 0) return PRAXIS_B200_OK;
  if (!a->q || !a->sf) return set_error(PRAXIS_B200_EINVAL, "expert_forward: null rows");
  cudaStream_t s = PRAXIS_STREAM(a->stream);
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  TileEntry* tiles = reinterpret_cast<TileEntry*>(ws + L.tiles);
  int32_t* num_tiles = reinterpret_cast<int32_t*>(ws + L.num_tiles);
  uint32_t* h_amax = reinterpret_cast<uint32_t*>(ws + L.h_amax);
  uint16_t* hidden = reinterpret_cast<uint16_t*>(ws + L.hidden);
  uint8_t* hq = ws + L.hq;
  int rc = run_segment_tiles(a->counts, a->starts, a->segments, tiles, L.max_tiles, num_tiles, s);
  if (rc) return rc;
  const uint8_t* asf = static_cast<const uint8_t*>(a->sf);
  if (gl == PRAXIS_B200_SF_REPLICATED) {
    rc = run_replicate_scales(asf, a->rows, a->dim, 128, ws + L.asf, s);
    if (rc) return rc;
    asf = ws + L.asf;
  }
  uint32_t* amax = hidden_mode ? a->hidden_amax : h_amax;
  cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(uint32_t) * a->segments, s);
  if (e != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "memset: %s", cudaGetErrorString(e));
  rc = run_grouped_gemm(a->q, asf, a->gate_up_q, a->gate_up_sf, tiles, num_tiles, L.max_tiles, a->rows,
                        2 * a->hidden, a->dim, a->experts, EPI_SWIGLU, hidden, a->hidden, a->act_global, nullptr,
                        a->gate_up_global, amax, gl, s, a->sm_limit);
  if (rc) return rc;
  if (hidden_mode)
    return run_quantize_rows(hidden, a->hidden, tiles, num_tiles, L.max_tiles, nullptr, amax,
                             static_cast<uint8_t*>(a->hidden_q), static_cast<uint8_t*>(a->hidden_sf),
                             PRAXIS_B200_SF_COMPACT, s);
  const bool down_rep = dl == PRAXIS_B200_SF_REPLICATED;
  rc = run_quantize_rows(hidden, a->hidden, tiles, num_tiles, L.max_tiles, nullptr, h_amax, hq,
                         down_rep ? ws + L.hsf_compact : ws + L.hsf, PRAXIS_B200_SF_COMPACT, s);
  if (rc) return rc;
  if (down_rep) {
    rc = run_replicate_scales(ws + L.hsf_compact, a->rows, a->hidden, 128, ws + L.hsf, s);
    if (rc) return rc;
  }
  return run_grouped_gemm(hq, ws + L.hsf, a->down_q, a->down_sf, tiles, num_tiles, L.max_tiles, a->rows, a->dim,
                          a->hidden, a->experts, EPI_RESCALE, static_cast<uint16_t*>(a->rows_out), a->dim, nullptr,
                          h_amax, a->down_global, nullptr, dl, s, a->sm_limit);
}

size_t praxis_b200_moe_workspace_size(int64_t tokens, int32_t top_k, int32_t experts, int32_t dim, int32_t hidden,
                                      int32_t with_router, int32_t passes) {
  return moe_layout(tokens, top_k, experts, passes == 2 ? 2 : 1, dim, hidden, with_router != 0).total;
}

int praxis_b200_moe_forward(const praxis_b200_moe_args* a) {
  if (!a) return set_error(PRAXIS_B200_EINVAL, "moe_forward: null args");
  PRAXIS_DEVICE_OR_RETURN(a->device);
  const bool with_router = a->router_weight != nullptr;
  if (!a->x || !a->top_idx || !a->gate || (!a->out && !a->tail) || !a->gate_up_q || !a->gate_up_sf || !a->gate_up_global ||
      !a->down_q || !a->down_sf || !a->down_global || !a->workspace)
    return set_error(PRAXIS_B200_EINVAL, "moe_forward: null pointer");
  const int gl = a->gate_up_sf_layout, dl = a->down_sf_layout;
  if ((gl != PRAXIS_B200_SF_COMPACT && gl != PRAXIS_B200_SF_REPLICATED) ||
      (dl != PRAXIS_B200_SF_COMPACT && dl != PRAXIS_B200_SF_REPLICATED))
    return set_error(PRAXIS_B200_EINVAL, "moe_forward: unknown weight scale layout (%d, %d)", gl, dl);
  if (dl == PRAXIS_B200_SF_REPLICATED && a->dim % 256 != 0)
    return set_error(PRAXIS_B200_EINVAL, "moe_forward: replicated down scales need C % 256 == 0");
  if (a->tokens < 0 || a->dim <= 0 || a->hidden <= 0 || a->experts <= 0 || a->top_k < 1 || a->top_k > 8 ||
      a->top_k > a->experts)
    return set_error(PRAXIS_B200_EINVAL, "moe_forward: bad sizes");
  if (a->dim % 128 || a->hidden % 128) return set_error(PRAXIS_B200_EINVAL, "moe_forward: C and F must be multiples of 128");
  if (a->passes != 0 && a->passes != 1 && a->passes != 2)
    return set_error(PRAXIS_B200_EINVAL, "moe_forward: passes must be 1 or 2");
  const Passes passes{a->passes == 2 ? 2 : 1, a->passes == 2 ? a->pass0_tokens : 0};
  if (passes.n == 2 && (passes.t0 < 0 || passes.t0 > a->tokens))
    return set_error(PRAXIS_B200_EINVAL, "moe_forward: pass 0 tokens outside 0..tokens");
  const int groups = a->experts * passes.n;
  const float fc1 = a->fc1_output_scale;
  if (fc1 < 0.0f || !(fc1 < 3.4e38f)) return set_error(PRAXIS_B200_EINVAL, "moe_forward: bad FC1 output scale");
  if (fc1 > 0.0f && (gl != PRAXIS_B200_SF_COMPACT || (2 * a->hidden) % 256 != 0))
    return set_error(PRAXIS_B200_EINVAL, "moe_forward: the FC1 FP4 output needs compact scales and F %% 128 == 0");
  const int64_t r = a->tokens * a->top_k;
  if ((r + 127 * (int64_t)groups) * (int64_t)(a->dim > 2 * a->hidden ? a->dim : 2 * a->hidden) >= ((int64_t)1 << 31) * 8)
    return set_error(PRAXIS_B200_EINVAL, "moe_forward: chunk exceeds the kernels' indexing range");
  const MoeLayout L = moe_layout(a->tokens, a->top_k, a->experts, passes.n, a->dim, a->hidden, with_router);
  if (a->workspace_size < L.total)
    return set_error(PRAXIS_B200_EINVAL, "moe_forward: workspace %zu < %zu bytes", a->workspace_size, L.total);
  if (a->tokens == 0) return PRAXIS_B200_OK;
  cudaStream_t s = PRAXIS_STREAM(a->stream);
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  uint16_t* row_amax = reinterpret_cast<uint16_t*>(ws + L.row_amax);
  int64_t* inverse = reinterpret_cast<int64_t*>(ws + L.inverse);
  int32_t* csr = reinterpret_cast<int32_t*>(ws + L.csr);
  int32_t* pcsr = reinterpret_cast<int32_t*>(ws + L.pcsr);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  TileEntry* tiles = reinterpret_cast<TileEntry*>(ws + L.tiles);
  int32_t* num_tiles = reinterpret_cast<int32_t*>(ws + L.num_tiles);
  uint32_t* act_amax = reinterpret_cast<uint32_t*>(ws + L.act_amax);
  float* act_global = reinterpret_cast<float*>(ws + L.act_global);
  uint32_t* h_amax = reinterpret_cast<uint32_t*>(ws + L.h_amax);
  uint8_t* aq = ws + L.aq;
  uint8_t* asf = ws + L.asf;
  uint16_t* hidden = reinterpret_cast<uint16_t*>(ws + L.hidden);
  uint8_t* hq = ws + L.hq;
  uint8_t* hsf = ws + L.hsf;
  uint16_t* rows = reinterpret_cast<uint16_t*>(ws + L.rows);
  const uint16_t* x = static_cast<const uint16_t*>(a->x);
  uint16_t* gate = static_cast<uint16_t*>(a->gate);
  int rc;
  if (with_router) {
    float* logits = reinterpret_cast<float*>(ws + L.logits);
    rc = run_router_logits(x, static_cast<const uint16_t*>(a->router_weight), a->router_splits, a->tokens, a->dim,
                           a->experts, logits, row_amax, s);
    if (rc) return rc;
    rc = run_route(logits, a->router_bias, a->tokens, a->experts, a->top_k, a->activation, a->top_idx, gate, s);
  } else {
    rc = run_row_amax(x, a->tokens, a->dim, row_amax, s);
  }
  if (rc) return rc;
  rc = run_dispatch(a->top_idx, gate, row_amax, a->tokens, a->top_k, a->experts, passes, ws + L.dispatch,
                    L.row_amax - L.dispatch, nullptr, inverse, nullptr, nullptr, nullptr, offsets, csr, pcsr, tiles,
                    L.max_tiles, num_tiles, act_global, act_amax, s);
  if (rc) return rc;
  // The quantizers write compact scales (one 4-byte word per row and 64
  // columns); a coalesced pass then builds the replicated copies, cheaper
  // than four scattered word stores per scale group.
  const bool rep = gl == PRAXIS_B200_SF_REPLICATED, down_rep = dl == PRAXIS_B200_SF_REPLICATED;
  rc = run_quantize_gather(x, a->tokens, a->dim, a->top_idx, inverse, csr, pcsr, act_global, nullptr, a->top_k,
                           a->experts, tiles, num_tiles, L.max_tiles, aq, rep ? ws + L.asf_compact : asf,
                           PRAXIS_B200_SF_COMPACT, s, passes);
  if (rc) return rc;
  if (rep) {
    rc = run_replicate_scales(ws + L.asf_compact, L.rp, a->dim, 128, asf, s);
    if (rc) return rc;
  }
  if (fc1 > 0.0f) {
    // calibrated FC1 output: FP4 hidden rows straight from the gate/up
    // epilogue at the frozen global, which the down GEMM's rescale uses too
    rc = run_grouped_gemm(aq, asf, a->gate_up_q, a->gate_up_sf, tiles, num_tiles, L.max_tiles, L.rp, 2 * a->hidden,
                          a->dim, a->experts, EPI_SWIGLU_FP4, nullptr, a->hidden, act_global, nullptr,
                          a->gate_up_global, nullptr, gl, s, 0, passes.n, hq, down_rep ? ws + L.hsf_compact : hsf,
                          fc1, 0.0f);
  } else {
    cudaError_t e = cudaMemsetAsync(h_amax, 0, sizeof(uint32_t) * groups, s);
    if (e != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "memset: %s", cudaGetErrorString(e));
    rc = run_grouped_gemm(aq, asf, a->gate_up_q, a->gate_up_sf, tiles, num_tiles, L.max_tiles, L.rp, 2 * a->hidden,
                          a->dim, a->experts, EPI_SWIGLU, hidden, a->hidden, act_global, nullptr, a->gate_up_global,
                          h_amax, gl, s, 0, passes.n);
    if (rc) return rc;
    rc = run_quantize_rows(hidden, a->hidden, tiles, num_tiles, L.max_tiles, nullptr, h_amax, hq,
                           down_rep ? ws + L.hsf_compact : hsf, PRAXIS_B200_SF_COMPACT, s);
  }
  if (rc) return rc;
  if (down_rep) {
    rc = run_replicate_scales(ws + L.hsf_compact, L.rp, a->hidden, 128, hsf, s);
    if (rc) return rc;
  }
  rc = run_grouped_gemm(hq, hsf, a->down_q, a->down_sf, tiles, num_tiles, L.max_tiles, L.rp, a->dim, a->hidden,
                        a->experts, EPI_RESCALE, rows, a->dim, nullptr, h_amax, a->down_global, nullptr, dl, s, 0,
                        passes.n, nullptr, nullptr, 0.0f, fc1);
  if (rc) return rc;
  if (a->tail != nullptr)
    return run_combine_tail(rows, a->dim, inverse, a->top_idx, gate, csr, pcsr, nullptr, h_amax, a->down_global, 1,
                            a->scaling, static_cast<const uint16_t*>(a->shared), tail_args(*a->tail), a->tokens,
                            a->top_k, a->experts, s, passes);
  return run_combine(rows, a->dim, inverse, a->top_idx, gate, csr, pcsr, nullptr, h_amax, a->down_global, 1,
                     a->scaling, static_cast<const uint16_t*>(a->shared), static_cast<uint16_t*>(a->out), a->tokens,
                     a->top_k, a->experts, s, passes);
}

// ---------------------------------------------------------------------------
// Peer buffers (CUDA IPC) and copies for the expert-parallel exchange
// ---------------------------------------------------------------------------
}  // extern "C"

namespace praxis {
// Copy by the SMs: 16-byte loads of this GPU's memory and stores to dst,
// which may be a peer's mapped buffer (NVLink writes); four loads in flight
// per thread.
constexpr int kPeerCopyThreads = 512;
__global__ void __launch_bounds__(kPeerCopyThreads) peer_copy_kernel(const uint4* __restrict__ src,
                                                                     uint4* __restrict__ dst, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * kPeerCopyThreads;
  int64_t i = (int64_t)blockIdx.x * kPeerCopyThreads + threadIdx.x;
  for (; i + 3 * stride < n; i += 4 * stride) {
    const uint4 a = ldg_stream(src + i), b = ldg_stream(src + i + stride);
    const uint4 c = ldg_stream(src + i + 2 * stride), d = ldg_stream(src + i + 3 * stride);
    dst[i] = a;
    dst[i + stride] = b;
    dst[i + 2 * stride] = c;
    dst[i + 3 * stride] = d;
  }
  for (; i < n; i += stride) dst[i] = ldg_stream(src + i);
}

// One thread waits until *flag (written by another GPU's copy engine into
// this GPU's memory) equals value, for at most timeout_ns of %globaltimer;
// past that it records kErrTimeoutPeer and returns, so the stream goes on and
// the host sees the error at its next check.
__global__ void wait_value_kernel(const int32_t* flag, int32_t value, int64_t timeout_ns) {
  if (threadIdx.x != 0) return;
  const uint64_t start = globaltimer_ns();
  while (true) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v == value) return;
    if (globaltimer_ns() - start > (uint64_t)timeout_ns) {
      record_error(kErrTimeoutPeer);
      return;
    }
    __nanosleep(256);
  }
}
}  // namespace praxis

extern "C" {
static_assert(sizeof(cudaIpcMemHandle_t) == PRAXIS_B200_IPC_HANDLE_BYTES, "IPC handle size");

int praxis_b200_ipc_alloc(size_t bytes, int device, void** ptr) {
  if (ptr == nullptr || bytes == 0) return set_error(PRAXIS_B200_EINVAL, "ipc_alloc: null pointer or zero size");
  int rc = use_device(device);
  if (rc) return rc;
  *ptr = nullptr;
  const cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "ipc_alloc(%zu): %s", bytes, cudaGetErrorString(e));
  return PRAXIS_B200_OK;
}

int praxis_b200_ipc_free(void* ptr, int device) {
  int rc = use_device(device);
  if (rc) return rc;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "ipc_free: %s", cudaGetErrorString(e));
  return PRAXIS_B200_OK;
}

int praxis_b200_ipc_handle(const void* ptr, int device, void* handle) {
  if (ptr == nullptr || handle == nullptr) return set_error(PRAXIS_B200_EINVAL, "ipc_handle: null pointer");
  int rc = use_device(device);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "ipc_handle: %s", cudaGetErrorString(e));
  memcpy(handle, &h, sizeof(h));
  return PRAXIS_B200_OK;
}

int praxis_b200_ipc_open(const void* handle, int device, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return set_error(PRAXIS_B200_EINVAL, "ipc_open: null pointer");
  int rc = use_device(device);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "ipc_open: %s", cudaGetErrorString(e));
  return PRAXIS_B200_OK;
}

int praxis_b200_ipc_close(void* ptr, int device) {
  int rc = use_device(device);
  if (rc) return rc;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "ipc_close: %s", cudaGetErrorString(e));
  return PRAXIS_B200_OK;
}

int praxis_b200_sm_copy(void* dst, const void* src, size_t bytes, int ctas, int device, void* stream) {
  if (bytes == 0) return PRAXIS_B200_OK;
  if (dst == nullptr || src == nullptr) return set_error(PRAXIS_B200_EINVAL, "sm_copy: null pointer");
  if ((((uintptr_t)dst | (uintptr_t)src | bytes) & 15) != 0)
    return set_error(PRAXIS_B200_EINVAL, "sm_copy: addresses and size must be multiples of 16 bytes");
  if (ctas < 1 || ctas > 1024) return set_error(PRAXIS_B200_EINVAL, "sm_copy: ctas must be 1..1024");
  int rc = use_device(device);
  if (rc) return rc;
  peer_copy_kernel<<<ctas, kPeerCopyThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), (int64_t)(bytes / 16));
  return check_launch("sm_copy");
}

int praxis_b200_wait_value(const int32_t* flag, int32_t value, int64_t timeout_ns, int device, void* stream) {
  if (flag == nullptr) return set_error(PRAXIS_B200_EINVAL, "wait_value: null pointer");
  if (((uintptr_t)flag & 3) != 0) return set_error(PRAXIS_B200_EINVAL, "wait_value: flag must be 4-byte aligned");
  if (timeout_ns <= 0 || timeout_ns > 60000000000ll)
    return set_error(PRAXIS_B200_EINVAL, "wait_value: timeout must be in (0, 60 s]");
  int rc = use_device(device);
  if (rc) return rc;
  wait_value_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flag, value, timeout_ns);
  return check_launch("wait_value");
}

int praxis_b200_copy_async(void* dst, const void* src, size_t bytes, int device, void* stream) {
  if (bytes == 0) return PRAXIS_B200_OK;
  if (dst == nullptr || src == nullptr) return set_error(PRAXIS_B200_EINVAL, "copy_async: null pointer");
  int rc = use_device(device);
  if (rc) return rc;
  const cudaError_t e =
      cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(PRAXIS_B200_ECUDA, "copy_async: %s", cudaGetErrorString(e));
  return PRAXIS_B200_OK;
}

}  // extern "C"
