// Internal declarations shared by the .cu files of the library (not part of
// the C ABI; see include/praxis_b200_moe.h for that).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace praxis {

constexpr int kMaxDevices = 64;

enum Epilogue : int { EPI_PLAIN = 0, EPI_SWIGLU = 1, EPI_RESCALE = 2, EPI_SWIGLU_FP4 = 3 };

struct GemmParams {
  CUtensorMap tmap_a;    // packed FP4 activation rows (padded, expert-grouped)
  CUtensorMap tmap_b;    // packed FP4 weights, E*N rows
  CUtensorMap tmap_sfa;  // A scales as 256-byte rows (2-CTA kernel)
  CUtensorMap tmap_sfb;  // B scales as 256-byte rows (2-CTA kernel)
  CUtensorMap tmap_out;  // bf16 output rows, 64-column x 32-row boxes (2-CTA kernel)
  const uint8_t* sfa;  // swizzled UE4M3 scales of A
  const uint8_t* sfb;  // swizzled UE4M3 scales of B, per expert
  const TileEntry* tiles;   // 128-row tiles; the 256-row pairs follow at tiles + max_tiles
  const int32_t* num_tiles; // {tiles, pairs}
  int32_t max_tiles;
  int32_t N;
  int32_t K;
  uint16_t* out;
  int32_t out_cols;
  int64_t out_rows;  // rows of the output (direct stores stay below)
  const float* act_global;
  const uint32_t* act_amax;
  const float* w_global;
  uint32_t* amax_out;
  int32_t weight_experts;  // tile expert e uses weights (e / groups_per_weight) % weight_experts
  int32_t groups_per_weight;
  uint8_t* q_out;            // EPI_SWIGLU_FP4: E2M1 hidden rows [rows, out_cols / 2]
  uint8_t* sf_out;           // EPI_SWIGLU_FP4: their UE4M3 scales, compact layout
  float fixed_global;        // EPI_SWIGLU_FP4: the frozen hidden global scale
  float act_global_scalar;   // > 0: the activation global of every tile (else act_global / act_amax)
  int32_t sm_limit;        // launch on at most this many SMs (0: all); host side only
};

// Records a message for praxis_b200_last_error and returns `code`.
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);

// Launch with programmatic stream serialization (the kernel starts with
// pdl_wait(), common.cuh); returns the launch status.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
int sm_count();

// Per-device, thread-safe one-time set-up. Kernel attributes such as the
// dynamic shared-memory limit belong to each device's context, so a process
// that drives several GPUs sets them once per device. device_once runs
// `init(device)` (with that device current) the first time `once` is used on
// it; a failed init returns its code and is retried on the next call.
struct DeviceOnce {
  std::mutex mu;
  std::atomic<bool> done[kMaxDevices];
};

template <class F>
inline int device_once(DeviceOnce& once, F&& init) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(PRAXIS_B200_EINVAL, "device index %d outside 0..%d", dev, kMaxDevices - 1);
  if (once.done[dev].load(std::memory_order_acquire)) return PRAXIS_B200_OK;
  std::lock_guard<std::mutex> lock(once.mu);
  if (once.done[dev].load(std::memory_order_relaxed)) return PRAXIS_B200_OK;
  const int rc = init(dev);
  if (rc == PRAXIS_B200_OK) once.done[dev].store(true, std::memory_order_release);
  return rc;
}

// f32(bf16(max(amax, 1e-12))) * f32(1/2688): the QAT global scale from the
// float bits of a bf16-valued maximum (praxis/kernels/nvfp4_moe.py:55-57).
__host__ __device__ __forceinline__ float global_from_amax_bits(uint32_t bits) {
#ifdef __CUDA_ARCH__
  float a = __uint_as_float(bits);
  a = fmaxf(a, 1.0e-12f);
  a = bf16_round(a);
  return __fmul_rn(a, 1.0f / 2688.0f);
#else
  float a;
  memcpy(&a, &bits, 4);
  (void)a;
  return 0.0f;
#endif
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda); nullptr when unavailable.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// Inputs and outputs of the fused MoE tail (combine_tail_kernel): the
// residual x and its new value x_out; w1 (1 + norm weight, fp32) and h_out
// when the RMSNorm follows; mod rows [R, 2C] (shift | scale) with the
// modulation row map {RF, RC, NREG, PW, WD, PH} of global token rows
// (token t of this launch is row t + mod_row0).
struct TailArgs {
  const uint16_t* x;
  uint16_t* x_out;
  const float* w1;
  uint16_t* h_out;
  float eps;
  float norm_scale;
  const uint16_t* mod;
  int mod_fma;
  int64_t mod_geom[6];
  int64_t mod_row0;
};

int run_grouped_gemm(const void* a_q, const void* a_sf, const void* b_q, const void* b_sf, const TileEntry* tiles,
                     const int32_t* num_tiles, int max_tiles, int64_t rows_padded, int32_t n, int32_t k,
                     int32_t experts, int epilogue, uint16_t* out, int32_t out_cols, const float* act_global,
                     const uint32_t* act_amax, const float* w_global, uint32_t* amax_out, int sf_layout,
                     cudaStream_t stream, int sm_limit = 0, int groups_per_weight = 1, uint8_t* q_out = nullptr,
                     uint8_t* sf_out = nullptr, float fixed_global = 0.0f, float act_global_scalar = 0.0f);

}  // namespace praxis
