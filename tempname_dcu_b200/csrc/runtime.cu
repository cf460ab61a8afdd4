// Library-wide runtime pieces of the native layer: the device status word,
// the C error channel, the driver entry point used for TMA descriptors and a
// bounded diagnostic delay kernel.
//
// Reference parity: the reference exports its codec through a ctypes C ABI
// (flux_dcu_codec_abi / flux_dcu_codec_error / flux_dcu_diagnostic_delay,
// src/taco/codec.hip:162-172).  This library keeps that style -- plain
// `extern "C"` entry points returning a CUDA error code -- for every kernel.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "tensor_map.h"

namespace tdb {
__device__ int g_status[4];
}

namespace tdb_host {
static thread_local char g_error[512];

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

static std::atomic<long long> g_launches{0};
void launched(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int* status_ptr() {
  static int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, tdb::g_status) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev] > 0 ? cache[dev] : 148;
}

// Per host thread: launches (and CUDA-graph captures) on one thread do not
// change another thread's grids.
static thread_local int t_grid_limit = 0;

int grid_sms() {
  const int n = sm_count();
  return (t_grid_limit > 0 && t_grid_limit < n) ? t_grid_limit : n;
}

// ---------------------------------------------------------------------------
// cuTensorMapEncodeTiled through the runtime's driver entry point, so that the
// library does not link libcuda directly.
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(int(cudaErrorNotSupported), "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16)
    return fail(int(cudaErrorInvalidValue), "TMA base address must be 16-byte aligned");
  if ((row_stride_elems * elem_bytes) % 16)
    return fail(int(cudaErrorInvalidValue), "TMA row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * uint64_t(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(int(cudaErrorInvalidValue), "cuTensorMapEncodeTiled failed (%d): inner=%llu outer=%llu box=%u,%u",
                int(r), (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
  return 0;
}
}  // namespace tdb_host

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
static constexpr int kAbiVersion = 5;

TDB_API int tdb_abi_version() { return kAbiVersion; }

// Number of kernels launched through this library since load (host counter).
TDB_API long long tdb_launch_count() { return tdb_host::g_launches.load(); }

TDB_API const char* tdb_last_error() { return tdb_host::g_error; }

TDB_API const char* tdb_error_string(int code) { return cudaGetErrorString(static_cast<cudaError_t>(code)); }

// Copies the device status word of the current device to host (synchronous).
TDB_API int tdb_read_status(int* out4) {
  cudaError_t e = cudaMemcpyFromSymbol(out4, tdb::g_status, sizeof(int) * 4);
  return int(e);
}

TDB_API int tdb_clear_status() {
  int zero[4] = {0, 0, 0, 0};
  return int(cudaMemcpyToSymbol(tdb::g_status, zero, sizeof(zero)));
}

// Bounded diagnostic delay: one thread spins on clock64 for `cycles` (at most
// 1e8, the same bound as the reference codec.hip:168).  Used only by the
// artificial lane-skew diagnostic, never in a timed forward.
__global__ void tdb_delay_kernel(unsigned long long cycles) {
  const unsigned long long start = clock64();
  while (clock64() - start < cycles) {
  }
}

TDB_API int tdb_diagnostic_delay(unsigned long long cycles, void* stream) {
  if (cycles == 0 || cycles > 100000000ull) return tdb_host::fail(int(cudaErrorInvalidValue), "delay cycles out of range");
  tdb_delay_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(cycles);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

// Per-device SM count cache for persistent grids.
// Cap the grid of the persistent GEMM-shaped kernels launched next from this
// host thread at `ctas` CTAs (2-CTA kernels: ctas / 2 clusters); 0 removes
// the cap.  Used to run a weight-gradient GEMM on one stream beside a
// communication-bound fused kernel on another, each on its own share of the
// SMs.  Returns the previous cap.
TDB_API int tdb_set_grid_limit(int ctas) {
  const int old = tdb_host::t_grid_limit;
  if (ctas >= 0) tdb_host::t_grid_limit = ctas;
  return old;
}

TDB_API int tdb_sm_count(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
  return n;
}
