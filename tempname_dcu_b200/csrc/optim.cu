// Fused optimizer-side kernels over flat parameter buffers:
//   * deterministic sum of squares (fp64 per-block partials, ordered finish)
//   * clip coefficient min(1, max_norm / (sqrt(total) + 1e-6)) on the device
//   * fused AdamW with fp32 masters: decoupled weight decay on the matrix
//     ranges only, Adam moments, bf16 parameter write-back and gradient reset
//     in one pass, reading the clip coefficient from device memory (no host
//     synchronisation inside the step).
//
// Reference parity: python/flux_dcu/model.py:279-292 (global_grad_norm with
// replicated parameters counted once), :381-388 (AdamW betas (0.9, 0.95),
// eps 1e-8, wd on ndim >= 2 only, fp32 masters) and :410-420 (clip, step,
// copy masters into the bf16 model parameters).
#include "common.cuh"

namespace tdb {
namespace optim {

constexpr int kThreads = 256;
constexpr int kBlocksMax = 1184;  // 8 per SM on 148 SMs

__global__ void sumsq_partial_kernel(const float* __restrict__ g, int64_t n, double* __restrict__ partial) {
  __shared__ double sh[kThreads];
  double s = 0.0;
  const int64_t n4 = n / 4;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x; i < n4; i += int64_t(gridDim.x) * kThreads) {
    const float4 v = g4[i];
    // squares of the fp32 values, accumulated in fp64
    s += double(v.x) * v.x + double(v.y) * v.y + double(v.z) * v.z + double(v.w) * v.w;
  }
  for (int64_t i = n4 * 4 + int64_t(blockIdx.x) * kThreads + threadIdx.x; i < n; i += int64_t(gridDim.x) * kThreads)
    s += double(g[i]) * g[i];
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int st = kThreads / 2; st; st >>= 1) {
    if (threadIdx.x < st) sh[threadIdx.x] += sh[threadIdx.x + st];
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = sh[0];
}

__global__ void sumsq_finish_kernel(const double* __restrict__ partial, int nparts, double* __restrict__ out,
                                    int accumulate) {
  if (threadIdx.x || blockIdx.x) return;
  double s = 0.0;
  for (int i = 0; i < nparts; ++i) s += partial[i];
  *out = accumulate ? *out + s : s;
}

// norm_out = sqrt(total); coef = min(1, max_norm / (norm + 1e-6)); finite
// flag cleared when the norm or the loss is not finite.
__global__ void clip_kernel(const double* __restrict__ total, float max_norm, double* __restrict__ norm_out,
                            float* __restrict__ coef, const float* __restrict__ loss, int* __restrict__ finite,
                            int* __restrict__ step_counter) {
  if (step_counter) *step_counter += 1;  // optimizer step number on the device (CUDA-graph replayable)
  const double norm = sqrt(*total);
  *norm_out = norm;
  const float c = float(double(max_norm) / (norm + 1e-6));
  *coef = c < 1.f ? c : 1.f;
  const bool ok = isfinite(norm) && (loss == nullptr || isfinite(*loss));
  if (!ok) *finite = 0;
}

// Adam bias corrections of optimizer step `step` (same expressions as the host path).
__device__ __forceinline__ void bias_corrections(int step, float beta1, float beta2, float& bc1, float& bc2_sqrt) {
  bc1 = 1.f - powf(beta1, float(step));
  bc2_sqrt = sqrtf(1.f - powf(beta2, float(step)));
}

struct WdRanges {
  int64_t lo0, hi0, lo1, hi1;
  __device__ __forceinline__ bool has_wd(int64_t i) const { return (i >= lo0 && i < hi0) || (i >= lo1 && i < hi1); }
};

__global__ void adamw_kernel(float* __restrict__ master, float* __restrict__ grad, float* __restrict__ m,
                             float* __restrict__ v, uint16_t* __restrict__ param, int64_t n, WdRanges wd, float lr,
                             float beta1, float beta2, float eps, float weight_decay, float bc1, float bc2_sqrt,
                             const float* __restrict__ coef_ptr, const int* __restrict__ finite, int zero_grad,
                             const int* __restrict__ step_dev) {
  if (finite && *finite == 0) return;  // non-finite step: leave state untouched
  if (step_dev) bias_corrections(*step_dev, beta1, beta2, bc1, bc2_sqrt);
  const float coef = coef_ptr ? *coef_ptr : 1.f;
  const float step = lr / bc1;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    float p = master[i];
    const float g = grad[i] * coef;
    if (wd.has_wd(i)) p *= 1.f - lr * weight_decay;
    const float mi = beta1 * m[i] + (1.f - beta1) * g;
    const float vi = beta2 * v[i] + (1.f - beta2) * g * g;
    m[i] = mi;
    v[i] = vi;
    const float denom = sqrtf(vi) / bc2_sqrt + eps;
    p -= step * (mi / denom);
    master[i] = p;
    param[i] = float_to_bf16_bits(p);
    if (zero_grad) grad[i] = 0.f;
  }
}

// Vectorised AdamW: four consecutive elements per thread and iteration
// (16-byte loads of master / grad / m / v, one 8-byte store of the bf16
// parameters).  Needs n % 4 == 0, 16-byte aligned buffers and decay ranges on
// multiples of 4 (the flat parameter layout aligns every tensor to 128).
__device__ __forceinline__ float adam_one(float p, float g, float& m, float& v, bool wd, float lr, float beta1,
                                          float beta2, float eps, float weight_decay, float step, float bc2_sqrt) {
  if (wd) p *= 1.f - lr * weight_decay;
  m = beta1 * m + (1.f - beta1) * g;
  v = beta2 * v + (1.f - beta2) * g * g;
  const float denom = sqrtf(v) / bc2_sqrt + eps;
  return p - step * (m / denom);
}

__global__ void __launch_bounds__(256) adamw4_kernel(float4* __restrict__ master, float4* __restrict__ grad,
                                                     float4* __restrict__ m, float4* __restrict__ v,
                                                     uint2* __restrict__ param, int64_t n4, WdRanges wd, float lr,
                                                     float beta1, float beta2, float eps, float weight_decay,
                                                     float bc1, float bc2_sqrt, const float* __restrict__ coef_ptr,
                                                     const int* __restrict__ finite, int zero_grad,
                                                     const int* __restrict__ step_dev) {
  if (finite && *finite == 0) return;  // non-finite step: leave state untouched
  if (step_dev) bias_corrections(*step_dev, beta1, beta2, bc1, bc2_sqrt);
  const float coef = coef_ptr ? *coef_ptr : 1.f;
  const float step = lr / bc1;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
    float4 p = master[i], g = grad[i], mm = m[i], vv = v[i];
    const bool w = wd.has_wd(4 * i);
    p.x = adam_one(p.x, g.x * coef, mm.x, vv.x, w, lr, beta1, beta2, eps, weight_decay, step, bc2_sqrt);
    p.y = adam_one(p.y, g.y * coef, mm.y, vv.y, w, lr, beta1, beta2, eps, weight_decay, step, bc2_sqrt);
    p.z = adam_one(p.z, g.z * coef, mm.z, vv.z, w, lr, beta1, beta2, eps, weight_decay, step, bc2_sqrt);
    p.w = adam_one(p.w, g.w * coef, mm.w, vv.w, w, lr, beta1, beta2, eps, weight_decay, step, bc2_sqrt);
    master[i] = p;
    m[i] = mm;
    v[i] = vv;
    param[i] = make_uint2(pack_bf16x2(p.x, p.y), pack_bf16x2(p.z, p.w));
    if (zero_grad) grad[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// fp32 -> bf16 copy (initial parameter materialisation).
__global__ void to_bf16_kernel(const float* __restrict__ src, uint16_t* __restrict__ dst, int64_t n) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    dst[i] = float_to_bf16_bits(src[i]);
}

static int grid_for(int64_t n) {
  int64_t b = (n + kThreads - 1) / kThreads;
  return int(b < kBlocksMax ? (b > 0 ? b : 1) : kBlocksMax);
}

}  // namespace optim
}  // namespace tdb

using namespace tdb::optim;

TDB_API int tdb_sumsq_partials_count() { return kBlocksMax; }

// out (+)= sum(g^2) in fp64; `partial` must hold tdb_sumsq_partials_count() doubles.
TDB_API int tdb_sumsq(const float* g, int64_t n, double* partial, double* out, int accumulate, void* stream) {
  if (n < 0 || (reinterpret_cast<uintptr_t>(g) % 16)) return tdb_host::fail(int(cudaErrorInvalidValue), "sumsq: bad args");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(n / 4 + 1);
  sumsq_partial_kernel<<<grid, kThreads, 0, s>>>(g, n, partial);
  tdb_host::launched(1);
  sumsq_finish_kernel<<<1, 32, 0, s>>>(partial, grid, out, accumulate);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

// step_counter (nullable): device int incremented once per call (the optimizer step).
TDB_API int tdb_clip_coef(const double* total, float max_norm, double* norm_out, float* coef, const float* loss,
                          int* finite, int* step_counter, void* stream) {
  clip_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(total, max_norm, norm_out, coef, loss, finite,
                                                              step_counter);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

TDB_API int tdb_adamw(float* master, float* grad, float* m, float* v, void* param, int64_t n, int64_t wd_lo0,
                      int64_t wd_hi0, int64_t wd_lo1, int64_t wd_hi1, float lr, float beta1, float beta2, float eps,
                      float weight_decay, int step, const float* coef, const int* finite, int zero_grad,
                      const int* step_dev, void* stream) {
  // step_dev (nullable): device step number read by the kernel instead of `step`
  if ((!step_dev && step < 1) || n <= 0) return tdb_host::fail(int(cudaErrorInvalidValue), "adamw: bad step/size");
  if (step < 1) step = 1;
  const float bc1 = 1.f - powf(beta1, float(step));
  const float bc2_sqrt = sqrtf(1.f - powf(beta2, float(step)));
  WdRanges wd{wd_lo0, wd_hi0, wd_lo1, wd_hi1};
  const bool vec = n % 4 == 0 && wd_lo0 % 4 == 0 && wd_hi0 % 4 == 0 && wd_lo1 % 4 == 0 && wd_hi1 % 4 == 0 &&
                   ((reinterpret_cast<uintptr_t>(master) | reinterpret_cast<uintptr_t>(grad) |
                     reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) % 16) == 0 &&
                   reinterpret_cast<uintptr_t>(param) % 8 == 0;
  if (vec) {
    const int64_t n4 = n / 4;
    const int64_t blocks = (n4 + 255) / 256;
    const int grid = int(blocks < int64_t(tdb_host::sm_count()) * 16 ? blocks : int64_t(tdb_host::sm_count()) * 16);
    adamw4_kernel<<<grid > 0 ? grid : 1, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<float4*>(master), reinterpret_cast<float4*>(grad), reinterpret_cast<float4*>(m),
        reinterpret_cast<float4*>(v), static_cast<uint2*>(param), n4, wd, lr, beta1, beta2, eps, weight_decay, bc1,
        bc2_sqrt, coef, finite, zero_grad, step_dev);
  } else {
    adamw_kernel<<<grid_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        master, grad, m, v, static_cast<uint16_t*>(param), n, wd, lr, beta1, beta2, eps, weight_decay, bc1, bc2_sqrt,
        coef, finite, zero_grad, step_dev);
  }
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

TDB_API int tdb_to_bf16(const float* src, void* dst, int64_t n, void* stream) {
  to_bf16_kernel<<<grid_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(src, static_cast<uint16_t*>(dst), n);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}
