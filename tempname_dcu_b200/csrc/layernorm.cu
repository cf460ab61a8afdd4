// LayerNorm forward / backward for the pre-LN transformer (hidden <= 8192).
//
// Reference parity: python/flux_dcu/model.py:229-233 (F.layer_norm with
// weight, bias and eps 1e-5 on the sequence-parallel residual rows).
//
// Forward: one warp per row (H a multiple of 256, <= 4096, 16-byte aligned
// rows) or one CTA per row (VPT contiguous elements per thread) otherwise;
// two-pass mean/variance from registers; saves mean and rstd (fp32) for the
// backward.
// Backward (H a multiple of 256, <= 4096, 16-byte aligned rows): dx by one
// warp per row with the row held in registers; dgamma / dbeta by the
// two-stage deterministic column reduction of colred.cuh.  Other shapes (and
// the allocation-free entry point): each CTA handles 16 rows, dgamma/dbeta
// partials per CTA, then a fixed-order reduction.  Both are bitwise
// deterministic (no floating-point atomics).
#include <atomic>
#include <mutex>

#include "colred.cuh"
#include "common.cuh"

namespace tdb {
namespace ln {

template <int VPT>
__device__ __forceinline__ void load_row(const uint16_t* p, float (&v)[VPT]) {
#pragma unroll
  for (int i = 0; i < VPT / 8; ++i) {
    const uint4 w = reinterpret_cast<const uint4*>(p)[i];
    const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[8 * i + 2 * j] = bf16_bits_to_float(a[j] & 0xffff);
      v[8 * i + 2 * j + 1] = bf16_bits_to_float(a[j] >> 16);
    }
  }
}

template <int VPT>
__device__ __forceinline__ void store_row(uint16_t* p, const float (&v)[VPT]) {
#pragma unroll
  for (int i = 0; i < VPT / 8; ++i) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * i], v[8 * i + 1]);
    w.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
    w.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
    w.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
    reinterpret_cast<uint4*>(p)[i] = w;
  }
}

// Block-wide sum (blockDim.x <= 1024, multiple of 32).
__device__ __forceinline__ float block_sum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += scratch[i];
  return t;
}

template <int VPT>
__global__ void ln_fwd_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ gamma,
                              const uint16_t* __restrict__ beta, uint16_t* __restrict__ y, float* __restrict__ mean_out,
                              float* __restrict__ rstd_out, int H, float eps) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const int c0 = threadIdx.x * VPT;
  float v[VPT];
  load_row<VPT>(x + row * H + c0, v);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) s += v[i];
  const float mean = block_sum(s, scratch) / float(H);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const float d = v[i] - mean;
    q += d * d;
  }
  const float var = block_sum(q, scratch) / float(H);
  const float rstd = rsqrtf(var + eps);
  float g[VPT], b[VPT];
  load_row<VPT>(gamma + c0, g);
  load_row<VPT>(beta + c0, b);
#pragma unroll
  for (int i = 0; i < VPT; ++i) v[i] = (v[i] - mean) * rstd * g[i] + b[i];
  store_row<VPT>(y + row * H + c0, v);
  if (threadIdx.x == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

constexpr int kBwdRows = 16;

template <int VPT>
__global__ void ln_bwd_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ gamma,
                              const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                              const uint16_t* __restrict__ dy, const uint16_t* __restrict__ dres,
                              uint16_t* __restrict__ dx, float* __restrict__ partial, int rows, int H) {
  __shared__ float scratch[32];
  const int c0 = threadIdx.x * VPT;
  float g[VPT], dg[VPT], db[VPT];
  load_row<VPT>(gamma + c0, g);
#pragma unroll
  for (int i = 0; i < VPT; ++i) dg[i] = db[i] = 0.f;
  const int first = blockIdx.x * kBwdRows;
  for (int r = first; r < first + kBwdRows && r < rows; ++r) {
    float xv[VPT], gy[VPT];
    load_row<VPT>(x + int64_t(r) * H + c0, xv);
    load_row<VPT>(dy + int64_t(r) * H + c0, gy);
    const float mean = mean_in[r], rstd = rstd_in[r];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const float xh = (xv[i] - mean) * rstd;
      xv[i] = xh;
      dg[i] += gy[i] * xh;
      db[i] += gy[i];
      const float d = gy[i] * g[i];
      gy[i] = d;
      s1 += d;
      s2 += d * xh;
    }
    const float c2 = block_sum(s1, scratch) / float(H);
    const float c1 = block_sum(s2, scratch) / float(H);
#pragma unroll
    for (int i = 0; i < VPT; ++i) gy[i] = (gy[i] - xv[i] * c1 - c2) * rstd;
    if (dres) {
      float rr[VPT];
      load_row<VPT>(dres + int64_t(r) * H + c0, rr);
#pragma unroll
      for (int i = 0; i < VPT; ++i) gy[i] += rr[i];
    }
    store_row<VPT>(dx + int64_t(r) * H + c0, gy);
  }
  float* pg = partial + int64_t(blockIdx.x) * 2 * H;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    pg[c0 + i] = dg[i];
    pg[H + c0 + i] = db[i];
  }
}

// dx for H = 256 * CH (CH <= 16): one warp per row, the row's x and dy kept in
// registers as packed bf16 (CH 16-byte chunks per lane), so each input is read
// once; no block-wide synchronisation.
template <int CH>
__global__ void __launch_bounds__(256) ln_bwd_dx_kernel(const uint16_t* __restrict__ x,
                                                        const uint16_t* __restrict__ gamma,
                                                        const float* __restrict__ mean_in,
                                                        const float* __restrict__ rstd_in,
                                                        const uint16_t* __restrict__ dy,
                                                        const uint16_t* __restrict__ dres, uint16_t* __restrict__ dx,
                                                        int rows) {
  constexpr int H = 256 * CH;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + int64_t(row) * H);
  const uint4* dr = reinterpret_cast<const uint4*>(dy + int64_t(row) * H);
  const uint4* gr = reinterpret_cast<const uint4*>(gamma);
  uint4 xv[CH], dv[CH];
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    xv[ch] = xr[ch * 32 + lane];
    dv[ch] = dr[ch * 32 + lane];
  }
  const float mean = mean_in[row], rstd = rstd_in[row];
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    float xf[8], df[8], gf[8];
    colred::unpack8(xv[ch], xf);
    colred::unpack8(dv[ch], df);
    colred::unpack8(gr[ch * 32 + lane], gf);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float d = df[j] * gf[j];
      s1 += d;
      s2 += d * ((xf[j] - mean) * rstd);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  const float c2 = s1 / float(H), c1 = s2 / float(H);
  const uint4* rr = dres ? reinterpret_cast<const uint4*>(dres + int64_t(row) * H) : nullptr;
  uint4* out = reinterpret_cast<uint4*>(dx + int64_t(row) * H);
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    float xf[8], df[8], gf[8], o[8];
    colred::unpack8(xv[ch], xf);
    colred::unpack8(dv[ch], df);
    colred::unpack8(gr[ch * 32 + lane], gf);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = (df[j] * gf[j] - ((xf[j] - mean) * rstd) * c1 - c2) * rstd;
    if (rr) {
      float rf[8];
      colred::unpack8(rr[ch * 32 + lane], rf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] += rf[j];
    }
    uint4 w;
    w.x = pack_bf16x2(o[0], o[1]);
    w.y = pack_bf16x2(o[2], o[3]);
    w.z = pack_bf16x2(o[4], o[5]);
    w.w = pack_bf16x2(o[6], o[7]);
    out[ch * 32 + lane] = w;
  }
}

template <int CH>
static int bwd_fast_launch(const void* x, const void* g, const float* mean, const float* rstd, const void* dy,
                           const void* dres, void* dx, float* dgamma, float* dbeta, float* partial, int rows,
                           int accumulate, cudaStream_t s) {
  constexpr int H = 256 * CH;
  ln_bwd_dx_kernel<CH><<<(rows + 7) / 8, 256, 0, s>>>(
      static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(g), mean, rstd, static_cast<const uint16_t*>(dy),
      static_cast<const uint16_t*>(dres), static_cast<uint16_t*>(dx), rows);
  tdb_host::launched(1);
  const int rpp = colred::rows_per_part(rows, H, tdb_host::sm_count());
  const int nparts = (rows + rpp - 1) / rpp;
  colred::colred_partial<true><<<dim3((H + colred::kColsPerCta - 1) / colred::kColsPerCta, nparts), colred::kThreads,
                                 0, s>>>(static_cast<const uint16_t*>(dy), H, static_cast<const uint16_t*>(x), H,
                                         mean, rstd, rows, H, rpp, partial);
  tdb_host::launched(1);
  colred::colred_finish<<<dim3((H + 63) / 64, 2), 256, 0, s>>>(partial, nparts, H, dgamma, dbeta, accumulate);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

// Forward for H = 256 * CH (CH <= 16): one warp per row, the row held in
// registers as packed bf16; two-pass mean / variance over the registers.
template <int CH>
__global__ void __launch_bounds__(256) ln_fwd_warp_kernel(const uint16_t* __restrict__ x,
                                                          const uint16_t* __restrict__ gamma,
                                                          const uint16_t* __restrict__ beta, uint16_t* __restrict__ y,
                                                          float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                          int rows, float eps) {
  constexpr int H = 256 * CH;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + int64_t(row) * H);
  uint4 xv[CH];
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) xv[ch] = xr[ch * 32 + lane];
  float s = 0.f;
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    float f[8];
    colred::unpack8(xv[ch], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += f[j];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / float(H);
  float q = 0.f;
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    float f[8];
    colred::unpack8(xv[ch], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) q += (f[j] - mean) * (f[j] - mean);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q / float(H) + eps);
  const uint4* gr = reinterpret_cast<const uint4*>(gamma);
  const uint4* br = reinterpret_cast<const uint4*>(beta);
  uint4* out = reinterpret_cast<uint4*>(y + int64_t(row) * H);
#pragma unroll
  for (int ch = 0; ch < CH; ++ch) {
    float f[8], g[8], b[8];
    colred::unpack8(xv[ch], f);
    colred::unpack8(gr[ch * 32 + lane], g);
    colred::unpack8(br[ch * 32 + lane], b);
    uint4 w;
    w.x = pack_bf16x2((f[0] - mean) * rstd * g[0] + b[0], (f[1] - mean) * rstd * g[1] + b[1]);
    w.y = pack_bf16x2((f[2] - mean) * rstd * g[2] + b[2], (f[3] - mean) * rstd * g[3] + b[3]);
    w.z = pack_bf16x2((f[4] - mean) * rstd * g[4] + b[4], (f[5] - mean) * rstd * g[5] + b[5]);
    w.w = pack_bf16x2((f[6] - mean) * rstd * g[6] + b[6], (f[7] - mean) * rstd * g[7] + b[7]);
    out[ch * 32 + lane] = w;
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

template <int CH>
static int fwd_warp_launch(const void* x, const void* g, const void* b, void* y, float* mean, float* rstd, int rows,
                           float eps, cudaStream_t s) {
  ln_fwd_warp_kernel<CH><<<(rows + 7) / 8, 256, 0, s>>>(static_cast<const uint16_t*>(x),
                                                        static_cast<const uint16_t*>(g),
                                                        static_cast<const uint16_t*>(b), static_cast<uint16_t*>(y),
                                                        mean, rstd, rows, eps);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

// Sum the per-CTA partials in CTA order and add into the fp32 accumulators.
__global__ void ln_reduce_partials(const float* __restrict__ partial, int nparts, int H, float* __restrict__ dgamma,
                                   float* __restrict__ dbeta, int accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= 2 * H) return;
  float s = 0.f;
  for (int p = 0; p < nparts; ++p) s += partial[int64_t(p) * 2 * H + c];
  float* dst = c < H ? dgamma + c : dbeta + (c - H);
  *dst = accumulate ? *dst + s : s;
}

template <int VPT>
static int fwd_launch(const void* x, const void* g, const void* b, void* y, float* mean, float* rstd, int rows, int H,
                      float eps, cudaStream_t s) {
  ln_fwd_kernel<VPT><<<rows, H / VPT, 0, s>>>(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(g),
                                              static_cast<const uint16_t*>(b), static_cast<uint16_t*>(y), mean, rstd,
                                              H, eps);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

template <int VPT>
static int bwd_launch(const void* x, const void* g, const float* mean, const float* rstd, const void* dy,
                      const void* dres, void* dx, float* partial, int rows, int H, cudaStream_t s) {
  const int blocks = (rows + kBwdRows - 1) / kBwdRows;
  ln_bwd_kernel<VPT><<<blocks, H / VPT, 0, s>>>(
      static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(g), mean, rstd, static_cast<const uint16_t*>(dy),
      static_cast<const uint16_t*>(dres), static_cast<uint16_t*>(dx), partial, rows, H);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

// Every row kernel moves bf16 rows 16 bytes at a time (uint4), so each bf16
// base pointer must be 16-byte aligned (H % 8 == 0 keeps every row aligned);
// a misaligned view is refused with an error code instead of faulting.
template <class... P>
static bool rows_aligned(const P*... ptrs) {
  return ((reinterpret_cast<uintptr_t>(ptrs) | ...) % 16) == 0;
}

static int pick_vpt(int H) {
  // threads = H / VPT must be a multiple of 32 and <= 1024
  for (int vpt : {8, 16, 32, 64}) {
    if (H % vpt == 0 && (H / vpt) % 32 == 0 && H / vpt <= 1024) return vpt;
  }
  return 0;
}

}  // namespace ln
}  // namespace tdb

using namespace tdb::ln;

TDB_API int tdb_layernorm_fwd(const void* x, const void* gamma, const void* beta, void* y, float* mean, float* rstd,
                              int rows, int H, float eps, void* stream) {
  const int vpt = pick_vpt(H);
  if (!vpt || rows <= 0) return tdb_host::fail(int(cudaErrorInvalidValue), "layernorm: unsupported hidden size %d", H);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!rows_aligned(x, y, gamma, beta))
    return tdb_host::fail(int(cudaErrorInvalidValue), "layernorm: x, y, gamma and beta must be 16-byte aligned");
  if (H % 256 == 0 && H <= 4096) {
    switch (H / 256) {
      case 1: return fwd_warp_launch<1>(x, gamma, beta, y, mean, rstd, rows, eps, s);
      case 2: return fwd_warp_launch<2>(x, gamma, beta, y, mean, rstd, rows, eps, s);
      case 4: return fwd_warp_launch<4>(x, gamma, beta, y, mean, rstd, rows, eps, s);
      case 8: return fwd_warp_launch<8>(x, gamma, beta, y, mean, rstd, rows, eps, s);
      case 16: return fwd_warp_launch<16>(x, gamma, beta, y, mean, rstd, rows, eps, s);
      default: break;
    }
  }
  switch (vpt) {
    case 8: return fwd_launch<8>(x, gamma, beta, y, mean, rstd, rows, H, eps, s);
    case 16: return fwd_launch<16>(x, gamma, beta, y, mean, rstd, rows, H, eps, s);
    case 32: return fwd_launch<32>(x, gamma, beta, y, mean, rstd, rows, H, eps, s);
    default: return fwd_launch<64>(x, gamma, beta, y, mean, rstd, rows, H, eps, s);
  }
}

// Scratch: `partial` holds ceil(rows/16) * 2 * H floats.
TDB_API int tdb_layernorm_bwd_scratch_floats(int rows, int H) { return ((rows + kBwdRows - 1) / kBwdRows) * 2 * H; }

TDB_API int tdb_layernorm_bwd(const void* x, const void* gamma, const float* mean, const float* rstd, const void* dy,
                              const void* dres, void* dx, float* dgamma, float* dbeta, float* partial, int rows, int H,
                              int accumulate, void* stream) {
  const int vpt = pick_vpt(H);
  if (!vpt || rows <= 0 || !partial)
    return tdb_host::fail(int(cudaErrorInvalidValue), "layernorm bwd: unsupported hidden size %d", H);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!rows_aligned(x, dy, dx, gamma, dres, partial))
    return tdb_host::fail(int(cudaErrorInvalidValue),
                          "layernorm bwd: x, dy, dx, gamma, dres and the scratch must be 16-byte aligned");
  // warp-per-row path (its partials need ceil(rows/16)*2*H floats at most,
  // which is what tdb_layernorm_bwd_scratch_floats promises)
  if (H % 256 == 0 && H <= 4096) {
    switch (H / 256) {
      case 1: return bwd_fast_launch<1>(x, gamma, mean, rstd, dy, dres, dx, dgamma, dbeta, partial, rows, accumulate, s);
      case 2: return bwd_fast_launch<2>(x, gamma, mean, rstd, dy, dres, dx, dgamma, dbeta, partial, rows, accumulate, s);
      case 4: return bwd_fast_launch<4>(x, gamma, mean, rstd, dy, dres, dx, dgamma, dbeta, partial, rows, accumulate, s);
      case 8: return bwd_fast_launch<8>(x, gamma, mean, rstd, dy, dres, dx, dgamma, dbeta, partial, rows, accumulate, s);
      case 16:
        return bwd_fast_launch<16>(x, gamma, mean, rstd, dy, dres, dx, dgamma, dbeta, partial, rows, accumulate, s);
      default: break;
    }
  }
  int rc;
  switch (vpt) {
    case 8: rc = bwd_launch<8>(x, gamma, mean, rstd, dy, dres, dx, partial, rows, H, s); break;
    case 16: rc = bwd_launch<16>(x, gamma, mean, rstd, dy, dres, dx, partial, rows, H, s); break;
    case 32: rc = bwd_launch<32>(x, gamma, mean, rstd, dy, dres, dx, partial, rows, H, s); break;
    default: rc = bwd_launch<64>(x, gamma, mean, rstd, dy, dres, dx, partial, rows, H, s); break;
  }
  if (rc) return rc;
  const int nparts = (rows + kBwdRows - 1) / kBwdRows;
  ln_reduce_partials<<<(2 * H + 255) / 256, 256, 0, s>>>(partial, nparts, H, dgamma, dbeta, accumulate);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

// ===========================================================================
// Allocation-free LayerNorm backward: tdb_layernorm_bwd_noalloc
//
// This entry point has no counterpart in the reference.  It exists for callers
// that cannot call cudaMalloc (or any allocating routine) at the point where
// they need the LayerNorm backward: for example a host application whose
// memory planner has already reserved all device memory up front, so a fresh
// allocation would fail or fragment it, or code in the middle of a stream of
// asynchronous work that must not risk the implicit device-wide
// synchronisation cudaMalloc / cudaFree can cause.  Such a caller supplies only
// the inputs and outputs; the per-block partial sums live in a fixed array of
// this library instead of a caller-provided scratch buffer.
//
// Limits and behaviour:
//   * The scratch is one file-scope device array of kNoAllocScratchFloats fp32
//     values (4 MiB).  Every GPU that loads this library holds it until the
//     process exits.  A call needs ceil(rows / 16) * 2 * H floats; larger
//     problems are rejected with cudaErrorInvalidValue and a message naming the
//     limit (use tdb_layernorm_bwd with your own scratch for those).
//   * The first call on a device looks up the array's device address with
//     cudaGetSymbolAddress while that device is current, and caches it per
//     device (an atomic per device ordinal; the lookup itself runs under a
//     mutex).  Make that first call before any stream capture begins.  The
//     cached address is not refreshed after a cudaDeviceReset of that device.
//   * x, dy, dx, gamma and dres (if given) must be 16-byte aligned, like every
//     LayerNorm entry point; misaligned pointers return cudaErrorInvalidValue.
//   * Nothing in the array has to start at zero: every partial that is read
//     is written earlier by the same call.  The array keeps the contents of the
//     last call.
//   * All calls on one device share the array, so calls that can overlap on
//     the GPU (different streams without ordering between them) race and give
//     wrong results.  Order such calls on one stream or with events.
//   * No cudaMalloc, cudaFree or other allocating routine is called.
// ===========================================================================
namespace tdb {
namespace ln {
constexpr int64_t kNoAllocScratchFloats = int64_t(1) << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
// device address of the array per device ordinal, looked up once; not
// refreshed if the process resets a device (cudaDeviceReset) afterwards
static std::atomic<float*> g_noalloc_addr[64];
static std::mutex g_noalloc_mutex;
}  // namespace ln
}  // namespace tdb

// Largest scratch (in floats) the allocation-free entry point can serve.
TDB_API long long tdb_layernorm_bwd_noalloc_max_floats() { return tdb::ln::kNoAllocScratchFloats; }

TDB_API int tdb_layernorm_bwd_noalloc(const void* x, const void* gamma, const float* mean, const float* rstd,
                                      const void* dy, const void* dres, void* dx, float* dgamma, float* dbeta,
                                      int rows, int H, int accumulate, void* stream) {
  const int vpt = pick_vpt(H);
  if (!vpt || rows <= 0)
    return tdb_host::fail(int(cudaErrorInvalidValue), "layernorm bwd (no-alloc): unsupported hidden size %d", H);
  if (!rows_aligned(x, dy, dx, gamma, dres))
    return tdb_host::fail(int(cudaErrorInvalidValue),
                          "layernorm bwd (no-alloc): x, dy, dx, gamma and dres must be 16-byte aligned");
  const int64_t need = int64_t((rows + kBwdRows - 1) / kBwdRows) * 2 * H;
  if (need > tdb::ln::kNoAllocScratchFloats)
    return tdb_host::fail(int(cudaErrorInvalidValue),
                          "layernorm bwd (no-alloc): rows=%d H=%d needs %lld scratch floats but the built-in array "
                          "holds at most %lld; call tdb_layernorm_bwd with caller-provided scratch instead",
                          rows, H, (long long)need, (long long)tdb::ln::kNoAllocScratchFloats);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return tdb_host::fail(int(e), "layernorm bwd (no-alloc): cudaGetDevice failed");
  if (dev < 0 || dev >= 64) return tdb_host::fail(int(cudaErrorInvalidDevice), "layernorm bwd (no-alloc): device %d", dev);
  float* scratch = tdb::ln::g_noalloc_addr[dev].load(std::memory_order_acquire);
  if (scratch == nullptr) {
    std::lock_guard<std::mutex> guard(tdb::ln::g_noalloc_mutex);
    scratch = tdb::ln::g_noalloc_addr[dev].load(std::memory_order_relaxed);
    if (scratch == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, tdb::ln::g_noalloc_scratch);
      if (e != cudaSuccess)
        return tdb_host::fail(int(e), "layernorm bwd (no-alloc): cudaGetSymbolAddress failed on device %d", dev);
      scratch = static_cast<float*>(p);
      tdb::ln::g_noalloc_addr[dev].store(scratch, std::memory_order_release);
    }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc;
  switch (vpt) {
    case 8: rc = bwd_launch<8>(x, gamma, mean, rstd, dy, dres, dx, scratch, rows, H, s); break;
    case 16: rc = bwd_launch<16>(x, gamma, mean, rstd, dy, dres, dx, scratch, rows, H, s); break;
    case 32: rc = bwd_launch<32>(x, gamma, mean, rstd, dy, dres, dx, scratch, rows, H, s); break;
    default: rc = bwd_launch<64>(x, gamma, mean, rstd, dy, dres, dx, scratch, rows, H, s); break;
  }
  if (rc) return rc;
  const int nparts = (rows + kBwdRows - 1) / kBwdRows;
  ln_reduce_partials<<<(2 * H + 255) / 256, 256, 0, s>>>(scratch, nparts, H, dgamma, dbeta, accumulate);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}
