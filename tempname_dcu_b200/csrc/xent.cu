// Vocab-parallel cross-entropy (fp32 softmax over bf16 logits).
//
// Reference parity: python/flux_dcu/model.py:143-176 (VocabCrossEntropy:
// max / sum-exp / target-logit all-reduces across the tensor-parallel group,
// backward softmax - onehot).  Here the per-rank statistics of one row are
// produced by one kernel (online max + rescaled sum-exp + target logit), the
// ranks exchange the [rows, 3] statistics with a single all-gather, a combine
// kernel forms the global (max, sum) and per-row loss, and the backward
// overwrites the logits in place with (softmax - onehot) * scale.  Padded
// vocabulary columns (vocab 50257 padded to a multiple of 8*128) are masked
// out of the softmax.
#include <cfloat>

#include "common.cuh"

namespace tdb {
namespace xent {

constexpr int kThreads = 256;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) {
    m = m2;
    s = s2;
    return;
  }
  const float mx = fmaxf(m, m2);
  s = s * __expf(m - mx) + s2 * __expf(m2 - mx);
  m = mx;
}

// stats[row] = {local max, local sum exp(l - local max), target logit or 0}
__global__ void __launch_bounds__(kThreads) stats_kernel(const uint16_t* __restrict__ logits, int64_t ld,
                                                         const int64_t* __restrict__ targets, int64_t vocab_start,
                                                         int valid_cols, int cols, float* __restrict__ stats) {
  const int64_t row = blockIdx.x;
  const uint16_t* p = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x * 8; c < cols; c += kThreads * 8) {
    const uint4 w = *reinterpret_cast<const uint4*>(p + c);
    const uint32_t a[4] = {w.x, w.y, w.z, w.w};
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = bf16_bits_to_float(a[j] & 0xffff);
      v[2 * j + 1] = bf16_bits_to_float(a[j] >> 16);
    }
    float lm = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (c + j < valid_cols) lm = fmaxf(lm, v[j]);
    if (lm == -INFINITY) continue;
    float ls = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (c + j < valid_cols) ls += __expf(v[j] - lm);
    online_merge(m, s, lm, ls);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm[kThreads / 32], ss[kThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -INFINITY, S = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) online_merge(M, S, sm[w], ss[w]);
    const int64_t t = targets[row] - vocab_start;
    const float tl = (t >= 0 && t < valid_cols) ? bf16_bits_to_float(p[t]) : 0.f;
    stats[row * 3 + 0] = M;
    stats[row * 3 + 1] = S;
    stats[row * 3 + 2] = tl;
  }
}

// all_stats: [world, rows, 3]; writes gstats [rows, 2] = {global max, global
// sum} and the per-row loss.
__global__ void combine_kernel(const float* __restrict__ all_stats, int world, int rows, float* __restrict__ gstats,
                               float* __restrict__ row_loss) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float M = -INFINITY, S = 0.f, T = 0.f;
  for (int w = 0; w < world; ++w) {
    const float* st = all_stats + (int64_t(w) * rows + r) * 3;
    online_merge(M, S, st[0], st[1]);
    T += st[2];
  }
  gstats[2 * r] = M;
  gstats[2 * r + 1] = S;
  row_loss[r] = logf(S) + M - T;
}

// Deterministic mean of the row losses (single block), optionally added to an
// accumulator: out = (accumulate ? out : 0) + scale * sum(row_loss).
__global__ void loss_sum_kernel(const float* __restrict__ row_loss, int rows, float scale, float* __restrict__ out,
                                int accumulate) {
  __shared__ double part[1024];
  double s = 0.0;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) s += double(row_loss[r]);
  part[threadIdx.x] = s;
  __syncthreads();
  for (int stride = blockDim.x / 2; stride; stride >>= 1) {
    if (threadIdx.x < stride) part[threadIdx.x] += part[threadIdx.x + stride];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float v = float(part[0]) * scale;
    *out = accumulate ? *out + v : v;
  }
}

// In place: logits <- (softmax - onehot) * scale; padded columns <- 0.
__global__ void __launch_bounds__(kThreads) grad_kernel(uint16_t* __restrict__ logits, int64_t ld,
                                                        const int64_t* __restrict__ targets, int64_t vocab_start,
                                                        int valid_cols, int cols, const float* __restrict__ gstats,
                                                        float scale) {
  const int64_t row = blockIdx.x;
  uint16_t* p = logits + row * ld;
  const float M = gstats[2 * row], inv = 1.0f / gstats[2 * row + 1];
  const int64_t t = targets[row] - vocab_start;
  for (int c = threadIdx.x * 8; c < cols; c += kThreads * 8) {
    uint4 w = *reinterpret_cast<const uint4*>(p + c);
    uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float lo = bf16_bits_to_float(a[j] & 0xffff), hi = bf16_bits_to_float(a[j] >> 16);
      const int c0 = c + 2 * j, c1 = c0 + 1;
      lo = c0 < valid_cols ? (__expf(lo - M) * inv - (c0 == t ? 1.f : 0.f)) * scale : 0.f;
      hi = c1 < valid_cols ? (__expf(hi - M) * inv - (c1 == t ? 1.f : 0.f)) * scale : 0.f;
      a[j] = pack_bf16x2(lo, hi);
    }
    w.x = a[0]; w.y = a[1]; w.z = a[2]; w.w = a[3];
    *reinterpret_cast<uint4*>(p + c) = w;
  }
}

}  // namespace xent
}  // namespace tdb

using namespace tdb::xent;

TDB_API int tdb_xent_stats(const void* logits, int64_t ld, const int64_t* targets, int64_t vocab_start,
                           int valid_cols, int cols, int rows, float* stats, void* stream) {
  if (!logits || !targets || !stats || rows <= 0 || cols <= 0 || cols % 8 || ld % 8)
    return tdb_host::fail(int(cudaErrorInvalidValue), "xent: columns and ld must be multiples of 8");
  stats_kernel<<<rows, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(logits), ld, targets, vocab_start, valid_cols, cols, stats);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

TDB_API int tdb_xent_combine(const float* all_stats, int world, int rows, float* gstats, float* row_loss,
                             float* loss_out, float loss_scale, int accumulate, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  combine_kernel<<<(rows + 255) / 256, 256, 0, s>>>(all_stats, world, rows, gstats, row_loss);
  tdb_host::launched(1);
  if (loss_out) {
    loss_sum_kernel<<<1, 1024, 0, s>>>(row_loss, rows, loss_scale, loss_out, accumulate);
    tdb_host::launched(1);
  }
  return int(cudaGetLastError());
}

TDB_API int tdb_xent_grad(void* logits, int64_t ld, const int64_t* targets, int64_t vocab_start, int valid_cols,
                          int cols, int rows, const float* gstats, float scale, void* stream) {
  if (cols % 8 || ld % 8) return tdb_host::fail(int(cudaErrorInvalidValue), "xent grad: bad alignment");
  grad_kernel<<<rows, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint16_t*>(logits), ld, targets,
                                                                        vocab_start, valid_cols, cols, gstats, scale);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}
