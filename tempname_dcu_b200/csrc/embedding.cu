// Vocab-parallel token embedding and learned positions, forward and a
// deterministic backward.
//
// Reference parity: python/flux_dcu/model.py:236-249 (masked lookup into the
// local vocabulary shard, SumScatter to the sequence-parallel rows, learned
// positions for the local rows) and the tied LM head (:264-266).
//
// Backward without atomics: the host passes the row indices stably sorted by
// token id; one CTA per sorted position checks whether it starts a segment of
// equal tokens and, if so, sums that segment's gradient rows in order and adds
// the sum into the fp32 gradient row of that token.  The position gradient
// sums rows r == p (mod seq) in row order.
#include "common.cuh"

namespace tdb {
namespace emb {

// out[r, :] = (tok in shard ? table[tok - start, :] : 0) (+ pos[(r + pos_offset) % seq, :])
__global__ void fwd_kernel(const int64_t* __restrict__ tokens, const uint16_t* __restrict__ table, int64_t start,
                           int64_t local_vocab, const uint16_t* __restrict__ pos, int64_t pos_offset, int seq, int H,
                           uint16_t* __restrict__ out) {
  const int64_t r = blockIdx.x;
  const int64_t t = tokens[r] - start;
  const bool mine = t >= 0 && t < local_vocab;
  const uint4* src = reinterpret_cast<const uint4*>(table + (mine ? t : 0) * H);
  const uint4* ps = pos ? reinterpret_cast<const uint4*>(pos + ((r + pos_offset) % seq) * int64_t(H)) : nullptr;
  uint4* dst = reinterpret_cast<uint4*>(out + r * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    float v[8];
    if (mine) {
      const uint4 w = src[c];
      const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[2 * j] = bf16_bits_to_float(a[j] & 0xffff);
        v[2 * j + 1] = bf16_bits_to_float(a[j] >> 16);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    if (ps) {
      const uint4 w = ps[c];
      const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[2 * j] += bf16_bits_to_float(a[j] & 0xffff);
        v[2 * j + 1] += bf16_bits_to_float(a[j] >> 16);
      }
    }
    uint4 o;
    o.x = pack_bf16x2(v[0], v[1]);
    o.y = pack_bf16x2(v[2], v[3]);
    o.z = pack_bf16x2(v[4], v[5]);
    o.w = pack_bf16x2(v[6], v[7]);
    dst[c] = o;
  }
}

// x[r, :] += pos[(r + offset) % seq, :]  (in place, bf16)
__global__ void add_pos_kernel(uint16_t* __restrict__ x, const uint16_t* __restrict__ pos, int64_t offset, int seq,
                               int H) {
  const int64_t r = blockIdx.x;
  uint4* xs = reinterpret_cast<uint4*>(x + r * H);
  const uint4* ps = reinterpret_cast<const uint4*>(pos + ((r + offset) % seq) * int64_t(H));
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    const uint4 a = xs[c], b = ps[c];
    const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, bb[4] = {b.x, b.y, b.z, b.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = pack_bf16x2(bf16_bits_to_float(aa[j] & 0xffff) + bf16_bits_to_float(bb[j] & 0xffff),
                         bf16_bits_to_float(aa[j] >> 16) + bf16_bits_to_float(bb[j] >> 16));
    xs[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// sorted_rows: row indices stably sorted by token id; sorted_tokens the ids in
// that order.  grad[tok - start, :] += sum of dy rows of the segment.
__global__ void bwd_table_kernel(const int64_t* __restrict__ sorted_tokens, const int64_t* __restrict__ sorted_rows,
                                 int rows, const uint16_t* __restrict__ dy, int64_t start, int64_t local_vocab, int H,
                                 float* __restrict__ grad) {
  const int i = blockIdx.x;
  const int64_t tok = sorted_tokens[i];
  if (i > 0 && sorted_tokens[i - 1] == tok) return;  // not a segment start
  const int64_t t = tok - start;
  if (t < 0 || t >= local_vocab) return;
  int end = i + 1;
  while (end < rows && sorted_tokens[end] == tok) ++end;
  float* g = grad + t * H;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float s = g[c];
    for (int j = i; j < end; ++j) s += bf16_bits_to_float(dy[sorted_rows[j] * H + c]);
    g[c] = s;
  }
}

// grad_pos[p, :] += sum_{r : (r + offset) % seq == p} dy[r, :], rows in order.
__global__ void bwd_pos_kernel(const uint16_t* __restrict__ dy, int rows, int64_t offset, int seq, int H,
                               float* __restrict__ grad_pos) {
  const int64_t p = blockIdx.x;  // position
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float s = grad_pos[p * H + c];
    bool any = false;
    // rows r with (r + offset) % seq == p, ascending
    int64_t r0 = ((p - offset) % seq + seq) % seq;
    for (int64_t r = r0; r < rows; r += seq) {
      s += bf16_bits_to_float(dy[r * H + c]);
      any = true;
    }
    if (any) grad_pos[p * H + c] = s;
  }
}

}  // namespace emb
}  // namespace tdb

using namespace tdb::emb;

namespace tdb {
namespace emb {
constexpr int kSortMax = 16384;  // 128 KB of keys in dynamic shared memory
constexpr int kSortThreads = 1024;

// Stable sort of a micro-batch's token ids (one CTA): bitonic sort of the
// unique keys (token << 32 | position) in shared memory, so equal tokens keep
// their position order -- the deterministic order the embedding gradient
// accumulates in.  Padding keys (all ones) sort last.
__global__ void __launch_bounds__(kSortThreads) sort_tokens_kernel(const int64_t* __restrict__ tokens, int n,
                                                                   int64_t* __restrict__ sorted_tokens,
                                                                   int64_t* __restrict__ order) {
  extern __shared__ unsigned long long key[];  // [size], size = next power of two >= n
  int size = 2;
  while (size < n) size <<= 1;
  for (int i = threadIdx.x; i < size; i += blockDim.x)
    key[i] = i < n ? (static_cast<unsigned long long>(tokens[i]) << 32) | static_cast<unsigned int>(i) : ~0ull;
  __syncthreads();
  for (int k = 2; k <= size; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < size; i += blockDim.x) {
        const int p = i ^ j;
        if (p > i) {
          const unsigned long long a = key[i], b = key[p];
          const bool ascending = (i & k) == 0;
          if ((a > b) == ascending) {
            key[i] = b;
            key[p] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    sorted_tokens[i] = static_cast<int64_t>(key[i] >> 32);
    order[i] = static_cast<int64_t>(key[i] & 0xffffffffull);
  }
}
}  // namespace emb
}  // namespace tdb

// tokens [n] (0 <= id < 2^31, n <= 16384) -> ids sorted ascending and the
// original positions, equal ids in position order (a stable sort).
TDB_API int tdb_sort_tokens(const int64_t* tokens, int n, int64_t* sorted_tokens, int64_t* order, void* stream) {
  if (!tokens || !sorted_tokens || !order || n <= 0 || n > tdb::emb::kSortMax)
    return tdb_host::fail(int(cudaErrorInvalidValue), "sort_tokens: 1..%d tokens", tdb::emb::kSortMax);
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(tdb::emb::sort_tokens_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         tdb::emb::kSortMax * 8);
    if (e != cudaSuccess) return tdb_host::fail(int(e), "sort_tokens: cudaFuncSetAttribute failed");
    attr[dev & 63] = true;
  }
  int size = 2;
  while (size < n) size <<= 1;
  tdb::emb::sort_tokens_kernel<<<1, tdb::emb::kSortThreads, size * 8, static_cast<cudaStream_t>(stream)>>>(
      tokens, n, sorted_tokens, order);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

TDB_API int tdb_embedding_fwd(const int64_t* tokens, const void* table, int64_t start, int64_t local_vocab,
                              const void* pos, int64_t pos_offset, int seq, int rows, int H, void* out, void* stream) {
  if (H % 8 || rows <= 0) return tdb_host::fail(int(cudaErrorInvalidValue), "embedding: H must be a multiple of 8");
  fwd_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(tokens, static_cast<const uint16_t*>(table), start,
                                                                  local_vocab, static_cast<const uint16_t*>(pos),
                                                                  pos_offset, seq, H, static_cast<uint16_t*>(out));
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

TDB_API int tdb_add_positions(void* x, const void* pos, int64_t offset, int seq, int rows, int H, void* stream) {
  if (H % 8 || rows <= 0) return tdb_host::fail(int(cudaErrorInvalidValue), "positions: H must be a multiple of 8");
  add_pos_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint16_t*>(x),
                                                                      static_cast<const uint16_t*>(pos), offset, seq, H);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

TDB_API int tdb_embedding_bwd(const int64_t* sorted_tokens, const int64_t* sorted_rows, int rows, const void* dy,
                              int64_t start, int64_t local_vocab, int H, float* grad, void* stream) {
  bwd_table_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      sorted_tokens, sorted_rows, rows, static_cast<const uint16_t*>(dy), start, local_vocab, H, grad);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

TDB_API int tdb_position_bwd(const void* dy, int rows, int64_t offset, int seq, int H, float* grad_pos,
                             void* stream) {
  bwd_pos_kernel<<<seq, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint16_t*>(dy), rows, offset,
                                                                      seq, H, grad_pos);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}
