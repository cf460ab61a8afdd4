// Sequence-parallel all-gather over NVLink peer memory (no NCCL on the data
// path).
//
// Reference parity: python/flux_dcu/model.py:75-81 (gather_rows: an
// all_gather of the row-sharded activations before every column-parallel
// layer, and of the row-parallel output gradient in the backward).
//
// Every rank owns, inside its symmetric heap, two "send slots" of
// [rows, cols] bf16 (alternating by call parity) and one flag word per
// source rank.  One call is three stream-ordered kernels:
//   ag_advance  (1 thread)   epoch += 1 in a device state word, so a captured
//                            CUDA graph replays with fresh epochs
//   ag_stage    (grid)       copy this rank's rows into its send slot[parity]
//                            (or, compressed, ag_stage_taco: TACO packets)
//   ag_pull     (grid)       CTA 0 publishes "epoch ready" to every peer
//                            (system fence, then a release store into the
//                            peer's flag[rank]); every CTA waits (bounded) for
//                            flag[s] >= epoch of each source s and copies
//                            that source's slot into the output with 16-byte
//                            peer loads, own rows included.
// Slot reuse: a rank rewrites slot[p] two calls later, after its previous
// pull kernel has seen every peer's publish of the call in between, which
// each peer issues only after finishing its own earlier pulls.
#include "call_state.cuh"
#include "codec.cuh"
#include "common.cuh"

namespace tdb {
namespace ag {

constexpr int kThreads = 512;
constexpr uint64_t kFlagsBytes = 256;  // flags[source] (uint32), then slots

struct Params {
  const uint64_t* peers;  // heap base of every rank
  const uint32_t* state;  // {epoch, parity}
  int W, rank;
  int64_t rows, cols;     // per-rank block
  uint64_t heap_off;      // this gather's region inside every heap
  uint16_t* out;          // [W * rows, cols]
  uint64_t wait_ns;
};

__device__ __forceinline__ uint8_t* region(const Params& p, int r) {
  return reinterpret_cast<uint8_t*>(p.peers[r] + p.heap_off);
}
__device__ __forceinline__ uint16_t* slot(const Params& p, int r, uint32_t parity) {
  return reinterpret_cast<uint16_t*>(region(p, r) + kFlagsBytes + uint64_t(parity) * p.rows * p.cols * 2);
}

__global__ void ag_advance_kernel(uint32_t* state) { advance_ag_state(state); }

__global__ void __launch_bounds__(kThreads) ag_stage_kernel(const uint16_t* __restrict__ x, int64_t ldx, Params p) {
  uint16_t* dst = slot(p, p.rank, __ldg(p.state + 1));
  const int64_t per_row = p.cols / 8;
  const int64_t n = p.rows * per_row;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row, c = i % per_row;
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(x + r * ldx)[c];
  }
}

// TACO staging (the compressed all-gather): one warp per H128 group of this
// rank's rows (row stride ldx), packets written into the send slot as
// [payload: rows*cols bytes][quant fp32 x groups][adaptive fp32 x groups].
__global__ void __launch_bounds__(256) ag_stage_taco_kernel(const uint16_t* __restrict__ x, int64_t ldx, Params p) {
  const int lane = threadIdx.x & 31;
  const int64_t gpr = p.cols / 128, groups = p.rows * gpr;
  const int64_t g = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (g >= groups) return;
  uint8_t* pk = reinterpret_cast<uint8_t*>(slot(p, p.rank, __ldg(p.state + 1)));
  const int64_t r = g / gpr, c = (g % gpr) * 128;
  const uint2 raw = reinterpret_cast<const uint2*>(x + r * ldx + c)[lane];
  float v[4] = {bf16_bits_to_float(raw.x & 0xffff), bf16_bits_to_float(raw.x >> 16),
                bf16_bits_to_float(raw.y & 0xffff), bf16_bits_to_float(raw.y >> 16)};
  taco::GroupScales sc;
  const uint32_t word = taco::encode_group_warp(v, lane, sc);
  reinterpret_cast<uint32_t*>(pk + g * 128)[lane] = word;
  if (lane == 0) {
    float* scales = reinterpret_cast<float*>(pk + p.rows * p.cols);
    scales[g] = sc.quant;
    scales[groups + g] = sc.adaptive;
  }
}


__global__ void __launch_bounds__(kThreads) ag_pull_kernel(Params p, int* status) {
  __shared__ int s_ok;
  const uint32_t epoch = __ldg(p.state), parity = __ldg(p.state + 1);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    __threadfence_system();  // the staged rows (previous kernel) before the publish
    for (int r = 0; r < p.W; ++r)
      if (r != p.rank) st_release_sys(reinterpret_cast<uint32_t*>(region(p, r)) + p.rank, epoch);
  }
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(region(p, p.rank));
  const int64_t per_row = p.cols / 8;
  const int64_t n = p.rows * per_row;  // 16-byte vectors per source
  for (int k = 0; k < p.W; ++k) {
    const int s = (p.rank + k) % p.W;  // own rows first, then the peers in ring order
    if (s != p.rank) {
      if (threadIdx.x == 0) {
        s_ok = 1;
        if (ld_acquire_sys(flags + s) < epoch) {
          const uint64_t t0 = globaltimer();
          while (ld_acquire_sys(flags + s) < epoch) {
            if (globaltimer() - t0 > p.wait_ns) {
              record_status(status, kTimeoutPeerFlag, 300, s, int(epoch));
              s_ok = 0;
              break;
            }
          }
        }
      }
      __syncthreads();
      if (!s_ok) return;
    }
    const uint4* src = reinterpret_cast<const uint4*>(slot(p, s, parity));
    uint4* dst = reinterpret_cast<uint4*>(p.out + int64_t(s) * p.rows * p.cols);
    // four independent 16-byte peer loads in flight per thread
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n; i += 4 * stride) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = src[i + u * stride];
#pragma unroll
      for (int u = 0; u < 4; ++u) dst[i + u * stride] = v[u];
    }
    for (; i < n; i += stride) dst[i] = src[i];
    __syncthreads();
  }
}

}  // namespace ag
}  // namespace tdb

// Bytes of one gather region inside the symmetric heap (flags + 2 slots).
TDB_API long long tdb_ag_region_bytes(long long rows, long long cols) {
  return (long long)(tdb::ag::kFlagsBytes + 2ull * uint64_t(rows) * uint64_t(cols) * 2ull);
}

// Advance the region's epoch and stage this rank's rows into its send slot
// (the first two steps of a gather; the fused all-gather GEMM pulls itself).
// taco = 1 stages TACO packets instead of BF16 rows (cols % 128 == 0).
TDB_API int tdb_ag_prepare(const void* x, long long ldx, long long rows, long long cols,
                           const unsigned long long* peers, int W, int rank, unsigned long long heap_off,
                           unsigned int* state, int taco, void* stream) {
  if (!x || !peers || !state || W < 2 || W > 64 || rank < 0 || rank >= W || rows <= 0 || cols <= 0 || cols % 8 ||
      ldx % 8 || heap_off % 16 || reinterpret_cast<uintptr_t>(x) % 16 || (taco && cols % 128))
    return tdb_host::fail(int(cudaErrorInvalidValue), "ag_prepare: bad arguments");
  using namespace tdb::ag;
  Params p;
  p.peers = reinterpret_cast<const uint64_t*>(peers);
  p.state = state;
  p.W = W;
  p.rank = rank;
  p.rows = rows;
  p.cols = cols;
  p.heap_off = heap_off;
  p.out = nullptr;
  p.wait_ns = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int sms = tdb_host::sm_count();
  ag_advance_kernel<<<1, 1, 0, s>>>(state);
  if (taco) {
    const int64_t groups = rows * (cols / 128);
    ag_stage_taco_kernel<<<unsigned((groups + 7) / 8), 256, 0, s>>>(static_cast<const uint16_t*>(x), ldx, p);
  } else {
    const int64_t vec = rows * cols / 8;
    const int stage_grid = int(vec / kThreads + 1 < 2 * sms ? vec / kThreads + 1 : 2 * sms);
    ag_stage_kernel<<<stage_grid, kThreads, 0, s>>>(static_cast<const uint16_t*>(x), ldx, p);
  }
  tdb_host::launched(2);
  return int(cudaGetLastError());
}

// out [W*rows, cols] = concat over ranks of every rank's x [rows, cols]
// (row stride ldx).  peers: [W] heap bases; heap_off: this gather's region
// (tdb_ag_region_bytes, zeroed once); state: device uint32 {epoch, parity}
// (zeroed once, one per region).
TDB_API int tdb_allgather(const void* x, long long ldx, long long rows, long long cols, void* out,
                          const unsigned long long* peers, int W, int rank, unsigned long long heap_off,
                          unsigned int* state, double wait_seconds, void* stream) {
  if (!x || !out || !peers || !state || W < 2 || W > 64 || rank < 0 || rank >= W || rows <= 0 || cols <= 0 ||
      cols % 8 || ldx % 8 || heap_off % 16 || ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) % 16))
    return tdb_host::fail(int(cudaErrorInvalidValue), "allgather: bad arguments (16-byte aligned rows needed)");
  using namespace tdb::ag;
  Params p;
  p.peers = reinterpret_cast<const uint64_t*>(peers);
  p.state = state;
  p.W = W;
  p.rank = rank;
  p.rows = rows;
  p.cols = cols;
  p.heap_off = heap_off;
  p.out = static_cast<uint16_t*>(out);
  p.wait_ns = uint64_t(wait_seconds * 1e9);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int sms = tdb_host::sm_count();
  ag_advance_kernel<<<1, 1, 0, s>>>(state);
  const int64_t vec = rows * cols / 8;
  const int stage_grid = int(vec / kThreads + 1 < 2 * sms ? vec / kThreads + 1 : 2 * sms);
  ag_stage_kernel<<<stage_grid, kThreads, 0, s>>>(static_cast<const uint16_t*>(x), ldx, p);
  ag_pull_kernel<<<sms, kThreads, 0, s>>>(p, tdb_host::status_ptr());
  tdb_host::launched(3);
  return int(cudaGetLastError());
}
