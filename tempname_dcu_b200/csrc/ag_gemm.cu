// All-gather fused into the tcgen05 GEMM: out = epilogue(AG(x) @ B^T).
//
// Reference parity: python/flux_dcu/model.py:110-126 (ColumnLinear: gather
// the sequence-parallel rows, then a local GEMM with the weight shard) and the
// row-parallel backward (:139-141: gather the output gradient, then the data
// gradient GEMM).  The reference runs an NCCL all_gather and then torch.mm;
// here ONE persistent kernel does both:
//
//   * the epilogue warps of every CTA first pull the gathered rows: work
//     items (source rank, 128-row block, slice) in the order the GEMM consumes
//     them -- this rank's rows first, then rank+1, rank+2, ... -- each copied
//     with 16-byte loads from the source's symmetric send slot (own rows from
//     the local slot) into the gathered output buffer; after an item the CTA
//     release-adds the block's counter (gpu scope);
//   * the TMA producer waits (bounded) for the counter of a tile's A rows,
//     issues `fence.proxy.async.global` and loads them with TMA -- so the
//     local tiles start at once and remote tiles follow their blocks' arrival
//     while later blocks are still crossing NVLink;
//   * the MMA warp and the TMA-store epilogue are the plain GEMM's.
// The copy waits on other CTAs of the same grid, so the kernel is launched
// cooperatively (all CTAs co-resident or no launch).  Variant 1
// (tdb_ag_set_variant) moves the pull onto four extra warps so that the
// epilogue warps drain finished tiles while rows are still arriving; variant
// 2 keeps sixteen loads in flight per pulling thread (the default from four
// ranks up).  Variant 3 turns the pull into a push: the four extra warps of
// every CTA write this rank's rows with plain 16-byte stores straight into
// every peer's receive buffer (posted writes, no round trip per load), stamp
// a per-slice flag there, and copy the slices that peers pushed into this
// rank's receive buffer on to the gathered output (a local copy, then the
// same per-block counters gate the TMA loads); no send slot is staged.
// Measured on 8 B200s it is no faster than the deep pull: the same bytes
// cross the switch at the same effective rate in either direction.  With
// taco = 1 the send slots hold TACO packets (allgather.cu stages them) and
// the pull decodes peers' rows; a rank's own rows are copied exact.  Peer readiness uses the
// all-gather protocol of allgather.cu (epoch published per source; slot
// parity and epochs on the device).  The gathered rows stay in the output
// buffer (the weight gradient reads them in the backward).  No TMA multicast.
#include <cmath>
#include <type_traits>

#include "call_state.cuh"
#include "codec.cuh"
#include "gemm.cuh"
#include "gemm2.cuh"
#include "gemm_epi.cuh"
#include "tensor_map.h"

namespace tdb {
namespace aggemm {

using gemm::BM;
using gemm::EpiParams;
using gemm::TileOrder;

constexpr uint64_t kFlagsBytes = 256;  // same region layout as allgather.cu

struct Pull {
  const uint64_t* peers;
  uint64_t heap_off;
  const uint32_t* state;  // {epoch, parity} advanced before the call
  int W, rank;
  int64_t rows, cols;     // per-rank block [rows, cols]
  uint16_t* full;         // gathered rows [W * rows, cols]
  uint32_t* ready;        // per 128-row block of `full`
  int slices;             // items per 128-row block
  uint64_t wait_ns;
  // compressed gather: peers' slots hold TACO packets (decoded here); this
  // rank's own rows are copied exact from x
  int taco;
  const uint16_t* x;
  int64_t ldx;
  uint64_t push_off;      // push area inside the region (variant 3): slice flags, then 2 receive buffers
};

constexpr int kSlices = 16;  // items per 128-row block (8 rows each)

// Push area (variant 3), at heap_off + push_off of every rank: epoch stamps
// flags[source][block][slice] (uint32, rounded up to 256 bytes), then two
// receive buffers [W * rows, cols] bf16 (by call parity).
__host__ __device__ __forceinline__ uint64_t push_flags_bytes(int64_t rows, int W) {
  return (uint64_t(W) * uint64_t(rows / 128) * kSlices * 4 + 255) / 256 * 256;
}
__host__ __device__ __forceinline__ uint64_t push_area_bytes(int64_t rows, int64_t cols, int W) {
  return push_flags_bytes(rows, W) + 2ull * uint64_t(W) * uint64_t(rows) * uint64_t(cols) * 2ull;
}
__device__ __forceinline__ uint8_t* push_area(const Pull& a, int r) {
  return reinterpret_cast<uint8_t*>(a.peers[r] + a.heap_off + a.push_off);
}
__device__ __forceinline__ uint16_t* recv_rows(const Pull& a, int r, uint32_t parity, int s, int64_t r0) {
  return reinterpret_cast<uint16_t*>(push_area(a, r) + push_flags_bytes(a.rows, a.W) +
                                     (uint64_t(parity) * a.W * a.rows + uint64_t(s) * a.rows + r0) * a.cols * 2);
}

__device__ __forceinline__ const uint16_t* src_slot(const Pull& a, int r, uint32_t parity) {
  return reinterpret_cast<const uint16_t*>(a.peers[r] + a.heap_off + kFlagsBytes +
                                           uint64_t(parity) * a.rows * a.cols * 2);
}

__device__ __forceinline__ void named_sync_epilogue() { asm volatile("bar.sync 1, 128;" ::: "memory"); }


// Compressed gather: decode `nrows` rows starting at r0 of source s's TACO
// packets into the gathered buffer; one warp per H128 group, four groups'
// loads in flight per warp.
__device__ __forceinline__ void decode_rows(const Pull& a, int s, uint32_t parity, int64_t r0, int nrows, int et) {
  const int warp = et >> 5, lane = et & 31;
  const uint8_t* pk = reinterpret_cast<const uint8_t*>(src_slot(a, s, parity));
  const int64_t gpr = a.cols / 128, groups = a.rows * gpr;
  const float* scales = reinterpret_cast<const float*>(pk + a.rows * a.cols);
  const int total = int(nrows * gpr);
  constexpr int U = 4;
  for (int g0 = warp * U; g0 < total; g0 += 4 * U) {
    uint32_t word[U];
    float q[U], ad[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (g0 + u < total) {
        const int64_t gi = (r0 + (g0 + u) / gpr) * gpr + (g0 + u) % gpr;
        word[u] = reinterpret_cast<const uint32_t*>(pk + gi * 128)[lane];
        q[u] = scales[gi];
        ad[u] = scales[groups + gi];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (g0 + u < total) {
        float v[4];
        taco::decode_group_warp(word[u], q[u], ad[u], lane, v);
        const int64_t row = r0 + (g0 + u) / gpr, col = ((g0 + u) % gpr) * 128;
        uint2 o;
        o.x = uint32_t(float_to_bf16_bits(v[0])) | (uint32_t(float_to_bf16_bits(v[1])) << 16);
        o.y = uint32_t(float_to_bf16_bits(v[2])) | (uint32_t(float_to_bf16_bits(v[3])) << 16);
        reinterpret_cast<uint2*>(a.full + (int64_t(s) * a.rows + row) * a.cols + col)[lane] = o;
      }
    }
  }
}

// Executed by the 128 epilogue threads of every CTA before their first tile.
// `s_ok` is the epilogue scratch word of the mainloop's barrier slot (no static
// shared memory: the dynamic allocation already uses the per-block maximum).
// `et` is the thread's index among the 128 pulling threads (four warps).
template <int U>
__device__ void pull_rows(const Pull& a, volatile int& s_ok, int* status, int et) {
  const uint32_t epoch = __ldg(a.state), parity = __ldg(a.state + 1);
  if (blockIdx.x == 0 && et == 0) {
    __threadfence_system();  // the staged rows (previous kernel) before the publish
    for (int r = 0; r < a.W; ++r)
      if (r != a.rank) st_release_sys(reinterpret_cast<uint32_t*>(a.peers[r] + a.heap_off) + a.rank, epoch);
  }
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(a.peers[a.rank] + a.heap_off);
  const int nblk = int(a.rows / 128);
  const int rows_per_item = 128 / a.slices;
  const int64_t vec_per_row = a.cols / 8;
  const int64_t n = int64_t(rows_per_item) * vec_per_row;  // 16-byte vectors per item
  const int items = a.W * nblk * a.slices;
  int checked = -1;  // last source whose publish this CTA has seen
  for (int w = blockIdx.x; w < items; w += gridDim.x) {
    const int k = w / (nblk * a.slices);
    const int s = (a.rank + k) % a.W;
    const int b = (w / a.slices) % nblk, j = w % a.slices;
    if (s != a.rank && s != checked) {
      if (et == 0) {
        s_ok = 1;
        if (ld_acquire_sys(flags + s) < epoch) {
          const uint64_t t0 = globaltimer();
          while (ld_acquire_sys(flags + s) < epoch) {
            if (globaltimer() - t0 > a.wait_ns) {
              record_status(status, kTimeoutPeerFlag, 310, s, int(epoch));
              s_ok = 0;
              break;
            }
          }
        }
      }
      named_sync_epilogue();
      if (!s_ok) return;
      checked = s;
    }
    const int64_t r0 = int64_t(b) * 128 + int64_t(j) * rows_per_item;  // row inside the source block
    if (a.taco && s != a.rank) {
      decode_rows(a, s, parity, r0, rows_per_item, et);
    } else {
      uint4* dst = reinterpret_cast<uint4*>(a.full + (int64_t(s) * a.rows + r0) * a.cols);
      if (a.taco) {  // own rows, exact, from the caller's input (row stride ldx)
        for (int64_t i = et; i < n; i += 128) {
          const int64_t rr = i / vec_per_row, c = i % vec_per_row;
          dst[i] = reinterpret_cast<const uint4*>(a.x + (r0 + rr) * a.ldx)[c];
        }
      } else {
        const uint4* src = reinterpret_cast<const uint4*>(src_slot(a, s, parity) + r0 * a.cols);
        int64_t i = et;
        for (; i + (U - 1) * 128 < n; i += U * 128) {  // U 16-byte loads in flight per thread
          uint4 v[U];
#pragma unroll
          for (int u = 0; u < U; ++u) v[u] = src[i + u * 128];
#pragma unroll
          for (int u = 0; u < U; ++u) dst[i + u * 128] = v[u];
        }
        for (; i < n; i += 128) dst[i] = src[i];
      }
    }
    named_sync_epilogue();
    if (et == 0) {
      __threadfence();
      red_release_gpu(a.ready + s * nblk + b, 1u);
    }
  }
}

// Variant 3, executed by the four auxiliary warps of every CTA.  Items, in
// index order (CTA c takes c, c + grid, ...; a CTA's pushes precede its
// collects, and pushes never wait, so every collect is eventually served):
//   own:     copy a slice of this rank's rows from x into the gathered output;
//   push:    write a slice of this rank's rows into peer d's receive buffer
//            (d = rank-1, rank-2, ...: the peer that consumes this rank's rows
//            soonest first), then stamp flags[rank][block][slice] = epoch there;
//   collect: wait (bounded) for source s's stamp (s = rank+1, rank+2, ...: the
//            GEMM's order), copy the slice from the receive buffer (local
//            memory, L2-only loads) into the gathered output.
// After own and collect items the block's counter is release-added (gpu
// scope) for the TMA producer's gate.  Receive-buffer reuse: a peer writes
// buffer[p] again two calls later, after its previous kernel has consumed this
// rank's pushes of the call in between, which this rank issues only after its
// own earlier kernel -- the one that read buffer[p] -- has ended.
template <int U>
__device__ __forceinline__ void copy_item(uint4* dst, const uint16_t* src, int64_t lds, int64_t vec_per_row, int64_t n,
                                          int et, bool l2_only) {
  int64_t i = et;
  for (; i + (U - 1) * 128 < n; i += U * 128) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t k = i + u * 128, rr = k / vec_per_row, c = k % vec_per_row;
      const uint4* sp = reinterpret_cast<const uint4*>(src + rr * lds) + c;
      v[u] = l2_only ? __ldcg(sp) : *sp;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) dst[i + u * 128] = v[u];
  }
  for (; i < n; i += 128) {
    const int64_t rr = i / vec_per_row, c = i % vec_per_row;
    const uint4* sp = reinterpret_cast<const uint4*>(src + rr * lds) + c;
    dst[i] = l2_only ? __ldcg(sp) : *sp;
  }
}

__device__ void push_rows(const Pull& a, volatile int& s_ok, int* status, int et) {
  const uint32_t epoch = __ldg(a.state), parity = __ldg(a.state + 1);
  const int nblk = int(a.rows / 128);
  const int rows_per_item = 128 / kSlices;
  const int64_t vec_per_row = a.cols / 8;
  const int64_t n = int64_t(rows_per_item) * vec_per_row;  // 16-byte vectors per item
  const int per_source = nblk * kSlices;
  const int own = per_source, pushes = (a.W - 1) * per_source;
  const int items = own + 2 * pushes;
  for (int w = blockIdx.x; w < items; w += gridDim.x) {
    if (w < own) {
      const int b = w / kSlices, j = w % kSlices;
      const int64_t r0 = int64_t(b) * 128 + int64_t(j) * rows_per_item;
      copy_item<8>(reinterpret_cast<uint4*>(a.full + (int64_t(a.rank) * a.rows + r0) * a.cols), a.x + r0 * a.ldx,
                   a.ldx, vec_per_row, n, et, false);
      named_sync_epilogue();
      if (et == 0) {
        __threadfence();
        red_release_gpu(a.ready + a.rank * nblk + b, 1u);
      }
    } else if (w < own + pushes) {
      const int q = w - own;
      const int d = (a.rank - 1 - q / per_source + a.W) % a.W;
      const int b = (q % per_source) / kSlices, j = q % kSlices;
      const int64_t r0 = int64_t(b) * 128 + int64_t(j) * rows_per_item;
      copy_item<8>(reinterpret_cast<uint4*>(recv_rows(a, d, parity, a.rank, r0)), a.x + r0 * a.ldx, a.ldx,
                   vec_per_row, n, et, false);
      __threadfence_system();  // this thread's peer stores, before the CTA's stamp
      named_sync_epilogue();
      if (et == 0) {
        uint32_t* flag = reinterpret_cast<uint32_t*>(push_area(a, d)) + (a.rank * nblk + b) * kSlices + j;
        st_release_sys(flag, epoch);
      }
    } else {
      const int q = w - own - pushes;
      const int s = (a.rank + 1 + q / per_source) % a.W;
      const int b = (q % per_source) / kSlices, j = q % kSlices;
      const int64_t r0 = int64_t(b) * 128 + int64_t(j) * rows_per_item;
      if (et == 0) {
        const uint32_t* flag = reinterpret_cast<const uint32_t*>(push_area(a, a.rank)) + (s * nblk + b) * kSlices + j;
        s_ok = 1;
        if (int32_t(ld_acquire_sys(flag) - epoch) < 0) {
          const uint64_t t0 = globaltimer();
          while (int32_t(ld_acquire_sys(flag) - epoch) < 0) {
            if (globaltimer() - t0 > a.wait_ns) {
              record_status(status, kTimeoutPeerFlag, 311, s, int(epoch));
              s_ok = 0;
              break;
            }
          }
        }
      }
      named_sync_epilogue();
      if (!s_ok) return;
      copy_item<8>(reinterpret_cast<uint4*>(a.full + (int64_t(s) * a.rows + r0) * a.cols),
                   recv_rows(a, a.rank, parity, s, r0), a.cols, vec_per_row, n, et, true);
      named_sync_epilogue();
      if (et == 0) {
        __threadfence();
        red_release_gpu(a.ready + s * nblk + b, 1u);
      }
    }
  }
}

// PULL = 0: the epilogue warps (2..5) pull before their first tile, so the
// epilogue of the first tiles waits for the whole pull.  PULL = 1: four
// extra warps (6..9) pull while the epilogue warps drain finished tiles, four
// 16-byte loads in flight per thread; PULL = 2: the same warps with sixteen
// loads in flight per thread (32 KB per SM), for a link whose latency under
// all-to-all load needs more bytes in flight to reach its bandwidth.
template <class Inner, int PULL>
struct PullEpi {
  static constexpr bool AUX = PULL != 0;
  const EpiParams& p;
  const Pull& a;
  Inner inner;
  static constexpr int kSmemBytes = Inner::kSmemBytes;
  static constexpr int kAuxWarps = AUX ? 4 : 0;
  __device__ __forceinline__ PullEpi(const EpiParams& ep, const Pull& pull) : p(ep), a(pull), inner{ep} {}
  int* scratch = nullptr;
  __device__ __forceinline__ void set_smem(uint8_t* s) {
    scratch = reinterpret_cast<int*>(s - 16);
    inner.set_smem(s);
  }
  __device__ __forceinline__ void prologue(int* status) {
    if constexpr (!AUX) pull_rows<4>(a, *scratch, status, int(threadIdx.x) - 64);
  }
  __device__ __forceinline__ void aux(int* status) {
    if constexpr (PULL == 3) push_rows(a, *scratch, status, int(threadIdx.x) - 192);
    else if constexpr (AUX) pull_rows<PULL == 2 ? 16 : 4>(a, *scratch, status, int(threadIdx.x) - 192);
  }
  __device__ __forceinline__ void tile_begin(int mb, int nb) { inner.tile_begin(mb, nb); }
  __device__ __forceinline__ void chunk(int row, int col, int c, const uint32_t (&r)[32]) { inner.chunk(row, col, c, r); }
  __device__ __forceinline__ void tile_end(int mb, int nb, int q, int lane) { inner.tile_end(mb, nb, q, lane); }
};

template <int BN, bool B_MN, int MODE, int PULL>
__global__ void __launch_bounds__(gemm::kThreads + (PULL ? 128 : 0), 1)
    ag_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int K,
                   TileOrder order, const __grid_constant__ EpiParams ep, const __grid_constant__ Pull pull,
                   int* status) {
  using Inner = typename gemm::EpiFor<MODE>::type;
  PullEpi<Inner, PULL> epi(ep, pull);
  gemm::gemm_mainloop<BN, false, B_MN>(&tmA, &tmB, K, order, epi, status);
}

constexpr int k2Stages = 6;

template <bool B_MN, int MODE, int PULL>
__global__ void __launch_bounds__(gemm2::kThreads + (PULL ? 128 : 0), 1)
    ag_gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int K,
                    TileOrder order, const __grid_constant__ EpiParams ep, const __grid_constant__ Pull pull,
                    int* status) {
  using Inner = typename gemm::EpiFor<MODE>::type;
  using Epi = PullEpi<Inner, PULL>;
  Epi epi(ep, pull);
  gemm2::mainloop<false, B_MN, Epi, k2Stages>(&tmA, &tmB, K, order, epi, status);
}

template <class Kern>
static int launch_coop(Kern kern, dim3 grid, int threads, int smem, int cluster, cudaStream_t s, const CUtensorMap& ta,
                       const CUtensorMap& tb, int K, const TileOrder& order, const EpiParams& ep, const Pull& pull,
                       int* status) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeCooperative;
  attr[na].val.cooperative = 1;
  ++na;
  if (cluster > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, K, order, ep, pull, status);
  tdb_host::launched(1);
  if (e != cudaSuccess) return tdb_host::fail(int(e), "ag_gemm: cooperative launch failed: %s", cudaGetErrorString(e));
  return 0;
}

template <int BN, bool B_MN, int MODE, int PULL>
static int launch1(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, TileOrder order,
                   const EpiParams& ep, const Pull& pull, cudaStream_t s) {
  using Cfg = gemm::Config<BN>;
  constexpr int kSmem = Cfg::kSmemBytes + gemm::EpiFor<MODE>::type::kSmemBytes;
  auto kern = ag_gemm_kernel<BN, B_MN, MODE, PULL>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return tdb_host::fail(int(e), "ag_gemm: smem attribute");
    attr[dev & 63] = true;
  }
  order.num_m = (M + BM - 1) / BM;
  order.num_n = (N + BN - 1) / BN;
  order.num_tiles = order.num_m * order.num_n;
  const int sms = tdb_host::grid_sms();
  const int grid = order.num_tiles < sms ? order.num_tiles : sms;
  return launch_coop(kern, dim3(grid), gemm::kThreads + (PULL ? 128 : 0), kSmem, 1, s, ta, tb, K, order, ep, pull,
                     tdb_host::status_ptr());
}

template <bool B_MN, int MODE, int PULL>
static int launch2(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, TileOrder order,
                   const EpiParams& ep, const Pull& pull, cudaStream_t s) {
  using Cfg = gemm2::Config<k2Stages>;
  constexpr int kSmem = Cfg::kSmemBytes + gemm::EpiFor<MODE>::type::kSmemBytes;
  constexpr int kBlock = gemm2::kThreads + (PULL ? 128 : 0);
  auto kern = ag_gemm2_kernel<B_MN, MODE, PULL>;
  static int max_clusters[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!max_clusters[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return tdb_host::fail(int(e), "ag_gemm2: smem attribute");
    // clusters that can be resident at once (the cooperative launch needs all of them)
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(tdb_host::sm_count());
    cfg.blockDim = dim3(kBlock);
    cfg.dynamicSmemBytes = kSmem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess || n <= 0) return tdb_host::fail(int(e), "ag_gemm2: no resident 2-CTA clusters");
    max_clusters[dev & 63] = n;
  }
  order.num_m = (M + 255) / 256;
  order.num_n = (N + 255) / 256;
  order.num_tiles = order.num_m * order.num_n;
  int pairs = max_clusters[dev & 63];
  if (pairs > tdb_host::grid_sms() / 2) pairs = tdb_host::grid_sms() / 2 > 0 ? tdb_host::grid_sms() / 2 : 1;
  const int clusters = order.num_tiles < pairs ? order.num_tiles : pairs;
  return launch_coop(kern, dim3(2 * clusters), kBlock, kSmem, 2, s, ta, tb, K, order, ep, pull,
                     tdb_host::status_ptr());
}

template <bool B_MN, int MODE, int PULL>
static int dispatch_tile_aux(int bn, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K,
                             const TileOrder& order, const EpiParams& ep, const Pull& pull, cudaStream_t s) {
  switch (bn) {
    case 512: return launch2<B_MN, MODE, PULL>(ta, tb, M, N, K, order, ep, pull, s);
    case 256: return launch1<256, B_MN, MODE, PULL>(ta, tb, M, N, K, order, ep, pull, s);
    case 192: return launch1<192, B_MN, MODE, PULL>(ta, tb, M, N, K, order, ep, pull, s);
    default: return launch1<128, B_MN, MODE, PULL>(ta, tb, M, N, K, order, ep, pull, s);
  }
}

// Row movement of the following calls: 0 epilogue-warp pull prologue, 1 four
// auxiliary warps pull, 2 the same with 16 loads in flight per thread, 3 four
// auxiliary warps push (set with tdb_ag_set_variant).  kAuto (the default)
// takes 2 from four ranks up and 0 below: measured on 8 B200 (QKV / FC1
// shapes, us) 0: 94.8 / 103.5, 2: 84.8 / 96.7, 3: 94.5 / 104.1; on 2 B200
// 0: 96.8 / 138.3, 2: 103.2 / 142.7, 3: 95.1 / 139.0.
constexpr int kAuto = -1;
static int g_variant = kAuto;
static int resolve_variant(int W) { return g_variant != kAuto ? g_variant : (W >= 4 ? 2 : 0); }

template <bool B_MN, int MODE>
static int dispatch_tile(int variant, int bn, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K,
                         const TileOrder& order, const EpiParams& ep, const Pull& pull, cudaStream_t s) {
  switch (variant) {
    case 1: return dispatch_tile_aux<B_MN, MODE, 1>(bn, ta, tb, M, N, K, order, ep, pull, s);
    case 2: return dispatch_tile_aux<B_MN, MODE, 2>(bn, ta, tb, M, N, K, order, ep, pull, s);
    case 3: return dispatch_tile_aux<B_MN, MODE, 3>(bn, ta, tb, M, N, K, order, ep, pull, s);
    default: return dispatch_tile_aux<B_MN, MODE, 0>(bn, ta, tb, M, N, K, order, ep, pull, s);
  }
}

template <bool B_MN>
static int dispatch_mode(int variant, int mode, int bn, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N,
                         int K, const TileOrder& order, const EpiParams& ep, const Pull& pull, cudaStream_t s) {
  using namespace gemm;
  switch (mode) {
    case kStore: return dispatch_tile<B_MN, kTmaBase + kStore>(variant, bn, ta, tb, M, N, K, order, ep, pull, s);
    case kBias: return dispatch_tile<B_MN, kTmaBase + kBias>(variant, bn, ta, tb, M, N, K, order, ep, pull, s);
    case kBiasGelu:
      return dispatch_tile<B_MN, kTmaBase + kBiasGelu>(variant, bn, ta, tb, M, N, K, order, ep, pull, s);
    case kGeluBwd:
      return dispatch_tile<B_MN, kTmaBase + kGeluBwd>(variant, bn, ta, tb, M, N, K, order, ep, pull, s);
  }
  return tdb_host::fail(int(cudaErrorInvalidValue), "ag_gemm: mode %d unsupported (0-3)", mode);
}

__global__ void push_advance_kernel(uint32_t* state) { advance_ag_state(state); }

}  // namespace aggemm
namespace gemm {
int make_operand_map(CUtensorMap* map, const void* ptr, bool mn_major, int mn, int K, int64_t ld, int tile_mn);
int pick_tile(int M, int N, int K, int sms);
}  // namespace gemm
}  // namespace tdb


// Bytes of the fused all-gather GEMM's region: the all-gather region
// (tdb_ag_region_bytes: flags and send slots for the pull variants) followed
// by the push area of variant 3 (slice flags and two receive buffers).
TDB_API long long tdb_ag_gemm_region_bytes(long long rows, long long cols, int W) {
  if (rows <= 0 || cols <= 0 || rows % 128 || W < 2 || W > 64) return 0;
  return tdb_ag_region_bytes(rows, cols) + (long long)tdb::aggemm::push_area_bytes(rows, cols, W);
}

// C = epilogue(AG(x) @ B^T) with the all-gather fused (see the header).
//   x: this rank's rows [rows, K] (row stride ldx); full: [W*rows, K] output of
//   the gathered rows; B: [N, K] or [K, N] (b_mn); C: [W*rows, N] bf16.
//   peers / heap_off / region_bytes / state: a fused all-gather region
//   (tdb_ag_gemm_region_bytes; with fewer bytes, tdb_ag_region_bytes, the
//   push variant is refused);
//   ready: uint32 [W*rows/128] zero-initialised counters owned by this call site;
//   tile_table: [tiles] production order (this rank's rows first) for tile code bn.
// mode: 0 store (alpha), 1 bias, 2 bias + GELU (aux_out = pre-activation), 3 GELU backward (aux).
// Row movement of the fused all-gather GEMM for the following calls
// (-1: automatic by world size; 0: the epilogue warps pull before their first
// tile; 1: four auxiliary warps pull concurrently; 2: as 1 with sixteen loads
// in flight per thread; 3: the auxiliary warps push); returns the previous
// value.  Any other value only returns the current one.
TDB_API int tdb_ag_set_variant(int variant) {
  const int old = tdb::aggemm::g_variant;
  if (variant >= tdb::aggemm::kAuto && variant <= 3) tdb::aggemm::g_variant = variant;
  return old;
}

TDB_API int tdb_ag_gemm(const void* x, long long ldx, void* full, long long rows, int K, const void* B, int b_mn,
                        long long ldb, void* C, long long ldc, int N, int mode, const void* bias, const void* aux,
                        long long ld_aux, void* aux_out, float alpha, int bn, const int* tile_table,
                        const unsigned long long* peers, int W, int rank, unsigned long long heap_off,
                        unsigned long long region_bytes, unsigned int* state, unsigned int* ready,
                        double wait_seconds, int taco, void* stream) {
  using namespace tdb;
  using namespace tdb::gemm;
  const long long M = rows * W;
  if (!x || !full || !B || !C || !tile_table || !peers || !state || !ready || W < 2 || W > 64 || rank < 0 ||
      rank >= W || rows % 256 || K % 64 || N % 8 || ldc % 8 || ldx % 8 || ldb % 8 ||
      (mode >= 2 && ld_aux % 8) || ((reinterpret_cast<uintptr_t>(C) | reinterpret_cast<uintptr_t>(full) |
                                     reinterpret_cast<uintptr_t>(x)) % 16))
    return tdb_host::fail(int(cudaErrorInvalidValue), "ag_gemm: bad arguments (rows %% 256, K %% 64, 16-byte rows)");
  if (bn != 128 && bn != 192 && bn != 256 && bn != 512)
    return tdb_host::fail(int(cudaErrorInvalidValue), "ag_gemm: bn must be 128, 192, 256 or 512");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (taco && K % 128)
    return tdb_host::fail(int(cudaErrorInvalidValue), "ag_gemm: the compressed gather needs K %% 128 == 0");
  // the compressed gather stages TACO packets, so it keeps the deep pull
  const int chosen = aggemm::resolve_variant(W);
  const int variant = (chosen == 3 && taco) ? 2 : chosen;
  if (variant == 3 && region_bytes < (unsigned long long)tdb_ag_gemm_region_bytes(rows, K, W))
    return tdb_host::fail(int(cudaErrorInvalidValue),
                          "ag_gemm: the push variant needs a region of tdb_ag_gemm_region_bytes(rows, K, W) bytes");
  int rc = 0;
  if (variant == 3) {  // no send slot: only the epoch advances
    aggemm::push_advance_kernel<<<1, 1, 0, s>>>(state);
    tdb_host::launched(1);
  } else if ((rc = tdb_ag_prepare(x, ldx, rows, K, peers, W, rank, heap_off, state, taco, stream))) {
    return rc;
  }
  CUtensorMap ta, tb;
  if ((rc = make_operand_map(&ta, full, false, int(M), K, K, BM))) return rc;
  if ((rc = make_operand_map(&tb, B, b_mn != 0, N, K, ldb, bn == 512 ? 128 : bn))) return rc;
  EpiParams ep;
  ep.C = C;
  ep.ldc = ldc;
  ep.M = int(M);
  ep.N = N;
  ep.bias = static_cast<const uint16_t*>(bias);
  ep.aux = static_cast<const uint16_t*>(aux);
  ep.ld_aux = ld_aux;
  ep.aux_out = static_cast<uint16_t*>(aux_out);
  ep.alpha = alpha;
  ep.beta = 0.f;
  if ((rc = tdb_host::make_tmap_2d(&ep.tmC, C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(N), uint64_t(M),
                                   uint64_t(ldc), 64, 32, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if (mode == kBiasGelu &&
      (rc = tdb_host::make_tmap_2d(&ep.tmAux, aux_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(N), uint64_t(M),
                                   uint64_t(ld_aux), 64, 32, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  aggemm::Pull pull;
  pull.peers = reinterpret_cast<const uint64_t*>(peers);
  pull.heap_off = heap_off;
  pull.state = state;
  pull.W = W;
  pull.rank = rank;
  pull.rows = rows;
  pull.cols = K;
  pull.full = static_cast<uint16_t*>(full);
  pull.ready = ready;
  pull.slices = aggemm::kSlices;
  pull.push_off = uint64_t(tdb_ag_region_bytes(rows, K));
  pull.wait_ns = uint64_t(wait_seconds * 1e9);
  pull.taco = taco;
  pull.x = static_cast<const uint16_t*>(x);
  pull.ldx = ldx;
  TileOrder order;
  order.group_m = 1;
  order.table = tile_table;
  order.gate_ready = ready;
  order.gate_epoch = state;
  order.gate_per_call = uint32_t(pull.slices);
  return b_mn ? aggemm::dispatch_mode<true>(variant, mode, bn, ta, tb, int(M), N, K, order, ep, pull, s)
              : aggemm::dispatch_mode<false>(variant, mode, bn, ta, tb, int(M), N, K, order, ep, pull, s);
}
