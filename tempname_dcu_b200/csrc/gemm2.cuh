// 2-CTA (cta_group::2) persistent tcgen05 GEMM mainloop: 256 x 256 output
// tiles computed by an SM pair (a cluster of two CTAs).
//
// CTA r of the pair holds rows [128r, 128r+128) of the A tile and rows
// [128r, 128r+128) of the B tile (i.e. half of the N columns).  One thread of
// the even CTA issues tcgen05.mma.cta_group::2 with M = 256, N = 256, K = 16;
// the hardware reads A and B from both CTAs' shared memory at the same
// offsets and writes each CTA's 128 output rows x 256 columns into that CTA's
// TMEM.  Compared with the 1-CTA 128 x 256 tile, each SM stages half of B, so
// the shared-memory traffic per MMA drops from 12 KB to 8 KB.
//
// Synchronisation (both CTAs run a TMA producer and four epilogue warps):
//   full[s]       even CTA; its producer posts expect_tx(64 KB); both CTAs'
//                 TMA loads (.cta_group::2, plain -- no multicast) complete
//                 bytes on it
//   empty[s]      each CTA; the MMA thread's tcgen05.commit is multicast to
//                 both CTAs
//   tmem_full[b]  each CTA; multicast commit after a tile's last MMA
//   tmem_empty[b] even CTA, 8 arrivals (4 epilogue warps x 2 CTAs, remote)
// All waits are bounded; teardown uses a bounded remote-flag handshake.
#pragma once
#include "gemm.cuh"

namespace tdb {
namespace gemm2 {

using gemm::BK;
constexpr int kThreads = 192;
constexpr int kHalf = 128;              // rows of A and of B per CTA
constexpr int kTileN = 256;             // output columns per tile (both CTAs)
constexpr int kABytes = kHalf * BK * 2;
constexpr int kBBytes = kHalf * BK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kTmemCols = 2 * kTileN;

template <int STAGES>
struct Config {
  static constexpr int kStages = STAGES;
  static constexpr int kSmemBytes = STAGES * kStageBytes + 1024 + 256;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cta address -> the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t mbar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(mbar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void umma2_f16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Commit arriving on the same barrier offset in both CTAs of the pair.
__device__ __forceinline__ void umma2_commit_both(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

__device__ __forceinline__ void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.release.cluster.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_cta_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.cluster.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}

struct alignas(8) Barriers {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  uint32_t peer_done;
};
// The barriers sit in a 256-byte slot before the epilogue's shared memory;
// its last 16 bytes are scratch of the epilogue warps (set_smem pointer - 16).
static_assert(sizeof(Barriers) <= 240, "barrier slot overlaps the epilogue scratch");

// `order` counts 256 x 256 tiles.  Epi receives 128-row block indices
// (tile_m * 2 + rank) and 256-column tile indices, like the 1-CTA mainloop
// with BN = 256.
template <bool A_MN, bool B_MN, class Epi, int STAGES>
__device__ __forceinline__ void mainloop(const CUtensorMap* tmA, const CUtensorMap* tmB, int K,
                                         const gemm::TileOrder& order, Epi& epi, int* status) {
  constexpr int S = STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + S * kStageBytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->tmem_full[b], 1);
      mbar_init(&bars->tmem_empty[b], 8);
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    bars->peer_done = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc2(&bars->tmem_base, kTmemCols);
    tmem_relinquish2();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(tmA);
    prefetch_tmap(tmB);
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised; TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int i = cluster; i < order.num_tiles && ok; i += nclusters) {
        int mt, nt;
        order.tile(i, mt, nt);
        const int m0 = mt * 256 + rank * kHalf, n0 = nt * kTileN + rank * kHalf;
        if (order.gate_ready && !gemm::gate_wait(order, m0 / 128, status)) { ok = false; *abort_flag = 1; break; }
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t round = it / S;
          if (!mbar_wait(&bars->empty[s], (round & 1) ^ 1, status, 110)) { ok = false; *abort_flag = 1; break; }
          if (*abort_flag) { ok = false; break; }
          uint8_t* sa = smem + s * kStageBytes;
          uint8_t* sb = sa + kABytes;
          if (rank == 0) mbar_arrive_expect_tx(&bars->full[s], 2 * kStageBytes);
          const uint32_t fb = mapa(smem_u32(&bars->full[s]), 0);
          const int k0 = kb * BK;
          if (!A_MN) {
            tma_load_2d_pair(sa, tmA, fb, k0, m0);
          } else {
            tma_load_2d_pair(sa, tmA, fb, m0, k0);
            tma_load_2d_pair(sa + BK * 128, tmA, fb, m0 + 64, k0);
          }
          if (!B_MN) {
            tma_load_2d_pair(sb, tmB, fb, k0, n0);
          } else {
            tma_load_2d_pair(sb, tmB, fb, n0, k0);
            tma_load_2d_pair(sb + BK * 128, tmB, fb, n0 + 64, k0);
          }
        }
      }
      if (!ok && rank == 0) {
        for (uint32_t j = (it >= S ? it - S : 0); j < it; ++j)
          mbar_wait(&bars->full[j % S], (j / S) & 1, status, 111);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_bf16(256, kTileN, A_MN, B_MN);
      uint32_t it = 0;
      int tc = 0;
      bool ok = true, issued = false;
      for (int i = cluster; i < order.num_tiles && ok; i += nclusters, ++tc) {
        const int b = tc & 1;
        const uint32_t use = tc >> 1;
        if (!mbar_wait(&bars->tmem_empty[b], (use & 1) ^ 1, status, 120)) { ok = false; *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t dcol = tmem_base + b * kTileN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t round = it / S;
          if (!mbar_wait(&bars->full[s], round & 1, status, 121)) { ok = false; *abort_flag = 1; break; }
          if (*abort_flag) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * kStageBytes);
          const uint32_t sb = sa + kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? gemm::desc_mnmajor(sa + k * 16 * 128) : gemm::desc_kmajor(sa + k * 32);
            const uint64_t bd = B_MN ? gemm::desc_mnmajor(sb + k * 16 * 128) : gemm::desc_kmajor(sb + k * 32);
            umma2_f16_ss(dcol, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued = true;
          umma2_commit_both(&bars->empty[s]);
        }
        if (ok) umma2_commit_both(&bars->tmem_full[b]);
      }
      if (issued) {
        umma2_commit_both(&bars->drain);
        mbar_wait(&bars->drain, 0, status, 122);
      }
    }
  } else if (gemm::AuxWarps<Epi>::value > 0 && warp >= 6) {
    // auxiliary warps (see gemm::AuxWarps)
    if constexpr (gemm::AuxWarps<Epi>::value > 0) {
      epi.set_smem(reinterpret_cast<uint8_t*>(bars) + 256);
      epi.aux(status);
    }
  } else {
    epi.set_smem(reinterpret_cast<uint8_t*>(bars) + 256);
    epi.prologue(status);
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int tc = 0;
    for (int i = cluster; i < order.num_tiles; i += nclusters, ++tc) {
      int mt, nt;
      order.tile(i, mt, nt);
      const int mb = mt * 2 + int(rank);
      const int b = tc & 1;
      const uint32_t use = tc >> 1;
      bool ok = mbar_wait(&bars->tmem_full[b], use & 1, status, 130);
      if (*abort_flag) ok = false;
      if (!ok) { *abort_flag = 1; break; }
      tc_fence_after();
      epi.tile_begin(mb, nt);
#pragma unroll 1
      for (int c = 0; c < kTileN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (uint32_t(quarter * 32) << 16) + b * kTileN + c * 32, r);
        tmem_wait_ld();
        if (c == kTileN / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa(smem_u32(&bars->tmem_empty[b]), 0));
        }
        epi.chunk(mb * gemm::BM + row_in_tile, nt * kTileN + c * 32, c, r);
      }
      epi.tile_end(mb, nt, quarter, lane);
    }
  }

  // Teardown: both CTAs finished their roles; a bounded handshake instead of
  // an unbounded cluster barrier, then the paired TMEM free.
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    st_cluster_u32(mapa(smem_u32(&bars->peer_done), rank ^ 1u), 1u);
    const uint64_t t0 = globaltimer();
    while (ld_acquire_cta_u32(&bars->peer_done) == 0u) {
      if (globaltimer() - t0 > kWaitLimitNs) {
        record_status(status, kTimeoutLocal, 140);
        break;
      }
    }
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc2(tmem_base, kTmemCols);
}

}  // namespace gemm2
}  // namespace tdb
