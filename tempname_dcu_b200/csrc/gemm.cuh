// Persistent warp-specialised tcgen05 GEMM mainloop for sm_100a.
//
//   D[M,N] = sum_k A[m,k] * B[n,k]        (fp32 accumulation in TMEM)
//
// A is "K-major" ([M,K] rows, K contiguous) or "MN-major" ([K,M] rows, M
// contiguous); likewise B ([N,K] or [K,N]).  Those three storage cases cover
// every linear layer of training: forward X*W^T (K,K), data gradient dY*W
// (K,MN) and weight gradient dY^T*X (MN,MN) without any transpose kernel.
//
// Roles (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer (one elected lane) + TMEM allocator
//   warp 1      MMA issuer: one thread issues tcgen05.mma.cta_group::1.kind::f16
//   warps 2..5  epilogue: tcgen05.ld 32x32b from TMEM -> registers -> Epi
// Pipelines:
//   smem ring of STAGES (A,B) tiles, full[] (TMA tx) / empty[] (tcgen05.commit)
//   two TMEM accumulators (2*BN columns), tmem_full[] / tmem_empty[] (one
//   for 256-wide block-scaled FP8 tiles, whose scale columns need the room)
// Optional: block-scaled FP8 tiles (MX = true, MxOperands) and auxiliary
// warps after the epilogue warps (Epi::kAuxWarps, see AuxWarps).
// Every mbarrier wait is bounded (common.cuh); on expiry the CTA abandons its
// loops, drains in-flight copies / MMAs with bounded waits, frees TMEM and
// returns with the status word set.  There is no TMA multicast.
#pragma once
#include <type_traits>

#include "common.cuh"

namespace tdb {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one 128B swizzle row
constexpr int kThreads = 192;

template <int BN, int STAGES = (BN == 128 ? 6 : 4), bool MX = false>
struct Config {
  static constexpr int kStages = STAGES;
  static constexpr int kABytes = BM * BK * 2;  // also 128 rows x 128 e4m3 (one block-scaled K step)
  static constexpr int kBBytes = BN * BK * 2;
  // block-scaled FP8 stages also carry the scale atoms of A (512 B) and B (BN*4 B)
  static constexpr int kSfBytes = MX ? (512 + BN * 4 + 1023) / 1024 * 1024 : 0;
  static constexpr int kStageBytes = kABytes + kBBytes + kSfBytes;
  // TMEM: accumulators of BN columns (two, so the epilogue of a tile overlaps
  // the next tile's MMAs; one for 256-wide FP8 tiles, whose scale ring would
  // not fit beside two), then (FP8) a ring of scale columns per stage
  static constexpr int kSfCols = 4 + BN / 32;
  static constexpr int kAccums = (MX && BN > 128) ? 1 : 2;
  static constexpr int kTmemCols = (MX || 2 * BN > 256) ? 512 : 256;
  static_assert(!MX || (BN % 128 == 0 && kAccums * BN + STAGES * kSfCols <= 512), "FP8 scale ring does not fit TMEM");
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// Block-scaled FP8 operands (kind::mxf8f6f4).  A is e4m3 [rows, K] and B is
// e4m3 [N, K], both K-major with TMA boxes of {128 bytes, 128 | BN rows}.
// Scales are ue8m0 (2^(byte-127)), one per 32 consecutive K values, stored
// as 512-byte atoms: the atom of 128-row block `blk` and 128-wide K chunk
// `kc` sits at (kc * blocks + blk) * 512, and inside it row r's scale for the
// 32-value block j at (r % 32) * 16 + (r / 32) * 4 + j -- the byte order in
// which one tcgen05.cp 32x128b.warpx4 lays them out in TMEM (lane r % 32,
// column r / 32, byte j).
struct MxOperands {
  const CUtensorMap* tmA;
  const CUtensorMap* tmB;
  const uint8_t* sfa;
  const uint8_t* sfb;
  int a_blocks, b_blocks;
  const uint8_t* mask;  // per 128-row m block: nonzero = block-scaled FP8 tile; null = every tile
  __device__ __forceinline__ bool on(int m_blk) const { return mask == nullptr || mask[m_blk] != 0; }
};

// TMA map of an e4m3 operand [rows, K] (K-major, 128-byte swizzle), box
// {128 bytes, box_rows} (csrc/gemm_mx.cu).
int make_fp8_map(CUtensorMap* map, const void* ptr, int rows, int K, int box_rows);

// Output-tile order.  Grouped raster (GROUP_M m-blocks per band) for L2 reuse,
// or an explicit device table of tile ids (used by the fused collective
// kernels to impose the common tile-to-rank production order).
struct TileOrder {
  int num_m, num_n;
  int group_m;
  const int* table;  // optional: table[i] = m_blk * num_n + n_blk
  int num_tiles;
  // Optional gate on the A rows (the all-gather fused into the GEMM): before
  // loading the A rows of a tile, the producer waits until the counter of
  // their 128-row block reaches (*gate_epoch) * gate_per_call.
  const uint32_t* gate_ready = nullptr;
  const uint32_t* gate_epoch = nullptr;
  uint32_t gate_per_call = 0;

  __host__ __device__ __forceinline__ void tile(int i, int& m_blk, int& n_blk) const {
    if (table) {
      const int t = table[i];
      m_blk = t / num_n;
      n_blk = t % num_n;
      return;
    }
    const int width = group_m * num_n;
    const int group = i / width;
    const int first = group * group_m;
    const int gsize = min(num_m - first, group_m);
    const int r = i % width;
    m_blk = first + r % gsize;
    n_blk = r / gsize;
  }
};

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Wait (bounded) until the A rows of 128-row block `blk` are in place, then
// order those generic-proxy writes before this thread's TMA (async-proxy)
// reads.  Returns false on timeout (status recorded).
__device__ __forceinline__ bool gate_wait(const TileOrder& order, int blk, int* status) {
  const uint32_t target = __ldg(order.gate_epoch) * order.gate_per_call;
  const uint32_t* ctr = order.gate_ready + blk;
  if (int32_t(ld_acquire_gpu_u32(ctr) - target) < 0) {
    const uint64_t t0 = globaltimer();
    while (int32_t(ld_acquire_gpu_u32(ctr) - target) < 0) {
      if (globaltimer() - t0 > kWaitLimitNs) {
        record_status(status, kTimeoutLocal, 40, blk, int(target));
        return false;
      }
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// Auxiliary warps: an Epi may declare `static constexpr int kAuxWarps = n`
// and a method `aux(int* status)`; the kernel then runs with n extra warps
// (after the epilogue warps 2..5) that execute aux() concurrently with the
// pipeline -- e.g. the fused all-gather's pull, so that it no longer delays
// the epilogue of the first tiles.  Launches must add 32 * n threads.
template <class E, class = void>
struct AuxWarps {
  static constexpr int value = 0;
};
template <class E>
struct AuxWarps<E, std::void_t<decltype(E::kAuxWarps)>> {
  static constexpr int value = E::kAuxWarps;
};

struct alignas(8) Barriers {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
// The barriers sit in a 256-byte slot before the epilogue's shared memory;
// its last 16 bytes are scratch of the epilogue warps (set_smem pointer - 16).
static_assert(sizeof(Barriers) <= 240, "barrier slot overlaps the epilogue scratch");

// Descriptor of a K-major SW128 tile: rows of 128 bytes, 8-row atoms of
// 1024 bytes.  LBO is unused for swizzled K-major operands (encoded as 16).
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr) { return smem_desc_sw128(saddr, 16, 1024); }

// Descriptor of an MN-major SW128 tile stored as boxes of [64 K rows][64 MN
// elements]: 8-row K groups are 1024 bytes apart (SBO), 64-element MN chunks
// are one box (64*128 bytes) apart (LBO).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t saddr) {
  return smem_desc_sw128(saddr, BK * 128, 1024);
}

// Epi may own shared memory (Epi::kSmemBytes, placed after the barriers);
// the epilogue warps receive it through epi.set_smem().
// MX = true adds block-scaled FP8 tiles (those whose m block mx->on()): they
// stream 128-wide K steps of e4m3 plus scale atoms through the same stage
// ring and issue kind::mxf8f6f4 MMAs; the other tiles run the bf16 path.
template <int BN, bool A_MN, bool B_MN, class Epi, int STAGES = Config<BN>::kStages, bool MX = false>
__device__ __forceinline__ void gemm_mainloop(const CUtensorMap* tmA, const CUtensorMap* tmB, int K,
                                              const TileOrder& order, Epi& epi, int* status,
                                              const MxOperands* mx = nullptr) {
  using Cfg = Config<BN, STAGES, MX>;
  static_assert(!MX || (!A_MN && !B_MN), "block-scaled FP8 operands are K-major");
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + S * Cfg::kStageBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = (K + BK - 1) / BK;
#ifdef TDB_DEBUG
  // Every thread checks this CTA's tiles before anything is allocated, so a
  // bad tile table makes the whole CTA return uniformly (status recorded).
  for (int i = blockIdx.x; i < order.num_tiles; i += gridDim.x) {
    int mb, nb;
    order.tile(i, mb, nb);
    if (!TDB_DEBUG_OK(status, mb >= 0 && mb < order.num_m && nb >= 0 && nb < order.num_n, 50, mb, nb)) return;
  }
#endif

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->tmem_full[b], 1);
      mbar_init(&bars->tmem_empty[b], 4);
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(tmA);
    prefetch_tmap(tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int i = blockIdx.x; i < order.num_tiles && ok; i += gridDim.x) {
        int mb, nb;
        order.tile(i, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        if (order.gate_ready && !gate_wait(order, m0 / 128, status)) { ok = false; *abort_flag = 1; break; }
        bool fp8 = false;
        if constexpr (MX) fp8 = mx->on(mb);
        const int tile_kb = fp8 ? K / 128 : num_kb;
        for (int kb = 0; kb < tile_kb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t round = it / S;
          if (!mbar_wait(&bars->empty[s], (round & 1) ^ 1, status, 10)) { ok = false; *abort_flag = 1; break; }
          if (*abort_flag) { ok = false; break; }
          uint8_t* sa = smem + s * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          if constexpr (MX) {
            if (fp8) {
              uint8_t* sf = sb + Cfg::kBBytes;
              mbar_arrive_expect_tx(&bars->full[s], Cfg::kABytes + Cfg::kBBytes + 512 + BN * 4);
              tma_load_2d(sa, mx->tmA, &bars->full[s], kb * 128, m0);
              tma_load_2d(sb, mx->tmB, &bars->full[s], kb * 128, n0);
              bulk_g2s(sf, mx->sfa + (size_t(kb) * mx->a_blocks + mb) * 512, 512, &bars->full[s]);
              bulk_g2s(sf + 512, mx->sfb + (size_t(kb) * mx->b_blocks + n0 / 128) * 512, BN * 4, &bars->full[s]);
              continue;
            }
          }
          mbar_arrive_expect_tx(&bars->full[s], Cfg::kABytes + Cfg::kBBytes);
          const int k0 = kb * BK;
          if (!A_MN) {
            tma_load_2d(sa, tmA, &bars->full[s], k0, m0);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(sa + j * (BK * 128), tmA, &bars->full[s], m0 + 64 * j, k0);
          }
          if (!B_MN) {
            tma_load_2d(sb, tmB, &bars->full[s], k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * (BK * 128), tmB, &bars->full[s], n0 + 64 * j, k0);
          }
        }
      }
      if (!ok) {
        // Drain: wait (bounded) for every stage that may still have bytes in flight.
        for (uint32_t j = (it >= S ? it - S : 0); j < it; ++j)
          mbar_wait(&bars->full[j % S], (j / S) & 1, status, 11);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN, A_MN, B_MN);
      uint32_t it = 0;
      int tc = 0;
      bool ok = true;
      bool issued = false;
      for (int i = blockIdx.x; i < order.num_tiles && ok; i += gridDim.x, ++tc) {
        const int b = Cfg::kAccums == 2 ? (tc & 1) : 0;
        const uint32_t use = Cfg::kAccums == 2 ? uint32_t(tc >> 1) : uint32_t(tc);
        if (!mbar_wait(&bars->tmem_empty[b], (use & 1) ^ 1, status, 20)) { ok = false; *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t dcol = tmem_base + b * BN;
        bool fp8 = false;
        if constexpr (MX) {
          int mb, nb;
          order.tile(i, mb, nb);
          fp8 = mx->on(mb);
        }
        const int tile_kb = fp8 ? K / 128 : num_kb;
        for (int kb = 0; kb < tile_kb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t round = it / S;
          if (!mbar_wait(&bars->full[s], round & 1, status, 21)) { ok = false; *abort_flag = 1; break; }
          if (*abort_flag) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * Cfg::kStageBytes);
          const uint32_t sb = sa + Cfg::kABytes;
          if constexpr (MX) {
            if (fp8) {
              // scales: smem atoms -> TMEM columns of this stage, then four K = 32 MMAs
              const uint32_t sf = sb + Cfg::kBBytes;
              const uint32_t sfa_col = tmem_base + Cfg::kAccums * BN + s * Cfg::kSfCols;
              const uint32_t sfb_col = sfa_col + 4;
              tmem_cp_32x128b_x4(sfa_col, smem_desc_plain(sf, 0, 128));
#pragma unroll
              for (int j = 0; j < BN / 128; ++j) tmem_cp_32x128b_x4(sfb_col + 4 * j, smem_desc_plain(sf + 512 + 512 * j, 0, 128));
              constexpr uint32_t idesc8 = idesc_mxf8(BM, BN);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_mxf8_ss(dcol, desc_kmajor(sa + k * 32), desc_kmajor(sb + k * 32), idesc8, sfa_col, sfb_col,
                             uint32_t(k), (kb | k) != 0 ? 1u : 0u);
              issued = true;
              umma_commit(&bars->empty[s]);
              continue;
            }
          }
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? desc_mnmajor(sa + k * 16 * 128) : desc_kmajor(sa + k * 32);
            const uint64_t bd = B_MN ? desc_mnmajor(sb + k * 16 * 128) : desc_kmajor(sb + k * 32);
            umma_f16_ss(dcol, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued = true;
          umma_commit(&bars->empty[s]);
        }
        if (ok) umma_commit(&bars->tmem_full[b]);
      }
      // Make sure every MMA has landed before TMEM can be released.
      if (issued) {
        umma_commit(&bars->drain);
        mbar_wait(&bars->drain, 0, status, 22);
      }
    }
  } else if (AuxWarps<Epi>::value > 0 && warp >= 6) {
    // ---------------- Auxiliary warps (6..) ----------------
    if constexpr (AuxWarps<Epi>::value > 0) {
      epi.set_smem(reinterpret_cast<uint8_t*>(bars) + 256);
      epi.aux(status);
    }
  } else {
    // ---------------- Epilogue (warps 2..5) ----------------
    epi.set_smem(reinterpret_cast<uint8_t*>(bars) + 256);
    epi.prologue(status);  // work before the first tile (e.g. the fused all-gather pull)
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32)
    const int row_in_tile = quarter * 32 + lane;
    int tc = 0;
    for (int i = blockIdx.x; i < order.num_tiles; i += gridDim.x, ++tc) {
      int mb, nb;
      order.tile(i, mb, nb);
      const int b = Cfg::kAccums == 2 ? (tc & 1) : 0;
      const uint32_t use = Cfg::kAccums == 2 ? uint32_t(tc >> 1) : uint32_t(tc);
      bool ok = mbar_wait(&bars->tmem_full[b], use & 1, status, 30);
      if (*abort_flag) ok = false;
      if (!ok) { *abort_flag = 1; break; }
      tc_fence_after();
      epi.tile_begin(mb, nb);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (uint32_t(quarter * 32) << 16) + b * BN + c * 32, r);
        tmem_wait_ld();
        if (c == BN / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->tmem_empty[b]);
        }
        epi.chunk(mb * BM + row_in_tile, nb * BN + c * 32, c, r);
      }
      epi.tile_end(mb, nb, quarter, lane);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace gemm
}  // namespace tdb
