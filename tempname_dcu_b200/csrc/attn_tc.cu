// Causal flash attention forward on the 5th-generation tensor cores
// (tcgen05.mma + TMEM accumulators + TMA), head_dim 128, bf16 in / fp32 acc.
//
// Reference parity: python/flux_dcu/model.py:250-256 (causal SDPA over the
// local heads, no dropout).  Same I/O contract as the mma.sync kernel in
// attention.cu: qkv [tokens, 3, Hl, 128] (row stride ld), out [tokens, Hl,
// 128] (row stride ld_out), lse [mb, Hl, seq] = m + log2(l) of the scores
// scaled by scale*log2(e).
//
// One CTA = 128 queries of one (batch, head); key/value tiles of 128.
//   warp 0      TMA producer: Q once, then K/V tiles through a 5-slot ring in
//               exactly the order the MMA warp consumes them
//               (K0, K1, V0, K2, V1, K3, ...); allocates 512 TMEM columns
//   warp 1      MMA issuer (one thread):  S_j = Q K_j^T into TMEM S[j%2]
//               (double-buffered, so S_{j+1} overlaps softmax j), then
//               O += P_j V_j into the TMEM O accumulator, with P_j read
//               straight from TMEM (written over S_j by the softmax warps), so
//               shared memory only carries Q, K and V
//   warps 2..9  softmax: two warps per TMEM lane quarter, each thread one
//               query row and 64 of its 128 columns, so row max and row sum
//               need no shuffles (the two halves meet once per step through
//               shared memory).  P_j (bf16) is stored back into TMEM.
//               The running max is only raised when it grows by more than
//               2^8 (exact: P <= 256 stays representable, O and l use the
//               same stale max), so the O correction (tcgen05.ld/st of the
//               accumulator) is rare.
// TMEM columns: S0 [0,128), S1 [128,256), O [256,384).
// All waits are bounded (common.cuh); there is no TMA multicast.
#include "common.cuh"
#include "tensor_map.h"

namespace tdb {
namespace attn_tc {

constexpr int BM = 128, BN = 128, D = 128;
constexpr int kBox = 128 * 128;  // one [128 rows][64 bf16] SW128 box = 16 KB
constexpr int kTile = 2 * kBox;  // a 128 x 128 bf16 tile = two boxes
constexpr int kSlots = 5;
constexpr int kTmemCols = 512;
constexpr int kOCol = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.0f;  // raise the running max only past 2^8 growth

struct alignas(8) Bars {
  uint64_t q_full;
  uint64_t kv_full[kSlots];
  uint64_t kv_empty[kSlots];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t pv_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int vote[2][2][4];    // per (parity, half, quarter): this warp can go on
  float red[2][2][BM];  // per (parity, half, row): partial row max (row sum at the end)
};

constexpr int kThreads = 320;  // TMA warp, MMA warp, 8 softmax / score warps
constexpr int kSmem = kTile + kSlots * kTile + 1024 + int(sizeof(Bars));
static_assert(kSmem <= 232448, "shared memory budget");

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Generic-proxy shared-memory writes -> visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// K-major SW128 operand spanning two 64-column boxes: K step k (16 elements).
__device__ __forceinline__ uint64_t desc_k(uint32_t base, int k) {
  return smem_desc_sw128(base + (k >> 2) * kBox + (k & 3) * 32, 16, 1024);
}
// MN-major SW128 operand (V: [128 keys][128 d], d contiguous, two 64-column
// boxes 16 KB apart): K step k = 16 key rows.
__device__ __forceinline__ uint64_t desc_mn(uint32_t base, int k) {
  return smem_desc_sw128(base + k * 16 * 128, kBox, 1024);
}

__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Row maximum over this thread's 64 columns; 8 independent chains.  MASK:
// columns c > lim are causally excluded.
template <bool MASK>
__device__ __forceinline__ float row_max64(const uint32_t (&sr)[2][32], int lim) {
  float mx[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
#pragma unroll
  for (int c = 0; c < 64; ++c) {
    const float v = __uint_as_float(sr[c >> 5][c & 31]);
    if (!MASK || c <= lim) mx[c & 7] = fmaxf(mx[c & 7], v);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) mx[i] = fmaxf(mx[i], mx[i + 4]);
  return fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
}

// P = exp2(s*sl2 - m) for this thread's 64 columns as 32 packed bf16 pairs;
// returns the partial row sum (8 accumulators).
template <bool MASK>
__device__ __forceinline__ float exp_row64(const uint32_t (&sr)[2][32], int lim, float sl2, float m,
                                           uint32_t (&pk)[32]) {
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  const float neg = -m;
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const int c0 = 2 * e;
    float p0 = ex2(fmaf(__uint_as_float(sr[c0 >> 5][c0 & 31]), sl2, neg));
    float p1 = ex2(fmaf(__uint_as_float(sr[(c0 + 1) >> 5][(c0 + 1) & 31]), sl2, neg));
    if (MASK) {
      p0 = c0 <= lim ? p0 : 0.f;
      p1 = c0 + 1 <= lim ? p1 : 0.f;
    }
    acc[(2 * e) & 7] += p0;
    acc[(2 * e + 1) & 7] += p1;
    pk[e] = pack_bf16x2(p0, p1);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] += acc[i + 4];
  return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16: A (M=128 rows = TMEM lanes,
// bf16 pairs packed along columns, 8 columns per K=16 step) read straight
// from tensor memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__global__ void __launch_bounds__(kThreads, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tm, uint16_t* __restrict__ out, int64_t ld_out,
               float* __restrict__ lse, int seq, int Hl, int mb, float scale, int* status,
               unsigned long long* __restrict__ tl) {
  // Optional diagnostic timeline (clock64 per pipeline event of the first
  // CTA, tl[16 * step + event]); null in normal use.
  const bool tl_on = tl != nullptr && blockIdx.x == 0 && blockIdx.y == 0;
#define TDB_TL(step, ev) \
  do {                     \
    if (tl_on) tl[16 * (step) + (ev)] = clock64(); \
  } while (0)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + kTile;
  Bars* bars = reinterpret_cast<Bars*>(sKV + kSlots * kTile);

  const int hb = blockIdx.x;  // (head, batch) fastest: all heads of the heaviest query tile launch first
  const int h = hb % Hl, b = hb / Hl;
  const int nq = seq / BM;
  const int qb = nq - 1 - int(blockIdx.y);
  const int n = qb + 1;  // causal: key tiles 0..qb
  const int row0 = b * seq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 8);
    }
    mbar_init(&bars->pv_done, 1);
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
    if (lane == 0) prefetch_tmap(&tm);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      mbar_arrive_expect_tx(&bars->q_full, kTile);
      tma_load_2d(sQ, &tm, &bars->q_full, h * D, row0 + qb * BM);
      tma_load_2d(sQ + kBox, &tm, &bars->q_full, h * D + 64, row0 + qb * BM);
      const int total = 2 * n;
      int i = 0;
      bool ok = true;
      for (; i < total && ok; ++i) {
        // item i of the consumption order K0, K1, V0, K2, V1, K3, ..., V_{n-1}
        bool is_v;
        int j;
        if (n == 1) {
          is_v = i == 1;
          j = 0;
        } else if (i < 2) {
          is_v = false;
          j = i;
        } else {
          const int t = i - 2;  // V_{t/2} (even t) then K_{t/2+2} (odd t) while K tiles remain
          const int k_left = n - 2;
          if (t < 2 * k_left) {
            is_v = (t & 1) == 0;
            j = is_v ? t >> 1 : (t >> 1) + 2;
          } else {
            is_v = true;
            j = t - k_left;
          }
        }
        const int s = i % kSlots;
        const uint32_t round = i / kSlots;
        if (!mbar_wait(&bars->kv_empty[s], (round & 1) ^ 1, status, 60)) { ok = false; *abort_flag = 1; break; }
        if (*abort_flag) { ok = false; break; }
        uint8_t* dst = sKV + s * kTile;
        const int col = (is_v ? 2 * Hl + h : Hl + h) * D;
        TDB_TL(j, is_v ? 1 : 0);
        mbar_arrive_expect_tx(&bars->kv_full[s], kTile);
        tma_load_2d(dst, &tm, &bars->kv_full[s], col, row0 + j * BN);
        tma_load_2d(dst + kBox, &tm, &bars->kv_full[s], col + 64, row0 + j * BN);
      }
      // Never leave a copy in flight: wait (bounded) for Q and the last loads.
      mbar_wait(&bars->q_full, 0, status, 61);
      if (!ok)
        for (int k = (i >= kSlots ? i - kSlots : 0); k < i; ++k)
          mbar_wait(&bars->kv_full[k % kSlots], (k / kSlots) & 1, status, 62);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idS = idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idO = idesc_bf16(BM, D, false, true);
      bool ok = mbar_wait(&bars->q_full, 0, status, 70);
      bool issued = false;
      uint32_t it = 0;
      const uint32_t sq = smem_u32(sQ);
      auto next_slot = [&](uint32_t& addr) -> bool {
        const int s = it % kSlots;
        if (!mbar_wait(&bars->kv_full[s], (it / kSlots) & 1, status, 71)) return false;
        if (*abort_flag) return false;
        tc_fence_after();
        addr = smem_u32(sKV + s * kTile);
        return true;
      };
      auto issue_s = [&](int j) -> bool {
        uint32_t sk;
        if (!next_slot(sk)) return false;
        TDB_TL(j, 2);
        const uint32_t d = tmem + (j & 1) * BN;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_f16_ss(d, desc_k(sq, k), desc_k(sk, k), idS, k > 0 ? 1u : 0u);
        umma_commit(&bars->kv_empty[it % kSlots]);
        umma_commit(&bars->s_full[j & 1]);
        ++it;
        issued = true;
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        if (!mbar_wait(&bars->p_full[j & 1], (j >> 1) & 1, status, 72)) return false;
        TDB_TL(j, 3);
        tc_fence_after();
        uint32_t sv;
        if (!next_slot(sv)) return false;
        TDB_TL(j, 4);
        // P_j (bf16 pairs) sits in the first 64 columns of TMEM buffer S[j%2].
        const uint32_t tp = tmem + (j & 1) * BN;
#pragma unroll
        for (int k = 0; k < BN / 16; ++k)
          umma_f16_ts(tmem + kOCol, tp + 8 * k, desc_mn(sv, k), idO, (j | k) != 0 ? 1u : 0u);
        umma_commit(&bars->kv_empty[it % kSlots]);
        umma_commit(&bars->pv_done);
        ++it;
        issued = true;
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && n > 1) ok = issue_s(1);
      for (int j = 0; j < n && ok; ++j) {
        ok = issue_pv(j);
        if (ok && j + 2 < n) ok = issue_s(j + 2);
      }
      if (!ok) *abort_flag = 1;
      if (issued) {
        umma_commit(&bars->drain);
        mbar_wait(&bars->drain, 0, status, 73);
      }
    }
  } else {
    // ---------------- softmax / correction / epilogue (warps 2..9) ----------------
    // Two warps per TMEM lane quarter: `half` owns key columns [64*half, +64)
    // of S and d columns [64*half, +64) of O.  The row max is combined
    // through shared memory (64-thread named barrier per quarter); each half
    // keeps its own partial row sum until the epilogue.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // query row within the tile (= TMEM lane)
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const uint32_t bar_id = 1 + quarter;
    const float sl2 = scale * kLog2e;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // Every iteration runs one exchange barrier in both warps of the pair,
    // whatever happens, so a bounded wait that expires in one of them can
    // never leave the other stuck on the named barrier.
    for (int j = 0; j < n; ++j) {
      if (ok && !mbar_wait(&bars->s_full[j & 1], (j >> 1) & 1, status, 80)) ok = false;
      const bool stamp = warp == 2 && lane == 0;
      if (stamp) TDB_TL(j, 5);
      if (*abort_flag) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      uint32_t sr[2][32];
      const bool diag = j == n - 1;
      const int lim = r - 64 * half;  // diagonal tile: column c of this half is visible iff c <= lim
      float mx = -INFINITY;
      if (ok) {
        tc_fence_after();
        const uint32_t sbase = tmem + lane_off + (j & 1) * BN + 64 * half;
        tmem_ld_32x32b_x32(sbase, sr[0]);
        tmem_ld_32x32b_x32(sbase + 32, sr[1]);
        tmem_wait_ld();
        if (stamp) TDB_TL(j, 6);
        mx = diag ? row_max64<true>(sr, lim) : row_max64<false>(sr, lim);
      }
      bars->red[j & 1][half][r] = mx;
      if (lane == 0) bars->vote[j & 1][half][quarter] = ok ? 1 : 0;
      named_barrier(bar_id, 64);
      if (stamp) TDB_TL(j, 7);
      ok = ok && bars->vote[j & 1][half ^ 1][quarter] != 0;
      if (!ok) continue;
      mx = fmaxf(mx, bars->red[j & 1][half ^ 1][r]);
      const float cand = fmaxf(m, mx * sl2);
      float alpha = 1.f;
      bool rescale = false;
      if (j == 0) {
        m = cand;
      } else if (cand > m + kRescale) {
        alpha = ex2(m - cand);
        m = cand;
        rescale = true;
      }
      // P overwrites S in place (columns [32*half, +32) of the buffer hold the
      // bf16 pairs of keys [64*half, +64)); both halves have read their S
      // values before the exchange barrier above.
      uint32_t pk[32];
      const float sum = diag ? exp_row64<true>(sr, lim, sl2, m, pk) : exp_row64<false>(sr, lim, sl2, m, pk);
      tmem_st_32x32b_x32(tmem + lane_off + (j & 1) * BN + 32 * half, pk);
      l = l * alpha + sum;
      tmem_wait_st();
      if (stamp) TDB_TL(j, 8);
      if (j > 0) {
        // O correction needs PV_{j-1} landed; it was issued a full softmax step ago.
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->pv_done, (j - 1) & 1, status, 81));
        if (stamp) TDB_TL(j, 9);
        if (!ok) continue;
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            const uint32_t oaddr = tmem + lane_off + kOCol + 64 * half + c * 32;
            tmem_ld_32x32b_x32(oaddr, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st_32x32b_x32(oaddr, o);
          }
          tmem_wait_st();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[j & 1]);
      if (stamp) TDB_TL(j, 10);
    }
    if (!ok) *abort_flag = 1;
    // combine the two partial row sums (one more barrier in both warps)
    // (parity n & 1: its last readers finished before the barrier of step n-1)
    bars->red[n & 1][half][r] = l;
    if (lane == 0) bars->vote[n & 1][half][quarter] = ok ? 1 : 0;
    named_barrier(bar_id, 64);
    ok = ok && bars->vote[n & 1][half ^ 1][quarter] != 0;
    l += bars->red[n & 1][half ^ 1][r];
    if (ok && mbar_wait(&bars->pv_done, (n - 1) & 1, status, 82)) {
      tc_fence_after();
      const float inv = 1.f / l;
      uint16_t* orow = out + int64_t(row0 + qb * BM + r) * ld_out + h * D + 64 * half;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tmem + lane_off + kOCol + 64 * half + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c * 32 + 8 * v) = w;
        }
      }
      if (half == 0) lse[(int64_t(b) * Hl + h) * seq + qb * BM + r] = m + log2f(l);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
  (void)mb;
#undef TDB_TL
}


// ===========================================================================
// Backward (deterministic, no atomics), two tcgen05 kernels after the
// Dsum pre-pass:  P = exp2(S*scale*log2e - lse),  dS = P * (dP - Dsum).
// ===========================================================================
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// K-major SW128 operand of 64 rows spanning two 64-column boxes (8 KB each).
__device__ __forceinline__ uint64_t desc_k64(uint32_t base, int k) {
  return smem_desc_sw128(base + (k >> 2) * 8192 + (k & 3) * 32, 16, 1024);
}
// MN-major SW128 operand [K = 64 rows][N = 128] stored as two [64][64] boxes.
__device__ __forceinline__ uint64_t desc_mn64(uint32_t base, int k) {
  return smem_desc_sw128(base + k * 16 * 128, 8192, 1024);
}


// dS for this thread's 32 key columns of the dQ kernel:
// ds = exp2(s*sl2 - lse) * (dp - Dsum).  MASK: columns c > lim are excluded.
template <bool MASK>
__device__ __forceinline__ void dq_row32(const uint32_t (&sv)[32], const uint32_t (&pv)[32], float sl2, float L,
                                         float Dr, int lim, uint32_t (&pk)[16]) {
  const float nl = -L;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    float d2[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = 2 * e + u;
      float p = ex2(fmaf(__uint_as_float(sv[c]), sl2, nl));
      if (MASK) p = c <= lim ? p : 0.f;
      d2[u] = p * (__uint_as_float(pv[c]) - Dr);
    }
    pk[e] = pack_bf16x2(d2[0], d2[1]);
  }
}

// P^T and dS^T for this thread's 32 query columns of the dK/dV kernel (lse /
// Dsum per column from shared memory).  MASK: columns c < lim are excluded.
template <bool MASK>
__device__ __forceinline__ void dkdv_row32(const uint32_t (&sv)[32], const uint32_t (&pv)[32], float sl2,
                                           const float* st, int lim, uint32_t (&pp)[16], uint32_t (&dd)[16]) {
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const float2 lse2 = *reinterpret_cast<const float2*>(st + 2 * e);
    const float2 ds2 = *reinterpret_cast<const float2*>(st + 64 + 2 * e);
    float p0 = ex2(fmaf(__uint_as_float(sv[2 * e]), sl2, -lse2.x));
    float p1 = ex2(fmaf(__uint_as_float(sv[2 * e + 1]), sl2, -lse2.y));
    if (MASK) {
      p0 = 2 * e >= lim ? p0 : 0.f;
      p1 = 2 * e + 1 >= lim ? p1 : 0.f;
    }
    pp[e] = pack_bf16x2(p0, p1);
    dd[e] = pack_bf16x2(p0 * (__uint_as_float(pv[2 * e]) - ds2.x), p1 * (__uint_as_float(pv[2 * e + 1]) - ds2.y));
  }
}

// Write `chunks` x 32 fp32 TMEM columns of this thread's row (times mul) as bf16.
__device__ __forceinline__ void tmem_cols_to_bf16(uint32_t taddr, int chunks, float mul, uint16_t* dst) {
#pragma unroll 1
  for (int c = 0; c < chunks; ++c) {
    uint32_t o[32];
    tmem_ld_32x32b_x32(taddr + c * 32, o);
    tmem_wait_ld();
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      uint4 w;
      w.x = pack_bf16x2(__uint_as_float(o[8 * v + 0]) * mul, __uint_as_float(o[8 * v + 1]) * mul);
      w.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]) * mul, __uint_as_float(o[8 * v + 3]) * mul);
      w.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]) * mul, __uint_as_float(o[8 * v + 5]) * mul);
      w.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]) * mul, __uint_as_float(o[8 * v + 7]) * mul);
      *reinterpret_cast<uint4*>(dst + c * 32 + 8 * v) = w;
    }
  }
}

// ---------------------------------------------------------------------------
// Backward warp layout (both kernels): warp 0 TMA, warp 1 MMA, warps 2..9
// score warps.  Score steps are independent (no running statistics), so the
// two warps of a TMEM lane quarter take alternate steps: half h owns steps
// i = h, h+2, ... and with them TMEM buffer h (scores and their gradient
// operands), which removes any sharing between warps.  The bf16 operand of
// the second GEMM pair (P^T, dS^T or dS) is written back into TMEM over the
// fp32 scores it came from and read from there by tcgen05.mma (A operand in
// tensor memory), so shared memory only carries the TMA tiles.  A buffer is
// rewritten by the MMA warp only after the GEMMs that read it (one thread,
// in-order issue), and the score warps see the new scores through the
// commit that also covers those GEMMs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// ---------------------------------------------------------------------------
// dQ: CTA = 128 queries; key/value tiles of 64 through a ring
// (K0, V0, K1, V1, ...).  K_j stays until dQ += dS_j K_j has read it.
// TMEM: S[2] cols 0/64 (dS bf16 pairs over their first 32 columns),
// dP[2] cols 128/192, dQ cols 256..383.
// ---------------------------------------------------------------------------
namespace dqk {
constexpr int kKV = 64 * 128 * 2;  // [64 keys][128 d] = two 8 KB boxes
constexpr int kSlots = 8;
struct alignas(8) Bars {
  uint64_t q_full;
  uint64_t kv_full[kSlots];
  uint64_t kv_empty[kSlots];
  uint64_t s_full[2];
  uint64_t ds_full[2];
  uint64_t done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr int kSmem = 2 * kTile + kSlots * kKV + 1024 + int(sizeof(Bars));
static_assert(kSmem <= 232448, "shared memory budget");
}  // namespace dqk

__global__ void __launch_bounds__(kThreads, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv,
                  const __grid_constant__ CUtensorMap tdo, const float* __restrict__ lse,
                  const float* __restrict__ dsum, uint16_t* __restrict__ dqkv, int64_t ld_dqkv, int seq, int Hl,
                  float scale, int* status) {
  constexpr int kSlots = dqk::kSlots, kKV = dqk::kKV;
  using Bars = dqk::Bars;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sDO = sQ + kTile;
  uint8_t* sKV = sDO + kTile;
  Bars* bars = reinterpret_cast<Bars*>(sKV + kSlots * kKV);

  const int hb = blockIdx.x;
  const int h = hb % Hl, b = hb / Hl;
  const int nq = seq / BM;
  const int qb = nq - 1 - int(blockIdx.y);
  const int n = 2 * qb + 2;  // 64-key tiles up to the diagonal
  const int row0 = b * seq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->ds_full[i], 4);
    }
    mbar_init(&bars->done, 1);
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tkv);
      prefetch_tmap(&tdo);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars->q_full, 2 * kTile);
      tma_load_2d(sQ, &tq, &bars->q_full, h * D, row0 + qb * BM);
      tma_load_2d(sQ + kBox, &tq, &bars->q_full, h * D + 64, row0 + qb * BM);
      tma_load_2d(sDO, &tdo, &bars->q_full, h * D, row0 + qb * BM);
      tma_load_2d(sDO + kBox, &tdo, &bars->q_full, h * D + 64, row0 + qb * BM);
      int i = 0;
      bool ok = true;
      for (; i < 2 * n; ++i) {
        const int s = i % kSlots;
        if (!mbar_wait(&bars->kv_empty[s], ((i / kSlots) & 1) ^ 1, status, 90)) { ok = false; *abort_flag = 1; break; }
        if (*abort_flag) { ok = false; break; }
        const int j = i >> 1;
        const int col = ((i & 1) ? 2 * Hl + h : Hl + h) * D;
        uint8_t* dst = sKV + s * kKV;
        mbar_arrive_expect_tx(&bars->kv_full[s], kKV);
        tma_load_2d(dst, &tkv, &bars->kv_full[s], col, row0 + j * 64);
        tma_load_2d(dst + 8192, &tkv, &bars->kv_full[s], col + 64, row0 + j * 64);
      }
      mbar_wait(&bars->q_full, 0, status, 91);
      if (!ok)
        for (int k = (i >= kSlots ? i - kSlots : 0); k < i; ++k)
          mbar_wait(&bars->kv_full[k % kSlots], (k / kSlots) & 1, status, 92);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(BM, 64, false, false);
      constexpr uint32_t idQ = idesc_bf16(BM, D, false, true);
      bool ok = mbar_wait(&bars->q_full, 0, status, 100);
      bool issued = false;
      const uint32_t sq = smem_u32(sQ), sdo = smem_u32(sDO);
      auto item = [&](int i, uint32_t& addr) -> bool {
        const int s = i % kSlots;
        if (!mbar_wait(&bars->kv_full[s], (i / kSlots) & 1, status, 101)) return false;
        if (*abort_flag) return false;
        tc_fence_after();
        addr = smem_u32(sKV + s * kKV);
        return true;
      };
      auto issue_sdp = [&](int j) -> bool {
        uint32_t sk, sv;
        if (!item(2 * j, sk)) return false;
        const uint32_t dS_ = tmem + (j & 1) * 64, dP_ = tmem + 128 + (j & 1) * 64;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_f16_ss(dS_, desc_k(sq, k), desc_k64(sk, k), idS, k > 0 ? 1u : 0u);
        if (!item(2 * j + 1, sv)) return false;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_f16_ss(dP_, desc_k(sdo, k), desc_k64(sv, k), idS, k > 0 ? 1u : 0u);
        umma_commit(&bars->kv_empty[(2 * j + 1) % kSlots]);
        umma_commit(&bars->s_full[j & 1]);
        issued = true;
        return true;
      };
      if (ok) ok = issue_sdp(0);
      if (ok && n > 1) ok = issue_sdp(1);
      for (int j = 0; j < n && ok; ++j) {
        if (!mbar_wait(&bars->ds_full[j & 1], (j >> 1) & 1, status, 102)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sk = smem_u32(sKV + ((2 * j) % kSlots) * kKV);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16_ts(tmem + 256, tmem + (j & 1) * 64 + 8 * k, desc_mn64(sk, k), idQ, (j | k) ? 1u : 0u);
        umma_commit(&bars->kv_empty[(2 * j) % kSlots]);
        if (j + 2 < n) ok = issue_sdp(j + 2);
      }
      if (ok) umma_commit(&bars->done);
      if (!ok) *abort_flag = 1;
      if (issued) {
        umma_commit(&bars->drain);
        mbar_wait(&bars->drain, 0, status, 103);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // this warp takes key tiles j = half, half + 2, ...
    const int r = quarter * 32 + lane;
    const int qi = qb * BM + r;
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const float sl2 = scale * kLog2e;
    const int64_t stat = (int64_t(b) * Hl + h) * seq + qi;
    const float L = lse[stat], Dr = dsum[stat];
    bool ok = true;
    const uint32_t sbuf = tmem + lane_off + half * 64, pbuf = sbuf + 128;
    for (int j = half; j < n && ok; j += 2) {
      if (!mbar_wait(&bars->s_full[half], (j >> 1) & 1, status, 110)) { ok = false; break; }
      if (*abort_flag) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // 32 keys at a time; dS of keys [32c, +32) -> columns [16c, +16)
        uint32_t sv[32], pv[32], pk[16];
        tmem_ld_32x32b_x32(sbuf + 32 * c, sv);
        tmem_ld_32x32b_x32(pbuf + 32 * c, pv);
        tmem_wait_ld();
        if (j >= 2 * qb) {
          dq_row32<true>(sv, pv, sl2, L, Dr, qi - j * 64 - 32 * c, pk);
        } else {
          dq_row32<false>(sv, pv, sl2, L, Dr, 0, pk);
        }
        tmem_st_32x32b_x16(sbuf + 16 * c, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ds_full[half]);
    }
    if (!ok) *abort_flag = 1;
    if (ok && mbar_wait(&bars->done, 0, status, 112)) {
      tc_fence_after();
      tmem_cols_to_bf16(tmem + lane_off + 256 + 64 * half, 2, scale,
                        dqkv + int64_t(row0 + qi) * ld_dqkv + h * D + 64 * half);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// ---------------------------------------------------------------------------
// dK, dV: CTA = 128 keys; query tiles of 64 (Q_i, dO_i, lse_i, Dsum_i)
// through a ring.  S^T = K Q_i^T, dP^T = V dO_i^T (thread = key row),
// dV += P^T dO_i, dK += dS^T Q_i (the Q_i / dO_i tiles serve as the K-major B
// operand of the first pair and the MN-major B operand of the second; P^T
// and dS^T are the TMEM A operands).
// TMEM: S^T[2] cols 0/64 (P^T over their first 32), dP^T[2] cols 128/192
// (dS^T over their first 32), dV 256.., dK 384..
// ---------------------------------------------------------------------------
namespace dkv {
constexpr int kQ = 64 * 128 * 2;  // [64 q][128 d] = two 8 KB boxes
constexpr int kSlot = 2 * kQ;     // Q_i then dO_i
constexpr int kSlots = 4;
struct alignas(8) Bars {
  uint64_t kv_full;
  uint64_t q_full[kSlots];
  uint64_t q_empty[kSlots];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr int kSmem = 2 * kTile + kSlots * kSlot + kSlots * 512 + 1024 + int(sizeof(Bars));
static_assert(kSmem <= 232448, "shared memory budget");
}  // namespace dkv

__global__ void __launch_bounds__(kThreads, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tkv, const __grid_constant__ CUtensorMap tq,
                    const __grid_constant__ CUtensorMap tdo, const float* __restrict__ lse,
                    const float* __restrict__ dsum, uint16_t* __restrict__ dqkv, int64_t ld_dqkv, int seq, int Hl,
                    float scale, int* status) {
  constexpr int kSlots = dkv::kSlots, kQ = dkv::kQ, kSlot = dkv::kSlot;
  using Bars = dkv::Bars;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + kTile;
  uint8_t* sRing = sV + kTile;
  float* sStat = reinterpret_cast<float*>(sRing + kSlots * kSlot);  // per slot: lse[64], dsum[64]
  Bars* bars = reinterpret_cast<Bars*>(reinterpret_cast<uint8_t*>(sStat) + kSlots * 512);

  const int hb = blockIdx.x;
  const int h = hb % Hl, b = hb / Hl;
  const int nq = seq / BM;
  const int kb = int(blockIdx.y);  // heaviest (kb = 0) first
  const int t0 = 2 * kb;           // first 64-query tile that sees these keys
  const int n = 2 * nq - t0;
  const int row0 = b * seq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* lse_h = lse + (int64_t(b) * Hl + h) * seq;
  const float* dsum_h = dsum + (int64_t(b) * Hl + h) * seq;

  if (threadIdx.x == 0) {
    mbar_init(&bars->kv_full, 1);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&bars->q_full[s], 1);
      mbar_init(&bars->q_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 4);
    }
    mbar_init(&bars->done, 1);
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
    if (lane == 0) {
      prefetch_tmap(&tkv);
      prefetch_tmap(&tq);
      prefetch_tmap(&tdo);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars->kv_full, 2 * kTile);
      tma_load_2d(sK, &tkv, &bars->kv_full, (Hl + h) * D, row0 + kb * BM);
      tma_load_2d(sK + kBox, &tkv, &bars->kv_full, (Hl + h) * D + 64, row0 + kb * BM);
      tma_load_2d(sV, &tkv, &bars->kv_full, (2 * Hl + h) * D, row0 + kb * BM);
      tma_load_2d(sV + kBox, &tkv, &bars->kv_full, (2 * Hl + h) * D + 64, row0 + kb * BM);
      int i = 0;
      bool ok = true;
      for (; i < n; ++i) {
        const int s = i % kSlots;
        if (!mbar_wait(&bars->q_empty[s], ((i / kSlots) & 1) ^ 1, status, 120)) { ok = false; *abort_flag = 1; break; }
        if (*abort_flag) { ok = false; break; }
        const int q0 = (t0 + i) * 64;
        uint8_t* dst = sRing + s * kSlot;
        float* st = sStat + s * 128;
        mbar_arrive_expect_tx(&bars->q_full[s], kSlot + 512);
        tma_load_2d(dst, &tq, &bars->q_full[s], h * D, row0 + q0);
        tma_load_2d(dst + 8192, &tq, &bars->q_full[s], h * D + 64, row0 + q0);
        tma_load_2d(dst + kQ, &tdo, &bars->q_full[s], h * D, row0 + q0);
        tma_load_2d(dst + kQ + 8192, &tdo, &bars->q_full[s], h * D + 64, row0 + q0);
        bulk_load(st, lse_h + q0, 256, &bars->q_full[s]);
        bulk_load(st + 64, dsum_h + q0, 256, &bars->q_full[s]);
      }
      mbar_wait(&bars->kv_full, 0, status, 121);
      if (!ok)
        for (int k = (i >= kSlots ? i - kSlots : 0); k < i; ++k)
          mbar_wait(&bars->q_full[k % kSlots], (k / kSlots) & 1, status, 122);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(BM, 64, false, false);
      constexpr uint32_t idG = idesc_bf16(BM, D, false, true);
      bool ok = mbar_wait(&bars->kv_full, 0, status, 130);
      bool issued = false;
      const uint32_t sk = smem_u32(sK), sv = smem_u32(sV);
      auto issue_sdp = [&](int i) -> bool {
        const int s = i % kSlots;
        if (!mbar_wait(&bars->q_full[s], (i / kSlots) & 1, status, 131)) return false;
        if (*abort_flag) return false;
        tc_fence_after();
        const uint32_t sq = smem_u32(sRing + s * kSlot), sdo = sq + kQ;
        const uint32_t dS_ = tmem + (i & 1) * 64, dP_ = tmem + 128 + (i & 1) * 64;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_f16_ss(dS_, desc_k(sk, k), desc_k64(sq, k), idS, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_f16_ss(dP_, desc_k(sv, k), desc_k64(sdo, k), idS, k > 0 ? 1u : 0u);
        umma_commit(&bars->s_full[i & 1]);
        issued = true;
        return true;
      };
      if (ok) ok = issue_sdp(0);
      if (ok && n > 1) ok = issue_sdp(1);
      for (int i = 0; i < n && ok; ++i) {
        if (!mbar_wait(&bars->p_full[i & 1], (i >> 1) & 1, status, 132)) { ok = false; break; }
        tc_fence_after();
        const int s = i % kSlots;
        const uint32_t sq = smem_u32(sRing + s * kSlot), sdo = sq + kQ;
        const uint32_t tpt = tmem + (i & 1) * 64, tdst = tmem + 128 + (i & 1) * 64;
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_f16_ts(tmem + 256, tpt + 8 * k, desc_mn64(sdo, k), idG, (i | k) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_f16_ts(tmem + 384, tdst + 8 * k, desc_mn64(sq, k), idG, (i | k) ? 1u : 0u);
        umma_commit(&bars->q_empty[s]);
        if (i + 2 < n) ok = issue_sdp(i + 2);
      }
      if (ok) umma_commit(&bars->done);
      if (!ok) *abort_flag = 1;
      if (issued) {
        umma_commit(&bars->drain);
        mbar_wait(&bars->drain, 0, status, 133);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // this warp takes query tiles i = half, half + 2, ...
    const int r = quarter * 32 + lane;
    const int kj = kb * BM + r;  // this thread's key
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const float sl2 = scale * kLog2e;
    bool ok = true;
    const uint32_t sbuf = tmem + lane_off + half * 64, pbuf = sbuf + 128;
    for (int i = half; i < n && ok; i += 2) {
      if (!mbar_wait(&bars->s_full[half], (i >> 1) & 1, status, 140)) { ok = false; break; }
      // the lse / Dsum rows of this tile arrived with Q_i (same transaction barrier)
      if (!mbar_wait(&bars->q_full[i % kSlots], (i / kSlots) & 1, status, 141)) { ok = false; break; }
      if (*abort_flag) { ok = false; break; }
      tc_fence_after();
      const float* st = sStat + (i % kSlots) * 128;
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // 32 queries at a time -> bf16 pairs in columns [16c, +16)
        uint32_t sv[32], pv[32], pp[16], dd[16];
        tmem_ld_32x32b_x32(sbuf + 32 * c, sv);
        tmem_ld_32x32b_x32(pbuf + 32 * c, pv);
        tmem_wait_ld();
        if (i < 2) {
          dkdv_row32<true>(sv, pv, sl2, st + 32 * c, kj - (t0 + i) * 64 - 32 * c, pp, dd);
        } else {
          dkdv_row32<false>(sv, pv, sl2, st + 32 * c, 0, pp, dd);
        }
        tmem_st_32x32b_x16(sbuf + 16 * c, pp);
        tmem_st_32x32b_x16(pbuf + 16 * c, dd);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[half]);
    }
    if (!ok) *abort_flag = 1;
    if (ok && mbar_wait(&bars->done, 0, status, 143)) {
      tc_fence_after();
      uint16_t* rowp = dqkv + int64_t(row0 + kj) * ld_dqkv + 64 * half;
      tmem_cols_to_bf16(tmem + lane_off + 256 + 64 * half, 2, 1.f, rowp + (2 * Hl + h) * D);
      tmem_cols_to_bf16(tmem + lane_off + 384 + 64 * half, 2, scale, rowp + (Hl + h) * D);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace attn_tc
}  // namespace tdb

// qkv [mb*seq, ld] (Q|K|V column blocks of Hl*128), out [mb*seq, ld_out],
// lse [mb, Hl, seq].  Requires seq % 128 == 0 and 16-byte aligned rows.
static int attn_fwd_tc_launch(const void* qkv, int64_t ld, void* out, int64_t ld_out, float* lse, int mb, int seq,
                              int Hl, float scale, void* stream, unsigned long long* tl) {
  using namespace tdb::attn_tc;
  if (!qkv || !out || !lse || mb <= 0 || seq <= 0 || Hl <= 0 || seq % BM || ld % 8 || ld_out % 8 ||
      ld < int64_t(3) * Hl * D || ld_out < int64_t(Hl) * D || reinterpret_cast<uintptr_t>(out) % 16)
    return tdb_host::fail(int(cudaErrorInvalidValue),
                          "attention fwd (tcgen05): needs seq %% 128 == 0, 16-byte aligned rows (seq=%d)", seq);
  CUtensorMap tm;
  int rc = tdb_host::make_tmap_2d(&tm, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(3) * Hl * D,
                                  uint64_t(mb) * seq, uint64_t(ld), 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static bool init = false;
  if (!init) {
    cudaError_t e = cudaFuncSetAttribute(fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return tdb_host::fail(int(e), "attention fwd (tcgen05): smem attribute");
    init = true;
  }
  dim3 grid(Hl * mb, seq / BM);
  fwd_kernel<<<grid, kThreads, kSmem, static_cast<cudaStream_t>(stream)>>>(
      tm, static_cast<uint16_t*>(out), ld_out, lse, seq, Hl, mb, scale, tdb_host::status_ptr(), tl);
  tdb_host::launched(1);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : tdb_host::fail(int(e), "attention fwd (tcgen05) launch: %s", cudaGetErrorString(e));
}

TDB_API int tdb_attn_fwd_tc(const void* qkv, int64_t ld, void* out, int64_t ld_out, float* lse, int mb, int seq,
                            int Hl, float scale, void* stream) {
  return attn_fwd_tc_launch(qkv, ld, out, ld_out, lse, mb, seq, Hl, scale, stream, nullptr);
}

// Diagnostic variant: also records the pipeline timeline of the first CTA
// into tl (uint64 [16 * steps], clock64 values; see fwd_kernel).
TDB_API int tdb_attn_fwd_tc_timeline(const void* qkv, int64_t ld, void* out, int64_t ld_out, float* lse, int mb,
                                     int seq, int Hl, float scale, void* stream, unsigned long long* tl) {
  return attn_fwd_tc_launch(qkv, ld, out, ld_out, lse, mb, seq, Hl, scale, stream, tl);
}

TDB_API int tdb_attn_bwd_pre(const void* out, int64_t ld_out, const void* dout, int64_t ld_dout, float* dsum, int mb,
                             int seq, int Hl, void* stream);

// The dK/dV and dQ kernels are independent (they read the same inputs and
// write disjoint columns of dqkv), so the dQ kernel runs on a second stream
// of this library, forked from and joined back into the caller's stream with
// events (a CUDA graph capture follows the fork and the join).  With few local
// heads -- 4 at TP8, i.e. 64 CTAs per kernel on 148 SMs -- the two then share
// the GPU instead of running one after the other.  Per host thread and device.
namespace {
struct BwdFork {
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
thread_local BwdFork t_bwd_fork[64];

int bwd_fork_for_device(BwdFork** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) return tdb_host::fail(int(cudaErrorInvalidDevice), "attention bwd: device");
  BwdFork& f = t_bwd_fork[dev];
  if (!f.side) {
    if ((e = cudaStreamCreateWithFlags(&f.side, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&f.fork, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&f.join, cudaEventDisableTiming)) != cudaSuccess)
      return tdb_host::fail(int(e), "attention bwd: second stream: %s", cudaGetErrorString(e));
  }
  *out = &f;
  return 0;
}
}  // namespace

// Backward on the tensor cores: Dsum pre-pass, then the dK/dV and dQ
// kernels (concurrently, see above).  Same contract as tdb_attn_bwd; needs
// seq % 128 == 0.
TDB_API int tdb_attn_bwd_tc(const void* qkv, int64_t ld, const void* out, int64_t ld_out, const void* dout,
                            int64_t ld_dout, const float* lse, float* dsum, void* dqkv, int64_t ld_dqkv, int mb,
                            int seq, int Hl, float scale, void* stream) {
  using namespace tdb::attn_tc;
  if (!qkv || !out || !dout || !lse || !dsum || !dqkv || mb <= 0 || seq <= 0 || Hl <= 0 || seq % BM || ld % 8 ||
      ld_dout % 8 || ld_dqkv % 8 || ld < int64_t(3) * Hl * D || ld_dqkv < int64_t(3) * Hl * D ||
      ld_dout < int64_t(Hl) * D || reinterpret_cast<uintptr_t>(dqkv) % 16 ||
      reinterpret_cast<uintptr_t>(lse) % 16 || reinterpret_cast<uintptr_t>(dsum) % 16)
    return tdb_host::fail(int(cudaErrorInvalidValue),
                          "attention bwd (tcgen05): needs seq %% 128 == 0 and 16-byte aligned rows (seq=%d)", seq);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = tdb_attn_bwd_pre(out, ld_out, dout, ld_dout, dsum, mb, seq, Hl, stream);
  if (rc) return rc;
  CUtensorMap tkv128, tkv64, tdo128, tdo64;
  const uint64_t rows = uint64_t(mb) * seq;
  if ((rc = tdb_host::make_tmap_2d(&tkv128, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(3) * Hl * D, rows,
                                   uint64_t(ld), 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = tdb_host::make_tmap_2d(&tkv64, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(3) * Hl * D, rows,
                                   uint64_t(ld), 64, 64, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = tdb_host::make_tmap_2d(&tdo128, dout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(Hl) * D, rows,
                                   uint64_t(ld_dout), 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = tdb_host::make_tmap_2d(&tdo64, dout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(Hl) * D, rows,
                                   uint64_t(ld_dout), 64, 64, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  static bool init = false;
  if (!init) {
    cudaError_t e = cudaFuncSetAttribute(bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dkv::kSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dqk::kSmem);
    if (e != cudaSuccess) return tdb_host::fail(int(e), "attention bwd (tcgen05): smem attribute");
    init = true;
  }
  BwdFork* fork = nullptr;
  if ((rc = bwd_fork_for_device(&fork))) return rc;
  const dim3 grid(Hl * mb, seq / BM);
  uint16_t* dq = static_cast<uint16_t*>(dqkv);
  cudaError_t e = cudaEventRecord(fork->fork, s);  // after the Dsum pre-pass
  if (e == cudaSuccess) e = cudaStreamWaitEvent(fork->side, fork->fork, 0);
  if (e != cudaSuccess) return tdb_host::fail(int(e), "attention bwd: fork: %s", cudaGetErrorString(e));
  bwd_dkdv_kernel<<<grid, kThreads, dkv::kSmem, s>>>(tkv128, tkv64, tdo64, lse, dsum, dq, ld_dqkv, seq, Hl, scale,
                                                      tdb_host::status_ptr());
  tdb_host::launched(1);
  bwd_dq_kernel<<<grid, kThreads, dqk::kSmem, fork->side>>>(tkv128, tkv64, tdo128, lse, dsum, dq, ld_dqkv, seq, Hl,
                                                             scale, tdb_host::status_ptr());
  tdb_host::launched(1);
  e = cudaGetLastError();
  if (e != cudaSuccess) return tdb_host::fail(int(e), "attention bwd (tcgen05) launch: %s", cudaGetErrorString(e));
  e = cudaEventRecord(fork->join, fork->side);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, fork->join, 0);
  return e == cudaSuccess ? 0 : tdb_host::fail(int(e), "attention bwd: join: %s", cudaGetErrorString(e));
}
