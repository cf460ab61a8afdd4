// Fused GEMM -> reduce-scatter over NVLink peer memory (the five-arm operator).
//
//   out[rows of this rank] = bias + residual + sum_{s=0..W-1} (A_s @ W_s^T)[rows of this rank]
//
// A call is a one-thread call-state advance (rs_advance_kernel) and two
// kernels on the caller's stream:
//
// 1. Produce (gemm_rs_kernel, persistent).  The tcgen05 mainloop (gemm.cuh)
//    computes the full [m, N] partial product tile by tile in the order of a
//    device tile table (the arm's production schedule: contiguous, the common
//    interleave, the calibrated arrival order, or remote-first for training).
//    The epilogue stores each 128 x BN tile straight into the destination
//    rank's receive slot [source = this rank] through its peer pointer: BF16,
//    or -- for blocks selected by the TACO mask and remote destinations --
//    H128/E4M3 encoded in registers (one thread owns one row's 128-column
//    group), so only compressed bytes cross NVLink.  After its last tile each
//    CTA issues one system-scope fence and release-adds the (block, source)
//    counters of every tile it produced.  gemm_rs_mx_kernel is the same
//    producer with the calibrated blocks' tiles as block-scaled FP8 MMAs.
// 2. Consume (rs_reduce_kernel, all co-resident CTAs).  Each CTA reduces this
//    rank's output blocks: it waits until all W sources of a block are
//    complete (bounded acquire polling), decodes TACO sources in registers
//    (one warp per H128 group) and adds the sources in rank order 0..W-1 with
//    BF16 rounding after every addition, then adds the residual and the bias.
//    Consumer policy "ordered" walks blocks in schedule order with all CTAs;
//    "per-lane ready" (arrival arms) splits the CTAs into two lanes
//    (lane = within % 2) and each lane consumes whichever of its blocks is
//    complete first.  Summation order never depends on arrival, so arms that
//    only reorder are bitwise identical.
//
// Params::variant selects alternatives (same results, measured slower):
// per-warp signals right after each tile, and the consumer run inside the
// producer kernel under a cooperative launch.
//
// Buffers live in the symmetric heap (symm.cu): receive slots
// [2 sets][W sources][per blocks][chunk_rows * N * 2 bytes] and counters
// [2 sets][per][W] (uint32, monotonically increasing; the call state holds
// the value that means "complete" for this call).  Calls alternate sets,
// which makes reuse safe: a rank can only start call k+2 after every rank
// finished consuming call k.  Every wait is bounded by %globaltimer and
// reports through the status word.
//
// Reference parity: python/flux_dcu/runtime.py:84-268 (FluxDCU: schedule,
// TACO encode of remote blocks, two lanes, ordered vs per-lane-ready
// consumers, ordered BF16 source reduction, final join) and
// src/taco/codec.hip:78-148 (codec math, ordered reduce).
#include <climits>
#include <utility>

#include "call_state.cuh"
#include "codec.cuh"
#include "gemm.cuh"
#include "tensor_map.h"

namespace tdb {
namespace rs {

using gemm::BM;

struct Params {
  const uint64_t* peers;  // [W] heap base of each rank
  int W, rank;
  int m, N;
  int chunk_rows, per;
  uint64_t recv_off, slot_bytes, flags_off;
  int set;
  uint32_t expected;       // counter value meaning "all tiles of (block, source) arrived"
  const uint8_t* qmask;    // [m / chunk_rows] 1 = TACO wire format (remote only)
  uint16_t* out;           // [per * chunk_rows, N]
  const uint16_t* bias;    // [N] or null
  const uint16_t* residual;  // [per * chunk_rows, N] or null
  const int* consume;      // [per] local blocks in consumption order
  int policy;              // 0 ordered, 1 per-lane ready
  unsigned long long* timeline;  // [2 * per] {first ready seen, last consumed} or null
  long long delay_cycles;  // diagnostic: delay the signal of tile (delay_mb, delay_nb)
  int delay_mb, delay_nb;
  uint64_t wait_ns;
  unsigned long long* phases;  // optional [grid][4]: start, produce done, first block ready, end
  // optional device call state {set, expected, epoch, target0, target1}
  // written by rs_advance_kernel before each call; when present it replaces
  // `set` / `expected`, so a captured CUDA graph replays with fresh values
  const uint32_t* call_state;
  // bit 0: every epilogue warp signals its tile right after pushing it (one
  //        system fence per warp and tile) instead of one fence per CTA after
  //        its whole produce phase;
  // bit 1: the consumer runs inside the producer kernel (cooperative launch,
  //        every CTA resident), each CTA reducing blocks once it has produced.
  int variant;
};

__device__ __forceinline__ int call_set(const Params& p) { return p.call_state ? int(__ldg(p.call_state)) : p.set; }
__device__ __forceinline__ uint32_t call_expected(const Params& p) {
  return p.call_state ? __ldg(p.call_state + 1) : p.expected;
}

__device__ __forceinline__ uint8_t* slot_ptr(const Params& p, int rank_of_heap, int source, int within) {
  return reinterpret_cast<uint8_t*>(p.peers[rank_of_heap] + p.recv_off +
                                    (uint64_t(call_set(p) * p.W + source) * p.per + within) * p.slot_bytes);
}

__device__ __forceinline__ uint32_t* flag_ptr(const Params& p, int rank_of_heap, int within, int source) {
  return reinterpret_cast<uint32_t*>(p.peers[rank_of_heap] + p.flags_off +
                                     (uint64_t(call_set(p) * p.per + within) * p.W + source) * 4);
}


// Variant bit 2: BF16 tiles leave the epilogue as TMA bulk stores
// (cp.async.bulk shared::cta -> the destination's global memory), one 8 KB
// store per warp and 128-column half, instead of 16-byte st.global from the
// warp's lanes; every warp then signals each tile once its stores are
// complete (deferred by one tile, so the wait overlaps the next tile).
// Operators with TACO blocks ignore the bit (their producer is built
// without the bulk path).
constexpr int kVariantBulk = 4;

__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Receive-slot layout of bulk-pushed BF16 tiles: 8 KB slabs of 32 rows x 128
// columns in slab-major order over the [chunk_rows / 32, N / 128] grid; in a
// slab, row r holds its sixteen 16-byte chunks XOR-swizzled (physical chunk =
// logical chunk ^ (r & 15)), exactly as the epilogue staged them.
constexpr int kSlabBytes = 32 * 128 * 2;

__device__ __forceinline__ int64_t slab_of(int row, int col, int N) { return int64_t(row >> 5) * (N >> 7) + (col >> 7); }

// 16-byte vector v of a slab-layout slot -> its vector index in the
// row-major [chunk_rows, N] block.
__device__ __forceinline__ int64_t slab_vec_to_rowmajor(int64_t v, int N) {
  const int64_t slab = v >> 9;  // 512 vectors per slab
  const int r = int(v >> 4) & 31, pc = int(v) & 15;
  const int per_band = N >> 7;
  const int64_t row = (slab / per_band) * 32 + r;
  const int64_t col8 = (slab % per_band) * 16 + (pc ^ (r & 15));
  return row * (N >> 3) + col8;
}

// Byte offset of element (row, col) (col % 4 == 0) in a slab-layout slot.
__device__ __forceinline__ int64_t slab_byte(int row, int col, int N) {
  const int r = row & 31, lc = (col & 127) >> 3;
  return slab_of(row, col, N) * kSlabBytes + r * 256 + ((lc ^ (r & 15)) << 4) + (col & 7) * 2;
}

// Consumer policy 2 (training operators, remote-first production order, BF16
// wire): there is no consumer kernel.  Remote tiles are bulk-pushed (slab
// layout) and each epilogue warp, once its stores are complete, writes the
// call's epoch into a per-(block, tile, quarter, source) flag at the
// destination.  The epilogue of a tile of this rank's own blocks waits for
// the matching quarter of every peer, then sums the sources in rank order
// 0..W-1 -- its own partial straight from TMEM, the peers' from the receive
// slots -- with BF16 rounding after every addition, adds residual and bias,
// and writes the output rows.  Same arithmetic, hence bitwise the same
// result, as the consumer kernel.
constexpr int kPolicyEpilogue = 2;
constexpr uint64_t kFineFlagsOff = 32768;  // inside the 64 KB flag region
constexpr uint64_t kFineFlagsBytes = 32768;

__device__ __forceinline__ uint32_t call_epoch(const Params& p) { return __ldg(p.call_state + 2); }

// Flag of (block `within`, tile `t` of the block, row quarter q, source) in
// the heap of `rank_of_heap`, for the current set.
__device__ __forceinline__ uint32_t* fine_flag_ptr(const Params& p, int rank_of_heap, int within, int t, int tiles,
                                                  int q, int source) {
  const uint64_t idx = ((uint64_t(call_set(p) * p.per + within) * tiles + t) * 4 + q) * p.W + source;
  return reinterpret_cast<uint32_t*>(p.peers[rank_of_heap] + p.flags_off + kFineFlagsOff + idx * 4);
}

// One thread encodes one H128 group held in registers (values already BF16
// rounded).  Same math as codec.cuh; the butterfly pairs and their order are
// those of the warp version.
__device__ __forceinline__ void encode_group_thread(float (&x)[128], uint32_t (&words)[32], float& q, float& a) {
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 128; ++j) ss += x[j] * x[j];
  const float variance = fmaxf(ss * (1.0f / 128.0f) + 1e-6f, 1e-12f);
  a = fminf(fmaxf(448.0f * rsqrtf(variance), 1e-3f), 1e3f);
#pragma unroll
  for (int j = 0; j < 128; ++j) x[j] *= a;
#pragma unroll
  for (int s = 1; s < 128; s <<= 1) {
#pragma unroll
    for (int i = 0; i < 128; ++i) {
      if ((i & s) == 0) {
        const float lo = x[i], hi = x[i + s];
        x[i] = lo + hi;
        x[i + s] = lo - hi;
      }
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 128; ++j) {
    x[j] *= taco::kInvSqrt128;
    amax = fmaxf(amax, fabsf(x[j]));
  }
  q = fminf(fmaxf(fmaxf(amax, 1e-12f) / 448.0f, 1e-12f), 1e6f);
  // Multiply by the correctly rounded reciprocal instead of 128 divisions;
  // differs from f / q by at most one ulp before the 3-bit-mantissa rounding.
  const float rq = __frcp_rn(q);
#pragma unroll
  for (int w = 0; w < 32; ++w) {
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float f = isfinite(x[4 * w + j]) ? x[4 * w + j] : 0.0f;
      y[j] = fminf(fmaxf(f * rq, -448.0f), 448.0f);
    }
    words[w] = uint32_t(taco::e4m3x2(y[0], y[1])) | (uint32_t(taco::e4m3x2(y[2], y[3])) << 16);
  }
}

constexpr int kMaxWorldEpi = 8;

// Called by lane 0 of an epilogue warp (bulk pushes): wait until this
// thread's bulk groups, except the `keep_one` most recent, have written,
// then fence and signal the tile at its destination -- +1 on the (block,
// source) counter, or (policy 2) the call's epoch in the tile quarter's flag.
// Out of line: it runs once per tile and keeps the epilogue's registers free.
__device__ __forceinline__ void signal_stored_tile_inline(const Params* p, int tiles, int dest, int within, int tile,
                                                         int quarter, int mb, int nb, bool keep_one) {
  if (keep_one) bulk_wait<1>();
  else bulk_wait<0>();
  asm volatile("fence.proxy.async.global;" ::: "memory");
  if (p->delay_cycles > 0 && mb == p->delay_mb && nb == p->delay_nb) {
    const long long t0 = clock64();
    while (clock64() - t0 < p->delay_cycles) {
    }
  }
  __threadfence_system();
  if (p->policy == kPolicyEpilogue)
    st_release_sys(fine_flag_ptr(*p, dest, within, tile, tiles, quarter, p->rank), call_epoch(*p));
  else
    red_release_sys(flag_ptr(*p, dest, within, p->rank), 1u);
}

__device__ __noinline__ void signal_stored_tile(const Params* p, int tiles, int dest, int within, int tile, int quarter,
                                                int mb, int nb, bool keep_one) {
  signal_stored_tile_inline(p, tiles, dest, within, tile, quarter, mb, nb, keep_one);
}

__device__ __forceinline__ void unpack8(const uint4& w, float (&v)[8]) {
  const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[2 * j] = bf16_bits_to_float(a[j] & 0xffff);
    v[2 * j + 1] = bf16_bits_to_float(a[j] >> 16);
  }
}

// Policy 2, own tile, after the epilogue staged one warp's 32 rows x 128
// columns (BF16, the slab layout of the receive slots) at `own`: the warp
// reduces them with 16-byte vectors -- lane i takes vectors i, i + 32, ... of
// the slab, so every load of a peer's slab is coalesced -- in rank order
// 0..W-1 with BF16 rounding after each addition, then residual and bias, and
// writes the output rows.  Out of line, so that its registers do not add to
// the epilogue's.
__device__ __noinline__ void reduce_staged_half(const Params* p, const uint8_t* own_stage, int within, int rib0, int n0) {
  const int lane = threadIdx.x & 31;
  const int N = p->N;
  const uint4* own = reinterpret_cast<const uint4*>(own_stage);
  const int64_t slab_off = slab_of(rib0, n0, N) * kSlabBytes;
  const int64_t out_row0 = int64_t(within) * p->chunk_rows + rib0;
  __syncwarp();
#pragma unroll 1
  for (int i0 = 0; i0 < 16; i0 += 4) {
    // the residual and bias of these four vectors load with the first
    // sources, so one memory round trip serves both
    int64_t o[4];
    uint4 rw[4], bw[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = lane + 32 * (i0 + u);
      const int r = v >> 4, lc = (v & 15) ^ (r & 15);
      o[u] = (out_row0 + r) * N + n0 + lc * 8;
      if (p->residual) rw[u] = *reinterpret_cast<const uint4*>(p->residual + o[u]);
      if (p->bias) bw[u] = __ldg(reinterpret_cast<const uint4*>(p->bias + n0 + lc * 8));
    }
    float acc[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[u][j] = 0.f;
#pragma unroll
    for (int s0 = 0; s0 < kMaxWorldEpi; s0 += 4) {
      uint4 w[4][4];  // [source][vector]
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int s = s0 + t;
        if (s >= p->W) continue;
        const uint4* src = s == p->rank ? own
                                        : reinterpret_cast<const uint4*>(slot_ptr(*p, p->rank, s, within) + slab_off);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int v = lane + 32 * (i0 + u);
          w[t][u] = s == p->rank ? src[v] : __ldcg(src + v);
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        if (s0 + t >= p->W) continue;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float x[8];
          unpack8(w[t][u], x);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[u][j] = bf16_bits_to_float(float_to_bf16_bits(acc[u][j] + x[j]));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (p->residual) {
        float x[8];
        unpack8(rw[u], x);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[u][j] = bf16_bits_to_float(float_to_bf16_bits(x[j] + acc[u][j]));
      }
      if (p->bias) {
        float x[8];
        unpack8(bw[u], x);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[u][j] = bf16_bits_to_float(float_to_bf16_bits(acc[u][j] + x[j]));
      }
      uint4 ov;
      ov.x = pack_bf16x2(acc[u][0], acc[u][1]);
      ov.y = pack_bf16x2(acc[u][2], acc[u][3]);
      ov.z = pack_bf16x2(acc[u][4], acc[u][5]);
      ov.w = pack_bf16x2(acc[u][6], acc[u][7]);
      *reinterpret_cast<uint4*>(p->out + o[u]) = ov;
    }
  }
  __syncwarp();  // the next half may overwrite the staging
}

// QUANT = false compiles the TACO wire path out (operators whose blocks all
// cross as BF16), which frees the 128 registers of the per-row encoder.
template <int BN, bool QUANT = true>
struct PushEpi {
  // Per epilogue warp: a 32-row x 128-column BF16 slab (or the TACO payload
  // of those rows), XOR-swizzled in 16-byte chunks so that both the
  // row-per-lane writes and the row-contiguous reads are conflict-free.  A
  // tile row is pushed in 128-column halves as soon as a half is complete,
  // which halves the staging and leaves room for a deeper TMA ring.
  static constexpr int kHalf = 128;
  static constexpr int kRowBytes = kHalf * 2;
  static constexpr int kChunks = kRowBytes / 16;  // 16-byte chunks per staged row
  static constexpr int kSmemBytes = 4 * 32 * kRowBytes;
  const Params* p;
  int* status;
  uint8_t* stage_base;
  int within, dest, row0, quarter, nbase;
  bool quant;
  uint8_t* slot;
  float grp[QUANT ? 128 : 1];
  float q_half, a_half;
  bool bulk = false;
  // bulk mode, lane 0 of each epilogue warp: the tile whose signal is pending
  int pend_dest = -1, pend_within = 0, pend_mb = 0, pend_nb = 0, pend_tile = 0;
  // policy 2: this tile belongs to this rank and is reduced here; its index in the block
  bool local_reduce = false;
  int tile_in_block = 0;

  __device__ __forceinline__ void set_smem(uint8_t* ptr) { stage_base = ptr; }
  __device__ __forceinline__ void prologue(int*) {}

  template <int Q>
  __device__ __forceinline__ void stash(const uint32_t (&r)[32]) {
    if constexpr (QUANT) {
#pragma unroll
      for (int j = 0; j < 32; ++j) grp[Q * 32 + j] = bf16_bits_to_float(float_to_bf16_bits(__uint_as_float(r[j])));
    }
  }

  __device__ __forceinline__ uint8_t* stage() const { return stage_base + ((threadIdx.x >> 5) & 3) * 32 * kRowBytes; }

  __device__ __forceinline__ static int swz(int row, int chunk) { return chunk ^ (row & (kChunks - 1)); }

  __device__ __forceinline__ void tile_begin(int mb, int nb) {
    const int m0 = mb * BM;
    const int physical = m0 / p->chunk_rows;
    dest = physical / p->per;
    within = physical % p->per;
    row0 = m0 - physical * p->chunk_rows;
    quant = QUANT && p->qmask[physical] != 0 && dest != p->rank;
    slot = slot_ptr(*p, dest, p->rank, within);
    quarter = (threadIdx.x >> 5) & 3;
    nbase = nb * BN;
    const bool epi_policy = p->policy == kPolicyEpilogue;
    // bulk pushes move BF16 slabs; operators with TACO blocks keep the lane stores
    bulk = !QUANT && (epi_policy || (p->variant & kVariantBulk) != 0);
    tile_in_block = (row0 / BM) * (p->N / BN) + nb;
    local_reduce = epi_policy && dest == p->rank;
    if (local_reduce) {
      // a peer may be waiting in its own epilogue for the tile pushed last:
      // release it before waiting here
      if ((threadIdx.x & 31) == 0) signal_pending(false);
      wait_peer_quarters();
    }
  }

  // Policy 2, own tile: every lane waits (bounded) until each peer's copy of
  // this warp's 32 rows of the tile is in the receive slot.
  __device__ __forceinline__ void wait_peer_quarters() {
    const uint32_t epoch = call_epoch(*p);
    const int tiles = (p->chunk_rows / BM) * (p->N / BN);
    for (int s = 0; s < p->W; ++s) {
      if (s == p->rank) continue;
      const uint32_t* f = fine_flag_ptr(*p, p->rank, within, tile_in_block, tiles, quarter, s);
      if (int32_t(ld_acquire_sys(f) - epoch) < 0) {
        const uint64_t t0 = globaltimer();
        while (int32_t(ld_acquire_sys(f) - epoch) < 0) {
          if (globaltimer() - t0 > p->wait_ns) {
            if ((threadIdx.x & 31) == 0) record_status(status, kTimeoutPeerFlag, 41, s, tile_in_block);
            return;  // the output of this call is invalid; the host raises on the status
          }
        }
      }
    }
  }

  __device__ __forceinline__ void reduce_half(int half) {
    reduce_staged_half(p, stage(), within, row0 + quarter * 32, nbase + half * kHalf);
  }

  // Lane 0, bulk mode: the pending tile's stores by this warp are complete
  // (all bulk groups but the `keep_one` most recent retired), then one system
  // fence and the signal (signal_stored_tile).
  __device__ __forceinline__ void signal_pending(bool keep_one) {
    if (pend_dest < 0) return;
    const int tiles = (p->chunk_rows / BM) * (p->N / BN);
    if constexpr (QUANT)  // a call here would have to save the encoder's registers
      signal_stored_tile_inline(p, tiles, pend_dest, pend_within, pend_tile, quarter, pend_mb, pend_nb, keep_one);
    else
      signal_stored_tile(p, tiles, pend_dest, pend_within, pend_tile, quarter, pend_mb, pend_nb, keep_one);
    pend_dest = -1;
  }

  // After the last tile (epilogue warps): signal what is still pending.
  __device__ __forceinline__ void finish() {
    if ((threadIdx.x & 31) == 0) signal_pending(false);
  }

  // Copy this warp's staged 32 rows x 128 columns (or their TACO payload and
  // scales) into the destination slot.
  __device__ __forceinline__ void push_half(int half) {
    const int lane = threadIdx.x & 31;
    const int N = p->N;
    const int n0 = nbase + half * kHalf;
    const int rib0 = row0 + quarter * 32;  // first block row of this warp
    const uint8_t* st = stage();
    if (bulk && !quant) {
      // the staged slab goes out as one bulk store; its smem is reusable once read
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        bulk_s2g(slot + slab_of(rib0, n0, N) * kSlabBytes, st, kSlabBytes);
        bulk_commit();
        if (half == 0) signal_pending(true);  // the previous tile's groups are older than this one
        bulk_wait_read<0>();
      }
      __syncwarp();
      return;
    }
    __syncwarp();
    if (!quant) {
      constexpr int kRowsPerIter = 32 / kChunks;  // 2 rows of 256 bytes per warp store
#pragma unroll 4
      for (int j = 0; j < 32; j += kRowsPerIter) {
        const int rr = j + lane / kChunks, ch = lane % kChunks;
        const uint4 v = reinterpret_cast<const uint4*>(st + rr * kRowBytes)[swz(rr, ch)];
        uint16_t* dst = reinterpret_cast<uint16_t*>(slot) + int64_t(rib0 + rr) * N + n0;
        reinterpret_cast<uint4*>(dst)[ch] = v;
      }
    } else if constexpr (QUANT) {
      constexpr int kPayChunks = kHalf / 16;       // 128 payload bytes per row
      constexpr int kRowsPerIter = 32 / kPayChunks;  // 4 rows per warp store
#pragma unroll 4
      for (int j = 0; j < 32; j += kRowsPerIter) {
        const int rr = j + lane / kPayChunks, ch = lane % kPayChunks;
        const uint4 v = reinterpret_cast<const uint4*>(st + rr * kRowBytes)[swz(rr, ch)];
        uint8_t* dst = slot + int64_t(rib0 + rr) * N + n0;
        reinterpret_cast<uint4*>(dst)[ch] = v;
      }
      const int64_t elements = int64_t(p->chunk_rows) * N;
      const int64_t groups = elements / 128;
      const int64_t g0 = (int64_t(rib0 + lane) * N + n0) / 128;
      float* scales = reinterpret_cast<float*>(slot + elements);
      scales[g0] = q_half;
      scales[groups + g0] = a_half;
    }
    __syncwarp();  // the next half may overwrite the staging
    if (bulk && half == 0 && lane == 0) signal_pending(false);  // no bulk group of this tile to keep
  }

  __device__ __forceinline__ void chunk(int /*row*/, int /*col*/, int c, const uint32_t (&r)[32]) {
    const int lane = threadIdx.x & 31;
    const int cl = c & 3;  // 32-column chunk inside the current 128-column half
    uint4* srow = reinterpret_cast<uint4*>(stage() + lane * kRowBytes);
    if (!quant) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 w;
        w.x = pack_bf16x2(__uint_as_float(r[8 * i + 0]), __uint_as_float(r[8 * i + 1]));
        w.y = pack_bf16x2(__uint_as_float(r[8 * i + 2]), __uint_as_float(r[8 * i + 3]));
        w.z = pack_bf16x2(__uint_as_float(r[8 * i + 4]), __uint_as_float(r[8 * i + 5]));
        w.w = pack_bf16x2(__uint_as_float(r[8 * i + 6]), __uint_as_float(r[8 * i + 7]));
        srow[swz(lane, cl * 4 + i)] = w;
      }
    } else if constexpr (QUANT) {
      // TACO: gather the 128-column group (4 chunks) in registers, BF16
      // rounded; the chunk index is a runtime value (the epilogue loop is not
      // unrolled), so dispatch to a compile-time register offset.
      switch (cl) {
        case 0: stash<0>(r); break;
        case 1: stash<1>(r); break;
        case 2: stash<2>(r); break;
        default: stash<3>(r); break;
      }
      if (cl == 3) {
        uint32_t words[32];
        encode_group_thread(grp, words, q_half, a_half);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          srow[swz(lane, i)] = make_uint4(words[4 * i], words[4 * i + 1], words[4 * i + 2], words[4 * i + 3]);
      }
    }
    if (cl == 3) {
      if constexpr (!QUANT) {  // policy 2 never runs with TACO blocks
        if (local_reduce) {
          reduce_half(c >> 2);
          return;
        }
      }
      push_half(c >> 2);
    }
  }

  __device__ __forceinline__ void tile_end(int mb, int nb, int, int lane) {
    if (local_reduce) return;  // reduced in place: nothing was sent
    if (bulk) {  // signalled once its stores are complete (next tile's first push or finish())
      if (lane == 0) {
        pend_dest = dest;
        pend_within = within;
        pend_mb = mb;
        pend_nb = nb;
        pend_tile = tile_in_block;
      }
      return;
    }
    // Variant bit 0: this warp's 32 rows of the tile are complete at the
    // destination once its stores are visible -- fence, then add 1 (four
    // warps make the 4 per tile that signal_tiles adds otherwise).
    if (!(p->variant & 1)) return;
    __syncwarp();
    if (lane == 0) {
      if (p->delay_cycles > 0 && mb == p->delay_mb && nb == p->delay_nb) {
        const long long t0 = clock64();
        while (clock64() - t0 < p->delay_cycles) {
        }
      }
      __threadfence_system();
      red_release_sys(flag_ptr(*p, dest, within, p->rank), 1u);
    }
  }
};

// After its produce phase a CTA makes all of its peer stores visible with a
// single system-scope fence and then adds 4 (one per epilogue warp) to the
// (block, source) counter of every tile it produced, in production order.
// The diagnostic delay holds back the signal of one tile only.
__device__ void signal_tiles(const Params& p, const gemm::TileOrder& order) {
  // signalled per tile by the epilogue warps (and policy 2 never touches the
  // per-block counters: its calls do not advance their targets)
  if ((p.variant & (1 | kVariantBulk)) || p.policy == kPolicyEpilogue) return;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int i = blockIdx.x; i < order.num_tiles; i += gridDim.x) {
    int mb, nb;
    order.tile(i, mb, nb);
    const int physical = (mb * BM) / p.chunk_rows;
    const int dest = physical / p.per, within = physical % p.per;
    if (p.delay_cycles > 0 && mb == p.delay_mb && nb == p.delay_nb) {
      const long long t0 = clock64();
      while (clock64() - t0 < p.delay_cycles) {
      }
    }
    red_release_sys(flag_ptr(p, dest, within, p.rank), 4u);
  }
}

// Block readiness: all W sources delivered (acquire).
__device__ __forceinline__ bool block_ready(const Params& p, int within) {
  for (int s = 0; s < p.W; ++s)
    if (ld_acquire_sys(flag_ptr(p, p.rank, within, s)) < call_expected(p)) return false;
  return true;
}


constexpr int kMaxWorld = 8;

// One 16-byte vector (8 outputs) of a BF16 block: ordered source sum, then
// residual, then bias.
// Vector v of a BF16 slot -> the block's row-major vector index (slab layout
// under bulk pushes, identity otherwise).
__device__ __forceinline__ int64_t out_vec(const Params& p, int64_t v) {
  return (p.variant & kVariantBulk) ? slab_vec_to_rowmajor(v, p.N) : v;
}

__device__ __forceinline__ uint4 reduce_vec8(const Params& p, uint64_t local_base, int within, int64_t v, int64_t vo) {
  uint4 src[kMaxWorld];
#pragma unroll
  for (int s = 0; s < kMaxWorld; ++s)
    if (s < p.W)
      src[s] = __ldcg(reinterpret_cast<const uint4*>(
                          local_base + p.recv_off + (uint64_t(call_set(p) * p.W + s) * p.per + within) * p.slot_bytes) + v);
  const int64_t ov = int64_t(within) * p.chunk_rows * p.N / 8 + vo;
  uint4 rw = make_uint4(0, 0, 0, 0), bw = make_uint4(0, 0, 0, 0);
  if (p.residual) rw = reinterpret_cast<const uint4*>(p.residual)[ov];
  if (p.bias) bw = reinterpret_cast<const uint4*>(p.bias)[uint32_t(vo) % uint32_t(p.N >> 3)];
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int s = 0; s < kMaxWorld; ++s) {
    if (s < p.W) {
      float x[8];
      unpack8(src[s], x);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = bf16_bits_to_float(float_to_bf16_bits(acc[j] + x[j]));
    }
  }
  if (p.residual) {
    float x[8];
    unpack8(rw, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = bf16_bits_to_float(float_to_bf16_bits(x[j] + acc[j]));
  }
  if (p.bias) {
    float x[8];
    unpack8(bw, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = bf16_bits_to_float(float_to_bf16_bits(acc[j] + x[j]));
  }
  uint4 o;
  o.x = pack_bf16x2(acc[0], acc[1]);
  o.y = pack_bf16x2(acc[2], acc[3]);
  o.z = pack_bf16x2(acc[4], acc[5]);
  o.w = pack_bf16x2(acc[6], acc[7]);
  return o;
}

// BF16 blocks of a batch (list of `count` block ids).  Vector v of a block
// always belongs to thread (v mod stride) of the partition -- independent of
// which blocks this CTA found ready -- and a thread chains its vectors across
// the batch's blocks so that four of them are in flight at once.
__device__ void consume_bf16_batch(const Params& p, const int* blocks, int count, int part, int nparts) {
  const int64_t nvec = int64_t(p.chunk_rows) * p.N / 8;
  const int64_t stride = int64_t(nparts) * blockDim.x;
  const int64_t t0 = int64_t(part) * blockDim.x + threadIdx.x;
  if (t0 >= nvec) return;
  const uint64_t local_base = p.peers[p.rank];
  constexpr int U = 4;
  int bi = 0;
  int64_t v = t0;
  while (bi < count) {
    int ib[U];
    int64_t iv[U];
    int n = 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (bi < count) {
        ib[u] = blocks[bi];
        iv[u] = v;
        n = u + 1;
        v += stride;
        if (v >= nvec) {
          ++bi;
          v = t0;
        }
      }
    }
    uint4 o[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (u < n) o[u] = reduce_vec8(p, local_base, ib[u], iv[u], out_vec(p, iv[u]));
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (u < n) reinterpret_cast<uint4*>(p.out)[int64_t(ib[u]) * nvec + out_vec(p, iv[u])] = o[u];
  }
}

// TACO block: one warp per H128 group; all sources' payload words and scales
// are loaded before the register decodes.
__device__ void consume_block_taco(const Params& p, int within, int part, int nparts) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const int gpr = p.N / 128;
  const int items = p.chunk_rows * gpr;
  const int64_t elements = int64_t(p.chunk_rows) * p.N;
  const int64_t groups = elements / 128;
  for (int it = part * nw + warp; it < items; it += nparts * nw) {
    const int rho = it / gpr, g = it % gpr;
    const int64_t e0 = int64_t(rho) * p.N + g * 128 + lane * 4;
    const int64_t gi = int64_t(rho) * gpr + g;
    uint32_t word[kMaxWorld];
    uint2 plain[kMaxWorld];
    float qv[kMaxWorld], av[kMaxWorld];
#pragma unroll
    for (int s = 0; s < kMaxWorld; ++s) {
      if (s >= p.W) continue;
      const uint8_t* slot = slot_ptr(p, p.rank, s, within);
      if (s != p.rank) {
        const float* scales = reinterpret_cast<const float*>(slot + elements);
        word[s] = __ldcg(reinterpret_cast<const unsigned int*>(slot + e0));
        qv[s] = __ldcg(scales + gi);
        av[s] = __ldcg(scales + groups + gi);
      } else if (p.variant & kVariantBulk) {  // this rank's own BF16 tile, bulk-pushed in slab layout
        plain[s] = __ldcg(reinterpret_cast<const uint2*>(slot + slab_byte(rho, g * 128 + lane * 4, p.N)));
      } else {
        plain[s] = __ldcg(reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(slot) + e0));
      }
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < kMaxWorld; ++s) {
      if (s >= p.W) continue;
      float v[4];
      if (s != p.rank) {
        taco::decode_group_warp(word[s], qv[s], av[s], lane, v);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = bf16_bits_to_float(float_to_bf16_bits(v[j]));
      } else {
        v[0] = bf16_bits_to_float(plain[s].x & 0xffff);
        v[1] = bf16_bits_to_float(plain[s].x >> 16);
        v[2] = bf16_bits_to_float(plain[s].y & 0xffff);
        v[3] = bf16_bits_to_float(plain[s].y >> 16);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = bf16_bits_to_float(float_to_bf16_bits(acc[j] + v[j]));
    }
    const int64_t o = (int64_t(within) * p.chunk_rows + rho) * p.N + g * 128 + lane * 4;
    if (p.residual) {
      const uint2 w = *reinterpret_cast<const uint2*>(p.residual + o);
      const float rr[4] = {bf16_bits_to_float(w.x & 0xffff), bf16_bits_to_float(w.x >> 16),
                           bf16_bits_to_float(w.y & 0xffff), bf16_bits_to_float(w.y >> 16)};
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = bf16_bits_to_float(float_to_bf16_bits(rr[j] + acc[j]));
    }
    if (p.bias) {
      const uint2 w = *reinterpret_cast<const uint2*>(p.bias + g * 128 + lane * 4);
      const float bb[4] = {bf16_bits_to_float(w.x & 0xffff), bf16_bits_to_float(w.x >> 16),
                           bf16_bits_to_float(w.y & 0xffff), bf16_bits_to_float(w.y >> 16)};
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = bf16_bits_to_float(float_to_bf16_bits(acc[j] + bb[j]));
    }
    uint2 ow;
    ow.x = pack_bf16x2(acc[0], acc[1]);
    ow.y = pack_bf16x2(acc[2], acc[3]);
    *reinterpret_cast<uint2*>(p.out + o) = ow;
  }
}

// Consumer.  Ordered policy: all CTAs take the longest prefix (in
// consumption order) of complete blocks; per-lane ready: the CTAs of lane l
// take every complete block of lane l.  Flags are polled by all threads in
// parallel with relaxed system-scope loads; a thread that sees a complete
// counter issues an acquire fence before the CTA barrier, after which the
// block's data is read (at L2).  The BF16 blocks of one batch are reduced
// together; TACO blocks one after another.
__device__ void consume_phase(const Params& p, int* status) {
  __shared__ int s_bf[64], s_tq[64];
  __shared__ int s_nb, s_nq;
  __shared__ int s_missing[64];
  __shared__ unsigned long long s_done;
  int part = blockIdx.x, nparts = gridDim.x, lane_id = -1;
  if (p.policy == 1) {
    lane_id = blockIdx.x & 1;
    part = blockIdx.x >> 1;
    nparts = (gridDim.x + 1 - lane_id) >> 1;
  }
  uint64_t mine = 0;
  for (int k = 0; k < p.per; ++k)
    if (lane_id < 0 || (p.consume[k] % 2) == lane_id) mine |= 1ull << k;
  if (threadIdx.x == 0) s_done = 0;
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(p.peers[p.rank] + p.flags_off) +
                          uint64_t(call_set(p)) * p.per * p.W;
  const uint64_t t_start = globaltimer();
  bool first = true;
  __syncthreads();
  while (s_done != mine) {
    // parallel poll: s_missing[w] = number of sources of block w not complete
    for (int i = threadIdx.x; i < p.per; i += blockDim.x) s_missing[i] = 0;
    __syncthreads();
    bool saw = false;
    for (int i = threadIdx.x; i < p.per * p.W; i += blockDim.x) {
      if (ld_relaxed_sys(flags + i) < call_expected(p)) atomicAdd(&s_missing[i / p.W], 1);
      else saw = true;
    }
    if (saw) fence_acq_rel_sys();
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint64_t done = s_done;
      int nb = 0, nq = 0;
      uint64_t taken = 0;
      for (int k = 0; k < p.per; ++k) {
        if (!((mine >> k) & 1) || ((done >> k) & 1)) continue;
        const int w = p.consume[k];
        if (!TDB_DEBUG_OK(status, w >= 0 && w < p.per, 51, k, w)) {
          taken |= 1ull << k;  // never read or written: the call reports the bad consumption table
          continue;
        }
        if (s_missing[w] == 0) {
          if (p.qmask[p.rank * p.per + w]) s_tq[nq++] = w;
          else s_bf[nb++] = w;
          taken |= 1ull << k;
        } else if (p.policy == 0) {
          break;  // ordered: stop at the first incomplete block
        }
      }
      if (nb + nq == 0 && globaltimer() - t_start > p.wait_ns) {
        record_status(status, kTimeoutPeerFlag, 40, p.rank, int(done));
        nb = -1;
      }
      s_nb = nb;
      s_nq = nq;
      const unsigned long long now = globaltimer();
      if (nb + nq > 0) {
        if (first && p.phases) p.phases[4 * (blockIdx.x % 1024) + 2] = now;
        if (p.timeline) {
          for (int i = 0; i < nb; ++i) atomicMin(&p.timeline[2 * s_bf[i]], now);
          for (int i = 0; i < nq; ++i) atomicMin(&p.timeline[2 * s_tq[i]], now);
        }
        s_done = done | taken;
      }
    }
    __syncthreads();
    const int nb = s_nb, nq = s_nq;
    if (nb < 0) return;
    if (nb + nq == 0) {
      __nanosleep(200);
      continue;
    }
    first = false;
    if (nb) consume_bf16_batch(p, s_bf, nb, part, nparts);
    for (int i = 0; i < nq; ++i) consume_block_taco(p, s_tq[i], part, nparts);
    if (p.timeline) {
      __syncthreads();
      if (threadIdx.x == 0) {
        const unsigned long long now = globaltimer();
        for (int i = 0; i < nb; ++i) atomicMax(&p.timeline[2 * s_bf[i] + 1], now);
        for (int i = 0; i < nq; ++i) atomicMax(&p.timeline[2 * s_tq[i] + 1], now);
      }
    }
    __syncthreads();
  }
}

// Shared memory: STAGES x (A + B tile) + the 4 x 32 x 128 staging of PushEpi:
// six stages of 128-wide tiles or four of 256-wide tiles.
template <int BN>
constexpr int kStagesFor = BN == 128 ? 6 : 4;

template <int BN, bool B_MN, bool QUANT>
__global__ void __launch_bounds__(gemm::kThreads, 1)
    gemm_rs_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int K,
                   gemm::TileOrder order, const __grid_constant__ Params p, int* status) {
  PushEpi<BN, QUANT> epi;
  epi.p = &p;
  epi.status = status;
  unsigned long long* ph = p.phases ? p.phases + 4 * blockIdx.x : nullptr;
  if (ph && threadIdx.x == 0) ph[0] = globaltimer();
  gemm::gemm_mainloop<BN, false, B_MN, PushEpi<BN, QUANT>, kStagesFor<BN>>(&tmA, &tmB, K, order, epi, status);
  if (threadIdx.x >= 64 && threadIdx.x < 192) epi.finish();
  signal_tiles(p, order);
  if (ph && threadIdx.x == 0) ph[1] = globaltimer();
  if (p.variant & 2) {
    consume_phase(p, status);
    if (ph && threadIdx.x == 0) ph[3] = globaltimer();
  }
}

// Consumer kernel: launched right after the producer on the same stream, at
// full occupancy.  It only waits for flags of blocks produced by other GPUs
// (the local producer kernel has completed), with bounded polling.
constexpr int kReduceThreads = 256;

// Per-call advance of the device call state (one thread): same arithmetic
// as the host-side Context.next_call, so both agree in eager mode.
__global__ void rs_advance_kernel(uint32_t* st, uint32_t signals) { advance_rs_state(st, signals); }

__global__ void __launch_bounds__(kReduceThreads, 2)
    rs_reduce_kernel(const __grid_constant__ Params p, int* status) {
  unsigned long long* ph = p.phases ? p.phases + 4 * (blockIdx.x % 1024) : nullptr;
  consume_phase(p, status);
  if (ph && threadIdx.x == 0) ph[3] = globaltimer();
}

// Producer for the selective arm's block-scaled FP8 mode: the tiles of the
// calibrated blocks (mx.on(m block)) run as kind::mxf8f6f4 MMAs on e4m3
// operands, the rest as bf16; every tile is pushed as bf16.
template <int BN>
constexpr int kMxStages = BN == 256 ? 3 : 5;

template <int BN>
__global__ void __launch_bounds__(gemm::kThreads, 1)
    gemm_rs_mx_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmA8, const __grid_constant__ CUtensorMap tmB8, int K,
                      gemm::TileOrder order, const __grid_constant__ Params p, const uint8_t* sfa, const uint8_t* sfb,
                      int a_blocks, int b_blocks, const uint8_t* mx_mask, int* status) {
  PushEpi<BN, false> epi;  // every block crosses as BF16
  epi.p = &p;
  epi.status = status;
  gemm::MxOperands mx{&tmA8, &tmB8, sfa, sfb, a_blocks, b_blocks, mx_mask};
  unsigned long long* ph = p.phases ? p.phases + 4 * blockIdx.x : nullptr;
  if (ph && threadIdx.x == 0) ph[0] = globaltimer();
  gemm::gemm_mainloop<BN, false, false, PushEpi<BN, false>, kMxStages<BN>, true>(&tmA, &tmB, K, order, epi, status,
                                                                                 &mx);
  if (threadIdx.x >= 64 && threadIdx.x < 192) epi.finish();
  signal_tiles(p, order);
  if (ph && threadIdx.x == 0) ph[1] = globaltimer();
  if (p.variant & 2) {
    consume_phase(p, status);
    if (ph && threadIdx.x == 0) ph[3] = globaltimer();
  }
}

static int launch_consumer(const Params& p, cudaStream_t stream);

// Producer launch: plain, or cooperative (all CTAs co-resident, grid capped
// at the resident count) when the consumer runs inside it (variant bit 1),
// in which case no separate consumer kernel follows.
template <class... KArgs, class... Args>
static int launch_producer(void (*kern)(KArgs...), int smem, int grid, const Params& p, cudaStream_t stream,
                           const char* what, Args&&... args) {
  const bool coop = (p.variant & 2) != 0;
  if (coop) {
    int nb = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, gemm::kThreads, smem);
    if (e != cudaSuccess || nb <= 0) return tdb_host::fail(int(e), "%s: no resident CTA possible", what);
    if (grid > nb * tdb_host::sm_count()) grid = nb * tdb_host::sm_count();
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(gemm::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = coop ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  tdb_host::launched(1);
  if (e != cudaSuccess) return tdb_host::fail(int(e), "%s: producer launch failed", what);
  return (coop || p.policy == kPolicyEpilogue) ? 0 : launch_consumer(p, stream);
}

template <int BN, bool B_MN, bool QUANT>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, int K, const gemm::TileOrder& order, const Params& p,
                  int grid, cudaStream_t stream) {
  using Cfg = gemm::Config<BN, kStagesFor<BN>>;
  constexpr int kSmem = Cfg::kSmemBytes + PushEpi<BN, QUANT>::kSmemBytes;
  static_assert(kSmem <= 227 * 1024, "fused GEMM-RS shared memory budget");
  auto kern = gemm_rs_kernel<BN, B_MN, QUANT>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return tdb_host::fail(int(e), "gemm_rs: cudaFuncSetAttribute failed");
    attr[dev & 63] = true;
  }
  int* status = tdb_host::status_ptr();
  return launch_producer(kern, kSmem, grid, p, stream, "gemm_rs", ta, tb, K, order, p, status);
}

template <int BN>
static int launch_mx(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta8, const CUtensorMap& tb8,
                     int K, const gemm::TileOrder& order, const Params& p, const uint8_t* sfa, const uint8_t* sfb,
                     const uint8_t* mx_mask, int grid, cudaStream_t stream) {
  using Cfg = gemm::Config<BN, kMxStages<BN>, true>;
  constexpr int kSmem = Cfg::kSmemBytes + PushEpi<BN, false>::kSmemBytes;
  static_assert(kSmem <= 227 * 1024, "fused FP8 GEMM-RS shared memory budget");
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_rs_mx_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return tdb_host::fail(int(e), "gemm_rs_mx: cudaFuncSetAttribute failed");
    attr[dev & 63] = true;
  }
  int* status = tdb_host::status_ptr();
  return launch_producer(gemm_rs_mx_kernel<BN>, kSmem, grid, p, stream, "gemm_rs_mx", ta, tb, ta8, tb8, K, order, p,
                         sfa, sfb, p.m / 128, p.N / 128, mx_mask, status);
}

static int launch_consumer(const Params& p, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  int* status = tdb_host::status_ptr();
  cudaError_t e;
  // Exactly the CTAs that are co-resident: every consumer CTA is polling and
  // reducing at the same time (a second wave would start only after the
  // first one drained, serialising the waits).
  static int per_sm[64] = {0};
  if (!per_sm[dev & 63]) {
    int nb = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, rs_reduce_kernel, kReduceThreads, 0);
    per_sm[dev & 63] = (e == cudaSuccess && nb > 0) ? nb : 1;
  }
  const int rgrid = per_sm[dev & 63] * tdb_host::grid_sms();
  rs_reduce_kernel<<<rgrid, kReduceThreads, 0, stream>>>(p, status);
  tdb_host::launched(1);
  e = cudaGetLastError();
  if (e != cudaSuccess) return tdb_host::fail(int(e), "gemm_rs: consumer launch failed");
  return 0;
}

int make_operand_map(CUtensorMap* map, const void* ptr, bool mn_major, int mn, int K, int64_t ld, int tile_mn) {
  if (!mn_major)
    return tdb_host::make_tmap_2d(map, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(K), uint64_t(mn),
                                  uint64_t(ld), gemm::BK, uint32_t(tile_mn), CU_TENSOR_MAP_SWIZZLE_128B);
  return tdb_host::make_tmap_2d(map, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, uint64_t(mn), uint64_t(K),
                                uint64_t(ld), 64, gemm::BK, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace rs
}  // namespace tdb

using namespace tdb;

// Fused GEMM + reduce-scatter.  A [m, K] (K contiguous, row stride lda);
// B = weight: [N, K] (b_mn = 0) or [K, N] (b_mn = 1), row stride ldb.
// tile_table: [num_tiles] production order (m_tile * (N / bn) + n_tile).
// quantized: nonzero when qmask selects any block for the TACO wire format
// (otherwise the producer is built without the encoder).
namespace tdb {
namespace rs {
// Default 0; see Params::variant.  Set with tdb_rs_set_variant (tuning).
static int g_variant = 0;

struct MxArgs {
  const void* a8;
  const void* sfa;
  const void* b8;
  const void* sfb;
  const uint8_t* mask;  // per 128-row m block of A
};

static int gemm_rs_impl(const void* A, int64_t lda, const void* B, int b_mn, int64_t ldb, int m, int N, int K, int bn,
                        const int* tile_table, const uint64_t* peers, int W, int rank, int chunk_rows,
                        uint64_t recv_off, uint64_t slot_bytes, uint64_t flags_off, int set, unsigned int expected,
                        const uint8_t* qmask, void* out, const void* bias, const void* residual, const int* consume,
                        int policy, unsigned long long* timeline, long long delay_cycles, int delay_mb, int delay_nb,
                        double wait_seconds, unsigned long long* phases, const uint32_t* call_state,
                        const MxArgs* mx, int quantized, void* stream) {
  if (!A || !B || !out || !tile_table || !peers || !qmask || !consume || W < 2 || W > rs::kMaxWorld || rank < 0 ||
      rank >= W)
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm_rs: bad pointers or ranks");
  if (bn != 128 && bn != 256) return tdb_host::fail(int(cudaErrorInvalidValue), "gemm_rs: bn must be 128 or 256");
  if (chunk_rows % rs::BM || m % (W * chunk_rows) || N % bn || N % 128 || K % 8)
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm_rs: shape (m=%d N=%d K=%d chunk=%d W=%d) unsupported", m,
                          N, K, chunk_rows, W);
  const int per = m / W / chunk_rows;
  if (per > 64) return tdb_host::fail(int(cudaErrorInvalidValue), "gemm_rs: at most 64 blocks per destination");
  if (slot_bytes < uint64_t(chunk_rows) * N * 2)
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm_rs: receive slot too small");
  if (delay_cycles < 0 || delay_cycles > 100000000ll)
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm_rs: diagnostic delay out of range");
  if (policy < 0 || policy > 2) return tdb_host::fail(int(cudaErrorInvalidValue), "gemm_rs: policy must be 0, 1 or 2");
  if (policy == rs::kPolicyEpilogue && quantized)
    return tdb_host::fail(int(cudaErrorInvalidValue), "gemm_rs: the epilogue-reduction policy sends BF16 only");
  if (policy == rs::kPolicyEpilogue) {
    const uint64_t fine = 2ull * per * (chunk_rows / rs::BM) * (N / bn) * 4 * W * 4;
    if (!call_state || W > rs::kMaxWorldEpi || fine > rs::kFineFlagsBytes || flags_off + rs::kFineFlagsOff + fine > recv_off)
      return tdb_host::fail(int(cudaErrorInvalidValue),
                            "gemm_rs: the epilogue-reduction policy needs a device call state, W <= 8 and %llu flag "
                            "bytes", (unsigned long long)fine);
  }
  CUtensorMap ta, tb;
  int rc = rs::make_operand_map(&ta, A, false, m, K, lda, rs::BM);
  if (rc) return rc;
  rc = rs::make_operand_map(&tb, B, b_mn != 0, N, K, ldb, bn);
  if (rc) return rc;
  gemm::TileOrder order;
  order.num_m = m / rs::BM;
  order.num_n = N / bn;
  order.group_m = 1;
  order.table = tile_table;
  order.num_tiles = order.num_m * order.num_n;
  rs::Params p;
  p.peers = peers;
  p.W = W;
  p.rank = rank;
  p.m = m;
  p.N = N;
  p.chunk_rows = chunk_rows;
  p.per = per;
  p.recv_off = recv_off;
  p.slot_bytes = slot_bytes;
  p.flags_off = flags_off;
  p.set = set;
  p.expected = expected;
  p.qmask = qmask;
  p.out = static_cast<uint16_t*>(out);
  p.bias = static_cast<const uint16_t*>(bias);
  p.residual = static_cast<const uint16_t*>(residual);
  p.consume = consume;
  p.policy = policy;
  p.timeline = timeline;
  p.delay_cycles = delay_cycles;
  p.delay_mb = delay_mb;
  p.delay_nb = delay_nb;
  p.wait_ns = uint64_t(wait_seconds * 1e9);
  p.phases = phases;
  p.call_state = call_state;
  // Producers of TACO blocks are built without the bulk-push path, so their
  // calls drop that bit: the tiles then travel (and are signalled and read
  // back by the reducer) as lane stores in row-major layout.
  p.variant = policy == kPolicyEpilogue ? 0 : (quantized ? (g_variant & ~kVariantBulk) : g_variant);
  const int sms = tdb_host::grid_sms();
  const int grid = order.num_tiles < sms ? order.num_tiles : sms;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (mx) {
    if (b_mn || K % 128 || !mx->a8 || !mx->b8 || !mx->sfa || !mx->sfb || !mx->mask ||
        (reinterpret_cast<uintptr_t>(mx->sfa) | reinterpret_cast<uintptr_t>(mx->sfb)) % 16)
      return tdb_host::fail(int(cudaErrorInvalidValue), "gemm_rs_mx: needs a K-major B, K %% 128, aligned scales");
    CUtensorMap ta8, tb8;
    rc = gemm::make_fp8_map(&ta8, mx->a8, m, K, rs::BM);
    if (rc) return rc;
    rc = gemm::make_fp8_map(&tb8, mx->b8, N, K, bn);
    if (rc) return rc;
    const uint8_t* sa = static_cast<const uint8_t*>(mx->sfa);
    const uint8_t* sb = static_cast<const uint8_t*>(mx->sfb);
    return bn == 256 ? rs::launch_mx<256>(ta, tb, ta8, tb8, K, order, p, sa, sb, mx->mask, grid, s)
                     : rs::launch_mx<128>(ta, tb, ta8, tb8, K, order, p, sa, sb, mx->mask, grid, s);
  }
  if (quantized) {
    if (bn == 256) return b_mn ? rs::launch<256, true, true>(ta, tb, K, order, p, grid, s)
                               : rs::launch<256, false, true>(ta, tb, K, order, p, grid, s);
    return b_mn ? rs::launch<128, true, true>(ta, tb, K, order, p, grid, s)
                : rs::launch<128, false, true>(ta, tb, K, order, p, grid, s);
  }
  if (bn == 256) return b_mn ? rs::launch<256, true, false>(ta, tb, K, order, p, grid, s)
                             : rs::launch<256, false, false>(ta, tb, K, order, p, grid, s);
  return b_mn ? rs::launch<128, true, false>(ta, tb, K, order, p, grid, s)
              : rs::launch<128, false, false>(ta, tb, K, order, p, grid, s);
}
}  // namespace rs
}  // namespace tdb

TDB_API int tdb_gemm_rs(const void* A, int64_t lda, const void* B, int b_mn, int64_t ldb, int m, int N, int K,
                        int bn, const int* tile_table, const uint64_t* peers, int W, int rank, int chunk_rows,
                        uint64_t recv_off, uint64_t slot_bytes, uint64_t flags_off, int set, unsigned int expected,
                        const uint8_t* qmask, void* out, const void* bias, const void* residual, const int* consume,
                        int policy, unsigned long long* timeline, long long delay_cycles, int delay_mb, int delay_nb,
                        double wait_seconds, unsigned long long* phases, const uint32_t* call_state, int quantized,
                        void* stream) {
  return rs::gemm_rs_impl(A, lda, B, b_mn, ldb, m, N, K, bn, tile_table, peers, W, rank, chunk_rows, recv_off,
                          slot_bytes, flags_off, set, expected, qmask, out, bias, residual, consume, policy, timeline,
                          delay_cycles, delay_mb, delay_nb, wait_seconds, phases, call_state, nullptr, quantized != 0,
                          stream);
}

// tdb_gemm_rs whose tiles in the m blocks flagged by mx_mask run as
// block-scaled FP8 MMAs on a8 / b8 (e4m3 copies of A and B, scale atoms
// sfa / sfb from tdb_mx_quantize).  B K-major, K % 128 == 0.
TDB_API int tdb_gemm_rs_mx(const void* A, int64_t lda, const void* B, int b_mn, int64_t ldb, int m, int N, int K,
                           int bn, const int* tile_table, const uint64_t* peers, int W, int rank, int chunk_rows,
                           uint64_t recv_off, uint64_t slot_bytes, uint64_t flags_off, int set, unsigned int expected,
                           const uint8_t* qmask, void* out, const void* bias, const void* residual, const int* consume,
                           int policy, unsigned long long* timeline, long long delay_cycles, int delay_mb,
                           int delay_nb, double wait_seconds, unsigned long long* phases, const uint32_t* call_state,
                           const void* a8, const void* sfa, const void* b8, const void* sfb, const uint8_t* mx_mask,
                           void* stream) {
  const rs::MxArgs mx{a8, sfa, b8, sfb, mx_mask};
  return rs::gemm_rs_impl(A, lda, B, b_mn, ldb, m, N, K, bn, tile_table, peers, W, rank, chunk_rows, recv_off,
                          slot_bytes, flags_off, set, expected, qmask, out, bias, residual, consume, policy, timeline,
                          delay_cycles, delay_mb, delay_nb, wait_seconds, phases, call_state, &mx, 0, stream);
}

// Select the fused GEMM-RS signalling / consumer variant of the following
// calls (bit 0 per-tile signals, bit 1 consumer inside the producer kernel,
// bit 2 bulk TMA pushes with per-tile signals after completion);
// returns the previous value.  Every rank must use the same variant.
TDB_API int tdb_rs_set_variant(int variant) {
  const int old = rs::g_variant;
  if (variant >= 0 && variant <= 7) rs::g_variant = variant;
  return old;
}

// Advance the device call state {set, expected, epoch, target0, target1}
// (uint32 x 5, zero-initialised) before a call that passes it to tdb_gemm_rs.
TDB_API int tdb_rs_advance(unsigned int* call_state, unsigned int signals, void* stream) {
  if (!call_state) return tdb_host::fail(int(cudaErrorInvalidValue), "rs_advance: null state");
  rs::rs_advance_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(call_state, signals);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

// Number of counter increments one (block, source) receives per call.
TDB_API int tdb_gemm_rs_signals_per_block(int chunk_rows, int N, int bn) { return (chunk_rows / 128) * (N / bn) * 4; }
