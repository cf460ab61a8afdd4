// Fused GEMM -> reduce-scatter over NVLink peer memory (the five-arm operator).
//
//   out[rows of this rank] = bias + residual + sum_{s=0..W-1} (A_s @ W_s^T)[rows of this rank]
//
// One persistent kernel per call, two phases:
//
// 1. Produce.  The tcgen05 mainloop (gemm.cuh) computes the full [m, N]
//    partial product tile by tile in the order of a device tile table (the
//    arm's production schedule: contiguous, the common interleave, or the
//    calibrated arrival order).  The epilogue stores each 128 x BN tile straight
//    into the destination rank's receive slot [source = this rank] through its
//    peer pointer: BF16, or -- for blocks selected by the TACO mask and remote
//    destinations -- H128/E4M3 encoded in registers (one thread owns one row's
//    128-column group), so only compressed bytes cross NVLink.  After its
//    stores each epilogue warp fences (system scope) and adds 1 to the
//    destination's (block, source) counter with a release-ordered remote
//    atomic.
// 2. Consume.  Each CTA then reduces this rank's output blocks: it waits until
//    all W sources of a block are complete (bounded acquire polling), decodes
//    TACO sources in registers (one warp per H128 group) and adds the sources
//    in rank order 0..W-1 with BF16 rounding after every addition, then adds
//    the residual and the bias.  Consumer policy "ordered" walks blocks in
//    schedule order with all CTAs; "per-lane ready" (arrival arms) splits the
//    CTAs into two lanes (lane = within % 2) and each lane consumes whichever
//    of its blocks is complete first.  Summation order never depends on
//    arrival, so arms that only reorder are bitwise identical.
//
// Buffers live in the symmetric heap (symm.cu): receive slots
// [2 sets][W sources][per blocks][chunk_rows * N * 2 bytes] and counters
// [2 sets][per][W] (uint32, monotonically increasing; the host passes the
// value that means "complete" for this call).  Calls alternate sets, which
// makes reuse safe: a rank can only start call k+2 after every rank finished
// consuming call k.  The launch is cooperative so all CTAs are co-resident.
// Every wait is bounded by %globaltimer and reports through the status word.
//
// Reference parity: python/flux_dcu/runtime.py:84-268 (FluxDCU: schedule,
// TACO encode of remote blocks, two lanes, ordered vs per-lane-ready
// consumers, ordered BF16 source reduction, final join) and
// src/taco/codec.hip:78-148 (codec math, ordered reduce).
#include <climits>

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
};

__device__ __forceinline__ uint8_t* slot_ptr(const Params& p, int rank_of_heap, int source, int within) {
  return reinterpret_cast<uint8_t*>(p.peers[rank_of_heap] + p.recv_off +
                                    (uint64_t(p.set * p.W + source) * p.per + within) * p.slot_bytes);
}

__device__ __forceinline__ uint32_t* flag_ptr(const Params& p, int rank_of_heap, int within, int source) {
  return reinterpret_cast<uint32_t*>(p.peers[rank_of_heap] + p.flags_off +
                                     (uint64_t(p.set * p.per + within) * p.W + source) * 4);
}

__device__ __forceinline__ void red_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
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
#pragma unroll
  for (int w = 0; w < 32; ++w) {
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float f = isfinite(x[4 * w + j]) ? x[4 * w + j] : 0.0f;
      y[j] = fminf(fmaxf(f / q, -448.0f), 448.0f);
    }
    words[w] = uint32_t(taco::e4m3x2(y[0], y[1])) | (uint32_t(taco::e4m3x2(y[2], y[3])) << 16);
  }
}

template <int BN>
struct PushEpi {
  const Params* p;
  int* status;
  // per-tile state
  int within, dest, row0;
  bool quant;
  uint8_t* slot;
  float grp[128];

  __device__ __forceinline__ void tile_begin(int mb, int nb) {
    const int m0 = mb * BM;
    const int physical = m0 / p->chunk_rows;
    dest = physical / p->per;
    within = physical % p->per;
    row0 = m0 - physical * p->chunk_rows;
    quant = p->qmask[physical] != 0 && dest != p->rank;
    slot = slot_ptr(*p, dest, p->rank, within);
  }

  __device__ __forceinline__ void chunk(int row, int col, int c, const uint32_t (&r)[32]) {
    const int rib = row0 + (row % BM);  // row inside the block
    const int N = p->N;
    if (!quant) {
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(slot) + int64_t(rib) * N + col);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 w;
        w.x = pack_bf16x2(__uint_as_float(r[8 * i + 0]), __uint_as_float(r[8 * i + 1]));
        w.y = pack_bf16x2(__uint_as_float(r[8 * i + 2]), __uint_as_float(r[8 * i + 3]));
        w.z = pack_bf16x2(__uint_as_float(r[8 * i + 4]), __uint_as_float(r[8 * i + 5]));
        w.w = pack_bf16x2(__uint_as_float(r[8 * i + 6]), __uint_as_float(r[8 * i + 7]));
        dst[i] = w;
      }
      return;
    }
    // TACO: gather the 128-column group (4 chunks) in registers, BF16 rounded.
#pragma unroll
    for (int j = 0; j < 32; ++j)
      grp[(c & 3) * 32 + j] = bf16_bits_to_float(float_to_bf16_bits(__uint_as_float(r[j])));
    if ((c & 3) == 3) {
      uint32_t words[32];
      float q, a;
      encode_group_thread(grp, words, q, a);
      const int gcol = col - 96;
      const int64_t elements = int64_t(p->chunk_rows) * N;
      const int64_t groups = elements / 128;
      const int64_t g = (int64_t(rib) * N + gcol) / 128;
      uint4* pay = reinterpret_cast<uint4*>(slot + int64_t(rib) * N + gcol);
#pragma unroll
      for (int i = 0; i < 8; ++i) pay[i] = make_uint4(words[4 * i], words[4 * i + 1], words[4 * i + 2], words[4 * i + 3]);
      float* scales = reinterpret_cast<float*>(slot + elements);
      scales[g] = q;
      scales[groups + g] = a;
    }
  }

  __device__ __forceinline__ void tile_end(int mb, int nb, int /*quarter*/, int lane) {
    __threadfence_system();
    __syncwarp();
    if (lane == 0) {
      if (p->delay_cycles > 0 && mb == p->delay_mb && nb == p->delay_nb) {
        const long long t0 = clock64();
        while (clock64() - t0 < p->delay_cycles) {
        }
      }
      red_release_sys(flag_ptr(*p, dest, within, p->rank), 1u);
    }
  }
};

// Block readiness: all W sources delivered (acquire).
__device__ __forceinline__ bool block_ready(const Params& p, int within) {
  for (int s = 0; s < p.W; ++s)
    if (ld_acquire_sys(flag_ptr(p, p.rank, within, s)) < p.expected) return false;
  return true;
}

__device__ void consume_block(const Params& p, int within, int part, int nparts) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const int gpr = p.N / 128;
  const int items = p.chunk_rows * gpr;
  const int physical = p.rank * p.per + within;
  const bool quant = p.qmask[physical] != 0;
  const int64_t elements = int64_t(p.chunk_rows) * p.N;
  const int64_t groups = elements / 128;
  for (int it = part * nw + warp; it < items; it += nparts * nw) {
    const int rho = it / gpr, g = it % gpr;
    const int64_t e0 = int64_t(rho) * p.N + g * 128 + lane * 4;  // element offset in block
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < p.W; ++s) {
      const uint8_t* slot = slot_ptr(p, p.rank, s, within);
      float v[4];
      if (quant && s != p.rank) {
        // Peer-written data: read at L2 (.cg) so no stale L1 line can be hit.
        const uint32_t word = __ldcg(reinterpret_cast<const unsigned int*>(slot + e0));
        const float* scales = reinterpret_cast<const float*>(slot + elements);
        const int64_t gi = int64_t(rho) * gpr + g;
        taco::decode_group_warp(word, __ldcg(scales + gi), __ldcg(scales + groups + gi), lane, v);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = bf16_bits_to_float(float_to_bf16_bits(v[j]));
      } else {
        const uint2 w = __ldcg(reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(slot) + e0));
        v[0] = bf16_bits_to_float(w.x & 0xffff);
        v[1] = bf16_bits_to_float(w.x >> 16);
        v[2] = bf16_bits_to_float(w.y & 0xffff);
        v[3] = bf16_bits_to_float(w.y >> 16);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = bf16_bits_to_float(float_to_bf16_bits(acc[j] + v[j]));
    }
    const int64_t orow = int64_t(within) * p.chunk_rows + rho;
    const int64_t o = orow * p.N + g * 128 + lane * 4;
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
    ow.x = uint32_t(float_to_bf16_bits(acc[0])) | (uint32_t(float_to_bf16_bits(acc[1])) << 16);
    ow.y = uint32_t(float_to_bf16_bits(acc[2])) | (uint32_t(float_to_bf16_bits(acc[3])) << 16);
    *reinterpret_cast<uint2*>(p.out + o) = ow;
  }
}

__device__ void consume_phase(const Params& p, int* status) {
  __shared__ int pick;
  // Partition: ordered = all CTAs; per-lane = CTAs of parity l consume lane-l blocks.
  int part = blockIdx.x, nparts = gridDim.x, lane_id = -1;
  if (p.policy == 1) {
    lane_id = blockIdx.x & 1;
    part = blockIdx.x >> 1;
    nparts = (gridDim.x + 1 - lane_id) >> 1;
  }
  uint64_t done = 0;
  int remaining = 0;
  for (int k = 0; k < p.per; ++k)
    if (lane_id < 0 || (p.consume[k] % 2) == lane_id) ++remaining;
  const uint64_t t_start = globaltimer();
  while (remaining > 0) {
    if (threadIdx.x == 0) {
      int chosen = -1;
      while (chosen < 0) {
        for (int k = 0; k < p.per; ++k) {
          const int w = p.consume[k];
          if ((done >> k) & 1) continue;
          if (lane_id >= 0 && (w % 2) != lane_id) continue;
          if (block_ready(p, w)) { chosen = k; break; }
          if (p.policy == 0) break;  // ordered: only the next block in order
        }
        if (chosen < 0 && globaltimer() - t_start > p.wait_ns) {
          record_status(status, kTimeoutPeerFlag, 40, p.rank, int(done));
          chosen = -2;
        }
      }
      pick = chosen;
      if (chosen >= 0 && p.timeline) atomicMin(&p.timeline[2 * p.consume[chosen]], (unsigned long long)globaltimer());
    }
    __syncthreads();
    const int k = pick;
    __syncthreads();
    if (k < 0) return;
    consume_block(p, p.consume[k], part, nparts);
    done |= 1ull << k;
    --remaining;
    if (p.timeline) {
      __syncthreads();
      if (threadIdx.x == 0) atomicMax(&p.timeline[2 * p.consume[k] + 1], (unsigned long long)globaltimer());
    }
  }
}

template <int BN, bool B_MN>
__global__ void __launch_bounds__(gemm::kThreads, 1)
    gemm_rs_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int K,
                   gemm::TileOrder order, const __grid_constant__ Params p, int* status) {
  PushEpi<BN> epi;
  epi.p = &p;
  epi.status = status;
  gemm::gemm_mainloop<BN, false, B_MN>(&tmA, &tmB, K, order, epi, status);
  consume_phase(p, status);
}

template <int BN, bool B_MN>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, int K, const gemm::TileOrder& order, const Params& p,
                  int grid, cudaStream_t stream) {
  using Cfg = gemm::Config<BN>;
  auto kern = gemm_rs_kernel<BN, B_MN>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return tdb_host::fail(int(e), "gemm_rs: cudaFuncSetAttribute failed");
    attr[dev & 63] = true;
  }
  int* status = tdb_host::status_ptr();
  CUtensorMap a = ta, b = tb;
  int k = K;
  gemm::TileOrder o = order;
  Params pp = p;
  void* args[] = {&a, &b, &k, &o, &pp, &status};
  cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(gemm::kThreads),
                                              args, Cfg::kSmemBytes, stream);
  if (e != cudaSuccess) return tdb_host::fail(int(e), "gemm_rs: cooperative launch failed (grid %d)", grid);
  tdb_host::launched(1);
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
TDB_API int tdb_gemm_rs(const void* A, int64_t lda, const void* B, int b_mn, int64_t ldb, int m, int N, int K,
                        int bn, const int* tile_table, const uint64_t* peers, int W, int rank, int chunk_rows,
                        uint64_t recv_off, uint64_t slot_bytes, uint64_t flags_off, int set, unsigned int expected,
                        const uint8_t* qmask, void* out, const void* bias, const void* residual, const int* consume,
                        int policy, unsigned long long* timeline, long long delay_cycles, int delay_mb, int delay_nb,
                        double wait_seconds, void* stream) {
  if (!A || !B || !out || !tile_table || !peers || !qmask || !consume || W < 2 || rank < 0 || rank >= W)
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
  const int sms = tdb_host::sm_count();
  const int grid = order.num_tiles < sms ? (order.num_tiles > 2 ? order.num_tiles : 2) : sms;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bn == 256) return b_mn ? rs::launch<256, true>(ta, tb, K, order, p, grid, s)
                             : rs::launch<256, false>(ta, tb, K, order, p, grid, s);
  return b_mn ? rs::launch<128, true>(ta, tb, K, order, p, grid, s) : rs::launch<128, false>(ta, tb, K, order, p, grid, s);
}

// Number of counter increments one (block, source) receives per call.
TDB_API int tdb_gemm_rs_signals_per_block(int chunk_rows, int N, int bn) { return (chunk_rows / 128) * (N / bn) * 4; }
