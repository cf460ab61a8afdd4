// Sparse vocabulary-parallel embedding exchange over NVLink peer memory.
//
// Reference parity: python/flux_dcu/model.py:236-249 (masked lookup into the
// local vocabulary shard, then SumScatter -- a reduce-scatter of the dense
// [m, h] lookup -- to the sequence-parallel rows) and the backward of that
// pair (an all-gather of the row gradients, then the masked table gradient).
//
// Every token's embedding row lives on exactly one rank (the owner of its
// vocabulary shard), so the dense reduce-scatter adds one nonzero row to W-1
// zero rows.  Here the owner instead writes the row straight into the
// receive buffer of the rank that holds that sequence position -- the same
// bits the reduce-scatter produces -- so a rank sends about m*h*2/W bytes
// instead of (W-1)/W of m*h*2.  In the backward each rank sends the gradient
// of each of its rows only to the owner of that row's token, which then runs
// the ordinary deterministic table backward on those rows.
//
// Region of every rank's symmetric heap (heap_off): flags [2 directions][W]
// uint32, two completion counters, then the forward slots [2 parities][ml, H]
// bf16 and the backward slots [2 parities][W * ml, H] bf16.  Per direction a
// device state {epoch, parity} is advanced before each call (graph replays
// see fresh epochs).  One call per direction is: advance, push (one CTA per
// row; the last CTA to finish fences and publishes the epoch to every rank),
// then collect: wait (bounded) for every rank's publish and copy the
// received rows into the caller's buffer (forward: plus positions).  A rank
// rewrites a slot two calls later, after it has seen every peer's publish of
// the call between.
#include "call_state.cuh"
#include "common.cuh"

namespace tdb {
namespace embx {

constexpr int kThreads = 256;
constexpr uint64_t kHeaderBytes = 256;  // flags[2][W] (W <= 8) and counters[2]

struct Params {
  const uint64_t* peers;
  uint64_t heap_off;
  const uint32_t* state;  // {epoch, parity} of this direction
  int W, rank;
  int64_t ml, H;          // rows per rank, hidden
  int dir;                // 0 forward, 1 backward
  uint64_t wait_ns;
};

__device__ __forceinline__ uint8_t* region(const Params& p, int r) {
  return reinterpret_cast<uint8_t*>(p.peers[r] + p.heap_off);
}
__device__ __forceinline__ uint32_t* flags(const Params& p, int r) {
  return reinterpret_cast<uint32_t*>(region(p, r)) + p.dir * 8;
}
__device__ __forceinline__ uint32_t* counter(const Params& p) {
  return reinterpret_cast<uint32_t*>(region(p, p.rank)) + 16 + p.dir;
}
__device__ __forceinline__ uint16_t* fwd_slot(const Params& p, int r, uint32_t parity) {
  return reinterpret_cast<uint16_t*>(region(p, r) + kHeaderBytes + uint64_t(parity) * p.ml * p.H * 2);
}
__device__ __forceinline__ uint16_t* bwd_slot(const Params& p, int r, uint32_t parity) {
  return reinterpret_cast<uint16_t*>(region(p, r) + kHeaderBytes + 2ull * p.ml * p.H * 2 +
                                     uint64_t(parity) * p.W * p.ml * p.H * 2);
}

__global__ void advance_kernel(uint32_t* state) { advance_ag_state(state); }

// The CTA that finishes last makes every CTA's peer stores visible, then
// publishes this call's epoch to every rank (this one included).
__device__ __forceinline__ void publish_when_last(const Params& p) {
  __threadfence_system();  // this thread's peer stores, before the CTA's arrival
  __syncthreads();
  if (threadIdx.x != 0) return;
  const uint32_t done = atomicAdd(counter(p), 1u);
  if (done != gridDim.x - 1) return;
  *counter(p) = 0;  // the next call's kernel starts after this one ends
  __threadfence_system();
  const uint32_t epoch = __ldg(p.state);
  for (int r = 0; r < p.W; ++r) st_release_sys(flags(p, r) + p.rank, epoch);
}

__device__ __forceinline__ void copy_row(uint16_t* dst, const uint16_t* src, int64_t H) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (int64_t c = threadIdx.x; c < H / 8; c += blockDim.x) d[c] = s[c];
}

// Forward: CTA g handles global row g; if its token is in this rank's shard
// the table row goes to row g % ml of rank g / ml's forward slot.
__global__ void __launch_bounds__(kThreads)
    push_fwd_kernel(Params p, const int64_t* __restrict__ tokens, const uint16_t* __restrict__ table, int64_t start,
                    int64_t local_vocab) {
  const int64_t g = blockIdx.x;
  const int64_t t = tokens[g] - start;
  if (t >= 0 && t < local_vocab) {
    const int dest = int(g / p.ml);
    copy_row(fwd_slot(p, dest, __ldg(p.state + 1)) + (g % p.ml) * p.H, table + t * p.H, p.H);
  }
  publish_when_last(p);
}

// Backward: CTA r handles this rank's row r (global row rank * ml + r) and
// sends its gradient to the owner of the token's shard, at the global row.
__global__ void __launch_bounds__(kThreads)
    push_bwd_kernel(Params p, const int64_t* __restrict__ tokens, const uint16_t* __restrict__ dy, int64_t ld,
                    int64_t local_vocab) {
  const int64_t r = blockIdx.x;
  const int64_t g = int64_t(p.rank) * p.ml + r;
  const int owner = int(tokens[g] / local_vocab);
  if (owner >= 0 && owner < p.W) copy_row(bwd_slot(p, owner, __ldg(p.state + 1)) + g * p.H, dy + r * ld, p.H);
  publish_when_last(p);
}

// Wait (bounded) until every rank published this call's epoch.  Returns
// false on expiry (status recorded).
__device__ __forceinline__ bool wait_all(const Params& p, int* status, int where) {
  const uint32_t epoch = __ldg(p.state);
  const uint32_t* f = flags(p, p.rank);
  for (int s = 0; s < p.W; ++s) {
    if (int32_t(ld_acquire_sys(f + s) - epoch) >= 0) continue;
    const uint64_t t0 = globaltimer();
    while (int32_t(ld_acquire_sys(f + s) - epoch) < 0) {
      if (globaltimer() - t0 > p.wait_ns) {
        record_status(status, kTimeoutPeerFlag, where, s, int(epoch));
        return false;
      }
    }
  }
  return true;
}

// Forward collect: every CTA waits for the publishes, then writes its row of
// x = received embedding row + learned position (row stride H).  The slot
// parity is read on the device, so a captured graph stays correct.
__global__ void __launch_bounds__(kThreads)
    collect_fwd_kernel(Params p, const uint16_t* __restrict__ pos, int64_t pos_offset, int seq, uint16_t* x,
                       int* status) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = wait_all(p, status, 320) ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  const int64_t r = blockIdx.x;
  const uint4* rs = reinterpret_cast<const uint4*>(fwd_slot(p, p.rank, __ldg(p.state + 1)) + r * p.H);
  const uint4* ps = reinterpret_cast<const uint4*>(pos + ((r + pos_offset) % seq) * p.H);
  uint4* xs = reinterpret_cast<uint4*>(x + r * p.H);
  for (int64_t c = threadIdx.x; c < p.H / 8; c += blockDim.x) {
    const uint4 a = __ldcg(rs + c), b = ps[c];
    const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, bb[4] = {b.x, b.y, b.z, b.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = pack_bf16x2(bf16_bits_to_float(aa[j] & 0xffff) + bf16_bits_to_float(bb[j] & 0xffff),
                         bf16_bits_to_float(aa[j] >> 16) + bf16_bits_to_float(bb[j] >> 16));
    xs[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Backward collect: CTA g waits for the publishes, then copies global row g
// into out if this rank owns its token (the only rows the table backward
// reads); other rows of out are left as they are.
__global__ void __launch_bounds__(kThreads)
    collect_bwd_kernel(Params p, const int64_t* __restrict__ tokens, int64_t start, int64_t local_vocab, uint16_t* out,
                       int* status) {
  const int64_t g = blockIdx.x;
  const int64_t t = tokens[g] - start;
  if (t < 0 || t >= local_vocab) return;
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = wait_all(p, status, 321) ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  const uint4* src = reinterpret_cast<const uint4*>(bwd_slot(p, p.rank, __ldg(p.state + 1)) + g * p.H);
  uint4* dst = reinterpret_cast<uint4*>(out + g * p.H);
  for (int64_t c = threadIdx.x; c < p.H / 8; c += blockDim.x) dst[c] = __ldcg(src + c);
}

static Params make(const unsigned long long* peers, unsigned long long heap_off, unsigned int* state, int W, int rank,
                   long long ml, long long H, int dir, double wait_seconds) {
  Params p;
  p.peers = reinterpret_cast<const uint64_t*>(peers);
  p.heap_off = heap_off;
  p.state = state;
  p.W = W;
  p.rank = rank;
  p.ml = ml;
  p.H = H;
  p.dir = dir;
  p.wait_ns = uint64_t(wait_seconds * 1e9);
  return p;
}

static int check(const void* a, const void* b, const unsigned long long* peers, unsigned int* state, int W, int rank,
                 long long ml, long long H, unsigned long long heap_off, double wait_seconds) {
  if (!a || !b || !peers || !state || W < 2 || W > 8 || rank < 0 || rank >= W || ml <= 0 || H <= 0 || H % 8 ||
      heap_off % 256 || !(wait_seconds > 0) || (reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) % 16)
    return tdb_host::fail(int(cudaErrorInvalidValue), "embedding exchange: bad arguments");
  return 0;
}

}  // namespace embx
}  // namespace tdb

using namespace tdb;

// Bytes of one exchange region (rows per rank ml, hidden H, W ranks).
TDB_API long long tdb_embx_region_bytes(long long ml, long long H, int W) {
  return (long long)embx::kHeaderBytes + 2ll * ml * H * 2 + 2ll * W * ml * H * 2;
}

// Forward: x [ml, H] (this rank's sequence-parallel rows) = the embedding
// rows of tokens[rank*ml : (rank+1)*ml] + positions.  tokens: all W*ml ids.
TDB_API int tdb_embx_forward(const int64_t* tokens, const void* table, long long start, long long local_vocab,
                             const void* pos, long long pos_offset, int seq, void* x, const unsigned long long* peers,
                             int W, int rank, long long ml, long long H, unsigned long long heap_off,
                             unsigned int* state, double wait_seconds, void* stream) {
  int rc = embx::check(tokens, table, peers, state, W, rank, ml, H, heap_off, wait_seconds);
  if (rc) return rc;
  if (!x || reinterpret_cast<uintptr_t>(x) % 16)
    return tdb_host::fail(int(cudaErrorInvalidValue), "embedding exchange: x must be 16-byte aligned");
  if (!pos || seq <= 0) return tdb_host::fail(int(cudaErrorInvalidValue), "embedding exchange: positions required");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  embx::Params p = embx::make(peers, heap_off, state, W, rank, ml, H, 0, wait_seconds);
  embx::advance_kernel<<<1, 1, 0, s>>>(state);
  embx::push_fwd_kernel<<<unsigned(W * ml), embx::kThreads, 0, s>>>(p, tokens, static_cast<const uint16_t*>(table),
                                                                     start, local_vocab);
  embx::collect_fwd_kernel<<<unsigned(ml), embx::kThreads, 0, s>>>(p, static_cast<const uint16_t*>(pos), pos_offset,
                                                                     seq, static_cast<uint16_t*>(x),
                                                                     tdb_host::status_ptr());
  tdb_host::launched(3);
  return int(cudaGetLastError());
}

// Backward: sends each of this rank's gradient rows dy [ml, H] (row stride
// ld) to the owner of its token; afterwards out [W*ml, H] holds, at every
// global row whose token lies in [start, start + local_vocab) (this rank's
// shard), that row's gradient -- the rows the table backward reads; its
// other rows are not written.
TDB_API int tdb_embx_backward(const int64_t* tokens, const void* dy, long long ld, long long start,
                              long long local_vocab, void* out, const unsigned long long* peers, int W, int rank,
                              long long ml, long long H, unsigned long long heap_off, unsigned int* state,
                              double wait_seconds, void* stream) {
  int rc = embx::check(tokens, dy, peers, state, W, rank, ml, H, heap_off, wait_seconds);
  if (rc) return rc;
  if (local_vocab <= 0 || ld < H || ld % 8 || !out || reinterpret_cast<uintptr_t>(out) % 16)
    return tdb_host::fail(int(cudaErrorInvalidValue), "embedding exchange: bad vocabulary, row stride or output");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  embx::Params p = embx::make(peers, heap_off, state, W, rank, ml, H, 1, wait_seconds);
  embx::advance_kernel<<<1, 1, 0, s>>>(state);
  embx::push_bwd_kernel<<<unsigned(ml), embx::kThreads, 0, s>>>(p, tokens, static_cast<const uint16_t*>(dy), ld,
                                                                 local_vocab);
  embx::collect_bwd_kernel<<<unsigned(W * ml), embx::kThreads, 0, s>>>(p, tokens, start, local_vocab,
                                                                         static_cast<uint16_t*>(out),
                                                                         tdb_host::status_ptr());
  tdb_host::launched(3);
  return int(cudaGetLastError());
}
