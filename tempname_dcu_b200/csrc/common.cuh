// Shared device helpers for the sm_100a kernels of tempname_dcu_b200.
//
// Everything here is hand-written PTX or plain CUDA for Blackwell (sm_100a):
// mbarrier pipelines, TMA tile loads (never with cluster multicast), tcgen05
// MMA / TMEM helpers and a bounded-wait discipline.  Every spin in this code
// base is bounded by %globaltimer: on expiry the waiting thread records an
// error code in the library-wide status word and the kernel unwinds normally
// (TMEM freed, no trap), so a lost flag never hangs the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "tdb.h"  // prototypes of every exported entry point (checked against the definitions)

#define TDB_API extern "C" __attribute__((visibility("default")))

namespace tdb {

// ---------------------------------------------------------------------------
// Status word.  One per process image of the library (per device it is used
// on).  Codes are small integers; the first error wins.
// ---------------------------------------------------------------------------
enum StatusCode : int {
  kOk = 0,
  kTimeoutPipeline = 1,   // an mbarrier wait inside a GEMM pipeline expired
  kTimeoutPeerFlag = 2,   // a cross-rank flag never arrived
  kTimeoutLocal = 3,      // an intra-kernel flag never arrived
  kBadArgument = 4,
  kDebugCheck = 5,        // a TDB_DEBUG index check failed (the access was skipped)
};

// The status word lives in runtime.cu; kernels receive its device address
// (layout [code, where, detail0, detail1]) as an argument.
__device__ __forceinline__ void record_status(int* status, int code, int where, int d0 = 0, int d1 = 0) {
  if (status == nullptr) return;
  if (atomicCAS(&status[0], 0, code) == 0) {
    status[1] = where;
    status[2] = d0;
    status[3] = d1;
  }
}

// Debug builds (-DTDB_DEBUG, the TDB_DEBUG=1 library): TDB_DEBUG_OK(status,
// cond, where, a, b) evaluates `cond`, records a failure (code kDebugCheck,
// location `where`, details a, b) and returns it, so the caller skips the
// access instead of faulting.  Release builds compile it to `true`.
#ifdef TDB_DEBUG
#define TDB_DEBUG_OK(status, cond, where, a, b) \
  ((cond) ? true : (::tdb::record_status((status), ::tdb::kDebugCheck, (where), int(a), int(b)), false))
#else
#define TDB_DEBUG_OK(status, cond, where, a, b) true
#endif

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Default bound for in-kernel waits: 2 seconds of wall time.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// ---------------------------------------------------------------------------
// Shared-memory address helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records the status)
// when the limit expires; callers then abandon their loop.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - start > kWaitLimitNs) {
      record_status(status, kTimeoutPipeline, where);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// Cross-CTA / cross-GPU flags: release stores and adds, acquire and relaxed
// loads, at system scope (peer GPUs) or GPU scope (this GPU's CTAs).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_gpu(uint32_t* addr, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) -- plain loads into this CTA's shared memory.
// No TMA or bulk load with .multicast::cluster exists in this code base (the
// only multicast is the 2-CTA MMA's tcgen05.commit to both CTAs' barriers).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 / TMEM
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_f16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Signal an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// row (lane_base + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Shared-memory matrix descriptor (tcgen05 "version 1" format), 128-byte
// swizzle.  Addresses and offsets are encoded in 16-byte units.
//   bits [0,14)  start address >> 4
//   bits [16,30) leading-dimension byte offset >> 4
//   bits [32,46) stride-dimension byte offset >> 4
//   bits [46,48) descriptor version (1 on sm_100)
//   bits [61,64) layout: 2 = SWIZZLE_128B
__host__ __device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
//   [4,6) D format (1 = f32); [7,10) A fmt (1 = bf16); [10,13) B fmt (1 = bf16)
//   [15] A major (1 = MN); [16] B major (1 = MN); [17,23) N>>3; [24,29) M>>4
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Block-scaled FP8 (kind::mxf8f6f4): e4m3 A/B, one ue8m0 scale per 32 K values.
// ---------------------------------------------------------------------------

// Untiled bulk copy global -> this CTA's shared memory (16-byte aligned
// addresses, size a multiple of 16), completing on an mbarrier.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Descriptor of an unswizzled K-major shared-memory matrix: 8-row core
// matrices of 16-byte rows, `sbo_bytes` apart along M/N; `lbo_bytes` apart
// along K (unused when K spans one 16-byte core column).
__host__ __device__ __forceinline__ uint64_t smem_desc_plain(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;  // version 1, layout 0 = no swizzle
  return d;
}

// 32 rows x 128 bits of shared memory -> TMEM lanes [0,32) x 4 columns,
// replicated into all four 32-lane sub-partitions (the scale-factor layout
// the block-scaled MMA reads for M = 128).
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Instruction descriptor of kind::mxf8f6f4 with e4m3 A/B (format 0), K-major
// operands, ue8m0 scales (bit 23) and the dense K = 32 shape (bit 31 = 0):
//   [4,6) B scale byte; [7,10) A fmt; [10,13) B fmt; [17,23) N>>3;
//   [24,29) M>>4; [29,31) A scale byte.
__host__ __device__ constexpr uint32_t idesc_mxf8(int m, int n) {
  return (static_cast<uint32_t>(n >> 3) << 17) | (1u << 23) | (static_cast<uint32_t>(m >> 4) << 24);
}

// D[tmem] (+)= (A * 2^sfa) (B * 2^sfb)^T for one K = 32 step.  sf_byte picks
// the scale byte (the 32-value K block inside the scale column word); it goes
// both into the descriptor and into bits [30,32) of the scale addresses.
__device__ __forceinline__ void umma_mxf8_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t sfa_col, uint32_t sfb_col, uint32_t sf_byte,
                                             uint32_t accumulate) {
  const uint32_t id = idesc | (sf_byte << 29) | (sf_byte << 4);
  const uint32_t ta = sfa_col | (sf_byte << 30), tb = sfb_col | (sf_byte << 30);
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(id), "r"(accumulate), "r"(ta), "r"(tb));
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t.reg .b32 r;\n\t"
      "elect.sync r|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// Numeric helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_float(uint16_t x) { return __uint_as_float(uint32_t(x) << 16); }

// Round-to-nearest-even fp32 -> bf16 bits.  On the device this is the
// single hardware cvt.rn.bf16.f32; the host version rounds the bit pattern
// (identical for every finite input; a NaN stays a NaN in both).
__host__ __device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
#ifdef __CUDA_ARCH__
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
#else
  uint32_t bits;
  memcpy(&bits, &f, 4);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return uint16_t((bits >> 16) | 0x0040u);
  bits += 0x7fffu + ((bits >> 16) & 1u);
  return uint16_t(bits >> 16);
#endif
}

// acc <- bf16(acc + x), the ordered-reduction step, in registers.
__device__ __forceinline__ float bf16_add(float acc, float x) {
  return __bfloat162float(__float2bfloat16_rn(acc + x));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

__device__ __forceinline__ float gelu_erf_grad(float x) {
  const float cdf = 0.5f * (1.0f + erff(x * 0.70710678118654752f));
  const float pdf = 0.3989422804014327f * __expf(-0.5f * x * x);
  return cdf + x * pdf;
}

}  // namespace tdb

// Host-side helpers shared by the launch wrappers.
namespace tdb_host {
// Thread-local last error text for the C ABI.
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
// Count kernels launched by the library (read with tdb_launch_count).
void launched(int n);
// Device address of the status word on the current device (cached per device).
int* status_ptr();
// SM count of the current device (cached).
int sm_count();
// SMs that persistent GEMM-shaped kernels (plain, fused collective) launched
// from this host thread may occupy: sm_count(), or less under
// tdb_set_grid_limit (so that a kernel on another stream can run beside them).
int grid_sms();
}  // namespace tdb_host
