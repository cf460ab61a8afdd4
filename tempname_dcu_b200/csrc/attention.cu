// Causal flash attention (head_dim 128), forward and deterministic backward,
// reading Q/K/V straight out of the fused QKV GEMM output.
//
// Reference parity: python/flux_dcu/model.py:250-256 (SDPA, causal, no
// dropout, per-rank local heads).  Layout: qkv is [tokens, 3, Hl, 128]
// (row stride `ld` elements; token t of micro-batch b is row b*seq + t);
// the output is [tokens, Hl, 128], the layout the attention-out projection
// consumes, so no permute/contiguous copies are made.
//
// Forward: FlashAttention-2 schedule.  CTA = 128 query rows of one (batch,
// head), 8 warps x 16 rows, key/value tiles of 64 double-buffered with
// cp.async into XOR-swizzled shared memory, bf16 mma.sync m16n8k16 with fp32
// accumulation, online softmax in exp2 form, log-sum-exp saved for backward.
// Backward (no atomics, bitwise deterministic):
//   pre:  Dsum[i] = rowsum(dO[i] * O[i])
//   dkdv: CTA = 64 keys (4 warps x 16 keys); loops over query tiles from the
//         diagonal, recomputing P^T; accumulates dV = P^T dO, dK = dS^T Q.
//   dq:   CTA = 64 queries; loops over key tiles up to the diagonal;
//         accumulates dQ = dS K.
#include "common.cuh"

namespace tdb {
namespace attn {

constexpr int D = 128;
constexpr int kRowBytes = D * 2;  // 256 bytes per row in shared memory

// --------------------------------------------------------------------------
// PTX wrappers
// --------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of (row, col) in a swizzled [rows][128] bf16 tile (col % 8 == 0).
__device__ __forceinline__ uint32_t swz(int row, int col) {
  return uint32_t(row * kRowBytes + ((((col >> 3) ^ (row & 7))) << 4));
}

// Copy `rows` x 128 bf16 from global (row stride ld elements) into a swizzled tile.
template <int ROWS, int THREADS>
__device__ __forceinline__ void load_tile(uint32_t sbase, const uint16_t* g, int64_t ld, int valid_rows) {
  constexpr int kChunks = ROWS * 16;
#pragma unroll
  for (int i = 0; i < kChunks / THREADS; ++i) {
    const int idx = threadIdx.x + i * THREADS;
    const int row = idx >> 4, ch = idx & 15;
    const int r = row < valid_rows ? row : valid_rows - 1;
    cp_async16(sbase + swz(row, ch * 8), g + int64_t(r) * ld + ch * 8);
  }
}

// A fragment (16 x 16) at (row0, col0) of a swizzled row-major tile.
__device__ __forceinline__ void lda(uint32_t base, int row0, int col0, uint32_t (&a)[4]) {
  const int l = threadIdx.x & 31;
  ldsm_x4(base + swz(row0 + (l & 15), col0 + (l >> 4) * 8), a[0], a[1], a[2], a[3]);
}

// Two B fragments (k 16 x n 8, n-tiles n0 and n0+8) from a tile stored [n][k].
__device__ __forceinline__ void ldb_nk(uint32_t base, int n0, int k0, uint32_t (&b)[4]) {
  const int l = threadIdx.x & 31;
  ldsm_x4(base + swz(n0 + (l & 7) + ((l >> 4) << 3), k0 + ((l >> 3) & 1) * 8), b[0], b[1], b[2], b[3]);
}

// Two B fragments (k 16 x n 8, n-tiles n0 and n0+8) from a tile stored [k][n].
__device__ __forceinline__ void ldb_kn(uint32_t base, int k0, int n0, uint32_t (&b)[4]) {
  const int l = threadIdx.x & 31;
  ldsm_x4_t(base + swz(k0 + (l & 7) + ((l >> 3) & 1) * 8, n0 + (l >> 4) * 8), b[0], b[1], b[2], b[3]);
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) { return pack_bf16x2(lo, hi); }

constexpr float kLog2e = 1.4426950408889634f;

// --------------------------------------------------------------------------
// Forward
// --------------------------------------------------------------------------
constexpr int FWD_BM = 128, FWD_BN = 64, FWD_THREADS = 256;

__global__ void __launch_bounds__(FWD_THREADS, 1)
    fwd_kernel(const uint16_t* __restrict__ qkv, int64_t ld, uint16_t* __restrict__ out, int64_t ld_out,
               float* __restrict__ lse, int seq, int Hl, float scale) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + FWD_BM * kRowBytes;
  const uint32_t sV0 = sK0 + 2 * FWD_BN * kRowBytes;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t tok0 = int64_t(b) * seq;
  const uint16_t* Qg = qkv + (tok0 + int64_t(qb) * FWD_BM) * ld + h * D;
  const uint16_t* Kg = qkv + tok0 * ld + (Hl + h) * D;
  const uint16_t* Vg = qkv + tok0 * ld + (2 * Hl + h) * D;
  const int q_valid = min(FWD_BM, seq - qb * FWD_BM);

  const int last_key = min(seq - 1, qb * FWD_BM + FWD_BM - 1);
  const int nkb = last_key / FWD_BN + 1;

  load_tile<FWD_BM, FWD_THREADS>(sQ, Qg, ld, q_valid);
  load_tile<FWD_BN, FWD_THREADS>(sK0, Kg, ld, min(FWD_BN, seq));
  load_tile<FWD_BN, FWD_THREADS>(sV0, Vg, ld, min(FWD_BN, seq));
  cp_commit();

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = scale * kLog2e;
  uint32_t qf[8][4];
  const int qrow0 = qb * FWD_BM + warp * 16 + g;  // absolute query index of c0/c1
  const int qrow1 = qrow0 + 8;

  for (int kb = 0; kb < nkb; ++kb) {
    if (kb + 1 < nkb) {
      const int nb = (kb + 1) & 1;
      const int kv_valid = min(FWD_BN, seq - (kb + 1) * FWD_BN);
      load_tile<FWD_BN, FWD_THREADS>(sK0 + nb * FWD_BN * kRowBytes, Kg + int64_t(kb + 1) * FWD_BN * ld, ld, kv_valid);
      load_tile<FWD_BN, FWD_THREADS>(sV0 + nb * FWD_BN * kRowBytes, Vg + int64_t(kb + 1) * FWD_BN * ld, ld, kv_valid);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) lda(sQ, warp * 16, k * 16, qf[k]);
    }
    const uint32_t sK = sK0 + (kb & 1) * FWD_BN * kRowBytes;
    const uint32_t sV = sV0 + (kb & 1) * FWD_BN * kRowBytes;
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        uint32_t bb[4];
        ldb_nk(sK, n * 8, k * 16, bb);
        mma16816(s[n], qf[k], bb[0], bb[1]);
        mma16816(s[n + 1], qf[k], bb[2], bb[3]);
      }
    }
    // causal mask + scale
    const int key0 = kb * FWD_BN;
    const bool need_mask = key0 + FWD_BN - 1 > qb * FWD_BM;
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int key = key0 + n * 8 + 2 * t + j;
        float v0 = s[n][j] * sl2, v1 = s[n][2 + j] * sl2;
        if (need_mask || key >= seq) {
          if (key > qrow0 || key >= seq) v0 = -INFINITY;
          if (key > qrow1 || key >= seq) v1 = -INFINITY;
        }
        s[n][j] = v0;
        s[n][2 + j] = v1;
        mx0 = fmaxf(mx0, v0);
        mx1 = fmaxf(mx1, v1);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float a0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - mx0);
    const float a1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pf[4][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = mx0 == -INFINITY ? 0.f : exp2f(s[n][0] - mx0);
      const float p1 = mx0 == -INFINITY ? 0.f : exp2f(s[n][1] - mx0);
      const float p2 = mx1 == -INFINITY ? 0.f : exp2f(s[n][2] - mx1);
      const float p3 = mx1 == -INFINITY ? 0.f : exp2f(s[n][3] - mx1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      const int kk = n >> 1;
      if ((n & 1) == 0) {
        pf[kk][0] = pack2(p0, p1);
        pf[kk][1] = pack2(p2, p3);
      } else {
        pf[kk][2] = pack2(p0, p1);
        pf[kk][3] = pack2(p2, p3);
      }
    }
    l0 = l0 * a0 + rs0;
    l1 = l1 * a1 + rs1;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= a0;
      o[i][1] *= a0;
      o[i][2] *= a1;
      o[i][3] *= a1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int n = 0; n < 16; n += 2) {
        uint32_t bb[4];
        ldb_kn(sV, kk * 16, n * 8, bb);
        mma16816(o[n], pf[kk], bb[0], bb[1]);
        mma16816(o[n + 1], pf[kk], bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int r0 = warp * 16 + g, r1 = r0 + 8;
  uint16_t* O0 = out + (tok0 + int64_t(qb) * FWD_BM + r0) * ld_out + h * D;
  uint16_t* O1 = out + (tok0 + int64_t(qb) * FWD_BM + r1) * ld_out + h * D;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int col = n * 8 + 2 * t;
    if (r0 < q_valid) *reinterpret_cast<uint32_t*>(O0 + col) = pack2(o[n][0] * inv0, o[n][1] * inv0);
    if (r1 < q_valid) *reinterpret_cast<uint32_t*>(O1 + col) = pack2(o[n][2] * inv1, o[n][3] * inv1);
  }
  if (t == 0) {
    float* L = lse + (int64_t(b) * Hl + h) * seq + qb * FWD_BM;
    // log-sum-exp in log2 units of the scaled scores: m + log2(l)
    if (r0 < q_valid) L[r0] = m0 + log2f(l0);
    if (r1 < q_valid) L[r1] = m1 + log2f(l1);
  }
}

// --------------------------------------------------------------------------
// Backward
// --------------------------------------------------------------------------
__global__ void bwd_pre_kernel(const uint16_t* __restrict__ out, int64_t ld_out, const uint16_t* __restrict__ dout,
                               int64_t ld_dout, float* __restrict__ dsum, int seq, int Hl, int total_rows) {
  // 16 lanes per (token, head) row of 128 values: one 16-byte load of O and
  // of dO per lane, then a 16-lane butterfly.
  const int64_t w = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 4;
  const int sub = threadIdx.x & 15;
  const bool live = w < int64_t(total_rows) * Hl;
  float s = 0.f;
  int64_t tok = 0;
  int h = 0;
  if (live) {
    tok = w / Hl;
    h = int(w % Hl);
    const uint4 a = *reinterpret_cast<const uint4*>(out + tok * ld_out + h * D + sub * 8);
    const uint4 c = *reinterpret_cast<const uint4*>(dout + tok * ld_dout + h * D + sub * 8);
    const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, cc[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      s += bf16_bits_to_float(aa[j] & 0xffff) * bf16_bits_to_float(cc[j] & 0xffff) +
           bf16_bits_to_float(aa[j] >> 16) * bf16_bits_to_float(cc[j] >> 16);
  }
#pragma unroll
  for (int o = 8; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (live && sub == 0) {
    const int64_t b = tok / seq, i = tok % seq;
    dsum[(b * Hl + h) * seq + i] = s;
  }
}

constexpr int BWD_B = 64, BWD_THREADS = 128;

// dK, dV for 64 keys. Shared: K, V (64 rows each), Q, dO (64 rows each, double
// buffered), LSE / Dsum of the query tile.
__global__ void __launch_bounds__(BWD_THREADS)
    bwd_dkdv_kernel(const uint16_t* __restrict__ qkv, int64_t ld, const uint16_t* __restrict__ dout, int64_t ld_dout,
                    const float* __restrict__ lse, const float* __restrict__ dsum, uint16_t* __restrict__ dqkv,
                    int64_t ld_dqkv, int seq, int Hl, float scale) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BWD_B * kRowBytes;
  const uint32_t sQ0 = sV + BWD_B * kRowBytes;            // 2 buffers
  const uint32_t sO0 = sQ0 + 2 * BWD_B * kRowBytes;       // 2 buffers (dO)
  float* sL = reinterpret_cast<float*>(smem + 6 * BWD_B * kRowBytes);  // [2][64]
  float* sD = sL + 2 * BWD_B;                                          // [2][64]
  const int kb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t tok0 = int64_t(b) * seq;
  const uint16_t* Qg = qkv + tok0 * ld + h * D;
  const uint16_t* Kg = qkv + (tok0 + int64_t(kb) * BWD_B) * ld + (Hl + h) * D;
  const uint16_t* Vg = qkv + (tok0 + int64_t(kb) * BWD_B) * ld + (2 * Hl + h) * D;
  const uint16_t* dOg = dout + tok0 * ld_dout + h * D;
  const float* Lg = lse + (int64_t(b) * Hl + h) * seq;
  const float* Dg = dsum + (int64_t(b) * Hl + h) * seq;
  const int k_valid = min(BWD_B, seq - kb * BWD_B);
  const float sl2 = scale * kLog2e;

  load_tile<BWD_B, BWD_THREADS>(sK, Kg, ld, k_valid);
  load_tile<BWD_B, BWD_THREADS>(sV, Vg, ld, k_valid);
  const int nqb = (seq + BWD_B - 1) / BWD_B;
  auto load_q = [&](int qb, int buf) {
    const int qv = min(BWD_B, seq - qb * BWD_B);
    load_tile<BWD_B, BWD_THREADS>(sQ0 + buf * BWD_B * kRowBytes, Qg + int64_t(qb) * BWD_B * ld, ld, qv);
    load_tile<BWD_B, BWD_THREADS>(sO0 + buf * BWD_B * kRowBytes, dOg + int64_t(qb) * BWD_B * ld_dout, ld_dout, qv);
    if (threadIdx.x < BWD_B) {
      const int i = qb * BWD_B + threadIdx.x;
      sL[buf * BWD_B + threadIdx.x] = i < seq ? Lg[i] : 0.f;
      sD[buf * BWD_B + threadIdx.x] = i < seq ? Dg[i] : 0.f;
    }
  };
  load_q(kb, 0);
  cp_commit();

  float dk[16][4], dv[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) dk[i][j] = dv[i][j] = 0.f;
  const int key_r0 = kb * BWD_B + warp * 16 + g;  // absolute key of c0/c1 rows
  const int key_r1 = key_r0 + 8;

  for (int qb = kb; qb < nqb; ++qb) {
    const int buf = (qb - kb) & 1;
    if (qb + 1 < nqb) {
      __syncthreads();  // sL/sD of the other buffer are free
      load_q(qb + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint32_t sQ = sQ0 + buf * BWD_B * kRowBytes;
    const uint32_t sO = sO0 + buf * BWD_B * kRowBytes;
    const float* L = sL + buf * BWD_B;
    const float* Ds = sD + buf * BWD_B;
    // S^T = K Q^T  (16 keys x 64 queries per warp)
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = dp[i][j] = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint32_t a[4];
      lda(sK, warp * 16, k * 16, a);
      uint32_t av[4];
      lda(sV, warp * 16, k * 16, av);
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        uint32_t bb[4];
        ldb_nk(sQ, n * 8, k * 16, bb);
        mma16816(s[n], a, bb[0], bb[1]);
        mma16816(s[n + 1], a, bb[2], bb[3]);
        uint32_t bo[4];
        ldb_nk(sO, n * 8, k * 16, bo);
        mma16816(dp[n], av, bo[0], bo[1]);
        mma16816(dp[n + 1], av, bo[2], bo[3]);
      }
    }
    // P^T and dS^T
    uint32_t pf[4][4], dsf[4][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      float p[4], ds[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int qi = qb * BWD_B + n * 8 + 2 * t + (j & 1);
        const int key = (j < 2) ? key_r0 : key_r1;
        const bool valid = qi >= key && qi < seq && key < seq;
        const float lq = L[n * 8 + 2 * t + (j & 1)];
        p[j] = valid ? exp2f(s[n][j] * sl2 - lq) : 0.f;
        ds[j] = p[j] * (dp[n][j] - Ds[n * 8 + 2 * t + (j & 1)]);
      }
      const int kk = n >> 1;
      if ((n & 1) == 0) {
        pf[kk][0] = pack2(p[0], p[1]);
        pf[kk][1] = pack2(p[2], p[3]);
        dsf[kk][0] = pack2(ds[0], ds[1]);
        dsf[kk][1] = pack2(ds[2], ds[3]);
      } else {
        pf[kk][2] = pack2(p[0], p[1]);
        pf[kk][3] = pack2(p[2], p[3]);
        dsf[kk][2] = pack2(ds[0], ds[1]);
        dsf[kk][3] = pack2(ds[2], ds[3]);
      }
    }
    // dV += P^T dO ; dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int n = 0; n < 16; n += 2) {
        uint32_t bo[4];
        ldb_kn(sO, kk * 16, n * 8, bo);
        mma16816(dv[n], pf[kk], bo[0], bo[1]);
        mma16816(dv[n + 1], pf[kk], bo[2], bo[3]);
        uint32_t bq[4];
        ldb_kn(sQ, kk * 16, n * 8, bq);
        mma16816(dk[n], dsf[kk], bq[0], bq[1]);
        mma16816(dk[n + 1], dsf[kk], bq[2], bq[3]);
      }
    }
  }
  // write dK (scaled) and dV into the dqkv buffer
  const int r0 = warp * 16 + g, r1 = r0 + 8;
  uint16_t* dK0 = dqkv + (tok0 + int64_t(kb) * BWD_B + r0) * ld_dqkv + (Hl + h) * D;
  uint16_t* dK1 = dqkv + (tok0 + int64_t(kb) * BWD_B + r1) * ld_dqkv + (Hl + h) * D;
  uint16_t* dV0 = dqkv + (tok0 + int64_t(kb) * BWD_B + r0) * ld_dqkv + (2 * Hl + h) * D;
  uint16_t* dV1 = dqkv + (tok0 + int64_t(kb) * BWD_B + r1) * ld_dqkv + (2 * Hl + h) * D;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int col = n * 8 + 2 * t;
    if (r0 < k_valid) {
      *reinterpret_cast<uint32_t*>(dK0 + col) = pack2(dk[n][0] * scale, dk[n][1] * scale);
      *reinterpret_cast<uint32_t*>(dV0 + col) = pack2(dv[n][0], dv[n][1]);
    }
    if (r1 < k_valid) {
      *reinterpret_cast<uint32_t*>(dK1 + col) = pack2(dk[n][2] * scale, dk[n][3] * scale);
      *reinterpret_cast<uint32_t*>(dV1 + col) = pack2(dv[n][2], dv[n][3]);
    }
  }
}

// dQ for 64 queries: loops over key tiles 0..diagonal.
__global__ void __launch_bounds__(BWD_THREADS)
    bwd_dq_kernel(const uint16_t* __restrict__ qkv, int64_t ld, const uint16_t* __restrict__ dout, int64_t ld_dout,
                  const float* __restrict__ lse, const float* __restrict__ dsum, uint16_t* __restrict__ dqkv,
                  int64_t ld_dqkv, int seq, int Hl, float scale) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sO = sQ + BWD_B * kRowBytes;
  const uint32_t sK0 = sO + BWD_B * kRowBytes;       // 2 buffers
  const uint32_t sV0 = sK0 + 2 * BWD_B * kRowBytes;  // 2 buffers
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t tok0 = int64_t(b) * seq;
  const uint16_t* Qg = qkv + (tok0 + int64_t(qb) * BWD_B) * ld + h * D;
  const uint16_t* Kg = qkv + tok0 * ld + (Hl + h) * D;
  const uint16_t* Vg = qkv + tok0 * ld + (2 * Hl + h) * D;
  const uint16_t* dOg = dout + (tok0 + int64_t(qb) * BWD_B) * ld_dout + h * D;
  const int q_valid = min(BWD_B, seq - qb * BWD_B);
  const float sl2 = scale * kLog2e;
  const int q_r0 = qb * BWD_B + warp * 16 + g, q_r1 = q_r0 + 8;
  const float* Lg = lse + (int64_t(b) * Hl + h) * seq;
  const float* Dg = dsum + (int64_t(b) * Hl + h) * seq;
  const float lq0 = q_r0 < seq ? Lg[q_r0] : 0.f, lq1 = q_r1 < seq ? Lg[q_r1] : 0.f;
  const float dq0s = q_r0 < seq ? Dg[q_r0] : 0.f, dq1s = q_r1 < seq ? Dg[q_r1] : 0.f;

  load_tile<BWD_B, BWD_THREADS>(sQ, Qg, ld, q_valid);
  load_tile<BWD_B, BWD_THREADS>(sO, dOg, ld_dout, q_valid);
  load_tile<BWD_B, BWD_THREADS>(sK0, Kg, ld, min(BWD_B, seq));
  load_tile<BWD_B, BWD_THREADS>(sV0, Vg, ld, min(BWD_B, seq));
  cp_commit();

  float dq[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  uint32_t qf[8][4], of[8][4];
  const int nkb = qb + 1;
  for (int kb = 0; kb < nkb; ++kb) {
    if (kb + 1 < nkb) {
      const int nb = (kb + 1) & 1;
      const int kv = min(BWD_B, seq - (kb + 1) * BWD_B);
      load_tile<BWD_B, BWD_THREADS>(sK0 + nb * BWD_B * kRowBytes, Kg + int64_t(kb + 1) * BWD_B * ld, ld, kv);
      load_tile<BWD_B, BWD_THREADS>(sV0 + nb * BWD_B * kRowBytes, Vg + int64_t(kb + 1) * BWD_B * ld, ld, kv);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        lda(sQ, warp * 16, k * 16, qf[k]);
        lda(sO, warp * 16, k * 16, of[k]);
      }
    }
    const uint32_t sK = sK0 + (kb & 1) * BWD_B * kRowBytes;
    const uint32_t sV = sV0 + (kb & 1) * BWD_B * kRowBytes;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = dp[i][j] = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        uint32_t bk[4], bv[4];
        ldb_nk(sK, n * 8, k * 16, bk);
        mma16816(s[n], qf[k], bk[0], bk[1]);
        mma16816(s[n + 1], qf[k], bk[2], bk[3]);
        ldb_nk(sV, n * 8, k * 16, bv);
        mma16816(dp[n], of[k], bv[0], bv[1]);
        mma16816(dp[n + 1], of[k], bv[2], bv[3]);
      }
    }
    uint32_t dsf[4][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      float ds[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = kb * BWD_B + n * 8 + 2 * t + (j & 1);
        const int qi = j < 2 ? q_r0 : q_r1;
        const bool valid = key <= qi && key < seq && qi < seq;
        const float p = valid ? exp2f(s[n][j] * sl2 - (j < 2 ? lq0 : lq1)) : 0.f;
        ds[j] = p * (dp[n][j] - (j < 2 ? dq0s : dq1s));
      }
      const int kk = n >> 1;
      if ((n & 1) == 0) {
        dsf[kk][0] = pack2(ds[0], ds[1]);
        dsf[kk][1] = pack2(ds[2], ds[3]);
      } else {
        dsf[kk][2] = pack2(ds[0], ds[1]);
        dsf[kk][3] = pack2(ds[2], ds[3]);
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int n = 0; n < 16; n += 2) {
        uint32_t bk[4];
        ldb_kn(sK, kk * 16, n * 8, bk);
        mma16816(dq[n], dsf[kk], bk[0], bk[1]);
        mma16816(dq[n + 1], dsf[kk], bk[2], bk[3]);
      }
    }
    __syncthreads();
  }
  const int r0 = warp * 16 + g, r1 = r0 + 8;
  uint16_t* dQ0 = dqkv + (tok0 + int64_t(qb) * BWD_B + r0) * ld_dqkv + h * D;
  uint16_t* dQ1 = dqkv + (tok0 + int64_t(qb) * BWD_B + r1) * ld_dqkv + h * D;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int col = n * 8 + 2 * t;
    if (r0 < q_valid) *reinterpret_cast<uint32_t*>(dQ0 + col) = pack2(dq[n][0] * scale, dq[n][1] * scale);
    if (r1 < q_valid) *reinterpret_cast<uint32_t*>(dQ1 + col) = pack2(dq[n][2] * scale, dq[n][3] * scale);
  }
}

constexpr int kFwdSmem = (FWD_BM + 4 * FWD_BN) * kRowBytes;
constexpr int kDkdvSmem = 6 * BWD_B * kRowBytes + 4 * BWD_B * 4;
constexpr int kDqSmem = 6 * BWD_B * kRowBytes;

}  // namespace attn
}  // namespace tdb

using namespace tdb::attn;

static int set_smem(const void* fn, int bytes) {
  return int(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

// qkv [mb*seq, ld] with Q|K|V column blocks of Hl*128; out [mb*seq, ld_out];
// lse [mb, Hl, seq] fp32.
TDB_API int tdb_attn_fwd(const void* qkv, int64_t ld, void* out, int64_t ld_out, float* lse, int mb, int seq, int Hl,
                         float scale, void* stream) {
  if (!qkv || !out || !lse || mb <= 0 || seq <= 0 || Hl <= 0 || ld % 8 || ld_out % 8)
    return tdb_host::fail(int(cudaErrorInvalidValue), "attention fwd: bad arguments");
  static bool init = false;
  if (!init) {
    int rc = set_smem(reinterpret_cast<const void*>(fwd_kernel), kFwdSmem);
    if (rc) return rc;
    init = true;
  }
  dim3 grid((seq + FWD_BM - 1) / FWD_BM, Hl, mb);
  fwd_kernel<<<grid, FWD_THREADS, kFwdSmem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(qkv), ld, static_cast<uint16_t*>(out), ld_out, lse, seq, Hl, scale);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

// dsum: scratch [mb, Hl, seq] fp32.  dqkv [mb*seq, ld_dqkv] receives dQ|dK|dV.
// Dsum[b, h, i] = sum_d dO[i, h, d] * O[i, h, d]  (one warp per (token, head)).
TDB_API int tdb_attn_bwd_pre(const void* out, int64_t ld_out, const void* dout, int64_t ld_dout, float* dsum, int mb,
                             int seq, int Hl, void* stream) {
  if (!out || !dout || !dsum || mb <= 0 || seq <= 0 || Hl <= 0 || ld_out % 8 || ld_dout % 8 ||
      (reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(dout)) % 16)
    return tdb_host::fail(int(cudaErrorInvalidValue), "attention bwd pre: bad arguments (16-byte aligned rows needed)");
  const int rows = mb * seq;
  const int64_t groups = int64_t(rows) * Hl;  // 16 threads each
  tdb::attn::bwd_pre_kernel<<<unsigned((groups * 16 + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(out), ld_out, static_cast<const uint16_t*>(dout), ld_dout, dsum, seq, Hl, rows);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}

TDB_API int tdb_attn_bwd(const void* qkv, int64_t ld, const void* out, int64_t ld_out, const void* dout,
                         int64_t ld_dout, const float* lse, float* dsum, void* dqkv, int64_t ld_dqkv, int mb, int seq,
                         int Hl, float scale, void* stream) {
  if (!qkv || !out || !dout || !lse || !dsum || !dqkv || seq <= 0 || Hl <= 0 || mb <= 0)
    return tdb_host::fail(int(cudaErrorInvalidValue), "attention bwd: bad arguments");
  static bool init = false;
  if (!init) {
    int rc = set_smem(reinterpret_cast<const void*>(bwd_dkdv_kernel), kDkdvSmem);
    if (rc) return rc;
    rc = set_smem(reinterpret_cast<const void*>(bwd_dq_kernel), kDqSmem);
    if (rc) return rc;
    init = true;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = tdb_attn_bwd_pre(out, ld_out, dout, ld_dout, dsum, mb, seq, Hl, stream);
  if (rc) return rc;
  dim3 grid((seq + BWD_B - 1) / BWD_B, Hl, mb);
  bwd_dkdv_kernel<<<grid, BWD_THREADS, kDkdvSmem, s>>>(static_cast<const uint16_t*>(qkv), ld,
                                                       static_cast<const uint16_t*>(dout), ld_dout, lse, dsum,
                                                       static_cast<uint16_t*>(dqkv), ld_dqkv, seq, Hl, scale);
  tdb_host::launched(1);
  bwd_dq_kernel<<<grid, BWD_THREADS, kDqSmem, s>>>(static_cast<const uint16_t*>(qkv), ld,
                                                   static_cast<const uint16_t*>(dout), ld_dout, lse, dsum,
                                                   static_cast<uint16_t*>(dqkv), ld_dqkv, seq, Hl, scale);
  tdb_host::launched(1);
  return int(cudaGetLastError());
}
