// Epilogues of the tcgen05 GEMMs (shared by gemm.cu and ag_gemm.cu):
// parameter block, register epilogue (PlainEpi) and the shared-memory + TMA
// bulk-store epilogues for fp32 (AccF32TmaEpi) and bf16 (TmaBf16Epi) outputs.
#pragma once
#include <type_traits>

#include "gemm.cuh"

namespace tdb {
namespace gemm {

enum EpiMode : int {
  kStore = 0,         // C(bf16) = alpha * acc
  kBias = 1,          // C(bf16) = acc + bias[n]
  kBiasGelu = 2,      // Z = bf16(acc + bias[n]) -> aux_out;  C(bf16) = gelu(Z)
  kGeluBwd = 3,       // C(bf16) = acc * gelu'(aux[m,n])
  kAccF32 = 4,        // C(fp32) = acc + beta * C
  kBiasResidual = 5,  // C(bf16) = acc + bias[n] + aux[m,n]
  // internal: kAccF32 with beta 0 or 1 and a 16-byte aligned C, written
  // through shared memory by TMA bulk stores / bulk reduce-adds
  kAccF32Tma = 6,
  // internal: kTmaBase + m = bf16 mode m (0, 1, 2, 3, 5) with TMA bulk stores
  kTmaBase = 8,
};

struct alignas(64) EpiParams {
  CUtensorMap tmC;    // TMA epilogues: C (fp32 box {32, 32} or bf16 box {64, 32}), 128B swizzle
  CUtensorMap tmAux;  // TMA bf16 epilogue of kBiasGelu: the saved pre-activation (aux_out)
  void* C;
  int64_t ldc;
  int M, N;
  const uint16_t* bias;
  const uint16_t* aux;
  int64_t ld_aux;
  uint16_t* aux_out;
  float alpha, beta;
};

__device__ __forceinline__ void load_bf16x32(const uint16_t* p, float (&v)[32]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 w = q[i];
    const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[8 * i + 2 * j] = bf16_bits_to_float(a[j] & 0xffff);
      v[8 * i + 2 * j + 1] = bf16_bits_to_float(a[j] >> 16);
    }
  }
}

__device__ __forceinline__ void store_bf16x32(uint16_t* p, const float (&v)[32]) {
  uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
    w.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
    w.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
    w.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
    q[i] = w;
  }
}

template <int MODE>
struct PlainEpi {
  const EpiParams& p;

  static constexpr int kSmemBytes = 0;
  __device__ __forceinline__ void set_smem(uint8_t*) {}
  __device__ __forceinline__ void prologue(int*) {}
  __device__ __forceinline__ void tile_begin(int, int) {}
  __device__ __forceinline__ void tile_end(int, int, int, int) {}

  __device__ __forceinline__ void chunk(int row, int col, int /*c*/, const uint32_t (&r)[32]) {
    if (row >= p.M || col >= p.N) return;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    const bool full = col + 32 <= p.N;
    if (MODE == kAccF32) {
      float* c = static_cast<float*>(p.C) + int64_t(row) * p.ldc + col;
      if (full) {
        float4* c4 = reinterpret_cast<float4*>(c);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float4 o = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          if (p.beta != 0.f) {
            const float4 old = c4[i];
            o.x += p.beta * old.x; o.y += p.beta * old.y; o.z += p.beta * old.z; o.w += p.beta * old.w;
          }
          c4[i] = o;
        }
      } else {
        _Pragma("unroll") for (int j = 0; j < 32; ++j) if (col + j < p.N) c[j] = v[j] + (p.beta != 0.f ? p.beta * c[j] : 0.f);
      }
      return;
    }
    if (MODE == kStore) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= p.alpha;
    }
    if (MODE == kBias || MODE == kBiasGelu || MODE == kBiasResidual) {
      if (p.bias) {
        if (full) {
          float b[32];
          load_bf16x32(p.bias + col, b);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += b[j];
        } else {
          _Pragma("unroll") for (int j = 0; j < 32; ++j) if (col + j < p.N) v[j] += bf16_bits_to_float(p.bias[col + j]);
        }
      }
    }
    if (MODE == kBiasResidual) {
      const uint16_t* a = p.aux + int64_t(row) * p.ld_aux + col;
      if (full) {
        float res[32];
        load_bf16x32(a, res);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += res[j];
      } else {
        _Pragma("unroll") for (int j = 0; j < 32; ++j) if (col + j < p.N) v[j] += bf16_bits_to_float(a[j]);
      }
    }
    if (MODE == kBiasGelu) {
      uint16_t* z = p.aux_out + int64_t(row) * p.ld_aux + col;
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = bf16_bits_to_float(float_to_bf16_bits(v[j]));
      if (full) {
        store_bf16x32(z, v);
      } else {
        _Pragma("unroll") for (int j = 0; j < 32; ++j) if (col + j < p.N) z[j] = float_to_bf16_bits(v[j]);
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
    }
    if (MODE == kGeluBwd) {
      const uint16_t* a = p.aux + int64_t(row) * p.ld_aux + col;
      if (full) {
        float zz[32];
        load_bf16x32(a, zz);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = bf16_bits_to_float(float_to_bf16_bits(v[j])) * gelu_erf_grad(zz[j]);
      } else {
        _Pragma("unroll") for (int j = 0; j < 32; ++j) if (col + j < p.N) v[j] = bf16_bits_to_float(float_to_bf16_bits(v[j])) * gelu_erf_grad(bf16_bits_to_float(a[j]));
      }
    }
    uint16_t* c = static_cast<uint16_t*>(p.C) + int64_t(row) * p.ldc + col;
    if (full) {
      store_bf16x32(c, v);
    } else {
      _Pragma("unroll") for (int j = 0; j < 32; ++j) if (col + j < p.N) c[j] = float_to_bf16_bits(v[j]);
    }
  }
};

// fp32 C through shared memory: each epilogue warp stages a 32 x 32 block
// (its 32 rows x one 32-column chunk) in a 128B-swizzled 4 KB buffer
// (double-buffered) and one lane issues a TMA bulk store (beta == 0) or a
// TMA bulk reduce-add (beta == 1) of the block.  Coalesced, asynchronous, and
// bitwise equal to the register path (one writer per element; the L2 add
// rounds to nearest like a load-add-store).  Out-of-range rows and columns
// are clipped by the tensor map.
struct AccF32TmaEpi {
  const EpiParams& p;
  static constexpr int kBuf = 32 * 32 * 4;
  static constexpr int kSmemBytes = 4 * 2 * kBuf + 1024;  // + alignment of the swizzled buffers
  uint32_t base = 0;
  int count = 0;

  __device__ __forceinline__ void set_smem(uint8_t* s) {
    const uint32_t a = smem_u32(s);
    base = ((a + 1023u) & ~1023u) + uint32_t(((threadIdx.x >> 5) & 3) * 2 * kBuf);
  }
  __device__ __forceinline__ void prologue(int*) {}
  __device__ __forceinline__ void tile_begin(int, int) {}
  __device__ __forceinline__ void tile_end(int, int, int, int) {}
  // Every bulk operation this thread issued has completed (its shared-memory
  // reads and its global writes) before the kernel returns, on every path.
  __device__ __forceinline__ ~AccF32TmaEpi() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
  __device__ __forceinline__ void chunk(int row, int col, int, const uint32_t (&r)[32]) {
    const int lane = threadIdx.x & 31;
    const uint32_t buf = base + uint32_t((count & 1) * kBuf);
    if (count >= 2) {  // the bulk op that last read this buffer must be done with it
      if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      __syncwarp();
    }
    const uint32_t rowa = buf + uint32_t(lane * 128), sw = uint32_t(lane & 7);
#pragma unroll
    for (int c = 0; c < 8; ++c)
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(rowa + ((uint32_t(c) ^ sw) << 4)), "r"(r[4 * c]),
                   "r"(r[4 * c + 1]), "r"(r[4 * c + 2]), "r"(r[4 * c + 3])
                   : "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
      const int row0 = row - lane;  // first row of this warp's block
      const uint64_t tmap = reinterpret_cast<uint64_t>(&p.tmC);
      if (p.beta != 0.f)
        asm volatile(
            "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
            "r"(buf), "r"(col), "r"(row0)
            : "memory");
      else
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
                     "r"(buf), "r"(col), "r"(row0)
                     : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    ++count;
  }
};

// bf16 outputs through shared memory: the same math as PlainEpi, then each
// epilogue warp stages 32 rows x 64 columns (two consecutive 32-column
// chunks) in a 128B-swizzled 4 KB buffer and one lane issues a TMA bulk
// store of the block (plus one of the pre-activation for kBiasGelu).  Two
// buffers per warp: double-buffered C, or C + pre-activation for kBiasGelu.
// Inputs (bias, residual, saved pre-activation) are read as in PlainEpi.
template <int MODE>
struct TmaBf16Epi {
  const EpiParams& p;
  static constexpr int kBuf = 32 * 128;
  static constexpr int kSmemBytes = 4 * 2 * kBuf + 1024;
  static constexpr bool kTwo = MODE == kBiasGelu;
  uint32_t base = 0;
  int blocks = 0;  // 64-column blocks issued by this warp

  __device__ __forceinline__ void set_smem(uint8_t* s) {
    const uint32_t a = smem_u32(s);
    base = ((a + 1023u) & ~1023u) + uint32_t(((threadIdx.x >> 5) & 3) * 2 * kBuf);
  }
  __device__ __forceinline__ void prologue(int*) {}
  __device__ __forceinline__ void tile_begin(int, int) {}
  __device__ __forceinline__ void tile_end(int, int, int, int) {}
  __device__ __forceinline__ ~TmaBf16Epi() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

  __device__ __forceinline__ static void stage(uint32_t buf, int lane, int half, const float (&v)[32]) {
    const uint32_t rowa = buf + uint32_t(lane * 128), sw = uint32_t(lane & 7);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(rowa + ((uint32_t(4 * half + k) ^ sw) << 4)),
                   "r"(pack_bf16x2(v[8 * k], v[8 * k + 1])), "r"(pack_bf16x2(v[8 * k + 2], v[8 * k + 3])),
                   "r"(pack_bf16x2(v[8 * k + 4], v[8 * k + 5])), "r"(pack_bf16x2(v[8 * k + 6], v[8 * k + 7]))
                   : "memory");
  }
  __device__ __forceinline__ static void store(const CUtensorMap* map, uint32_t buf, int col, int row) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(buf), "r"(col), "r"(row)
                 : "memory");
  }

  __device__ __forceinline__ void chunk(int row, int col, int c, const uint32_t (&r)[32]) {
    const int lane = threadIdx.x & 31;
    const int half = c & 1;
    float v[32], z[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    const bool inb = row < p.M;
    const bool full = inb && col + 32 <= p.N;
    if (MODE == kStore) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= p.alpha;
    }
    if ((MODE == kBias || MODE == kBiasGelu || MODE == kBiasResidual) && p.bias) {
      if (full) {
        float b[32];
        load_bf16x32(p.bias + col, b);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += b[j];
      } else if (inb) {
        _Pragma("unroll") for (int j = 0; j < 32; ++j) if (col + j < p.N) v[j] += bf16_bits_to_float(p.bias[col + j]);
      }
    }
    if (MODE == kBiasResidual) {
      const uint16_t* a = p.aux + int64_t(row) * p.ld_aux + col;
      if (full) {
        float res[32];
        load_bf16x32(a, res);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += res[j];
      } else if (inb) {
        _Pragma("unroll") for (int j = 0; j < 32; ++j) if (col + j < p.N) v[j] += bf16_bits_to_float(a[j]);
      }
    }
    if (MODE == kBiasGelu) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        z[j] = bf16_bits_to_float(float_to_bf16_bits(v[j]));
        v[j] = gelu_erf(z[j]);
      }
    }
    if (MODE == kGeluBwd) {
      const uint16_t* a = p.aux + int64_t(row) * p.ld_aux + col;
      if (full) {
        float zz[32];
        load_bf16x32(a, zz);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = bf16_bits_to_float(float_to_bf16_bits(v[j])) * gelu_erf_grad(zz[j]);
      } else if (inb) {
        _Pragma("unroll") for (int j = 0; j < 32; ++j) if (col + j < p.N) v[j] = bf16_bits_to_float(float_to_bf16_bits(v[j])) * gelu_erf_grad(bf16_bits_to_float(a[j]));
      }
    }
    // buffers: [b0][b1]; kBiasGelu uses b0 for C and b1 for the pre-activation
    const uint32_t bufC = base + uint32_t((kTwo ? 0 : (blocks & 1)) * kBuf);
    const uint32_t bufZ = base + uint32_t(kBuf);
    if (half == 0 && blocks >= (kTwo ? 1 : 2)) {  // the bulk store that last read these buffers is done with them
      if (lane == 0) {
        if (kTwo)
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        else
          asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      }
      __syncwarp();
    }
    stage(bufC, lane, half, v);
    if (kTwo) stage(bufZ, lane, half, z);
    if (half == 1) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        store(&p.tmC, bufC, col - 32, row - lane);
        if (kTwo) store(&p.tmAux, bufZ, col - 32, row - lane);
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
      ++blocks;
    }
  }
};

template <int MODE>
struct EpiFor {
  using type = typename std::conditional<(MODE >= kTmaBase), TmaBf16Epi<MODE - kTmaBase>, PlainEpi<MODE>>::type;
};
template <>
struct EpiFor<kAccF32Tma> {
  using type = AccF32TmaEpi;
};

}  // namespace gemm
}  // namespace tdb
