// Shared device helpers for the kvssd B200 decode kernels.
//
// Bit layout (the contract of kvssd's quantizer, src/kvssd/quant.py:28-46 and 68-73):
//   * a row of `head_dim` unsigned codes is packed low-bits-first: element i lives in byte
//     i / (8/bits) at bit offset (i % (8/bits)) * bits;
//   * a value is (code - 2^(bits-1)) * scale, with one FP16 scale per `group_size` elements.
//
// The unpackers below turn packed codes into FP16 without integer conversions: a code n is
// OR-ed into the mantissa of the FP16 constant 1024 (0x6400), giving the exact value
// 1024 + n * 2^s, and one HSUB2/HFMA2 with exactly representable constants removes the
// offset. Every intermediate is an exactly representable small integer, so the centred
// code (n - midpoint) is exact and the single HMUL2 by the FP16 scale is one
// round-to-nearest-even step: bit-identical to kvssd's dequantize_tensor(q, torch.float16),
// which rounds the exact FP32 product (code - mid) * scale to FP16 once.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>

namespace kvb {

// Query element types accepted by the C ABI (the reference dispatches f32/f64/f16/bf16,
// csrc/fused_decode.cu:131-140).
enum QueryDtype : int { kQF32 = 0, kQF16 = 1, kQBF16 = 2, kQF64 = 3 };

// Status bits OR-ed into the workspace header word by device code.
enum DeviceStatusBits : unsigned {
  kDevBadBlockIndex = 1u,   // a block-table entry outside [0, n_pool_blocks)
  kDevBadValidCount = 2u,   // a valid_tokens entry outside [0, block_tokens]
  kDevCombineTimeout = 4u,  // a fused combine gave up waiting for the other CTAs' parts
  kDevExchangeTimeout = 8u,  // a cross-GPU exchange gave up waiting for another rank's slice
  kDevBadProblem = 16u,      // a batched problem descriptor was refused (misaligned/invalid)
  kDevStreamTimeout = 32u,   // a TMA-fed kernel gave up waiting for its copies or ring slots
};

// The G FP16 scales of one (token, KV head) row, loaded as one 8- or 4-byte word.
template <int G>
struct ScaleRow {
  __half s[G];
  __device__ __forceinline__ void load(const uint8_t* p) {
    if constexpr (G == 4) {
      const uint2 w = *reinterpret_cast<const uint2*>(p);
      memcpy(s, &w, 8);
    } else {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
      memcpy(s, &w, 4);
    }
  }
  // Scales 2i and 2i + 1 as one FP16 pair (low half = scale 2i); i may differ per thread (a
  // select between the row's two words, never an indexed access).
  __device__ __forceinline__ uint32_t word(int i) const {
    uint32_t w0, w1 = 0u;
    memcpy(&w0, s, 4);
    if constexpr (G == 4) memcpy(&w1, s + 2, 4);
    return (G == 4 && i) ? w1 : w0;
  }
};

// System-scope relaxed 64-bit load / store (words written across GPUs over NVLink; an
// aligned 64-bit access is single-copy atomic, so a {value, tag} word arrives whole).
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// GPU-scope acquire load (pairs with __threadfence + atomicAdd on the writer side).
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float load_query(const void* q, int dtype, long long idx) {
  switch (dtype) {
    case kQF16: return __half2float(reinterpret_cast<const __half*>(q)[idx]);
    case kQBF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(q)[idx]);
    case kQF64: return static_cast<float>(reinterpret_cast<const double*>(q)[idx]);
    default: return reinterpret_cast<const float*>(q)[idx];
  }
}

// Eight consecutive query elements q[idx .. idx + 7] as FP32, idx a multiple of 8: vector
// loads when the tensor is 16-byte aligned (two or four of them, all issued before use), else
// element by element.
__device__ __forceinline__ void load_query8(const void* q, int dtype, long long idx, float (&f)[8]) {
  const bool vec = (reinterpret_cast<uintptr_t>(q) & 15u) == 0;
  if (vec && (dtype == kQF16 || dtype == kQBF16)) {
    const uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(q) + idx);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (dtype == kQF16) {
        const __half2 h = *reinterpret_cast<const __half2*>(&u[i]);
        f[2 * i] = __low2float(h);
        f[2 * i + 1] = __high2float(h);
      } else {
        const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&u[i]);
        f[2 * i] = __low2float(h);
        f[2 * i + 1] = __high2float(h);
      }
    }
  } else if (vec && dtype == kQF32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(q) + idx);
    const float4 a = p[0], b = p[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else if (vec && dtype == kQF64) {
    const double2* p = reinterpret_cast<const double2*>(reinterpret_cast<const double*>(q) + idx);
    const double2 a = p[0], b = p[1], c = p[2], d = p[3];
    f[0] = static_cast<float>(a.x); f[1] = static_cast<float>(a.y);
    f[2] = static_cast<float>(b.x); f[3] = static_cast<float>(b.y);
    f[4] = static_cast<float>(c.x); f[5] = static_cast<float>(c.y);
    f[6] = static_cast<float>(d.x); f[7] = static_cast<float>(d.y);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = load_query(q, dtype, idx + i);
  }
}

__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) {
  __half2 h;
  memcpy(&h, &u, 4);
  return h;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) {
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}

__device__ __forceinline__ __half2 h2_const(uint32_t bits) { return u32_as_h2(bits); }

// (x & MASK) | 0x64006400: places the selected code bits of both 16-bit lanes into the
// mantissa of FP16 1024.
template <uint32_t MASK>
__device__ __forceinline__ uint32_t or_magic(uint32_t x) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "n"(MASK), "n"(0x64006400u));
  return r;
}

// Centred codes of a 32-bit word viewed as two 16-bit lanes. Lane 0 is bits 0-15, lane 1 is
// bits 16-31; each lane holds 16/BITS codes in element order. Output pair k is
// (lane0 code k - mid, lane1 code k - mid) as an exact FP16 pair.
template <int BITS>
struct LanePairs;

template <>
struct LanePairs<4> {
  static constexpr int kPairs = 4;  // codes per 16-bit lane
  __device__ __forceinline__ static void centred(uint32_t x, __half2 (&o)[4]) {
    const uint32_t x8 = x >> 8;
    // code at bits 0-3 of each lane: 1024 + n, minus 1032 (0x6408)
    o[0] = __hsub2(u32_as_h2(or_magic<0x000F000Fu>(x)), h2_const(0x64086408u));
    // code at bits 4-7: 1024 + 16n; times 1/16 (0x2C00) minus 72 (0xD480 = -72)
    o[1] = __hfma2(u32_as_h2(or_magic<0x00F000F0u>(x)), h2_const(0x2C002C00u),
                   h2_const(0xD480D480u));
    o[2] = __hsub2(u32_as_h2(or_magic<0x000F000Fu>(x8)), h2_const(0x64086408u));
    o[3] = __hfma2(u32_as_h2(or_magic<0x00F000F0u>(x8)), h2_const(0x2C002C00u),
                   h2_const(0xD480D480u));
  }
};

// Uncentred INT4 pairs: even code slots as FP16 1024 + n, odd slots as 1024 + 16n (one LOP3
// each); consumers fold the 1/16 and the offsets (1032, 1152) into their other operand.
__device__ __forceinline__ void raw_pairs4(uint32_t x, uint32_t (&o)[4]) {
  const uint32_t x8 = x >> 8;
  o[0] = or_magic<0x000F000Fu>(x);
  o[1] = or_magic<0x00F000F0u>(x);
  o[2] = or_magic<0x000F000Fu>(x8);
  o[3] = or_magic<0x00F000F0u>(x8);
}

template <>
struct LanePairs<2> {
  static constexpr int kPairs = 8;
  __device__ __forceinline__ static void centred(uint32_t x, __half2 (&o)[8]) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t y = half ? (x >> 8) : x;
      // bits 0-1: 1024 + n, minus 1026 (0x6402)
      o[4 * half + 0] = __hsub2(u32_as_h2(or_magic<0x00030003u>(y)), h2_const(0x64026402u));
      // bits 2-3: 1024 + 4n; * 1/4 (0x3400) - 258 (0xDC08)
      o[4 * half + 1] = __hfma2(u32_as_h2(or_magic<0x000C000Cu>(y)), h2_const(0x34003400u),
                                h2_const(0xDC08DC08u));
      // bits 4-5: 1024 + 16n; * 1/16 (0x2C00) - 66 (0xD420)
      o[4 * half + 2] = __hfma2(u32_as_h2(or_magic<0x00300030u>(y)), h2_const(0x2C002C00u),
                                h2_const(0xD420D420u));
      // bits 6-7: 1024 + 64n; * 1/64 (0x2400) - 18 (0xCC80)
      o[4 * half + 3] = __hfma2(u32_as_h2(or_magic<0x00C000C0u>(y)), h2_const(0x24002400u),
                                h2_const(0xCC80CC80u));
    }
  }
};

// Dequantized pairs: centred code times the per-lane FP16 scale, one RN-even rounding.
template <int BITS>
__device__ __forceinline__ void dequant_pairs(uint32_t x, __half2 scale,
                                              __half2 (&o)[LanePairs<BITS>::kPairs]) {
  LanePairs<BITS>::centred(x, o);
#pragma unroll
  for (int k = 0; k < LanePairs<BITS>::kPairs; ++k) o[k] = __hmul2(o[k], scale);
}

// Combines 16-bit lane `hw` of two 32-bit words (two token rows) into one word whose low
// lane comes from `a` and high lane from `b`.
__device__ __forceinline__ uint32_t pair_lanes(uint32_t a, uint32_t b, int hw_in_word) {
  return __byte_perm(a, b, hw_in_word ? 0x7632u : 0x5410u);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// D = A * B + D for one m16n8k16 FP16 tile with FP32 accumulation (PTX ISA
// "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32").
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transposes an 8x8 b16 matrix held in the mma row-fragment layout.
__device__ __forceinline__ uint32_t transpose_8x8(uint32_t x) {
  uint32_t y;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// Four 8x8 b16 matrices from shared memory; lane i supplies the address of row i%8 of matrix
// i/8 (PTX ldmatrix). The .trans form hands thread (g, c) elements [2c][g] and [2c+1][g].
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// GPU-wide nanosecond clock (%globaltimer), the time base of every bounded wait.
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// L2 policy for data read exactly once: evicted first, so it does not push out data that is
// reused soon (e.g. the split-KV parts the combine kernel reads next).
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// 16-byte asynchronous global -> shared copy, cached in L2 only (PTX cp.async.cg).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst),
               "l"(src), "l"(policy)
               : "memory");
}

// 8-byte asynchronous global -> shared copy (PTX cp.async.ca; 8-byte aligned addresses).
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 8, %2;" ::"r"(dst),
               "l"(src), "l"(policy)
               : "memory");
}

// 4-byte asynchronous global -> shared copy (PTX cp.async.ca; 4-byte aligned addresses).
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 4, %2;" ::"r"(dst),
               "l"(src), "l"(policy)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int N>
struct VecBytes;  // streaming loads of N contiguous bytes into 32-bit words

template <>
struct VecBytes<32> {
  __device__ __forceinline__ static void load(const uint8_t* p, uint32_t* w) {
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "l"(p));
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7]) : "l"(p + 16));
  }
};
template <>
struct VecBytes<16> {
  __device__ __forceinline__ static void load(const uint8_t* p, uint32_t* w) {
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "l"(p));
  }
};
template <>
struct VecBytes<8> {
  __device__ __forceinline__ static void load(const uint8_t* p, uint32_t* w) {
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(w[0]), "=r"(w[1]) : "l"(p));
  }
};
template <>
struct VecBytes<4> {
  __device__ __forceinline__ static void load(const uint8_t* p, uint32_t* w) {
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(w[0]) : "l"(p));
  }
};
template <>
struct VecBytes<2> {
  __device__ __forceinline__ static void load(const uint8_t* p, uint32_t* w) {
    unsigned short s;
    asm("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(s) : "l"(p));
    w[0] = s;
  }
};

template <int N>
struct LdsBytes;  // shared-memory loads of N contiguous bytes into 32-bit words

template <>
struct LdsBytes<32> {
  __device__ __forceinline__ static void load(const uint8_t* p, uint32_t* w) {
    const uint4 a = reinterpret_cast<const uint4*>(p)[0], b = reinterpret_cast<const uint4*>(p)[1];
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
    w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
  }
};
template <>
struct LdsBytes<16> {
  __device__ __forceinline__ static void load(const uint8_t* p, uint32_t* w) {
    const uint4 a = *reinterpret_cast<const uint4*>(p);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  }
};
template <>
struct LdsBytes<8> {
  __device__ __forceinline__ static void load(const uint8_t* p, uint32_t* w) {
    const uint2 a = *reinterpret_cast<const uint2*>(p);
    w[0] = a.x; w[1] = a.y;
  }
};
template <>
struct LdsBytes<4> {
  __device__ __forceinline__ static void load(const uint8_t* p, uint32_t* w) {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
};
template <>
struct LdsBytes<2> {
  __device__ __forceinline__ static void load(const uint8_t* p, uint32_t* w) {
    w[0] = *reinterpret_cast<const unsigned short*>(p);
  }
};

__device__ __forceinline__ __half load_scale(const __half* p) {
  unsigned short s;
  asm("ld.global.nc.u16 %0, [%1];" : "=h"(s) : "l"(p));
  return __ushort_as_half(s);
}

}  // namespace kvb
