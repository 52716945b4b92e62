// awq_common.cuh -- device helpers shared by the W4A16 AWQ kernels (sm_100a).
//
// AWQ packing (anvil-q1/tests/verify.py:38, anvil-q1/design/SPEC.md:181-192):
// logical output lane i of a packed int32 is the nibble at bit shift
// (0,16,4,20,8,24,12,28)[i].  Read the other way, nibble j (bits 4j..4j+3)
// holds lane (0,2,4,6,1,3,5,7)[j], so the nibbles at bits 0 and 16 are lanes
// 0 and 1, bits 4 and 20 lanes 2 and 3, bits 8 and 24 lanes 4 and 5, and bits
// 12 and 28 lanes 6 and 7: every pair of adjacent output columns sits in the
// two 16-bit halves of the word at the same offset.  One AND/OR places such a
// pair into a half2.
//
// Nibble -> binary16 without a conversion instruction: binary16 0x6400 is
// 1024.0, whose unit in the last place is 1.0, so OR-ing a 4-bit value v into
// mantissa bits 0..3 gives exactly 1024 + v, and OR-ing it into bits 4..7
// gives exactly 1024 + 16 v.  Subtracting the zero point encoded the same way
// yields the signed delta q - z exactly (|q - z| <= 15 is exact in binary16).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace anvilq {

constexpr uint32_t kLoPairMask = 0x000F000Fu;   // nibbles at bits 0 and 16
constexpr uint32_t kHiPairMask = 0x00F000F0u;   // nibbles at bits 4 and 20
constexpr uint32_t kMagic1024 = 0x64006400u;    // half2(1024, 1024)

__device__ __forceinline__ half2 u32_as_half2(uint32_t u) {
  return *reinterpret_cast<half2*>(&u);
}
__device__ __forceinline__ uint32_t half2_as_u32(half2 h) {
  return *reinterpret_cast<uint32_t*>(&h);
}

// Zero-point constants of one packed qzeros word (8 output lanes):
//   z01 = (1024+z0, 1024+z1), z45 = (1024+z4, 1024+z5)
//   n23 = (-(64+z2), -(64+z3)), n67 = (-(64+z6), -(64+z7))
struct ZeroPoint {
  half2 z01, n23, z45, n67;
};

__device__ __forceinline__ ZeroPoint make_zero_point(uint32_t zw) {
  const half2 minus_sixteenth = __float2half2_rn(-0.0625f);
  const uint32_t z8 = zw >> 8;
  ZeroPoint zp;
  zp.z01 = u32_as_half2((zw & kLoPairMask) | kMagic1024);
  zp.z45 = u32_as_half2((z8 & kLoPairMask) | kMagic1024);
  // (1024 + 16 z) * (-1/16) = -(64 + z), exact.
  zp.n23 = __hmul2(u32_as_half2((zw & kHiPairMask) | kMagic1024), minus_sixteenth);
  zp.n67 = __hmul2(u32_as_half2((z8 & kHiPairMask) | kMagic1024), minus_sixteenth);
  return zp;
}

// Signed deltas q - z of the 8 lanes of one qweight word, as 4 half2 holding
// output columns (0,1), (2,3), (4,5), (6,7).  All values exact.
// Cost: 5 integer ops (4 AND/OR, 1 shift) + 4 half2 ops for 8 weights.
__device__ __forceinline__ void unpack_deltas(uint32_t w, const ZeroPoint& zp, half2 d[4]) {
  const half2 sixteenth = __float2half2_rn(0.0625f);
  const uint32_t w8 = w >> 8;
  d[0] = __hsub2(u32_as_half2((w & kLoPairMask) | kMagic1024), zp.z01);
  d[1] = __hfma2(u32_as_half2((w & kHiPairMask) | kMagic1024), sixteenth, zp.n23);
  d[2] = __hsub2(u32_as_half2((w8 & kLoPairMask) | kMagic1024), zp.z45);
  d[3] = __hfma2(u32_as_half2((w8 & kHiPairMask) | kMagic1024), sixteenth, zp.n67);
}

// a0 += x * d.lo and a1 += x * d.hi in binary32: the product of two binary16
// operands is exact in binary32 (11 + 11 significant bits), so each step of a
// sum of x (q - z) rounds once, in fp32, as FP32Model.linear's accumulation does.
__device__ __forceinline__ void fma2_f32_f16(float& a0, float& a1, half2 d, __half x) {
  asm("{\n .reg .f16 d0, d1;\n mov.b32 {d0, d1}, %2;\n"
      " fma.rn.f32.f16 %0, %3, d0, %0;\n fma.rn.f32.f16 %1, %3, d1, %1;\n}"
      : "+f"(a0), "+f"(a1)
      : "r"(half2_as_u32(d)), "h"(__half_as_ushort(x)));
}

// Nonzero iff either binary16 half of `u` is an invalid AWQ scale: exponent 31
// (Inf/NaN) or negative and nonzero (anvil-q1/design/SPEC.md:175-177).
// Per half: (e & 0x7C00) + 0x0400 carries into bit 15 exactly when e == 31;
// (h & 0x7FFF) + 0x7FFF carries into bit 15 exactly when the magnitude is
// nonzero, which is then AND-ed with the sign bit.
__device__ __forceinline__ uint32_t invalid_scale_pair(uint32_t u) {
  const uint32_t inf_nan = (u & 0x7C007C00u) + 0x04000400u;
  const uint32_t neg_nonzero = ((u & 0x7FFF7FFFu) + 0x7FFF7FFFu) & u;
  return (inf_nan | neg_nonzero) & 0x80008000u;
}

// ---- global loads --------------------------------------------------------
// Streamed once: read-only path, do not keep in L1.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ld_stream_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
// Reused across threads (activations, scales, zeros): read-only path, cached.
__device__ __forceinline__ uint4 ld_ro_v4(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

template <int WORDS>
struct Words;
template <>
struct Words<4> {
  uint32_t w[4];
  __device__ __forceinline__ void load_stream(const int32_t* p) {
    uint4 v = ld_stream_v4(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  }
  __device__ __forceinline__ void load_ro(const int32_t* p) {
    uint4 v = ld_ro_v4(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  }
};
template <>
struct Words<2> {
  uint32_t w[2];
  __device__ __forceinline__ void load_stream(const int32_t* p) {
    uint2 v = ld_stream_v2(p);
    w[0] = v.x; w[1] = v.y;
  }
  __device__ __forceinline__ void load_ro(const int32_t* p) {
    uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = v.x; w[1] = v.y;
  }
};
template <>
struct Words<1> {
  uint32_t w[1];
  __device__ __forceinline__ void load_stream(const int32_t* p) { w[0] = ld_stream_u32(p); }
  __device__ __forceinline__ void load_ro(const int32_t* p) {
    w[0] = __ldg(reinterpret_cast<const unsigned int*>(p));
  }
};

}  // namespace anvilq
