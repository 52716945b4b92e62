// kv_int8.cu -- the per-head INT8 KV-cache encoding with FP32 escape of the
// Anvil-Q4 cache (anvil-q4/design/SPEC.md:209-235; rational model
// anvil-q4/tests/cache_reference.py:54-83), written straight into the cache
// layout that gqa_decode_kernel<D, true> reads.
//
// One warp encodes one (token, kv head) row of D values:
//   * escape when the row holds a NaN, an infinity or -0.0: metadata
//     0x7FC00000, codes 0, the values (every NaN made 0x7FC00000) in the fp32
//     escape payload;
//   * otherwise scale = fp32(maxabs / 127) (1.0 for an all-+0 row; escape if it
//     underflows to 0), code = clamp(round-half-even(|fp32(v / scale)|), 127)
//     with v's sign, metadata = the scale's bits, payload zero.
// Each step is one IEEE binary32 operation (__fdiv_rn, rintf), so the codes and
// scales are bit-identical to the rational model.
//
// Cache layout: codes int8 [B][Tmax][Hkv][D]; metadata uint32 [B][Hkv][Tmax]
// (a kv head's tokens contiguous, so 16 of them are one 64-byte TMA box);
// escape payload fp32 [B][Tmax][Hkv][D].
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/anvilq.h"

namespace anvilq {
namespace kv8 {

constexpr uint32_t kMarker = 0x7FC00000u;
constexpr int kMaxD = 256;

struct StoreParams {
  const void* src;          // [B][T][H][D] fp16 or fp32
  int src_half;
  const int* start;         // [B] first cache position of each sequence's rows (NULL: 0)
  int8_t* codes;
  uint32_t* meta;
  float* escape;            // NULL: escaped rows set ANVILQ_DEV_ERR_NONFINITE
  int* dev_err;
  int B, T, H, D, Tmax;
};

__global__ void kv_int8_store_kernel(const StoreParams p) {
  const int lane = threadIdx.x % 32;
  const long long w = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;   // (b, t, h)
  if (w >= (long long)p.B * p.T * p.H) return;
  const int h = (int)(w % p.H), t = (int)((w / p.H) % p.T), b = (int)(w / ((long long)p.H * p.T));
  const int pos = (p.start ? p.start[b] : 0) + t;
  if (pos < 0 || pos >= p.Tmax) {
    if (lane == 0 && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SEQLEN);
    return;
  }
  constexpr int kPer = kMaxD / 32;
  const size_t src_row = (((size_t)b * p.T + t) * p.H + h) * p.D;
  uint32_t bits[kPer];
  bool special = false;
  float maxabs = 0.0f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int d = lane + 32 * i;
    bits[i] = 0;
    if (d < p.D) {
      const float v = p.src_half ? __half2float(static_cast<const __half*>(p.src)[src_row + d])
                                 : static_cast<const float*>(p.src)[src_row + d];
      bits[i] = __float_as_uint(v);
      special |= (bits[i] & 0x7F800000u) == 0x7F800000u || bits[i] == 0x80000000u;
      maxabs = fmaxf(maxabs, fabsf(v));
    }
  }
  const bool nonfinite_or_negzero = __any_sync(0xffffffffu, special);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) maxabs = fmaxf(maxabs, __shfl_xor_sync(0xffffffffu, maxabs, o));
  float scale = 1.0f;
  bool esc = nonfinite_or_negzero;
  if (!esc && maxabs > 0.0f) {
    scale = __fdiv_rn(maxabs, 127.0f);
    esc = scale == 0.0f;   // maxabs of 63 or fewer subnormal units
  }
  const size_t cache_row = (((size_t)b * p.Tmax + pos) * p.H + h) * p.D;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int d = lane + 32 * i;
    if (d >= p.D) continue;
    int code = 0;
    uint32_t payload = 0;
    if (esc) {
      const bool nan = (bits[i] & 0x7F800000u) == 0x7F800000u && (bits[i] & 0x7FFFFFu);
      payload = nan ? kMarker : bits[i];
    } else {
      const float ratio = __fdiv_rn(__uint_as_float(bits[i]), scale);
      const float mag = fminf(rintf(fabsf(ratio)), 127.0f);
      code = (int)(ratio < 0.0f ? -mag : mag);
    }
    p.codes[cache_row + d] = (int8_t)code;
    if (p.escape) p.escape[cache_row + d] = __uint_as_float(payload);
  }
  if (lane == 0) {
    p.meta[((size_t)b * p.H + h) * p.Tmax + pos] = esc ? kMarker : __float_as_uint(scale);
    if (esc && !p.escape && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_NONFINITE);
  }
}

}  // namespace kv8
}  // namespace anvilq

extern "C" int anvilq_kv_int8_store(const void* src, int src_half, int B, int T, int H, int D, int Tmax,
                                    const int32_t* start, int8_t* codes, uint32_t* meta, float* escape,
                                    int* dev_err, anvilq_stream_t stream) {
  using namespace anvilq::kv8;
  if (!src || !codes || !meta) return ANVILQ_EINVAL;
  if (B < 1 || T < 1 || H < 1 || D < 1 || D > kMaxD || Tmax < 1 || (src_half != 0 && src_half != 1))
    return ANVILQ_EINVAL;
  if (!start && T > Tmax) return ANVILQ_EINVAL;
  StoreParams p;
  p.src = src;
  p.src_half = src_half;
  p.start = start;
  p.codes = codes;
  p.meta = meta;
  p.escape = escape;
  p.dev_err = dev_err;
  p.B = B; p.T = T; p.H = H; p.D = D; p.Tmax = Tmax;
  const long long rows = (long long)B * T * H;
  const int warps_per_block = 8;
  const long long blocks = (rows + warps_per_block - 1) / warps_per_block;
  if (blocks > 0x7FFFFFFFll) return ANVILQ_ESHAPE;
  kv_int8_store_kernel<<<(unsigned)blocks, warps_per_block * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}
