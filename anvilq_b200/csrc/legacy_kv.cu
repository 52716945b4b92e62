// legacy_kv.cu -- the legacy KV-cache codecs of the Q16.16 datapath: INT8
// symmetric, INT4 symmetric and INT4 asymmetric blocks with a power-of-two
// exponent per block (anvil-q4/design/SPEC.md:250-262; model
// anvil-q4/tests/legacy_reference.py:71-97 cache_block, payload layout
// :186-203).
//
// A block is `block` consecutive Q16.16 values of one head (the last block of a
// head may be shorter).  Symmetric: e = the smallest exponent <= Emax (25 for
// INT8, 29 for INT4) with max|v| <= L 2^e (L = 127 or 7, on the unrounded
// magnitude); code = clamp(round-half-away(v / 2^e), -L, L).  Asymmetric: the
// first e in 0..32 for which the rounded extrema plus a zero point z in [-8, 7]
// fit [-8, 7], z the fitting value closest to 0; code = rounded + z.
// Metadata = e | (z & 15) << 8; the value decodes to sat32((code - z) 2^e).
// Payload: W = ceil(block * bits / 32) words per block, codes in ascending
// bytes / nibbles, padding zero; word column (head * B + block) * W + word,
// metadata column head * B + block, B = ceil(D / block).
//
// Encode: one warp per block (two values per lane, block <= 64), extrema by
// warp reductions in 64-bit integers, codes gathered into words through shared
// memory.  Decode: one thread per value, with the format's checks (exponent
// range, reserved metadata bits, the forbidden symmetric codes -128 / -8,
// nonzero padding) reported through ANVILQ_DEV_ERR_CODEC.
#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>

#include "../../include/anvilq.h"

namespace anvilq {
namespace legacy {

constexpr int kMaxBlock = 64;
constexpr int kWarpsPerCta = 8;

__device__ __forceinline__ long long round_away_shift(long long v, int e) {
  if (e == 0) return v;
  const long long m = ((v < 0 ? -v : v) + (1LL << (e - 1))) >> e;
  return v < 0 ? -m : m;
}
__device__ __forceinline__ long long warp_max(long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  return v;
}
__device__ __forceinline__ long long warp_min(long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u < v ? u : v;
  }
  return v;
}

struct Shape {
  int R, H, D, block, fmt;
  int B, W, bits;
};

__global__ void __launch_bounds__(kWarpsPerCta * 32) legacy_encode_kernel(const int32_t* __restrict__ in,
                                                                        uint32_t* __restrict__ payload,
                                                                        uint32_t* __restrict__ meta, const Shape s) {
  __shared__ int8_t codes_s[kWarpsPerCta][2 * kMaxBlock];
  const int lane = threadIdx.x % 32, wl = threadIdx.x / 32;
  const long long w = (long long)blockIdx.x * kWarpsPerCta + wl;   // (row, head, block)
  if (w >= (long long)s.R * s.H * s.B) return;
  const int b = (int)(w % s.B), h = (int)((w / s.B) % s.H);
  const long long r = w / ((long long)s.B * s.H);
  const int n = min(s.block, s.D - b * s.block);
  const int32_t* src = in + (r * s.H + h) * s.D + (long long)b * s.block;
  const bool ok0 = lane < n, ok1 = lane + 32 < n;
  const long long v0 = ok0 ? src[lane] : 0, v1 = ok1 ? src[lane + 32] : 0;
  int e = 0, z = 0;
  long long c0 = 0, c1 = 0;
  if (s.fmt == 3) {
    for (e = 0; e <= 32; ++e) {
      const long long r0 = round_away_shift(v0, e), r1 = round_away_shift(v1, e);
      const long long mn = warp_min(min(ok0 ? r0 : LLONG_MAX, ok1 ? r1 : LLONG_MAX));
      const long long mx = warp_max(max(ok0 ? r0 : LLONG_MIN, ok1 ? r1 : LLONG_MIN));
      const long long low = max(-8LL, -8 - mn), high = min(7LL, 7 - mx);
      if (low <= high) {
        z = (int)(low > 0 ? low : (high < 0 ? high : 0));
        c0 = r0 + z;
        c1 = r1 + z;
        break;
      }
    }
  } else {
    const long long L = s.fmt == 1 ? 127 : 7;
    const int emax = s.fmt == 1 ? 25 : 29;
    const long long a = warp_max(max(ok0 ? (v0 < 0 ? -v0 : v0) : 0LL, ok1 ? (v1 < 0 ? -v1 : v1) : 0LL));
    while (e < emax && a > (L << e)) ++e;
    c0 = min(L, max(-L, round_away_shift(v0, e)));
    c1 = min(L, max(-L, round_away_shift(v1, e)));
  }
  // codes of the block, padding zero, gathered into words
  const int per = 32 / s.bits;
  int8_t* cs = codes_s[wl];
  cs[lane] = ok0 ? (int8_t)c0 : 0;
  cs[lane + 32] = ok1 ? (int8_t)c1 : 0;
  __syncwarp();
  const long long base = ((r * s.H + h) * s.B + b) * s.W;
  if (lane < s.W) {
    const uint32_t mask = (1u << s.bits) - 1u;
    uint32_t word = 0;
    for (int k = 0; k < per; ++k) {
      const int i = lane * per + k;
      const int c = i < n ? cs[i] : 0;
      word |= ((uint32_t)c & mask) << (k * s.bits);
    }
    payload[base + lane] = word;
  }
  if (lane == 0) meta[(r * s.H + h) * s.B + b] = (uint32_t)e | ((uint32_t)(z & 15) << 8);
}

__global__ void legacy_decode_kernel(const uint32_t* __restrict__ payload, const uint32_t* __restrict__ meta,
                                     int32_t* __restrict__ out, int* dev_err, const Shape s) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;   // (row, head, dim)
  if (t >= (long long)s.R * s.H * s.D) return;
  const int d = (int)(t % s.D), h = (int)((t / s.D) % s.H);
  const long long r = t / ((long long)s.D * s.H);
  const int b = d / s.block, i = d % s.block;
  const int per = 32 / s.bits;
  const long long blk = (r * s.H + h) * s.B + b;
  const uint32_t m = meta[blk];
  const uint32_t word = payload[blk * s.W + i / per];
  const uint32_t raw = (word >> ((i % per) * s.bits)) & ((1u << s.bits) - 1u);
  const int code = s.bits == 8 ? (int)(int8_t)raw : (int)((raw ^ 8u) - 8u);   // sign-extended
  const int e = (int)(m & 0xFFu);
  const int zraw = (int)((m >> 8) & 15u);
  const int z = s.fmt == 3 ? (zraw ^ 8) - 8 : 0;
  bool bad = e > (s.fmt == 1 ? 25 : s.fmt == 2 ? 29 : 32) || (m >> 12) != 0u || (s.fmt != 3 && zraw != 0) ||
             (s.fmt == 1 && code == -128) || (s.fmt == 2 && code == -8);
  // the thread of a block's last value also checks the block's padding codes
  const int n = min(s.block, s.D - b * s.block);
  if (i == n - 1) {
    for (int k = n; k < s.W * per; ++k) {
      const uint32_t wk = payload[blk * s.W + k / per];
      bad |= ((wk >> ((k % per) * s.bits)) & ((1u << s.bits) - 1u)) != 0u;
    }
  }
  if (bad) atomicOr(dev_err, ANVILQ_DEV_ERR_CODEC);
  const long long v = (long long)(code - z) << (e > 32 ? 32 : e);
  out[t] = (int32_t)(v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : v));
}

static bool make_shape(Shape* s, int R, int H, int D, int block, int fmt) {
  if (R < 1 || H < 1 || D < 1 || block < 1 || block > kMaxBlock || fmt < 1 || fmt > 3) return false;
  if ((long long)R * H * D > (1LL << 40)) return false;
  s->R = R; s->H = H; s->D = D; s->block = block; s->fmt = fmt;
  s->bits = fmt == 1 ? 8 : 4;
  s->B = (D + block - 1) / block;
  s->W = (block * s->bits + 31) / 32;
  return true;
}

}  // namespace legacy
}  // namespace anvilq

extern "C" {

int anvilq_legacy_kv_encode(const int32_t* values, uint32_t* payload, uint32_t* metadata, int rows, int H, int D,
                            int block, int format, anvilq_stream_t stream) {
  using namespace anvilq::legacy;
  if (!values || !payload || !metadata) return ANVILQ_EINVAL;
  Shape s;
  if (!make_shape(&s, rows, H, D, block, format)) return ANVILQ_ESHAPE;
  const long long warps = (long long)rows * H * s.B;
  const long long grid = (warps + kWarpsPerCta - 1) / kWarpsPerCta;
  if (grid > 0x7FFFFFFFLL) return ANVILQ_ESHAPE;
  legacy_encode_kernel<<<(unsigned)grid, kWarpsPerCta * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      values, payload, metadata, s);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}

int anvilq_legacy_kv_decode(const uint32_t* payload, const uint32_t* metadata, int32_t* values, int rows, int H,
                            int D, int block, int format, int* dev_err, anvilq_stream_t stream) {
  using namespace anvilq::legacy;
  if (!values || !payload || !metadata || !dev_err) return ANVILQ_EINVAL;
  Shape s;
  if (!make_shape(&s, rows, H, D, block, format)) return ANVILQ_ESHAPE;
  const long long n = (long long)rows * H * D;
  const long long grid = (n + 255) / 256;
  if (grid > 0x7FFFFFFFLL) return ANVILQ_ESHAPE;
  legacy_decode_kernel<<<(unsigned)grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(payload, metadata,
                                                                                          values, dev_err, s);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}

}  // extern "C"
