// gemm_w4a16.cu -- W4A16 AWQ GEMV / small-M GEMM on CUDA cores, the AWQ
// dequantiser and the AWQ pack/unpack kernels, with their C-ABI entry points.
//
// Reference semantics: FP32Model.linear (anvil-q1/tests/official_weights.py:418-437),
// dequant (anvil-q1/tests/verify.py:241-250), pack / pack_lanes / unpack_lanes
// (verify.py:252-253, anvil-q1-fp/tests/awq_prepare.py:84-99).
//
// Fast path ("stream-K" over column bands):
//   * A band is 32 consecutive qweight words of a row = 128 bytes = 256 output
//     columns.  A slot is 16 consecutive rows of one band (2 KB of int4 data).
//     The bands x slots items are linearised band-major and split into equal
//     contiguous ranges, one per CTA of a persistent grid of (#SM x occupancy)
//     CTAs, so every SM streams the same number of bytes (+-1 slot).
//   * Inside a CTA, lane-groups (8 lanes x 4 words for M=1, a warp x 1 word for
//     M>1) take the slots of the current band round-robin.  Each thread keeps
//     16 row loads in flight, unpacks nibbles in registers (awq_common.cuh),
//     accumulates x * (q - z) for the 16 rows in half2, then folds the partial
//     into fp32 accumulators with the group's scale (a slot never straddles a
//     group: G % 16 == 0).  The scale multiplies once per 16 products.
//   * At the end of a band segment the lane-groups are reduced through shared
//     memory in a fixed order.  A band covered by one CTA is written directly;
//     a band split between CTAs leaves one fp32 partial per CTA in the
//     workspace, and the CTA that arrives last (atomic ticket) sums them in
//     CTA order -- deterministic, no spin-wait -- adds bias, rounds to fp16 and
//     re-arms the ticket.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "../../include/anvilq.h"
#include "awq_common.cuh"
#include "internal.h"

namespace anvilq {

constexpr int kSlotRows = 16;
constexpr int kBandWords = 32;
constexpr int kBandCols = kBandWords * 8;   // 256
constexpr int kThreads = 128;

struct GemmParams {
  const __half* x;        // [M][K]
  const int32_t* qweight; // [K][W8]
  const int32_t* qzeros;  // [K/G][W8]
  const __half* scales;   // [K/G][N]
  const __half* bias;     // [N] or null
  __half* y;              // [M][N]
  float* partials;        // [P][2][M][256]
  int* tickets;           // [bands]
  int* dev_err;
  int K, N, W8, G;
  int bands, slots;       // slots per band = K / 16
  long long items;        // bands * slots
};

__device__ __forceinline__ long long range_begin(long long c, long long items, long long P) {
  return c * items / P;
}
// CTA owning item i: the largest c with floor(c * items / P) <= i.
__device__ __forceinline__ int owner_of(long long i, long long items, long long P) {
  return (int)(((i + 1) * P + items - 1) / items - 1);
}

// Broadcast binary16 #j (0..7) of a uint4 into both halves of a half2.
__device__ __forceinline__ half2 bcast_half(const uint4& v, int j) {
  const uint32_t w = (j >> 1) == 0 ? v.x : (j >> 1) == 1 ? v.y : (j >> 1) == 2 ? v.z : v.w;
  return u32_as_half2(__byte_perm(w, w, (j & 1) ? 0x3232 : 0x1010));
}

// Writes the CTA's reduced segment result for band `band` (M x 256 floats in
// `seg`, one per thread-strided column) to y directly or through the workspace.
template <int M>
__device__ void finish_segment(const GemmParams& p, const float* seg, int band, bool whole,
                               long long it, int* s_flag) {
  const int col0 = band * kBandCols;
  if (whole) {
    for (int e = threadIdx.x; e < M * kBandCols; e += blockDim.x) {
      const int m = e / kBandCols, c = e % kBandCols, col = col0 + c;
      if (col < p.N) {
        float v = seg[e];
        if (p.bias) v += __half2float(p.bias[col]);
        p.y[(size_t)m * p.N + col] = __float2half_rn(v);
      }
    }
    return;
  }
  const long long P = gridDim.x;
  const int me = blockIdx.x;
  const int slot_j = (it == range_begin(me, p.items, P)) ? 0 : 1;
  float* mine = p.partials + ((size_t)me * 2 + slot_j) * (M * kBandCols);
  for (int e = threadIdx.x; e < M * kBandCols; e += blockDim.x) __stcg(mine + e, seg[e]);
  __threadfence();
  __syncthreads();
  const long long band_first = (long long)band * p.slots;
  const int c_lo = owner_of(band_first, p.items, P);
  const int c_hi = owner_of(band_first + p.slots - 1, p.items, P);
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(p.tickets + band, 1);
    const bool last = ticket == c_hi - c_lo;
    if (last) p.tickets[band] = 0;   // re-arm for the next launch
    *s_flag = last;
  }
  __syncthreads();
  if (!*s_flag) return;
  __threadfence();
  // Contributor q stored its partial for its first band in slot 0, for its last
  // band in slot 1.  Every contributor after c_lo starts inside this band (slot
  // 0); c_lo used slot 1 unless its range starts exactly at the band start.
  const int j_lo = range_begin(c_lo, p.items, P) < band_first ? 1 : 0;
  const float* first = p.partials + ((size_t)c_lo * 2 + j_lo) * (M * kBandCols);
  const float* rest = p.partials + ((size_t)(c_lo + 1) * 2) * (M * kBandCols);
  const size_t stride = (size_t)2 * M * kBandCols;
  const int n_rest = c_hi - c_lo;
  for (int e = threadIdx.x; e < M * kBandCols; e += blockDim.x) {
    const int m = e / kBandCols, c = e % kBandCols, col = col0 + c;
    float v = __ldcg(first + e);
    int q = 0;
    for (; q + 4 <= n_rest; q += 4) {   // independent loads, summed in contributor order
      const float a = __ldcg(rest + (size_t)q * stride + e);
      const float b = __ldcg(rest + (size_t)(q + 1) * stride + e);
      const float cc = __ldcg(rest + (size_t)(q + 2) * stride + e);
      const float d = __ldcg(rest + (size_t)(q + 3) * stride + e);
      v += a;
      v += b;
      v += cc;
      v += d;
    }
    for (; q < n_rest; ++q) v += __ldcg(rest + (size_t)q * stride + e);
    if (col < p.N) {
      if (p.bias) v += __half2float(p.bias[col]);
      p.y[(size_t)m * p.N + col] = __float2half_rn(v);
    }
  }
}

// ---------------------------------------------------------------------------
// M = 1: 8 lanes x 4 words (16-byte loads) per band row, 16 lane-groups.
__global__ void __launch_bounds__(kThreads, 3) gemv_m1_kernel(const GemmParams p) {
  constexpr int WPT = 4, LPR = 8, LG = kThreads / LPR;
  __shared__ float red[LG][kBandCols + 4];
  __shared__ float seg[kBandCols];
  __shared__ int s_flag;
  const int lane_in_row = threadIdx.x % LPR;
  const int lg = threadIdx.x / LPR;
  const long long P = gridDim.x;
  const long long it0 = range_begin(blockIdx.x, p.items, P);
  const long long it1 = range_begin(blockIdx.x + 1, p.items, P);
  uint32_t bad = 0;

  for (long long it = it0; it < it1;) {
    const int band = (int)(it / p.slots);
    const int s0 = (int)(it % p.slots);
    const long long seg_end = min(it1, (long long)(band + 1) * p.slots);
    const int s1 = (int)(seg_end - (long long)band * p.slots);
    const int w0 = band * kBandWords + lane_in_row * WPT;
    const bool active = w0 < p.W8;
    float acc[WPT * 8];
#pragma unroll
    for (int j = 0; j < WPT * 8; ++j) acc[j] = 0.0f;

    if (active) {
      for (int s = s0 + lg; s < s1; s += LG) {
        const int k0 = s * kSlotRows;
        const int g = k0 / p.G;
        Words<4> q[kSlotRows];
#pragma unroll
        for (int r = 0; r < kSlotRows; ++r)
          q[r].load_stream(p.qweight + (size_t)(k0 + r) * p.W8 + w0);
        Words<4> z;
        z.load_ro(p.qzeros + (size_t)g * p.W8 + w0);
        const uint4 xa = ld_ro_v4(p.x + k0);
        const uint4 xb = ld_ro_v4(p.x + k0 + 8);
        uint4 sc[WPT];
#pragma unroll
        for (int i = 0; i < WPT; ++i) sc[i] = ld_ro_v4(p.scales + (size_t)g * p.N + 8 * (w0 + i));

        ZeroPoint zp[WPT];
#pragma unroll
        for (int i = 0; i < WPT; ++i) zp[i] = make_zero_point(z.w[i]);
        float part[WPT * 8];   // the slot's sums of x (q - z), fp32
#pragma unroll
        for (int j = 0; j < WPT * 8; ++j) part[j] = 0.0f;
#pragma unroll
        for (int r = 0; r < kSlotRows; ++r) {
          const __half xx = __low2half(bcast_half(r < 8 ? xa : xb, r & 7));
#pragma unroll
          for (int i = 0; i < WPT; ++i) {
            half2 d[4];
            unpack_deltas(q[r].w[i], zp[i], d);
#pragma unroll
            for (int e = 0; e < 4; ++e) fma2_f32_f16(part[i * 8 + 2 * e], part[i * 8 + 2 * e + 1], d[e], xx);
          }
        }
        if (k0 % p.G == 0) {   // each (group, column) scale is checked exactly once
#pragma unroll
          for (int i = 0; i < WPT; ++i)
            bad |= invalid_scale_pair(sc[i].x) | invalid_scale_pair(sc[i].y) |
                   invalid_scale_pair(sc[i].z) | invalid_scale_pair(sc[i].w);
        }
#pragma unroll
        for (int i = 0; i < WPT; ++i) {
          const uint32_t sw[4] = {sc[i].x, sc[i].y, sc[i].z, sc[i].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 s2 = __half22float2(u32_as_half2(sw[e]));
            acc[i * 8 + 2 * e] = fmaf(part[i * 8 + 2 * e], s2.x, acc[i * 8 + 2 * e]);
            acc[i * 8 + 2 * e + 1] = fmaf(part[i * 8 + 2 * e + 1], s2.y, acc[i * 8 + 2 * e + 1]);
          }
        }
      }
    }
    // Reduce the lane-groups in a fixed order.
#pragma unroll
    for (int j = 0; j < WPT * 8; j += 4)
      *reinterpret_cast<float4*>(&red[lg][lane_in_row * WPT * 8 + j]) =
          make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
    __syncthreads();
    for (int c = threadIdx.x; c < kBandCols; c += blockDim.x) {
      float v = 0.0f;
#pragma unroll
      for (int l = 0; l < LG; ++l) v += red[l][c];
      seg[c] = v;
    }
    __syncthreads();
    finish_segment<1>(p, seg, band, s0 == 0 && s1 == p.slots, it, &s_flag);
    __syncthreads();
    it = seg_end;
  }
  if (bad && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SCALE);
}

// ---------------------------------------------------------------------------
// 2 <= M <= 8: one warp per band row (1 word per lane), 4 warps; activations of
// the slot are staged transposed in shared memory, xs[warp][row][m].
template <int M>
__global__ void __launch_bounds__(kThreads) gemm_smallm_kernel(const GemmParams p) {
  constexpr int LG = kThreads / 32;
  __shared__ float red[LG][M][kBandCols + 4];
  __shared__ float seg[M * kBandCols];
  __shared__ __align__(16) __half xs[LG][kSlotRows][8];
  __shared__ int s_flag;
  const int lane = threadIdx.x % 32;
  const int lg = threadIdx.x / 32;
  const long long P = gridDim.x;
  const long long it0 = range_begin(blockIdx.x, p.items, P);
  const long long it1 = range_begin(blockIdx.x + 1, p.items, P);
  uint32_t bad = 0;

  for (long long it = it0; it < it1;) {
    const int band = (int)(it / p.slots);
    const int s0 = (int)(it % p.slots);
    const long long seg_end = min(it1, (long long)(band + 1) * p.slots);
    const int s1 = (int)(seg_end - (long long)band * p.slots);
    const int w0 = band * kBandWords + lane;
    const bool active = w0 < p.W8;
    float acc[M][8];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[m][j] = 0.0f;

    for (int s = s0 + lg; s < s1; s += LG) {   // warp-uniform loop
      const int k0 = s * kSlotRows;
      const int g = k0 / p.G;
      uint32_t q[kSlotRows];
      if (active) {
#pragma unroll
        for (int r = 0; r < kSlotRows; ++r)
          q[r] = ld_stream_u32(p.qweight + (size_t)(k0 + r) * p.W8 + w0);
      }
      __syncwarp();
      if (lane < 2 * M) {   // stage x[m][k0..k0+16) transposed
        const int m = lane >> 1, h = lane & 1;
        const uint4 v = ld_ro_v4(p.x + (size_t)m * p.K + k0 + 8 * h);
        const __half* hv = reinterpret_cast<const __half*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) xs[lg][8 * h + j][m] = hv[j];
      }
      __syncwarp();
      if (active) {
        const uint32_t zw = __ldg(reinterpret_cast<const unsigned int*>(p.qzeros + (size_t)g * p.W8 + w0));
        const uint4 sc = ld_ro_v4(p.scales + (size_t)g * p.N + 8 * w0);
        const ZeroPoint zp = make_zero_point(zw);
        float part[M][8];   // the slot's sums of x (q - z), fp32
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
          for (int j = 0; j < 8; ++j) part[m][j] = 0.0f;
#pragma unroll
        for (int r = 0; r < kSlotRows; ++r) {
          half2 d[4];
          unpack_deltas(q[r], zp, d);
          const uint4 xr = *reinterpret_cast<const uint4*>(&xs[lg][r][0]);
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const __half xx = __low2half(bcast_half(xr, m));
#pragma unroll
            for (int e = 0; e < 4; ++e) fma2_f32_f16(part[m][2 * e], part[m][2 * e + 1], d[e], xx);
          }
        }
        if (k0 % p.G == 0)
          bad |= invalid_scale_pair(sc.x) | invalid_scale_pair(sc.y) |
                 invalid_scale_pair(sc.z) | invalid_scale_pair(sc.w);
        const uint32_t sw[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 s2 = __half22float2(u32_as_half2(sw[e]));
#pragma unroll
          for (int m = 0; m < M; ++m) {
            acc[m][2 * e] = fmaf(part[m][2 * e], s2.x, acc[m][2 * e]);
            acc[m][2 * e + 1] = fmaf(part[m][2 * e + 1], s2.y, acc[m][2 * e + 1]);
          }
        }
      }
      __syncwarp();
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      *reinterpret_cast<float4*>(&red[lg][m][lane * 8]) =
          make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
      *reinterpret_cast<float4*>(&red[lg][m][lane * 8 + 4]) =
          make_float4(acc[m][4], acc[m][5], acc[m][6], acc[m][7]);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < M * kBandCols; e += blockDim.x) {
      const int m = e / kBandCols, c = e % kBandCols;
      float v = 0.0f;
#pragma unroll
      for (int l = 0; l < LG; ++l) v += red[l][m][c];
      seg[e] = v;
    }
    __syncthreads();
    finish_segment<M>(p, seg, band, s0 == 0 && s1 == p.slots, it, &s_flag);
    __syncthreads();
    it = seg_end;
  }
  if (bad && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SCALE);
}

// ---------------------------------------------------------------------------
// Reference-order kernel: one thread per (row m, output column c), sequential
// k, every binary32 operation rounded separately (no FMA contraction), as in
// FP32Model.linear.  Bit-identical to the reference before the output store;
// OutT = float keeps it, OutT = __half rounds it once (the fallback for shapes
// the fast kernels do not take).
__device__ __forceinline__ void store_out(float* y, long long i, float v) { y[i] = v; }
__device__ __forceinline__ void store_out(__half* y, long long i, float v) { y[i] = __float2half_rn(v); }

template <typename OutT>
__global__ void gemm_exact_kernel(const __half* __restrict__ x, const int32_t* __restrict__ qweight,
                                  const int32_t* __restrict__ qzeros, const __half* __restrict__ scales,
                                  const __half* __restrict__ bias, OutT* __restrict__ y,
                                  int M, int K, int N, int G, int* dev_err) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)M * N) return;
  const int m = (int)(idx / N), c = (int)(idx % N);
  const int W8 = N / 8, word = c / 8, lane = c % 8;
  const int shift = (0x73625140 >> (4 * lane)) & 0xF;   // nibble index of lane: 0,4,1,5,2,6,3,7
  float total = 0.0f;
  bool bad = false;
  for (int k = 0; k < K; ++k) {
    const int g = k / G;
    const __half hs = scales[(size_t)g * N + c];
    const uint16_t hb = __half_as_ushort(hs);
    if (((hb >> 10) & 31) == 31 || ((hb & 0x8000) && (hb & 0x7FFF))) { bad = true; break; }
    const uint32_t qw = (uint32_t)qweight[(size_t)k * W8 + word];
    const uint32_t qz = (uint32_t)qzeros[(size_t)g * W8 + word];
    const int delta = (int)((qw >> (4 * shift)) & 15u) - (int)((qz >> (4 * shift)) & 15u);
    const float weight = __fmul_rn((float)delta, __half2float(hs));
    const float product = __fmul_rn(__half2float(x[(size_t)m * K + k]), weight);
    total = __fadd_rn(total, product);
  }
  if (!bad && bias) total = __fadd_rn(total, __half2float(bias[c]));
  store_out(y, idx, bad ? 0.0f : total);
  if (bad && dev_err) atomicOr(dev_err, ANVILQ_DEV_ERR_SCALE);
}

// ---------------------------------------------------------------------------
// Dequantiser: one thread per (row k, packed word), through unpack_deltas.
__global__ void dequant_kernel(const int32_t* __restrict__ qweight, const int32_t* __restrict__ qzeros,
                               const __half* __restrict__ scales, int8_t* __restrict__ delta_out,
                               float* __restrict__ w_out, int K, int N, int G, int* dev_err) {
  const int W8 = N / 8;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)K * W8) return;
  const int k = (int)(idx / W8), w = (int)(idx % W8), g = k / G;
  const ZeroPoint zp = make_zero_point((uint32_t)qzeros[(size_t)g * W8 + w]);
  half2 d[4];
  unpack_deltas((uint32_t)qweight[idx], zp, d);
  uint32_t bad = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int c = 8 * w + 2 * e;
    const uint32_t s = *reinterpret_cast<const uint32_t*>(scales + (size_t)g * N + c);
    const uint32_t b = invalid_scale_pair(s);
    bad |= b;
    const float2 df = __half22float2(d[e]);
    const float2 sf = __half22float2(u32_as_half2(s));
    if (delta_out) {
      delta_out[(size_t)k * N + c] = (int8_t)df.x;
      delta_out[(size_t)k * N + c + 1] = (int8_t)df.y;
    }
    if (w_out) {
      w_out[(size_t)k * N + c] = (b & 0x8000u) ? 0.0f : __fmul_rn(df.x, sf.x);
      w_out[(size_t)k * N + c + 1] = (b & 0x80000000u) ? 0.0f : __fmul_rn(df.y, sf.y);
    }
  }
  if (bad && dev_err) atomicOr(dev_err, ANVILQ_DEV_ERR_SCALE);
}

__global__ void pack_kernel(const uint8_t* __restrict__ codes, int32_t* __restrict__ packed, long long words) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= words) return;
  const uint8_t* c = codes + idx * 8;
  uint32_t w = 0;
#pragma unroll
  for (int lane = 0; lane < 8; ++lane) {
    const int nib = (0x73625140 >> (4 * lane)) & 0xF;
    w |= (uint32_t)(c[lane] & 15u) << (4 * nib);
  }
  packed[idx] = (int32_t)w;
}

__global__ void unpack_kernel(const int32_t* __restrict__ packed, uint8_t* __restrict__ codes, long long words) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= words) return;
  const uint32_t w = (uint32_t)packed[idx];
#pragma unroll
  for (int lane = 0; lane < 8; ++lane) {
    const int nib = (0x73625140 >> (4 * lane)) & 0xF;
    codes[idx * 8 + lane] = (uint8_t)((w >> (4 * nib)) & 15u);
  }
}

// ---------------------------------------------------------------------------
// Host side.
struct DeviceInfo {
  int sms = 0;
  int occ_m1 = 0;
  int occ_small[9] = {0};
};

constexpr int kMaxDevices = 64;
static DeviceInfo g_info[kMaxDevices];
static std::once_flag g_once[kMaxDevices];

static const DeviceInfo* device_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(g_once[dev], [dev] {
    DeviceInfo& d = g_info[dev];
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.occ_m1, gemv_m1_kernel, kThreads, 0);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.occ_small[2], gemm_smallm_kernel<2>, kThreads, 0);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.occ_small[3], gemm_smallm_kernel<3>, kThreads, 0);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.occ_small[4], gemm_smallm_kernel<4>, kThreads, 0);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.occ_small[5], gemm_smallm_kernel<5>, kThreads, 0);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.occ_small[6], gemm_smallm_kernel<6>, kThreads, 0);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.occ_small[7], gemm_smallm_kernel<7>, kThreads, 0);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.occ_small[8], gemm_smallm_kernel<8>, kThreads, 0);
    cudaGetLastError();
  });
  return &g_info[dev];
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static bool fast_path_ok(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                         const uint16_t* scales, int M, int K, int N, int G) {
  (void)M;
  return G % kSlotRows == 0 && K % kSlotRows == 0 && N % 32 == 0 && aligned16(x) &&
         aligned16(qweight) && aligned16(qzeros) && aligned16(scales);
}

struct Plan {
  int chunk_m;      // rows per launch (1 or 2..8)
  int grid;         // persistent CTAs
  int bands, slots;
  long long items;
  size_t partial_floats, bytes;
};

static Plan plan_for(const DeviceInfo& d, int M, int K, int N) {
  Plan pl{};
  pl.chunk_m = M <= 1 ? 1 : std::min(M, 8);
  pl.bands = (N / 8 + kBandWords - 1) / kBandWords;
  pl.slots = K / kSlotRows;
  pl.items = (long long)pl.bands * pl.slots;
  const int occ = pl.chunk_m == 1 ? d.occ_m1 : d.occ_small[pl.chunk_m];
  long long grid = (long long)d.sms * std::max(occ, 1);
  // at least 8 slots (16 KB of int4 data) per CTA bounds the contributors per band
  grid = std::max<long long>(1, std::min<long long>(grid, pl.items / 8));
  pl.grid = (int)grid;
  pl.partial_floats = (size_t)pl.grid * 2 * pl.chunk_m * kBandCols;
  pl.bytes = ANVILQ_WORKSPACE_COUNTER_BYTES + pl.partial_floats * sizeof(float);
  return pl;
}

static int launch_fast(const Plan& pl, const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                       const uint16_t* scales, const uint16_t* bias, uint16_t* y, int M, int K, int N,
                       int G, void* workspace, int* dev_err, cudaStream_t stream) {
  GemmParams p;
  p.qweight = qweight;
  p.qzeros = qzeros;
  p.scales = reinterpret_cast<const __half*>(scales);
  p.bias = reinterpret_cast<const __half*>(bias);
  // counters first (left zero by every call), partial sums after them
  p.tickets = reinterpret_cast<int*>(workspace);
  p.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + ANVILQ_WORKSPACE_COUNTER_BYTES);
  p.dev_err = dev_err;
  p.K = K; p.N = N; p.W8 = N / 8; p.G = G;
  p.bands = pl.bands; p.slots = pl.slots; p.items = pl.items;
  for (int m0 = 0; m0 < M; m0 += pl.chunk_m) {
    const int mc = std::min(pl.chunk_m, M - m0);
    p.x = reinterpret_cast<const __half*>(x) + (size_t)m0 * K;
    p.y = reinterpret_cast<__half*>(y) + (size_t)m0 * N;
    switch (mc) {
      case 1: gemv_m1_kernel<<<pl.grid, kThreads, 0, stream>>>(p); break;
      case 2: gemm_smallm_kernel<2><<<pl.grid, kThreads, 0, stream>>>(p); break;
      case 3: gemm_smallm_kernel<3><<<pl.grid, kThreads, 0, stream>>>(p); break;
      case 4: gemm_smallm_kernel<4><<<pl.grid, kThreads, 0, stream>>>(p); break;
      case 5: gemm_smallm_kernel<5><<<pl.grid, kThreads, 0, stream>>>(p); break;
      case 6: gemm_smallm_kernel<6><<<pl.grid, kThreads, 0, stream>>>(p); break;
      case 7: gemm_smallm_kernel<7><<<pl.grid, kThreads, 0, stream>>>(p); break;
      default: gemm_smallm_kernel<8><<<pl.grid, kThreads, 0, stream>>>(p); break;
    }
    if (cudaGetLastError() != cudaSuccess) return ANVILQ_ECUDA;
  }
  return ANVILQ_OK;
}

static bool shape_ok(int M, int K, int N, int G) {
  return M >= 1 && K >= 1 && N >= 8 && N % 8 == 0 && G >= 1;
}

template <typename OutT>
static int launch_exact(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                        const uint16_t* scales, const uint16_t* bias, OutT* y, int M, int K, int N,
                        int G, int* dev_err, cudaStream_t stream) {
  const long long n = (long long)M * N;
  const int threads = 128;
  gemm_exact_kernel<OutT><<<(unsigned)((n + threads - 1) / threads), threads, 0, stream>>>(
      reinterpret_cast<const __half*>(x), qweight, qzeros, reinterpret_cast<const __half*>(scales),
      reinterpret_cast<const __half*>(bias), y, M, K, N, G, dev_err);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}

}  // namespace anvilq

using namespace anvilq;

// The M = 1 plan: the stream-K kernel for deep layers (K >= 8192) of at least
// kStreamMinBytes of int4 weights, the cluster kernel otherwise.  Measured on
// B200 (CUDA graph, L2-cold): stream-K wins 3-52 % on 8192x3584 .. 28672x8192
// and 28672x1024 (the cluster kernel's deep-K split costs a fix-up per band),
// the cluster kernel wins 4-20 % on the K = 4096 layers of 7B-class models and
// on every decode-size (0.5B) layer.
static constexpr long long kStreamMinBytes = 12ll << 20;
static constexpr int kStreamMinK = 8192;
static bool default_gemv_plan(const void* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                              int K, int N, int G, GemvPlan* plan) {
  if (K >= kStreamMinK && (long long)K * N / 2 >= kStreamMinBytes &&
      gemv_stream_supported(x, qweight, qzeros, scales, K, N, G) &&
      gemv_stream_default_plan(K, N, plan) && gemv_stream_check_plan(K, N, *plan) == ANVILQ_OK)
    return true;
  return gemv_tma_supported(x, qweight, qzeros, scales, K, N, G) && gemv_cluster_default_plan(K, N, plan);
}

extern "C" {

int anvilq_abi_version(void) { return ANVILQ_ABI_VERSION; }

const char* anvilq_strerror(int status) {
  switch (status) {
    case ANVILQ_OK: return "ok";
    case ANVILQ_EINVAL: return "invalid argument (null pointer or inconsistent size)";
    case ANVILQ_EALIGN: return "pointer alignment required by the kernel is missing";
    case ANVILQ_ECUDA: return "CUDA kernel launch failed";
    case ANVILQ_EWORKSPACE: return "workspace missing or too small";
    case ANVILQ_ESHAPE: return "shape outside the supported range";
    case ANVILQ_ENOSCRATCH: return "request needs more scratch than the fixed no-allocation buffer holds";
    default: return "unknown anvilq status";
  }
}

size_t anvilq_w4a16_gemm_workspace_size(int M, int K, int N, int G) {
  if (!shape_ok(M, K, N, G)) return 0;
  const DeviceInfo* d = device_info();
  if (!d) return 0;
  size_t b = plan_for(*d, M, K, N).bytes;
  if (M == 1) {
    b = std::max(b, gemv_tma_workspace_bytes(K, N));
    GemvPlan sp;
    if (gemv_stream_default_plan(K, N, &sp)) b = std::max(b, gemv_stream_workspace_bytes(sp));
  }
  // the tensor-core path may serve any M (anvilq_w4a16_verify_gemm)
  if (G == 128 && K % 128 == 0 && N % 32 == 0) b = std::max(b, verify_tc_workspace_bytes(M, K, N));
  return b;
}

int anvilq_w4a16_gemm(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                      const uint16_t* scales, const uint16_t* bias, uint16_t* y,
                      int M, int K, int N, int G, void* workspace, size_t workspace_bytes,
                      int* dev_err, anvilq_stream_t stream) {
  return anvilq_w4a16_gemm_ex(x, qweight, qzeros, scales, bias, y, M, K, N, G, workspace, workspace_bytes,
                              dev_err, 0u, stream);
}

int anvilq_w4a16_gemm_ex(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                         const uint16_t* scales, const uint16_t* bias, uint16_t* y,
                         int M, int K, int N, int G, void* workspace, size_t workspace_bytes,
                         int* dev_err, unsigned flags, anvilq_stream_t stream) {
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  if (!x || !qweight || !qzeros || !scales || !y) return ANVILQ_EINVAL;
  if (!shape_ok(M, K, N, G)) return ANVILQ_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (!fast_path_ok(x, qweight, qzeros, scales, M, K, N, G))
    return launch_exact(x, qweight, qzeros, scales, bias, reinterpret_cast<__half*>(y), M, K, N, G,
                        dev_err, s);
  if (M == 1) {
    GemvPlan pl;
    if (default_gemv_plan(x, qweight, qzeros, scales, K, N, G, &pl)) {
      const bool overlap = (flags & ANVILQ_GEMM_OVERLAP_PRIOR) != 0;
      if (pl.kernel == ANVILQ_GEMV_KERNEL_STREAM)
        return launch_gemv_stream(pl, x, qweight, qzeros, scales, bias, y, K, N, G, workspace, workspace_bytes,
                                  dev_err, s, overlap);
      GemvIo io;
      io.x = x;
      io.y = y;
      return launch_gemv_tma(io, qweight, qzeros, scales, bias, K, N, G, workspace, workspace_bytes, dev_err, s,
                             overlap);
    }
  }
  if (M >= ANVILQ_VERIFY_TC_MIN_M && verify_tc_supported(x, qweight, qzeros, scales, M, K, N, G))
    return launch_verify_tc(x, qweight, nullptr, qzeros, scales, bias, y, M, K, N, workspace, workspace_bytes,
                            dev_err, s, (flags & ANVILQ_GEMM_OVERLAP_PRIOR) != 0);
  const DeviceInfo* d = device_info();
  if (!d) return ANVILQ_ECUDA;
  const Plan pl = plan_for(*d, M, K, N);
  if ((size_t)pl.bands * sizeof(int) > ANVILQ_WORKSPACE_COUNTER_BYTES) return ANVILQ_ESHAPE;
  if (!workspace || workspace_bytes < pl.bytes) return ANVILQ_EWORKSPACE;
  if (!aligned16(workspace)) return ANVILQ_EALIGN;
  return launch_fast(pl, x, qweight, qzeros, scales, bias, y, M, K, N, G, workspace, dev_err, s);
}

int anvilq_w4a16_gemv_plan(int K, int N, int G, anvilq_gemv_plan* plan) {
  if (!plan || !shape_ok(1, K, N, G)) return ANVILQ_EINVAL;
  // any 16-byte aligned operands: the plan depends on the shape only
  const void* a = reinterpret_cast<const void*>(uintptr_t(256));
  if (!default_gemv_plan(a, static_cast<const int32_t*>(a), static_cast<const int32_t*>(a),
                         static_cast<const uint16_t*>(a), K, N, G, plan))
    return ANVILQ_ESHAPE;
  return ANVILQ_OK;
}

int anvilq_w4a16_gemv_kernel_plan(int kernel, int K, int N, int G, anvilq_gemv_plan* plan) {
  if (!plan || !shape_ok(1, K, N, G)) return ANVILQ_EINVAL;
  const void* a = reinterpret_cast<const void*>(uintptr_t(256));
  const int32_t* w = static_cast<const int32_t*>(a);
  const uint16_t* h = static_cast<const uint16_t*>(a);
  if (kernel == ANVILQ_GEMV_KERNEL_STREAM)
    return gemv_stream_supported(a, w, w, h, K, N, G) && gemv_stream_default_plan(K, N, plan) &&
                   gemv_stream_check_plan(K, N, *plan) == ANVILQ_OK
               ? ANVILQ_OK
               : ANVILQ_ESHAPE;
  if (kernel == ANVILQ_GEMV_KERNEL_CLUSTER)
    return gemv_tma_supported(a, w, w, h, K, N, G) && gemv_cluster_default_plan(K, N, plan) ? ANVILQ_OK
                                                                                           : ANVILQ_ESHAPE;
  return ANVILQ_EINVAL;
}

size_t anvilq_w4a16_gemv_plan_workspace_size(int K, int N, int G, const anvilq_gemv_plan* plan) {
  if (!plan || !shape_ok(1, K, N, G)) return 0;
  GemvPlan pl = *plan;
  if (pl.kernel == ANVILQ_GEMV_KERNEL_STREAM)
    return gemv_stream_check_plan(K, N, pl) == ANVILQ_OK ? gemv_stream_workspace_bytes(pl) : 0;
  if (pl.kernel == ANVILQ_GEMV_KERNEL_CLUSTER)
    return gemv_cluster_check_plan(K, N, &pl) == ANVILQ_OK ? gemv_cluster_workspace_bytes(K, N, pl) : 0;
  return 0;
}

int anvilq_w4a16_gemv_planned(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                              const uint16_t* scales, const uint16_t* bias, uint16_t* y, int K, int N, int G,
                              const anvilq_gemv_plan* plan, void* workspace, size_t workspace_bytes,
                              int* dev_err, unsigned flags, anvilq_stream_t stream) {
  if (!x || !qweight || !qzeros || !scales || !y || !plan) return ANVILQ_EINVAL;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  if (!shape_ok(1, K, N, G)) return ANVILQ_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool overlap = (flags & ANVILQ_GEMM_OVERLAP_PRIOR) != 0;
  GemvPlan pl = *plan;
  if (pl.kernel == ANVILQ_GEMV_KERNEL_STREAM) {
    if (!aligned16(y) || !gemv_stream_supported(x, qweight, qzeros, scales, K, N, G)) return ANVILQ_ESHAPE;
    return launch_gemv_stream(pl, x, qweight, qzeros, scales, bias, y, K, N, G, workspace, workspace_bytes,
                              dev_err, s, overlap);
  }
  if (pl.kernel != ANVILQ_GEMV_KERNEL_CLUSTER) return ANVILQ_EINVAL;
  const int rc = gemv_cluster_check_plan(K, N, &pl);
  if (rc != ANVILQ_OK) return rc;
  if (!gemv_tma_supported(x, qweight, qzeros, scales, K, N, G)) return ANVILQ_ESHAPE;
  GemvIo io;
  io.x = x;
  io.y = y;
  return launch_gemv_tma(io, qweight, qzeros, scales, bias, K, N, G, workspace, workspace_bytes, dev_err, s,
                         overlap, &pl);
}

int anvilq_w4a16_verify_gemm(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                             const uint16_t* scales, const uint16_t* bias, uint16_t* y,
                             int M, int K, int N, int G, void* workspace, size_t workspace_bytes,
                             int* dev_err, anvilq_stream_t stream) {
  if (!x || !qweight || !qzeros || !scales || !y) return ANVILQ_EINVAL;
  if (!shape_ok(M, K, N, G)) return ANVILQ_EINVAL;
  if (!verify_tc_supported(x, qweight, qzeros, scales, M, K, N, G)) return ANVILQ_ESHAPE;
  return launch_verify_tc(x, qweight, nullptr, qzeros, scales, bias, y, M, K, N, workspace, workspace_bytes,
                          dev_err, reinterpret_cast<cudaStream_t>(stream));
}

size_t anvilq_w4a16_tc_pack_size(int K, int N, int G) {
  return G == 128 ? tc_pack_bytes(K, N) : 0;
}

int anvilq_w4a16_tc_pack(const int32_t* qweight, int32_t* packed, int K, int N, int G, anvilq_stream_t stream) {
  if (!qweight || !packed) return ANVILQ_EINVAL;
  if (!shape_ok(1, K, N, G)) return ANVILQ_EINVAL;
  if (anvilq_w4a16_tc_pack_size(K, N, G) == 0) return ANVILQ_ESHAPE;
  return launch_tc_pack(qweight, packed, K, N, reinterpret_cast<cudaStream_t>(stream));
}

int anvilq_w4a16_verify_gemm_packed(const uint16_t* x, const int32_t* packed, const int32_t* qzeros,
                                    const uint16_t* scales, const uint16_t* bias, uint16_t* y, int M, int K,
                                    int N, int G, void* workspace, size_t workspace_bytes, int* dev_err,
                                    anvilq_stream_t stream) {
  if (!x || !packed || !qzeros || !scales || !y) return ANVILQ_EINVAL;
  if (!shape_ok(M, K, N, G)) return ANVILQ_EINVAL;
  if (!aligned16(packed) || !verify_tc_supported(x, packed, qzeros, scales, M, K, N, G)) return ANVILQ_ESHAPE;
  return launch_verify_tc(x, nullptr, packed, qzeros, scales, bias, y, M, K, N, workspace, workspace_bytes,
                          dev_err, reinterpret_cast<cudaStream_t>(stream));
}

int anvilq_w4a16_gemv_fused(const void* x, int x_mode, const uint16_t* gamma, float eps,
                            const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                            const uint16_t* bias, void* y, int y_mode, int K, int N, int G, void* workspace,
                            size_t workspace_bytes, int* dev_err, unsigned flags, anvilq_stream_t stream) {
  if (!x || !qweight || !qzeros || !scales || !y) return ANVILQ_EINVAL;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  if (x_mode < ANVILQ_GEMV_X_HALF || x_mode > ANVILQ_GEMV_X_SILU_MUL) return ANVILQ_EINVAL;
  if (y_mode < ANVILQ_GEMV_Y_HALF || y_mode > ANVILQ_GEMV_Y_SILU_MUL) return ANVILQ_EINVAL;
  if (x_mode == ANVILQ_GEMV_X_RMSNORM && (!gamma || !(eps >= 0.0f))) return ANVILQ_EINVAL;
  if (y_mode == ANVILQ_GEMV_Y_SILU_MUL && (x_mode == ANVILQ_GEMV_X_SILU_MUL || bias || N % 64))
    return ANVILQ_EINVAL;
  if (!shape_ok(1, K, N, G)) return ANVILQ_EINVAL;
  const bool a16 = aligned16(x) && aligned16(y) && (!gamma || aligned16(gamma));
  if (!a16 || !gemv_tma_supported(x, qweight, qzeros, scales, K, N, G)) return ANVILQ_ESHAPE;
  GemvIo io;
  io.xmode = x_mode;
  io.ymode = y_mode == ANVILQ_GEMV_Y_SILU_MUL ? 5 : y_mode;   // the kernel's activation epilogue
  io.x = static_cast<const uint16_t*>(x);
  io.xr = static_cast<const float*>(x);
  io.gamma = gamma;
  io.eps = eps;
  io.y = static_cast<uint16_t*>(y);
  io.yr = static_cast<float*>(y);
  return launch_gemv_tma(io, qweight, qzeros, scales, bias, K, N, G, workspace, workspace_bytes, dev_err,
                         reinterpret_cast<cudaStream_t>(stream), (flags & ANVILQ_GEMM_OVERLAP_PRIOR) != 0);
}

size_t anvilq_w4a16_mlp_workspace_size(int H, int I, int G) {
  if (H <= 0 || I <= 0 || G <= 0) return 0;
  // the partial outputs of every band of at least 16 words (128 gate/up columns)
  return ANVILQ_WORKSPACE_COUNTER_BYTES + (size_t)((2 * (size_t)I / 8 + 15) / 16) * H * sizeof(float);
}

int anvilq_w4a16_mlp(float* r, const uint16_t* gamma, float eps, const int32_t* gu_qweight,
                     const int32_t* gu_qzeros, const uint16_t* gu_scales, const int32_t* dn_qweight,
                     const int32_t* dn_qzeros, const uint16_t* dn_scales, int H, int I, int G, void* workspace,
                     size_t workspace_bytes, int* dev_err, unsigned flags, anvilq_stream_t stream) {
  if (!r || !gamma || !gu_qweight || !gu_qzeros || !gu_scales || !dn_qweight || !dn_qzeros || !dn_scales)
    return ANVILQ_EINVAL;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  if (!(eps >= 0.0f) || I <= 0 || I % 32 || !shape_ok(1, H, 2 * I, G) || !shape_ok(1, I, H, G)) return ANVILQ_EINVAL;
  if (!aligned16(r) || !aligned16(gamma) || !gemv_tma_supported(r, gu_qweight, gu_qzeros, gu_scales, H, 2 * I, G))
    return ANVILQ_ESHAPE;
  GemvIo io;
  io.xmode = 1;   // RMSNorm of the residual
  io.ymode = 4;   // the MLP epilogue
  io.xr = r;
  io.gamma = gamma;
  io.eps = eps;
  io.yr = r;
  io.dn_qweight = dn_qweight;
  io.dn_qzeros = dn_qzeros;
  io.dn_scales = dn_scales;
  io.dn_H = H;
  return launch_gemv_tma(io, gu_qweight, gu_qzeros, gu_scales, nullptr, H, 2 * I, G, workspace, workspace_bytes,
                         dev_err, reinterpret_cast<cudaStream_t>(stream), (flags & ANVILQ_GEMM_OVERLAP_PRIOR) != 0);
}

int anvilq_w4a16_gemv_qkv_rope(const void* x, int x_mode, const uint16_t* gamma, float eps,
                               const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                               const uint16_t* bias, int K, int G, const int32_t* pos, uint16_t* q_out,
                               uint16_t* k_cache, uint16_t* v_cache, int32_t* seqlen, int Hq, int Hkv, int D,
                               int Tmax, float theta, void* workspace, size_t workspace_bytes, int* dev_err,
                               unsigned flags, anvilq_stream_t stream) {
  if (!x || !qweight || !qzeros || !scales || !pos || !q_out || !k_cache || !v_cache) return ANVILQ_EINVAL;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  if (x_mode < ANVILQ_GEMV_X_HALF || x_mode > ANVILQ_GEMV_X_SILU_MUL) return ANVILQ_EINVAL;
  if (x_mode == ANVILQ_GEMV_X_RMSNORM && (!gamma || !(eps >= 0.0f))) return ANVILQ_EINVAL;
  if (Hq < 1 || Hkv < 1 || Hq % Hkv || D < 2 || D % 2 || Tmax < 1 || !(theta > 0.0f)) return ANVILQ_EINVAL;
  const long long n = (long long)(Hq + 2 * Hkv) * D;
  if (n > (1 << 24)) return ANVILQ_ESHAPE;
  const int N = (int)n;
  if (!shape_ok(1, K, N, G)) return ANVILQ_EINVAL;
  const bool a16 = aligned16(x) && (!gamma || aligned16(gamma));
  if (!a16 || !gemv_tma_supported(x, qweight, qzeros, scales, K, N, G)) return ANVILQ_ESHAPE;
  GemvIo io;
  io.xmode = x_mode;
  io.ymode = 2;
  io.x = static_cast<const uint16_t*>(x);
  io.xr = static_cast<const float*>(x);
  io.gamma = gamma;
  io.eps = eps;
  io.rope_pos = pos;
  io.q_out = q_out;
  io.k_cache = k_cache;
  io.v_cache = v_cache;
  io.seqlen = seqlen;
  io.Hq = Hq;
  io.Hkv = Hkv;
  io.D = D;
  io.Tmax = Tmax;
  io.theta = theta;
  return launch_gemv_tma(io, qweight, qzeros, scales, bias, K, N, G, workspace, workspace_bytes, dev_err,
                         reinterpret_cast<cudaStream_t>(stream), (flags & ANVILQ_GEMM_OVERLAP_PRIOR) != 0);
}

int anvilq_w4a16_gemv_allgather(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                                const uint16_t* scales, const uint16_t* bias, int K, int N, int G, int rank,
                                int world, int col_base, int n_full, uint16_t* const* peer_y,
                                unsigned int* const* peer_flags, unsigned int* epoch, void* workspace,
                                size_t workspace_bytes, int* dev_err, unsigned flags, anvilq_stream_t stream) {
  if (!x || !qweight || !qzeros || !scales || !peer_y || !peer_flags || !epoch) return ANVILQ_EINVAL;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  if (world < 1 || world > 8 || rank < 0 || rank >= world) return ANVILQ_EINVAL;
  if (!shape_ok(1, K, N, G)) return ANVILQ_EINVAL;
  if (col_base < 0 || col_base % 8 || n_full < col_base + N) return ANVILQ_EINVAL;
  for (int r = 0; r < world; ++r)
    if (!peer_y[r] || !peer_flags[r]) return ANVILQ_EINVAL;
  GemvPlan pl;
  if (!aligned16(x) || !default_gemv_plan(x, qweight, qzeros, scales, K, N, G, &pl)) return ANVILQ_ESHAPE;
  GemvIo io;
  io.xmode = 0;
  io.ymode = 3;
  io.x = x;
  for (int r = 0; r < world; ++r) {
    io.peer_y[r] = peer_y[r];
    io.peer_flags[r] = peer_flags[r];
  }
  io.epoch = epoch;
  io.world = world;
  io.tp_rank = rank;
  io.col_base = col_base;
  // the kernel and plan of anvilq_w4a16_gemm for this slice, so the fused call's
  // values are bit-identical to the GEMV followed by an all-gather
  const bool overlap = (flags & ANVILQ_GEMM_OVERLAP_PRIOR) != 0;
  if (pl.kernel == ANVILQ_GEMV_KERNEL_STREAM)
    return launch_gemv_stream(pl, x, qweight, qzeros, scales, bias, nullptr, K, N, G, workspace, workspace_bytes,
                              dev_err, reinterpret_cast<cudaStream_t>(stream), overlap, &io);
  return launch_gemv_tma(io, qweight, qzeros, scales, bias, K, N, G, workspace, workspace_bytes, dev_err,
                         reinterpret_cast<cudaStream_t>(stream), overlap);
}

int anvilq_w4a16_gemv_allgather_planned(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                                        const uint16_t* scales, const uint16_t* bias, int K, int N, int G,
                                        int rank, int world, int col_base, int n_full, uint16_t* const* peer_y,
                                        unsigned int* const* peer_flags, unsigned int* epoch,
                                        const anvilq_gemv_plan* plan, void* workspace, size_t workspace_bytes,
                                        int* dev_err, unsigned flags, anvilq_stream_t stream) {
  if (!x || !qweight || !qzeros || !scales || !peer_y || !peer_flags || !epoch || !plan) return ANVILQ_EINVAL;
  if (flags & ~(unsigned)(ANVILQ_GEMM_OVERLAP_PRIOR | ANVILQ_GATHER_DEFERRED)) return ANVILQ_EINVAL;
  if (world < 1 || world > 8 || rank < 0 || rank >= world) return ANVILQ_EINVAL;
  if (!shape_ok(1, K, N, G)) return ANVILQ_EINVAL;
  if (col_base < 0 || col_base % 8 || n_full < col_base + N) return ANVILQ_EINVAL;
  for (int r = 0; r < world; ++r)
    if (!peer_y[r] || !peer_flags[r]) return ANVILQ_EINVAL;
  const GemvPlan pl = *plan;
  if (pl.kernel != ANVILQ_GEMV_KERNEL_STREAM) return ANVILQ_EINVAL;
  if (!aligned16(x) || !gemv_stream_supported(x, qweight, qzeros, scales, K, N, G)) return ANVILQ_ESHAPE;
  GemvIo io;
  io.xmode = 0;
  io.ymode = 3;
  io.x = x;
  for (int r = 0; r < world; ++r) {
    io.peer_y[r] = peer_y[r];
    io.peer_flags[r] = peer_flags[r];
  }
  io.epoch = epoch;
  io.world = world;
  io.tp_rank = rank;
  io.col_base = col_base;
  io.deferred = (flags & ANVILQ_GATHER_DEFERRED) != 0;
  return launch_gemv_stream(pl, x, qweight, qzeros, scales, bias, nullptr, K, N, G, workspace, workspace_bytes,
                            dev_err, reinterpret_cast<cudaStream_t>(stream),
                            (flags & ANVILQ_GEMM_OVERLAP_PRIOR) != 0, &io);
}

int anvilq_peer_wait(const unsigned int* flags, int world, const unsigned int* epoch, int* dev_err,
                     anvilq_stream_t stream) {
  if (!flags || !epoch || world < 1 || world > 8) return ANVILQ_EINVAL;
  return launch_peer_wait(flags, world, epoch, dev_err, reinterpret_cast<cudaStream_t>(stream));
}

int anvilq_w4a16_gemm_exact(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                            const uint16_t* scales, const uint16_t* bias, float* y32,
                            int M, int K, int N, int G, int* dev_err, anvilq_stream_t stream) {
  if (!x || !qweight || !qzeros || !scales || !y32) return ANVILQ_EINVAL;
  if (!shape_ok(M, K, N, G)) return ANVILQ_EINVAL;
  return launch_exact(x, qweight, qzeros, scales, bias, y32, M, K, N, G, dev_err,
                      reinterpret_cast<cudaStream_t>(stream));
}

int anvilq_awq_dequant(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                       int8_t* delta_out, float* w_out, int K, int N, int G, int* dev_err,
                       anvilq_stream_t stream) {
  if (!qweight || !qzeros || !scales) return ANVILQ_EINVAL;
  if (K < 1 || N < 8 || N % 8 || G < 1) return ANVILQ_EINVAL;
  if ((reinterpret_cast<uintptr_t>(scales) & 3u) != 0) return ANVILQ_EALIGN;
  const long long n = (long long)K * (N / 8);
  const int threads = 256;
  dequant_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0,
                   reinterpret_cast<cudaStream_t>(stream)>>>(
      qweight, qzeros, reinterpret_cast<const __half*>(scales), delta_out, w_out, K, N, G, dev_err);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}

int anvilq_awq_pack(const uint8_t* codes, int32_t* packed, int rows, int N, anvilq_stream_t stream) {
  if (!codes || !packed || rows < 1 || N < 8 || N % 8) return ANVILQ_EINVAL;
  const long long words = (long long)rows * (N / 8);
  pack_kernel<<<(unsigned)((words + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      codes, packed, words);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}

int anvilq_awq_unpack(const int32_t* packed, uint8_t* codes, int rows, int N, anvilq_stream_t stream) {
  if (!codes || !packed || rows < 1 || N < 8 || N % 8) return ANVILQ_EINVAL;
  const long long words = (long long)rows * (N / 8);
  unpack_kernel<<<(unsigned)((words + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      packed, codes, words);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}

}  // extern "C"
