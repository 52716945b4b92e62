// gemv_tma.cu -- batch-1 W4A16 AWQ GEMV for B200: TMA-staged int4 stream,
// thread-block-cluster split-K, DSMEM reduction.
//
// Reference semantics: FP32Model.linear (anvil-q1/tests/official_weights.py:418-437),
//   y[c] = sum_k x[k] * (u4 q[k][c] - u4 z[k/G][c]) * scale[k/G][c]  (+ bias[c]).
//
// Data movement.  The int4 matrix is the only large operand.  A band is 64
// consecutive qweight words of every row (256 B per row, 512 output columns);
// a tile is 32 rows of a band (8 KB), fetched by ONE cp.async.bulk.tensor.2d
// from a tensor map over qweight [K][N/8].  Every warp streams its own range
// of tiles through a private 3-stage shared-memory ring (one mbarrier per
// stage), so the bytes in flight (up to 2 CTAs x 4 warps x 3 tiles = 192 KB
// per SM) cost no registers.  Tiles past the last row or column are
// zero-filled by the TMA unit and contribute nothing.
//
// Split-K.  The c CTAs of a thread-block cluster share one band and split its
// tiles between their 4c warps; warps are reduced in shared memory, CTAs
// through distributed shared memory in cluster-rank order (deterministic, no
// global scratch, no atomics).  c in {1,2,4,8,16} is chosen on the host so that
// all CTAs are resident at once and every warp has work.
//
// Arithmetic (per thread: 4 words = 32 columns x 16 consecutive rows):
//   * q is used as a binary16 SUBNORMAL: (w & 0x000F000F) reinterpreted as
//     half2 is exactly (q0, q1) * 2^-24, (w & 0x00F000F0) is 16 (q2, q3) 2^-24,
//     and the same on w >> 8 for lanes 4..7.  One AND per column pair.
//   * x is pre-scaled per 16-row slot by an exact power of two 2^S (S from the
//     slot's largest |x|, so |x 2^S| < 2^15): products x q land in the normal
//     binary16 range and the 16-row partial sum acc = sum x 2^S q 2^-24 is
//     accumulated with one HFMA2 per column pair per row.
//   * The slot's partial is folded into fp32 as A += acc * 2^(24-S) (/16 for
//     the shifted pairs), exact scaling.
//   * The zero point is applied once per group through the slot sums of x:
//     sum x (q - z) = sum x q - z sum x, and the group's scale once:
//     y += s (A - z X).  Only the 16-product partials are binary16.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "../../include/anvilq.h"
#include "awq_common.cuh"
#include "internal.h"

namespace anvilq {
namespace tma_gemv {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kBandWords = 64;                        // 256 B per row, 512 columns
constexpr int kBandCols = kBandWords * 8;
constexpr int kTileRows = 32;
constexpr int kStages = 3;
constexpr int kTileBytes = kTileRows * kBandWords * 4;   // 8 KB
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

// dynamic shared memory layout
constexpr int kRingOff = 0;
constexpr int kRingBytes = kWarps * kStages * kTileBytes;
constexpr int kXsOff = kRingOff + kRingBytes;                    // [warp][32 rows] half2
constexpr int kXrawOff = kXsOff + kWarps * kTileRows * 4;        // [warp][stage][32 rows] half
constexpr int kBarOff = kXrawOff + kWarps * kStages * kTileRows * 2;   // [warp][stage] u64
constexpr int kRedOff = kBarOff + kWarps * kStages * 8 + 64;     // [warp][512] f32
constexpr int kPartOff = kRedOff + kWarps * kBandCols * 4;       // [512] f32
constexpr int kSmemBytes = kPartOff + kBandCols * 4;

struct Params {
  const __half* x;
  const int32_t* qzeros;
  const __half* scales;
  const __half* bias;
  __half* y;
  int* dev_err;
  int K, N, W8, G;
  int cluster;   // CTAs per band
  int tiles;     // tiles per band = ceil(K / 32)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 63u && globaltimer() - t0 > kWaitLimitNs) return false;
  }
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_dsmem_f32(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}
__device__ __forceinline__ half2 h2(uint32_t u) { return *reinterpret_cast<half2*>(&u); }
__device__ __forceinline__ uint32_t u32(half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

__global__ void __launch_bounds__(kThreads, 2)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tmap, const Params p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int c = p.cluster;
  const int rank = c > 1 ? (int)cluster_rank() : 0;
  const int band = blockIdx.x / c;
  const int wi = rank * kWarps + warp, nw = c * kWarps;
  const int t0 = (int)((long long)wi * p.tiles / nw);
  const int t1 = (int)((long long)(wi + 1) * p.tiles / nw);
  const int ntiles = t1 - t0;

  unsigned char* ring = smem + kRingOff + warp * kStages * kTileBytes;
  uint32_t* xs = reinterpret_cast<uint32_t*>(smem + kXsOff) + warp * kTileRows;
  const __half* xraw = reinterpret_cast<const __half*>(smem + kXrawOff) + warp * kStages * kTileRows;
  const uint32_t xraw0 = smem_u32(smem + kXrawOff) + warp * kStages * kTileRows * 2;
  const uint32_t bar0 = smem_u32(smem + kBarOff + warp * kStages * 8);
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * s) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap) : "memory");
  }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  // let the next kernel on the stream start its own weight prefetch (programmatic
  // dependent launch); it still waits for this grid before touching our output
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __syncwarp();

  // Stage j % kStages receives tile t0 + j (8 KB of int4 words) and the tile's
  // 32 activations (64 B), both counted on the stage's mbarrier.
  auto x_bytes = [&](int j) { return (uint32_t)min(kTileRows, p.K - (t0 + j) * kTileRows) * 2u; };
  auto issue_tile = [&](int j, bool with_x) {   // lane 0 only
    const int st = j % kStages;
    const uint32_t bar = bar0 + 8 * st;
    // the stage was last read through the generic proxy; order that before the TMA write
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (with_x)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                   "r"(kTileBytes + x_bytes(j))
                   : "memory");
    else
      asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(kTileBytes) : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(ring + st * kTileBytes)),
        "l"(&tmap), "r"(band * kBandWords), "r"((t0 + j) * kTileRows), "r"(bar)
        : "memory");
    if (with_x)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       xraw0 + st * kTileRows * 2),
                   "l"(p.x + (size_t)(t0 + j) * kTileRows), "r"(x_bytes(j)), "r"(bar)
                   : "memory");
  };
  auto issue_x = [&](int j) {   // lane 0 only: activations of a tile whose weights are in flight
    const int st = j % kStages;
    const uint32_t bar = bar0 + 8 * st;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(x_bytes(j)) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     xraw0 + st * kTileRows * 2),
                 "l"(p.x + (size_t)(t0 + j) * kTileRows), "r"(x_bytes(j)), "r"(bar)
                 : "memory");
  };

  const int q = lane % 16, rg = lane / 16;         // 4 words of the band, 16-row half of the tile
  const int w0 = band * kBandWords + q * 4;
  const bool active = w0 < p.W8;
  auto slot_row = [&](int j) { return (t0 + j) * kTileRows + 16 * rg; };

  float A[32], Y[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) A[j] = Y[j] = 0.0f;
  float Xg = 0.0f;
  uint4 sc[4] = {}, zq = {}, nsc[4] = {}, nzq = {};
  uint32_t bad = 0;
  bool ok = true;

  auto load_group = [&](int row, uint4* s4, uint4& z) {   // scales and zeros of the group of `row`
    if (active && row < p.K) {
      const int g = row / p.G;
      const __half* sp = p.scales + (size_t)g * p.N + 8 * (size_t)w0;
#pragma unroll
      for (int i = 0; i < 4; ++i) s4[i] = __ldg(reinterpret_cast<const uint4*>(sp + 8 * i));
      z = __ldg(reinterpret_cast<const uint4*>(p.qzeros + (size_t)g * p.W8 + w0));
    }
  };
  auto check_group = [&](int row) {   // the slot that opens a group checks its scales, once
    if (active && row < p.K && row % p.G == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        bad |= invalid_scale_pair(sc[i].x) | invalid_scale_pair(sc[i].y) | invalid_scale_pair(sc[i].z) |
               invalid_scale_pair(sc[i].w);
    }
  };

  // y += s (A - z X) for the finished group; s, z of this lane's 32 columns
  auto flush_group = [&]() {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t zw = i == 0 ? zq.x : i == 1 ? zq.y : i == 2 ? zq.z : zq.w;
      const uint32_t sw[4] = {sc[i].x, sc[i].y, sc[i].z, sc[i].w};
      // zero points as fp32 via the binary16 magic 1024 + z, pairs (0,1),(2,3),(4,5),(6,7)
      const uint32_t zp[4] = {(zw & 0x000F000Fu) | 0x64006400u, ((zw >> 4) & 0x000F000Fu) | 0x64006400u,
                              ((zw >> 8) & 0x000F000Fu) | 0x64006400u, ((zw >> 12) & 0x000F000Fu) | 0x64006400u};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 s2 = __half22float2(h2(sw[e]));
        const float2 z2 = __half22float2(h2(zp[e]));
        const float t0v = fmaf(-(z2.x - 1024.0f), Xg, A[i * 8 + 2 * e]);
        const float t1v = fmaf(-(z2.y - 1024.0f), Xg, A[i * 8 + 2 * e + 1]);
        Y[i * 8 + 2 * e] = fmaf(s2.x, t0v, Y[i * 8 + 2 * e]);
        Y[i * 8 + 2 * e + 1] = fmaf(s2.y, t1v, Y[i * 8 + 2 * e + 1]);
        A[i * 8 + 2 * e] = 0.0f;
        A[i * 8 + 2 * e + 1] = 0.0f;
      }
    }
    Xg = 0.0f;
  };

  // -- prologue: weights first (they do not depend on the previous kernel) ---
  int issued = 0;
  const int pro = min(kStages - 1, ntiles);
  if (lane == 0)
    for (int j = 0; j < pro; ++j) issue_tile(j, false);
  issued = pro;
  if (ntiles > 0) load_group(slot_row(0), sc, zq);
  asm volatile("griddepcontrol.wait;" ::: "memory");   // x may come from the previous kernel
  if (lane == 0)
    for (int j = 0; j < pro; ++j) issue_x(j);
  if (ntiles > 0) check_group(slot_row(0));

  for (int j = 0; j < ntiles; ++j) {
    if (issued < ntiles) {
      if (lane == 0) issue_tile(issued, true);
      ++issued;
    }
    const bool next_group = j + 1 < ntiles && slot_row(j + 1) / p.G != slot_row(j) / p.G;
    if (next_group) load_group(slot_row(j + 1), nsc, nzq);   // lands while this tile computes
    const int st = j % kStages;
    const bool landed = mbar_wait_bounded(bar0 + 8 * st, (j / kStages) & 1);
    if (!__all_sync(0xffffffffu, landed)) {
      ok = false;
      break;
    }
    // -- activations of the tile: lane l holds row l; a slot (16 rows) is 16 lanes
    float Sxs, pow_lo;
    {
      static_assert(kTileRows == 32, "one activation row per lane");
      const int kr = (t0 + j) * kTileRows + lane;
      const float xf = kr < p.K ? __half2float(xraw[st * kTileRows + lane]) : 0.0f;
      float mx = fabsf(xf);
      float sum = xf;
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
      }
      // |x| < 2^e with e the binary exponent of mx; scale by 2^(15 - e)
      const int e = mx > 0.0f ? ((__float_as_int(mx) >> 23) & 255) - 126 : 0;
      const int S = 15 - e;
      const float f = __int_as_float((127 + S) << 23);
      const half hs = __float2half_rn(xf * f);
      xs[lane] = u32(__halves2half2(hs, hs));
      // this thread's slot is rows 16 rg .. 16 rg + 15, held by lanes 16 rg .. 16 rg + 15
      Sxs = __shfl_sync(0xffffffffu, sum, 16 * rg);
      const int Smine = __shfl_sync(0xffffffffu, S, 16 * rg);
      pow_lo = __int_as_float((127 + 24 - Smine) << 23);
    }
    __syncwarp();
    const unsigned char* tile = ring + st * kTileBytes + (16 * rg) * (kBandWords * 4) + q * 16;
    half2 part[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) part[i] = __float2half2_rn(0.0f);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const uint4 w = *reinterpret_cast<const uint4*>(tile + r * (kBandWords * 4));
      const half2 xx = h2(xs[16 * rg + r]);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t w8 = ws[i] >> 8;
        part[4 * i + 0] = __hfma2(xx, h2(ws[i] & 0x000F000Fu), part[4 * i + 0]);   // columns 0,1
        part[4 * i + 1] = __hfma2(xx, h2(ws[i] & 0x00F000F0u), part[4 * i + 1]);   // columns 2,3 (x16)
        part[4 * i + 2] = __hfma2(xx, h2(w8 & 0x000F000Fu), part[4 * i + 2]);      // columns 4,5
        part[4 * i + 3] = __hfma2(xx, h2(w8 & 0x00F000F0u), part[4 * i + 3]);      // columns 6,7 (x16)
      }
    }
    __syncwarp();   // stage st and xs are free again
    const float pow_hi = pow_lo * 0.0625f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f2 = __half22float2(part[4 * i + e]);
        const float pw = (e & 1) ? pow_hi : pow_lo;
        A[i * 8 + 2 * e] = fmaf(f2.x, pw, A[i * 8 + 2 * e]);
        A[i * 8 + 2 * e + 1] = fmaf(f2.y, pw, A[i * 8 + 2 * e + 1]);
      }
    Xg += Sxs;
    if (next_group) {
      flush_group();
#pragma unroll
      for (int i = 0; i < 4; ++i) sc[i] = nsc[i];
      zq = nzq;
      check_group(slot_row(j + 1));
    }
  }
  const bool ended_in_group = ntiles > 0;
  if (ok && ended_in_group) flush_group();
  if (!ok) {
    if (lane == 0 && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
    for (int j = max(0, issued - kStages); j < issued; ++j)
      mbar_wait_bounded(bar0 + 8 * (j % kStages), (j / kStages) & 1);
#pragma unroll
    for (int j = 0; j < 32; ++j) Y[j] = 0.0f;
  }
  if (bad && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SCALE);

  // -- reduce: the two row halves of the warp, then the warps, then the cluster
#pragma unroll
  for (int j = 0; j < 32; ++j) Y[j] += __shfl_xor_sync(0xffffffffu, Y[j], 16);
  float* red = reinterpret_cast<float*>(smem + kRedOff) + warp * kBandCols;
  if (rg == 0) {
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4*>(red + q * 32 + j) = make_float4(Y[j], Y[j + 1], Y[j + 2], Y[j + 3]);
  }
  __syncthreads();
  float* part = reinterpret_cast<float*>(smem + kPartOff);
  for (int col = threadIdx.x; col < kBandCols; col += kThreads) {
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += reinterpret_cast<const float*>(smem + kRedOff)[w * kBandCols + col];
    part[col] = v;
  }
  const int col0 = band * kBandCols;
  if (c == 1) {
    __syncthreads();
    for (int col = threadIdx.x; col < kBandCols; col += kThreads) {
      if (col0 + col < p.N) {
        float v = part[col];
        if (p.bias) v += __half2float(p.bias[col0 + col]);
        p.y[col0 + col] = __float2half_rn(v);
      }
    }
    return;
  }
  cluster_sync();   // every CTA of the cluster reaches this point, errors included
  const int per = kBandCols / c;
  for (int t = threadIdx.x; t < per; t += kThreads) {
    const int col = rank * per + t;
    float v = 0.0f;
    for (int r = 0; r < c; ++r) v += ld_dsmem_f32(part + col, (uint32_t)r);
    if (col0 + col < p.N) {
      if (p.bias) v += __half2float(p.bias[col0 + col]);
      p.y[col0 + col] = __float2half_rn(v);
    }
  }
  cluster_sync();   // peers may still be reading this CTA's partial
}

// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    cudaGetLastError();
  });
  return g_encode;
}

constexpr int kMaxDevices = 64;
struct DeviceInfo {
  int sms = 0;
  int max_clusters[5] = {0, 0, 0, 0, 0};   // co-resident clusters of size 1, 2, 4, 8, 16
};
static DeviceInfo g_dev[kMaxDevices];
static std::once_flag g_dev_once[kMaxDevices];

static const DeviceInfo* device_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(g_dev_once[dev], [dev] {
    DeviceInfo& d = g_dev[dev];
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(gemv_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    cudaFuncSetAttribute(gemv_tma_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    for (int i = 0; i < 5; ++i) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1u << i, 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = kSmemBytes;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1u << i;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, gemv_tma_kernel, &cfg) != cudaSuccess) n = 0;
      d.max_clusters[i] = n;
    }
    cudaGetLastError();
  });
  return &g_dev[dev];
}

// Largest cluster size whose clusters (one per band) are all co-resident and
// whose warps each get at least half a tile on average.
int choose_cluster(int bands, int tiles, const DeviceInfo& d) {
  int c = 1;
  for (int i = 1; i < 5; ++i) {
    const int cand = 1 << i;
    if (d.max_clusters[i] >= bands && 2 * cand <= tiles) c = cand;
  }
  return c;
}

}  // namespace tma_gemv

bool gemv_tma_supported(const void* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                        int K, int N, int G) {
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  return K % 16 == 0 && G % 16 == 0 && N % 32 == 0 && a16(x) && a16(qweight) && a16(qzeros) && a16(scales) &&
         tma_gemv::encode_fn() != nullptr;
}

int launch_gemv_tma(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                    const uint16_t* bias, uint16_t* y, int K, int N, int G, int* dev_err, cudaStream_t stream,
                    bool overlap_prior) {
  using namespace tma_gemv;
  const DeviceInfo* d = device_info();
  auto encode = encode_fn();
  if (!d || d->sms <= 0 || !encode) return ANVILQ_ECUDA;
  const int W8 = N / 8;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)W8, (cuuint64_t)K};
  const cuuint64_t strides[1] = {(cuuint64_t)W8 * 4};
  const cuuint32_t box[2] = {(cuuint32_t)kBandWords, (cuuint32_t)kTileRows};
  const cuuint32_t estr[2] = {1, 1};
  if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(qweight), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return ANVILQ_EALIGN;
  Params p;
  p.x = reinterpret_cast<const __half*>(x);
  p.qzeros = qzeros;
  p.scales = reinterpret_cast<const __half*>(scales);
  p.bias = reinterpret_cast<const __half*>(bias);
  p.y = reinterpret_cast<__half*>(y);
  p.dev_err = dev_err;
  p.K = K; p.N = N; p.W8 = W8; p.G = G;
  const int bands = (W8 + kBandWords - 1) / kBandWords;
  p.tiles = (K + kTileRows - 1) / kTileRows;
  p.cluster = choose_cluster(bands, p.tiles, *d);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(bands * p.cluster, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap_prior ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, gemv_tma_kernel, map, p) != cudaSuccess) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  return ANVILQ_OK;
}

}  // namespace anvilq
