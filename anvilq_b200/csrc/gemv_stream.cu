// gemv_stream.cu -- batch-1 W4A16 AWQ GEMV for large layers (7B / 70B class):
// stream-K over 4 KB chunks of the int4 stream, one TMA ring per warp.
//
// Reference semantics: FP32Model.linear (anvil-q1/tests/official_weights.py:418-437),
//   y[c] = sum_k x[k] * (u4 q[k][c] - u4 z[k/G][c]) * scale[k/G][c]  (+ bias[c]).
//
// Work.  A band is 32 consecutive qweight words of every row (128 B per row,
// 256 output columns); a chunk is 32 rows of a band (4 KB), the unit of one
// cp.async.bulk.tensor.2d.  The chunks are numbered band-major and the grid
// takes them as one stream: CTA i owns chunks [i T / P, (i + 1) T / P), and
// its warps split that range evenly, so every SM streams the same number of
// bytes whatever the layer's shape (deep-K, wide-N or a tensor-parallel
// slice).  A CTA's range covers at most two bands (the host guarantees
// T / P <= chunks per band).
//
// Streaming.  Each warp owns a ring of S stages; lane 0 keeps S chunks in
// flight, each with its 32 activations (a 64-byte bulk copy) on the same
// mbarrier.  The weights of the first S chunks are requested before
// griddepcontrol.wait, so under programmatic dependent launch they stream
// while the previous kernel drains; activations are requested after it.
//
// Arithmetic (lane l owns word 32 band + l = 8 columns, for every row of
// its chunks): the nibble pairs (w & 0x000F000F), (w & 0x00F000F0) and the
// same on w >> 8 are binary16 subnormals (q0, q1) 2^-24 and 16 (q2, q3) 2^-24;
// each product x * q is exact and added into an fp32 accumulator by the
// mixed-precision fma.rn.f32.f16 (one rounding per weight, no binary16 partial
// sums).  Per group the zero point enters once through the group's sum of x
// (sum x (q - z) = sum x q - z sum x) and the scale once, in fp32.
//
// Reduction.  Warps sum in shared memory in warp order; a band finished
// inside one CTA is written directly, otherwise every CTA that touched it
// leaves its partial in the workspace and the CTA arriving last at the band's
// ticket adds the partials in CTA order.  Every sum has a fixed order, so the
// result is bit-reproducible; no CTA ever waits for another.  A CTA whose range
// crosses a band boundary takes both bands' steps together (both partials
// stored, both tickets taken by two threads, both fix-ups in one batch of
// loads), and the CTA bounds of its bands -- 64-bit divisions -- are computed
// before griddepcontrol.wait, while the first chunks are in flight.
//
// Fused all-gather (PEER, one rank's column slice of a tensor-parallel split):
// the CTA that finishes a band stores its 256 fp16 columns into every rank's
// full-width output with 16-byte stores (peer memory over NVLink, plain
// stores), fences them at system scope and counts the band on the rank's
// ticket; the CTA completing the rank's last band raises the rank's flag in
// every rank and waits, bounded by ~1 s of %globaltimer, for every rank's flag.
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
namespace stream_gemv {

constexpr int kBandWords = 32;                         // 128 B per row, 256 columns
constexpr int kBandCols = kBandWords * 8;
constexpr int kChunkRows = 32;
constexpr int kChunkBytes = kChunkRows * kBandWords * 4;   // 4 KB
constexpr int kXBytes = kChunkRows * 2;                    // the chunk's 32 fp16 activations
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

template <int W, int S>
struct Layout {
  static constexpr int kRingOff = 0;
  static constexpr int kRingBytes = W * S * kChunkBytes;
  static constexpr int kXOff = kRingBytes;                  // [warp][stage][64 B]
  static constexpr int kBarOff = kXOff + W * S * kXBytes;   // [warp][stage] u64
  static constexpr int kBytes = kBarOff + W * S * 8;
  static constexpr int kRedBytes = 2 * W * kBandCols * 4;   // [slot][warp][256] f32, aliases the ring
  static_assert(kRedBytes <= kRingBytes, "the reduction buffer reuses the ring");
};

constexpr int kMaxPeers = 8;
// the rank's completed-band counter of the fused all-gather: the last int of
// the workspace's counter region (band tickets use the first `bands` ints)
constexpr int kRankTicket = ANVILQ_WORKSPACE_COUNTER_BYTES / 4 - 1;

struct Params {
  const __half* x;
  const int32_t* qzeros;
  const __half* scales;
  const __half* bias;
  __half* y;
  float* parts;      // [ctas][2][256]
  int* tickets;      // [bands] (+ the rank ticket at kRankTicket)
  int* dev_err;
  int K, N, W8, G;
  int cpb;           // chunks per band = K / 32
  int cpg;           // chunks per group = G / 32
  int total;         // bands * cpb
  int bands;
  // PEER only: one rank's column slice of a tensor-parallel split; y is stored
  // at columns [col_base, col_base + N) of every rank's full-width output
  __half* peer_y[kMaxPeers];
  unsigned* peer_flags[kMaxPeers];
  unsigned* epoch;
  int world, tp_rank, col_base;
  int deferred;      // PEER: raise the flag without waiting; wait for the previous call before reading x
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
// true once the phase completed; false after ~1 s (the caller reports a timeout)
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 63u && globaltimer() - t0 > kWaitLimitNs) return false;
  }
}
__device__ __forceinline__ half2 h2(uint32_t u) { return *reinterpret_cast<half2*>(&u); }

// a0 += x * q.lo, a1 += x * q.hi: binary16 x and q, binary32 accumulators,
// exact products rounded once into the accumulators
__device__ __forceinline__ void fma_f32_f16x2(float& a0, float& a1, uint32_t q2, unsigned short x) {
  asm("{\n .reg .f16 q0, q1;\n mov.b32 {q0, q1}, %2;\n"
      " fma.rn.f32.f16 %0, %3, q0, %0;\n fma.rn.f32.f16 %1, %3, q1, %1;\n}"
      : "+f"(a0), "+f"(a1)
      : "r"(q2), "h"(x));
}

// CTA that owns chunk c when T chunks are split over P CTAs as [i T / P, (i + 1) T / P)
__device__ __forceinline__ int cta_of(long long c, int T, int P) {
  return (int)(((c + 1) * P - 1) / T);
}

// system-scope flag accesses between GPUs of the node
// a strong store at system scope; after a system fence it is a release (fence
// + relaxed stores: one fence for every rank's flag, where a release store per
// rank would wait for each remote store before issuing the next)
__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <int W, int S, bool PEER>
__global__ void __launch_bounds__(W * 32, W <= 8 ? 2 : 1)
    gemv_stream_kernel(const __grid_constant__ CUtensorMap tmap, const Params p) {
  using L = Layout<W, S>;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_last[2], s_done;
  // the CTAs sharing the CTA's two bands (first, last) and the slot that
  // band's first contributor stored it in: {first0, first1, last0, last1, slot0, slot1}
  __shared__ int s_bounds[6];
  __shared__ __align__(16) __half s_y[2 * kBandCols];   // PEER: finished bands, staged for 16-byte stores
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x, T = p.total;
  const int c0 = (int)((long long)blockIdx.x * T / P), c1 = (int)((long long)(blockIdx.x + 1) * T / P);
  const int n = c1 - c0;
  const int wc0 = c0 + (int)((long long)warp * n / W);
  const int nch = c0 + (int)((long long)(warp + 1) * n / W) - wc0;   // this warp's chunks
  const int band0 = c0 / p.cpb;                                      // the CTA's first band (slot 0)

  unsigned char* ring = smem + L::kRingOff + warp * S * kChunkBytes;
  unsigned char* xbuf = smem + L::kXOff + warp * S * kXBytes;
  const uint32_t ring0 = smem_u32(ring), xbuf0 = smem_u32(xbuf);
  const uint32_t bar0 = smem_u32(smem + L::kBarOff + warp * S * 8);
  if (lane == 0) {
    for (int s = 0; s < S; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * s) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap) : "memory");
  }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  // the next kernel on the stream may start its own weight prefetch now
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __syncwarp();

  // chunk iterators (band, chunk-in-band) without divisions in the loop
  int ib = wc0 / p.cpb, ik = wc0 % p.cpb;   // next chunk to request (lane 0)
  auto issue_w = [&](int j) {               // lane 0: weights of chunk j (at ib, ik)
    const uint32_t bar = bar0 + 8 * (j % S);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(kChunkBytes) : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(ring0 + (j % S) * kChunkBytes),
        "l"(&tmap), "r"(ib * kBandWords), "r"(ik * kChunkRows), "r"(bar)
        : "memory");
  };
  auto issue_x = [&](int j, int row) {      // lane 0: activations of chunk j (rows row .. row + 31)
    const uint32_t bar = bar0 + 8 * (j % S);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kXBytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     xbuf0 + (j % S) * kXBytes),
                 "l"(p.x + row), "r"(kXBytes), "r"(bar)
                 : "memory");
  };
  auto advance = [&](int& b, int& k) {
    if (++k == p.cpb) {
      k = 0;
      ++b;
    }
  };

  const int pro = min(S, nch);
  int xb = ib, xk = ik;   // activations of the prologue chunks follow after griddepcontrol.wait
  if (lane == 0)
    for (int j = 0; j < pro; ++j) {
      issue_w(j);
      advance(ib, ik);
    }

  // this lane's word and the scales / zeros of the current (band, group) segment
  int cb = wc0 / p.cpb, ck = wc0 % p.cpb;   // chunk being consumed
  auto word_of = [&](int band) { return band * kBandWords + lane; };
  uint4 sc = {}, nsc = {};
  uint32_t zq = 0, nzq = 0;
  uint32_t bad = 0;
  auto load_seg = [&](int band, int k, uint4& s, uint32_t& z) {
    const int w = word_of(band);
    if (w < p.W8) {
      const int g = k / p.cpg;
      s = ld_stream_v4(p.scales + (size_t)g * p.N + 8 * (size_t)w);
      z = ld_stream_u32(p.qzeros + (size_t)g * p.W8 + w);
    }
  };
  if (nch > 0) load_seg(cb, ck, sc, zq);

  // the reduction's 64-bit divisions, done while the first chunks are in flight
  // (read only after the barrier that ends the tile loop)
  if (warp == W - 1 && lane < 6) {
    const int band = band0 + (lane & 1);
    const long long c = lane >> 1 == 1 ? (long long)(band + 1) * p.cpb - 1 : (long long)band * p.cpb;
    int val = cta_of(c, T, P);
    if (lane >> 1 == 2) val = (int)((long long)val * T / P) / p.cpb < band ? 1 : 0;
    s_bounds[lane] = val;
  }

  asm volatile("griddepcontrol.wait;" ::: "memory");   // x may come from the previous kernel
  if (PEER && p.deferred && lane == 0) {
    // every rank has finished the previous fused call: its slice of x (when x is
    // that call's gathered row) is here, and no rank still reads the output slot
    // this call is about to overwrite.  Bounded like the flag wait at the end.
    const unsigned e_prev = *reinterpret_cast<volatile unsigned*>(p.epoch);
    const unsigned* mine = p.peer_flags[p.tp_rank];
    const unsigned long long t_start = globaltimer();
    bool all = false;
    for (uint32_t i = 0; !all; ++i) {
      all = true;
      for (int r = 0; r < p.world; ++r) all &= (int)(ld_acquire_sys(mine + r) - e_prev) >= 0;
      if (!all && (i & 63u) == 63u && globaltimer() - t_start > kWaitLimitNs) {
        if (p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
        break;
      }
    }
    // the peers' stores (generic proxy) before the bulk copies of x (async proxy)
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  if (lane == 0)
    for (int j = 0; j < pro; ++j) {
      issue_x(j, xk * kChunkRows);
      advance(xb, xk);
    }

  float A[8], Y[8], Yf[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) A[i] = Y[i] = Yf[i] = 0.0f;
  float Xg = 0.0f;
  bool split = false;   // Yf holds the warp's first band (the CTA's slot 0)
  int stop = nch;       // first chunk not consumed (nch unless a wait expired)
  if (nch > 0) bad |= invalid_scale_pair(sc.x) | invalid_scale_pair(sc.y) | invalid_scale_pair(sc.z) |
                      invalid_scale_pair(sc.w);

  // y += s (A - z X) for the finished segment
  auto flush = [&]() {
    const uint32_t sw[4] = {sc.x, sc.y, sc.z, sc.w};
    const uint32_t zp[4] = {(zq & 0x000F000Fu) | 0x64006400u, ((zq >> 4) & 0x000F000Fu) | 0x64006400u,
                            ((zq >> 8) & 0x000F000Fu) | 0x64006400u, ((zq >> 12) & 0x000F000Fu) | 0x64006400u};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 s2 = __half22float2(h2(sw[e]));
      const float2 z2 = __half22float2(h2(zp[e]));
      const float pw = (e & 1) ? 1048576.0f : 16777216.0f;   // 2^20 (shifted pairs) or 2^24
      const float a0 = fmaf(-(z2.x - 1024.0f), Xg, A[2 * e] * pw);
      const float a1 = fmaf(-(z2.y - 1024.0f), Xg, A[2 * e + 1] * pw);
      Y[2 * e] = fmaf(s2.x, a0, Y[2 * e]);
      Y[2 * e + 1] = fmaf(s2.y, a1, Y[2 * e + 1]);
      A[2 * e] = 0.0f;
      A[2 * e + 1] = 0.0f;
    }
    Xg = 0.0f;
  };

  for (int j = 0; j < nch; ++j) {
    // the segment of the next chunk: prefetch its scales and zeros now
    int nb = cb, nk = ck;
    advance(nb, nk);
    const bool more = j + 1 < nch;
    const bool new_seg = more && (nb != cb || nk % p.cpg == 0);
    if (new_seg) load_seg(nb, nk, nsc, nzq);

    const int st = j % S;
    const bool landed = mbar_wait_bounded(bar0 + 8 * st, (j / S) & 1);
    if (!__all_sync(0xffffffffu, landed)) {
      stop = j;
      break;
    }
    const unsigned char* tile = ring + st * kChunkBytes + lane * 4;
    const uint4* xq = reinterpret_cast<const uint4*>(xbuf + st * kXBytes);
    // the chunk's sum of activations (for the zero points)
    {
      float xs = __half2float(reinterpret_cast<const __half*>(xbuf + st * kXBytes)[lane]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) xs += __shfl_xor_sync(0xffffffffu, xs, o);
      Xg += xs;
    }
#pragma unroll
    for (int r8 = 0; r8 < kChunkRows; r8 += 8) {
      const uint4 xv = xq[r8 / 8];   // rows r8 .. r8 + 7 (broadcast)
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const uint32_t wd = *reinterpret_cast<const uint32_t*>(tile + (r8 + r) * (kBandWords * 4));
        const unsigned short xh = (unsigned short)(r & 1 ? xw[r / 2] >> 16 : xw[r / 2] & 0xFFFFu);
        const uint32_t w8 = wd >> 8;
        fma_f32_f16x2(A[0], A[1], wd & 0x000F000Fu, xh);   // columns 0,1
        fma_f32_f16x2(A[2], A[3], wd & 0x00F000F0u, xh);   // columns 2,3 (x16)
        fma_f32_f16x2(A[4], A[5], w8 & 0x000F000Fu, xh);   // columns 4,5
        fma_f32_f16x2(A[6], A[7], w8 & 0x00F000F0u, xh);   // columns 6,7 (x16)
      }
    }
    __syncwarp();   // stage st is free again
    if (lane == 0 && j + S < nch) {
      issue_w(j + S);
      issue_x(j + S, ik * kChunkRows);
      advance(ib, ik);
    }
    if (!more || new_seg) {
      flush();
      if (more && nb != cb) {   // the warp moves on to the CTA's second band
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          Yf[i] = Y[i];
          Y[i] = 0.0f;
        }
        split = true;
      }
      if (more) {
        sc = nsc;
        zq = nzq;
        if (word_of(nb) < p.W8)
          bad |= invalid_scale_pair(sc.x) | invalid_scale_pair(sc.y) | invalid_scale_pair(sc.z) |
                 invalid_scale_pair(sc.w);
      }
    }
    cb = nb;
    ck = nk;
  }
  if (stop < nch) {
    if (lane == 0 && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
    // chunks [stop, stop + S) were requested and not consumed: wait (bounded)
    // for them before the ring is reused as the reduction buffer
    for (int j = stop; j < min(nch, stop + S); ++j) mbar_wait_bounded(bar0 + 8 * (j % S), (j / S) & 1);
#pragma unroll
    for (int i = 0; i < 8; ++i) Y[i] = Yf[i] = 0.0f;
  }
  if (bad && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SCALE);

  // -- reduce: warps in shared memory (slot 0 = the CTA's first band), then CTAs
  __syncthreads();   // every warp is done with its ring
  float* red = reinterpret_cast<float*>(smem + L::kRingOff);   // [2][W][256]
  {
    const int last_band = nch > 0 ? (wc0 + nch - 1) / p.cpb : band0;   // the band of this warp's Y
    const int slot_y = last_band - band0;
    float* r0 = red + (0 * W + warp) * kBandCols + lane * 8;
    float* r1 = red + (1 * W + warp) * kBandCols + lane * 8;
    float v0[8], v1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v0[i] = split ? Yf[i] : (slot_y == 0 ? Y[i] : 0.0f);
      v1[i] = split ? Y[i] : (slot_y == 1 ? Y[i] : 0.0f);
    }
    *reinterpret_cast<float4*>(r0) = make_float4(v0[0], v0[1], v0[2], v0[3]);
    *reinterpret_cast<float4*>(r0 + 4) = make_float4(v0[4], v0[5], v0[6], v0[7]);
    *reinterpret_cast<float4*>(r1) = make_float4(v1[0], v1[1], v1[2], v1[3]);
    *reinterpret_cast<float4*>(r1 + 4) = make_float4(v1[4], v1[5], v1[6], v1[7]);
  }
  __syncthreads();
  // The CTA's bands (slot 0, and slot 1 when its range crosses a band boundary)
  // go through the cross-CTA steps together: both partials are stored, both
  // tickets taken by two threads at once, and both fix-ups loaded in one pass.
  const int last_band_cta = n > 0 ? (c1 - 1) / p.cpb : band0 - 1;
  const int nslots = last_band_cta - band0 + 1;   // 0, 1 or 2 (uniform over the CTA)
  const int first_s[2] = {s_bounds[0], s_bounds[1]}, last_s[2] = {s_bounds[2], s_bounds[3]};
  // (slot, column) entries of this thread: e = threadIdx.x + u W 32, slot e / 256
  constexpr int kE = (2 * kBandCols + W * 32 - 1) / (W * 32);
  float v[kE];
#pragma unroll
  for (int u = 0; u < kE; ++u) {
    const int e = threadIdx.x + u * W * 32, s = e / kBandCols, t = e % kBandCols;
    v[u] = 0.0f;
    if (e < 2 * kBandCols && s < nslots) {
#pragma unroll
      for (int w = 0; w < W; ++w) v[u] += red[(s * W + w) * kBandCols + t];
      if (s == 0 ? first_s[0] != last_s[0] : first_s[1] != last_s[1])
        __stcg(p.parts + ((size_t)blockIdx.x * 2 + s) * kBandCols + t, v[u]);
    }
  }
  if (threadIdx.x < 2) s_last[threadIdx.x] = 0;
  if (PEER && threadIdx.x == 0) s_done = 0;
  __syncthreads();
  // lane 0 of warp s fences for the CTA (the barrier orders every thread's
  // stores before it, cumulatively) and takes slot s's ticket; the last
  // arriver's fence orders its CTA's loads after every contributor's stores
  if (lane == 0 && warp < nslots && (warp == 0 ? first_s[0] != last_s[0] : first_s[1] != last_s[1])) {
    const int band = band0 + warp;
    __threadfence();
    const int arrived = atomicAdd(p.tickets + band, 1);
    if (arrived == (warp == 0 ? last_s[0] - first_s[0] : last_s[1] - first_s[1])) {
      p.tickets[band] = 0;   // re-armed for the next launch
      __threadfence();
      s_last[warp] = 1;
    }
  }
  __syncthreads();
  bool own[2], fix[2];   // this CTA writes the slot's band / adds its contributors first
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    fix[s] = s < nslots && first_s[s] != last_s[s] && s_last[s];
    own[s] = s < nslots && (first_s[s] == last_s[s] || s_last[s]);
  }
  if (fix[0] || fix[1]) {
    // the contributors of both slots as one list of rows (slot 0's, then slot
    // 1's, each in CTA order), loaded by all threads at once and staged through
    // the ring (free again) in batches, then summed per slot in CTA order
    constexpr int kFixRows = L::kRingBytes / (kBandCols * 4) < 64 ? L::kRingBytes / (kBandCols * 4) : 64;
    float* stage = reinterpret_cast<float*>(smem + L::kRingOff + L::kRedBytes);
    constexpr int kStageRows = (L::kRingBytes - L::kRedBytes) / (kBandCols * 4) < kFixRows
                                   ? (L::kRingBytes - L::kRedBytes) / (kBandCols * 4)
                                   : kFixRows;
    static_assert(kStageRows >= 4, "room to stage the fix-up");
    const int rows0 = fix[0] ? last_s[0] - first_s[0] + 1 : 0;
    const int rows_all = rows0 + (fix[1] ? last_s[1] - first_s[1] + 1 : 0);
    float acc[kE];
#pragma unroll
    for (int u = 0; u < kE; ++u) acc[u] = 0.0f;
    for (int r0 = 0; r0 < rows_all; r0 += kStageRows) {
      const int rows = min(kStageRows, rows_all - r0);
      constexpr int kU = 8;   // loads in flight per thread (a whole batch at 256 or 512 threads)
      for (int e0 = threadIdx.x; e0 < rows * (kBandCols / 4); e0 += kU * W * 32) {
        float4 vv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int e = e0 + u * W * 32, r = r0 + e / (kBandCols / 4), c4 = e % (kBandCols / 4);
          const int s = r < rows0 ? 0 : 1;
          const int i = s == 0 ? first_s[0] + r : first_s[1] + (r - rows0);   // contributor CTA
          // the band's slot in CTA i: every contributor after the first starts inside the band
          const int slot = i != (s == 0 ? first_s[0] : first_s[1]) ? 0 : s_bounds[4 + s];
          if (e < rows * (kBandCols / 4))
            vv[u] = __ldcg(reinterpret_cast<const float4*>(p.parts + ((size_t)i * 2 + slot) * kBandCols) + c4);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u)
          if (e0 + u * W * 32 < rows * (kBandCols / 4)) reinterpret_cast<float4*>(stage)[e0 + u * W * 32] = vv[u];
      }
      __syncthreads();
#pragma unroll
      for (int u = 0; u < kE; ++u) {
        const int e = threadIdx.x + u * W * 32, s = e / kBandCols, t = e % kBandCols;
        if (e < 2 * kBandCols && (s == 0 ? fix[0] : fix[1])) {
          const int rb = s == 0 ? r0 : max(r0, rows0);
          const int re = s == 0 ? min(r0 + rows, rows0) : r0 + rows;
          for (int r = rb; r < re; ++r) acc[u] += stage[(r - r0) * kBandCols + t];   // in CTA order
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < kE; ++u) {
      const int e = threadIdx.x + u * W * 32, s = e / kBandCols;
      if (e < 2 * kBandCols && (s == 0 ? fix[0] : fix[1])) v[u] = acc[u];
    }
  }
  // the final values of the bands this CTA owns
#pragma unroll
  for (int u = 0; u < kE; ++u) {
    const int e = threadIdx.x + u * W * 32, s = e / kBandCols, t = e % kBandCols;
    if (e >= 2 * kBandCols || !(s == 0 ? own[0] : own[1])) continue;
    const int col = (band0 + s) * kBandCols + t;
    float out = v[u];
    if (col < p.N && p.bias) out += __half2float(p.bias[col]);
    if (!PEER) {
      if (col < p.N) p.y[col] = __float2half_rn(out);
    } else {
      s_y[s * kBandCols + t] = __float2half_rn(out);
    }
  }
  if (PEER) {
    __syncthreads();
    // 16-byte stores of 8 columns each into every rank's output (its own included)
    if (threadIdx.x < 2 * (kBandCols / 8)) {
      const int s = threadIdx.x / (kBandCols / 8), c8 = threadIdx.x % (kBandCols / 8);
      const int col = (band0 + s) * kBandCols + 8 * c8;
      if ((s == 0 ? own[0] : own[1]) && col < p.N) {
        const uint4 val = reinterpret_cast<const uint4*>(s_y)[threadIdx.x];
        for (int r = 0; r < p.world; ++r) *reinterpret_cast<uint4*>(p.peer_y[r] + p.col_base + col) = val;
      }
    }
    __syncthreads();
    const int nfin = (int)own[0] + (int)own[1];
    if (threadIdx.x == 0 && nfin > 0) {
      __threadfence_system();   // the CTA's peer stores (ordered by the barrier) reach every rank first
      const int done = atomicAdd(p.tickets + kRankTicket, nfin);
      if (done + nfin == p.bands) {
        p.tickets[kRankTicket] = 0;   // re-armed for the next launch
        s_done = 1;
      }
    }
    __syncthreads();
  }
  // PEER: the CTA that completed the rank's last band raises this rank's flag in
  // every rank and waits (bounded) until every rank's flag reached this call
  if (PEER && s_done && threadIdx.x == 0) {
    __threadfence_system();   // with the relaxed stores below: the release of this rank's flag
    const unsigned e = *p.epoch + 1;
    for (int r = 0; r < p.world; ++r) st_relaxed_sys(p.peer_flags[r] + p.tp_rank, e);
    if (p.deferred) {   // the next deferred call (or peer_wait_kernel) waits for the others
      *p.epoch = e;
      return;
    }
    const unsigned* mine = p.peer_flags[p.tp_rank];
    const unsigned long long t_start = globaltimer();
    bool all = false;
    for (uint32_t i = 0; !all; ++i) {
      all = true;
      for (int r = 0; r < p.world; ++r) all &= (int)(ld_acquire_sys(mine + r) - e) >= 0;
      if (!all && (i & 63u) == 63u && globaltimer() - t_start > kWaitLimitNs) {
        if (p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
        break;
      }
    }
    *p.epoch = e;
  }
}

// One thread: waits, bounded by ~1 s, until every rank's flag in this rank's
// array has reached *epoch (this rank's count of fused calls), i.e. until the
// last deferred fused call's row is complete here.
__global__ void peer_wait_kernel(const unsigned* flags, int world, const unsigned* epoch, int* dev_err) {
  const unsigned e = *epoch;
  const unsigned long long t_start = globaltimer();
  bool all = false;
  for (uint32_t i = 0; !all; ++i) {
    all = true;
    for (int r = 0; r < world; ++r) all &= (int)(ld_acquire_sys(flags + r) - e) >= 0;
    if (!all && (i & 63u) == 63u && globaltimer() - t_start > kWaitLimitNs) {
      if (dev_err) atomicOr(dev_err, ANVILQ_DEV_ERR_TIMEOUT);
      break;
    }
  }
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

using KernelFn = void (*)(CUtensorMap, Params);
struct Variant {
  int warps, stages;
  KernelFn fn, peer_fn;   // y to this GPU / y stored into every rank (the fused all-gather)
  int smem;
};
#define ANVILQ_STREAM_VARIANT(W, S) \
  {W, S, gemv_stream_kernel<W, S, false>, gemv_stream_kernel<W, S, true>, Layout<W, S>::kBytes}
// (warps per CTA, ring stages per warp)
static const Variant kVariants[] = {
    ANVILQ_STREAM_VARIANT(8, 3),  ANVILQ_STREAM_VARIANT(8, 2),  ANVILQ_STREAM_VARIANT(8, 4),
    ANVILQ_STREAM_VARIANT(16, 2), ANVILQ_STREAM_VARIANT(16, 3), ANVILQ_STREAM_VARIANT(4, 4),
};
#undef ANVILQ_STREAM_VARIANT

static const Variant* variant(int warps, int stages) {
  for (const Variant& v : kVariants)
    if (v.warps == warps && v.stages == stages) return &v;
  return nullptr;
}

constexpr int kMaxDevices = 64;
struct DeviceInfo {
  int sms = 0;
};
static DeviceInfo g_dev[kMaxDevices];
static std::once_flag g_dev_once[kMaxDevices];

static const DeviceInfo* device_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(g_dev_once[dev], [dev] {
    DeviceInfo& d = g_dev[dev];
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    for (size_t i = 0; i < sizeof(kVariants) / sizeof(kVariants[0]); ++i) {
      const Variant& v = kVariants[i];
      cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, v.smem);
      cudaFuncSetAttribute(v.peer_fn, cudaFuncAttributeMaxDynamicSharedMemorySize, v.smem);
    }
    cudaGetLastError();
  });
  return &g_dev[dev];
}

}  // namespace stream_gemv

bool gemv_stream_supported(const void* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                           int K, int N, int G) {
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  return K % stream_gemv::kChunkRows == 0 && G % stream_gemv::kChunkRows == 0 && K % G == 0 && N % 32 == 0 &&
         a16(x) && a16(qweight) && a16(qzeros) && a16(scales) &&
         (long long)((N / 8 + stream_gemv::kBandWords - 1) / stream_gemv::kBandWords) * (K / stream_gemv::kChunkRows) <
             (1ll << 30) &&
         stream_gemv::encode_fn() != nullptr;
}

// Default plan, from sweeps on B200 over the 7B / 70B-class projection shapes
// (the 16 KB and 8 KB ring variants x 1 or 2 CTAs per SM): one CTA per SM
// (two per SM lost 5-60 %: the per-CTA fix-up and tail cost more than the
// extra warps hide), two ring stages, 16 warps for layers of >= 8192 columns
// and 8 below; never fewer CTAs than bands, never more than chunks.
bool gemv_stream_default_plan(int K, int N, GemvPlan* plan) {
  using namespace stream_gemv;
  const DeviceInfo* d = device_info();
  if (!d || d->sms <= 0) return false;
  const Variant* v = variant(N >= 8192 ? 16 : 8, 2);
  const int bands = (N / 8 + kBandWords - 1) / kBandWords;
  const long long T = (long long)bands * (K / kChunkRows);
  long long ctas = std::max<long long>(d->sms, bands);
  ctas = std::min<long long>(ctas, T);
  plan->kernel = ANVILQ_GEMV_KERNEL_STREAM;
  plan->band_cols = kBandCols;
  plan->cluster = 1;
  plan->kc = 1;
  plan->warps = v->warps;
  plan->stages = v->stages;
  plan->ctas = (int)ctas;
  return true;
}

// The plan's shape rules; returns ANVILQ_OK or the status to report.
int gemv_stream_check_plan(int K, int N, const GemvPlan& pl) {
  using namespace stream_gemv;
  const DeviceInfo* d = device_info();
  if (!d || d->sms <= 0) return ANVILQ_ECUDA;
  const Variant* v = variant(pl.warps, pl.stages);
  if (!v || pl.band_cols != kBandCols || pl.cluster != 1 || pl.kc != 1) return ANVILQ_EINVAL;
  const int bands = (N / 8 + kBandWords - 1) / kBandWords;
  const int cpb = K / kChunkRows;
  const long long T = (long long)bands * cpb;
  // every CTA holds at least one chunk and its range touches at most two bands
  if (pl.ctas < 1 || pl.ctas > T || (T + pl.ctas - 1) / pl.ctas > cpb) return ANVILQ_ESHAPE;
  if (bands >= kRankTicket) return ANVILQ_ESHAPE;   // band tickets and the rank ticket share the counters
  return ANVILQ_OK;
}

size_t gemv_stream_workspace_bytes(const GemvPlan& pl) {
  return ANVILQ_WORKSPACE_COUNTER_BYTES + (size_t)pl.ctas * 2 * stream_gemv::kBandCols * sizeof(float);
}

int launch_gemv_stream(const GemvPlan& pl, const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                       const uint16_t* scales, const uint16_t* bias, uint16_t* y, int K, int N, int G,
                       void* workspace, size_t workspace_bytes, int* dev_err, cudaStream_t stream,
                       bool overlap_prior, const GemvIo* peer) {
  using namespace stream_gemv;
  const int rc = gemv_stream_check_plan(K, N, pl);
  if (rc != ANVILQ_OK) return rc;
  auto encode = encode_fn();
  if (!encode) return ANVILQ_ECUDA;
  const Variant* v = variant(pl.warps, pl.stages);
  const int W8 = N / 8;
  const int bands = (W8 + kBandWords - 1) / kBandWords;
  if (peer) {
    if (peer->world < 1 || peer->world > kMaxPeers || peer->tp_rank < 0 || peer->tp_rank >= peer->world ||
        !peer->epoch || peer->col_base % 8)
      return ANVILQ_EINVAL;
    for (int r = 0; r < peer->world; ++r) {
      if (!peer->peer_y[r] || !peer->peer_flags[r]) return ANVILQ_EINVAL;
      if (reinterpret_cast<uintptr_t>(peer->peer_y[r]) & 15u) return ANVILQ_EALIGN;
    }
  } else if (!y) {
    return ANVILQ_EINVAL;
  }
  if (!workspace || workspace_bytes < gemv_stream_workspace_bytes(pl)) return ANVILQ_EWORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) return ANVILQ_EALIGN;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)W8, (cuuint64_t)K};
  const cuuint64_t strides[1] = {(cuuint64_t)W8 * 4};
  const cuuint32_t box[2] = {(cuuint32_t)kBandWords, (cuuint32_t)kChunkRows};
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
  p.tickets = reinterpret_cast<int*>(workspace);
  p.parts = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + ANVILQ_WORKSPACE_COUNTER_BYTES);
  p.dev_err = dev_err;
  p.K = K;
  p.N = N;
  p.W8 = W8;
  p.G = G;
  p.cpb = K / kChunkRows;
  p.cpg = G / kChunkRows;
  p.total = bands * p.cpb;
  p.bands = bands;
  for (int r = 0; r < kMaxPeers; ++r) {
    p.peer_y[r] = peer && r < peer->world ? reinterpret_cast<__half*>(peer->peer_y[r]) : nullptr;
    p.peer_flags[r] = peer && r < peer->world ? peer->peer_flags[r] : nullptr;
  }
  p.epoch = peer ? peer->epoch : nullptr;
  p.world = peer ? peer->world : 0;
  p.tp_rank = peer ? peer->tp_rank : 0;
  p.col_base = peer ? peer->col_base : 0;
  p.deferred = peer && peer->deferred ? 1 : 0;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.ctas, 1, 1);
  cfg.blockDim = dim3(v->warps * 32, 1, 1);
  cfg.dynamicSmemBytes = v->smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap_prior ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, peer ? v->peer_fn : v->fn, map, p) != cudaSuccess) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  return ANVILQ_OK;
}

int launch_peer_wait(const unsigned* flags, int world, const unsigned* epoch, int* dev_err, cudaStream_t stream) {
  stream_gemv::peer_wait_kernel<<<1, 1, 0, stream>>>(flags, world, epoch, dev_err);
  if (cudaGetLastError() != cudaSuccess) return ANVILQ_ECUDA;
  return ANVILQ_OK;
}

}  // namespace anvilq
