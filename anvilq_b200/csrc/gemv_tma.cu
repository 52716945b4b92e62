// gemv_tma.cu -- batch-1 W4A16 AWQ GEMV for B200: TMA-staged int4 stream,
// two-level split-K (thread-block cluster + workspace), DSMEM push reduction.
//
// Reference semantics: FP32Model.linear (anvil-q1/tests/official_weights.py:418-437),
//   y[c] = sum_k x[k] * (u4 q[k][c] - u4 z[k/G][c]) * scale[k/G][c]  (+ bias[c]).
//
// Data movement.  The int4 matrix is the only large operand.  A band is 64
// consecutive qweight words of every row (256 B per row, 512 output columns);
// a tile is 16 rows of a band (4 KB), fetched by ONE cp.async.bulk.tensor.2d
// from a tensor map over qweight [K][N/8], together with the tile's 16
// activations (a 32-byte bulk copy) on the same mbarrier.  Every warp streams
// its own range of tiles through a private ring of 3 or 4 stages (chosen per
// plan), so bytes in flight cost no registers: four 4-warp CTAs fit on an SM
// with 3 stages, three with 4 (up to 192 KB in flight either way).  Tiles past
// the last row or column are zero-filled by the TMA unit and contribute nothing.
//
// Split-K, two levels.  The c CTAs of a thread-block cluster and kc clusters
// share one band; the band's tiles are split evenly over all their warps.
// Warps are reduced in shared memory; the CTA of rank r owns column slice r
// of the band, every CTA stores its sum of that slice straight into the
// owner's shared memory (DSMEM), and after a single cluster barrier the owner
// adds the c partials in rank order.  With kc > 1 every cluster leaves
// one partial per column slice in the workspace and the CTA that arrives last
// at the slice's ticket adds the kc partials in cluster order.  Every sum has a
// fixed order, so results are bit-reproducible; there are no atomics on data
// and no waits on other CTAs.
//
// Arithmetic (per thread: 2 words = 16 columns x the 16 rows of a tile):
//   * q is used as a binary16 SUBNORMAL: (w & 0x000F000F) reinterpreted as
//     half2 is exactly (q0, q1) * 2^-24, (w & 0x00F000F0) is 16 (q2, q3) 2^-24,
//     and the same on w >> 8 for lanes 4..7.  One AND per column pair.
//   * Each product x * q 2^-24 is formed exactly and added into an fp32
//     accumulator by the mixed-precision fma.rn.f32.f16 (binary16 operands,
//     binary32 addend and result): one instruction per weight, one rounding,
//     no binary16 partial sums.
//   * Per group the accumulators hold 2^-24 sum x q (2^-20 for the shifted
//     pairs); the zero point is applied once through the group's sum of x,
//     sum x (q - z) = sum x q - z sum x, and the scale once: y += s (A - z X).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "../../include/anvilq.h"
#include "awq_common.cuh"
#include "internal.h"

namespace anvilq {
namespace tma_gemv {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kBandWords = 64;                          // 256 B per row, 512 columns
constexpr int kBandCols = kBandWords * 8;
constexpr int kTileRows = 16;
constexpr int kMinStages = 3, kMaxStages = 4;   // ring depth per warp (template parameter S)
constexpr int kTileBytes = kTileRows * kBandWords * 4;  // 4 KB
constexpr int kMaxCluster = 16;
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

// dynamic shared memory layout for a ring of S stages per warp: S = 3 fits
// four CTAs on an SM, S = 4 three (each warp with a third more bytes in flight)
template <int S>
struct Smem {
  static constexpr int kRingOff = 0;
  static constexpr int kRingBytes = kWarps * S * kTileBytes;                 // 48 / 64 KB
  static constexpr int kXsOff = kRingOff + kRingBytes;                       // [warp][16] half (+pad)
  // per stage: 128 B of raw activation rows: [0, 64) primary (fp16 x, fp32 residual
  // or fp16 gate rows), [64, 128) secondary (fp16 gamma or fp16 up rows)
  static constexpr int kXrawStage = 128;
  static constexpr int kXrawOff = kXsOff + kWarps * kTileRows * 4;           // [warp][stage][128 B]
  static constexpr int kBarOff = kXrawOff + kWarps * S * kXrawStage;         // [warp][stage] u64
  static constexpr int kPartOff = kBarOff + kWarps * S * 8 + 32;             // [512] f32
  static constexpr int kBytes = kPartOff + kBandCols * 4;
};
constexpr int kRedBytes = kWarps * kBandCols * 4;                            // 8 KB, aliases the ring
static_assert(kRedBytes <= Smem<kMinStages>::kRingBytes, "reduction buffer reuses the ring");
constexpr int smem_bytes(int stages) { return stages == 3 ? Smem<3>::kBytes : Smem<4>::kBytes; }

// Where the GEMV's activation row k comes from (template parameter XMODE):
//   kXHalf     x[k] (fp16)
//   kXRmsNorm  fp16( r[k] * gamma[k] / sqrt(mean(r^2) + eps) ), r an fp32 residual stream
//   kXSiluMul  fp16( silu(g[k]) * u[k] ), g = x[0:K], u = x[K:2K] (a fused gate/up output)
// and where the result goes (YMODE):
//   kYHalf     y[c] = fp16(result (+ bias))
//   kYResidual r_out[c] += result (+ bias), fp32 in place
//   kYRope     the QKV projection of a decode step: y = fp16(result (+ bias))
//              is never stored; its q and k heads are rotated (split-half RoPE
//              at position *pos) into q_out and row *pos of the K cache, its
//              v heads copied to row *pos of the V cache, *seqlen = *pos + 1
//              -- the same operations, in the same precision, as the separate
//              RoPE/append kernel applied to the stored y.
//   kYPeer     one rank's column slice of a tensor-parallel split: y = fp16(result
//              (+ bias)) stored at columns [col0, col0 + N) of every rank's
//              full-width output (peer memory over NVLink), then the ranks'
//              completion flags exchanged, so that when the kernel completes
//              the full row is present on every rank (the all-gather fused in).
//   kYMlp      the decode step's MLP: this GEMV is gate/up in unit-interleaved
//              columns (per 32 intermediate rows: 32 gate then 32 up columns);
//              each slice owner forms fp16(silu(fp16 g) * fp16 u) for its rows
//              (as kXSiluMul would from the stored gate/up output), multiplies
//              them with its rows of the down matrix (prefetched at the start),
//              and the partials are summed over the cluster (distributed shared
//              memory, rank order) and then over the bands (workspace, band
//              order, by the last band to arrive) into the fp32 residual.
enum XMode { kXHalf = 0, kXRmsNorm = 1, kXSiluMul = 2 };
//   kYAct      gate/up in the same unit-interleaved columns; y = the activations
//              fp16(silu(fp16 g) * fp16 u) [N / 2] -- what the SiLU prologue of
//              the down projection would compute from the stored gate/up output,
//              so the down projection reads them as fp16 x (kXHalf), bit-identical.
enum YMode { kYHalf = 0, kYResidual = 1, kYRope = 2, kYPeer = 3, kYMlp = 4, kYAct = 5 };
constexpr int kMaxRopePairs = 64;   // head_dim <= 128 in the fused RoPE epilogue
constexpr int kMlpMaxBytes = 64 * 1024;   // kYMlp: down rows, meta and slots per CTA
constexpr int kMaxPeers = 8;        // ranks of a fused all-gather

struct Params {
  const __half* x;         // kXHalf, kXSiluMul
  const float* xr;         // kXRmsNorm: fp32 residual [K]
  const __half* gamma;     // kXRmsNorm: [K]
  float eps;
  const int32_t* qzeros;
  const __half* scales;
  const __half* bias;
  __half* y;               // kYHalf
  float* yr;               // kYResidual: fp32 residual [N], updated in place
  float* partials;   // [bands][kc][512]   (kc > 1)
  int* tickets;      // [bands][c]         (kc > 1)
  int* dev_err;
  int K, N, W8, G;
  int cluster;       // c: CTAs per cluster
  int kc;            // clusters per band
  int tiles;         // tiles per band = ceil(K / 16)
  // kYRope only
  const int* rope_pos;     // position of the token
  __half* q_out;           // [Hq][D]
  __half* k_cache;         // [Tmax][Hkv][D]
  __half* v_cache;
  int* seqlen;             // optional
  int Hq, Hkv, D, Tmax;
  double rope_inv[kMaxRopePairs];   // theta^(-2i/D), binary64, computed on the host
  // kYPeer only
  __half* peer_y[kMaxPeers];         // every rank's full-width y [n_full] (this rank's included)
  unsigned* peer_flags[kMaxPeers];   // every rank's flag array [kMaxPeers]
  unsigned* epoch;                   // this rank's count of fused calls (device)
  int world, tp_rank, col_base;      // col_base: first column of this rank's slice
  // kYMlp only (yr: the residual the down projection is added to)
  const int32_t* dn_qweight;   // down [I][H / 8]
  const int32_t* dn_qzeros;    // [I / G][H / 8]
  const __half* dn_scales;     // [I / G][H]
  int dn_H;                    // H: the down projection's output width
  int dn_rows;                 // intermediate rows per slice owner (per / 2)
  int dn_groups;               // down groups a slice owner's rows can touch (1 or 2)
  int bands;                   // clusters of the launch (kc == 1)
  int mlp_off;                 // dynamic shared memory offset of the down region
};
// kYMlp shared memory after the GEMV's own layout: the owner's down rows
// [rows][H/8] words, its groups' zero points [groups][H/8] words and scales
// [groups][H] fp16, its rows' activations (fp16), the cluster's partial slices
// [c][H/c] fp32 and one mbarrier for the prefetch.
struct MlpSmem {
  int w, z, s, act, dslots, bar, bytes;
  __host__ __device__ MlpSmem(int H, int rows, int groups, int c) {
    w = 0;
    z = w + rows * H / 2;
    s = z + groups * H / 2;
    act = s + groups * H * 2;
    dslots = act + ((rows * 2 + 15) / 16) * 16;
    bar = dslots + c * (H / c) * 4;
    bytes = bar + 16;
  }
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
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the same shared-memory address in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t dsmem_addr_u32(uint32_t local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  return remote;
}
__device__ __forceinline__ void st_dsmem_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// v into another CTA's shared memory, its 4 bytes counted on that CTA's mbarrier
__device__ __forceinline__ void st_async_f32(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(addr),
               "r"(__float_as_uint(v)), "r"(bar)
               : "memory");
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
__device__ __forceinline__ half2 h2(uint32_t u) { return *reinterpret_cast<half2*>(&u); }
__device__ __forceinline__ uint32_t u32(half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// a0 += x * q.lo, a1 += x * q.hi with binary16 x and q, binary32 accumulators:
// the products are exact and rounded once into the accumulators.
__device__ __forceinline__ void fma_f32_f16x2(float& a0, float& a1, uint32_t q2, unsigned short x) {
  asm("{\n .reg .f16 q0, q1;\n mov.b32 {q0, q1}, %2;\n"
      " fma.rn.f32.f16 %0, %3, q0, %0;\n fma.rn.f32.f16 %1, %3, q1, %1;\n}"
      : "+f"(a0), "+f"(a1)
      : "r"(q2), "h"(x));
}

template <int XMODE, int YMODE, int BW, int kStages>
__global__ void __launch_bounds__(kThreads, 4)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tmap, const Params p) {
  using L = Smem<kStages>;
  constexpr int kRingOff = L::kRingOff, kXsOff = L::kXsOff, kXrawStage = L::kXrawStage, kXrawOff = L::kXrawOff,
                kBarOff = L::kBarOff, kPartOff = L::kPartOff;
  // Band geometry: BW qweight words (8 BW columns) per band.  A lane owns PW
  // consecutive words of a row; LPR lanes cover a row, and the warp's NRS row
  // sets take the tile's rows in turn (row r belongs to row set r % NRS).
  constexpr int PW = BW == 64 ? 2 : 1;
  constexpr int LPR = BW / PW;
  constexpr int NRS = 32 / LPR;
  constexpr int kCols = BW * 8;
  constexpr int kTileB = kTileRows * BW * 4;
  static_assert(BW == 64 || BW == 32 || BW == 16, "bands of 512, 256 or 128 columns");
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_last;
  __shared__ float s_norm[kWarps + 1];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int c = p.cluster;
  const int rank = c > 1 ? (int)cluster_rank() : 0;
  const int cluster_id = blockIdx.x / c;
  const int band = cluster_id / p.kc, kidx = cluster_id % p.kc;
  const int wi = (kidx * c + rank) * kWarps + warp, nw = p.kc * c * kWarps;
  const int t0 = (int)((long long)wi * p.tiles / nw);
  const int t1 = (int)((long long)(wi + 1) * p.tiles / nw);
  const int ntiles = t1 - t0;

  unsigned char* ring = smem + kRingOff + warp * kStages * kTileBytes;
  uint32_t* xs = reinterpret_cast<uint32_t*>(smem + kXsOff) + warp * kTileRows;
  const unsigned char* xraw = smem + kXrawOff + warp * kStages * kXrawStage;
  const uint32_t xraw0 = smem_u32(smem + kXrawOff) + warp * kStages * kXrawStage;
  const uint32_t bar0 = smem_u32(smem + kBarOff + warp * kStages * 8);
  // the cluster's partial sums arrive as st.async on this CTA's slot barrier
  // (kBarOff pad), which expects all kCols values of its slice from every rank
  const uint32_t slot_bar = smem_u32(smem + kBarOff + kWarps * kStages * 8);
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * s) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap) : "memory");
    if (warp == 0 && c > 1) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(slot_bar) : "memory");
  }
  // kYMlp: this CTA's rows of the down matrix and their groups' zero points and
  // scales do not depend on any earlier kernel: request them now
  const MlpSmem ml(YMODE == kYMlp ? p.dn_H : 32, YMODE == kYMlp ? p.dn_rows : 16, YMODE == kYMlp ? p.dn_groups : 1,
                   YMODE == kYMlp ? c : 1);
  const uint32_t mlp0 = smem_u32(smem + (YMODE == kYMlp ? p.mlp_off : 0));
  const int mlp_i0 = band * (kCols / 2) + rank * p.dn_rows;                      // first intermediate row
  const int mlp_nr = YMODE == kYMlp ? max(0, min(p.dn_rows, p.N / 2 - mlp_i0)) : 0;   // rows below I
  if (YMODE == kYMlp && threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mlp0 + ml.bar) : "memory");
  }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  if (c > 1) {
    if (threadIdx.x == 0)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(slot_bar), "r"(kCols * 4)
                   : "memory");
    // every CTA's slot barrier is initialised before any rank pushes to it: this
    // arrive pairs with the wait just before the pushes
    cluster_arrive_release();
  }
  if (YMODE == kYMlp && threadIdx.x == 0) {
    const int H = p.dn_H, g0 = mlp_i0 / p.G;
    const int ng = mlp_nr > 0 ? (mlp_i0 + mlp_nr - 1) / p.G - g0 + 1 : 0;   // <= dn_groups (host)
    const uint32_t bytes = (uint32_t)mlp_nr * H / 2 + (uint32_t)ng * (H / 2 + 2 * H);
    const uint32_t bar = mlp0 + ml.bar;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    auto bulk = [&](uint32_t d, const void* src, uint32_t n) {
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(d),
                   "l"(src), "r"(n), "r"(bar)
                   : "memory");
    };
    if (mlp_nr > 0) bulk(mlp0 + ml.w, p.dn_qweight + (size_t)mlp_i0 * (H / 8), (uint32_t)mlp_nr * H / 2);
    for (int k = 0; k < ng; ++k) {
      bulk(mlp0 + ml.z + k * (H / 2), p.dn_qzeros + (size_t)(g0 + k) * (H / 8), H / 2);
      bulk(mlp0 + ml.s + k * (2 * H), p.dn_scales + (size_t)(g0 + k) * H, 2 * H);
    }
  }
  // let the next kernel on the stream start its own weight prefetch (programmatic
  // dependent launch); it still waits for this grid before touching our output
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __syncwarp();

  // Stage j % kStages receives tile t0 + j (4 KB of int4 words) and the tile's
  // 16 activation rows (one or two short bulk copies), all counted on the
  // stage's mbarrier.  K % 16 == 0, so every tile has 16 rows.
  constexpr uint32_t x_bytes = XMODE == kXRmsNorm ? 16 * 4 + 16 * 2 : XMODE == kXSiluMul ? 2 * 16 * 2 : 16 * 2;
  auto copy_x = [&](int j, uint32_t bar) {
    const int st = j % kStages;
    const size_t r0 = (size_t)(t0 + j) * kTileRows;
    const uint32_t dst = xraw0 + st * kXrawStage;
    auto bulk = [&](uint32_t d, const void* src, uint32_t n) {
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(d),
                   "l"(src), "r"(n), "r"(bar)
                   : "memory");
    };
    if (XMODE == kXHalf) bulk(dst, p.x + r0, 32);
    if (XMODE == kXRmsNorm) {
      bulk(dst, p.xr + r0, 64);
      bulk(dst + 64, p.gamma + r0, 32);
    }
    if (XMODE == kXSiluMul) {
      bulk(dst, p.x + r0, 32);
      bulk(dst + 64, p.x + p.K + r0, 32);
    }
  };
  auto issue_tile = [&](int j, bool with_x) {   // lane 0 only
    const int st = j % kStages;
    const uint32_t bar = bar0 + 8 * st;
    // the stage was last read through the generic proxy; order that before the TMA write
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (with_x)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kTileB + x_bytes)
                   : "memory");
    else
      asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(kTileB) : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(ring + st * kTileBytes)),
        "l"(&tmap), "r"(band * BW), "r"((t0 + j) * kTileRows), "r"(bar)
        : "memory");
    if (with_x) copy_x(j, bar);
  };
  auto issue_x = [&](int j) {   // lane 0 only: activations of a tile whose weights are in flight
    const uint32_t bar = bar0 + 8 * (j % kStages);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(x_bytes) : "memory");
    copy_x(j, bar);
  };

  const int lw = lane % LPR, rs = lane / LPR;   // word slot and row set of this lane
  const int w0 = band * BW + lw * PW;             // this lane's PW words = 8 PW columns
  const bool active = w0 < p.W8;
  auto tile_row = [&](int j) { return (t0 + j) * kTileRows; };

  float A[16], Y[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) A[j] = Y[j] = 0.0f;
  float Xg = 0.0f;
  uint4 sc[2] = {}, nsc[2] = {};
  uint2 zq = {}, nzq = {};
  uint32_t bad = 0;
  bool ok = true;

  // scales and zeros of the group of `row`.  Volatile loads: issued here, a
  // group ahead of their use (a plain read-only load may be sunk by the
  // compiler to its use, putting a memory round trip on the critical path).
  auto load_group = [&](int row, uint4* s2, uint2& z) {
    if (active) {
      const int g = row / p.G;
      const __half* sp = p.scales + (size_t)g * p.N + 8 * (size_t)w0;
      s2[0] = ld_stream_v4(sp);
      if (PW == 2) {
        s2[1] = ld_stream_v4(sp + 8);
        z = ld_stream_v2(p.qzeros + (size_t)g * p.W8 + w0);
      } else {
        z.x = ld_stream_u32(p.qzeros + (size_t)g * p.W8 + w0);
      }
    }
  };
  auto check_group = [&](int row) {   // the tile that opens a group checks its scales, once
    if (active && row % p.G == 0) {
#pragma unroll
      for (int i = 0; i < PW; ++i)
        bad |= invalid_scale_pair(sc[i].x) | invalid_scale_pair(sc[i].y) | invalid_scale_pair(sc[i].z) |
               invalid_scale_pair(sc[i].w);
    }
  };
  // y += s (A - z X) for the finished group, this lane's 8 PW columns (X: the
  // group's activations summed over this lane's row set)
  auto flush_group = [&]() {
#pragma unroll
    for (int i = 0; i < PW; ++i) {
      const uint32_t zw = i == 0 ? zq.x : zq.y;
      const uint32_t sw[4] = {sc[i].x, sc[i].y, sc[i].z, sc[i].w};
      // zero points via the binary16 magic 1024 + z, pairs (0,1),(2,3),(4,5),(6,7)
      const uint32_t zp[4] = {(zw & 0x000F000Fu) | 0x64006400u, ((zw >> 4) & 0x000F000Fu) | 0x64006400u,
                              ((zw >> 8) & 0x000F000Fu) | 0x64006400u, ((zw >> 12) & 0x000F000Fu) | 0x64006400u};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 s2 = __half22float2(h2(sw[e]));
        const float2 z2 = __half22float2(h2(zp[e]));
        const float pw = (e & 1) ? 1048576.0f : 16777216.0f;   // 2^20 (shifted pairs) or 2^24
        const float a0 = fmaf(-(z2.x - 1024.0f), Xg, A[i * 8 + 2 * e] * pw);
        const float a1 = fmaf(-(z2.y - 1024.0f), Xg, A[i * 8 + 2 * e + 1] * pw);
        Y[i * 8 + 2 * e] = fmaf(s2.x, a0, Y[i * 8 + 2 * e]);
        Y[i * 8 + 2 * e + 1] = fmaf(s2.y, a1, Y[i * 8 + 2 * e + 1]);
        A[i * 8 + 2 * e] = 0.0f;
        A[i * 8 + 2 * e + 1] = 0.0f;
      }
    }
    Xg = 0.0f;
  };

  // -- prologue: weights first (they do not depend on the previous kernel) ---
  const int pro = min(kStages - 1, ntiles);
  if (lane == 0)
    for (int j = 0; j < pro; ++j) issue_tile(j, false);
  int issued = pro;
  if (ntiles > 0) load_group(tile_row(0), sc, zq);
  asm volatile("griddepcontrol.wait;" ::: "memory");   // x may come from the previous kernel
  if (lane == 0)
    for (int j = 0; j < pro; ++j) issue_x(j);
  float norm_inv = 1.0f;   // kXRmsNorm: 1 / sqrt(mean(r^2) + eps), computed by every CTA
  if (XMODE == kXRmsNorm) {
    // every CTA needs the whole row's norm: 8 vector loads per thread in
    // flight at once (one L2 round trip per 4096 elements), summed in a fixed order
    const float4* xr4 = reinterpret_cast<const float4*>(p.xr);
    const int n4 = p.K / 4;
    float ss = 0.0f;
    for (int base = threadIdx.x; base < n4; base += 8 * kThreads) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        v[u] = base + u * kThreads < n4 ? __ldcg(xr4 + base + u * kThreads) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        ss = fmaf(v[u].x, v[u].x, ss);
        ss = fmaf(v[u].y, v[u].y, ss);
        ss = fmaf(v[u].z, v[u].z, ss);
        ss = fmaf(v[u].w, v[u].w, ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) s_norm[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) t += s_norm[w];
      s_norm[kWarps] = 1.0f / sqrtf(t / (float)p.K + p.eps);
    }
    __syncthreads();
    norm_inv = s_norm[kWarps];
  }
  if (ntiles > 0) check_group(tile_row(0));

  for (int j = 0; j < ntiles; ++j) {
    if (issued < ntiles) {
      if (lane == 0) issue_tile(issued, true);
      ++issued;
    }
    const bool next_group = j + 1 < ntiles && tile_row(j + 1) / p.G != tile_row(j) / p.G;
    if (next_group) load_group(tile_row(j + 1), nsc, nzq);   // lands while this tile computes
    const int st = j % kStages;
    const bool landed = mbar_wait_bounded(bar0 + 8 * st, (j / kStages) & 1);
    if (!__all_sync(0xffffffffu, landed)) {
      ok = false;
      break;
    }
    // -- the tile's activations: lanes l and l + 16 both hold row l % 16
    float Xt;
    {
      // this row's activation, rounded to binary16 (the A16 of W4A16)
      const unsigned char* xr0 = xraw + st * kXrawStage;
      const int r = lane & 15;
      float xf;
      if (XMODE == kXHalf) xf = __half2float(reinterpret_cast<const __half*>(xr0)[r]);
      if (XMODE == kXRmsNorm) {
        const float v = reinterpret_cast<const float*>(xr0)[r];
        const float gm = __half2float(reinterpret_cast<const __half*>(xr0 + 64)[r]);
        xf = __half2float(__float2half_rn(v * gm * norm_inv));
      }
      if (XMODE == kXSiluMul) {
        const float g = __half2float(reinterpret_cast<const __half*>(xr0)[r]);
        const float u = __half2float(reinterpret_cast<const __half*>(xr0 + 64)[r]);
        const float e = expf(-fabsf(g));   // stable silu (official_weights.py:494-499)
        const float sg = g >= 0.0f ? g / (1.0f + e) : (g * e) / (1.0f + e);
        xf = __half2float(__float2half_rn(sg * u));
      }
      // the sum of this lane's row set: all 16 rows (NRS 1), or the rows of one
      // parity (xor 2..8), taken from lane rs, whose row has parity rs (NRS 2)
      float sum = xf;
#pragma unroll
      for (int o = NRS; o < 16; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (NRS == 2) sum = __shfl_sync(0xffffffffu, sum, rs);
      if (lane < 16) reinterpret_cast<__half*>(xs)[lane] = __float2half_rn(xf);
      Xt = sum;
    }
    __syncwarp();
    const unsigned char* tile = ring + st * kTileBytes + lw * PW * 4;
    // one qweight word (8 columns) times one activation into A[8 i .. 8 i + 7]
    auto word_fma = [&](int i, uint32_t wd, unsigned short xv) {
      const uint32_t w8 = wd >> 8;
      fma_f32_f16x2(A[i * 8 + 0], A[i * 8 + 1], wd & 0x000F000Fu, xv);   // columns 0,1
      fma_f32_f16x2(A[i * 8 + 2], A[i * 8 + 3], wd & 0x00F000F0u, xv);   // columns 2,3 (x16)
      fma_f32_f16x2(A[i * 8 + 4], A[i * 8 + 5], w8 & 0x000F000Fu, xv);   // columns 4,5
      fma_f32_f16x2(A[i * 8 + 6], A[i * 8 + 7], w8 & 0x00F000F0u, xv);   // columns 6,7 (x16)
    };
    if (NRS == 1) {
#pragma unroll
      for (int r = 0; r < kTileRows; r += 2) {
        const uint32_t xpair = xs[r / 2];   // rows r, r + 1
        const unsigned short xr_[2] = {(unsigned short)(xpair & 0xFFFFu), (unsigned short)(xpair >> 16)};
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          if (PW == 2) {
            const uint2 w = *reinterpret_cast<const uint2*>(tile + (r + rr) * (BW * 4));
            word_fma(0, w.x, xr_[rr]);
            word_fma(1, w.y, xr_[rr]);
          } else {
            word_fma(0, *reinterpret_cast<const uint32_t*>(tile + (r + rr) * (BW * 4)), xr_[rr]);
          }
        }
      }
    } else {
      const unsigned short* xh = reinterpret_cast<const unsigned short*>(xs);
#pragma unroll
      for (int i2 = 0; i2 < kTileRows / NRS; ++i2) {
        const int r = NRS * i2 + rs;
        word_fma(0, *reinterpret_cast<const uint32_t*>(tile + r * (BW * 4)), xh[r]);
      }
    }
    __syncwarp();   // stage st and xs are free again
    Xg += Xt;
    if (next_group) {
      flush_group();
      sc[0] = nsc[0];
      sc[1] = nsc[1];
      zq = nzq;
      check_group(tile_row(j + 1));
    }
  }
  if (ok && ntiles > 0) flush_group();
  if (!ok) {
    if (lane == 0 && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
    for (int j = max(0, issued - kStages); j < issued; ++j)
      mbar_wait_bounded(bar0 + 8 * (j % kStages), (j / kStages) & 1);
#pragma unroll
    for (int j = 0; j < 16; ++j) Y[j] = 0.0f;
  }
  if (bad && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SCALE);
  if (NRS == 2) {   // the two row sets of a word slot: lanes l and l ^ 16
#pragma unroll
    for (int j = 0; j < 8; ++j) Y[j] += __shfl_xor_sync(0xffffffffu, Y[j], 16);
  }

  // -- reduce: warps (shared memory, reusing the ring), then the cluster (pushed
  //    over DSMEM to the slice owners), then the kc clusters of the band (workspace)
  __syncthreads();   // every warp is done with its ring
  float* red = reinterpret_cast<float*>(smem + kRingOff);   // [warp][512]
  if (lane < LPR) {
#pragma unroll
    for (int j = 0; j < 8 * PW; j += 4)
      *reinterpret_cast<float4*>(red + warp * kCols + lw * 8 * PW + j) =
          make_float4(Y[j], Y[j + 1], Y[j + 2], Y[j + 3]);
  }
  __syncthreads();
  // The band's columns are owned in slices of per = 512 / c columns, slice r
  // by the CTA of rank r.  Each CTA sums its warps and pushes slice r of that
  // sum into slot [its rank] of owner r (distributed shared memory); after one
  // cluster barrier every owner holds all c partials of its slice locally.
  float* slots = reinterpret_cast<float*>(smem + kPartOff);   // [c][per]
  const int per = kCols / c;              // this CTA's column slice of the band
  const int col0 = band * kCols + rank * per;
  const uint32_t slots_u32 = smem_u32(slots);
  // slot position L of a band column: the column itself, or for kYRope the
  // pair order (head, i, half) that gives every owner both columns i and
  // i + D/2 of the heads' dims it owns (bands hold whole heads)
  auto slot_of = [&](int col) {
    // kYMlp: band column (unit u, gate/up half, i) -> 2 (32 u + i) + half, so an
    // owner's slice holds (gate, up) pairs of per / 2 intermediate rows
    if (YMODE == kYMlp || YMODE == kYAct) return 2 * ((col / 64) * 32 + col % 32) + (col % 64) / 32;
    if (YMODE != kYRope) return col;
    const int hd = p.D / 2, head = col / p.D, j = col % p.D;
    return 2 * (head * hd + j % hd) + (j >= hd ? 1 : 0);
  };
  if (c > 1) cluster_wait_acquire();   // every rank's slot barrier is initialised
  for (int col = threadIdx.x; col < kCols; col += kThreads) {
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[w * kCols + col];
    const int L = slot_of(col);
    if (c > 1) {
      const uint32_t owner = (uint32_t)(L / per);
      st_async_f32(dsmem_addr_u32(slots_u32 + (rank * per + L % per) * 4, owner), v,
                   dsmem_addr_u32(slot_bar, owner));
    } else {
      slots[L] = v;
    }
  }
  if (c > 1) {
    // the owner proceeds once all c slices of its columns have landed (every
    // CTA of the cluster pushes every column, errors included); no cluster-wide
    // barrier: the mbarrier's completion makes the asynchronous stores visible
    if (!mbar_wait_bounded(slot_bar, 0) && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
  } else {
    __syncthreads();
  }
  if (YMODE == kYPeer) {   // kc == 1 (the host plan guarantees it)
    for (int t = threadIdx.x; t < per; t += kThreads) {
      if (col0 + t >= p.N) continue;
      float out = slots[t];
      for (int k = 1; k < c; ++k) out += slots[k * per + t];   // in rank order, as for kYHalf
      if (p.bias) out += __half2float(p.bias[col0 + t]);
      const __half h = __float2half_rn(out);
      for (int r = 0; r < p.world; ++r) p.peer_y[r][p.col_base + col0 + t] = h;
    }
    // every CTA's stores are ordered before its ticket; the last CTA to arrive
    // raises this rank's flag in every rank, then waits (bounded) for all flags
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const int n = atomicAdd_system(p.tickets, 1);
      s_last = n == (int)gridDim.x - 1;
      if (s_last) p.tickets[0] = 0;   // re-armed for the next launch
    }
    __syncthreads();
    if (!s_last || threadIdx.x != 0) return;
    __threadfence_system();   // with the relaxed stores below: the release of this rank's flag
    const unsigned e = *p.epoch + 1;
    for (int r = 0; r < p.world; ++r) st_relaxed_sys(p.peer_flags[r] + p.tp_rank, e);
    const unsigned* mine = p.peer_flags[p.tp_rank];
    const unsigned long long t_start = globaltimer();
    bool done = false;
    for (uint32_t i = 0; !done; ++i) {
      done = true;
      for (int r = 0; r < p.world; ++r) done &= (int)(ld_acquire_sys(mine + r) - e) >= 0;
      if (!done && (i & 63u) == 63u && globaltimer() - t_start > kWaitLimitNs) {
        if (p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
        break;
      }
    }
    *p.epoch = e;
    return;
  }
  if (YMODE == kYRope) {   // kc == 1 (the host plan guarantees it)
    const int hd = p.D / 2;
    const int pos = *p.rope_pos;
    const bool pos_ok = pos >= 0 && pos < p.Tmax;
    if (!pos_ok) {
      if (band == 0 && rank == 0 && threadIdx.x == 0 && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SEQLEN);
      return;
    }
    for (int q2 = threadIdx.x; q2 < per / 2; q2 += kThreads) {
      float va = slots[2 * q2], vb = slots[2 * q2 + 1];
      for (int k = 1; k < c; ++k) {   // in rank order, as for the stored projection
        va += slots[k * per + 2 * q2];
        vb += slots[k * per + 2 * q2 + 1];
      }
      const int pr = (rank * per) / 2 + q2;   // pair index within the band
      const int i = pr % hd;
      const int ca = band * kCols + (pr / hd) * p.D + i, cb = ca + hd;
      if (ca >= p.N) continue;
      if (p.bias) {
        va += __half2float(p.bias[ca]);
        vb += __half2float(p.bias[cb]);
      }
      const __half ha = __float2half_rn(va), hb = __float2half_rn(vb);
      const int head = ca / p.D;
      if (head < p.Hq + p.Hkv) {
        const float angle = (float)((double)pos * p.rope_inv[i]);
        float si, co;
        sincosf(angle, &si, &co);
        const float xa = __half2float(ha), xb = __half2float(hb);
        const float ra = __fsub_rn(__fmul_rn(xa, co), __fmul_rn(xb, si));
        const float rb = __fadd_rn(__fmul_rn(xb, co), __fmul_rn(xa, si));
        __half* dst = head < p.Hq ? p.q_out + (size_t)head * p.D
                                  : p.k_cache + ((size_t)pos * p.Hkv + (head - p.Hq)) * p.D;
        dst[i] = __float2half_rn(ra);
        dst[i + hd] = __float2half_rn(rb);
      } else {
        __half* dst = p.v_cache + ((size_t)pos * p.Hkv + (head - p.Hq - p.Hkv)) * p.D;
        dst[i] = ha;
        dst[i + hd] = hb;
      }
    }
    if (p.seqlen && band == 0 && rank == 0 && threadIdx.x == 0) *p.seqlen = pos + 1;
    return;
  }
  if (YMODE == kYAct) {   // kc == 1 (the host plan guarantees it)
    // this owner's per / 2 intermediate rows: g and u summed in rank order (as
    // for the stored projection), rounded to fp16, then silu(g) u rounded to fp16
    const int i0 = band * (kCols / 2) + rank * (per / 2);
    for (int j = threadIdx.x; j < per / 2; j += kThreads) {
      if (i0 + j >= p.N / 2) continue;
      float g = slots[2 * j], u = slots[2 * j + 1];
      for (int k = 1; k < c; ++k) {
        g += slots[k * per + 2 * j];
        u += slots[k * per + 2 * j + 1];
      }
      const float gh = __half2float(__float2half_rn(g)), uh = __half2float(__float2half_rn(u));
      const float e = expf(-fabsf(gh));   // stable silu (official_weights.py:494-499)
      const float sg = gh >= 0.0f ? gh / (1.0f + e) : (gh * e) / (1.0f + e);
      p.y[i0 + j] = __float2half_rn(sg * uh);
    }
    return;
  }
  if (YMODE == kYMlp) {   // kc == 1 (the host plan guarantees it)
    const int H = p.dn_H, W8d = H / 8, cs = H / c;   // cs: output columns owned per rank
    __half* act = reinterpret_cast<__half*>(smem + p.mlp_off + ml.act);
    const uint32_t* dnw = reinterpret_cast<const uint32_t*>(smem + p.mlp_off + ml.w);
    const uint32_t* dnz = reinterpret_cast<const uint32_t*>(smem + p.mlp_off + ml.z);
    const __half* dns = reinterpret_cast<const __half*>(smem + p.mlp_off + ml.s);
    float* dslots = reinterpret_cast<float*>(smem + p.mlp_off + ml.dslots);   // [c][cs]
    const uint32_t dslots_u32 = mlp0 + ml.dslots;
    // this owner's rows: g and u summed in rank order (as for the stored
    // projection), rounded to fp16, then silu(g) u rounded to fp16
    for (int j = threadIdx.x; j < p.dn_rows; j += kThreads) {
      float g = slots[2 * j], u = slots[2 * j + 1];
      for (int k = 1; k < c; ++k) {
        g += slots[k * per + 2 * j];
        u += slots[k * per + 2 * j + 1];
      }
      const float gh = __half2float(__float2half_rn(g)), uh = __half2float(__float2half_rn(u));
      const float e = expf(-fabsf(gh));   // stable silu (official_weights.py:494-499)
      const float sg = gh >= 0.0f ? gh / (1.0f + e) : (gh * e) / (1.0f + e);
      act[j] = j < mlp_nr ? __float2half_rn(sg * uh) : __float2half_rn(0.0f);
    }
    const bool landed = mbar_wait_bounded(mlp0 + ml.bar, 0);
    if (!landed && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
    __syncthreads();
    // down partial of this owner's rows: thread t takes words t, t + 128, ...
    // (8 output columns each), one group at a time, flushed as in the tile loop
    const int g0 = mlp_i0 / p.G;
    uint32_t mbad = 0;   // an invalid down scale fails the operation, as in the down GEMV
    for (int w = threadIdx.x; w < W8d; w += kThreads) {
      float Ad[8], Yd[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) Ad[i] = Yd[i] = 0.0f;
      float Xs = 0.0f;
      auto flush_down = [&](int gl) {   // gl: the group's index among this owner's groups
        const uint32_t zw = dnz[gl * W8d + w];
        const uint4 s4 = reinterpret_cast<const uint4*>(dns + (size_t)gl * H)[w];
        const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
        mbad |= invalid_scale_pair(s4.x) | invalid_scale_pair(s4.y) | invalid_scale_pair(s4.z) |
                invalid_scale_pair(s4.w);
        const uint32_t zp[4] = {(zw & 0x000F000Fu) | 0x64006400u, ((zw >> 4) & 0x000F000Fu) | 0x64006400u,
                                ((zw >> 8) & 0x000F000Fu) | 0x64006400u, ((zw >> 12) & 0x000F000Fu) | 0x64006400u};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 s2 = __half22float2(h2(sw[e]));
          const float2 z2 = __half22float2(h2(zp[e]));
          const float pw = (e & 1) ? 1048576.0f : 16777216.0f;   // 2^20 (shifted pairs) or 2^24
          const float a0 = fmaf(-(z2.x - 1024.0f), Xs, Ad[2 * e] * pw);
          const float a1 = fmaf(-(z2.y - 1024.0f), Xs, Ad[2 * e + 1] * pw);
          Yd[2 * e] = fmaf(s2.x, a0, Yd[2 * e]);
          Yd[2 * e + 1] = fmaf(s2.y, a1, Yd[2 * e + 1]);
          Ad[2 * e] = 0.0f;
          Ad[2 * e + 1] = 0.0f;
        }
        Xs = 0.0f;
      };
      if (landed) {
        for (int j = 0; j < mlp_nr; ++j) {
          if (j > 0 && (mlp_i0 + j) % p.G == 0) flush_down((mlp_i0 + j - 1) / p.G - g0);
          const unsigned short xh = __half_as_ushort(act[j]);
          const uint32_t wd = dnw[j * W8d + w], w8 = wd >> 8;
          fma_f32_f16x2(Ad[0], Ad[1], wd & 0x000F000Fu, xh);   // columns 0,1
          fma_f32_f16x2(Ad[2], Ad[3], wd & 0x00F000F0u, xh);   // columns 2,3 (x16)
          fma_f32_f16x2(Ad[4], Ad[5], w8 & 0x000F000Fu, xh);   // columns 4,5
          fma_f32_f16x2(Ad[6], Ad[7], w8 & 0x00F000F0u, xh);   // columns 6,7 (x16)
          Xs += __half2float(act[j]);
        }
        if (mlp_nr > 0) flush_down((mlp_i0 + mlp_nr - 1) / p.G - g0);
      }
      // columns 8w .. 8w + 7 belong to owner 8w / cs (cs % 8 == 0)
      const int owner = (8 * w) / cs, lc = 8 * w - owner * cs;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (c > 1) {
          st_dsmem_f32(dsmem_addr_u32(dslots_u32 + (rank * cs + lc + i) * 4, owner), Yd[i]);
        } else {
          dslots[lc + i] = Yd[i];
        }
      }
    }
    if (mbad && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SCALE);
    if (!landed) mbar_wait_bounded(mlp0 + ml.bar, 0);   // copies in flight land before the CTA can exit
    if (c > 1) {
      cluster_arrive_release();
      cluster_wait_acquire();
    } else {
      __syncthreads();
    }
    // the cluster's (the band's) partial of this rank's columns, summed in rank
    // order, into the workspace; the band arriving last adds every band's
    // partial in band order to the residual
    float* part = p.partials + (size_t)band * H + rank * cs;
    for (int t = threadIdx.x; t < cs; t += kThreads) {
      float v = dslots[t];
      for (int k = 1; k < c; ++k) v += dslots[k * cs + t];
      __stcg(part + t, v);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const int n = atomicAdd(p.tickets + rank, 1);
      s_last = n == p.bands - 1;
      if (s_last) p.tickets[rank] = 0;   // re-armed for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int t = threadIdx.x; t < cs; t += kThreads) {
      const float* col = p.partials + rank * cs + t;
      float acc = 0.0f;
      int b = 0;
      for (; b + 8 <= p.bands; b += 8) {   // eight loads in flight, then the ordered sum
        float r8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) r8[k] = __ldcg(col + (size_t)(b + k) * H);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc += r8[k];
      }
      for (; b < p.bands; ++b) acc += __ldcg(col + (size_t)b * H);
      p.yr[rank * cs + t] += acc;
    }
    return;
  }
  constexpr int kMaxPer = kCols / kThreads;   // up to 4 columns per thread (c == 1)
  float v[kMaxPer];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    v[i] = 0.0f;
    const int t = threadIdx.x + i * kThreads;
    if (t < per) {
      v[i] = slots[t];
      for (int k = 1; k < c; ++k) v[i] += slots[k * per + t];   // in rank order
    }
  }

  if (p.kc > 1) {
    float* slot = p.partials + ((size_t)band * p.kc + kidx) * kCols + rank * per;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int t = threadIdx.x + i * kThreads;
      if (t < per) __stcg(slot + t, v[i]);
    }
    __threadfence();
    __syncthreads();
    int* ticket = p.tickets + band * c + rank;
    if (threadIdx.x == 0) {
      const int n = atomicAdd(ticket, 1);
      s_last = n == p.kc - 1;
      if (s_last) *ticket = 0;   // re-arm for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* base = p.partials + (size_t)band * p.kc * kCols + rank * per;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int t = threadIdx.x + i * kThreads;
      if (t < per) {
        float r[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)   // kc <= 8: all loads first, then the ordered sum
          if (k < p.kc) r[k] = __ldcg(base + (size_t)k * kCols + t);
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (k < p.kc) acc += r[k];
        v[i] = acc;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int t = threadIdx.x + i * kThreads;
    if (t < per && col0 + t < p.N) {
      float out = v[i];
      if (p.bias) out += __half2float(p.bias[col0 + t]);
      if (YMODE == kYHalf) p.y[col0 + t] = __float2half_rn(out);
      if (YMODE == kYResidual) p.yr[col0 + t] += out;
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

constexpr int kMaxDevices = 64;
struct DeviceInfo {
  int sms = 0;
  // co-resident clusters of size 1, 2, 4, 8, 16, for each ring depth
  int max_clusters[kMaxStages - kMinStages + 1][5] = {};
};
static DeviceInfo g_dev[kMaxDevices];
static std::once_flag g_dev_once[kMaxDevices];

using KernelFn = void (*)(CUtensorMap, Params);
constexpr int kBandWidths[3] = {64, 32, 16};   // qweight words per band
template <int XM, int YM, int S>
static KernelFn kernel_bw(int bw) {
  return bw == 64 ? gemv_tma_kernel<XM, YM, 64, S> : bw == 32 ? gemv_tma_kernel<XM, YM, 32, S>
                                                              : gemv_tma_kernel<XM, YM, 16, S>;
}
template <int XM, int S>
static KernelFn kernel_y(int ymode, int bw) {
  if (ymode == kYPeer) {   // the fused all-gather takes fp16 activations
    if constexpr (XM == kXHalf) return kernel_bw<kXHalf, kYPeer, S>(bw);
    return nullptr;
  }
  if (ymode == kYMlp) {   // the MLP reads the residual stream through RMSNorm
    if constexpr (XM == kXRmsNorm) return kernel_bw<kXRmsNorm, kYMlp, S>(bw);
    return nullptr;
  }
  if (ymode == kYAct) {   // gate/up: the residual through RMSNorm, or fp16 x
    if constexpr (XM == kXRmsNorm || XM == kXHalf) return kernel_bw<XM, kYAct, S>(bw);
    return nullptr;
  }
  return ymode == kYHalf ? kernel_bw<XM, kYHalf, S>(bw) : ymode == kYResidual ? kernel_bw<XM, kYResidual, S>(bw)
                                                                            : kernel_bw<XM, kYRope, S>(bw);
}
template <int S>
static KernelFn kernel_s(int xmode, int ymode, int bw) {
  return xmode == kXHalf ? kernel_y<kXHalf, S>(ymode, bw) : xmode == kXRmsNorm ? kernel_y<kXRmsNorm, S>(ymode, bw)
                                                                              : kernel_y<kXSiluMul, S>(ymode, bw);
}
static KernelFn kernel_for(int xmode, int ymode, int bw, int stages) {
  return stages == 3 ? kernel_s<3>(xmode, ymode, bw) : kernel_s<4>(xmode, ymode, bw);
}

static const DeviceInfo* device_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(g_dev_once[dev], [dev] {
    DeviceInfo& d = g_dev[dev];
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    for (int st = kMinStages; st <= kMaxStages; ++st)
      for (int xm = 0; xm < 3; ++xm)
        for (int ym = 0; ym < 6; ++ym)
          for (int bw : kBandWidths) {
            KernelFn k = kernel_for(xm, ym, bw, st);
            if (!k) continue;
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem_bytes(st) + (ym == kYMlp ? kMlpMaxBytes + 128 : 0));
            cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
          }
    for (int st = kMinStages; st <= kMaxStages; ++st)
    for (int i = 0; i < 5; ++i) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1u << i, 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = smem_bytes(st);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1u << i;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kernel_for(kXHalf, kYHalf, 64, st), &cfg) != cudaSuccess) n = 0;
      d.max_clusters[st - kMinStages][i] = n;
    }
    cudaGetLastError();
  });
  return &g_dev[dev];
}

struct Plan {
  int bw, bands, tiles, c, kc, stages;
  size_t bytes;   // workspace bytes (counters included)
};

// Grid of bands x kc clusters of c CTAs, in one of two regimes (measured on
// B200 across the 0.5B, 7B and 70B projection shapes; each rule picks the
// fastest plan or one within a few percent):
//   * Latency bound (each warp would stream fewer than 8 tiles at two CTAs
//     per SM; all decode projections up to 7B-class): a warp spends ~2.5
//     instructions per weight and lane on a tile and a cluster's reduction
//     costs a barrier, so the plan looks for many CTAs, all co-resident, none
//     idle.  Among band widths of 512, 256 and 128 columns and cluster sizes
//     up to 16 (clusters co-resident, at most half the warps without a tile)
//     it takes the CTA count closest to two per SM; on a tie, the larger
//     cluster, unless some of its warps would have no tile.
//   * Bandwidth bound: 512-column bands (narrower boxes cost DRAM efficiency)
//     and the largest co-resident cluster.  The workspace fix-up of kc > 1
//     costs a few microseconds of tail; only deep-K layers, where every warp
//     would stream 16 or more tiles, trade that tail for more warps (c = 8,
//     kc = 3 on 28672 x 8192).
static Plan make_plan(const DeviceInfo& d, int K, int N, int stages) {
  Plan pl{};
  pl.stages = stages;
  const int* max_clusters = d.max_clusters[stages - kMinStages];
  const int W8 = N / 8;
  pl.tiles = (K + kTileRows - 1) / kTileRows;
  const double tiles_per_warp = (double)W8 * pl.tiles / (64.0 * 2.0 * d.sms * kWarps);
  int kc = 1;
  if (tiles_per_warp < 8.0) {
    const double target = 2.0 * d.sms;
    double best_score = 1e30;
    int best_ctas = 0;
    pl.bw = kBandWidths[0];
    pl.c = 1;
    for (int bw : kBandWidths) {
      const int bands = (W8 + bw - 1) / bw;
      for (int i = 4; i >= 0; --i) {
        const int c = 1 << i;
        if (max_clusters[i] < bands || c * kWarps > 2 * pl.tiles) continue;
        const int ctas = bands * c;
        const double score = std::fabs(std::log((double)ctas / target));
        bool take = score < best_score - 1e-9;
        if (!take && ctas == best_ctas) {   // a tie: the larger cluster, if all its warps stream
          const bool full = c * kWarps <= pl.tiles, best_full = pl.c * kWarps <= pl.tiles;
          take = (full && !best_full) || (full == best_full && c > pl.c);
        }
        if (take) {
          best_score = score;
          best_ctas = ctas;
          pl.bw = bw;
          pl.c = c;
        }
      }
    }
    pl.bands = (W8 + pl.bw - 1) / pl.bw;
  } else {
    pl.bw = kBandWidths[0];
    pl.bands = (W8 + pl.bw - 1) / pl.bw;
    pl.c = 1;
    for (int i = 4; i >= 1; --i) {
      const int cand = 1 << i;
      if (max_clusters[i] >= pl.bands && cand * kWarps <= pl.tiles) {
        pl.c = cand;
        break;
      }
    }
    if (pl.tiles / (kWarps * pl.c) >= 16) {
      for (int cand_c : {8, 16}) {
        const int i = cand_c == 8 ? 3 : 4;
        for (int cand_kc = 3; cand_kc >= 2; --cand_kc)
          if (kc == 1 && max_clusters[i] >= pl.bands * cand_kc && pl.bands * cand_c * cand_kc <= 4 * d.sms) {
            pl.c = cand_c;
            kc = cand_kc;
          }
      }
    }
  }
  pl.kc = kc;
  pl.bytes = ANVILQ_WORKSPACE_COUNTER_BYTES +
             (pl.kc > 1 ? (size_t)pl.bands * pl.kc * pl.bw * 8 * sizeof(float) : 0);
  return pl;
}

// Ring depth: four stages give every warp a third more bytes in flight but fit
// three CTAs on an SM instead of four.  Measured on B200 (CUDA graphs of
// distinct-weight launches), four stages are 6-14 % faster wherever the plan
// keeps its CTA count (4096x11008, 4096x22016, 11008x4096, 8192x8192,
// 28672x8192, 4864x896, 896x1152) and equal elsewhere, but 30 % slower on
// 8192x28672, where 56 bands of 8-CTA clusters no longer fit co-resident and
// the plan halves its CTAs.  So: four stages unless that plan launches fewer CTAs.
static Plan choose_plan(const DeviceInfo& d, int K, int N) {
  const Plan p3 = make_plan(d, K, N, kMinStages);
  const Plan p4 = make_plan(d, K, N, kMaxStages);
  const long long c3 = (long long)p3.bands * p3.kc * p3.c, c4 = (long long)p4.bands * p4.kc * p4.c;
  return c4 >= c3 ? p4 : p3;
}

static Plan plan_from(const GemvPlan& g, int K, int N) {
  Plan pl{};
  pl.bw = g.band_cols / 8;
  pl.bands = (N / 8 + pl.bw - 1) / pl.bw;
  pl.tiles = (K + kTileRows - 1) / kTileRows;
  pl.c = g.cluster;
  pl.kc = g.kc;
  pl.stages = g.stages;
  pl.bytes = ANVILQ_WORKSPACE_COUNTER_BYTES +
             (pl.kc > 1 ? (size_t)pl.bands * pl.kc * pl.bw * 8 * sizeof(float) : 0);
  return pl;
}

}  // namespace tma_gemv

bool gemv_cluster_default_plan(int K, int N, GemvPlan* out) {
  using namespace tma_gemv;
  const DeviceInfo* d = device_info();
  if (!d || d->sms <= 0) return false;
  const Plan pl = choose_plan(*d, K, N);
  out->kernel = ANVILQ_GEMV_KERNEL_CLUSTER;
  out->band_cols = pl.bw * 8;
  out->cluster = pl.c;
  out->kc = pl.kc;
  out->warps = kWarps;
  out->stages = pl.stages;
  out->ctas = pl.bands * pl.kc * pl.c;
  return true;
}

int gemv_cluster_check_plan(int K, int N, GemvPlan* g) {
  using namespace tma_gemv;
  const DeviceInfo* d = device_info();
  if (!d || d->sms <= 0) return ANVILQ_ECUDA;
  const int bw = g->band_cols / 8;
  if (g->kernel != ANVILQ_GEMV_KERNEL_CLUSTER || bw * 8 != g->band_cols || (bw != 64 && bw != 32 && bw != 16))
    return ANVILQ_EINVAL;
  const int c = g->cluster;
  if (c < 1 || c > kMaxCluster || (c & (c - 1)) || g->kc < 1 || g->kc > 8 || g->warps != kWarps ||
      g->stages < kMinStages || g->stages > kMaxStages)
    return ANVILQ_EINVAL;
  int li = 0;
  while ((1 << li) < c) ++li;
  if (d->max_clusters[g->stages - kMinStages][li] < 1) return ANVILQ_ESHAPE;   // a cluster does not fit
  const long long bands = (N / 8 + bw - 1) / bw;
  if (g->kc > 1 && bands * c * (long long)sizeof(int) > ANVILQ_WORKSPACE_COUNTER_BYTES) return ANVILQ_ESHAPE;
  if (bands * g->kc * c > (1ll << 31) - 1) return ANVILQ_ESHAPE;
  g->ctas = (int)(bands * g->kc * c);
  return ANVILQ_OK;
}

size_t gemv_cluster_workspace_bytes(int K, int N, const GemvPlan& g) {
  return tma_gemv::plan_from(g, K, N).bytes;
}

bool gemv_tma_supported(const void* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                        int K, int N, int G) {
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  return K % 16 == 0 && G % 16 == 0 && N % 32 == 0 && a16(x) && a16(qweight) && a16(qzeros) && a16(scales) &&
         tma_gemv::encode_fn() != nullptr;
}

size_t gemv_tma_workspace_bytes(int K, int N) {
  const tma_gemv::DeviceInfo* d = tma_gemv::device_info();
  if (!d || d->sms <= 0) return 0;
  return tma_gemv::choose_plan(*d, K, N).bytes;
}

int launch_gemv_tma(const GemvIo& io, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                    const uint16_t* bias, int K, int N, int G, void* workspace, size_t workspace_bytes, int* dev_err,
                    cudaStream_t stream, bool overlap_prior, const GemvPlan* plan) {
  using namespace tma_gemv;
  const DeviceInfo* d = device_info();
  auto encode = encode_fn();
  if (!d || d->sms <= 0 || !encode) return ANVILQ_ECUDA;
  if (io.xmode < 0 || io.xmode > 2 || io.ymode < 0 || io.ymode > 5) return ANVILQ_EINVAL;
  if (io.ymode == kYAct && (io.xmode == kXSiluMul || bias || N % 64)) return ANVILQ_EINVAL;
  if (io.ymode == kYPeer && io.xmode != kXHalf) return ANVILQ_EINVAL;
  if (io.ymode == kYMlp && (io.xmode != kXRmsNorm || bias || !io.yr)) return ANVILQ_EINVAL;
  if (plan && (io.xmode != kXHalf || io.ymode != kYHalf)) return ANVILQ_EINVAL;
  Plan pl = plan ? plan_from(*plan, K, N) : choose_plan(*d, K, N);
  const int* max_clusters = d->max_clusters[pl.stages - kMinStages];
  if (io.ymode == kYPeer) {
    if (io.world < 1 || io.world > kMaxPeers || io.tp_rank < 0 || io.tp_rank >= io.world || !io.epoch)
      return ANVILQ_EINVAL;
    if (pl.kc > 1) pl.kc = 1;   // one completion ticket per launch: no workspace fix-up
  }
  if (io.ymode == kYRope) {
    // the epilogue needs whole heads in a band and one cluster per band; the
    // usual plan of every decode QKV shape qualifies, anything else falls back
    // to 512-column bands
    if (io.D < 2 || io.D % 2 || io.D / 2 > kMaxRopePairs || (kBandWidths[0] * 8) % io.D) return ANVILQ_ESHAPE;
    if (pl.kc > 1 || (pl.bw * 8) % io.D) {
      pl.bw = kBandWidths[0];
      pl.bands = (N / 8 + pl.bw - 1) / pl.bw;
      pl.c = 1;
      for (int i = 4; i >= 1; --i)
        if (max_clusters[i] >= pl.bands && (1 << i) * kWarps <= pl.tiles) {
          pl.c = 1 << i;
          break;
        }
      pl.kc = 1;
    }
  }
  if (io.ymode == kYAct) pl.kc = 1;   // the owners' (gate, up) sums are final after the cluster sum
  int dn_rows = 0, dn_groups = 0, mlp_off = 0, mlp_bytes = 0;
  if (io.ymode == kYMlp) {
    // one cluster per band (the owners' rows are final after the cluster sum),
    // and every owner's share of the H outputs a whole number of 8-column words
    const int H = io.dn_H;
    if (H < 8 || H % 32 || N % 64 || !io.dn_qweight || !io.dn_qzeros || !io.dn_scales) return ANVILQ_ESHAPE;
    auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    if (!a16(io.dn_qweight) || !a16(io.dn_qzeros) || !a16(io.dn_scales) || !a16(io.yr)) return ANVILQ_EALIGN;
    pl.kc = 1;
    while (pl.c > 1 && H % (8 * pl.c)) pl.c /= 2;
    // the 3-stage ring: with the down region a CTA stays within a third of an
    // SM's shared memory, so the plan's clusters remain co-resident in one wave
    pl.stages = kMinStages;
    dn_rows = pl.bw * 8 / pl.c / 2;
    // groups an owner's rows can touch: owners start at multiples of dn_rows
    dn_groups = G % dn_rows == 0 ? 1 : (dn_rows + G - 1) / G + 1;
    mlp_bytes = MlpSmem(H, dn_rows, dn_groups, pl.c).bytes;
    if (mlp_bytes > kMlpMaxBytes) return ANVILQ_ESHAPE;
    mlp_off = (smem_bytes(pl.stages) + 127) / 128 * 128;
    if (!workspace || workspace_bytes < ANVILQ_WORKSPACE_COUNTER_BYTES + (size_t)pl.bands * H * sizeof(float))
      return ANVILQ_EWORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) return ANVILQ_EALIGN;
  }
  if (pl.kc > 1) {
    if (!workspace || workspace_bytes < pl.bytes) return ANVILQ_EWORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) return ANVILQ_EALIGN;
    if ((size_t)pl.bands * pl.c * sizeof(int) > ANVILQ_WORKSPACE_COUNTER_BYTES) return ANVILQ_ESHAPE;
  }
  if (io.ymode == kYPeer) {   // the launch's completion ticket lives in the counter region
    if (!workspace || workspace_bytes < ANVILQ_WORKSPACE_COUNTER_BYTES) return ANVILQ_EWORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) return ANVILQ_EALIGN;
  }
  const int W8 = N / 8;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)W8, (cuuint64_t)K};
  const cuuint64_t strides[1] = {(cuuint64_t)W8 * 4};
  const cuuint32_t box[2] = {(cuuint32_t)pl.bw, (cuuint32_t)kTileRows};
  const cuuint32_t estr[2] = {1, 1};
  if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(qweight), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return ANVILQ_EALIGN;
  Params p = {};
  p.x = reinterpret_cast<const __half*>(io.x);
  p.xr = io.xr;
  p.gamma = reinterpret_cast<const __half*>(io.gamma);
  p.eps = io.eps;
  p.qzeros = qzeros;
  p.scales = reinterpret_cast<const __half*>(scales);
  p.bias = reinterpret_cast<const __half*>(bias);
  p.y = reinterpret_cast<__half*>(io.y);
  p.yr = io.yr;
  p.tickets = reinterpret_cast<int*>(workspace);
  p.partials = workspace ? reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) +
                                                    ANVILQ_WORKSPACE_COUNTER_BYTES)
                         : nullptr;
  p.dev_err = dev_err;
  p.K = K; p.N = N; p.W8 = W8; p.G = G;
  p.rope_pos = io.rope_pos;
  p.q_out = reinterpret_cast<__half*>(io.q_out);
  p.k_cache = reinterpret_cast<__half*>(io.k_cache);
  p.v_cache = reinterpret_cast<__half*>(io.v_cache);
  p.seqlen = io.seqlen;
  p.Hq = io.Hq; p.Hkv = io.Hkv; p.D = io.D; p.Tmax = io.Tmax;
  for (int r = 0; r < kMaxPeers; ++r) {
    p.peer_y[r] = r < io.world ? reinterpret_cast<__half*>(io.peer_y[r]) : nullptr;
    p.peer_flags[r] = r < io.world ? io.peer_flags[r] : nullptr;
  }
  p.epoch = io.epoch;
  p.world = io.world;
  p.tp_rank = io.tp_rank;
  p.col_base = io.col_base;
  for (int i = 0; i < kMaxRopePairs; ++i)
    p.rope_inv[i] = io.ymode == kYRope && i < io.D / 2 ? std::pow((double)io.theta, -2.0 * i / io.D) : 0.0;
  p.cluster = pl.c;
  p.kc = pl.kc;
  p.tiles = pl.tiles;
  p.dn_qweight = io.dn_qweight;
  p.dn_qzeros = io.dn_qzeros;
  p.dn_scales = reinterpret_cast<const __half*>(io.dn_scales);
  p.dn_H = io.dn_H;
  p.dn_rows = dn_rows;
  p.dn_groups = dn_groups;
  p.bands = pl.bands;
  p.mlp_off = mlp_off;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.bands * pl.kc * pl.c, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = io.ymode == kYMlp ? mlp_off + mlp_bytes : smem_bytes(pl.stages);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = pl.c;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap_prior ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, kernel_for(io.xmode, io.ymode, pl.bw, pl.stages), map, p) != cudaSuccess) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  return ANVILQ_OK;
}

}  // namespace anvilq
