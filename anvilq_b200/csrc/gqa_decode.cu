// gqa_decode.cu -- GQA decode attention over an fp16 KV cache (flash-decoding,
// split-KV), with its C-ABI entry points.
//
// Reference semantics: attention(q, keys, values) of
// anvil-q1-fp/tests/fp64_reference.py:164-170 and the FP32 loop of
// anvil-q1/tests/official_weights.py:471-486: for every query head,
// softmax(q . k_t * scale) over positions t < seqlen, weighted sum of v_t, with
// kv head = query head / (Hq / Hkv) (contiguous groups).  The online-softmax
// form (running max, running sum, rescale by exp(m_old - m_new)) follows the
// tiled contract of anvil-q1-ht3/design/SPEC.md:545-556.
//
// Design (B200, latency first: a decode step calls this once per layer with
// a few kv heads, so the critical path, not bandwidth, sets the time):
//   * Grid (CTAs per pair, Hkv, B); a pair = (sequence, kv head).  The CTAs of
//     a pair split its live tiles into contiguous ranges; up to 8 of them form
//     one thread-block cluster and merge their partial softmax states through
//     distributed shared memory (one cluster barrier, one DSMEM round trip),
//     so a short context finishes with no global-memory handshake at all.
//     Longer contexts give a pair several clusters; each writes one merged
//     partial, and the cluster CTA that arrives last at the pair's ticket
//     merges those partials in cluster order (deterministic, no spin-wait),
//     loading every partial of its elements in one L2 round trip.
//   * The query heads of a GQA group (<= 8) share every K/V row, so each row is
//     read from HBM once per group.  A 16-token K tile and V tile arrive as
//     TMA boxes of a 4-D tensor map over the cache (D, Hkv, Tmax, B): one box
//     per 64 dims of each, 128-byte swizzled, into a per-warp ring guarded by
//     mbarriers; each of the 8 warps streams its own tiles, so no inter-warp
//     handshake sits on the critical path.  The fragment loads below undo the
//     swizzle (16-byte chunk c of row r sits at c ^ (r % 8)).  Cache rows past
//     the live length inside the last tile are not part of the sequence: their
//     K scores are masked and their V rows zeroed in shared memory, so whatever
//     they hold cannot reach the output.
//   * S = Q K^T on the tensor cores (mma.m16n8k16, fp16 in, fp32 accumulate):
//     the group's query heads are the 16-row A operand (rows >= group size are
//     zero), 8 tokens per n-tile.  The S accumulator layout is exactly the B
//     operand layout of O^T += V^T P^T, so P never leaves registers; V^T comes
//     from ldmatrix.trans.
//   * Online softmax in the log2 domain, per warp; the 8 warps are merged in
//     shared memory, then the cluster, then (long contexts) the clusters.
//   * Every mbarrier wait is bounded (about one second of %globaltimer); on
//     expiry the kernel sets ANVILQ_DEV_ERR_TIMEOUT, stops using its tiles and
//     waits, again bounded, for its own copies before it exits.  The cluster
//     barriers are reached by every thread of every CTA on every path (there is
//     no return before them), and a cluster's CTAs are co-scheduled by the
//     hardware, so they always complete.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "../../include/anvilq.h"
#include "internal.h"

namespace anvilq {
namespace attn {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 16;          // tokens per tile
constexpr int kMaxGroup = 8;       // query heads per kv head handled by one CTA
constexpr int kMaxCluster = 8;     // CTAs of a pair merged in one cluster (portable size)
constexpr int kMaxClusters = 16;   // clusters per pair
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

struct Params {
  const __half* q;      // [B][Hq][D]
  const __half* k;      // [B][Tmax][Hkv][D]
  const __half* v;
  const int* seqlens;   // [B]
  __half* out;          // [B][Hq][D]
  float* partials;      // [B][Hkv][clusters][group][D + 4]: o[D], max, sum, pad
  int* tickets;         // [B][Hkv]
  int* dev_err;
  int Hq, Hkv, Tmax, group;
  int cluster, clusters;   // CTAs per cluster, clusters per pair (gridDim.x = their product)
  float scale_log2;        // softmax scale * log2(e)
  // INT8 cache only: fp32 payloads of escaped (token, kv head) rows, [B][Tmax][Hkv][D] (may be NULL)
  const float* k_escape;
  const float* v_escape;
  // paged fp16 cache only (else NULL): logical page j of sequence b lives in
  // physical page page_table[b][j] (bit 31 valid, bits 30:0 the page) of a
  // pool [num_pages][page_tokens][Hkv][D]; the tensor maps then cover the
  // pool as one sequence of num_pages * page_tokens rows
  const uint32_t* page_table;   // [B][max_pages]
  int page_tokens, max_pages, num_pages;
  // optional [B][Hq]: each head's log-sum-exp of its scaled scores in the log2
  // domain, log2(sum_t 2^(q.k_t scale log2(e))) (-inf for an empty sequence),
  // so that a caller can merge this softmax with scores over further keys
  float* lse;
};

constexpr uint32_t kEscapeMarker = 0x7FC00000u;   // INT8-cache metadata of an escaped row

// Q8: the cache holds INT8 codes with per-(token, kv head) scales (kv_int8.cu);
// a stage then carries the K and V code tiles and their 16 metadata words, and
// each warp stages them into fp16 tiles of the same swizzled layout for the MMAs.
template <int D, bool Q8 = false>
struct Layout {
  static constexpr int kStages = 2;                            // ring depth per warp
  static constexpr int kHalves = D / 64;                       // 128-byte boxes per row
  static constexpr int kBoxBytes = kTile * 128;                // 16 rows x 64 dims, swizzled
  static constexpr int kTileBytes = kHalves * kBoxBytes;       // fp16 tile: [half][row][128 B]
  static constexpr int kCodeBytes = kTile * D;                 // INT8 tile: [row][D]
  static constexpr int kMetaBytes = kTile * 4;                 // 16 metadata words (one TMA box)
  static constexpr int kMetaSlot = 128;                        // a TMA destination is 128-byte aligned
  static constexpr int kStageBytes = Q8 ? 2 * kCodeBytes + 2 * kMetaSlot : 2 * kTileBytes;
  static constexpr int kStageTx = Q8 ? 2 * kCodeBytes + 2 * kMetaBytes : 2 * kTileBytes;   // bytes landed
  static constexpr int kStagingOffset = kStages * kStageBytes; // Q8: fp16 K tile + V tile, per warp
  static constexpr int kWarpBytes = kStagingOffset + (Q8 ? 2 * kTileBytes : 0);
  static constexpr int kRingBytes = kWarps * kWarpBytes;
  static constexpr int kRow = D + 2;                           // one head's state: o[D], max, sum
  static constexpr int kStateBytes = kMaxGroup * kRow * 4;     // a warp's or a CTA's state
  static constexpr int kBarOffset = kRingBytes;                // kWarps * kStages mbarriers
  static constexpr int kAuxOffset = kBarOffset + kWarps * kStages * 8;
  static constexpr int kAuxBytes = (kMaxGroup * kWarps + 2 * kMaxGroup) * 4;   // warp weights, head max/sum
  static constexpr int kSlotOffset = kAuxOffset + kAuxBytes;   // rank 0: one state per CTA of the cluster
  static constexpr int kSlotBytes = kMaxCluster * kStateBytes;
  static constexpr int kTotal = kSlotOffset + kSlotBytes + 1024;   // + slack to align the ring to 1024
  static_assert(kBoxBytes % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
  static_assert(kStageBytes % 128 == 0 && kWarpBytes % 128 == 0 && kCodeBytes % 128 == 0,
                "stages, warp areas and every TMA destination stay 128-byte aligned");
  static_assert(kWarpBytes >= kStateBytes, "a warp's state fits its idle ring");
  static_assert(kTotal <= 227 * 1024, "fits one SM's shared memory");
  // byte offset of the 16-byte chunk c (of 8 dims) of row r inside a tile
  __device__ static __forceinline__ int chunk(int r, int c) {
    return (c >> 3) * kBoxBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4);
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
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
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
// Bounded wait: true when the phase completed, false after ~kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 63u && globaltimer() - t0 > kWaitLimitNs) return false;
  }
}
__device__ __forceinline__ void tma_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                       uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// cluster barrier halves: arrive.release orders this thread's earlier
// shared-memory writes (remote ones included) before the wait.acquire of the
// others; a thread may exit after arriving
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
// address of the same shared-memory variable in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_dsmem(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col)
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
// four INT8 codes (ascending bytes) as four fp16 values (exact: |code| <= 127)
__device__ __forceinline__ uint2 codes_to_half4(uint32_t w) {
  return make_uint2(pack_half2((float)(int8_t)(w & 0xFFu), (float)(int8_t)((w >> 8) & 0xFFu)),
                    pack_half2((float)(int8_t)((w >> 16) & 0xFFu), (float)(int8_t)(w >> 24)));
}
// a row's scale from its metadata word (1 for an escaped row, whose payload is the value itself)
__device__ __forceinline__ float meta_scale(uint32_t m) { return m == kEscapeMarker ? 1.0f : __uint_as_float(m); }

// mk / mv: the K / V cache (fp16, or Q8: INT8 codes); mkm / mvm (Q8 only): their
// metadata [B][Hkv][Tmax] uint32.
template <int D, bool Q8>
__global__ void __launch_bounds__(kThreads, D == 64 ? 2 : 1)
    gqa_decode_kernel(const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv,
                      const __grid_constant__ CUtensorMap mkm, const __grid_constant__ CUtensorMap mvm,
                      const Params p) {
  using L = Layout<D, Q8>;
  constexpr int KS = D / 16;   // k-steps of QK, m-tiles of PV
  constexpr int kStages = L::kStages;
  constexpr int R = L::kRow;
  constexpr int RG = D + 4;    // a head's row in the global partials (16-byte multiple)
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ int s_flag;
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int C = p.cluster, rank = split % C, cl = split / C;
  // launched with programmatic dependent launch (ANVILQ_GEMM_OVERLAP_PRIOR) the
  // CTAs may be resident before the previous kernel -- the one that wrote q,
  // the new cache row and the length -- completes: wait for it before reading
  // any of them (a no-op otherwise)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int seqlen = p.seqlens[b];
  const bool bad_len = seqlen < 1 || seqlen > p.Tmax;
  const int ntiles = bad_len ? 0 : (seqlen + kTile - 1) / kTile;
  // the live sequence is spread over all CTAs of the pair (the grid is sized for Tmax)
  const int per_split = (ntiles + gridDim.x - 1) / gridDim.x;
  const int tb = split * per_split;
  const int te = min(ntiles, tb + per_split);
  // warp-local tiles: tb + warp + kWarps * j
  const int my_tiles = te > tb + warp ? (te - tb - warp + kWarps - 1) / kWarps : 0;

  unsigned char* ring = smem + warp * L::kWarpBytes;
  const uint32_t bar0 = smem_u32(smem + L::kBarOffset + warp * kStages * 8);
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(bar0 + 8 * s, 1);
    if (warp == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&mk) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&mv) : "memory");
      if (Q8) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&mkm) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&mvm) : "memory");
      }
    }
  }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  // a kernel launched after this one with programmatic dependent launch (the
  // next projection) may start now and stream its weights; it still waits
  // for this grid to complete before it reads the attention output
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __syncwarp();

  auto issue = [&](int j) {   // tile j of this warp into stage j % kStages
    const int st = j % kStages;
    const uint32_t bar = bar0 + 8 * st;
    // the stage may hold zeros written through the generic proxy (tail rows)
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      const int t0 = (tb + warp + kWarps * j) * kTile;
      const uint32_t kd = smem_u32(ring + st * L::kStageBytes);
      int row = t0, seq = b;   // the tile's coordinates in the tensor maps
      if (!Q8 && p.page_table) {
        // a 16-token tile never straddles a page (page_tokens % 16 == 0); an
        // absent or out-of-range page is an error, and the copy then reads
        // physical page 0 so that it stays inside the pool
        const uint32_t e = p.page_table[(size_t)b * p.max_pages + t0 / p.page_tokens];
        uint32_t page = e & 0x7FFFFFFFu;
        if (!(e >> 31) || page >= (uint32_t)p.num_pages) {
          atomicOr(p.dev_err, ANVILQ_DEV_ERR_PAGE);
          page = 0;
        }
        row = (int)page * p.page_tokens + t0 % p.page_tokens;
        seq = 0;
      }
      if (Q8) {
        mbar_expect_tx(bar, L::kStageTx);
        tma_4d(kd, &mk, 0, h, t0, b, bar);
        tma_4d(kd + L::kCodeBytes, &mv, 0, h, t0, b, bar);
        tma_3d(kd + 2 * L::kCodeBytes, &mkm, t0, h, b, bar);
        tma_3d(kd + 2 * L::kCodeBytes + L::kMetaSlot, &mvm, t0, h, b, bar);
      } else {
        mbar_expect_tx(bar, 2 * kTile * D * 2);
#pragma unroll
        for (int hf = 0; hf < L::kHalves; ++hf) {
          tma_4d(kd + hf * L::kBoxBytes, &mk, 64 * hf, h, row, seq, bar);
          tma_4d(kd + L::kTileBytes + hf * L::kBoxBytes, &mv, 64 * hf, h, row, seq, bar);
        }
      }
    }
    __syncwarp();
  };

  int issued = 0;
  for (; issued < min(kStages - 1, my_tiles); ++issued) issue(issued);

  // Q as the A operand: row g = query head of the group (zero beyond the group).
  const int g = lane / 4;
  uint32_t qa[KS][2];
  {
    const bool valid = g < p.group;
    const __half* qrow = p.q + ((size_t)b * p.Hq + (size_t)h * p.group + (valid ? g : 0)) * D;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qa[ks][0] = valid ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 2 * (lane % 4)) : 0u;
      qa[ks][1] = valid ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 8 + 2 * (lane % 4)) : 0u;
    }
  }

  float o[KS][4];
#pragma unroll
  for (int mt = 0; mt < KS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;
  bool ok = true;
  // Q8: o holds the output divided by F, the largest V scale of the last tile
  // (the V scales are folded into P, normalised per tile to stay clear of fp16 underflow)
  float F = 1.0f;

  for (int j = 0; j < my_tiles && ok; ++j) {
    if (issued < my_tiles) issue(issued++);
    const int st = j % kStages;
    // every lane polls; the warp proceeds only if all lanes saw the tile land
    const bool landed = mbar_wait_bounded(bar0 + 8 * st, (j / kStages) & 1);
    if (!__all_sync(0xffffffffu, landed)) {
      ok = false;
      break;
    }
    const int t0 = (tb + warp + kWarps * j) * kTile;
    const unsigned char* kt = ring + st * L::kStageBytes;
    const unsigned char* vt = kt + L::kTileBytes;
    const uint32_t* km = reinterpret_cast<const uint32_t*>(kt + 2 * L::kCodeBytes);   // Q8 metadata
    const uint32_t* vm = reinterpret_cast<const uint32_t*>(kt + 2 * L::kCodeBytes + L::kMetaSlot);
    if (Q8) {
      // codes -> fp16 tiles in the swizzled layout; escaped rows from their fp32
      // payload; rows past the sequence zero
      unsigned char* sk = ring + L::kStagingOffset;
      unsigned char* sv = sk + L::kTileBytes;
      for (int e = lane; e < kTile * D / 4; e += 32) {
        const int r = e / (D / 4), d = 4 * (e % (D / 4));
        const int tok = t0 + r;
        uint2 hk = make_uint2(0, 0), hv = make_uint2(0, 0);
        if (tok < seqlen) {
          const size_t esc_at = (((size_t)b * p.Tmax + tok) * p.Hkv + h) * D + d;
          if (km[r] != kEscapeMarker) {
            hk = codes_to_half4(*reinterpret_cast<const uint32_t*>(kt + r * D + d));
          } else if (p.k_escape) {
            const float4 f = *reinterpret_cast<const float4*>(p.k_escape + esc_at);
            hk = make_uint2(pack_half2(f.x, f.y), pack_half2(f.z, f.w));
          } else if (d == 0) {
            atomicOr(p.dev_err, ANVILQ_DEV_ERR_NONFINITE);
          }
          if (vm[r] != kEscapeMarker) {
            hv = codes_to_half4(*reinterpret_cast<const uint32_t*>(kt + L::kCodeBytes + r * D + d));
          } else if (p.v_escape) {
            const float4 f = *reinterpret_cast<const float4*>(p.v_escape + esc_at);
            hv = make_uint2(pack_half2(f.x, f.y), pack_half2(f.z, f.w));
          } else if (d == 0) {
            atomicOr(p.dev_err, ANVILQ_DEV_ERR_NONFINITE);
          }
        }
        *reinterpret_cast<uint2*>(sk + L::chunk(r, d >> 3) + (d & 7) * 2) = hk;
        *reinterpret_cast<uint2*>(sv + L::chunk(r, d >> 3) + (d & 7) * 2) = hv;
      }
      __syncwarp();
      kt = sk;
      vt = sv;
    } else if (t0 + kTile > seqlen) {
      // rows past the sequence: zero their V (scores are masked below)
      unsigned char* vz = ring + st * L::kStageBytes + L::kTileBytes;
      for (int e = lane; e < kTile * L::kHalves * 8; e += 32) {
        const int r = e / (L::kHalves * 8), c = e % (L::kHalves * 8);
        if (t0 + r >= seqlen) *reinterpret_cast<uint4*>(vz + L::chunk(r, c)) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }

    // S = Q K^T for tokens t0..t0+15 (two n-tiles of 8)
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < KS; ks += 2) {
        const int mj = lane / 8, r = lane % 8;
        const uint32_t addr = smem_u32(kt + L::chunk(nt * 8 + r, 2 * (ks + mj / 2) + (mj % 2)));
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(addr, b0, b1, b2, b3);
        mma16816(s[nt], qa[ks][0], 0u, qa[ks][1], 0u, b0, b1);
        mma16816(s[nt], qa[ks + 1][0], 0u, qa[ks + 1][1], 0u, b2, b3);
      }
    }
    // online softmax on rows g (c0, c1); rows g + 8 are padding
    float x[4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tok = t0 + nt * 8 + 2 * (lane % 4) + e;
        const float ks = Q8 && tok < seqlen ? meta_scale(km[tok - t0]) : 1.0f;   // Q8: code scale of K
        x[nt * 2 + e] = tok < seqlen ? s[nt][e] * ks * p.scale_log2 : -INFINITY;
      }
    float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);           // finite: every tile holds a valid token
    const float alpha = exp2f(m_run - m_new);
    float pr[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pr[e] = exp2f(x[e] - m_new);
    l_run = l_run * alpha + (pr[0] + pr[1]) + (pr[2] + pr[3]);
    m_run = m_new;
    float rescale = 1.0f;   // Q8: F_old / F_new on top of the softmax rescale
    if (Q8) {
      // P times each token's V scale over the tile's largest one
      float vs = lane < kTile && t0 + lane < seqlen ? meta_scale(vm[lane]) : 0.0f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) vs = fmaxf(vs, __shfl_xor_sync(0xffffffffu, vs, o));
      const float inv = 1.0f / vs;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = (e >> 1) * 8 + 2 * (lane % 4) + (e & 1);
        pr[e] = t0 + r < seqlen ? pr[e] * (meta_scale(vm[r]) * inv) : 0.0f;
      }
      rescale = F * inv;
      F = vs;
    }
    const uint32_t pb0 = pack_half2(pr[0], pr[1]);   // tokens 2(l%4), +1   (k rows 0..7)
    const uint32_t pb1 = pack_half2(pr[2], pr[3]);   // tokens 8 + 2(l%4)   (k rows 8..15)
    const float alpha_a = __shfl_sync(0xffffffffu, alpha, 8 * (lane % 4)) * rescale;
    const float alpha_b = __shfl_sync(0xffffffffu, alpha, 8 * (lane % 4) + 4) * rescale;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      o[mt][0] *= alpha_a;
      o[mt][1] *= alpha_b;
      o[mt][2] *= alpha_a;
      o[mt][3] *= alpha_b;
      const int mj = lane / 8, r = lane % 8;
      const uint32_t addr = smem_u32(vt + L::chunk(r + 8 * (mj / 2), 2 * mt + (mj % 2)));
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4_trans(addr, a0, a1, a2, a3);
      mma16816(o[mt], a0, a1, a2, a3, pb0, pb1);
    }
    __syncwarp();
  }
  if (!ok) {
    atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
    // wait, bounded, for every copy this warp still has in flight
    for (int j = max(0, issued - kStages); j < issued; ++j) mbar_wait_bounded(bar0 + 8 * (j % kStages), (j / kStages) & 1);
  }
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);

  // ---- merge the warps: each warp's state goes to its own ring, idle now ----
  float* mine = reinterpret_cast<float*>(ring);   // [head][R]
  if (!ok) {
    m_run = -INFINITY;
    l_run = 0.0f;
  }
  if (!Q8) F = 1.0f;
#pragma unroll
  for (int mt = 0; mt < KS; ++mt) {
    const int d = 16 * mt + lane / 4, hh = 2 * (lane % 4);
    mine[hh * R + d] = ok ? o[mt][0] * F : 0.0f;
    mine[(hh + 1) * R + d] = ok ? o[mt][1] * F : 0.0f;
    mine[hh * R + d + 8] = ok ? o[mt][2] * F : 0.0f;
    mine[(hh + 1) * R + d + 8] = ok ? o[mt][3] * F : 0.0f;
  }
  if (lane % 4 == 0) {
    mine[g * R + D] = m_run;
    mine[g * R + D + 1] = l_run;
  }
  __syncthreads();
  if (bad_len && threadIdx.x == 0) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SEQLEN);

  const int G = p.group;
  const int pair = b * p.Hkv + h;
  const int S2 = p.clusters;
  float* fw = reinterpret_cast<float*>(smem + L::kAuxOffset);   // [head][warp] weights
  float* hstat = fw + kMaxGroup * kWarps;                        // [head]: max, sum
  // weights of the warps per head: lanes (head, warp) of warps 0-1, tree sums
  // over the 8 lanes of a head in a fixed order
  if (threadIdx.x < kMaxGroup * kWarps) {
    const int hh = threadIdx.x / kWarps, w = threadIdx.x % kWarps;
    const float* st = reinterpret_cast<const float*>(smem + w * L::kWarpBytes) + hh * R;
    const float mw = hh < G ? st[D] : -INFINITY;
    const float lw = hh < G ? st[D + 1] : 0.0f;
    float M = mw;
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 1));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 2));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 4));
    const float f = M == -INFINITY ? 0.0f : exp2f(mw - M);
    float ls = f * lw;
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    ls += __shfl_xor_sync(0xffffffffu, ls, 4);
    fw[hh * kWarps + w] = f;
    if (w == 0) {
      hstat[2 * hh] = M;
      hstat[2 * hh + 1] = ls;
    }
  }
  __syncthreads();

  // The pair's merged state of element (hh, d): with one cluster it is the
  // output, otherwise this cluster's partial.
  auto finish = [&](int hh, int d, float M, float lsum, float acc) {
    if (S2 == 1) {
      const float out = lsum > 0.0f ? acc / lsum : 0.0f;
      p.out[((size_t)b * p.Hq + (size_t)h * G + hh) * D + d] = __float2half_rn(out);
      if (p.lse && d == 0) p.lse[(size_t)b * p.Hq + (size_t)h * G + hh] = lsum > 0.0f ? M + log2f(lsum) : -INFINITY;
    } else {
      float* row = p.partials + (((size_t)pair * S2 + cl) * G + hh) * RG;
      __stcg(row + d, acc);
      if (d == 0) {
        __stcg(row + D, M);
        __stcg(row + D + 1, lsum);
      }
    }
  };
  // the CTA's state; with a cluster it goes to slot `rank` of the cluster's rank 0
  const uint32_t slot0 = smem_u32(smem + L::kSlotOffset);
  const uint32_t my_slot = C > 1 ? dsmem_addr(slot0 + rank * L::kStateBytes, 0) : 0u;
  for (int e = threadIdx.x; e < G * D; e += kThreads) {
    const int hh = e / D, d = e % D;
    float acc = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w)
      acc += fw[hh * kWarps + w] * reinterpret_cast<const float*>(smem + w * L::kWarpBytes)[hh * R + d];
    const float M = hstat[2 * hh], lsum = hstat[2 * hh + 1];
    if (C == 1) {
      finish(hh, d, M, lsum, acc);
    } else {
      st_dsmem(my_slot + (hh * R + d) * 4, acc);
      if (d == 0) {
        st_dsmem(my_slot + (hh * R + D) * 4, M);
        st_dsmem(my_slot + (hh * R + D + 1) * 4, lsum);
      }
    }
  }

  // ---- merge the cluster's CTAs on rank 0, in rank order ----
  if (C > 1) {
    cluster_arrive();
    if (rank != 0) return;   // nothing reads this CTA's shared memory
    cluster_wait();
    const float* slots = reinterpret_cast<const float*>(smem + L::kSlotOffset);
    for (int e = threadIdx.x; e < G * D; e += kThreads) {
      const int hh = e / D, d = e % D;
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < kMaxCluster; ++r)
        if (r < C) M = fmaxf(M, slots[(r * kMaxGroup + hh) * R + D]);
      float acc = 0.0f, lsum = 0.0f;
      if (M != -INFINITY) {
#pragma unroll
        for (int r = 0; r < kMaxCluster; ++r) {
          if (r < C) {
            const float* row = slots + (r * kMaxGroup + hh) * R;
            const float f = exp2f(row[D] - M);
            lsum += f * row[D + 1];
            acc += f * row[d];
          }
        }
      }
      finish(hh, d, M, lsum, acc);
    }
  }
  if (S2 == 1) return;

  // ---- merge the pair's clusters: the last rank 0 to arrive, in cluster order ----
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(p.tickets + pair, 1);
    const bool last = ticket == S2 - 1;   // one arrival per cluster (its rank 0)
    if (last) p.tickets[pair] = 0;
    s_flag = last;
  }
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  const float* parts = p.partials + (size_t)pair * S2 * G * RG;
  // the clusters' (max, sum) of every head, loaded in one parallel pass into
  // the slot area (free again: the cluster merge is behind the barriers above)
  float* gstat = reinterpret_cast<float*>(smem + L::kSlotOffset);   // [cluster][head][2]
  for (int i = threadIdx.x; i < S2 * G; i += kThreads) {
    const float* row = parts + (size_t)i * RG;
    gstat[2 * i] = __ldcg(row + D);
    gstat[2 * i + 1] = __ldcg(row + D + 1);
  }
  __syncthreads();
  // two consecutive dims of one head per thread; all their partials are loaded
  // before any is used (one L2 round trip), summed in cluster order
  for (int e = threadIdx.x; e < G * (D / 2); e += kThreads) {
    const int hh = e / (D / 2), d2 = 2 * (e % (D / 2));
    const float* col = parts + (size_t)hh * RG + d2;
    float2 oc[kMaxClusters];
#pragma unroll
    for (int c = 0; c < kMaxClusters; ++c)
      if (c < S2) oc[c] = __ldcg(reinterpret_cast<const float2*>(col + (size_t)c * G * RG));
    float M = -INFINITY;
    for (int c = 0; c < S2; ++c) M = fmaxf(M, gstat[2 * (c * G + hh)]);
    float lsum = 0.0f;
    float2 acc = make_float2(0.0f, 0.0f);
    if (M != -INFINITY) {
#pragma unroll
      for (int c = 0; c < kMaxClusters; ++c) {
        if (c < S2) {
          const float f = exp2f(gstat[2 * (c * G + hh)] - M);
          lsum += f * gstat[2 * (c * G + hh) + 1];
          acc.x += f * oc[c].x;
          acc.y += f * oc[c].y;
        }
      }
    }
    const float inv = lsum > 0.0f ? 1.0f / lsum : 0.0f;
    *reinterpret_cast<__half2*>(p.out + ((size_t)b * p.Hq + (size_t)h * G + hh) * D + d2) =
        __floats2half2_rn(acc.x * inv, acc.y * inv);
    if (p.lse && d2 == 0) p.lse[(size_t)b * p.Hq + (size_t)h * G + hh] = lsum > 0.0f ? M + log2f(lsum) : -INFINITY;
  }
}

// ---------------------------------------------------------------------------
struct Plan {
  int cluster, clusters;   // CTAs per cluster, clusters per pair
  size_t partial_bytes, bytes;
};

constexpr int kMaxDevices = 64;
struct DeviceInfo {
  int sms;
  int max_clusters[2];   // co-resident clusters of kMaxCluster CTAs, head_dim 64 / 128
};
static DeviceInfo g_info[kMaxDevices];
static std::once_flag g_once[kMaxDevices];

template <int D>
static int max_active_clusters() {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kMaxCluster * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Layout<D, false>::kTotal;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kMaxCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gqa_decode_kernel<D, false>, &cfg) != cudaSuccess) n = 0;
  return n;
}

static const DeviceInfo* device_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(g_once[dev], [dev] {
    DeviceInfo& in = g_info[dev];
    cudaDeviceGetAttribute(&in.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(gqa_decode_kernel<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Layout<64, false>::kTotal);
    cudaFuncSetAttribute(gqa_decode_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Layout<128, false>::kTotal);
    cudaFuncSetAttribute(gqa_decode_kernel<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Layout<64, true>::kTotal);
    cudaFuncSetAttribute(gqa_decode_kernel<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Layout<128, true>::kTotal);
    in.max_clusters[0] = max_active_clusters<64>();
    in.max_clusters[1] = max_active_clusters<128>();
    cudaGetLastError();
  });
  return g_info[dev].sms > 0 ? &g_info[dev] : nullptr;
}

// CTAs per pair: one wave of the GPU, but no more than one tile per warp at
// the cache's capacity.  Up to 8 of them form a cluster; beyond that, whole
// clusters, as many as can be resident at once.
static Plan plan_for(int B, int Hq, int Hkv, int D, int Tmax, const DeviceInfo& dev) {
  Plan pl{};
  const long long tiles = (Tmax + kTile - 1) / kTile;
  const long long pairs = (long long)B * Hkv;
  const int per_sm = D == 64 ? 2 : 1;   // shared memory per CTA: ~83 KB / ~165 KB
  const long long slots = (long long)dev.sms * per_sm;
  long long ctas = std::max<long long>(1, std::min<long long>(slots / pairs, (tiles + kWarps - 1) / kWarps));
  const int max_clusters = dev.max_clusters[D == 64 ? 0 : 1];
  pl.cluster = 1;
  if (max_clusters >= 1)
    while (pl.cluster * 2 <= std::min<long long>(ctas, kMaxCluster)) pl.cluster *= 2;
  long long clusters = std::min<long long>(kMaxClusters, ctas / pl.cluster);
  if (pl.cluster == kMaxCluster) clusters = std::min<long long>(clusters, max_clusters / pairs);
  pl.clusters = (int)std::max<long long>(1, clusters);
  const int group = Hq / Hkv;
  pl.partial_bytes = pl.clusters > 1 ? (size_t)pairs * pl.clusters * group * (D + 4) * sizeof(float) : 0;
  pl.bytes = ANVILQ_WORKSPACE_COUNTER_BYTES + pl.partial_bytes;
  return pl;
}

static bool args_ok(int B, int Hq, int Hkv, int D, int Tmax) {
  return B >= 1 && Hq >= 1 && Hkv >= 1 && Hq % Hkv == 0 && Hq / Hkv <= kMaxGroup && (D == 64 || D == 128) &&
         Tmax >= 1 && (long long)B * Hkv * (long long)sizeof(int) <= ANVILQ_WORKSPACE_COUNTER_BYTES;
}

static bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static std::once_flag g_encode_once;
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
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

// The cache [B][Tmax][Hkv][D] fp16 as a 4-D tensor (D, Hkv, Tmax, B); one box
// = 64 dims x 1 head x 16 tokens, 128-byte swizzled.
static bool cache_map(CUtensorMap* map, const void* cache, int B, int Hkv, int D, int Tmax) {
  auto encode = encode_fn();
  if (!encode) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)Hkv, (cuuint64_t)Tmax, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)Hkv * D * 2, (cuuint64_t)Tmax * Hkv * D * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)kTile, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(cache), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// INT8 codes [B][Tmax][Hkv][D] as a 4-D tensor (D, Hkv, Tmax, B); one box = a
// 16-token tile of one kv head, unswizzled.
static bool code_map(CUtensorMap* map, const void* codes, int B, int Hkv, int D, int Tmax) {
  auto encode = encode_fn();
  if (!encode) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)Hkv, (cuuint64_t)Tmax, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)D, (cuuint64_t)Hkv * D, (cuuint64_t)Tmax * Hkv * D};
  const cuuint32_t box[4] = {(cuuint32_t)D, 1, (cuuint32_t)kTile, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(codes), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Metadata [B][Hkv][Tmax] uint32 as (Tmax, Hkv, B); one box = 16 tokens' words.
static bool meta_map(CUtensorMap* map, const void* meta, int B, int Hkv, int Tmax) {
  auto encode = encode_fn();
  if (!encode) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)Tmax, (cuuint64_t)Hkv, (cuuint64_t)B};
  const cuuint64_t strides[2] = {(cuuint64_t)Tmax * 4, (cuuint64_t)Hkv * Tmax * 4};
  const cuuint32_t box[3] = {(cuuint32_t)kTile, 1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void*>(meta), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// One launch, clusters of p.cluster CTAs along x.
template <int D, bool Q8>
static cudaError_t launch_d(const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mkm,
                            const CUtensorMap& mvm, const Params& p, int B, cudaStream_t st, bool pdl = false) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.cluster * p.clusters, p.Hkv, B);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Layout<D, Q8>::kTotal;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, gqa_decode_kernel<D, Q8>, mk, mv, mkm, mvm, p);
}

static int finish_launch(cudaError_t e) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}

// fp16 caches: tensor maps for both, then one launch.
static int launch(const Params& p, int B, int D, const void* k_cache, const void* v_cache, cudaStream_t st,
                  bool pdl = false) {
  CUtensorMap mk, mv;
  if (!cache_map(&mk, k_cache, B, p.Hkv, D, p.Tmax) || !cache_map(&mv, v_cache, B, p.Hkv, D, p.Tmax))
    return ANVILQ_EALIGN;
  return finish_launch(D == 64 ? launch_d<64, false>(mk, mv, mk, mv, p, B, st, pdl)
                               : launch_d<128, false>(mk, mv, mk, mv, p, B, st, pdl));
}

// INT8 caches: code and metadata tensor maps, then one launch.
static int launch_q8(const Params& p, int B, int D, const void* k_codes, const void* k_meta, const void* v_codes,
                     const void* v_meta, cudaStream_t st) {
  CUtensorMap mk, mv, mkm, mvm;
  if (!code_map(&mk, k_codes, B, p.Hkv, D, p.Tmax) || !code_map(&mv, v_codes, B, p.Hkv, D, p.Tmax) ||
      !meta_map(&mkm, k_meta, B, p.Hkv, p.Tmax) || !meta_map(&mvm, v_meta, B, p.Hkv, p.Tmax))
    return ANVILQ_EALIGN;
  return finish_launch(D == 64 ? launch_d<64, true>(mk, mv, mkm, mvm, p, B, st)
                               : launch_d<128, true>(mk, mv, mkm, mvm, p, B, st));
}

}  // namespace attn
}  // namespace anvilq

namespace anvilq {

size_t gqa_decode_workspace_bytes(int B, int Hq, int Hkv, int D, int Tmax) {
  using namespace attn;
  if (!args_ok(B, Hq, Hkv, D, Tmax)) return 0;
  const DeviceInfo* dev = device_info();
  if (!dev) return 0;
  return plan_for(B, Hq, Hkv, D, Tmax, *dev).bytes;
}

int launch_gqa_decode_paged(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                            const uint32_t* page_table, const int32_t* seqlens, uint16_t* out, float* lse, int B,
                            int Hq, int Hkv, int D, int page_tokens, int max_pages, int num_pages, float scale,
                            void* workspace, size_t workspace_bytes, int* dev_err, cudaStream_t st) {
  using namespace attn;
  if (!q || !k_pool || !v_pool || !page_table || !seqlens || !out || !dev_err) return ANVILQ_EINVAL;
  if (page_tokens < kTile || page_tokens % kTile || max_pages < 1 || num_pages < 1 ||
      (long long)page_tokens * max_pages > (1LL << 30) || (long long)page_tokens * num_pages > (1LL << 30))
    return ANVILQ_ESHAPE;
  const int Tmax = page_tokens * max_pages;   // logical capacity of a sequence
  if (!args_ok(B, Hq, Hkv, D, Tmax)) return ANVILQ_ESHAPE;
  if (!a16(q) || !a16(k_pool) || !a16(v_pool) || !a16(out)) return ANVILQ_EALIGN;
  const DeviceInfo* dev = device_info();
  if (!dev) return ANVILQ_ECUDA;
  const Plan pl = plan_for(B, Hq, Hkv, D, Tmax, *dev);
  if (!workspace || workspace_bytes < pl.bytes) return ANVILQ_EWORKSPACE;
  if (!a16(workspace)) return ANVILQ_EALIGN;
  Params p{};
  p.q = reinterpret_cast<const __half*>(q);
  p.k = reinterpret_cast<const __half*>(k_pool);
  p.v = reinterpret_cast<const __half*>(v_pool);
  p.seqlens = seqlens;
  p.out = reinterpret_cast<__half*>(out);
  p.tickets = reinterpret_cast<int*>(workspace);
  p.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + ANVILQ_WORKSPACE_COUNTER_BYTES);
  p.dev_err = dev_err;
  p.Hq = Hq; p.Hkv = Hkv; p.Tmax = Tmax; p.group = Hq / Hkv;
  p.cluster = pl.cluster; p.clusters = pl.clusters;
  const float s = scale > 0.0f ? scale : 1.0f / std::sqrt((float)D);
  p.scale_log2 = s * 1.4426950408889634f;
  p.page_table = page_table;
  p.page_tokens = page_tokens;
  p.max_pages = max_pages;
  p.num_pages = num_pages;
  p.lse = lse;
  // the pool as one sequence of num_pages * page_tokens rows
  CUtensorMap mk, mv;
  if (!cache_map(&mk, k_pool, 1, Hkv, D, page_tokens * num_pages) ||
      !cache_map(&mv, v_pool, 1, Hkv, D, page_tokens * num_pages))
    return ANVILQ_EALIGN;
  return finish_launch(D == 64 ? launch_d<64, false>(mk, mv, mk, mv, p, B, st)
                               : launch_d<128, false>(mk, mv, mk, mv, p, B, st));
}

}  // namespace anvilq

using namespace anvilq::attn;

extern "C" {

size_t anvilq_gqa_decode_workspace_size(int B, int Hq, int Hkv, int D, int Tmax) {
  if (!args_ok(B, Hq, Hkv, D, Tmax)) return 0;
  const DeviceInfo* dev = device_info();
  if (!dev) return 0;
  return plan_for(B, Hq, Hkv, D, Tmax, *dev).bytes;
}

int anvilq_gqa_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* seqlens,
                      uint16_t* out, int B, int Hq, int Hkv, int D, int Tmax, float scale, void* workspace,
                      size_t workspace_bytes, int* dev_err, anvilq_stream_t stream) {
  return anvilq_gqa_decode_ex(q, k_cache, v_cache, seqlens, out, B, Hq, Hkv, D, Tmax, scale, workspace,
                              workspace_bytes, dev_err, 0u, stream);
}

int anvilq_gqa_decode_ex(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                         const int32_t* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D, int Tmax,
                         float scale, void* workspace, size_t workspace_bytes, int* dev_err, unsigned flags,
                         anvilq_stream_t stream) {
  if (!q || !k_cache || !v_cache || !seqlens || !out || !dev_err) return ANVILQ_EINVAL;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  if (!args_ok(B, Hq, Hkv, D, Tmax)) return ANVILQ_ESHAPE;
  if (!a16(q) || !a16(k_cache) || !a16(v_cache) || !a16(out)) return ANVILQ_EALIGN;
  const DeviceInfo* dev = device_info();
  if (!dev) return ANVILQ_ECUDA;
  const Plan pl = plan_for(B, Hq, Hkv, D, Tmax, *dev);
  if (!workspace || workspace_bytes < pl.bytes) return ANVILQ_EWORKSPACE;
  if (!a16(workspace)) return ANVILQ_EALIGN;
  Params p{};   // value-initialised: no page table, no escape payloads unless set
  p.q = reinterpret_cast<const __half*>(q);
  p.k = reinterpret_cast<const __half*>(k_cache);
  p.v = reinterpret_cast<const __half*>(v_cache);
  p.seqlens = seqlens;
  p.out = reinterpret_cast<__half*>(out);
  p.tickets = reinterpret_cast<int*>(workspace);   // counters first, partials after them
  p.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + ANVILQ_WORKSPACE_COUNTER_BYTES);
  p.dev_err = dev_err;
  p.Hq = Hq; p.Hkv = Hkv; p.Tmax = Tmax; p.group = Hq / Hkv;
  p.cluster = pl.cluster; p.clusters = pl.clusters;
  const float s = scale > 0.0f ? scale : 1.0f / std::sqrt((float)D);
  p.scale_log2 = s * 1.4426950408889634f;
  p.k_escape = p.v_escape = nullptr;
  return launch(p, B, D, k_cache, v_cache, reinterpret_cast<cudaStream_t>(stream),
                (flags & ANVILQ_GEMM_OVERLAP_PRIOR) != 0);
}

int anvilq_gqa_decode_int8(const uint16_t* q, const int8_t* k_codes, const uint32_t* k_meta, const float* k_escape,
                           const int8_t* v_codes, const uint32_t* v_meta, const float* v_escape,
                           const int32_t* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D, int Tmax,
                           float scale, void* workspace, size_t workspace_bytes, int* dev_err,
                           anvilq_stream_t stream) {
  if (!q || !k_codes || !k_meta || !v_codes || !v_meta || !seqlens || !out || !dev_err) return ANVILQ_EINVAL;
  if (!args_ok(B, Hq, Hkv, D, Tmax) || Tmax % kTile) return ANVILQ_ESHAPE;
  if (!a16(q) || !a16(k_codes) || !a16(v_codes) || !a16(k_meta) || !a16(v_meta) || !a16(out) ||
      (k_escape && !a16(k_escape)) || (v_escape && !a16(v_escape)))
    return ANVILQ_EALIGN;
  const DeviceInfo* dev = device_info();
  if (!dev) return ANVILQ_ECUDA;
  const Plan pl = plan_for(B, Hq, Hkv, D, Tmax, *dev);
  if (!workspace || workspace_bytes < pl.bytes) return ANVILQ_EWORKSPACE;
  if (!a16(workspace)) return ANVILQ_EALIGN;
  Params p{};   // value-initialised: no page table, no escape payloads unless set
  p.q = reinterpret_cast<const __half*>(q);
  p.k = p.v = nullptr;
  p.seqlens = seqlens;
  p.out = reinterpret_cast<__half*>(out);
  p.tickets = reinterpret_cast<int*>(workspace);
  p.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + ANVILQ_WORKSPACE_COUNTER_BYTES);
  p.dev_err = dev_err;
  p.Hq = Hq; p.Hkv = Hkv; p.Tmax = Tmax; p.group = Hq / Hkv;
  p.cluster = pl.cluster; p.clusters = pl.clusters;
  const float s = scale > 0.0f ? scale : 1.0f / std::sqrt((float)D);
  p.scale_log2 = s * 1.4426950408889634f;
  p.k_escape = k_escape;
  p.v_escape = v_escape;
  return launch_q8(p, B, D, k_codes, k_meta, v_codes, v_meta, reinterpret_cast<cudaStream_t>(stream));
}

int anvilq_gqa_decode_paged(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                            const uint32_t* page_table, const int32_t* seqlens, uint16_t* out, int B, int Hq, int Hkv,
                            int D, int page_tokens, int max_pages, int num_pages, float scale, void* workspace,
                            size_t workspace_bytes, int* dev_err, anvilq_stream_t stream) {
  return anvilq::launch_gqa_decode_paged(q, k_pool, v_pool, page_table, seqlens, out, nullptr, B, Hq, Hkv, D,
                                         page_tokens, max_pages, num_pages, scale, workspace, workspace_bytes,
                                         dev_err, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Attention with no allocation and no caller workspace.
//
// Some callers cannot hand this library any device memory of their own:
// a host whose allocator owns all of HBM and offers nothing per call, a
// binding that only passes the tensors it was given, or a loop that must not
// trigger cudaMalloc's implicit device synchronisation.  For them the split-KV
// scratch (arrival counters, then per-split partial results) lives in a fixed
// array in this library's device image instead.  Every GPU that loads the
// library holds these bytes until the process exits.
namespace anvilq {
namespace attn {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;   // 4 MiB, counters included
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static void* g_noalloc_ptr[kMaxDevices];
static int g_noalloc_rc[kMaxDevices];
static std::once_flag g_noalloc_once[kMaxDevices];

// Device address of g_noalloc_scratch on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is asked from the
// runtime once per device, with that device current.
static int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  std::call_once(g_noalloc_once[dev], [dev] {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    g_noalloc_rc[dev] = e == cudaSuccess && p != nullptr ? ANVILQ_OK : ANVILQ_ECUDA;
    g_noalloc_ptr[dev] = e == cudaSuccess ? p : nullptr;
    if (e != cudaSuccess) cudaGetLastError();
  });
  *out = g_noalloc_ptr[dev];
  return g_noalloc_rc[dev];
}

}  // namespace attn
}  // namespace anvilq

extern "C" int anvilq_gqa_decode_noalloc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                         const int32_t* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D,
                                         int Tmax, float scale, int* dev_err, anvilq_stream_t stream) {
  using namespace anvilq::attn;
  if (!q || !k_cache || !v_cache || !seqlens || !out || !dev_err) return ANVILQ_EINVAL;
  if (!args_ok(B, Hq, Hkv, D, Tmax)) return ANVILQ_ESHAPE;
  if (!a16(q) || !a16(k_cache) || !a16(v_cache) || !a16(out)) return ANVILQ_EALIGN;
  const DeviceInfo* dev = device_info();
  if (!dev) return ANVILQ_ECUDA;
  const Plan pl = plan_for(B, Hq, Hkv, D, Tmax, *dev);
  if (pl.bytes > kNoAllocScratchBytes) return ANVILQ_ENOSCRATCH;
  void* ws = nullptr;
  const int rc = noalloc_scratch(&ws);
  if (rc != ANVILQ_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // The array keeps whatever the previous call left.  Counters must start at
  // zero; a call cut short by a bounded wait may not have re-armed them.
  if (cudaMemsetAsync(ws, 0, (size_t)B * Hkv * sizeof(int), st) != cudaSuccess) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  Params p{};   // value-initialised: no page table, no escape payloads unless set
  p.q = reinterpret_cast<const __half*>(q);
  p.k = reinterpret_cast<const __half*>(k_cache);
  p.v = reinterpret_cast<const __half*>(v_cache);
  p.seqlens = seqlens;
  p.out = reinterpret_cast<__half*>(out);
  p.tickets = reinterpret_cast<int*>(ws);
  p.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + ANVILQ_WORKSPACE_COUNTER_BYTES);
  p.dev_err = dev_err;
  p.Hq = Hq; p.Hkv = Hkv; p.Tmax = Tmax; p.group = Hq / Hkv;
  p.cluster = pl.cluster; p.clusters = pl.clusters;
  const float s = scale > 0.0f ? scale : 1.0f / std::sqrt((float)D);
  p.scale_log2 = s * 1.4426950408889634f;
  p.k_escape = p.v_escape = nullptr;
  return launch(p, B, D, k_cache, v_cache, st);
}
