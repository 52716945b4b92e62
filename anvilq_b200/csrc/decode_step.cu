// decode_step.cu -- every decoder layer of one greedy decode token in ONE
// persistent kernel (one CTA per SM, all CTAs co-resident by cooperative launch).
//
// Reference semantics: FP32Model.token (anvil-q1/tests/official_weights.py:451-509)
// and QwenFP64.step (anvil-q1-fp/tests/fp64_reference.py:210-246), per layer:
//   h = rmsnorm(x); q,k,v = h W_qkv + b; rope(q, k); cache k, v
//   a = attention(q, K, V); x += a W_o
//   h = rmsnorm(x); g, u = h W_gate, h W_up; x += (silu(g) u) W_down
// with the W4A16 datapath's roundings: the normalised activations, q / k / v,
// the attention output, g and u and silu(g) u are binary16; the residual stream
// and every accumulation are binary32.
//
// Why one kernel.  A 0.5B-class layer moves ~8 MB of int4 weights, 1.3 us of
// HBM time, but as five launches (QKV, attention, O, gate/up, down) it costs
// ~24 us: every launch pays its ramp and tail.  Here the five phases of a layer
// are roles that CTAs take (one CTA per SM for the whole launch).
//
// Tagged words instead of counters.  A decode layer is a chain of five
// dependent phases, so latency bounds it, and a counter handoff costs three
// serial trips through L2: the producer's fence, the consumer's poll of the
// counter, then its loads of the data.  Here every value a phase hands on is
// stored as one 8-byte word (value bits | tag << 32; 8-byte relaxed stores and
// loads are single-copy atomic), the tag naming launch and layer.  A consumer
// loads exactly the words it needs and re-loads those whose tag is not yet
// this layer's: one trip, no fence, and no CTA waits for data it does not use
// (a down split waits only for the gate/up units of its rows).  Every poll is
// bounded (~1 s, or another CTA gave up), then ANVILQ_DEV_ERR_TIMEOUT.  A
// buffer is rewritten only by a later layer, whose producers depend, through
// the data they consume, on every read of the earlier layer's words.
//
// Nothing is merged or fixed up in a phase of its own:
//   - attention units hand on unnormalised partials (m, l, o); every O CTA
//     merges all of them as it stages its inputs (redundant across O CTAs, a
//     few tens of KB of L2 reads each, instead of a serial phase);
//   - down splits hand on partial column sums; the residual after layer l is
//     never stored: the next layer's QKV and O CTAs add x_a and the splits in
//     split order as part of their input load.
//
// Weights stream ahead.  Each CTA's slice of a phase's weights (int4 words,
// zeros, scales, and the RMSNorm gamma) and, for attention, the first chunk of
// its KV range up to the previous position, are copied into shared memory with
// cp.async as soon as the CTA has finished the same phase of the previous
// layer: a whole layer of lead time, so the copies never sit on the critical
// path.  Three groups are in flight per CTA (roles A = QKV or attention or O,
// B = gate/up, C = down).
//
// Work per layer (P = #CTAs, 512 threads each):
//   QKV   one head (D columns, all H rows) per CTA: RoPE and the K / V cache
//         append need both halves of a head, so the head is the unit.
//   attn  (kv head, range of 64-token chunks) per CTA, online softmax over the
//         range's chunks in fp32.
//   O     32 output columns (4 qweight words) per CTA; residual added.
//   g/u   32 intermediate columns of gate AND of up per CTA as ONE tile of 8
//         words a row (gate and up interleaved at load time), so silu(g) u is
//         formed locally; units beyond P go to the last CTAs, which have no
//         down split, and the rows of those units form the last split alone.
//   down  32 output columns x a split of the groups of K = I per CTA.
// The GEMV arithmetic is that of the batch-1 kernels: binary16-subnormal
// nibbles, exact products by fma.rn.f32.f16 into fp32, zero points through
// the group's sum of x, scales in fp32.  Every sum has a fixed order.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "../../include/anvilq.h"
#include "awq_common.cuh"
#include "internal.h"

namespace anvilq {
namespace dstep {

using u64 = unsigned long long;

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kG = 128;            // AWQ group (rows)
constexpr int kBW = 4;             // words of an O / down unit (32 columns)
constexpr int kGU = 8;             // words of a gate/up unit (32 gate + 32 up columns)
constexpr int kChunk = 64;         // attention tokens per chunk
constexpr int kMaxGroup = 8;       // q heads per kv head
constexpr int kMaxD = 128;
constexpr int kMaxUnits = 32;      // attention units per kv head (one merge lane each)
constexpr int kMaxSplit = 16;      // down splits (each adds a load to the residual)
constexpr unsigned long long kWaitNs = 1000000000ull;

// shared-memory scratch `misc` (floats)
constexpr int kMiscY = 32;         // GEMV outputs, up to 128
constexpr int kMiscAct = 96;       // gate/up: the unit's 32 silu(g) u (binary16)
constexpr int kMiscBig = 160;      // per role: RoPE table and QKV output, attention state, O merge weights
constexpr int kQkvOut = kMiscBig + kMaxD;                     // QKV: the head's D binary16 outputs
constexpr int kAttQs = kMiscBig;                              // [grp][D] scaled q
constexpr int kAttP = kAttQs + kMaxGroup * kMaxD;             // [grp][64] probabilities
constexpr int kAttWmax = kAttP + kMaxGroup * kChunk;          // [grp][2]
constexpr int kAttWsum = kAttWmax + 2 * kMaxGroup;            // [grp][2]
constexpr int kAttM = kAttWsum + 2 * kMaxGroup;               // [2][grp] running max by chunk parity
constexpr int kAttL = kAttM + 2 * kMaxGroup;                  // [grp] running sum
constexpr int kAttRaw = kAttL + kMaxGroup;                    // staged q (grp D halves), k and v rows (2 D halves)
constexpr int kAttEnd = kAttRaw + (kMaxGroup * kMaxD + 2 * kMaxD) / 2;

struct Params {
  const anvilq_decode_layer* layers;
  int L, H, I, QH, KVH, D, Tmax, V;
  float eps;
  const __half* emb;
  const int* token;
  const int* pos;
  int* seqlen;
  float* x_out;
  u64* key;
  int* dev_err;
  // workspace: launch bookkeeping
  int* exit_ctr;    // CTAs out of this launch
  int* abort_flag;  // a CTA gave up
  unsigned* seq;    // launches completed (the tags' launch part)
  // workspace: tagged words (value bits | tag << 32), one buffer per handoff
  u64* ll_xa;       // [H] residual after attention
  u64* ll_dpart;    // [H / 32][nsplit][32] down partial sums
  u64* ll_q;        // [QH * D / 2] rotated q, two binary16 a word
  u64* ll_kv;       // [2][KVH][D / 2] this token's k rows, then its v rows
  u64* ll_apart;    // [KVH][nu_max][perP] attention partials: [group][D + 2] (m, l, o), padded
  u64* ll_act;      // [I / 2] silu(g) u, two binary16 a word
  // roles: A = QKV heads [0, n1), attention [n1, n1 + n2), O blocks [n1 + n2, n1 + n2 + n3)
  int n1, n2, n3, nsplit, nu_max;
  int perP;         // words of one unit's partials, group * (D + 2) rounded up to a multiple of 4
  int gx;           // > 0: the last down split is groups [gx, I / 128) (the extra gate/up units' rows)
  // shared-memory carve-up (bytes)
  int offA, offB, offC, offX, offRed, offMisc, offBst, smem;
  int offStage;     // within region A, after every role's tile: staged inputs, attention's P V sums
  double rope_inv[kMaxD / 2];
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// ---- bulk copies into shared memory, completion counted on an mbarrier -------
__device__ __forceinline__ void mbar_init(u64* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)) : "memory");
}
// The one arrival of a phase, by the thread that then issues its copies; the
// proxy fence orders the CTA's earlier shared-memory reads (made visible to it
// by the barrier before the prefetch) before the bulk copies' writes.
__device__ __forceinline__ void mbar_expect(u64* bar, uint32_t bytes) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(u64* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// `bytes` (a multiple of 16, both addresses 16-byte aligned) from global memory,
// counted on `bar` (no multicast)
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, u64* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ int ld_relaxed(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ half2 h2(uint32_t u) { return *reinterpret_cast<half2*>(&u); }
__device__ __forceinline__ uint32_t h2u(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
__device__ __forceinline__ void fma_f32_f16x2(float& a0, float& a1, uint32_t q2, unsigned short x) {
  asm("{\n .reg .f16 q0, q1;\n mov.b32 {q0, q1}, %2;\n"
      " fma.rn.f32.f16 %0, %3, q0, %0;\n fma.rn.f32.f16 %1, %3, q1, %1;\n}"
      : "+f"(a0), "+f"(a1)
      : "r"(q2), "h"(x));
}
__device__ __forceinline__ bool misaligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

// ---- tagged words ------------------------------------------------------------
__device__ __forceinline__ void ll_put(u64* dst, uint32_t bits, uint32_t tag) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(dst), "l"(((u64)tag << 32) | bits) : "memory");
}
__device__ __forceinline__ ulonglong2 ll_get2(const u64* src) {
  ulonglong2 v;
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(src));
  return v;
}

// Where a gather reads: up to three segments, each `rows` runs of
// `row_chunks` 16-byte chunks (two tagged words) `stride` words apart, all
// expected to carry `tag`.
struct LLSeg {
  const u64* base;
  int rows, row_chunks, stride;
  unsigned tag;
};
struct LLSrc {
  LLSeg s[3];
  int nseg;
};
__device__ __forceinline__ LLSrc ll_src(LLSeg a) { return LLSrc{{a, a, a}, 1}; }
__device__ __forceinline__ LLSrc ll_src(LLSeg a, LLSeg b) { return LLSrc{{a, b, b}, 2}; }
__device__ __forceinline__ LLSrc ll_src(LLSeg a, LLSeg b, LLSeg c) { return LLSrc{{a, b, c}, 3}; }
__device__ __forceinline__ LLSeg ll_run(const u64* base, int words, unsigned tag) {   // one contiguous run
  return LLSeg{base, 1, words / 2, 0, tag};
}

// Gather the chunks of `src` into shared memory as their value bits, chunk i
// (counted across the segments in order) to dst[2i], dst[2i + 1], once both
// its words carry the segment's tag.  Each thread re-loads only its chunks
// not yet complete, four loads in flight.  Bounded: after ~1 s, or when
// another CTA gave up, the CTA gives up.  Ends with a barrier; returns the
// CTA's verdict.
__device__ __noinline__ bool ll_gather(const Params& p, uint32_t* dst, const LLSrc src) {
  constexpr int kFly = 4;
  int n = 0;
  for (int k = 0; k < src.nseg; ++k) n += src.s[k].rows * src.s[k].row_chunks;
  auto where = [&](int i, unsigned* tag) {
    int k = 0;
    for (; k + 1 < src.nseg; ++k) {
      const int c = src.s[k].rows * src.s[k].row_chunks;
      if (i < c) break;
      i -= c;
    }
    const LLSeg& g = src.s[k];
    *tag = g.tag;
    const int r = g.rows > 1 ? i / g.row_chunks : 0;
    return g.base + (size_t)r * g.stride + 2 * (i - r * g.row_chunks);
  };
  bool ok = true;
  for (int base = 0; base < n; base += 32 * kThreads) {
    uint32_t pending = 0;
    for (int k = 0; k < 32; ++k)
      if (base + (int)threadIdx.x + k * kThreads < n) pending |= 1u << k;
    unsigned long long t0 = 0;
    uint32_t rounds = 0;
    while (pending && ok) {
      uint32_t rest = pending;
      while (rest) {
        int ks[kFly];
        unsigned tg[kFly];
        ulonglong2 v[kFly];
#pragma unroll
        for (int j = 0; j < kFly; ++j) {
          ks[j] = rest ? __ffs(rest) - 1 : -1;
          rest &= rest - 1;
        }
#pragma unroll
        for (int j = 0; j < kFly; ++j)
          if (ks[j] >= 0) v[j] = ll_get2(where(base + (int)threadIdx.x + ks[j] * kThreads, &tg[j]));
#pragma unroll
        for (int j = 0; j < kFly; ++j)
          if (ks[j] >= 0 && (uint32_t)(v[j].x >> 32) == tg[j] && (uint32_t)(v[j].y >> 32) == tg[j]) {
            const int i = base + (int)threadIdx.x + ks[j] * kThreads;
            dst[2 * i] = (uint32_t)v[j].x;
            dst[2 * i + 1] = (uint32_t)v[j].y;
            pending &= ~(1u << ks[j]);
          }
      }
      if (pending && (++rounds & 15u) == 0) {
        const unsigned long long now = globaltimer();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > kWaitNs) {
          ok = false;
          if (p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
          atomicExch(p.abort_flag, 1);
        }
        if (ok && ld_relaxed(p.abort_flag)) ok = false;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// Bytes of one column block of a projection (see anvilq_block_columns):
// `rows` rows of `words` int4 words, the zeros [ng][words] and the scales
// [ng][8 words] (binary16) of its ng groups -- three contiguous ranges.
__host__ __device__ inline uint32_t block_bytes(int rows, int words, int ng) {
  return (uint32_t)(rows * words * 4 + ng * words * 4 + ng * words * 16);
}
// The three ranges of a column block as three bulk copies (one thread).
__device__ void load_block(uint32_t* wdst, uint32_t* zdst, uint32_t* sdst, const int32_t* wsrc, const int32_t* zsrc,
                           const __half* ssrc, int rows, int words, int ng, u64* bar) {
  bulk_load(wdst, wsrc, rows * words * 4, bar);
  bulk_load(zdst, zsrc, ng * words * 4, bar);
  bulk_load(sdst, ssrc, ng * words * 16, bar);
}

// dst[b][r][e] = src[r][b * block + e]: the column blocks of a row-major matrix
// laid out one after another (16-byte pieces; block * elem_bytes % 16 == 0).
__global__ void block_columns_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, long long rows,
                                     long long row_vecs, long long block_vecs) {
  const long long n = rows * row_vecs;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / row_vecs, c = i % row_vecs, b = c / block_vecs, e = c % block_vecs;
    dst[(b * rows + r) * block_vecs + e] = src[i];
  }
}

// out[8 W] = x[0:R] . dequant(W[0:R][0:W]) for a tile in shared memory whose
// row 0 is row `row0` of the matrix (groups of 128 rows).  Thread t takes word
// t % W and the contiguous rows of row set t / W; row sets are summed within
// the warp by shuffles, then the warps' sums by every thread: the 512 / (8 W)
// lanes of an output add 16 W / 32 warps' values each and a shuffle tree adds
// the lanes (a fixed order).  `red` holds kWarps x 8 W floats.  Returns
// nonzero if a scale of the tile was invalid.
template <int W>
__device__ uint32_t tile_gemv(const uint32_t* wsm, const __half* xs, const uint32_t* zsm, const uint32_t* ssm,
                              int R, int row0, float* red, float* out) {
  constexpr int S = kThreads / W;
  const int t = threadIdx.x, word = t % W, s = t / W, lane = t & 31, warp = t >> 5;
  const int rb = (int)((long long)s * R / S), re = (int)((long long)(s + 1) * R / S);
  float A[8], Y[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) A[i] = Y[i] = 0.0f;
  float Xg = 0.0f;
  uint32_t bad = 0;
  const int g0 = row0 / kG;
  int g = (row0 + rb) / kG;
  int bnd = (g + 1) * kG - row0;
  auto flush = [&](int gl) {
    const uint32_t zw = zsm[gl * W + word];
    const uint32_t zp[4] = {(zw & 0x000F000Fu) | 0x64006400u, ((zw >> 4) & 0x000F000Fu) | 0x64006400u,
                            ((zw >> 8) & 0x000F000Fu) | 0x64006400u, ((zw >> 12) & 0x000F000Fu) | 0x64006400u};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t sw = ssm[gl * 4 * W + 4 * word + e];
      bad |= invalid_scale_pair(sw);
      const float2 s2 = __half22float2(h2(sw));
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
  const unsigned short* xh = reinterpret_cast<const unsigned short*>(xs);
  auto rows = [&](int r0, int r1) {   // rows of one group
#pragma unroll 4
    for (int r = r0; r < r1; ++r) {
      const uint32_t wd = wsm[r * W + word];
      const unsigned short xv = xh[r];
      Xg += __half2float(__ushort_as_half(xv));
      const uint32_t w8 = wd >> 8;
      fma_f32_f16x2(A[0], A[1], wd & 0x000F000Fu, xv);   // columns 0,1
      fma_f32_f16x2(A[2], A[3], wd & 0x00F000F0u, xv);   // columns 2,3 (x16)
      fma_f32_f16x2(A[4], A[5], w8 & 0x000F000Fu, xv);   // columns 4,5
      fma_f32_f16x2(A[6], A[7], w8 & 0x00F000F0u, xv);   // columns 6,7 (x16)
    }
  };
  // a thread's contiguous rows (fewer than 128) cross at most one group boundary
  for (int r = rb; r < re;) {
    const int e = min(re, bnd);
    rows(r, e);
    flush(g - g0);
    r = e;
    ++g;
    bnd += kG;
  }
#pragma unroll
  for (int o = W; o < 32; o <<= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i) Y[i] += __shfl_xor_sync(0xffffffffu, Y[i], o);
  if (lane < W)
#pragma unroll
    for (int i = 0; i < 8; ++i) red[warp * 8 * W + 8 * lane + i] = Y[i];
  __syncthreads();
  constexpr int G = kThreads / (8 * W);   // lanes per output (W >= 2: within a warp)
  static_assert(G <= 32 && kWarps % G == 0, "tile width");
  {
    const int o = t / G, k = t % G;
    float v = 0.0f;
#pragma unroll
    for (int j = 0; j < kWarps / G; ++j) v += red[(k + j * G) * 8 * W + o];
#pragma unroll
    for (int m = G / 2; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    if (k == 0) out[o] = v;
  }
  __syncthreads();
  return bad;
}

// The residual entering a layer after the first at column k of a 32-column
// block: x_a of the previous layer plus its down splits added in split order,
// from values staged as xa[k] and splits[s * 32 + k % 32] of the block.
__device__ __forceinline__ float residual_sum(float xa, const float* splits, int nsplit, int k) {
  float acc = 0.0f;
  for (int s = 0; s < nsplit; ++s) acc += splits[s * 32 + (k & 31)];
  return xa + acc;
}

// x_norm[k] = fp16(x[k] * gamma[k] / sqrt(mean(x^2) + eps)) into shared memory,
// x[k] = val(k) (from shared memory), gamma in shared memory.  Every thread
// keeps its (at most kMaxPerThread) values: one pass over x.
constexpr int kMaxPerThread = 8;   // H <= 4096
template <class Val>
__device__ void rmsnorm_to_smem(const Params& p, Val val, const __half* gamma, __half* xs, float* misc) {
  float v[kMaxPerThread];
  float ss = 0.0f;
#pragma unroll
  for (int u = 0; u < kMaxPerThread; ++u) {
    const int k = threadIdx.x + u * kThreads;
    v[u] = k < p.H ? val(k) : 0.0f;
  }
#pragma unroll
  for (int u = 0; u < kMaxPerThread; ++u) ss = fmaf(v[u], v[u], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) misc[threadIdx.x >> 5] = ss;
  __syncthreads();
  // every warp adds the 16 warp sums by the same shuffle tree (no second barrier)
  float tsum = misc[threadIdx.x & (kWarps - 1)];
#pragma unroll
  for (int o = kWarps / 2; o > 0; o >>= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, o);
  const float inv = 1.0f / sqrtf(tsum / (float)p.H + p.eps);
#pragma unroll
  for (int u = 0; u < kMaxPerThread; ++u) {
    const int k = threadIdx.x + u * kThreads;
    if (k < p.H) xs[k] = __float2half_rn(v[u] * __half2float(gamma[k]) * inv);
  }
  __syncthreads();
}

__device__ __host__ inline int a_words(int D) { return D / 8; }
__device__ __host__ inline int kv_stride(int D) { return D + 8; }   // halves; 16-byte rows, no bank conflicts
// groups [*g0, *g1) of K = I in down split ds
__device__ __host__ inline void down_split(int ds, int nsplit, int ngI, int gx, int* g0, int* g1) {
  if (gx > 0) {
    *g0 = ds < nsplit - 1 ? ds * gx / (nsplit - 1) : gx;
    *g1 = ds < nsplit - 1 ? (ds + 1) * gx / (nsplit - 1) : ngI;
  } else {
    *g0 = ds * ngI / nsplit;
    *g1 = (ds + 1) * ngI / nsplit;
  }
}

__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int cta = blockIdx.x, P = gridDim.x, tid = threadIdx.x;
  unsigned char* regA = smem + p.offA;
  unsigned char* regB = smem + p.offB;
  unsigned char* regC = smem + p.offC;
  __half* xs = reinterpret_cast<__half*>(smem + p.offX);
  float* red = reinterpret_cast<float*>(smem + p.offRed);
  float* misc = reinterpret_cast<float*>(smem + p.offMisc);
  float* bst = reinterpret_cast<float*>(smem + p.offBst);   // gate/up: x_a staged
  const int H = p.H, I = p.I, QH = p.QH, KVH = p.KVH, D = p.D, grp = QH / KVH;
  const int nb = H / 32;                  // 32-column blocks of H
  const int n_gu = I / 32;                // gate/up units
  const int ngI = I / kG;                 // groups of K = I
  const int ngH = H / kG;
  const int KS = kv_stride(D);
  uint32_t bad = 0;

  int pos = *p.pos;
  int token = *p.token;
  if (pos < 0 || pos >= p.Tmax || token < 0 || token >= p.V) {
    if (cta == 0 && tid == 0 && p.dev_err)
      atomicOr(p.dev_err, pos < 0 || pos >= p.Tmax ? ANVILQ_DEV_ERR_SEQLEN : ANVILQ_DEV_ERR_TOKEN);
    return;   // every CTA returns here alike: nothing was written
  }
  const unsigned seq = *p.seq;            // the tag of layer l: seq * L + l + 1 (never 0 before it wraps)
  auto tag_of = [&](int l) { return seq * (unsigned)p.L + (unsigned)l + 1u; };
  const int T = pos + 1;                  // attention length
  const int nch = (T + kChunk - 1) / kChunk;
  const int nu = min(p.nu_max, nch);      // attention units per kv head this token
  const __half* xemb = p.emb + (size_t)token * H;
  if (cta == 0 && tid == 0) {
    if (p.seqlen) *p.seqlen = T;
    if (p.key) *p.key = 0ull;
  }

  // ---- roles of this CTA --------------------------------------------------
  const int roleA = cta < p.n1 ? 1 : cta < p.n1 + p.n2 ? 2 : cta < p.n1 + p.n2 + p.n3 ? 3 : 0;
  const int idxA = roleA == 1 ? cta : roleA == 2 ? cta - p.n1 : cta - p.n1 - p.n2;
  const int ah = roleA == 2 ? idxA / p.nu_max : 0, au = roleA == 2 ? idxA % p.nu_max : 0;   // kv head, unit
  const int ac0 = au * nch / nu, ac1 = (au + 1) * nch / nu;                                   // its chunks
  const bool att_on = roleA == 2 && au < nu;
  const int extra = max(0, n_gu - P);                              // units beyond one a CTA
  const int gu0 = cta < n_gu ? cta : -1;
  const int gu1 = cta >= P - extra ? P + (P - 1 - cta) : -1;       // the extra units, from the last CTA down
  const bool has_down = cta < nb * p.nsplit;
  const int db = cta / p.nsplit, ds = cta % p.nsplit;              // down block and split
  int dg0 = 0, dg1 = 0;
  down_split(ds, p.nsplit, ngI, p.gx, &dg0, &dg1);
  const int drow0 = dg0 * kG, drows = (dg1 - dg0) * kG;

  // role-A tile layout (QKV head / O block): weights, zeros, scales[, gamma]
  const int wA = roleA == 1 ? a_words(D) : kBW;
  const int rowsA = roleA == 1 ? H : QH * D;
  uint32_t* A_w = reinterpret_cast<uint32_t*>(regA);
  uint32_t* A_z = A_w + rowsA * wA;
  uint32_t* A_s = A_z + ((rowsA + kG - 1) / kG) * wA;
  __half* A_gamma = reinterpret_cast<__half*>(A_s + ((rowsA + kG - 1) / kG) * 4 * wA);
  float* stage = reinterpret_cast<float*>(regA + p.offStage);   // staged inputs; attention: P V sums
  __half* Kc = reinterpret_cast<__half*>(regA);                  // attention: [64][KS]
  __half* Vc = Kc + kChunk * KS;
  // gate/up: up to two units, each [H][8 words] + zeros + scales, then gamma_post
  const int guTile = H * kGU + ngH * kGU + ngH * 4 * kGU;        // uint32 per unit
  auto gu_w = [&](int slot) { return reinterpret_cast<uint32_t*>(regB) + slot * guTile; };
  __half* B_gamma = reinterpret_cast<__half*>(gu_w(2));
  uint32_t* C_w = reinterpret_cast<uint32_t*>(regC);
  uint32_t* C_z = C_w + drows * kBW;
  uint32_t* C_s = C_z + (drows / kG) * kBW;

  // QKV role: sin / cos of this launch's position for each rotated pair (every layer alike)
  float* rope_sc = misc + kMiscBig;   // [sin: D / 2][cos: D / 2], the QKV role's part of misc
  if (roleA == 1)
    for (int i = tid; i < D / 2; i += kThreads) {
      const float angle = (float)((double)pos * p.rope_inv[i]);
      sincosf(angle, &rope_sc[i], &rope_sc[kMaxD / 2 + i]);
    }
  bool ok = true, misal = false;   // misal: a tensor of the layer table is not 16-byte aligned
  // Prefetches: bulk copies counted on one mbarrier per region (A, B, C, and
  // K for the attention's later chunks), one phase per layer; `armed` marks a
  // phase issued and not yet waited for.
  __shared__ __align__(8) u64 s_bar[4];
  uint32_t parity[4] = {0u, 0u, 0u, 0u};
  bool armed[4] = {false, false, false, false};
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&s_bar[i]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // every thread waits for region r's phase, bounded; false when it expired
  auto wait_region = [&](int r) {
    if (!armed[r]) return true;
    armed[r] = false;
    const uint32_t ph = parity[r];
    parity[r] ^= 1u;
    if (mbar_test(&s_bar[r], ph)) return true;
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 0;; ++i) {
      if (mbar_test(&s_bar[r], ph)) return true;
      if ((i & 255u) == 255u && globaltimer() - t0 > kWaitNs) {
        if (p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
        atomicExch(p.abort_flag, 1);
        return false;
      }
    }
  };
  // a chunk of kv head h: rows t0 .. t0 + cnt - 1 except the current position
  // (this token's row comes from the QKV phase's tagged words), one bulk copy a
  // row of K and of V, issued by warp 0
  auto load_chunk = [&](const anvilq_decode_layer& Ly, int h, int c, int r) {
    const int t0 = c * kChunk, cnt = min(kChunk, T - t0);
    if (tid < 32) {
      const uint32_t rowb = D * 2;
      const int rows = cnt - (pos >= t0 && pos < t0 + cnt ? 1 : 0);
      if (tid == 0) mbar_expect(&s_bar[r], 2u * rowb * rows);
      __syncwarp();
      const __half* kc = reinterpret_cast<const __half*>(Ly.k_cache);
      const __half* vc = reinterpret_cast<const __half*>(Ly.v_cache);
      for (int i = tid; i < cnt; i += 32) {
        const int tok = t0 + i;
        if (tok == pos) continue;
        const size_t off = ((size_t)tok * KVH + h) * D;
        bulk_load(Kc + i * KS, kc + off, rowb, &s_bar[r]);
        bulk_load(Vc + i * KS, vc + off, rowb, &s_bar[r]);
      }
    }
    armed[r] = true;
  };
  // Each prefetch first checks the alignment the bulk copies need, and runs
  // after a barrier: nothing still reads the region it overwrites.
  auto prefetchA = [&](int l) {
    const anvilq_decode_layer& Ly = p.layers[l];
    if (roleA == 1) {   // column block idxA (one head) of the blocked QKV projection, and gamma_in
      const int wd = a_words(D);
      if (misaligned16(Ly.qkv_qweight) || misaligned16(Ly.qkv_qzeros) || misaligned16(Ly.qkv_scales) ||
          misaligned16(Ly.gamma_in) || misaligned16(Ly.k_cache) || misaligned16(Ly.v_cache)) {
        misal = true, ok = false;
      } else {
        if (tid == 0) {
          mbar_expect(&s_bar[0], block_bytes(H, wd, ngH) + H * 2);
          load_block(A_w, A_z, A_s, Ly.qkv_qweight + (size_t)idxA * H * wd, Ly.qkv_qzeros + (size_t)idxA * ngH * wd,
                     reinterpret_cast<const __half*>(Ly.qkv_scales) + (size_t)idxA * ngH * 8 * wd, H, wd, ngH,
                     &s_bar[0]);
          bulk_load(A_gamma, Ly.gamma_in, H * 2, &s_bar[0]);
        }
        armed[0] = true;
      }
    } else if (att_on) {   // the unit's first chunk
      if (misaligned16(Ly.k_cache) || misaligned16(Ly.v_cache)) misal = true, ok = false;
      else load_chunk(Ly, ah, ac0, 0);
    } else if (roleA == 3) {   // column block idxA of the blocked O projection
      const int K = QH * D, ng = K / kG;
      if (misaligned16(Ly.o_qweight) || misaligned16(Ly.o_qzeros) || misaligned16(Ly.o_scales)) {
        misal = true, ok = false;
      } else {
        if (tid == 0) {
          mbar_expect(&s_bar[0], block_bytes(K, kBW, ng));
          load_block(A_w, A_z, A_s, Ly.o_qweight + (size_t)idxA * K * kBW, Ly.o_qzeros + (size_t)idxA * ng * kBW,
                     reinterpret_cast<const __half*>(Ly.o_scales) + (size_t)idxA * ng * 8 * kBW, K, kBW, ng,
                     &s_bar[0]);
        }
        armed[0] = true;
      }
    }
  };
  auto prefetchB = [&](int l) {
    if (gu0 < 0) return;
    const anvilq_decode_layer& Ly = p.layers[l];
    if (misaligned16(Ly.gu_qweight) || misaligned16(Ly.gu_qzeros) || misaligned16(Ly.gu_scales) ||
        misaligned16(Ly.gamma_post)) {
      misal = true, ok = false;
      return;
    }
    if (tid == 0) {
      mbar_expect(&s_bar[1], (gu1 >= 0 ? 2u : 1u) * block_bytes(H, kGU, ngH) + H * 2);
      const int units[2] = {gu0, gu1};
      for (int sl = 0; sl < 2; ++sl) {
        const int u = units[sl];
        if (u < 0) continue;
        uint32_t* w = gu_w(sl);
        load_block(w, w + H * kGU, w + H * kGU + ngH * kGU, Ly.gu_qweight + (size_t)u * H * kGU,
                   Ly.gu_qzeros + (size_t)u * ngH * kGU,
                   reinterpret_cast<const __half*>(Ly.gu_scales) + (size_t)u * ngH * 8 * kGU, H, kGU, ngH, &s_bar[1]);
      }
      bulk_load(B_gamma, Ly.gamma_post, H * 2, &s_bar[1]);
    }
    armed[1] = true;
  };
  auto prefetchC = [&](int l) {
    if (!has_down) return;
    const anvilq_decode_layer& Ly = p.layers[l];
    if (misaligned16(Ly.down_qweight) || misaligned16(Ly.down_qzeros) || misaligned16(Ly.down_scales)) {
      misal = true, ok = false;
      return;
    }
    if (tid == 0) {   // rows [drow0, drow0 + drows) of column block db of the blocked down projection
      mbar_expect(&s_bar[2], block_bytes(drows, kBW, dg1 - dg0));
      load_block(C_w, C_z, C_s, Ly.down_qweight + ((size_t)db * I + drow0) * kBW,
                 Ly.down_qzeros + ((size_t)db * ngI + dg0) * kBW,
                 reinterpret_cast<const __half*>(Ly.down_scales) + ((size_t)db * ngI + dg0) * 8 * kBW, drows, kBW,
                 dg1 - dg0, &s_bar[2]);
    }
    armed[2] = true;
  };
  prefetchA(0);
  prefetchB(0);
  prefetchC(0);

  for (int l = 0; l < p.L && ok; ++l) {
    const anvilq_decode_layer& Ly = p.layers[l];
    const unsigned tag = tag_of(l), tag_prev = tag_of(l - 1);

    // ---- role A --------------------------------------------------------------
    if (!(ok = __syncthreads_and(wait_region(0)) != 0)) break;
    if (roleA == 1) {   // QKV head idxA: rmsnorm -> GEMV -> bias -> RoPE -> q / cache
      if (l > 0) {   // x_a and every down split of the previous layer: one trip
        if (!(ok = ll_gather(p, reinterpret_cast<uint32_t*>(stage),
                             ll_src(ll_run(p.ll_xa, H, tag_prev), ll_run(p.ll_dpart, H * p.nsplit, tag_prev)))))
          break;
        rmsnorm_to_smem(
            p, [&](int k) { return residual_sum(stage[k], stage + H + (k >> 5) * p.nsplit * 32, p.nsplit, k); },
            A_gamma, xs, misc);
      } else {
        rmsnorm_to_smem(p, [&](int k) { return __half2float(xemb[k]); }, A_gamma, xs, misc);
      }
      float* y = misc + kMiscY;
      bad |= D == 64 ? tile_gemv<8>(A_w, xs, A_z, A_s, H, 0, red, y) : tile_gemv<16>(A_w, xs, A_z, A_s, H, 0, red, y);
      const int head = idxA, hd = D / 2;
      const __half* bias = reinterpret_cast<const __half*>(Ly.qkv_bias);
      __half* hout = reinterpret_cast<__half*>(misc + kQkvOut);   // the head's D outputs
      for (int i = tid; i < hd; i += kThreads) {
        float va = y[i], vb = y[i + hd];
        if (bias) {
          va += __half2float(bias[head * D + i]);
          vb += __half2float(bias[head * D + i + hd]);
        }
        const __half ha = __float2half_rn(va), hb = __float2half_rn(vb);
        if (head < QH + KVH) {
          const float si = rope_sc[i], co = rope_sc[kMaxD / 2 + i];
          const float xa = __half2float(ha), xb = __half2float(hb);
          const float ra = __fsub_rn(__fmul_rn(xa, co), __fmul_rn(xb, si));
          const float rb = __fadd_rn(__fmul_rn(xb, co), __fmul_rn(xa, si));
          hout[i] = __float2half_rn(ra);
          hout[i + hd] = __float2half_rn(rb);
        } else {
          hout[i] = ha;
          hout[i + hd] = hb;
        }
      }
      __syncthreads();
      // hand on as tagged pairs; k and v also into the cache (plain stores, read by later launches)
      u64* dst = head < QH ? p.ll_q + (size_t)head * hd : p.ll_kv + (size_t)(head - QH) * hd;
      for (int w = tid; w < hd; w += kThreads) {
        const uint32_t pair = h2u(hout[2 * w], hout[2 * w + 1]);
        ll_put(dst + w, pair, tag);
        if (head >= QH) {
          const bool isv = head >= QH + KVH;
          __half* c = reinterpret_cast<__half*>(isv ? Ly.v_cache : Ly.k_cache) +
                      ((size_t)pos * KVH + (head - QH - (isv ? KVH : 0))) * D;
          reinterpret_cast<uint32_t*>(c)[w] = pair;
        }
      }
    } else if (att_on) {   // kv head ah, chunks [ac0, ac1): online softmax, unnormalised partial out
      const int h = ah;
      float* qs = misc + kAttQs;
      float* Pp = misc + kAttP;
      float* wmax = misc + kAttWmax;
      float* wsum = misc + kAttWsum;
      float* mbuf = misc + kAttM;
      float* lrun = misc + kAttL;
      uint32_t* raw = reinterpret_cast<uint32_t*>(misc + kAttRaw);   // q pairs, then k and v row pairs
      {   // q of the group and, for the unit holding this token's row, its k and v: one trip
        const int qw = grp * D / 2;                            // q words of the group
        const LLSeg q = ll_run(p.ll_q + (size_t)h * qw, qw, tag);
        // k row of head h, then its v row (the v rows follow the KVH k rows)
        const LLSeg kv{p.ll_kv + (size_t)h * (D / 2), 2, D / 4, KVH * (D / 2), tag};
        if (!(ok = ll_gather(p, raw, ac1 == nch ? ll_src(q, kv) : ll_src(q)))) break;
      }
      const float qscale = 1.4426950408889634f / sqrtf((float)D);   // log2(e) / sqrt(D)
      for (int i = tid; i < grp * D; i += kThreads)   // grp * D <= 1024
        qs[i] = __half2float(reinterpret_cast<const __half*>(raw)[i]) * qscale;
      if (tid < grp) {
        mbuf[tid] = -INFINITY;
        lrun[tid] = 0.0f;
      }
      const int lane = tid & 31, warp = tid >> 5;
      const int sj = warp >> 1, srh = warp & 1;                      // scores: head, row half
      const int pairs = D / 2, nrg = kThreads / pairs, rpg = kChunk / nrg;
      const int dp = tid % pairs, rg = tid / pairs;                  // PV: dim pair, row group
      float O[2] = {0.0f, 0.0f};
      for (int c = ac0; c < ac1; ++c) {
        const int t0 = c * kChunk, cnt = min(kChunk, T - t0), ci = c - ac0;
        if (c != ac0) {   // later chunks of the range: copied now
          __syncthreads();
          load_chunk(Ly, h, c, 3);
          if (!(ok = __syncthreads_and(wait_region(3)) != 0)) break;
        }
        if (pos >= t0 && pos < t0 + cnt) {   // this token's row, from the staged k and v pairs
          const uint4* kr = reinterpret_cast<const uint4*>(raw + grp * D / 2);
          for (int i = tid; i < D / 8; i += kThreads) {
            *reinterpret_cast<uint4*>(Kc + (pos - t0) * KS + 8 * i) = kr[i];
            *reinterpret_cast<uint4*>(Vc + (pos - t0) * KS + 8 * i) = kr[D / 8 + i];
          }
        }
        __syncthreads();
        // scores: warp (head sj, rows srh*32 + lane); 16-byte K loads, q broadcast
        const int r = srh * 32 + lane;
        float sc = -INFINITY;
        if (sj < grp) {
          if (r < cnt) {
            const __half* kr = Kc + r * KS;
            const float* qj = qs + sj * D;
            float acc = 0.0f;
            for (int d = 0; d < D; d += 8) {
              const uint4 kv = *reinterpret_cast<const uint4*>(kr + d);
              const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 k2 = __half22float2(h2(kw[e]));
                acc = fmaf(qj[d + 2 * e], k2.x, acc);
                acc = fmaf(qj[d + 2 * e + 1], k2.y, acc);
              }
            }
            sc = acc;
          }
          float m = sc;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0) wmax[2 * sj + srh] = m;
        }
        __syncthreads();
        float* mold = mbuf + (ci & 1) * kMaxGroup;
        float* mnew = mbuf + ((ci + 1) & 1) * kMaxGroup;
        if (sj < grp) {
          const float mn = fmaxf(mold[sj], fmaxf(wmax[2 * sj], wmax[2 * sj + 1]));
          const float pr = r < cnt ? exp2f(sc - mn) : 0.0f;
          Pp[sj * kChunk + r] = pr;
          float s = pr;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
          if (lane == 0) {
            wsum[2 * sj + srh] = s;
            if (srh == 0) mnew[sj] = mn;
          }
        }
        __syncthreads();
        // P V: thread (row group rg, dims 2 dp, 2 dp + 1) over its rows, all heads
        float acc[kMaxGroup][2];
#pragma unroll
        for (int j = 0; j < kMaxGroup; ++j) acc[j][0] = acc[j][1] = 0.0f;
        for (int i = 0; i < rpg; ++i) {
          const int rr = rg * rpg + i;
          if (rr < cnt) {
            const float2 v2 = __half22float2(*reinterpret_cast<const half2*>(Vc + rr * KS + 2 * dp));
#pragma unroll
            for (int j = 0; j < kMaxGroup; ++j)
              if (j < grp) {
                const float pj = Pp[j * kChunk + rr];
                acc[j][0] = fmaf(pj, v2.x, acc[j][0]);
                acc[j][1] = fmaf(pj, v2.y, acc[j][1]);
              }
          }
        }
#pragma unroll
        for (int j = 0; j < kMaxGroup; ++j)
          if (j < grp)
            *reinterpret_cast<float2*>(stage + (rg * grp + j) * D + 2 * dp) = make_float2(acc[j][0], acc[j][1]);
        __syncthreads();
        {   // (head, dim) pairs tid and tid + 512 (grp * D <= 1024), two chains
          const int i0 = tid, i1 = min(tid + kThreads, grp * D - 1);
          const int j0 = i0 / D, j1 = i1 / D;
          const float* s0 = stage + j0 * D + i0 % D;
          const float* s1 = stage + j1 * D + i1 % D;
          float a0 = 0.0f, a1 = 0.0f;
          for (int g2 = 0; g2 < nrg; ++g2) {   // in row-group order
            a0 += s0[g2 * grp * D];
            a1 += s1[g2 * grp * D];
          }
          if (i0 < grp * D) O[0] = fmaf(O[0], exp2f(mold[j0] - mnew[j0]), a0);
          if (tid + kThreads < grp * D) O[1] = fmaf(O[1], exp2f(mold[j1] - mnew[j1]), a1);
        }
        if (tid < grp) lrun[tid] = fmaf(lrun[tid], exp2f(mold[tid] - mnew[tid]), wsum[2 * tid] + wsum[2 * tid + 1]);
      }
      if (!ok) break;
      const float* mfin = mbuf + ((ac1 - ac0) & 1) * kMaxGroup;
      u64* part_out = p.ll_apart + (size_t)(h * p.nu_max + au) * p.perP;
      for (int k = 0; k < 2; ++k) {
        const int i = tid + k * kThreads;
        if (i < grp * D) ll_put(part_out + (i / D) * (D + 2) + 2 + i % D, __float_as_uint(O[k]), tag);
      }
      if (tid < grp) {
        ll_put(part_out + tid * (D + 2), __float_as_uint(mfin[tid]), tag);
        ll_put(part_out + tid * (D + 2) + 1, __float_as_uint(lrun[tid]), tag);
      }
      for (int i = grp * (D + 2) + tid; i < p.perP; i += kThreads) ll_put(part_out + i, 0u, tag);   // padding words
    } else if (roleA == 3) {   // O block idxA: merge the partials, x_a = x + attn W_o
      const int per = p.perP, unit = nu * per, n = KVH * unit;   // words; per % 4 == 0
      float* ew = misc + kMiscBig;      // [QH][nu] merge weights
      float* Ls = ew + QH * nu;         // [QH]
      // every unit's (m, l, o), then this block's x_a and down splits: one trip
      const LLSeg parts{p.ll_apart, KVH, unit / 2, p.nu_max * per, tag};
      const LLSeg xblk = ll_run(p.ll_xa + idxA * 32, 32, tag_prev);
      const LLSeg dblk = ll_run(p.ll_dpart + (size_t)idxA * p.nsplit * 32, 32 * p.nsplit, tag_prev);
      if (!(ok = ll_gather(p, reinterpret_cast<uint32_t*>(stage), l > 0 ? ll_src(parts, xblk, dblk) : ll_src(parts))))
        break;
      // per q head: M = max m_u, e_u = 2^(m_u - M), L = sum l_u e_u (warp per head, lane per unit)
      const int lane = tid & 31, warp = tid >> 5;
      for (int jj = warp; jj < QH; jj += kWarps) {
        const float* pc = stage + (size_t)(jj / grp) * unit + min(lane, nu - 1) * per + (jj % grp) * (D + 2);
        const float m = lane < nu ? pc[0] : -INFINITY;
        float M = m;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float e = lane < nu ? exp2f(m - M) : 0.0f;
        float s = lane < nu ? pc[1] * e : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane < nu) ew[jj * nu + lane] = e;
        if (lane == 0) Ls[jj] = s;
      }
      __syncthreads();
      for (int i0 = tid; i0 < QH * D; i0 += 2 * kThreads) {   // two independent chains a thread
        const int i1 = min(i0 + kThreads, QH * D - 1), j0 = i0 / D, j1 = i1 / D;
        const float* pc0 = stage + (size_t)(j0 / grp) * unit + (j0 % grp) * (D + 2) + 2 + i0 % D;
        const float* pc1 = stage + (size_t)(j1 / grp) * unit + (j1 % grp) * (D + 2) + 2 + i1 % D;
        float a0 = 0.0f, a1 = 0.0f;
        for (int u = 0; u < nu; ++u) {   // in unit order
          a0 = fmaf(ew[j0 * nu + u], pc0[u * per], a0);
          a1 = fmaf(ew[j1 * nu + u], pc1[u * per], a1);
        }
        xs[i0] = __float2half_rn(a0 / Ls[j0]);
        if (i0 + kThreads < QH * D) xs[i1] = __float2half_rn(a1 / Ls[j1]);
      }
      __syncthreads();
      float* y = misc + kMiscY;
      bad |= tile_gemv<kBW>(A_w, xs, A_z, A_s, QH * D, 0, red, y);
      if (tid < 32) {
        const int k = idxA * 32 + tid;
        const float x = l > 0 ? residual_sum(stage[n + tid], stage + n + 32, p.nsplit, k) : __half2float(xemb[k]);
        ll_put(p.ll_xa + k, __float_as_uint(x + y[tid]), tag);
      }
    }
    __syncthreads();
    if (l + 1 < p.L) prefetchA(l + 1);

    // ---- role B: gate/up -----------------------------------------------------
    if (!(ok = ok && __syncthreads_and(wait_region(1)) != 0)) break;
    if (gu0 >= 0) {
      if (!(ok = ok && ll_gather(p, reinterpret_cast<uint32_t*>(bst), ll_src(ll_run(p.ll_xa, H, tag))))) break;
      rmsnorm_to_smem(p, [&](int k) { return bst[k]; }, B_gamma, xs, misc);
      for (int sl = 0; sl < 2; ++sl) {
        const int u = sl == 0 ? gu0 : gu1;
        if (u < 0) continue;
        float* g = misc + kMiscY;   // g[0:32] gate, g[32:64] up
        __half* act = reinterpret_cast<__half*>(misc + kMiscAct);
        uint32_t* w = gu_w(sl);
        bad |= tile_gemv<kGU>(w, xs, w + H * kGU, w + H * kGU + ngH * kGU, H, 0, red, g);
        if (tid < 32) {
          const float gh = __half2float(__float2half_rn(g[tid])), uh = __half2float(__float2half_rn(g[32 + tid]));
          const float e = expf(-fabsf(gh));   // stable silu (official_weights.py:494-499)
          const float sg = gh >= 0.0f ? gh / (1.0f + e) : (gh * e) / (1.0f + e);
          act[tid] = __float2half_rn(sg * uh);
        }
        __syncthreads();
        if (tid < 16) ll_put(p.ll_act + u * 16 + tid, h2u(act[2 * tid], act[2 * tid + 1]), tag);
      }
    }
    __syncthreads();
    if (l + 1 < p.L) prefetchB(l + 1);

    // ---- role C: down split --------------------------------------------------
    if (!(ok = ok && __syncthreads_and(wait_region(2)) != 0)) break;
    if (has_down) {   // the act rows of this split, staged as the GEMV's binary16 x
      if (!(ok = ok && ll_gather(p, reinterpret_cast<uint32_t*>(xs), ll_src(ll_run(p.ll_act + drow0 / 2, drows / 2, tag)))))
        break;
      float* y = misc + kMiscY;
      bad |= tile_gemv<kBW>(C_w, xs, C_z, C_s, drows, drow0, red, y);
      if (tid < 32) ll_put(p.ll_dpart + ((size_t)db * p.nsplit + ds) * 32 + tid, __float_as_uint(y[tid]), tag);
    }
    __syncthreads();
    if (l + 1 < p.L) prefetchC(l + 1);
  }
  for (int r = 0; r < 4; ++r) wait_region(r);   // copies still in flight land before the CTA exits (bounded)
  if (!ok && tid == 0) {   // a misaligned tensor, a wait that expired, or another CTA gave up
    if (misal && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_ALIGN);
    atomicExch(p.abort_flag, 1);
  }
  // ---- the residual after the last layer: column block cta ---------------------
  if (ok && cta < nb) {
    float* st = misc + kMiscBig;
    const unsigned tl = tag_of(p.L - 1);
    if (ll_gather(p, reinterpret_cast<uint32_t*>(st),
                  ll_src(ll_run(p.ll_xa + cta * 32, 32, tl), ll_run(p.ll_dpart + (size_t)cta * p.nsplit * 32,
                                                                     32 * p.nsplit, tl))) &&
        tid < 32)
      p.x_out[cta * 32 + tid] = residual_sum(st[tid], st + 32, p.nsplit, tid);
  }
  if (bad && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SCALE);

  // ---- exit: the last CTA out advances the launch count and re-arms the flags --
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    __shared__ int s_exit;
    s_exit = atomicAdd(p.exit_ctr, 1) == P - 1;
    if (s_exit) {
      __threadfence();
      *p.seq = seq + 1u;
      *p.abort_flag = 0;
      __threadfence();
      *p.exit_ctr = 0;
    }
  }
}

// ---------------------------------------------------------------------------
struct Plan {
  int P, n1, n2, n3, nsplit, nu_max, perP, gx;
  int offA, offB, offC, offX, offRed, offMisc, offBst, offStage, smem;
  size_t ws_bytes;
  size_t off_exit, off_abort, off_seq, off_xa, off_dpart, off_q, off_kv, off_apart, off_act;
};

constexpr int kMaxDevices = 64;
static int g_sms[kMaxDevices];
static std::once_flag g_once[kMaxDevices];

static int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  std::call_once(g_once[dev], [dev] {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sms[dev] = n;
  });
  return g_sms[dev];
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
constexpr size_t kSmemLimit = 220 * 1024;

// ANVILQ_OK and the plan, or the status that rejects the shape.
static int make_plan(int L, int H, int I, int QH, int KVH, int D, int G, int Tmax, Plan* pl) {
  if (L < 1 || H < 128 || I < 128 || QH < 1 || KVH < 1 || Tmax < 1) return ANVILQ_EINVAL;
  if (G != kG || H % kG || I % kG || QH % KVH || QH / KVH > kMaxGroup || (D != 64 && D != 128) ||
      (QH * D) % kG || H > kThreads * kMaxPerThread)
    return ANVILQ_ESHAPE;
  const int P = sm_count();
  if (P <= 0) return ANVILQ_ECUDA;
  pl->P = P;
  const int nb = H / 32, ngI = I / kG, ngH = H / kG, grp = QH / KVH, n_gu = I / 32;
  pl->n1 = QH + 2 * KVH;
  pl->n3 = nb;
  pl->nsplit = std::min(std::min(P / nb, ngI), kMaxSplit);
  if (pl->nsplit < 1 || n_gu > 2 * P || pl->n1 + pl->n3 + KVH > P) return ANVILQ_ESHAPE;
  // the rows of the units beyond P form the last down split alone, when every
  // other split keeps at least one group
  const int gx = (P * 32) / kG;
  pl->gx = n_gu > P && pl->nsplit >= 2 && gx >= pl->nsplit - 1 && gx < ngI ? gx : 0;
  int maxdg = 0;
  for (int s = 0; s < pl->nsplit; ++s) {
    int g0 = 0, g1 = 0;
    down_split(s, pl->nsplit, ngI, pl->gx, &g0, &g1);
    maxdg = std::max(maxdg, g1 - g0);
  }
  // shared memory other than region A
  const size_t guTile = ((size_t)H * kGU + ngH * kGU + ngH * 4 * kGU) * 4;
  const size_t regB = align_up(2 * guTile + (size_t)H * 2, 128);
  const size_t regC = align_up((size_t)maxdg * kG * kBW * 4 + maxdg * kBW * 4 + maxdg * 32 * 2, 128);
  const size_t xsB = align_up((size_t)std::max(std::max(H, QH * D), maxdg * kG) * 2, 128);
  const size_t redB = align_up((size_t)kWarps * 8 * 16 * 4, 128);
  const size_t bstB = align_up((size_t)H * 4, 128);
  // region A: the role's tile (QKV head + gamma, attention chunk, O block),
  // then from offStage the role's staged inputs (QKV: x_a and the down splits;
  // O: the partials of every unit, x_a and the splits of its block) or the
  // attention's P V sums
  const size_t qkvA = align_up((size_t)H * (D / 8) * 4 + ngH * (D / 8) * 4 + ngH * D * 2 + (size_t)H * 2, 128);
  const size_t attKV = align_up((size_t)2 * kChunk * kv_stride(D) * 2, 128);
  const size_t attPV = (size_t)kThreads * 2 * grp * 4;          // [512 / (D/2)][grp][D] floats
  const size_t oW = align_up((size_t)QH * D * kBW * 4 + (QH * D / kG) * kBW * 4 + (QH * D / kG) * 32 * 2, 128);
  const int perP = (grp * (D + 2) + 3) / 4 * 4;
  const size_t unitB = (size_t)KVH * perP * 4;                   // staged bytes per unit index
  const size_t offStage = std::max(qkvA, std::max(attKV, oW));
  const size_t qkvStage = (size_t)H * (pl->nsplit + 1) * 4, oRes = (size_t)32 * (pl->nsplit + 1) * 4;
  const size_t fixed = regB + regC + xsB + redB + bstB;
  auto regA_bytes = [&](int u) {
    return align_up(offStage + std::max(std::max(qkvStage, attPV), (size_t)u * unitB + oRes), 128);
  };
  auto misc_bytes = [&](int u) {   // the largest role's part, and the final residual's staging
    const int big = std::max(std::max(kAttEnd, kQkvOut + kMaxD / 2),
                             std::max(kMiscBig + QH * (u + 1), kMiscBig + 32 * (kMaxSplit + 1)));
    return align_up((size_t)big * 4, 128);
  };
  // units per kv head: the spare CTAs, at most one per chunk, and what region A can stage
  int nu = std::min((P - pl->n1 - pl->n3) / KVH, std::min(kMaxUnits, (Tmax + kChunk - 1) / kChunk));
  while (nu > 1 && regA_bytes(nu) + fixed + misc_bytes(nu) > kSmemLimit) --nu;
  if (nu < 1 || regA_bytes(nu) + fixed + misc_bytes(nu) > kSmemLimit) return ANVILQ_ESHAPE;   // must fit one SM
  pl->nu_max = nu;
  pl->perP = perP;
  pl->n2 = KVH * nu;
  const size_t regA = regA_bytes(nu);
  pl->offA = 0;
  pl->offStage = (int)offStage;
  pl->offB = (int)regA;
  pl->offC = (int)(regA + regB);
  pl->offX = (int)(regA + regB + regC);
  pl->offRed = pl->offX + (int)xsB;
  pl->offBst = pl->offRed + (int)redB;
  pl->offMisc = pl->offBst + (int)bstB;
  pl->smem = pl->offMisc + (int)misc_bytes(nu);
  // workspace
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  pl->off_exit = take(4);
  pl->off_abort = take(4);
  pl->off_seq = take(4);
  pl->off_xa = take((size_t)H * 8);
  pl->off_dpart = take((size_t)nb * pl->nsplit * 32 * 8);
  pl->off_q = take((size_t)QH * D / 2 * 8);
  pl->off_kv = take((size_t)KVH * D * 8);
  pl->off_apart = take((size_t)KVH * nu * perP * 8);
  pl->off_act = take((size_t)I / 2 * 8);
  pl->ws_bytes = o;
  return ANVILQ_OK;
}

}  // namespace dstep
}  // namespace anvilq

using namespace anvilq::dstep;

extern "C" size_t anvilq_decode_layers_workspace_size(int L, int H, int I, int QH, int KVH, int D, int G, int Tmax) {
  Plan pl;
  return make_plan(L, H, I, QH, KVH, D, G, Tmax, &pl) == ANVILQ_OK ? pl.ws_bytes : 0;
}

extern "C" int anvilq_decode_layers(const anvilq_decode_layer* layers, int L, int H, int I, int QH, int KVH, int D,
                                    int G, int Tmax, float eps, float theta, const uint16_t* embedding, int V,
                                    const int32_t* token, const int32_t* pos, int32_t* seqlen, float* x_out,
                                    unsigned long long* argmax_key, void* workspace, size_t workspace_bytes,
                                    int* dev_err, anvilq_stream_t stream) {
  if (!layers || !embedding || !token || !pos || !x_out || V < 1 || !(eps >= 0.0f) || !(theta > 0.0f))
    return ANVILQ_EINVAL;
  Plan pl;
  const int rc = make_plan(L, H, I, QH, KVH, D, G, Tmax, &pl);
  if (rc != ANVILQ_OK) return rc;
  if (!workspace || workspace_bytes < pl.ws_bytes) return ANVILQ_EWORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) || (reinterpret_cast<uintptr_t>(embedding) & 15u))
    return ANVILQ_EALIGN;
  Params p{};
  p.layers = layers;
  p.L = L; p.H = H; p.I = I; p.QH = QH; p.KVH = KVH; p.D = D; p.Tmax = Tmax; p.V = V;
  p.eps = eps;
  p.emb = reinterpret_cast<const __half*>(embedding);
  p.token = token;
  p.pos = pos;
  p.seqlen = seqlen;
  p.x_out = x_out;
  p.key = argmax_key;
  p.dev_err = dev_err;
  char* w = static_cast<char*>(workspace);
  p.exit_ctr = reinterpret_cast<int*>(w + pl.off_exit);
  p.abort_flag = reinterpret_cast<int*>(w + pl.off_abort);
  p.seq = reinterpret_cast<unsigned*>(w + pl.off_seq);
  p.ll_xa = reinterpret_cast<u64*>(w + pl.off_xa);
  p.ll_dpart = reinterpret_cast<u64*>(w + pl.off_dpart);
  p.ll_q = reinterpret_cast<u64*>(w + pl.off_q);
  p.ll_kv = reinterpret_cast<u64*>(w + pl.off_kv);
  p.ll_apart = reinterpret_cast<u64*>(w + pl.off_apart);
  p.ll_act = reinterpret_cast<u64*>(w + pl.off_act);
  p.n1 = pl.n1; p.n2 = pl.n2; p.n3 = pl.n3; p.nsplit = pl.nsplit; p.nu_max = pl.nu_max; p.perP = pl.perP;
  p.gx = pl.gx;
  p.offA = pl.offA; p.offB = pl.offB; p.offC = pl.offC; p.offX = pl.offX; p.offRed = pl.offRed;
  p.offMisc = pl.offMisc; p.offBst = pl.offBst; p.offStage = pl.offStage; p.smem = pl.smem;
  for (int i = 0; i < D / 2; ++i) p.rope_inv[i] = std::pow((double)theta, -2.0 * i / D);

  if (cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem) != cudaSuccess) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.P, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;   // every CTA resident at once (they wait on one another)
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, decode_step_kernel, p) != cudaSuccess) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  return ANVILQ_OK;
}

extern "C" int anvilq_block_columns(const void* src, void* dst, int rows, int cols, int block, int elem_bytes,
                                    anvilq_stream_t stream) {
  if (!src || !dst || rows < 1 || cols < 1 || block < 1 || (elem_bytes != 2 && elem_bytes != 4)) return ANVILQ_EINVAL;
  if (cols % block || (block * elem_bytes) % 16) return ANVILQ_ESHAPE;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) return ANVILQ_EALIGN;
  const long long row_vecs = (long long)cols * elem_bytes / 16, block_vecs = (long long)block * elem_bytes / 16;
  const long long n = (long long)rows * row_vecs;
  const int threads = 256;
  const long long blocks = std::min<long long>((n + threads - 1) / threads, 1 << 20);
  block_columns_kernel<<<(unsigned)blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), rows, row_vecs, block_vecs);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}
