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
// ~22 us: every launch pays its ramp and tail.  Here the five phases of a layer
// are roles that CTAs take, and a phase starts when the counter its producers
// increment reaches the number of producers (release / acquire at GPU scope,
// bounded waits).  No CTA waits for CTAs that do not produce its input.
//
// Weights stream ahead.  Each CTA's slice of a phase's weights (int4 words,
// zeros, scales) and, for attention, its chunk of the KV cache up to the
// previous position, are copied into shared memory with cp.async as soon as
// the CTA has finished the same phase of the previous layer: a whole layer of
// lead time, so the copies never sit on the critical path.  Three groups are
// in flight per CTA (roles A = QKV or attention or O, B = gate/up, C = down).
//
// Work per layer (P = #CTAs, 512 threads each):
//   QKV   one head (D columns, all H rows) per CTA: RoPE and the K / V cache
//         append need both halves of a head, so the head is the unit.
//   attn  (kv head, 64-token chunk) per CTA: fp32 scores and softmax over the
//         chunk; the CTA arriving last at its kv head's ticket merges the
//         chunks in chunk order.
//   O     32 output columns (4 qweight words) per CTA; residual added.
//   g/u   32 intermediate columns of gate AND of up per CTA, so silu(g) u is
//         formed locally; I / 32 units over P CTAs.
//   down  32 output columns x a split of the groups of K = I per CTA; the last
//         split to arrive at the block's ticket adds the splits in order and
//         writes the layer's residual.
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

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kG = 128;            // AWQ group (rows)
constexpr int kBW = 4;             // words of an O / gate-up / down unit (32 columns)
constexpr int kChunk = 64;         // attention tokens per unit
constexpr int kPhases = 5;
constexpr int kMaxGroup = 8;       // q heads per kv head
constexpr int kMaxD = 128;
constexpr unsigned long long kWaitNs = 1000000000ull;

struct Params {
  const anvilq_decode_layer* layers;
  int L, H, I, QH, KVH, D, Tmax, V;
  float eps;
  const __half* emb;
  const int* token;
  const int* pos;
  int* seqlen;
  float* x_out;
  unsigned long long* key;
  int* dev_err;
  // workspace
  float* xbuf;      // [2][H] residual after each layer (ping-pong)
  float* xa;        // [H] residual after attention
  __half* q;        // [QH * D] rotated q
  float* apart;     // [KVH][maxch][group][D + 2] attention chunk partials (m, l, o)
  __half* attn;     // [QH * D] attention output
  __half* act;      // [I] silu(g) u
  float* dpart;     // [H / 32][nsplit][32] down partials
  int* ctr;         // [L][kPhases] producer counters
  int* aticket;     // [L][KVH]
  int* dticket;     // [L][H / 32]
  int* exit_ctr;    // [1]
  int* abort_flag;  // [1]
  // roles: A = QKV heads [0, n1), attention [n1, n1 + n2), O blocks [n1 + n2, n1 + n2 + n3)
  int n1, n2, n3, nsplit, maxch;
  // shared-memory carve-up (bytes)
  int offA, offB, offC, offX, offRed, offMisc, smem;
  int regA_bytes;
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
__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait2() { asm volatile("cp.async.wait_group 2;" ::: "memory"); }
__device__ __forceinline__ void cp_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ half2 h2(uint32_t u) { return *reinterpret_cast<half2*>(&u); }
__device__ __forceinline__ void fma_f32_f16x2(float& a0, float& a1, uint32_t q2, unsigned short x) {
  asm("{\n .reg .f16 q0, q1;\n mov.b32 {q0, q1}, %2;\n"
      " fma.rn.f32.f16 %0, %3, q0, %0;\n fma.rn.f32.f16 %1, %3, q1, %1;\n}"
      : "+f"(a0), "+f"(a1)
      : "r"(q2), "h"(x));
}

// Block until *ctr >= target (thread 0 polls, the CTA follows); false when the
// wait expired (~1 s) or another CTA already gave up: the launch then aborts.
__device__ bool wait_count(const Params& p, const int* ctr, int target) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    if (ld_acquire(ctr) < target) {
      const unsigned long long t0 = globaltimer();
      for (uint32_t i = 0;; ++i) {
        if (ld_acquire(ctr) >= target) break;
        if ((i & 63u) == 63u && (globaltimer() - t0 > kWaitNs || ld_acquire(p.abort_flag))) {
          ok = 0;
          if (p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
          atomicExch(p.abort_flag, 1);
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}
// every thread's stores of this phase are visible at GPU scope, then the counter
// moves: the barrier orders the CTA's stores before thread 0's fence (cumulative)
__device__ void publish(int* ctr, int n) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(ctr, n);
  }
}

// this CTA's stores so far visible, then a ticket; true for the last arriver
// (whose loads after the call see every other arriver's stores)
__device__ bool last_arrival(int* ticket, int arrivals) {
  __shared__ int s_last_arrival;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const bool last = atomicAdd(ticket, 1) == arrivals - 1;
    if (last) __threadfence();
    s_last_arrival = last;
  }
  __syncthreads();
  return s_last_arrival != 0;
}

// dst[0:n] = src[0:n] (L2-coherent loads), 8 loads in flight per thread
__device__ void stage_floats(float* dst, const float* src, int n) {
  for (int i0 = threadIdx.x; i0 < n; i0 += 8 * kThreads) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = i0 + u * kThreads < n ? __ldcg(src + i0 + u * kThreads) : 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (i0 + u * kThreads < n) dst[i0 + u * kThreads] = v[u];
  }
}

// Copy one column block of a projection (see anvilq_block_columns): `rows`
// rows of `words` int4 words, then the zeros [ng][words] and the scales
// [ng][8 words] (binary16) of its ng groups -- three contiguous ranges, so the
// 16-byte copies of consecutive threads are consecutive in memory.
__device__ void prefetch_block(uint32_t* wdst, uint32_t* zdst, uint32_t* sdst, const int32_t* wsrc,
                               const int32_t* zsrc, const __half* ssrc, int rows, int words, int ng) {
  const int nw = rows * words / 4, nz = ng * words / 4, ns = ng * words;
  for (int i = threadIdx.x; i < nw; i += kThreads) cp16(wdst + 4 * i, wsrc + 4 * i);
  for (int i = threadIdx.x; i < nz; i += kThreads) cp16(zdst + 4 * i, zsrc + 4 * i);
  for (int i = threadIdx.x; i < ns; i += kThreads) cp16(sdst + 4 * i, ssrc + 8 * i);
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
// the warp by shuffles and across warps in warp order.  `red` holds
// kWarps x 8 W floats.  Returns nonzero if a scale of the tile was invalid.
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
  if (t < 8 * W) {
    float v = 0.0f;
    for (int w = 0; w < kWarps; ++w) v += red[w * 8 * W + t];   // in warp order
    out[t] = v;
  }
  __syncthreads();
  return bad;
}

// x_norm[k] = fp16(x[k] * gamma[k] / sqrt(mean(x^2) + eps)) into shared memory.
// x: the residual (fp32, L2-coherent loads) or, for layer 0, the embedding row.
// One pass over x: every thread keeps its (at most kMaxPerThread) values.
constexpr int kMaxPerThread = 8;   // H <= 4096
__device__ void rmsnorm_to_smem(const Params& p, const float* x, const __half* xemb, const __half* gamma,
                                __half* xs, float* misc) {
  float v[kMaxPerThread];
  float ss = 0.0f;
#pragma unroll
  for (int u = 0; u < kMaxPerThread; ++u) {
    const int k = threadIdx.x + u * kThreads;
    v[u] = k < p.H ? (x ? __ldcg(x + k) : __half2float(xemb[k])) : 0.0f;
  }
#pragma unroll
  for (int u = 0; u < kMaxPerThread; ++u) ss = fmaf(v[u], v[u], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) misc[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int w = 0; w < kWarps; ++w) t += misc[w];
    misc[kWarps] = 1.0f / sqrtf(t / (float)p.H + p.eps);
  }
  __syncthreads();
  const float inv = misc[kWarps];
#pragma unroll
  for (int u = 0; u < kMaxPerThread; ++u) {
    const int k = threadIdx.x + u * kThreads;
    if (k < p.H) xs[k] = __float2half_rn(v[u] * __half2float(gamma[k]) * inv);
  }
  __syncthreads();
}

// sizes of the role-A shared-memory tiles
__device__ __host__ inline int a_words(int D) { return D / 8; }

__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int cta = blockIdx.x, P = gridDim.x, tid = threadIdx.x;
  unsigned char* regA = smem + p.offA;
  unsigned char* regB = smem + p.offB;
  unsigned char* regC = smem + p.offC;
  __half* xs = reinterpret_cast<__half*>(smem + p.offX);
  float* red = reinterpret_cast<float*>(smem + p.offRed);
  float* misc = reinterpret_cast<float*>(smem + p.offMisc);
  const int H = p.H, I = p.I, QH = p.QH, KVH = p.KVH, D = p.D, grp = QH / KVH;
  const int nb = H / 32;                  // 32-column blocks of H
  const int n_gu = I / 32;                // gate/up units
  const int ngI = I / kG;                 // groups of K = I
  uint32_t bad = 0;

  int pos = *p.pos;
  int token = *p.token;
  if (pos < 0 || pos >= p.Tmax || token < 0 || token >= p.V) {
    if (cta == 0 && tid == 0 && p.dev_err)
      atomicOr(p.dev_err, pos < 0 || pos >= p.Tmax ? ANVILQ_DEV_ERR_SEQLEN : ANVILQ_DEV_ERR_TOKEN);
    return;   // every CTA returns here alike: nothing was counted
  }
  const int T = pos + 1;                  // attention length
  const int nch = (T + kChunk - 1) / kChunk;
  const __half* xemb = p.emb + (size_t)token * H;
  if (cta == 0 && tid == 0) {
    if (p.seqlen) *p.seqlen = T;
    if (p.key) *p.key = 0ull;
  }

  // ---- roles of this CTA --------------------------------------------------
  const int roleA = cta < p.n1 ? 1 : cta < p.n1 + p.n2 ? 2 : cta < p.n1 + p.n2 + p.n3 ? 3 : 0;
  const int idxA = roleA == 1 ? cta : roleA == 2 ? cta - p.n1 : cta - p.n1 - p.n2;
  const int gu0 = cta, gu1 = cta + P < n_gu ? cta + P : -1;        // gate/up units
  const bool has_down = cta < nb * p.nsplit;
  const int db = cta / p.nsplit, ds = cta % p.nsplit;              // down block and split
  const int dg0 = ds * ngI / p.nsplit, dg1 = (ds + 1) * ngI / p.nsplit;
  const int drow0 = dg0 * kG, drows = (dg1 - dg0) * kG;

  // role-A tile layout (QKV head / attention chunk / O block)
  const int wA = roleA == 1 ? a_words(D) : kBW;
  const int rowsA = roleA == 1 ? H : QH * D;
  uint32_t* A_w = reinterpret_cast<uint32_t*>(regA);
  uint32_t* A_z = A_w + rowsA * wA;
  uint32_t* A_s = A_z + ((rowsA + kG - 1) / kG) * wA;
  __half* Kc = reinterpret_cast<__half*>(regA);                   // attention: [64][D]
  __half* Vc = Kc + kChunk * D;
  // gate/up: two units of (gate, up) tiles, each [H][4] + zeros + scales
  const int guTile = H * kBW + (H / kG) * kBW + (H / kG) * 4 * kBW;   // uint32 per tile
  auto gu_w = [&](int slot, int which) { return reinterpret_cast<uint32_t*>(regB) + (2 * slot + which) * guTile; };
  uint32_t* C_w = reinterpret_cast<uint32_t*>(regC);
  uint32_t* C_z = C_w + drows * kBW;
  uint32_t* C_s = C_z + (drows / kG) * kBW;

  auto prefetchA = [&](int l) {
    const anvilq_decode_layer& Ly = p.layers[l];
    if (roleA == 1) {   // column block idxA (one head) of the blocked QKV projection
      const int wd = a_words(D), ng = H / kG;
      prefetch_block(A_w, A_z, A_s, Ly.qkv_qweight + (size_t)idxA * H * wd, Ly.qkv_qzeros + (size_t)idxA * ng * wd,
                     reinterpret_cast<const __half*>(Ly.qkv_scales) + (size_t)idxA * ng * 8 * wd, H, wd, ng);
    } else if (roleA == 2) {
      // the first chunk this CTA owns: rows before the current position only
      const int u = idxA;
      if (u < KVH * nch) {
        const int h = u % KVH, c = u / KVH, t0 = c * kChunk, cnt = min(kChunk, T - t0);
        const int d8 = D / 8;
        const __half* kc = reinterpret_cast<const __half*>(Ly.k_cache);
        const __half* vc = reinterpret_cast<const __half*>(Ly.v_cache);
        for (int i = tid; i < cnt * d8; i += kThreads) {
          const int r = i / d8, c8 = i % d8, tok = t0 + r;
          if (tok == pos) continue;   // written by this token's QKV phase; read after it
          const size_t off = ((size_t)tok * KVH + h) * D + 8 * c8;
          cp16(Kc + r * D + 8 * c8, kc + off);
          cp16(Vc + r * D + 8 * c8, vc + off);
        }
      }
    } else if (roleA == 3) {   // column block idxA of the blocked O projection
      const int K = QH * D, ng = K / kG;
      prefetch_block(A_w, A_z, A_s, Ly.o_qweight + (size_t)idxA * K * kBW, Ly.o_qzeros + (size_t)idxA * ng * kBW,
                     reinterpret_cast<const __half*>(Ly.o_scales) + (size_t)idxA * ng * 8 * kBW, K, kBW, ng);
    }
    cp_commit();
  };
  auto prefetchB = [&](int l) {
    const anvilq_decode_layer& Ly = p.layers[l];
    const int units[2] = {gu0, gu1};
    for (int sl = 0; sl < 2; ++sl) {
      const int u = units[sl];
      if (u < 0 || u >= n_gu) continue;
      for (int which = 0; which < 2; ++which) {   // column blocks u (gate) and I / 32 + u (up)
        uint32_t* w = gu_w(sl, which);
        const size_t b = (size_t)(which ? n_gu : 0) + u;
        const int ng = H / kG;
        prefetch_block(w, w + H * kBW, w + H * kBW + ng * kBW, Ly.gu_qweight + b * H * kBW,
                       Ly.gu_qzeros + b * ng * kBW, reinterpret_cast<const __half*>(Ly.gu_scales) + b * ng * 8 * kBW,
                       H, kBW, ng);
      }
    }
    cp_commit();
  };
  auto prefetchC = [&](int l) {
    if (has_down) {
      const anvilq_decode_layer& Ly = p.layers[l];
      // rows [drow0, drow0 + drows) of column block db of the blocked down projection
      prefetch_block(C_w, C_z, C_s, Ly.down_qweight + ((size_t)db * I + drow0) * kBW,
                     Ly.down_qzeros + ((size_t)db * ngI + dg0) * kBW,
                     reinterpret_cast<const __half*>(Ly.down_scales) + ((size_t)db * ngI + dg0) * 8 * kBW, drows, kBW,
                     dg1 - dg0);
    }
    cp_commit();
  };
  prefetchA(0);
  prefetchB(0);
  prefetchC(0);

  bool ok = true;
  for (int l = 0; l < p.L && ok; ++l) {
    const anvilq_decode_layer& Ly = p.layers[l];
    int* ctr = p.ctr + l * kPhases;
    const float* x_in = l == 0 ? nullptr : p.xbuf + (l & 1) * H;   // null: the embedding row
    float* x_next = l == p.L - 1 ? p.x_out : p.xbuf + ((l + 1) & 1) * H;

    // ---- role A --------------------------------------------------------------
    cp_wait2();
    __syncthreads();
    if (roleA == 1) {   // QKV head idxA: rmsnorm -> GEMV -> bias -> RoPE -> q / cache
      if (l > 0 && !(ok = wait_count(p, p.ctr + (l - 1) * kPhases + 4, nb))) break;
      rmsnorm_to_smem(p, x_in, xemb, reinterpret_cast<const __half*>(Ly.gamma_in), xs, misc);
      float* y = misc + 32;
      bad |= D == 64 ? tile_gemv<8>(A_w, xs, A_z, A_s, H, 0, red, y) : tile_gemv<16>(A_w, xs, A_z, A_s, H, 0, red, y);
      const int head = idxA, hd = D / 2;
      const __half* bias = reinterpret_cast<const __half*>(Ly.qkv_bias);
      for (int i = tid; i < hd; i += kThreads) {
        float va = y[i], vb = y[i + hd];
        if (bias) {
          va += __half2float(bias[head * D + i]);
          vb += __half2float(bias[head * D + i + hd]);
        }
        const __half ha = __float2half_rn(va), hb = __float2half_rn(vb);
        if (head < QH + KVH) {
          const float angle = (float)((double)pos * p.rope_inv[i]);
          float si, co;
          sincosf(angle, &si, &co);
          const float xa = __half2float(ha), xb = __half2float(hb);
          const float ra = __fsub_rn(__fmul_rn(xa, co), __fmul_rn(xb, si));
          const float rb = __fadd_rn(__fmul_rn(xb, co), __fmul_rn(xa, si));
          __half* dst = head < QH ? p.q + (size_t)head * D
                                  : reinterpret_cast<__half*>(Ly.k_cache) + ((size_t)pos * KVH + (head - QH)) * D;
          dst[i] = __float2half_rn(ra);
          dst[i + hd] = __float2half_rn(rb);
        } else {
          __half* dst = reinterpret_cast<__half*>(Ly.v_cache) + ((size_t)pos * KVH + (head - QH - KVH)) * D;
          dst[i] = ha;
          dst[i + hd] = hb;
        }
      }
      publish(ctr + 0, 1);
    } else if (roleA == 2) {   // attention chunks u = idxA, idxA + n2, ...
      if (!(ok = wait_count(p, ctr + 0, QH + 2 * KVH))) break;
      for (int u = idxA, first = 1; u < KVH * nch; u += p.n2, first = 0) {
        const int h = u % KVH, c = u / KVH, t0 = c * kChunk, cnt = min(kChunk, T - t0);
        const __half* kc = reinterpret_cast<const __half*>(Ly.k_cache);
        const __half* vc = reinterpret_cast<const __half*>(Ly.v_cache);
        const int d8 = D / 8;
        if (!first) {   // later chunks of this CTA: copied now
          for (int i = tid; i < cnt * d8; i += kThreads) {
            const int r = i / d8, c8 = i % d8, tok = t0 + r;
            if (tok == pos) continue;
            const size_t off = ((size_t)tok * KVH + h) * D + 8 * c8;
            cp16(Kc + r * D + 8 * c8, kc + off);
            cp16(Vc + r * D + 8 * c8, vc + off);
          }
          cp_commit();
          cp_wait0();
        }
        if (pos >= t0 && pos < t0 + cnt) {   // this token's row, written by the QKV phase
          for (int i = tid; i < d8; i += kThreads) {
            const size_t off = ((size_t)pos * KVH + h) * D + 8 * i;
            *reinterpret_cast<uint4*>(Kc + (pos - t0) * D + 8 * i) = __ldcg(reinterpret_cast<const uint4*>(kc + off));
            *reinterpret_cast<uint4*>(Vc + (pos - t0) * D + 8 * i) = __ldcg(reinterpret_cast<const uint4*>(vc + off));
          }
        }
        // q of the group, scaled by log2(e) / sqrt(D), as fp32 in shared memory
        float* qs = misc + 32;                     // [grp][D]
        float* sc = qs + kMaxGroup * kMaxD;         // [grp][64] scores, then probabilities
        const float qscale = 1.4426950408889634f / sqrtf((float)D);
        for (int i = tid; i < grp * D; i += kThreads)   // grp * D <= 1024: two loads per thread at most
          qs[i] = __half2float(__ldcg(p.q + (size_t)h * grp * D + i)) * qscale;
        __syncthreads();
        // scores: warp w takes rows w, w + 16, ...; lanes split the head dim
        const int lane = tid & 31, warp = tid >> 5;
        for (int r = warp; r < kChunk; r += kWarps) {
          float part[kMaxGroup];
#pragma unroll
          for (int j = 0; j < kMaxGroup; ++j) part[j] = 0.0f;
          if (r < cnt) {
            for (int d = 2 * lane; d < D; d += 64) {
              const float2 kv = __half22float2(*reinterpret_cast<const half2*>(Kc + r * D + d));
#pragma unroll
              for (int j = 0; j < kMaxGroup; ++j)
                if (j < grp) part[j] = fmaf(qs[j * D + d + 1], kv.y, fmaf(qs[j * D + d], kv.x, part[j]));
            }
          }
#pragma unroll
          for (int j = 0; j < kMaxGroup; ++j) {
            float v = part[j];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && j < grp) sc[j * kChunk + r] = r < cnt ? v : -INFINITY;
          }
        }
        __syncthreads();
        // per head: max, exp2, sum over the chunk (warp j)
        float* ml = sc + kMaxGroup * kChunk;        // [grp][2]
        if (warp < grp) {
          const float a = sc[warp * kChunk + lane], b = sc[warp * kChunk + lane + 32];
          float m = fmaxf(a, b);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          const float pa = lane < cnt ? exp2f(a - m) : 0.0f, pb = lane + 32 < cnt ? exp2f(b - m) : 0.0f;
          sc[warp * kChunk + lane] = pa;
          sc[warp * kChunk + lane + 32] = pb;
          float s = pa + pb;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
          if (lane == 0) {
            ml[2 * warp] = m;
            ml[2 * warp + 1] = s;
          }
        }
        __syncthreads();
        float* part_out = p.apart + ((size_t)(h * p.maxch + c) * grp) * (D + 2);
        for (int i = tid; i < grp * D; i += kThreads) {
          const int j = i / D, d = i % D;
          float o = 0.0f;
          for (int r = 0; r < cnt; ++r) o = fmaf(sc[j * kChunk + r], __half2float(Vc[r * D + d]), o);
          __stcg(part_out + j * (D + 2) + 2 + d, o);
        }
        if (tid < grp) {
          __stcg(part_out + tid * (D + 2), ml[2 * tid]);
          __stcg(part_out + tid * (D + 2) + 1, ml[2 * tid + 1]);
        }
        // the last chunk of kv head h to arrive merges the chunks in chunk order
        if (last_arrival(p.aticket + l * KVH + h, nch)) {
          // every chunk's (m, l, o) of this head, loaded at once into shared
          // memory (the K / V tiles are no longer needed), in batches that fit
          float* st = reinterpret_cast<float*>(regA);
          const int per_chunk = grp * (D + 2);
          const int batch = max(1, (int)(p.regA_bytes / (per_chunk * 4)));
          float M[2], Ls[2], O[2];
          for (int k = 0; k < 2; ++k) M[k] = -INFINITY, Ls[k] = O[k] = 0.0f;
          for (int c0 = 0; c0 < nch; c0 += batch) {
            const int nb_ = min(batch, nch - c0);
            stage_floats(st, p.apart + (size_t)(h * p.maxch + c0) * per_chunk, nb_ * per_chunk);
            __syncthreads();
            for (int k = 0; k < 2; ++k) {   // (head, dim) pairs tid and tid + 512 (grp * D <= 1024)
              const int i = tid + k * kThreads;
              if (i >= grp * D) continue;
              const int j = i / D, d = i % D;
              for (int cc = 0; cc < nb_; ++cc) {   // online merge in chunk order
                const float* pc = st + cc * per_chunk + j * (D + 2);
                const float m = pc[0];
                const float mn = fmaxf(M[k], m);
                const float a = exp2f(M[k] - mn), b = exp2f(m - mn);
                Ls[k] = fmaf(Ls[k], a, pc[1] * b);
                O[k] = fmaf(O[k], a, pc[2 + d] * b);
                M[k] = mn;
              }
            }
            __syncthreads();
          }
          for (int k = 0; k < 2; ++k) {
            const int i = tid + k * kThreads;
            if (i < grp * D) p.attn[(size_t)h * grp * D + i] = __float2half_rn(O[k] / Ls[k]);
          }
          publish(ctr + 1, 1);
        }
        __syncthreads();
      }
    } else if (roleA == 3) {   // O block idxA: x_a = x + attn W_o
      if (!(ok = wait_count(p, ctr + 1, KVH))) break;
      for (int i = tid; i < QH * D / 8; i += kThreads)
        reinterpret_cast<uint4*>(xs)[i] = __ldcg(reinterpret_cast<const uint4*>(p.attn) + i);
      __syncthreads();
      float* y = misc + 32;
      bad |= tile_gemv<kBW>(A_w, xs, A_z, A_s, QH * D, 0, red, y);
      if (tid < 32) {
        const int col = idxA * 32 + tid;
        const float xin = x_in ? __ldcg(x_in + col) : __half2float(xemb[col]);
        p.xa[col] = xin + y[tid];
      }
      publish(ctr + 2, 1);
    }
    __syncthreads();
    if (l + 1 < p.L) prefetchA(l + 1);
    else cp_commit();

    // ---- role B: gate/up -----------------------------------------------------
    cp_wait2();
    __syncthreads();
    if (!(ok = wait_count(p, ctr + 2, nb))) break;
    rmsnorm_to_smem(p, p.xa, nullptr, reinterpret_cast<const __half*>(Ly.gamma_post), xs, misc);
    int produced = 0;
    for (int sl = 0; sl < 2; ++sl) {
      const int u = sl == 0 ? gu0 : gu1;
      if (u < 0 || u >= n_gu) continue;
      float* g = misc + 32;
      float* up = g + 32;
      uint32_t* wg = gu_w(sl, 0);
      uint32_t* wu = gu_w(sl, 1);
      bad |= tile_gemv<kBW>(wg, xs, wg + H * kBW, wg + H * kBW + (H / kG) * kBW, H, 0, red, g);
      bad |= tile_gemv<kBW>(wu, xs, wu + H * kBW, wu + H * kBW + (H / kG) * kBW, H, 0, red, up);
      if (tid < 32) {
        const float gh = __half2float(__float2half_rn(g[tid])), uh = __half2float(__float2half_rn(up[tid]));
        const float e = expf(-fabsf(gh));   // stable silu (official_weights.py:494-499)
        const float sg = gh >= 0.0f ? gh / (1.0f + e) : (gh * e) / (1.0f + e);
        p.act[u * 32 + tid] = __float2half_rn(sg * uh);
      }
      ++produced;
    }
    if (produced) publish(ctr + 3, produced);
    __syncthreads();
    if (l + 1 < p.L) prefetchB(l + 1);
    else cp_commit();

    // ---- role C: down + residual ----------------------------------------------
    cp_wait2();
    __syncthreads();
    if (has_down) {
      if (!(ok = wait_count(p, ctr + 3, n_gu))) break;
      for (int i = tid; i < drows / 8; i += kThreads)
        reinterpret_cast<uint4*>(xs)[i] = __ldcg(reinterpret_cast<const uint4*>(p.act + drow0) + i);
      __syncthreads();
      float* y = misc + 32;
      bad |= tile_gemv<kBW>(C_w, xs, C_z, C_s, drows, drow0, red, y);
      if (tid < 32) __stcg(p.dpart + ((size_t)db * p.nsplit + ds) * 32 + tid, y[tid]);
      if (last_arrival(p.dticket + l * nb + db, p.nsplit)) {
        float* st = misc + 32;   // [nsplit][32], every split loaded at once
        stage_floats(st, p.dpart + (size_t)db * p.nsplit * 32, p.nsplit * 32);
        __syncthreads();
        if (tid < 32) {
          float acc = 0.0f;
          for (int s2 = 0; s2 < p.nsplit; ++s2) acc += st[s2 * 32 + tid];   // in split order
          const int col = db * 32 + tid;
          x_next[col] = __ldcg(p.xa + col) + acc;
        }
        publish(ctr + 4, 1);
      }
    }
    __syncthreads();
    if (l + 1 < p.L) prefetchC(l + 1);
    else cp_commit();
  }
  cp_wait0();
  if (bad && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SCALE);

  // ---- exit: the last CTA out re-arms every counter for the next launch ------
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    __shared__ int s_exit;
    s_exit = atomicAdd(p.exit_ctr, 1) == P - 1;
    if (s_exit) {
      __threadfence();
      for (int i = 0; i < p.L * kPhases; ++i) p.ctr[i] = 0;
      for (int i = 0; i < p.L * KVH; ++i) p.aticket[i] = 0;
      for (int i = 0; i < p.L * nb; ++i) p.dticket[i] = 0;
      *p.abort_flag = 0;
      __threadfence();
      *p.exit_ctr = 0;
    }
  }
}

// ---------------------------------------------------------------------------
struct Plan {
  int P, n1, n2, n3, nsplit, maxch;
  int offA, offB, offC, offX, offRed, offMisc, smem;
  size_t ws_bytes;
  size_t off_xbuf, off_xa, off_q, off_apart, off_attn, off_act, off_dpart, off_ctr, off_at, off_dt, off_exit,
      off_abort;
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

// ANVILQ_OK and the plan, or the status that rejects the shape.
static int make_plan(int L, int H, int I, int QH, int KVH, int D, int G, int Tmax, Plan* pl) {
  if (L < 1 || H < 128 || I < 128 || QH < 1 || KVH < 1 || Tmax < 1) return ANVILQ_EINVAL;
  if (G != kG || H % kG || I % kG || QH % KVH || QH / KVH > kMaxGroup || (D != 64 && D != 128) ||
      (QH * D) % kG || H > kThreads * kMaxPerThread)
    return ANVILQ_ESHAPE;
  const int P = sm_count();
  if (P <= 0) return ANVILQ_ECUDA;
  pl->P = P;
  const int nb = H / 32, ngI = I / kG;
  pl->n1 = QH + 2 * KVH;
  pl->n3 = nb;
  pl->maxch = (Tmax + kChunk - 1) / kChunk;
  pl->n2 = std::min(KVH * pl->maxch, P - pl->n1 - pl->n3);
  if (pl->n2 < 1) return ANVILQ_ESHAPE;
  pl->nsplit = std::min(std::min(P / nb, ngI), 48);   // the fix-up stages nsplit x 32 floats in `misc`
  if (pl->nsplit < 1 || (I / 32 + P - 1) / P > 2) return ANVILQ_ESHAPE;
  // shared memory
  const size_t qkvA = (size_t)H * (D / 8) * 4 + (H / kG) * (D / 8) * 4 + (H / kG) * D * 2;
  const size_t attA = (size_t)2 * kChunk * D * 2;
  const size_t oA = (size_t)QH * D * kBW * 4 + (QH * D / kG) * kBW * 4 + (QH * D / kG) * 32 * 2;
  const size_t regA = align_up(std::max(qkvA, std::max(attA, oA)), 128);
  const size_t guTile = ((size_t)H * kBW + (H / kG) * kBW + (H / kG) * 4 * kBW) * 4;
  const size_t regB = align_up(4 * guTile, 128);
  const int maxdg = (ngI + pl->nsplit - 1) / pl->nsplit;
  const size_t regC = align_up((size_t)maxdg * kG * kBW * 4 + maxdg * kBW * 4 + maxdg * 32 * 2, 128);
  const size_t xsB = align_up((size_t)std::max(std::max(H, QH * D), maxdg * kG) * 2, 128);
  const size_t redB = align_up((size_t)kWarps * 8 * 16 * 4, 128);
  const size_t miscB = align_up((size_t)(32 + kMaxGroup * kMaxD + kMaxGroup * kChunk + 2 * kMaxGroup) * 4, 128);
  pl->offA = 0;
  pl->offB = (int)regA;
  pl->offC = (int)(regA + regB);
  pl->offX = (int)(regA + regB + regC);
  pl->offRed = pl->offX + (int)xsB;
  pl->offMisc = pl->offRed + (int)redB;
  pl->smem = pl->offMisc + (int)miscB;
  if (pl->smem > 220 * 1024) return ANVILQ_ESHAPE;   // a layer's slices must fit one SM's shared memory
  // workspace
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  pl->off_ctr = take((size_t)L * kPhases * 4);
  pl->off_at = take((size_t)L * KVH * 4);
  pl->off_dt = take((size_t)L * nb * 4);
  pl->off_exit = take(4);
  pl->off_abort = take(4);
  pl->off_xbuf = take((size_t)2 * H * 4);
  pl->off_xa = take((size_t)H * 4);
  pl->off_q = take((size_t)QH * D * 2);
  pl->off_apart = take((size_t)KVH * pl->maxch * (QH / KVH) * (D + 2) * 4);
  pl->off_attn = take((size_t)QH * D * 2);
  pl->off_act = take((size_t)I * 2);
  pl->off_dpart = take((size_t)nb * pl->nsplit * 32 * 4);
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
  p.ctr = reinterpret_cast<int*>(w + pl.off_ctr);
  p.aticket = reinterpret_cast<int*>(w + pl.off_at);
  p.dticket = reinterpret_cast<int*>(w + pl.off_dt);
  p.exit_ctr = reinterpret_cast<int*>(w + pl.off_exit);
  p.abort_flag = reinterpret_cast<int*>(w + pl.off_abort);
  p.xbuf = reinterpret_cast<float*>(w + pl.off_xbuf);
  p.xa = reinterpret_cast<float*>(w + pl.off_xa);
  p.q = reinterpret_cast<__half*>(w + pl.off_q);
  p.apart = reinterpret_cast<float*>(w + pl.off_apart);
  p.attn = reinterpret_cast<__half*>(w + pl.off_attn);
  p.act = reinterpret_cast<__half*>(w + pl.off_act);
  p.dpart = reinterpret_cast<float*>(w + pl.off_dpart);
  p.n1 = pl.n1; p.n2 = pl.n2; p.n3 = pl.n3; p.nsplit = pl.nsplit; p.maxch = pl.maxch;
  p.offA = pl.offA; p.offB = pl.offB; p.offC = pl.offC; p.offX = pl.offX; p.offRed = pl.offRed;
  p.offMisc = pl.offMisc; p.smem = pl.smem;
  p.regA_bytes = pl.offB - pl.offA;
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
