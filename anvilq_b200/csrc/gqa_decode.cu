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
// Design (one CTA = one (sequence, kv head, KV split); 4 warps):
//   * The query heads of a GQA group (<= 8) share every K/V row, so each row is
//     read from HBM once per group.  Rows are moved by the TMA engine
//     (cp.async.bulk, one 128/256-byte row per lane, 32 rows = one 16-token K
//     tile + V tile per instruction round) into a per-warp ring of 4 stages
//     guarded by mbarriers; each warp streams its own tiles, so no inter-warp
//     handshake sits on the critical path.  Rows are padded by 16 bytes so the
//     fragment loads below are bank-conflict free.
//   * S = Q K^T on the tensor cores (mma.m16n8k16, fp16 in, fp32 accumulate):
//     the group's query heads are the 16-row A operand (rows >= group size are
//     zero), 8 tokens per n-tile.  The S accumulator layout is exactly the B
//     operand layout of O^T += V^T P^T, so P never leaves registers; V^T comes
//     from ldmatrix.trans.
//   * Online softmax in the log2 domain, per warp; warps are merged in shared
//     memory, KV splits through a caller-provided workspace: the CTA that
//     arrives last at a (sequence, kv head) ticket merges the splits in split
//     order (deterministic, no spin-wait) and writes fp16 output.
//   * Every mbarrier wait is bounded (about one second of %globaltimer); on
//     expiry the kernel sets ANVILQ_DEV_ERR_TIMEOUT, stops using its tiles and
//     waits, again bounded, for its own copies before it exits.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "../../include/anvilq.h"

namespace anvilq {
namespace attn {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 16;          // tokens per tile
constexpr int kStages = 4;         // ring depth per warp
constexpr int kMaxGroup = 8;       // query heads per kv head handled by one CTA
constexpr int kMaxSplits = 32;     // KV splits per (sequence, kv head)
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

struct Params {
  const __half* q;      // [B][Hq][D]
  const __half* k;      // [B][Tmax][Hkv][D]
  const __half* v;
  const int* seqlens;   // [B]
  __half* out;          // [B][Hq][D]
  float* partials;      // [B][Hkv][splits][group][D + 2]
  int* tickets;         // [B][Hkv]
  int* dev_err;
  int Hq, Hkv, Tmax, group, splits, tiles_per_split;
  float scale_log2;     // softmax scale * log2(e)
};

template <int D>
struct Layout {
  static constexpr int kRowBytes = D * 2 + 16;                 // padded row
  static constexpr int kStageBytes = 2 * kTile * kRowBytes;    // K tile + V tile
  static constexpr int kWarpBytes = kStages * kStageBytes;
  static constexpr int kRingBytes = kWarps * kWarpBytes;
  static constexpr int kBarOffset = kRingBytes;                // kWarps * kStages mbarriers
  static constexpr int kCombOffset = kBarOffset + kWarps * kStages * 8;
  static constexpr int kCombBytes = kWarps * kMaxGroup * (D + 2) * 4;
  static_assert(kCombBytes >= (3 * kMaxSplits * kMaxGroup + kMaxGroup) * 4, "split merge fits the warp-merge area");
  static constexpr int kTotal = kCombOffset + kCombBytes;
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
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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

template <int D>
__global__ void __launch_bounds__(kThreads) gqa_decode_kernel(const Params p) {
  using L = Layout<D>;
  constexpr int KS = D / 16;   // k-steps of QK, m-tiles of PV
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_flag;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int seqlen = p.seqlens[b];
  const bool bad_len = seqlen < 1 || seqlen > p.Tmax;
  const int ntiles = bad_len ? 0 : (seqlen + kTile - 1) / kTile;
  const int tb = split * p.tiles_per_split;
  const int te = min(ntiles, tb + p.tiles_per_split);
  // warp-local tiles: tb + warp + kWarps * j
  const int my_tiles = te > tb + warp ? (te - tb - warp + kWarps - 1) / kWarps : 0;

  unsigned char* ring = smem + warp * L::kWarpBytes;
  const uint32_t bar0 = smem_u32(smem + L::kBarOffset + warp * kStages * 8);
  if (lane == 0)
    for (int s = 0; s < kStages; ++s) mbar_init(bar0 + 8 * s, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncwarp();

  const size_t row_stride = (size_t)p.Hkv * D;   // elements between consecutive tokens
  const __half* kbase = p.k + ((size_t)b * p.Tmax * p.Hkv + h) * D;
  const __half* vbase = p.v + ((size_t)b * p.Tmax * p.Hkv + h) * D;

  auto issue = [&](int j) {   // tile j of this warp into stage j % kStages
    const int st = j % kStages;
    const uint32_t bar = bar0 + 8 * st;
    if (lane == 0) mbar_expect_tx(bar, 2 * kTile * D * 2);
    __syncwarp();
    fence_proxy_async();
    const int tok = min((tb + warp + kWarps * j) * kTile + (lane % kTile), seqlen - 1);
    const __half* src = (lane < kTile ? kbase : vbase) + (size_t)tok * row_stride;
    const uint32_t dst = smem_u32(ring + st * L::kStageBytes + (lane / kTile) * kTile * L::kRowBytes +
                                  (lane % kTile) * L::kRowBytes);
    bulk_copy_g2s(dst, src, D * 2, bar);
  };

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
  int issued = 0;

  for (; issued < min(kStages - 1, my_tiles); ++issued) issue(issued);
  for (int j = 0; j < my_tiles && ok; ++j) {
    if (issued < my_tiles) issue(issued++);
    const int st = j % kStages;
    // every lane polls; the warp proceeds only if all lanes saw the tile land
    const bool landed = mbar_wait_bounded(bar0 + 8 * st, (j / kStages) & 1);
    if (!__all_sync(0xffffffffu, landed)) {
      ok = false;
      break;
    }
    const unsigned char* kt = ring + st * L::kStageBytes;
    const unsigned char* vt = kt + kTile * L::kRowBytes;
    const int t0 = (tb + warp + kWarps * j) * kTile;

    // S = Q K^T for tokens t0..t0+15 (two n-tiles of 8)
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < KS; ks += 2) {
        const int mj = lane / 8, r = lane % 8;
        const uint32_t addr = smem_u32(kt + (nt * 8 + r) * L::kRowBytes + (16 * (ks + mj / 2) + 8 * (mj % 2)) * 2);
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
        x[nt * 2 + e] = tok < seqlen ? s[nt][e] * p.scale_log2 : -INFINITY;
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
    const uint32_t pb0 = pack_half2(pr[0], pr[1]);   // tokens 2(l%4), +1   (k rows 0..7)
    const uint32_t pb1 = pack_half2(pr[2], pr[3]);   // tokens 8 + 2(l%4)   (k rows 8..15)
    const float alpha_a = __shfl_sync(0xffffffffu, alpha, 8 * (lane % 4));
    const float alpha_b = __shfl_sync(0xffffffffu, alpha, 8 * (lane % 4) + 4);
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      o[mt][0] *= alpha_a;
      o[mt][1] *= alpha_b;
      o[mt][2] *= alpha_a;
      o[mt][3] *= alpha_b;
      const int mj = lane / 8, r = lane % 8;
      const uint32_t addr = smem_u32(vt + (r + 8 * (mj / 2)) * L::kRowBytes + (16 * mt + 8 * (mj % 2)) * 2);
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

  // ---- merge the warps (shared memory) ----
  float* comb = reinterpret_cast<float*>(smem + L::kCombOffset);   // [warp][head][D + 2]
  float* mine = comb + (size_t)warp * kMaxGroup * (D + 2);
  if (!ok) {
    m_run = -INFINITY;
    l_run = 0.0f;
  }
#pragma unroll
  for (int mt = 0; mt < KS; ++mt) {
    const int d = 16 * mt + lane / 4, hh = 2 * (lane % 4);
    mine[hh * (D + 2) + d] = ok ? o[mt][0] : 0.0f;
    mine[(hh + 1) * (D + 2) + d] = ok ? o[mt][1] : 0.0f;
    mine[hh * (D + 2) + d + 8] = ok ? o[mt][2] : 0.0f;
    mine[(hh + 1) * (D + 2) + d + 8] = ok ? o[mt][3] : 0.0f;
  }
  if (lane % 4 == 0) {
    mine[g * (D + 2) + D] = m_run;
    mine[g * (D + 2) + D + 1] = l_run;
  }
  __syncthreads();
  const int G = p.group;
  const int pair = b * p.Hkv + h;
  const bool single = p.splits == 1;
  float* part = p.partials + ((size_t)pair * p.splits + split) * G * (D + 2);
  for (int e = threadIdx.x; e < G * (D + 2); e += blockDim.x) {
    const int hh = e / (D + 2), d = e % (D + 2);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, comb[(w * kMaxGroup + hh) * (D + 2) + D]);
    float acc = 0.0f, lsum = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float* row = comb + (w * kMaxGroup + hh) * (D + 2);
        const float f = exp2f(row[D] - M);
        lsum += f * row[D + 1];
        if (d < D) acc += f * row[d];
      }
    }
    const float val = d < D ? acc : (d == D ? M : lsum);
    if (single) {
      if (d < D) {
        const float out = (lsum > 0.0f) ? acc / lsum : 0.0f;
        p.out[((size_t)b * p.Hq + (size_t)h * G + hh) * D + d] = __float2half_rn(out);
      }
    } else {
      __stcg(part + e, val);
    }
  }
  if (bad_len && threadIdx.x == 0) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SEQLEN);
  if (single) return;

  // ---- merge the KV splits: last CTA of the (sequence, kv head) pair ----
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(p.tickets + pair, 1);
    const bool last = ticket == p.splits - 1;
    if (last) p.tickets[pair] = 0;
    s_flag = last;
  }
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  const float* parts = p.partials + (size_t)pair * p.splits * G * (D + 2);
  // split statistics (running max, running sum) of every head, loaded in one
  // parallel pass into shared memory (reusing the warp-merge area)
  float* s_stat = comb;   // [splits][G][2]
  for (int i = threadIdx.x; i < p.splits * G; i += blockDim.x) {
    const float* row = parts + (size_t)i * (D + 2);
    s_stat[2 * i] = __ldcg(row + D);
    s_stat[2 * i + 1] = __ldcg(row + D + 1);
  }
  __syncthreads();
  float* s_w = comb + 2 * kMaxSplits * kMaxGroup;   // [splits][G] merge weights, then [G] 1/L
  for (int hh = threadIdx.x; hh < G; hh += blockDim.x) {
    float M = -INFINITY;
    for (int sp = 0; sp < p.splits; ++sp) M = fmaxf(M, s_stat[2 * (sp * G + hh)]);
    float lsum = 0.0f;
    for (int sp = 0; sp < p.splits; ++sp) {
      const float f = M == -INFINITY ? 0.0f : exp2f(s_stat[2 * (sp * G + hh)] - M);
      s_w[sp * G + hh] = f;
      lsum += f * s_stat[2 * (sp * G + hh) + 1];
    }
    s_w[kMaxSplits * G + hh] = lsum > 0.0f ? 1.0f / lsum : 0.0f;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int hh = e / D, d = e % D;
    float acc = 0.0f;
    int sp = 0;
    for (; sp + 8 <= p.splits; sp += 8) {   // independent loads, summed in split order
      float o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = __ldcg(parts + ((size_t)(sp + k) * G + hh) * (D + 2) + d);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc += s_w[(sp + k) * G + hh] * o[k];
    }
    for (; sp < p.splits; ++sp) acc += s_w[sp * G + hh] * __ldcg(parts + ((size_t)sp * G + hh) * (D + 2) + d);
    p.out[((size_t)b * p.Hq + (size_t)h * G + hh) * D + d] = __float2half_rn(acc * s_w[kMaxSplits * G + hh]);
  }
}

// ---------------------------------------------------------------------------
struct Plan {
  int splits, tiles_per_split;
  size_t partial_bytes, bytes;
};

constexpr int kMaxDevices = 64;
static int g_sms[kMaxDevices];
static std::once_flag g_once[kMaxDevices];

static int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  std::call_once(g_once[dev], [dev] {
    cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(gqa_decode_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout<64>::kTotal);
    cudaFuncSetAttribute(gqa_decode_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout<128>::kTotal);
    cudaGetLastError();
  });
  return g_sms[dev];
}

static Plan plan_for(int B, int Hq, int Hkv, int D, int Tmax, int sms) {
  Plan pl{};
  const int tiles = (Tmax + kTile - 1) / kTile;
  const long long pairs = (long long)B * Hkv;
  const int ctas_per_sm = D == 64 ? 3 : 1;
  const long long slots = (long long)std::max(sms, 1) * ctas_per_sm;
  // enough CTAs for about two full waves, each split holding >= one tile per warp
  long long want = (2 * slots + pairs - 1) / pairs;
  const int max_splits = std::max(1, std::min(kMaxSplits, tiles / kWarps));
  pl.splits = (int)std::max<long long>(1, std::min<long long>(want, max_splits));
  pl.tiles_per_split = (tiles + pl.splits - 1) / pl.splits;
  pl.splits = (tiles + pl.tiles_per_split - 1) / pl.tiles_per_split;
  const int group = Hq / Hkv;
  pl.partial_bytes = pl.splits > 1 ? (size_t)pairs * pl.splits * group * (D + 2) * sizeof(float) : 0;
  pl.bytes = ANVILQ_WORKSPACE_COUNTER_BYTES + pl.partial_bytes;
  return pl;
}

static bool args_ok(int B, int Hq, int Hkv, int D, int Tmax) {
  return B >= 1 && Hq >= 1 && Hkv >= 1 && Hq % Hkv == 0 && Hq / Hkv <= kMaxGroup && (D == 64 || D == 128) &&
         Tmax >= 1 && (long long)B * Hkv * (long long)sizeof(int) <= ANVILQ_WORKSPACE_COUNTER_BYTES;
}

static bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace attn
}  // namespace anvilq

using namespace anvilq::attn;

extern "C" {

size_t anvilq_gqa_decode_workspace_size(int B, int Hq, int Hkv, int D, int Tmax) {
  if (!args_ok(B, Hq, Hkv, D, Tmax)) return 0;
  const int sms = sm_count();
  if (sms <= 0) return 0;
  return plan_for(B, Hq, Hkv, D, Tmax, sms).bytes;
}

int anvilq_gqa_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* seqlens,
                      uint16_t* out, int B, int Hq, int Hkv, int D, int Tmax, float scale, void* workspace,
                      size_t workspace_bytes, int* dev_err, anvilq_stream_t stream) {
  if (!q || !k_cache || !v_cache || !seqlens || !out || !dev_err) return ANVILQ_EINVAL;
  if (!args_ok(B, Hq, Hkv, D, Tmax)) return ANVILQ_ESHAPE;
  if (!a16(q) || !a16(k_cache) || !a16(v_cache) || !a16(out)) return ANVILQ_EALIGN;
  const int sms = sm_count();
  if (sms <= 0) return ANVILQ_ECUDA;
  const Plan pl = plan_for(B, Hq, Hkv, D, Tmax, sms);
  if (!workspace || workspace_bytes < pl.bytes) return ANVILQ_EWORKSPACE;
  if (!a16(workspace)) return ANVILQ_EALIGN;
  Params p;
  p.q = reinterpret_cast<const __half*>(q);
  p.k = reinterpret_cast<const __half*>(k_cache);
  p.v = reinterpret_cast<const __half*>(v_cache);
  p.seqlens = seqlens;
  p.out = reinterpret_cast<__half*>(out);
  p.tickets = reinterpret_cast<int*>(workspace);   // counters first, partials after them
  p.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + ANVILQ_WORKSPACE_COUNTER_BYTES);
  p.dev_err = dev_err;
  p.Hq = Hq; p.Hkv = Hkv; p.Tmax = Tmax; p.group = Hq / Hkv;
  p.splits = pl.splits; p.tiles_per_split = pl.tiles_per_split;
  const float s = scale > 0.0f ? scale : 1.0f / std::sqrt((float)D);
  p.scale_log2 = s * 1.4426950408889634f;
  const dim3 grid(pl.splits, Hkv, B);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (D == 64)
    gqa_decode_kernel<64><<<grid, kThreads, Layout<64>::kTotal, st>>>(p);
  else
    gqa_decode_kernel<128><<<grid, kThreads, Layout<128>::kTotal, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
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
  const int sms = sm_count();
  if (sms <= 0) return ANVILQ_ECUDA;
  const Plan pl = plan_for(B, Hq, Hkv, D, Tmax, sms);
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
  Params p;
  p.q = reinterpret_cast<const __half*>(q);
  p.k = reinterpret_cast<const __half*>(k_cache);
  p.v = reinterpret_cast<const __half*>(v_cache);
  p.seqlens = seqlens;
  p.out = reinterpret_cast<__half*>(out);
  p.tickets = reinterpret_cast<int*>(ws);
  p.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + ANVILQ_WORKSPACE_COUNTER_BYTES);
  p.dev_err = dev_err;
  p.Hq = Hq; p.Hkv = Hkv; p.Tmax = Tmax; p.group = Hq / Hkv;
  p.splits = pl.splits; p.tiles_per_split = pl.tiles_per_split;
  const float s = scale > 0.0f ? scale : 1.0f / std::sqrt((float)D);
  p.scale_log2 = s * 1.4426950408889634f;
  const dim3 grid(pl.splits, Hkv, B);
  if (D == 64)
    gqa_decode_kernel<64><<<grid, kThreads, Layout<64>::kTotal, st>>>(p);
  else
    gqa_decode_kernel<128><<<grid, kThreads, Layout<128>::kTotal, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}
