// tree_attn.cu -- attention of speculative draft nodes over the committed prefix
// plus each node's ancestors (tree attention with ancestor masks).
//
// Reference semantics: the batched draft-tree decoder of Anvil-Q3-HT2
// (anvil-q3-ht2/design/SPEC.md:71-86: "per-node causal tree attention" over the
// committed prefix and the node's ancestors) with the ancestor contract of
// anvil-q1-ht3/design/SPEC.md:528-533 (each active node includes itself and
// only earlier ancestors, and includes the ancestors of its ancestors);
// prefix coordinates first, then provisional nodes in ascending node order
// (:535-538).  Node m's softmax runs over cache rows [0, P) and the rows P + j
// of the nodes j whose bit is set in ancestors[m].
//
// Design.  The prefix is the expensive part (P rows, each read once per kv
// head per node) and is exactly decode attention, so it runs on the paged
// split-KV kernel: every node is one "sequence" whose page table maps onto the
// same cache pages (the cache viewed as a pool of 16-token pages), with the
// kernel also returning each head's log-sum-exp.  The provisional part (at
// most 32 rows) runs in tree_tail_kernel, one warp per (node, query head): the
// ancestor scores in fp32 from the fp16 q and K rows, then one softmax over
// {prefix state, ancestors} merged through the prefix log-sum-exp:
//   out = (o_p 2^(lse_p - M) + sum_j 2^(s_j - M) v_j) / (2^(lse_p - M) + sum_j 2^(s_j - M)).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>

#include "../../include/anvilq.h"
#include "internal.h"

namespace anvilq {
namespace tree {

constexpr int kMaxNodes = 32;   // one ancestor bit per node
constexpr int kPageTokens = 16;

struct TailParams {
  const __half* q;             // [M][Hq][D]
  const __half* k;             // [Tmax][Hkv][D]
  const __half* v;
  const uint32_t* ancestors;   // [M]
  const __half* o_prefix;      // [M][Hq][D] prefix attention, or null when P == 0
  const float* lse_prefix;     // [M][Hq]
  __half* out;                 // [M][Hq][D]
  int* dev_err;
  int M, Hq, Hkv, D, P;
  float scale_log2;
};

// One warp per (node m, query head hq): lane l holds dims l, l + 32, ... of D.
__global__ void __launch_bounds__(128) tree_tail_kernel(const TailParams p) {
  const int lane = threadIdx.x % 32;
  const int hq = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int m = blockIdx.y;
  if (hq >= p.Hq) return;
  const int kvh = hq / (p.Hq / p.Hkv);
  const uint32_t mask = p.ancestors[m];
  // the ancestor contract: itself included, no later node, closed under ancestry
  bool ok = (mask >> m) & 1u;
  if (m + 1 < 32) ok = ok && (mask >> (m + 1)) == 0u;
  for (int j = 0; j < m && ok; ++j)
    if ((mask >> j) & 1u) ok = (p.ancestors[j] & ~mask) == 0u;
  if (!ok && hq == 0 && lane == 0) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TREE);

  constexpr int kPer = 4;   // D <= 128
  float qv[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int d = lane + 32 * i;
    qv[i] = d < p.D ? __half2float(p.q[((size_t)m * p.Hq + hq) * p.D + d]) : 0.0f;
  }
  // scores of the ancestors, in ascending node order; lane j keeps score j
  float s_mine = -INFINITY;
  for (int j = 0; j <= m; ++j) {
    if (!((mask >> j) & 1u)) continue;
    const __half* kr = p.k + ((size_t)(p.P + j) * p.Hkv + kvh) * p.D;
    float dot = 0.0f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int d = lane + 32 * i;
      if (d < p.D) dot = fmaf(qv[i], __half2float(kr[d]), dot);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == j) s_mine = dot * p.scale_log2;
  }
  const float lse_p = p.o_prefix ? p.lse_prefix[(size_t)m * p.Hq + hq] : -INFINITY;
  float mx = s_mine;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  mx = fmaxf(mx, lse_p);   // finite: node m sees itself
  const float w_mine = s_mine == -INFINITY ? 0.0f : exp2f(s_mine - mx);
  const float w_p = lse_p == -INFINITY ? 0.0f : exp2f(lse_p - mx);
  // the denominator in a fixed order: prefix, then nodes 0..31
  float den = w_mine;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  den += w_p;
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int d = lane + 32 * i;
    acc[i] = w_p > 0.0f && d < p.D ? w_p * __half2float(p.o_prefix[((size_t)m * p.Hq + hq) * p.D + d]) : 0.0f;
  }
  for (int j = 0; j <= m; ++j) {
    if (!((mask >> j) & 1u)) continue;
    const float wj = __shfl_sync(0xffffffffu, w_mine, j);
    const __half* vr = p.v + ((size_t)(p.P + j) * p.Hkv + kvh) * p.D;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int d = lane + 32 * i;
      if (d < p.D) acc[i] = fmaf(wj, __half2float(vr[d]), acc[i]);
    }
  }
  const float inv = den > 0.0f ? 1.0f / den : 0.0f;   // 0 only for a mask flagged above
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int d = lane + 32 * i;
    if (d < p.D) p.out[((size_t)m * p.Hq + hq) * p.D + d] = __float2half_rn(acc[i] * inv);
  }
}

// the prefix pages of every node: entry j = valid | page j (the cache as a pool
// of 16-token pages); every node's prefix length is P
__global__ void tree_setup_kernel(uint32_t* table, int32_t* seqlens, int M, int pages, int P) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < M * pages) table[i] = 0x80000000u | (uint32_t)(i % pages);
  if (i < M) seqlens[i] = P;
}

struct Layout {
  size_t attn, table, oprefix, lse, seqlens, total;
};
static size_t up16(size_t n) { return (n + 15) & ~size_t(15); }
static Layout layout(int M, int Hq, int Hkv, int D, int Tmax) {
  Layout l{};
  const size_t attn = gqa_decode_workspace_bytes(M, Hq, Hkv, D, Tmax);
  if (!attn) return l;
  const int pages = Tmax / kPageTokens;
  l.attn = 0;
  l.table = up16(attn);
  l.oprefix = l.table + up16((size_t)M * pages * 4);
  l.lse = l.oprefix + up16((size_t)M * Hq * D * 2);
  l.seqlens = l.lse + up16((size_t)M * Hq * 4);
  l.total = l.seqlens + up16((size_t)M * 4);
  return l;
}

static bool shape_ok(int M, int Hq, int Hkv, int D, int Tmax) {
  return M >= 1 && M <= kMaxNodes && Hq >= 1 && Hkv >= 1 && Hq % Hkv == 0 && (D == 64 || D == 128) &&
         Tmax >= kPageTokens && Tmax % kPageTokens == 0;
}

}  // namespace tree
}  // namespace anvilq

extern "C" {

size_t anvilq_tree_attention_workspace_size(int M, int Hq, int Hkv, int D, int Tmax) {
  using namespace anvilq::tree;
  if (!shape_ok(M, Hq, Hkv, D, Tmax)) return 0;
  return layout(M, Hq, Hkv, D, Tmax).total;
}

int anvilq_tree_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                          const uint32_t* ancestors, int prefix_len, uint16_t* out, int M, int Hq, int Hkv, int D,
                          int Tmax, float scale, void* workspace, size_t workspace_bytes, int* dev_err,
                          anvilq_stream_t stream) {
  using namespace anvilq::tree;
  if (!q || !k_cache || !v_cache || !ancestors || !out || !dev_err) return ANVILQ_EINVAL;
  if (!shape_ok(M, Hq, Hkv, D, Tmax) || prefix_len < 0 || (long long)prefix_len + M > Tmax) return ANVILQ_ESHAPE;
  auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (!a16(q) || !a16(k_cache) || !a16(v_cache) || !a16(out)) return ANVILQ_EALIGN;
  const Layout l = layout(M, Hq, Hkv, D, Tmax);
  if (!l.total) return ANVILQ_ESHAPE;
  if (!workspace || workspace_bytes < l.total) return ANVILQ_EWORKSPACE;
  if (!a16(workspace)) return ANVILQ_EALIGN;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  TailParams tp{};
  tp.q = reinterpret_cast<const __half*>(q);
  tp.k = reinterpret_cast<const __half*>(k_cache);
  tp.v = reinterpret_cast<const __half*>(v_cache);
  tp.ancestors = ancestors;
  tp.out = reinterpret_cast<__half*>(out);
  tp.dev_err = dev_err;
  tp.M = M; tp.Hq = Hq; tp.Hkv = Hkv; tp.D = D; tp.P = prefix_len;
  const float s = scale > 0.0f ? scale : 1.0f / std::sqrt((float)D);
  tp.scale_log2 = s * 1.4426950408889634f;
  if (prefix_len > 0) {
    const int pages = Tmax / kPageTokens;
    auto* table = reinterpret_cast<uint32_t*>(ws + l.table);
    auto* seqlens = reinterpret_cast<int32_t*>(ws + l.seqlens);
    auto* o_prefix = reinterpret_cast<uint16_t*>(ws + l.oprefix);
    auto* lse = reinterpret_cast<float*>(ws + l.lse);
    const int n = M * pages;
    tree_setup_kernel<<<(n + 255) / 256, 256, 0, st>>>(table, seqlens, M, pages, prefix_len);
    if (cudaGetLastError() != cudaSuccess) return ANVILQ_ECUDA;
    const int rc = anvilq::launch_gqa_decode_paged(q, k_cache, v_cache, table, seqlens, o_prefix, lse, M, Hq, Hkv,
                                                   D, kPageTokens, pages, pages, scale, ws + l.attn, l.table,
                                                   dev_err, st);
    if (rc != ANVILQ_OK) return rc;
    tp.o_prefix = reinterpret_cast<const __half*>(o_prefix);
    tp.lse_prefix = lse;
  }
  const dim3 grid((Hq + 3) / 4, M);
  tree_tail_kernel<<<grid, 128, 0, st>>>(tp);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}

}  // extern "C"
