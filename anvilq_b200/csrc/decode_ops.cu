// decode_ops.cu -- the decode-step operations around the W4A16 GEMVs and the
// attention kernel: embedding lookup, RoPE + KV-cache append, the tied fp16
// lm_head GEMV with the final RMSNorm and the greedy argmax fused in, and the
// on-device commit of the sampled token.
//
// Reference semantics: FP32Model.token (anvil-q1/tests/official_weights.py:451-509):
// embedding row (:463), split-half RoPE with theta 1e6 (:439-449, :468-469),
// cache write (:470), final norm (:504) and tied logits (:505-506); greedy
// selection with the lowest index winning ties (anvil-q4/tests/transformer_reference.py:212-217).
//
// Every kernel here is launched with programmatic dependent launch when the
// caller passes ANVILQ_GEMM_OVERLAP_PRIOR: it signals its dependents at once
// and waits for its predecessor before touching global memory.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "../../include/anvilq.h"

namespace anvilq {
namespace decode {

__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// x[c] = E[token][c] (fp32 residual stream); clears the argmax key.
__global__ void embed_kernel(const __half* __restrict__ table, const int* __restrict__ token,
                             float* __restrict__ x, int H, int V, unsigned long long* argmax_key, int* dev_err) {
  pdl_enter();
  int t = *token;
  if (t < 0 || t >= V) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && dev_err) atomicOr(dev_err, ANVILQ_DEV_ERR_TOKEN);
    t = 0;
  }
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < H; c += gridDim.x * blockDim.x)
    x[c] = __half2float(table[(size_t)t * H + c]);
  if (argmax_key && blockIdx.x == 0 && threadIdx.x == 0) *argmax_key = 0ull;
}

// qkv = [q (Hq*D) | k (Hkv*D) | v (Hkv*D)] fp16.  q and k are rotated in split
// halves: for pair i < D/2, angle = pos * theta^(-2i/D) (binary64 product of the
// host-computed frequency, rounded to binary32 as the reference does; sine and
// cosine of that binary32 angle in binary32), then
//   a' = a cos - b sin,  b' = b cos + a sin   (a = x[i], b = x[i + D/2]).
// q goes to q_out, rotated k and raw v to row `pos` of the caches
// [Tmax][Hkv][D]; seqlen = pos + 1.
constexpr int kMaxRopePairs = 128;   // head_dim <= 256
struct RopeFreq {
  double inv[kMaxRopePairs];          // theta^(-2i/D), binary64, computed on the host
};

__global__ void rope_append_kernel(const __half* __restrict__ qkv, const int* __restrict__ pos_p,
                                   const int* __restrict__ row_p, __half* __restrict__ q_out,
                                   __half* __restrict__ k_cache, __half* __restrict__ v_cache,
                                   int* __restrict__ seqlen, int Hq, int Hkv, int D, int Tmax,
                                   const __grid_constant__ RopeFreq freq, int* dev_err) {
  pdl_enter();
  const int pos = *pos_p;                     // the rotation's position
  const int crow = row_p ? *row_p : pos;      // the cache row written
  if (pos < 0 || pos >= Tmax || crow < 0 || crow >= Tmax) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && dev_err) atomicOr(dev_err, ANVILQ_DEV_ERR_SEQLEN);
    return;
  }
  const int half_d = D / 2;
  const int rot = (Hq + Hkv) * half_d;   // rotated pairs
  const int copies = Hkv * D;            // v elements
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rot + copies; i += gridDim.x * blockDim.x) {
    if (i < rot) {
      const int head = i / half_d, pair = i % half_d;
      const float angle = (float)((double)pos * freq.inv[pair]);
      float si, co;
      sincosf(angle, &si, &co);
      const int a = head * D + pair, b = a + half_d;
      const float xa = __half2float(qkv[a]), xb = __half2float(qkv[b]);
      const float ra = __fsub_rn(__fmul_rn(xa, co), __fmul_rn(xb, si));
      const float rb = __fadd_rn(__fmul_rn(xb, co), __fmul_rn(xa, si));
      if (head < Hq) {
        q_out[a] = __float2half_rn(ra);
        q_out[b] = __float2half_rn(rb);
      } else {
        const int kh = head - Hq;
        __half* row = k_cache + ((size_t)crow * Hkv + kh) * D;
        row[pair] = __float2half_rn(ra);
        row[pair + half_d] = __float2half_rn(rb);
      }
    } else {
      const int e = i - rot, kh = e / D, d = e % D;
      v_cache[((size_t)crow * Hkv + kh) * D + d] = qkv[(Hq + Hkv) * D + e];
    }
  }
  if (seqlen && blockIdx.x == 0 && threadIdx.x == 0) *seqlen = crow + 1;
}

// Orderable key of (logit, row): larger logit wins, then the lower row index.
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)row);
}

constexpr int kLmThreads = 256;
constexpr int kLmWarps = kLmThreads / 32;
constexpr int kLmRowsPerIter = 4;     // rows per warp iteration, 8 lanes each
constexpr int kLmBatch = 8;           // 16-byte loads in flight per lane

// logits[v] = h . E[v], h = rmsnorm(x, gamma) in fp32; argmax over v into a
// 64-bit key with one atomicMax per CTA.  H % 64 == 0.
__global__ void __launch_bounds__(kLmThreads) lmhead_argmax_kernel(const float* __restrict__ x,
                                                                    const __half* __restrict__ gamma, float eps,
                                                                    const __half* __restrict__ table,
                                                                    float* __restrict__ logits,
                                                                    unsigned long long* __restrict__ key_out, int H,
                                                                    int V) {
  extern __shared__ float h[];   // [H]
  __shared__ float s_red[kLmWarps];
  __shared__ unsigned long long s_best[kLmWarps];
  pdl_enter();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // final RMSNorm, every CTA for itself (H floats)
  float ss = 0.0f;
  for (int k = threadIdx.x; k < H; k += kLmThreads) {
    const float v = __ldcg(x + k);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) s_red[warp] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kLmWarps; ++w) tot += s_red[w];
  const float denom = sqrtf(tot / (float)H + eps);
  for (int k = threadIdx.x; k < H; k += kLmThreads) h[k] = __ldcg(x + k) * __half2float(gamma[k]) / denom;
  __syncthreads();

  const int chunks = H / 8;                 // 16-byte chunks per row
  const int warps_total = gridDim.x * kLmWarps;
  const int gw = blockIdx.x * kLmWarps + warp;
  const int rows_per_warp = (V + warps_total - 1) / warps_total;
  const int r_begin = gw * rows_per_warp, r_end = min(V, r_begin + rows_per_warp);
  const int sub = lane / 8, sl = lane % 8;  // row within the iteration, lane within the row
  unsigned long long best = 0ull;
  for (int r0 = r_begin; r0 < r_end; r0 += kLmRowsPerIter) {
    const int row = r0 + sub;
    const bool valid = row < r_end;
    const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)(valid ? row : r_begin) * H);
    float acc = 0.0f;
    for (int c0 = sl; c0 < chunks; c0 += 8 * kLmBatch) {
      uint4 w[kLmBatch];
#pragma unroll
      for (int b = 0; b < kLmBatch; ++b) {
        const int c = c0 + 8 * b;
        if (c < chunks) w[b] = __ldcs(src + c);
      }
#pragma unroll
      for (int b = 0; b < kLmBatch; ++b) {
        const int c = c0 + 8 * b;
        if (c < chunks) {
          const __half2* hw = reinterpret_cast<const __half2*>(&w[b]);
          const float4 h0 = *reinterpret_cast<const float4*>(h + 8 * c);
          const float4 h1 = *reinterpret_cast<const float4*>(h + 8 * c + 4);
          const float2 e0 = __half22float2(hw[0]), e1 = __half22float2(hw[1]);
          const float2 e2 = __half22float2(hw[2]), e3 = __half22float2(hw[3]);
          acc = fmaf(h0.x, e0.x, acc);
          acc = fmaf(h0.y, e0.y, acc);
          acc = fmaf(h0.z, e1.x, acc);
          acc = fmaf(h0.w, e1.y, acc);
          acc = fmaf(h1.x, e2.x, acc);
          acc = fmaf(h1.y, e2.y, acc);
          acc = fmaf(h1.z, e3.x, acc);
          acc = fmaf(h1.w, e3.y, acc);
        }
      }
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (valid && sl == 0) {
      if (logits) logits[row] = acc;
      const unsigned long long k = argmax_key(acc, row);
      best = k > best ? k : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if (lane == 0) s_best[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < kLmWarps; ++w) b = s_best[w] > b ? s_best[w] : b;
    if (b) atomicMax(key_out, b);
  }
}

// token = row of the argmax key; pos += 1 (the next step's position).
__global__ void commit_kernel(const unsigned long long* __restrict__ key, int* __restrict__ token,
                              int* __restrict__ pos) {
  pdl_enter();
  const unsigned long long k = *key;
  *token = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
  if (pos) *pos += 1;
}

// ---- M-row forms of the GEMV prologues / epilogues (the batched verification
// pass, where the projections run as M-row GEMMs) --------------------------

// out[m] = fp16(x[m] * gamma / sqrt(mean(x[m]^2) + eps)): one CTA per row, the
// same binary32 expression as the RMSNorm prologue of the batch-1 GEMV.
constexpr int kRowThreads = 256;
__global__ void __launch_bounds__(kRowThreads) rmsnorm_rows_kernel(const float* __restrict__ x,
                                                                   const __half* __restrict__ gamma, float eps,
                                                                   __half* __restrict__ out, int H) {
  pdl_enter();
  __shared__ float s_part[kRowThreads / 32];
  const float* xr = x + (size_t)blockIdx.x * H;
  float ss = 0.0f;
  for (int c = threadIdx.x; c < H; c += kRowThreads) ss = fmaf(xr[c], xr[c], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (threadIdx.x % 32 == 0) s_part[threadIdx.x / 32] = ss;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; ++w) t += s_part[w];
  const float inv = 1.0f / sqrtf(t / (float)H + eps);
  for (int c = threadIdx.x; c < H; c += kRowThreads)
    out[(size_t)blockIdx.x * H + c] = __float2half_rn(xr[c] * __half2float(gamma[c]) * inv);
}

// x[i] += y[i] (fp32 residual stream plus an fp16 projection output)
__global__ void add_rows_kernel(float* __restrict__ x, const __half* __restrict__ y, long long n) {
  pdl_enter();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    x[i] += __half2float(y[i]);
}

// out[m][i] = fp16(silu(g) * u), g = gu[m][i], u = gu[m][I + i]: the stable
// SiLU of the batch-1 GEMV prologue (official_weights.py:494-499)
__global__ void silu_mul_rows_kernel(const __half* __restrict__ gu, __half* __restrict__ out, int M, int I) {
  pdl_enter();
  const long long n = (long long)M * I;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (long long)gridDim.x * blockDim.x) {
    const long long m = t / I, i = t % I;
    const float g = __half2float(gu[m * 2 * I + i]);
    const float u = __half2float(gu[m * 2 * I + I + i]);
    const float e = expf(-fabsf(g));
    const float sg = g >= 0.0f ? g / (1.0f + e) : (g * e) / (1.0f + e);
    out[t] = __float2half_rn(sg * u);
  }
}

constexpr int kMaxDevices = 64;
static int g_sms[kMaxDevices];
static std::once_flag g_once[kMaxDevices];
static int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  std::call_once(g_once[dev], [dev] {
    cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(lmhead_argmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    cudaGetLastError();
  });
  return g_sms[dev];
}

template <typename... KArgs, typename... Args>
static int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, unsigned flags,
                  Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & ANVILQ_GEMM_OVERLAP_PRIOR) ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, kernel, args...) != cudaSuccess) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  return ANVILQ_OK;
}

}  // namespace decode
}  // namespace anvilq

using namespace anvilq::decode;

extern "C" {

int anvilq_embed(const uint16_t* table, const int32_t* token, float* x, int H, int V,
                 unsigned long long* argmax_key, int* dev_err, unsigned flags, anvilq_stream_t stream) {
  if (!table || !token || !x || H < 1 || V < 1) return ANVILQ_EINVAL;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  const int threads = 256, blocks = std::min(64, (H + threads - 1) / threads);
  return launch(embed_kernel, dim3(blocks), dim3(threads), 0, reinterpret_cast<cudaStream_t>(stream), flags,
                reinterpret_cast<const __half*>(table), (const int*)token, x, H, V, argmax_key, dev_err);
}

static int rope_kv_append(const uint16_t* qkv, const int32_t* pos, const int32_t* row, uint16_t* q_out,
                          uint16_t* k_cache, uint16_t* v_cache, int32_t* seqlen, int Hq, int Hkv, int D, int Tmax,
                          float theta, int* dev_err, unsigned flags, anvilq_stream_t stream) {
  if (!qkv || !pos || !q_out || !k_cache || !v_cache) return ANVILQ_EINVAL;
  if (Hq < 1 || Hkv < 1 || Hq % Hkv || D < 2 || D % 2 || Tmax < 1 || !(theta > 0.0f)) return ANVILQ_EINVAL;
  if (D / 2 > kMaxRopePairs) return ANVILQ_ESHAPE;
  RopeFreq freq;
  for (int i = 0; i < D / 2; ++i) freq.inv[i] = std::pow((double)theta, -2.0 * i / D);
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  const int work = (Hq + Hkv) * (D / 2) + Hkv * D;
  const int threads = 256, blocks = std::min(32, (work + threads - 1) / threads);
  return launch(rope_append_kernel, dim3(blocks), dim3(threads), 0, reinterpret_cast<cudaStream_t>(stream), flags,
                reinterpret_cast<const __half*>(qkv), (const int*)pos, (const int*)row,
                reinterpret_cast<__half*>(q_out), reinterpret_cast<__half*>(k_cache),
                reinterpret_cast<__half*>(v_cache), (int*)seqlen, Hq, Hkv, D, Tmax, freq, dev_err);
}

int anvilq_rope_kv_append(const uint16_t* qkv, const int32_t* pos, uint16_t* q_out, uint16_t* k_cache,
                          uint16_t* v_cache, int32_t* seqlen, int Hq, int Hkv, int D, int Tmax, float theta,
                          int* dev_err, unsigned flags, anvilq_stream_t stream) {
  return rope_kv_append(qkv, pos, nullptr, q_out, k_cache, v_cache, seqlen, Hq, Hkv, D, Tmax, theta, dev_err, flags,
                        stream);
}

int anvilq_rope_kv_append_at(const uint16_t* qkv, const int32_t* pos, const int32_t* row, uint16_t* q_out,
                             uint16_t* k_cache, uint16_t* v_cache, int Hq, int Hkv, int D, int Tmax, float theta,
                             int* dev_err, unsigned flags, anvilq_stream_t stream) {
  if (!row) return ANVILQ_EINVAL;
  return rope_kv_append(qkv, pos, row, q_out, k_cache, v_cache, nullptr, Hq, Hkv, D, Tmax, theta, dev_err, flags,
                        stream);
}

int anvilq_lmhead_argmax(const float* x, const uint16_t* gamma, float eps, const uint16_t* table, float* logits,
                         unsigned long long* argmax_key, int H, int V, unsigned flags, anvilq_stream_t stream) {
  if (!x || !gamma || !table || !argmax_key || H < 64 || H % 64 || V < 1 || !(eps >= 0.0f)) return ANVILQ_EINVAL;
  if (H * sizeof(float) > 64 * 1024) return ANVILQ_ESHAPE;
  if ((reinterpret_cast<uintptr_t>(table) & 15u) != 0) return ANVILQ_EALIGN;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  const int sms = sm_count();
  if (sms <= 0) return ANVILQ_ECUDA;
  const int rows_per_cta = kLmWarps * kLmRowsPerIter;
  const int blocks = std::max(1, std::min(4 * sms, (V + rows_per_cta - 1) / rows_per_cta));
  return launch(lmhead_argmax_kernel, dim3(blocks), dim3(kLmThreads), (size_t)H * sizeof(float),
                reinterpret_cast<cudaStream_t>(stream), flags, x, reinterpret_cast<const __half*>(gamma), eps,
                reinterpret_cast<const __half*>(table), logits, argmax_key, H, V);
}

int anvilq_argmax_commit(const unsigned long long* argmax_key, int32_t* token, int32_t* pos, unsigned flags,
                         anvilq_stream_t stream) {
  if (!argmax_key || !token) return ANVILQ_EINVAL;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  return launch(commit_kernel, dim3(1), dim3(1), 0, reinterpret_cast<cudaStream_t>(stream), flags, argmax_key,
                (int*)token, (int*)pos);
}

int anvilq_rmsnorm_rows(const float* x, const uint16_t* gamma, float eps, uint16_t* out, int M, int H,
                        unsigned flags, anvilq_stream_t stream) {
  if (!x || !gamma || !out || M < 1 || H < 1) return ANVILQ_EINVAL;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  return launch(rmsnorm_rows_kernel, dim3(M), dim3(kRowThreads), 0, reinterpret_cast<cudaStream_t>(stream), flags,
                x, reinterpret_cast<const __half*>(gamma), eps, reinterpret_cast<__half*>(out), H);
}

int anvilq_residual_add_rows(float* x, const uint16_t* y, int M, int H, unsigned flags, anvilq_stream_t stream) {
  if (!x || !y || M < 1 || H < 1) return ANVILQ_EINVAL;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  const long long n = (long long)M * H;
  const int blocks = (int)std::min<long long>((n + 255) / 256, 4096);
  return launch(add_rows_kernel, dim3(blocks), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), flags, x,
                reinterpret_cast<const __half*>(y), n);
}

int anvilq_silu_mul_rows(const uint16_t* gu, uint16_t* out, int M, int I, unsigned flags, anvilq_stream_t stream) {
  if (!gu || !out || M < 1 || I < 1) return ANVILQ_EINVAL;
  if (flags & ~(unsigned)ANVILQ_GEMM_OVERLAP_PRIOR) return ANVILQ_EINVAL;
  const long long n = (long long)M * I;
  const int blocks = (int)std::min<long long>((n + 255) / 256, 4096);
  return launch(silu_mul_rows_kernel, dim3(blocks), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), flags,
                reinterpret_cast<const __half*>(gu), reinterpret_cast<__half*>(out), M, I);
}

}  // extern "C"
