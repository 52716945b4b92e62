// internal.h -- launchers shared between the translation units of libanvilq.so
// (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/anvilq.h"

namespace anvilq {

using GemvPlan = anvilq_gemv_plan;

// Batch-1 W4A16 GEMV on the TMA + cluster kernel (gemv_tma.cu).
bool gemv_tma_supported(const void* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                        int K, int N, int G);
size_t gemv_tma_workspace_bytes(int K, int N);
bool gemv_cluster_default_plan(int K, int N, GemvPlan* plan);
int gemv_cluster_check_plan(int K, int N, GemvPlan* plan);   // validates, fills in ctas
size_t gemv_cluster_workspace_bytes(int K, int N, const GemvPlan& plan);

// Source of the activations and destination of the result of one GEMV launch
// (modes as in ANVILQ_GEMV_X_* / ANVILQ_GEMV_Y_* of anvilq.h).
struct GemvIo {
  int xmode = 0, ymode = 0;
  const uint16_t* x = nullptr;   // fp16 x [K] or fp16 [gate | up] [2K]
  const float* xr = nullptr;     // fp32 residual [K]
  const uint16_t* gamma = nullptr;
  float eps = 0.0f;
  uint16_t* y = nullptr;         // fp16 out [N]
  float* yr = nullptr;           // fp32 residual [N], += result
  // ymode 2 (QKV projection with RoPE and the KV-cache append)
  const int32_t* rope_pos = nullptr;
  uint16_t* q_out = nullptr;
  uint16_t* k_cache = nullptr;
  uint16_t* v_cache = nullptr;
  int32_t* seqlen = nullptr;
  int Hq = 0, Hkv = 0, D = 0, Tmax = 0;
  float theta = 0.0f;
  // ymode 3 (column slice of a tensor-parallel split, all-gather fused in)
  uint16_t* peer_y[8] = {};
  unsigned* peer_flags[8] = {};
  unsigned* epoch = nullptr;
  int world = 0, tp_rank = 0, col_base = 0;
  bool deferred = false;   // stream-K only: no flag wait at the end; the next call waits before reading x
  // ymode 4 (the MLP: gate/up in unit-interleaved columns, down in the
  // epilogue, added into yr)
  const int32_t* dn_qweight = nullptr;
  const int32_t* dn_qzeros = nullptr;
  const uint16_t* dn_scales = nullptr;
  int dn_H = 0;
};
// plan: null for the default plan of the shape; a given plan is only taken
// for x_mode/y_mode 0 and must have passed gemv_cluster_check_plan.
int launch_gemv_tma(const GemvIo& io, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                    const uint16_t* bias, int K, int N, int G, void* workspace, size_t workspace_bytes, int* dev_err,
                    cudaStream_t stream, bool overlap_prior, const GemvPlan* plan = nullptr);

// Batch-1 W4A16 GEMV on the stream-K kernel (gemv_stream.cu).  peer: null, or
// the tensor-parallel fields of a GemvIo (peer_y, peer_flags, epoch, world,
// tp_rank, col_base) for the all-gather fused into the epilogue (y unused).
bool gemv_stream_supported(const void* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                           int K, int N, int G);
bool gemv_stream_default_plan(int K, int N, GemvPlan* plan);
int gemv_stream_check_plan(int K, int N, const GemvPlan& plan);
size_t gemv_stream_workspace_bytes(const GemvPlan& plan);
// one thread waits (bounded) until flags[0 .. world) all reached *epoch
int launch_peer_wait(const unsigned* flags, int world, const unsigned* epoch, int* dev_err, cudaStream_t stream);
int launch_gemv_stream(const GemvPlan& plan, const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                       const uint16_t* scales, const uint16_t* bias, uint16_t* y, int K, int N, int G,
                       void* workspace, size_t workspace_bytes, int* dev_err, cudaStream_t stream,
                       bool overlap_prior, const GemvIo* peer = nullptr);

// Small-M (speculative verify) GEMM on tcgen05 tensor cores (verify_gemm_tc.cu):
// G == 128, K % 128 == 0, N % 32 == 0, 16-byte aligned operands; M rows in
// launches of at most 64.
bool verify_tc_supported(const void* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                         int M, int K, int N, int G);
size_t verify_tc_workspace_bytes(int M, int K, int N);
// qweight: AWQ layout, or null when `packed` (anvilq_w4a16_tc_pack layout) is given.
int launch_verify_tc(const uint16_t* x, const int32_t* qweight, const int32_t* packed, const int32_t* qzeros,
                     const uint16_t* scales, const uint16_t* bias, uint16_t* y, int M, int K, int N,
                     void* workspace, size_t workspace_bytes, int* dev_err, cudaStream_t stream,
                     bool overlap_prior = false);
size_t tc_pack_bytes(int K, int N);
int launch_tc_pack(const int32_t* qweight, int32_t* packed, int K, int N, cudaStream_t stream);

// Bit-accurate Q16.16 integer GEMV (gemv_q16.cu).
size_t gemm_q16_workspace_bytes(int K, int N, int G);
int launch_gemm_q16(const int32_t* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                    const uint16_t* bias, int32_t* y, int M, int K, int N, int G, void* workspace,
                    size_t workspace_bytes, int* dev_err, cudaStream_t stream);

// Decode attention over a paged fp16 cache (gqa_decode.cu), as
// anvilq_gqa_decode_paged, optionally also writing each head's log2-domain
// log-sum-exp to lse [B][Hq] (null: not written).
size_t gqa_decode_workspace_bytes(int B, int Hq, int Hkv, int D, int Tmax);
int launch_gqa_decode_paged(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                            const uint32_t* page_table, const int32_t* seqlens, uint16_t* out, float* lse, int B,
                            int Hq, int Hkv, int D, int page_tokens, int max_pages, int num_pages, float scale,
                            void* workspace, size_t workspace_bytes, int* dev_err, cudaStream_t stream);

}  // namespace anvilq
