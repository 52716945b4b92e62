/*
 * anvilq.h -- C ABI of libanvilq.so, the B200 (sm_100a) W4A16 AWQ decode datapath.
 *
 * Conventions
 *  - Every pointer argument is a DEVICE pointer owned by the caller, except
 *    where stated.  Nothing here allocates device memory: scratch space is a
 *    caller-provided workspace whose size is given by the *_workspace_size
 *    query.
 *  - binary16 tensors are passed as `uint16_t*` bit patterns; AWQ packed
 *    tensors as `int32_t*` in the reference's layout:
 *        qweight [K][N/8]   qzeros [ceil(K/G)][N/8]   scales [ceil(K/G)][N]   bias [N]
 *    (input row k uses group k / G; the last group may be partial, as in
 *    anvil-q1/tests/official_weights.py:427-429)
 *    where logical output lane i of a packed word sits at bit shift
 *    (0,16,4,20,8,24,12,28)[i] (anvil-q1/tests/verify.py:38).
 *  - All work is asynchronous on `stream` (NULL = legacy default stream).
 *  - Return value: ANVILQ_OK, or a negative ANVILQ_E* code for an argument
 *    rejected on the host before anything was launched.  A condition found
 *    on the device (an invalid AWQ scale) is OR-ed into *dev_err (optional,
 *    device int, never cleared by the library); the whole operation is then
 *    failed and its output must not be used, mirroring the reference, where
 *    an invalid scale fails the GEMV instead of being consumed
 *    (anvil-q1/design/SPEC.md:175-177).
 *  - Calls are stateless and thread-safe; two calls that share a workspace
 *    must be ordered on the GPU (same stream or events).
 */
#ifndef ANVILQ_H
#define ANVILQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* anvilq_stream_t; /* same type as cudaStream_t */

#define ANVILQ_ABI_VERSION 1

#define ANVILQ_OK 0
#define ANVILQ_EINVAL (-1)     /* null pointer, negative or inconsistent size */
#define ANVILQ_EALIGN (-2)     /* pointer alignment the kernel needs is missing */
#define ANVILQ_ECUDA (-3)      /* kernel launch failed (cudaGetLastError) */
#define ANVILQ_EWORKSPACE (-4) /* workspace missing or smaller than required */
#define ANVILQ_ESHAPE (-5)     /* shape outside the supported range */
#define ANVILQ_ENOSCRATCH (-6) /* needs more than the fixed scratch of a no-allocation entry point */

/* Bits OR-ed into *dev_err by a kernel. */
#define ANVILQ_DEV_ERR_SCALE 1   /* an AWQ scale was negative-nonzero or nonfinite */
#define ANVILQ_DEV_ERR_SEQLEN 2  /* a sequence length outside [1, Tmax] */
#define ANVILQ_DEV_ERR_TIMEOUT 4 /* a bounded wait inside a kernel expired */
#define ANVILQ_DEV_ERR_TOKEN 8   /* a token id outside [0, V) */
#define ANVILQ_DEV_ERR_NONFINITE 16 /* a binary16 parameter (bias) was Inf or NaN */
#define ANVILQ_DEV_ERR_PAGE 32     /* a page-table entry of a live page was absent or out of range */
#define ANVILQ_DEV_ERR_TREE 64     /* a draft node's ancestor mask broke the tree contract */
#define ANVILQ_DEV_ERR_CODEC 128   /* a legacy cache block held a forbidden code, padding or metadata */
#define ANVILQ_DEV_ERR_ALIGN 256   /* a tensor named by a device-side table was not 16-byte aligned */

/* Workspace layout shared by every entry point that takes one: the first
 * ANVILQ_WORKSPACE_COUNTER_BYTES hold arrival counters that must be zero
 * before a call and that every call leaves zero; the bytes after them are
 * scratch that a call overwrites.  One workspace, zero-filled once, can
 * therefore serve any sequence of calls ordered on one stream. */
#define ANVILQ_WORKSPACE_COUNTER_BYTES 65536

int anvilq_abi_version(void);
const char* anvilq_strerror(int status);

/* ---------------------------------------------------------------------------
 * W4A16 AWQ GEMV / small-M GEMM:  y[M][N] = x[M][K] @ dequant(W)[K][N] (+ bias)
 *
 * Replaces FP32Model.linear(x, layer, projection)
 * (anvil-q1/tests/official_weights.py:418-437): for each output column c,
 * sum over k of x[k] * ((u4 q[k][c] - u4 z[k/G][c]) * scale[k/G][c]), plus
 * bias[c] for Q/K/V projections; M independent rows (the speculative-verify
 * batch of anvil-q4/rtl/anvil_q4_speculative.sv:57-92 computed in one pass).
 *
 * x fp16 [M][K], y fp16 [M][N], bias fp16 [N] or NULL.  Products are
 * accumulated in fp32 (each x (q - z) product exact, every partial sum fp32),
 * then rounded once to fp16: results differ from the reference's
 * strictly sequential binary32 sum only by accumulation order and the final
 * fp16 rounding.
 * Requirements: M >= 1, K >= 1, N >= 8, N % 8 == 0, G >= 1.
 * The fast kernels additionally use G % 16 == 0, K % 16 == 0, N % 32 == 0 and
 * 16-byte aligned pointers; other shapes fall back to the sequential kernel.
 * workspace: at least anvilq_w4a16_gemm_workspace_size(M, K, N, G) bytes,
 * 16-byte aligned, with the layout described at ANVILQ_WORKSPACE_COUNTER_BYTES.
 * Supports N <= 4,194,304.
 */
size_t anvilq_w4a16_gemm_workspace_size(int M, int K, int N, int G);
int anvilq_w4a16_gemm(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                      const uint16_t* scales, const uint16_t* bias, uint16_t* y,
                      int M, int K, int N, int G,
                      void* workspace, size_t workspace_bytes,
                      int* dev_err, anvilq_stream_t stream);

/* Same operation with flags:
 *   ANVILQ_GEMM_OVERLAP_PRIOR  the weights (qweight, qzeros, scales, bias) are
 *     not written by the work enqueued just before this call on `stream`, so
 *     the kernel may be launched before that work finishes and start
 *     streaming its weights early (programmatic dependent launch).  x is
 *     still read only after the preceding work has completed, and y written
 *     after that.  Used for chains of GEMMs over resident model weights. */
#define ANVILQ_GEMM_OVERLAP_PRIOR 1u
int anvilq_w4a16_gemm_ex(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                         const uint16_t* scales, const uint16_t* bias, uint16_t* y,
                         int M, int K, int N, int G,
                         void* workspace, size_t workspace_bytes,
                         int* dev_err, unsigned flags, anvilq_stream_t stream);

/* ---- batch-1 GEMV plans ------------------------------------------------------
 * The M = 1 GEMV runs on one of two kernels, chosen per shape:
 *   ANVILQ_GEMV_KERNEL_CLUSTER  bands of band_cols columns; `cluster` CTAs of a
 *     thread-block cluster and `kc` clusters split K per band (partials summed
 *     over distributed shared memory, then, for kc > 1, by the cluster arriving
 *     last at the band's workspace ticket); 4 warps per CTA.  Decode-size layers.
 *   ANVILQ_GEMV_KERNEL_STREAM  256-column bands cut into 32-row chunks, the
 *     chunks split evenly over `ctas` CTAs of `warps` warps (stream-K); a band
 *     shared by several CTAs is summed by the CTA arriving last at its ticket.
 *     7B / 70B-class layers.  Needs K % 32 == 0, G % 32 == 0, K % G == 0.
 * `stages` is the depth of every warp's TMA ring.  Every sum has a fixed
 * order: a plan's results are bit-reproducible.
 * anvilq_w4a16_gemv_plan fills in the plan anvilq_w4a16_gemm(_ex) uses for
 * M = 1 (ANVILQ_ESHAPE when no fast kernel serves the shape);
 * anvilq_w4a16_gemv_kernel_plan the best plan of one named kernel for the
 * shape (ANVILQ_EINVAL for an unknown kernel, ANVILQ_ESHAPE when that kernel
 * cannot serve it);
 * anvilq_w4a16_gemv_planned runs y = x @ dequant(W) (+ bias) under a given
 * plan, checked against the kernel's rules (ANVILQ_EINVAL for a plan the
 * kernel does not have, ANVILQ_ESHAPE for one that does not fit the shape);
 * its workspace is anvilq_w4a16_gemv_plan_workspace_size bytes (0: the plan
 * does not fit).  Same meaning and tolerance as anvilq_w4a16_gemm with M = 1.
 * Replaces FP32Model.linear (anvil-q1/tests/official_weights.py:418-437) like
 * anvilq_w4a16_gemm; the plan is the launch shape a caller may pin. */
#define ANVILQ_GEMV_KERNEL_CLUSTER 0
#define ANVILQ_GEMV_KERNEL_STREAM 1
typedef struct anvilq_gemv_plan {
  int kernel;     /* ANVILQ_GEMV_KERNEL_* */
  int band_cols;  /* output columns per band: 512, 256 or 128 (cluster), 256 (stream) */
  int cluster;    /* CTAs per thread-block cluster (power of two <= 16); 1 for stream */
  int kc;         /* clusters per band (1..8); 1 for stream */
  int warps;      /* warps per CTA: 4 (cluster); 4, 8 or 16 (stream) */
  int stages;     /* ring depth per warp: 3 or 4 (cluster); 2..4 (stream) */
  int ctas;       /* CTAs launched (cluster: bands * kc * cluster, filled in) */
} anvilq_gemv_plan;
int anvilq_w4a16_gemv_plan(int K, int N, int G, anvilq_gemv_plan* plan);
int anvilq_w4a16_gemv_kernel_plan(int kernel, int K, int N, int G, anvilq_gemv_plan* plan);
size_t anvilq_w4a16_gemv_plan_workspace_size(int K, int N, int G, const anvilq_gemv_plan* plan);
int anvilq_w4a16_gemv_planned(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                              const uint16_t* scales, const uint16_t* bias, uint16_t* y, int K, int N, int G,
                              const anvilq_gemv_plan* plan, void* workspace, size_t workspace_bytes,
                              int* dev_err, unsigned flags, anvilq_stream_t stream);

/* The speculative-verify GEMM on the tensor cores: M token rows against one
 * AWQ weight matrix with tcgen05.mma from shared memory into TMEM
 * accumulators (integer deltas q - z on the tensor cores, the group scale
 * applied in fp32 afterwards).  Replaces the M full weight passes of the
 * reference's sequential verify (anvil-q4/rtl/anvil_q4_speculative.sv:57-92,
 * anvil-q4/design/SPEC.md:271-272) and its 4-token batched projection
 * (anvil-q3-ht2/design/SPEC.md:81-86); every row equals FP32Model.linear
 * (official_weights.py:418-437) within the fp32 accumulation-order tolerance.
 * anvilq_w4a16_gemm(_ex) routes M >= ANVILQ_VERIFY_TC_MIN_M here by itself;
 * this entry point uses the tensor cores for any M >= 1 (launches of at most
 * 64 rows).  Requires G == 128, K % 128 == 0, N % 32 == 0 and 16-byte aligned
 * x, qweight, qzeros and scales (ANVILQ_ESHAPE otherwise).  Workspace: at
 * least anvilq_w4a16_gemm_workspace_size(M, K, N, G) bytes. */
#define ANVILQ_VERIFY_TC_MIN_M 16
int anvilq_w4a16_verify_gemm(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                             const uint16_t* scales, const uint16_t* bias, uint16_t* y,
                             int M, int K, int N, int G,
                             void* workspace, size_t workspace_bytes,
                             int* dev_err, anvilq_stream_t stream);

/* Resident-weight form of the verify GEMM.  anvilq_w4a16_tc_pack rewrites an
 * AWQ qweight [K][N/8] once (at model load) into the order the tensor-core
 * kernel's dequantisers consume -- the same nibbles, regrouped per 128-column
 * x 128-row unit so that each output column's 8 consecutive rows share one
 * 32-bit word (8 KB per unit, anvilq_w4a16_tc_pack_size bytes in all; columns
 * past N zero).  anvilq_w4a16_verify_gemm_packed then computes exactly what
 * anvilq_w4a16_verify_gemm computes from the original layout, with qzeros,
 * scales and bias unchanged.  G must be 128, K % 128 == 0, N % 32 == 0, and
 * `packed` 16-byte aligned (ANVILQ_ESHAPE otherwise). */
size_t anvilq_w4a16_tc_pack_size(int K, int N, int G);
int anvilq_w4a16_tc_pack(const int32_t* qweight, int32_t* packed, int K, int N, int G,
                         anvilq_stream_t stream);
int anvilq_w4a16_verify_gemm_packed(const uint16_t* x, const int32_t* packed, const int32_t* qzeros,
                                    const uint16_t* scales, const uint16_t* bias, uint16_t* y,
                                    int M, int K, int N, int G,
                                    void* workspace, size_t workspace_bytes,
                                    int* dev_err, anvilq_stream_t stream);

/* Batch-1 W4A16 GEMV with the decode step's neighbouring operations fused in.
 *
 * Replaces FP32Model.linear (official_weights.py:418-437) together with the
 * operation that produces its input and the one that consumes its output in
 * FP32Model.token (official_weights.py:451-509):
 *   x_mode ANVILQ_GEMV_X_HALF     input row k = x[k]            (x: fp16 [K])
 *          ANVILQ_GEMV_X_RMSNORM  input row k = fp16( r[k] * gamma[k] / sqrt(mean(r^2) + eps) )
 *                                 (x: fp32 residual r [K], gamma fp16 [K]; norm :411-416)
 *          ANVILQ_GEMV_X_SILU_MUL input row k = fp16( silu(g[k]) * u[k] )
 *                                 (x: fp16 [2K] = [g | u], a fused gate/up output; :493-501)
 *   y_mode ANVILQ_GEMV_Y_HALF     y fp16 [N] = result (+ bias)
 *          ANVILQ_GEMV_Y_RESIDUAL y fp32 [N] += result (+ bias), the residual add (:489, :503)
 *          ANVILQ_GEMV_Y_SILU_MUL the fused gate/up projection with the SiLU product
 *                                 in its epilogue: the weights' N = 2I columns are
 *                                 unit-interleaved (per 32 intermediate rows, 32 gate
 *                                 columns then 32 up columns, as for anvilq_w4a16_mlp),
 *                                 y fp16 [N/2] = fp16( silu(g) * u ) with g, u the
 *                                 fp16-rounded projections (:492-501) -- exactly what
 *                                 ANVILQ_GEMV_X_SILU_MUL computes from a stored [g | u],
 *                                 so the down projection then takes y as HALF input.
 *                                 No bias, N % 64 == 0, x_mode HALF or RMSNORM.
 * Same weights, workspace and requirements as anvilq_w4a16_gemm with M = 1
 * (fast-kernel shapes only: K % 16 == 0, G % 16 == 0, N % 32 == 0, 16-byte
 * aligned pointers; ANVILQ_ESHAPE otherwise).  flags: ANVILQ_GEMM_OVERLAP_PRIOR. */
#define ANVILQ_GEMV_X_HALF 0
#define ANVILQ_GEMV_X_RMSNORM 1
#define ANVILQ_GEMV_X_SILU_MUL 2
#define ANVILQ_GEMV_Y_HALF 0
#define ANVILQ_GEMV_Y_RESIDUAL 1
#define ANVILQ_GEMV_Y_SILU_MUL 2
int anvilq_w4a16_gemv_fused(const void* x, int x_mode, const uint16_t* gamma, float eps,
                            const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                            const uint16_t* bias, void* y, int y_mode, int K, int N, int G,
                            void* workspace, size_t workspace_bytes, int* dev_err, unsigned flags,
                            anvilq_stream_t stream);

/* The decode step's MLP in one launch (FP32Model.token's feed-forward block,
 * official_weights.py:491-503):
 *   h = fp16(RMSNorm(r) * gamma);  g, u = fp16(h @ W_gate), fp16(h @ W_up)
 *   r += fp16(silu(g) * u) @ W_down                      (r: fp32 [H], in place)
 * with the same operations and precisions as anvilq_w4a16_gemv_fused
 * (RMSNORM in, HALF out) on [gate | up] followed by anvilq_w4a16_gemv_fused
 * (SILU_MUL in, RESIDUAL out) on down; only the order of the down projection's
 * fp32 sums differs (per-row-slice partials summed over the cluster, then over
 * the bands in band order: bit-reproducible).
 * gate/up weights in unit-interleaved columns: for every 32 intermediate rows
 * u, 32 gate columns then 32 up columns, i.e. qweight [H][2I/8] with word
 * 8u + w = gate word 4u + w and word 8u + 4 + w = up word 4u + w (w < 4),
 * qzeros [H/G][2I/8] the same, scales [H/G][2I] with column 64u + i = gate
 * 32u + i and 64u + 32 + i = up 32u + i.  down: AWQ [I][H/8].  Needs
 * I % 32 == 0, H % 32 == 0, G % 16 == 0, 16-byte aligned pointers
 * (ANVILQ_ESHAPE / ANVILQ_EALIGN otherwise); workspace of
 * anvilq_w4a16_mlp_workspace_size bytes, counters zeroed before the first call
 * (the kernel re-arms them).  flags: ANVILQ_GEMM_OVERLAP_PRIOR. */
size_t anvilq_w4a16_mlp_workspace_size(int H, int I, int G);
int anvilq_w4a16_mlp(float* r, const uint16_t* gamma, float eps, const int32_t* gu_qweight,
                     const int32_t* gu_qzeros, const uint16_t* gu_scales, const int32_t* dn_qweight,
                     const int32_t* dn_qzeros, const uint16_t* dn_scales, int H, int I, int G, void* workspace,
                     size_t workspace_bytes, int* dev_err, unsigned flags, anvilq_stream_t stream);

/* The decode step's QKV projection with RoPE and the KV-cache append fused
 * into its epilogue: y = the GEMV of anvilq_w4a16_gemv_fused (same x_mode
 * inputs; N = (Hq + 2 Hkv) * D) rounded to fp16 (y_mode ANVILQ_GEMV_Y_HALF),
 * then exactly anvilq_rope_kv_append on that y -- q heads rotated into q_out,
 * k heads rotated into row *pos of k_cache, v heads copied to row *pos of
 * v_cache, *seqlen = *pos + 1 -- without y ever being stored.  Results are
 * bit-identical to the two calls whenever the GEMV plan keeps whole heads in
 * a band and one cluster per band (every decode QKV shape; otherwise equal
 * within the GEMV tolerance).  Replaces FP32Model.linear for the q/k/v
 * projections with the rotation and cache write that follow it
 * (official_weights.py:418-437, 439-449, 466-470).  D even, D <= 128; a *pos
 * outside [0, Tmax) sets ANVILQ_DEV_ERR_SEQLEN and writes nothing.
 * flags: ANVILQ_GEMM_OVERLAP_PRIOR. */
int anvilq_w4a16_gemv_qkv_rope(const void* x, int x_mode, const uint16_t* gamma, float eps,
                               const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                               const uint16_t* bias, int K, int G, const int32_t* pos, uint16_t* q_out,
                               uint16_t* k_cache, uint16_t* v_cache, int32_t* seqlen, int Hq, int Hkv, int D,
                               int Tmax, float theta, void* workspace, size_t workspace_bytes, int* dev_err,
                               unsigned flags, anvilq_stream_t stream);

/* Reference-order W4A16 GEMM: one thread per output column sums its K products
 * in increasing k from +0.0 with every binary32 multiply and add rounded
 * separately (no FMA), exactly as FP32Model.linear does
 * (official_weights.py:393-397, 418-437).  y32 (fp32 [M][N]) is therefore
 * bit-identical to the reference; slow, meant for verification.
 * Same layout and requirements as anvilq_w4a16_gemm (any G, no workspace). */
int anvilq_w4a16_gemm_exact(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                            const uint16_t* scales, const uint16_t* bias, float* y32,
                            int M, int K, int N, int G, int* dev_err, anvilq_stream_t stream);

/* Bit-accurate Q16.16 integer W4A16 GEMV: the integer golden model's projection
 * (anvil-q1/tests/official_weights.py:592-612) and the RTL datapath it
 * specifies (anvil-q1/design/SPEC.md:151-158):
 *   total = sum_k x[k] * (q - z) * round_away(scale * 2^16)   (exact integer)
 *   total += clip32(round_away(bias * 2^16)) * 65536           (bias may be NULL)
 *   y = clip32(round_away(total / 65536))
 * x_q16 int32 [M][K] and y_q16 int32 [M][N] are signed Q16.16; weights in the
 * AWQ layout of anvilq_w4a16_gemm, any G >= 1 (a partial last group allowed).
 * Results are bit-identical to the reference for every input.  Invalid scales
 * set ANVILQ_DEV_ERR_SCALE, a nonfinite bias ANVILQ_DEV_ERR_NONFINITE.
 * workspace: anvilq_w4a16_gemm_q16_workspace_size bytes, 16-byte aligned, with
 * the shared layout of ANVILQ_WORKSPACE_COUNTER_BYTES (the counter region is
 * neither read nor written; the scratch after it need not be zeroed). */
size_t anvilq_w4a16_gemm_q16_workspace_size(int M, int K, int N, int G);
int anvilq_w4a16_gemm_q16(const int32_t* x_q16, const int32_t* qweight, const int32_t* qzeros,
                          const uint16_t* scales, const uint16_t* bias, int32_t* y_q16,
                          int M, int K, int N, int G, void* workspace, size_t workspace_bytes,
                          int* dev_err, anvilq_stream_t stream);

/* ---------------------------------------------------------------------------
 * AWQ dequantisation of a whole [K][N] matrix, using the same in-register
 * unpack as the GEMM kernels.
 * Replaces dequant(qw, qz, h, lane) (anvil-q1/tests/verify.py:241-250) and
 * the weight f32(delta*scale) of official_weights.py:428-431:
 *   delta_out int8 [K][N] = u4 q - u4 z          (may be NULL)
 *   w_out   float  [K][N] = delta * scale, exact  (may be NULL; 0 where invalid)
 * Invalid scales set ANVILQ_DEV_ERR_SCALE in *dev_err.  Any G >= 1. */
int anvilq_awq_dequant(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                       int8_t* delta_out, float* w_out, int K, int N, int G,
                       int* dev_err, anvilq_stream_t stream);

/* AWQ packing of row-major 4-bit codes: codes uint8 [rows][N] (values 0..15,
 * higher bits ignored) <-> packed int32 [rows][N/8].
 * Replaces pack(values) (anvil-q1/tests/verify.py:252-253) and
 * pack_lanes / unpack_lanes (anvil-q1-fp/tests/awq_prepare.py:84-99), which
 * use the output-major transpose of the same layout. */
int anvilq_awq_pack(const uint8_t* codes, int32_t* packed, int rows, int N,
                    anvilq_stream_t stream);
int anvilq_awq_unpack(const int32_t* packed, uint8_t* codes, int rows, int N,
                      anvilq_stream_t stream);

/* ---------------------------------------------------------------------------
 * GQA decode attention over an fp16 KV cache (flash-decoding, split-KV).
 *
 * Replaces attention(q, keys, values) (anvil-q1-fp/tests/fp64_reference.py:164-170)
 * and the attention loop of FP32Model.token (anvil-q1/tests/official_weights.py:471-486),
 * batched: for sequence b and query head j,
 *   out[b][j] = softmax_t(q[b][j] . k[b][t][j / (Hq/Hkv)] * scale) @ v[b][t][...]
 * over positions t < seqlens[b].
 *   q fp16 [B][Hq][D], k_cache / v_cache fp16 [B][Tmax][Hkv][D],
 *   seqlens int32 [B] (device, each in [1, Tmax]), out fp16 [B][Hq][D].
 * scale <= 0 selects 1/sqrt(D).  Scores and the softmax run in fp32
 * (probabilities rounded to fp16 for the P.V product on the tensor cores).
 * Requirements: Hq % Hkv == 0, Hq / Hkv <= 8, D in {64, 128}, B*Hkv <= 16384,
 * 16-byte aligned q, caches and out; dev_err is required.  A sequence length
 * outside [1, Tmax] sets ANVILQ_DEV_ERR_SEQLEN and yields zeros for it.
 * workspace: at least anvilq_gqa_decode_workspace_size(...) bytes, layout as
 * described at ANVILQ_WORKSPACE_COUNTER_BYTES. */
size_t anvilq_gqa_decode_workspace_size(int B, int Hq, int Hkv, int D, int Tmax);
int anvilq_gqa_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                      const int32_t* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D, int Tmax,
                      float scale, void* workspace, size_t workspace_bytes, int* dev_err,
                      anvilq_stream_t stream);
/* The same with flags: ANVILQ_GEMM_OVERLAP_PRIOR launches the kernel with
 * programmatic dependent launch -- its CTAs may become resident while the work
 * enqueued before it (the QKV projection that writes q, the new cache row and
 * the lengths) still runs, and wait for that work before reading anything.
 * Results are identical to anvilq_gqa_decode. */
int anvilq_gqa_decode_ex(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                         const int32_t* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D, int Tmax,
                         float scale, void* workspace, size_t workspace_bytes, int* dev_err, unsigned flags,
                         anvilq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Decode-step operations around the GEMVs and the attention (batch 1).
 * Replace the pieces of FP32Model.token (anvil-q1/tests/official_weights.py:451-509).
 * flags: ANVILQ_GEMM_OVERLAP_PRIOR launches them as programmatic dependents
 * of the preceding kernel (they wait for it before touching memory). */

/* x (fp32 [H]) = E[*token] (fp16 table [V][H]); sets *argmax_key = 0 when given.
 * Embedding lookup, official_weights.py:463.  A token outside [0, V) sets
 * ANVILQ_DEV_ERR_TOKEN and row 0 is used. */
int anvilq_embed(const uint16_t* table, const int32_t* token, float* x, int H, int V,
                 unsigned long long* argmax_key, int* dev_err, unsigned flags, anvilq_stream_t stream);

/* RoPE and KV-cache append for the current position *pos (device int):
 * qkv fp16 [(Hq + 2 Hkv) * D] = [q | k | v]; q and k rotated in split halves,
 * angle = pos * theta^(-2i/D) (official_weights.py:439-449); q_out fp16
 * [Hq * D]; rotated k and v written to row *pos of k_cache / v_cache
 * fp16 [Tmax][Hkv][D] (:470); *seqlen = *pos + 1 when seqlen is given. */
int anvilq_rope_kv_append(const uint16_t* qkv, const int32_t* pos, uint16_t* q_out, uint16_t* k_cache,
                          uint16_t* v_cache, int32_t* seqlen, int Hq, int Hkv, int D, int Tmax, float theta,
                          int* dev_err, unsigned flags, anvilq_stream_t stream);
/* The same with the cache row given apart from the rotation's position: k and
 * v are written to row *row, rotated by angle *pos * theta^(-2i/D).  The
 * draft-tree verifier stages node m of a tree at row prefix + m while rotating
 * it to its own position, prefix + depth(m) (per-node positions and RoPE of
 * anvil-q3-ht2/design/SPEC.md:71-86).  Both in [0, Tmax), else
 * ANVILQ_DEV_ERR_SEQLEN and nothing is written. */
int anvilq_rope_kv_append_at(const uint16_t* qkv, const int32_t* pos, const int32_t* row, uint16_t* q_out,
                             uint16_t* k_cache, uint16_t* v_cache, int Hq, int Hkv, int D, int Tmax, float theta,
                             int* dev_err, unsigned flags, anvilq_stream_t stream);

/* ---- tensor-parallel column split with the all-gather fused in ---------------
 *
 * Replaces the column-split projection followed by its all-gather (the
 * 70B-class layer split: rank r of W holds output columns [r N/W, (r+1) N/W); reference analog:
 * the column interleave of anvil-q2/rtl/anvil_q2_gemv_lane.sv:117,187).
 *
 * Peer buffers: a rank exports any device pointer (e.g. a tensor's) as an IPC
 * handle (anvilq_peer_handle_size() bytes) plus its offset within its
 * allocation; the other ranks of the node import it and write into it with
 * plain stores over NVLink.  No multicast object is involved. */
size_t anvilq_peer_handle_size(void);
int anvilq_peer_export(const void* dev_ptr, void* handle_out, size_t* offset_out);
int anvilq_peer_import(const void* handle, size_t offset, void** base_out, void** dev_ptr_out);
int anvilq_peer_close(void* base);

/* This rank's slice of y = x W (+ bias) for an M = 1 projection (x fp16 [K],
 * the rank's qweight/qzeros/scales/bias of N columns as anvilq_w4a16_gemm)
 * stored as fp16 at columns [col_base, col_base + N) of every rank's full-width
 * output peer_y[r] (fp16 [n_full]; host array of `world` device pointers,
 * this rank's own included).  After all its stores the rank raises its flag,
 * value = its count of fused calls, in every rank's flag array peer_flags[r]
 * (unsigned [8] each, zero-initialised, host array of device pointers) and
 * waits, bounded by ~1 s (ANVILQ_DEV_ERR_TIMEOUT), until every rank's flag
 * has reached that count; *epoch (device, this rank's, starts at 0) advances
 * by one.  When the call completes on `stream` the full row is in
 * peer_y[rank].  Every rank must make the same sequence of calls, and a
 * peer_y buffer must not be written again until every rank has passed a
 * later fused call (alternate two or more buffers).  The workspace is as for
 * anvilq_w4a16_gemm (its counter region holds the completion tickets).
 * The slice is computed with the kernel and plan anvilq_w4a16_gemm uses for
 * these K, N (anvilq_w4a16_gemv_plan), so the gathered row is bit-identical
 * to a GEMV on every rank followed by an all-gather; the stream-K kernel
 * stores each finished 256-column band with 16-byte stores.
 * After ANVILQ_DEV_ERR_TIMEOUT (a rank that never made the call) *epoch has
 * still advanced and peer_y[rank] may lack other ranks' slices: the ranks'
 * flags and epochs no longer agree, so every rank must zero its flag array
 * and epoch (and rewrite the outputs) before the next fused call.
 * flags: ANVILQ_GEMM_OVERLAP_PRIOR. */
int anvilq_w4a16_gemv_allgather(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                                const uint16_t* scales, const uint16_t* bias, int K, int N, int G, int rank,
                                int world, int col_base, int n_full, uint16_t* const* peer_y,
                                unsigned int* const* peer_flags, unsigned int* epoch, void* workspace,
                                size_t workspace_bytes, int* dev_err, unsigned flags, anvilq_stream_t stream);

/* The same fused call under an explicit stream-K plan (kernel ANVILQ_GEMV_KERNEL_STREAM,
 * e.g. one CTA shape for every slice of a rank's chain; any other kernel:
 * ANVILQ_EINVAL), with one more flag:
 *
 * ANVILQ_GATHER_DEFERRED: the call raises its flag and advances *epoch without
 * waiting for the other ranks.  Instead, before reading x, every CTA waits
 * (bounded by ~1 s, ANVILQ_DEV_ERR_TIMEOUT) until every rank's flag has reached
 * the count of the previous fused call -- so x may be the previous call's
 * gathered row (a chain of projections whose exchange overlaps the next
 * projection's weight stream), and no rank still reads the output buffer this
 * call overwrites when two or more buffers alternate.  The gathered row of a
 * deferred call is complete on this rank only once every rank's flag has
 * reached its count: the next deferred call waits for that before reading x,
 * and anvilq_peer_wait makes it complete for any other consumer (end a chain
 * with it).  Buffer reuse: with S output buffers alternating, another rank's
 * call e + S may overwrite the row of call e as soon as every rank has raised
 * the flag of call e + S - 1 -- so on every rank, whatever reads the row of
 * call e other than call e + 1 must be enqueued before that rank's call
 * e + S - 1.  Same values as the plain fused call, and as a GEMV under `plan`
 * followed by an all-gather, bit for bit.
 * flags: ANVILQ_GEMM_OVERLAP_PRIOR, ANVILQ_GATHER_DEFERRED. */
#define ANVILQ_GATHER_DEFERRED 2u
int anvilq_w4a16_gemv_allgather_planned(const uint16_t* x, const int32_t* qweight, const int32_t* qzeros,
                                        const uint16_t* scales, const uint16_t* bias, int K, int N, int G,
                                        int rank, int world, int col_base, int n_full, uint16_t* const* peer_y,
                                        unsigned int* const* peer_flags, unsigned int* epoch,
                                        const anvilq_gemv_plan* plan, void* workspace, size_t workspace_bytes,
                                        int* dev_err, unsigned flags, anvilq_stream_t stream);

/* Waits on `stream` (one thread, bounded by ~1 s: ANVILQ_DEV_ERR_TIMEOUT) until
 * flags[0 .. world) -- this rank's flag array, peer_flags[rank] of the fused
 * calls -- have all reached *epoch, i.e. until the last fused call's gathered
 * row is complete on this rank. */
int anvilq_peer_wait(const unsigned int* flags, int world, const unsigned int* epoch, int* dev_err,
                     anvilq_stream_t stream);

/* ---- every decoder layer of one decode token in one persistent kernel ---------
 *
 * Replaces the per-layer body of FP32Model.token (anvil-q1/tests/official_weights.py:462-503)
 * / QwenFP64.step (anvil-q1-fp/tests/fp64_reference.py:210-246) for all L layers
 * of a Qwen2-architecture W4A16 AWQ model at batch 1: x = E[*token] (the
 * embedding row), then per layer h = rmsnorm(x) gamma_in; q,k,v = h W_qkv + b
 * with split-half RoPE at *pos (theta); k, v written to row *pos of the
 * layer's caches [Tmax][KVH][D]; causal attention over rows [0, *pos];
 * x += attn W_o; h = rmsnorm(x) gamma_post; x += (silu(h W_gate) (h W_up)) W_down.
 * The final residual goes to x_out (fp32 [H]) for anvilq_lmhead_argmax;
 * *seqlen = *pos + 1; *argmax_key = 0 when given.  Numerics as the per-kernel
 * path (anvilq_w4a16_gemv_qkv_rope, anvilq_gqa_decode, anvilq_w4a16_gemv_fused):
 * binary16 activations, fp32 residual and accumulation; attention scores,
 * softmax and P.V in fp32.
 *
 * `layers` is a DEVICE array of L descriptors.  Per layer: qkv = the q, k, v
 * projections concatenated along N (AWQ [H][(QH+2KVH) D / 8], bias fp16
 * [(QH+2KVH) D] or NULL); o [QH D][H / 8]; gu = gate and up concatenated
 * along N ([H][2 I / 8]); down [I][H / 8]; gammas fp16 [H]; caches fp16.
 * The AWQ tensors are given COLUMN-BLOCKED (anvilq_block_columns), so that the
 * slice a CTA streams is one contiguous range: qkv in blocks of one head
 * (qweight and qzeros D / 8 words, scales D halves), o and down in blocks of
 * 4 words (scales 32 halves): a block's rows follow one another.  gate and up
 * are interleaved by 32-column unit u: gu_qweight [I/32][H][8] holds in words
 * 0-3 of a row the gate's columns 32u..32u+31 and in words 4-7 the up's,
 * gu_qzeros [I/32][H/G][8] likewise, gu_scales [I/32][H/G][64] the gate's 32
 * scales then the up's (a column permutation of whole AWQ words: the packing
 * is unchanged).
 * Requirements: G == 128, H % 128 == 0, I % 128 == 0, QH % KVH == 0,
 * QH / KVH <= 8, D in {64, 128}, (QH D) % 128 == 0, 16-byte aligned tensors,
 * and one SM's shared memory must hold a CTA's slices of a layer (ANVILQ_ESHAPE
 * otherwise: larger models use the per-kernel path).  The grid is one CTA per
 * SM, launched cooperatively: CTAs wait on one another's counters (bounded,
 * ~1 s, then ANVILQ_DEV_ERR_TIMEOUT and the launch gives up).  An invalid
 * *token or *pos sets ANVILQ_DEV_ERR_TOKEN / _SEQLEN and does nothing; a
 * tensor of the table that is not 16-byte aligned sets ANVILQ_DEV_ERR_ALIGN
 * and the launch gives up before copying from it (x_out is then not written).
 * workspace: anvilq_decode_layers_workspace_size bytes, 256-byte aligned,
 * zero-filled once (every launch leaves its counters zero). */
/* dst[b][r][e] = src[r][b * block + e] for a row-major [rows][cols] matrix of
 * elem_bytes-byte elements (2 or 4): its column blocks of `block` elements
 * stored one after another.  block * elem_bytes % 16 == 0, cols % block == 0,
 * 16-byte aligned pointers.  A layout step for anvilq_decode_layers; no
 * counterpart computation in the reference (the AWQ words are moved, never changed). */
int anvilq_block_columns(const void* src, void* dst, int rows, int cols, int block, int elem_bytes,
                         anvilq_stream_t stream);
typedef struct anvilq_decode_layer {
  const int32_t* qkv_qweight;
  const int32_t* qkv_qzeros;
  const uint16_t* qkv_scales;
  const uint16_t* qkv_bias;
  const int32_t* o_qweight;
  const int32_t* o_qzeros;
  const uint16_t* o_scales;
  const int32_t* gu_qweight;
  const int32_t* gu_qzeros;
  const uint16_t* gu_scales;
  const int32_t* down_qweight;
  const int32_t* down_qzeros;
  const uint16_t* down_scales;
  const uint16_t* gamma_in;
  const uint16_t* gamma_post;
  uint16_t* k_cache;
  uint16_t* v_cache;
} anvilq_decode_layer;
size_t anvilq_decode_layers_workspace_size(int L, int H, int I, int QH, int KVH, int D, int G, int Tmax);
int anvilq_decode_layers(const anvilq_decode_layer* layers, int L, int H, int I, int QH, int KVH, int D, int G,
                         int Tmax, float eps, float theta, const uint16_t* embedding, int V, const int32_t* token,
                         const int32_t* pos, int32_t* seqlen, float* x_out, unsigned long long* argmax_key,
                         void* workspace, size_t workspace_bytes, int* dev_err, anvilq_stream_t stream);

/* Tied fp16 lm_head with the final RMSNorm and greedy argmax fused:
 * h = x * gamma / sqrt(mean(x^2) + eps) in fp32 (official_weights.py:504),
 * logits[v] = h . E[v] (:505-506; written when logits != NULL), and
 * *argmax_key = max over v of an orderable (logit, lowest v) key, combined
 * with atomicMax (the key must be 0 before the call: anvilq_embed clears it).
 * H % 64 == 0, H <= 16384, table 16-byte aligned. */
int anvilq_lmhead_argmax(const float* x, const uint16_t* gamma, float eps, const uint16_t* table, float* logits,
                         unsigned long long* argmax_key, int H, int V, unsigned flags, anvilq_stream_t stream);

/* *token = the row encoded in *argmax_key (greedy choice, lowest index on
 * ties as in anvil-q4/tests/transformer_reference.py:212-217); *pos += 1
 * when pos is given.  Keeps the autoregressive loop on the device. */
int anvilq_argmax_commit(const unsigned long long* argmax_key, int32_t* token, int32_t* pos, unsigned flags,
                         anvilq_stream_t stream);

/* GQA decode attention that allocates nothing and takes no workspace.
 *
 * No counterpart in the reference: an addition for callers that cannot give
 * this library device memory -- a host whose allocator already owns all of
 * HBM and offers nothing per call, a binding that can only pass the tensors it
 * was handed, or a decode loop that must not trigger cudaMalloc's implicit
 * device synchronisation.
 *
 * Same operation, arguments and requirements as anvilq_gqa_decode, minus the
 * workspace.  The split-KV scratch is a fixed 4 MiB array inside the library's
 * device image, held by every GPU that loads the library until the process
 * exits; a request whose scratch would exceed it is rejected with
 * ANVILQ_ENOSCRATCH before anything is launched.  Nothing is allocated: no
 * cudaMalloc, no cudaFree, no allocating library call.
 * The first call on a device looks up the array's device address (once per
 * device, with that device current); make that first call before any stream
 * capture.  Every call on the device shares the one array, so calls that may
 * overlap on the GPU (different streams without ordering) race and must not
 * be issued; calls ordered on one stream are fine.  Each call zeroes the
 * array's counters on `stream` before its kernel. */
int anvilq_gqa_decode_noalloc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                              const int32_t* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D,
                              int Tmax, float scale, int* dev_err, anvilq_stream_t stream);

/* ---- INT8 KV cache (Anvil-Q4 per-head encoding with FP32 escape) ------------
 *
 * Format (anvil-q4/design/SPEC.md:209-235, rational model
 * anvil-q4/tests/cache_reference.py:54-83), one (token, kv head) row of D values
 * at a time: scale = fp32(maxabs / 127) (1.0 for an all-+0 row), code =
 * clamp(round-half-even(|fp32(v / scale)|), 127) with v's sign, value =
 * fp32(code * scale); a row holding NaN, +-inf or -0.0, or whose scale
 * underflows to 0, escapes: metadata 0x7FC00000, codes 0, and its values (NaN
 * made 0x7FC00000) in the fp32 escape payload.  Layout:
 *   codes    int8   [B][Tmax][Hkv][D]
 *   meta     uint32 [B][Hkv][Tmax]   (scale bits or 0x7FC00000)
 *   escape   float  [B][Tmax][Hkv][D] (optional; zero for ordinary rows)
 *
 * anvilq_kv_int8_store encodes rows src [B][T][H][D] (fp16 when src_half, else
 * fp32) into positions start[b] + t of sequence b (start: device int32 [B], or
 * NULL for 0); codes and metadata are bit-identical to the rational model.
 * Without an escape buffer an escaped row sets ANVILQ_DEV_ERR_NONFINITE.
 * D <= 256; a position outside [0, Tmax) sets ANVILQ_DEV_ERR_SEQLEN. */
int anvilq_kv_int8_store(const void* src, int src_half, int B, int T, int H, int D, int Tmax,
                         const int32_t* start, int8_t* codes, uint32_t* meta, float* escape, int* dev_err,
                         anvilq_stream_t stream);

/* anvilq_gqa_decode over INT8 caches of the format above: scores use each K row's
 * scale (escaped rows their fp32 payload, rounded to fp16 for the tensor cores),
 * the V scales are folded into the probabilities.  Same q, seqlens, out, scale
 * and workspace (anvilq_gqa_decode_workspace_size) as anvilq_gqa_decode;
 * Tmax % 16 == 0; all pointers 16-byte aligned.  An escaped row without an
 * escape payload sets ANVILQ_DEV_ERR_NONFINITE and counts as zeros. */
int anvilq_gqa_decode_int8(const uint16_t* q, const int8_t* k_codes, const uint32_t* k_meta, const float* k_escape,
                           const int8_t* v_codes, const uint32_t* v_meta, const float* v_escape,
                           const int32_t* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D, int Tmax,
                           float scale, void* workspace, size_t workspace_bytes, int* dev_err,
                           anvilq_stream_t stream);

/* anvilq_gqa_decode over a PAGED fp16 cache (the Anvil-Q4 page table,
 * anvil-q4/design/SPEC.md:205-208: an entry's bit 31 marks it valid, bits 30:0
 * give the physical page).  Logical position t of sequence b lives in row
 * t % page_tokens of physical page page_table[b][t / page_tokens] of the pools
 *   k_pool / v_pool fp16 [num_pages][page_tokens][Hkv][D],
 *   page_table uint32 [B][max_pages] (device).
 * A sequence holds at most Tmax = page_tokens * max_pages positions; q, seqlens,
 * out, scale and the workspace (anvilq_gqa_decode_workspace_size(B, Hq, Hkv, D,
 * Tmax)) are as for anvilq_gqa_decode, whose result this equals bit for bit
 * for the same logical cache contents.  page_tokens % 16 == 0.  A live page
 * whose entry is not valid or names a page >= num_pages sets
 * ANVILQ_DEV_ERR_PAGE (the output is then not to be used). */
int anvilq_gqa_decode_paged(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                            const uint32_t* page_table, const int32_t* seqlens, uint16_t* out, int B, int Hq, int Hkv,
                            int D, int page_tokens, int max_pages, int num_pages, float scale, void* workspace,
                            size_t workspace_bytes, int* dev_err, anvilq_stream_t stream);

/* ---- tree attention of speculative draft nodes -----------------------------
 *
 * Replaces the per-node causal tree attention of the batched draft-tree decoder
 * (anvil-q3-ht2/design/SPEC.md:71-86) under the ancestor contract of
 * anvil-q1-ht3/design/SPEC.md:528-533.  Draft node m (0 <= m < M <= 32) attends
 * to cache rows [0, prefix_len) -- the committed prefix -- and to the rows
 * prefix_len + j of the nodes j whose bit is set in ancestors[m] (device
 * uint32 [M]); node j's K/V must already be in those rows.  A mask must hold
 * bit m, no bit above m, and every ancestor's own mask (else
 * ANVILQ_DEV_ERR_TREE; the output is then not to be used).
 *   q fp16 [M][Hq][D], k_cache / v_cache fp16 [Tmax][Hkv][D] (one sequence),
 *   out fp16 [M][Hq][D]; prefix_len + M <= Tmax, Tmax % 16 == 0,
 *   Hq % Hkv == 0, Hq / Hkv <= 8, D in {64, 128}, 16-byte aligned pointers.
 * scale <= 0 selects 1/sqrt(D).  workspace: at least
 * anvilq_tree_attention_workspace_size(M, Hq, Hkv, D, Tmax) bytes, layout as
 * described at ANVILQ_WORKSPACE_COUNTER_BYTES.  No counterpart function in the
 * reference's Python goldens: the golden is attention() of
 * anvil-q1-fp/tests/fp64_reference.py:164-170 over each node's key rows. */
size_t anvilq_tree_attention_workspace_size(int M, int Hq, int Hkv, int D, int Tmax);
int anvilq_tree_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                          const uint32_t* ancestors, int prefix_len, uint16_t* out, int M, int Hq, int Hkv, int D,
                          int Tmax, float scale, void* workspace, size_t workspace_bytes, int* dev_err,
                          anvilq_stream_t stream);

/* ---- M-row decode operations (the batched verification of M draft tokens) ----
 *
 * The prologues / epilogues that the batch-1 GEMV fuses, for M rows whose
 * projections run as M-row GEMMs (official_weights.py:466-503 per token):
 * anvilq_rmsnorm_rows: out fp16 [M][H] = x * gamma / sqrt(mean(x^2) + eps), x fp32 [M][H];
 * anvilq_residual_add_rows: x fp32 [M][H] += y fp16 [M][H];
 * anvilq_silu_mul_rows: out fp16 [M][I] = silu(g) * u with [g | u] = gu fp16 [M][2I].
 * flags: ANVILQ_GEMM_OVERLAP_PRIOR. */
int anvilq_rmsnorm_rows(const float* x, const uint16_t* gamma, float eps, uint16_t* out, int M, int H,
                        unsigned flags, anvilq_stream_t stream);
int anvilq_residual_add_rows(float* x, const uint16_t* y, int M, int H, unsigned flags, anvilq_stream_t stream);
int anvilq_silu_mul_rows(const uint16_t* gu, uint16_t* out, int M, int I, unsigned flags, anvilq_stream_t stream);

/* ---- legacy KV-cache codecs of the Q16.16 datapath ---------------------------
 *
 * The legacy quantised caches of the Anvil-Q chips (anvil-q4/design/SPEC.md:250-262;
 * model anvil-q4/tests/legacy_reference.py:71-97 cache_block, payload layout
 * :186-203): format 1 INT8 symmetric, 2 INT4 symmetric, 3 INT4 asymmetric, one
 * power-of-two exponent (and for format 3 a zero point) per block of `block`
 * consecutive Q16.16 values of a head (1 <= block <= 64; a head's last block may
 * be shorter).  Rows of H heads x D values:
 *   values   int32  [rows][H * D]        Q16.16
 *   payload  uint32 [rows][H * B * W]    B = ceil(D / block), W = ceil(block * bits / 32),
 *                                        codes in ascending bytes / nibbles, padding zero
 *   metadata uint32 [rows][H * B]        exponent | (zero point & 15) << 8
 * Encoding is bit-identical to the reference model; decoding gives
 * sat32((code - z) 2^e) and sets ANVILQ_DEV_ERR_CODEC for an exponent past
 * the format's range, reserved metadata bits, the forbidden symmetric codes
 * (-128, -8) or nonzero padding. */
int anvilq_legacy_kv_encode(const int32_t* values, uint32_t* payload, uint32_t* metadata, int rows, int H, int D,
                            int block, int format, anvilq_stream_t stream);
int anvilq_legacy_kv_decode(const uint32_t* payload, const uint32_t* metadata, int32_t* values, int rows, int H,
                            int D, int block, int format, int* dev_err, anvilq_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ANVILQ_H */
