// verify_gemm_tc.cu -- W4A16 AWQ small-M GEMM (the speculative-verify batch,
// up to 64 token rows per launch) on the fifth-generation tensor cores:
// tcgen05.mma with the dequantised weights in TMEM, the activations in shared
// memory and fp32 accumulators in TMEM.
//
// Reference semantics: M independent rows of FP32Model.linear
// (anvil-q1/tests/official_weights.py:418-437) -- the M-token batched projection
// of anvil-q3-ht2/design/SPEC.md:81-86 and the verify step of
// anvil-q4/design/SPEC.md:271-272 -- y[m][c] = sum_k x[m][k] (q[k][c] - z[g][c]) s[g][c].
//
// Orientation ("swap AB").  One MMA computes D[col][token] = sum_k A[col][k] B[token][k]:
// A = the integer deltas of 128 output columns (MMA M = 128, one TMEM lane per
// column), B = the activations (MMA N = MPAD = M rounded up to 16, one TMEM
// column per token; rows past M are zero-filled by the TMA unit), K = 16 per
// instruction.
//
// Exactness.  The tensor cores are fed q - z, which binary16 holds exactly
// (|q - z| <= 15), never binary16(delta * scale): the products with the fp16
// activations are exact and accumulate in fp32 in TMEM over one AWQ group
// (128 rows, 8 instructions).  The epilogue applies the group's scale in fp32,
// y += s * D_g.
//
// Why A lives in TMEM.  With A in shared memory every unit moves 64 KB through
// the shared-memory port (the dequantiser writes 32 KB, the tensor core reads
// them back at ~140 B/clk), twice the time the unit's 8 KB of int4 weights
// take to arrive from HBM.  Here the dequantisers write A straight from
// registers into TMEM (tcgen05.st) and the MMA reads it from there; shared
// memory carries only the TMA-staged int4 tile, the activations and the
// unit's zero points and scales.
//
// The dequantiser's transpose.  A TMEM lane holds one output column along k,
// while a qweight word holds 8 columns at one k.  The qweight tile is staged by
// one TMA box of 128 rows x 64 bytes with the 64-byte swizzle (16-byte chunk c
// of row k lands at chunk c ^ ((k >> 1) & 3)), so the 16 bytes of a 32-column
// lane quarter in 8 consecutive rows fall in 8 different bank groups.  For
// each block of 8 rows a warp loads those 128 bytes (one word per lane: lane
// 4r + l holds word l of row awq_lane(r)), then an 8 x 8 nibble transpose over
// the lanes {4r + l : r} (shfl.xor 16 / 8 / 4 with prmt and nibble masks)
// leaves lane 4r + l with the 8 rows of one column, rows 2i and 2i+1 in the
// nibble pairs the binary16 magic-number unpack reads (awq_common.cuh).  After
// the transpose nibble position r of a word is AWQ lane awq_lane(r), so lane
// 4r + l of quarter q holds tile column 32q + 8l + awq_lane(r); the epilogue
// uses the same mapping.
//
// Work split (stream-K).  A unit is (column tile of 128 columns, group of 128
// rows); units are ordered tile-major and split into equal contiguous ranges,
// one per CTA of a persistent grid (one CTA per SM).  A tile covered by one CTA
// is written directly; a tile split between CTAs leaves one fp32 partial per
// CTA in the workspace ([cta][slot][column][row]: a column's rows contiguous,
// moved as 16-byte vectors) and the warp that arrives last at the (tile, warp)
// ticket sums them in CTA order, two contributors' loads in flight at a time
// -- deterministic, no spin-wait on other CTAs.
//
// Warp roles (14 warps, one CTA per SM):
//   0-3   epilogue: warp q reads TMEM lanes 32q..32q+31 (one output column each)
//   4-11  dequantisers: warp 4 + 4e + q writes lane quarter q (all 128 rows) of
//         the units e, e + 2, e + 4, ...: two teams, two units in flight
//   12    TMA producer (the whole warp loops, one elected lane issues)
//   13    MMA issuer (likewise) and TMEM owner
// Pipelines (mbarriers): a TMA ring of kSR stages carrying a unit's int4 tile,
// activation tile, zero points and scales (full: tx bytes; empty: MMA commit
// and the 4 epilogue warps, which read the scales), four TMEM A buffers (full:
// the 4 warps of a dequant team; empty: MMA commit), 4 TMEM accumulators (full:
// MMA commit; empty: 4 epilogue warps).  Waits spin on try_wait (no suspend-time
// hint) and every wait is bounded (1 s); on expiry the CTA
// raises ANVILQ_DEV_ERR_TIMEOUT, all roles leave their loops, copies and MMAs
// in flight are drained (bounded) and TMEM is released.
//
// B (activations) in shared memory: K-major, 128-byte swizzle, row = token
// (128 bytes = 64 k), 8-row atoms of 1024 bytes (stride byte offset 1024); the
// k-th 16-column slice starts 32 k bytes into the atom.  A in TMEM: lane =
// column, 32-bit column j = (k = 2j, 2j+1) as binary16 (low half = even k).
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
namespace tc_verify {

constexpr int kEpiWarps = 4;
constexpr int kDeqWarps = 8;
constexpr int kProducerWarp = kEpiWarps + kDeqWarps;   // 12
constexpr int kMmaWarp = kProducerWarp + 1;            // 13
constexpr int kThreads = (kMmaWarp + 1) * 32;          // 448
constexpr int kTileCols = 128;                         // MMA M
constexpr int kTileWords = kTileCols / 8;              // 16 qweight words per row
constexpr int kGroupRows = 128;                        // AWQ group = one accumulation
constexpr int kKSteps = kGroupRows / 16;               // 8 MMAs per unit
constexpr int kNAcc = 4;                               // TMEM accumulators
constexpr int kSA = 4;                                 // TMEM A buffers (columns 256 .. 511)
constexpr int kQBytes = kGroupRows * kTileWords * 4;   // 8 KB: [128 rows][64 B], 64-byte swizzle
constexpr int kZBytes = kTileWords * 4;                // qzeros of one unit: 64 B
constexpr int kSBytes = kTileCols * 2;                 // scales of one unit: 256 B
constexpr int kMetaBytes = kZBytes + kSBytes;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA = 256;                       // A buffers: columns 256 + 64 a
constexpr uint32_t kACols = kGroupRows / 2;            // 64 columns of binary16 pairs
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

template <int MPAD>
struct Cfg {
  static_assert(MPAD % 16 == 0 && MPAD >= 16 && MPAD <= 64, "MMA N = 16..64 tokens");
  static constexpr int kXBytes = MPAD * 256;                 // 2 boxes x MPAD rows x 128 B
  static constexpr int kStageR = kXBytes + kQBytes;          // multiple of 1024
  static constexpr int kSR = (180 * 1024) / kStageR < 12 ? (180 * 1024) / kStageR : 12;
  static constexpr int kOffMeta = kSR * kStageR;             // [kSR][kMetaBytes]: zeros, scales
  static constexpr int kOffBar = kOffMeta + kSR * kMetaBytes;
  static constexpr int kNumBars = 3 * kSR + 2 * kSA + 2 * kNAcc;
  static constexpr int kOffMisc = kOffBar + 8 * kNumBars;
  static constexpr int kSmem = kOffMisc + 64 + 1024;        // + slack to align the base to 1024
  static_assert(kNAcc * MPAD <= (int)kTmemA, "accumulators below the A buffers");
  static_assert(kStageR % 1024 == 0, "swizzled boxes need 1024-byte alignment");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
};

struct Params {
  const int32_t* packed;   // PACKED: [units][8 KB] (anvilq_w4a16_tc_pack)
  const int32_t* qzeros;   // [K/128][W8]
  const __half* scales;    // [K/128][N]
  const __half* bias;      // [N] or null
  __half* y;               // [M][N]
  float* partials;         // [P][2][128][MPAD]
  int* tickets;            // [tiles][4]: one per epilogue warp
  int* dev_err;
  int M, K, N, W8;
  int tiles, groups;
  long long units;         // tiles * groups
};

// ---- PTX wrappers -----------------------------------------------------------
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
// Waits for the phase of `parity` to complete; gives up after kWaitLimitNs or
// once another role has raised the CTA's abort flag.  A wait whose phase has
// already completed costs a single try_wait.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag || globaltimer() - t0 > kWaitLimitNs) return false;
  }
}
// Bounded wait that ignores the abort flag: drains copies and MMAs in flight.
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > kWaitLimitNs) return;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// One lane of a converged warp: the issuing roles keep the whole warp in the
// loop so addresses and descriptors stay warp-uniform.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile("{\n .reg .pred e;\n .reg .b32 r;\n elect.sync r|e, 0xffffffff;\n selp.u32 %0, 1, 0, e;\n}"
               : "=r"(pred));
  return pred != 0;
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 (binary16 operands, fp32 accumulate).
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  const uint32_t mask = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n}" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask)
      : "memory");
}
// 32 lanes x 16 consecutive 32-bit TMEM columns: thread t gets lane (base lane + t).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// the same load without the wait (the caller waits once for several loads)
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// thread t writes 32 consecutive 32-bit columns of lane (base lane + t)
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// the same store without the wait (the caller waits once for several stores)
__device__ __forceinline__ void tmem_st32_nowait(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// Shared-memory matrix descriptor (tcgen05): start, leading and stride byte
// offsets in 16-byte units, version 1, base offset 0, layout type in bits 61..63
// (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), A and B
// binary16 (formats 0), both K-major (A from TMEM is always K-major), N >> 3 at
// bit 17, M >> 4 at bit 24.
template <int MPAD>
__host__ __device__ constexpr uint32_t instr_desc() {
  return (1u << 4) | ((uint32_t)(MPAD >> 3) << 17) | ((uint32_t)(kTileCols >> 4) << 24);
}

__device__ __forceinline__ long long range_begin(long long c, long long units, long long P) {
  return c * units / P;
}
__device__ __forceinline__ int owner_of(long long u, long long units, long long P) {
  return (int)(((u + 1) * P + units - 1) / units - 1);
}

// AWQ lane held by nibble position j of a packed word: (0,2,4,6,1,3,5,7)[j]
// (anvil-q1/tests/verify.py:38).
__device__ __forceinline__ int awq_lane(int j) { return j < 4 ? 2 * j : 2 * j - 7; }

// One step of the 8 x 8 nibble transpose across lanes {4r + l}: with D the
// step's bit of r, nibble position j takes the partner's nibble j ^ D whenever
// bit D of j differs from bit D of r.
// The selector, rotation and mask depend only on the lane and are hoisted.
template <int D>
__device__ __forceinline__ uint32_t transpose_step(uint32_t v, int r) {
  const uint32_t p = __shfl_xor_sync(0xffffffffu, v, 4 * D);
  if (D == 4) return __byte_perm(v, p, (r & 4) ? 0x3276 : 0x5410);   // 16-bit halves
  if (D == 2) return __byte_perm(v, p, (r & 2) ? 0x3715 : 0x6240);   // bytes
  // nibbles: odd r keeps the high nibble of every byte and takes the partner's
  // high nibbles shifted down (a rotate by 28 whose wrapped bits are masked
  // off), even r the reverse with a rotate by 4
  const uint32_t keep = (r & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
  const uint32_t moved = __funnelshift_l(p, p, (r & 1) ? 28 : 4);
  return (v & keep) | (moved & ~keep);
}

// PACKED: the int4 weights come pre-transposed (anvilq_w4a16_tc_pack): each
// unit is 8 KB in the order the dequantisers consume, fetched by one bulk copy,
// and the nibble transpose is skipped.
template <int MPAD, bool PACKED>
__global__ void __launch_bounds__(kThreads, 1)
    verify_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmx,
                     const Params p) {
  using C = Cfg<MPAD>;
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  unsigned char* smem = smem_raw + (base - raw0);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  const long long P = gridDim.x;
  const long long u0 = range_begin(blockIdx.x, p.units, P);
  const int nunits = (int)(range_begin(blockIdx.x + 1, p.units, P) - u0);

  const uint32_t bars = base + C::kOffBar;
  auto full_r = [&](int s) { return bars + 8u * s; };
  auto empty_r = [&](int s) { return bars + 8u * (C::kSR + s); };
  auto empty_m = [&](int s) { return bars + 8u * (2 * C::kSR + s); };
  auto full_a = [&](int a) { return bars + 8u * (3 * C::kSR + a); };
  auto empty_a = [&](int a) { return bars + 8u * (3 * C::kSR + kSA + a); };
  auto acc_full = [&](int b) { return bars + 8u * (3 * C::kSR + 2 * kSA + b); };
  auto acc_empty = [&](int b) { return bars + 8u * (3 * C::kSR + 2 * kSA + kNAcc + b); };
  const uint32_t meta0 = base + C::kOffMeta;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

  // programmatic dependent launch (a no-op without the launch attribute): the
  // next kernel on the stream may launch now; the activations (TMA) and every
  // global write (epilogue) wait for this kernel's predecessor below
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // unit u0 + li = (column tile t, group g), advanced without divisions
  const int first_t = (int)(u0 / p.groups), first_g = (int)(u0 % p.groups);
  auto next_unit = [&](int& t, int& g) {
    if (++g == p.groups) {
      g = 0;
      ++t;
    }
  };
  // one unit's copies into stage li % kSR: weights, zero points and scales
  // (never written by a preceding kernel), then, separately, the activations
  auto issue_weights = [&](int li, int t, int g) {
    const int s = li % C::kSR;
    // the last column tile copies only its columns below N
    const uint32_t zb = (uint32_t)min(kTileWords, p.W8 - t * kTileWords) * 4;
    const uint32_t sb = (uint32_t)min(kTileCols, p.N - t * kTileCols) * 2;
    const uint32_t dst = base + s * C::kStageR;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(full_r(s)),
                 "r"(C::kStageR + zb + sb)
                 : "memory");
    if (PACKED)
      bulk_copy(dst + C::kXBytes, p.packed + (size_t)(u0 + li) * (kQBytes / 4), kQBytes, full_r(s));
    else
      tma_2d(dst + C::kXBytes, &tmq, t * kTileWords, g * kGroupRows, full_r(s));
    bulk_copy(meta0 + s * kMetaBytes, p.qzeros + (size_t)g * p.W8 + t * kTileWords, zb, full_r(s));
    bulk_copy(meta0 + s * kMetaBytes + kZBytes, p.scales + (size_t)g * p.N + t * kTileCols, sb, full_r(s));
  };
  auto issue_acts = [&](int li, int g) {
    const int s = li % C::kSR;
    const uint32_t dst = base + s * C::kStageR;
    tma_2d(dst, &tmx, g * kGroupRows, 0, full_r(s));
    tma_2d(dst + MPAD * 128, &tmx, g * kGroupRows + 64, 0, full_r(s));
  };
  // the producer warp initialises the barriers and sends the first few units'
  // copies before the CTA barrier, while the MMA warp allocates TMEM (a few: every
  // copy issued here delays the other roles' start by ~70 cycles)
  const int pro = min(min(C::kSR, 4), nunits);
  if (warp == kProducerWarp) {
    if (lane == 0) {
      for (int s = 0; s < C::kSR; ++s) {
        mbar_init(full_r(s), 1);
        mbar_init(empty_r(s), 1);
        mbar_init(empty_m(s), kEpiWarps);
      }
      for (int a = 0; a < kSA; ++a) {
        mbar_init(full_a(a), kDeqWarps / 2);
        mbar_init(empty_a(a), 1);
      }
      for (int b = 0; b < kNAcc; ++b) {
        mbar_init(acc_full(b), 1);
        mbar_init(acc_empty(b), kEpiWarps);
      }
      *s_abort = 0;
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      if (!PACKED) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmq) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmx) : "memory");
      int t = first_t, g = first_g;
      for (int li = 0; li < pro; ++li, next_unit(t, g)) issue_weights(li, t, g);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");   // x may come from the previous kernel
    if (lane == 0) {
      int t = first_t, g = first_g;
      for (int li = 0; li < pro; ++li, next_unit(t, g)) issue_acts(li, g);
    }
    __syncwarp();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  auto fail = [&]() {
    *s_abort = 1;
    if (p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_TIMEOUT);
  };

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------------- TMA
    int issued = pro;
    int t = first_t, g = first_g;
    for (int li = 0; li < pro; ++li) next_unit(t, g);
    for (int li = pro; li < nunits; ++li, next_unit(t, g)) {
      const int s = li % C::kSR;
      const uint32_t par = ((li / C::kSR) & 1) ^ 1;
      const bool ok = mbar_wait(empty_r(s), par, s_abort) && mbar_wait(empty_m(s), par, s_abort);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) fail();
        break;
      }
      if (elect_one()) {
        issue_weights(li, t, g);
        issue_acts(li, g);
      }
      __syncwarp();
      issued = li + 1;
    }
    if (*s_abort && lane == 0) {   // let the copies still in flight land before the CTA exits
      for (int li = std::max(0, issued - C::kSR); li < issued; ++li)
        mbar_drain(full_r(li % C::kSR), (li / C::kSR) & 1);
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA
    constexpr uint32_t idesc = instr_desc<MPAD>();
    int issued = 0;
    for (int li = 0; li < nunits; ++li) {
      const int s = li % C::kSR, a = li % kSA, b = li % kNAcc;
      // full_a implies full_r: the dequant team waited for the stage's copies
      // (activations included) before it dequantised and arrived
      const bool ok = mbar_wait(full_a(a), (li / kSA) & 1, s_abort) &&
                      mbar_wait(acc_empty(b), ((li / kNAcc) & 1) ^ 1, s_abort);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) fail();
        break;
      }
      tc_fence_after();
      const uint32_t x0 = base + s * C::kStageR;
      const uint32_t d = tmem + b * MPAD;
      const uint32_t at = tmem + kTmemA + a * kACols;
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < kKSteps; ++kk) {
          const uint64_t bd = smem_desc(x0 + (kk / 4) * MPAD * 128 + (kk % 4) * 32, 16, 1024, 2);
          tc_mma_ts(d, at + kk * 8, bd, idesc, kk > 0 ? 1u : 0u);
        }
        tc_commit(empty_r(s));
        tc_commit(empty_a(a));
        tc_commit(acc_full(b));
      }
      __syncwarp();
      issued = li + 1;
    }
    if (*s_abort && issued > 0 && lane == 0) {   // MMAs still running write TMEM: wait for the last commit
      const int li = issued - 1;
      mbar_drain(acc_full(li % kNAcc), (li / kNAcc) & 1);
    }
  } else if (warp >= kEpiWarps) {
    // ---------------------------------------------------------------- dequantisers
    const int q = warp % 4;                    // lane quarter: tile columns 32q .. 32q + 31
    const int team = (warp - kEpiWarps) / 4;   // units team, team + 2, ...: two units in flight
    const int r = lane / 4, l = lane % 4;
    const uint32_t tlane = (uint32_t)(q * 32) << 16;
    const half2 sixteenth = __float2half2_rn(0.0625f);
    for (int li = team; li < nunits; li += 2) {
      const int s = li % C::kSR, a = li % kSA;
      bool ok = mbar_wait(full_r(s), (li / C::kSR) & 1, s_abort);
      ok = ok && mbar_wait(empty_a(a), ((li / kSA) & 1) ^ 1, s_abort);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) fail();
        break;
      }
      tc_fence_after();
      // zero point of this lane's column: after the transpose nibble position r
      // of a word is AWQ lane awq_lane(r), the same nibble as in the zero word.
      // Columns past N read stale zero points; their qweight words are
      // zero-filled and their results are never stored.
      uint32_t zw;
      asm volatile("ld.shared.u32 %0, [%1];" : "=r"(zw) : "r"(meta0 + s * kMetaBytes + (4 * q + l) * 4));
      const uint32_t z = (zw >> (4 * r)) & 0xFu;
      const half2 zz = u32_as_half2((z | (z << 16)) | kMagic1024);   // (1024 + z) in both halves
      // (1024 + 16 z) / 16 = 64 + z, exact
      const half2 nzz16 = __hneg2(__hmul2(u32_as_half2(((z << 4) | (z << 20)) | kMagic1024), sixteenth));
#pragma unroll
      for (int h = 0; h < 2; ++h) {   // rows 64h .. 64h + 63 of the unit
      uint32_t w[8];
      if (PACKED) {
        // [h][q][blk / 4][lane][blk % 4]: two conflict-free 16-byte loads per lane
        const uint32_t pk = base + s * C::kStageR + C::kXBytes + ((h * 4 + q) * 2 * 32 + lane) * 16;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                     : "r"(pk));
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
                     : "r"(pk + 512));
      } else {
        // lane 4r + l reads word l of quarter q in row k = 64h + 8 blk + awq_lane(r);
        // (k >> 1) & 3 depends only on awq_lane(r), the same for every block
        const int kr = awq_lane(r);
        const uint32_t qt = base + s * C::kStageR + C::kXBytes + (64 * h + kr) * 64 +
                            ((q ^ ((kr >> 1) & 3)) << 4) + l * 4;
#pragma unroll
        for (int blk = 0; blk < 8; ++blk)
          asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w[blk]) : "r"(qt + blk * 512));
        // the three transpose steps, each over all 8 blocks so their shuffles overlap
#pragma unroll
        for (int blk = 0; blk < 8; ++blk) w[blk] = transpose_step<4>(w[blk], r);
#pragma unroll
        for (int blk = 0; blk < 8; ++blk) w[blk] = transpose_step<2>(w[blk], r);
#pragma unroll
        for (int blk = 0; blk < 8; ++blk) w[blk] = transpose_step<1>(w[blk], r);
      }
      uint32_t cells[32];
#pragma unroll
      for (int blk = 0; blk < 8; ++blk) {
        // rows (2i, 2i+1) of the block sit at nibble positions (i, i + 4)
        const uint32_t v = w[blk];
        const uint32_t v8 = v >> 8;
        cells[4 * blk + 0] = half2_as_u32(__hsub2(u32_as_half2((v & kLoPairMask) | kMagic1024), zz));
        // (1024 + 16 q) / 16 - (64 + z) = q - z, exact
        cells[4 * blk + 1] = half2_as_u32(__hfma2(u32_as_half2((v & kHiPairMask) | kMagic1024), sixteenth, nzz16));
        cells[4 * blk + 2] = half2_as_u32(__hsub2(u32_as_half2((v8 & kLoPairMask) | kMagic1024), zz));
        cells[4 * blk + 3] = half2_as_u32(__hfma2(u32_as_half2((v8 & kHiPairMask) | kMagic1024), sixteenth, nzz16));
      }
      tmem_st32_nowait(tmem + kTmemA + a * kACols + tlane + 32 * h, cells);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(full_a(a));
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp;                      // TMEM lanes 32q .. 32q + 31
    const int ct = q * 32 + 8 * (lane % 4) + awq_lane(lane / 4);   // column within the tile
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    asm volatile("griddepcontrol.wait;" ::: "memory");   // y and the workspace are shared with the predecessor
    float acc[MPAD];
#pragma unroll
    for (int m = 0; m < MPAD; ++m) acc[m] = 0.0f;
    uint32_t bad = 0;
    long long seg_u0 = u0;
    int t = first_t, g = first_g;
    for (int li = 0; li < nunits; ++li, next_unit(t, g)) {
      const long long u = u0 + li;
      const int col = t * kTileCols + ct;
      if (g == 0) seg_u0 = u;
      const int b = li % kNAcc, s = li % C::kSR;
      // acc_full implies full_r (through the MMA's full_a): the scales have landed
      const bool ok = mbar_wait(acc_full(b), (li / kNAcc) & 1, s_abort);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) fail();
        break;
      }
      float sc = 0.0f;
      if (col < p.N) {
        unsigned short sb;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(sb) : "r"(meta0 + s * kMetaBytes + kZBytes + ct * 2));
        bad |= invalid_scale_pair(sb);
        sc = __half2float(__ushort_as_half(sb));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_m(s));
      tc_fence_after();
      // two 16-column loads in flight per wait
#pragma unroll
      for (int c = 0; c < MPAD / 16; c += 2) {
        uint32_t v0[16], v1[16];
        tmem_ld16_nowait(lane_addr + b * MPAD + c * 16, v0);
        if (c + 1 < MPAD / 16) tmem_ld16_nowait(lane_addr + b * MPAD + (c + 1) * 16, v1);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[c * 16 + i] = fmaf(sc, __uint_as_float(v0[i]), acc[c * 16 + i]);
        if (c + 1 < MPAD / 16) {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            acc[(c + 1) * 16 + i] = fmaf(sc, __uint_as_float(v1[i]), acc[(c + 1) * 16 + i]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty(b));

      if (g != p.groups - 1 && li != nunits - 1) continue;
      // ---- end of a segment of tile t: [seg_u0, u] ----
      const long long tile_u0 = (long long)t * p.groups;
      const bool whole = seg_u0 == tile_u0 && g == p.groups - 1;
      const float bv = (p.bias && col < p.N) ? __half2float(p.bias[col]) : 0.0f;
      if (whole) {
        if (col < p.N) {
#pragma unroll
          for (int m = 0; m < MPAD; ++m)
            if (m < p.M) p.y[(size_t)m * p.N + col] = __float2half_rn(acc[m] + bv);
        }
      } else {
        // Each epilogue warp owns 32 columns of the tile and settles them on its
        // own ticket (tile, warp): no barrier between the epilogue warps.
        const int slot_j = seg_u0 == u0 ? 0 : 1;
        // partials [cta][slot][column][MPAD]: a column's rows are contiguous, so
        // both sides move them as 16-byte vectors (rows past M hold zeros)
        float* mine = p.partials + ((size_t)blockIdx.x * 2 + slot_j) * (MPAD * kTileCols) + (size_t)ct * MPAD;
#pragma unroll
        for (int m = 0; m < MPAD; m += 4)
          __stcg(reinterpret_cast<float4*>(mine + m), make_float4(acc[m], acc[m + 1], acc[m + 2], acc[m + 3]));
        __threadfence();
        __syncwarp();
        const int c_lo = owner_of(tile_u0, p.units, P);
        const int c_hi = owner_of(tile_u0 + p.groups - 1, p.units, P);
        int last = 0;
        if (lane == 0) {
          int* ticket = p.tickets + (size_t)t * kEpiWarps + q;
          last = atomicAdd(ticket, 1) == c_hi - c_lo;
          if (last) *ticket = 0;   // re-arm for the next launch
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          // contributor c_lo stored this tile as its last segment (slot 1) unless
          // its range starts at the tile start; every later contributor starts
          // inside the tile (slot 0)
          const int j_lo = range_begin(c_lo, p.units, P) < tile_u0 ? 1 : 0;
          const float* first = p.partials + ((size_t)c_lo * 2 + j_lo) * (MPAD * kTileCols) + (size_t)ct * MPAD;
          const float* rest = p.partials + ((size_t)(c_lo + 1) * 2) * (MPAD * kTileCols) + (size_t)ct * MPAD;
          const size_t stride = (size_t)2 * MPAD * kTileCols;
          const int n_rest = c_hi - c_lo;
          if (col < p.N) {
            // up to 32 rows at a time; the loads of two contributors are in
            // flight together, and the sum still runs in CTA order
            constexpr int kCh = MPAD < 32 ? MPAD : 32;
#pragma unroll
            for (int m0 = 0; m0 < MPAD; m0 += kCh) {
              if (m0 >= p.M) break;
              float4 v[kCh / 4];
#pragma unroll
              for (int i = 0; i < kCh / 4; ++i) v[i] = __ldcg(reinterpret_cast<const float4*>(first + m0) + i);
              for (int rr = 0; rr < n_rest; rr += 2) {
                const bool two = rr + 1 < n_rest;
                float4 w0[kCh / 4], w1[kCh / 4];
#pragma unroll
                for (int i = 0; i < kCh / 4; ++i) {
                  w0[i] = __ldcg(reinterpret_cast<const float4*>(rest + rr * stride + m0) + i);
                  w1[i] = two ? __ldcg(reinterpret_cast<const float4*>(rest + (rr + 1) * stride + m0) + i)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int i = 0; i < kCh / 4; ++i) {
                  v[i].x += w0[i].x; v[i].y += w0[i].y; v[i].z += w0[i].z; v[i].w += w0[i].w;
                  if (two) { v[i].x += w1[i].x; v[i].y += w1[i].y; v[i].z += w1[i].z; v[i].w += w1[i].w; }
                }
              }
#pragma unroll
              for (int i = 0; i < kCh / 4; ++i) {
                const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  if (m0 + 4 * i + k < p.M) p.y[(size_t)(m0 + 4 * i + k) * p.N + col] = __float2half_rn(e[k] + bv);
              }
            }
          }
        }
      }
#pragma unroll
      for (int m = 0; m < MPAD; ++m) acc[m] = 0.0f;
    }
    if (bad && p.dev_err) atomicOr(p.dev_err, ANVILQ_DEV_ERR_SCALE);
    tc_fence_before();
  }

  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
  }
}

// ---- host side ----------------------------------------------------------------
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

constexpr int kMaxDevices = 64;
static int g_sms[kMaxDevices];
static std::once_flag g_dev_once[kMaxDevices];

template <int MPAD>
static void set_smem_attr() {
  cudaFuncSetAttribute(verify_tc_kernel<MPAD, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<MPAD>::kSmem);
  cudaFuncSetAttribute(verify_tc_kernel<MPAD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<MPAD>::kSmem);
}

// One thread per word of the packed layout: unit (t, g) is 2048 words in the
// order [h][q][blk / 4][lane][blk % 4] (see the dequantisers), lane 4r + l of
// block blk holding nibble r of the words l of quarter q in the block's rows
// 64h + 8blk + awq_lane(j) at nibble positions j -- the transpose's result.
__global__ void tc_pack_kernel(const int32_t* __restrict__ qweight, uint32_t* __restrict__ packed, int W8,
                               int groups, long long words) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= words) return;
  const long long unit = i >> 11;
  const int e = (int)(i & 2047);
  const int j = e & 3, lane = (e >> 2) & 31, half = (e >> 7) & 1, q = (e >> 8) & 3, h = (e >> 10) & 1;
  const int t = (int)(unit / groups), g = (int)(unit % groups);
  const int blk = half * 4 + j, r = lane >> 2, l = lane & 3;
  const int k0 = g * kGroupRows + 64 * h + 8 * blk;
  const int w = t * kTileWords + 4 * q + l;
  uint32_t out = 0;
  if (w < W8) {
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const uint32_t word = (uint32_t)__ldg(qweight + (size_t)(k0 + awq_lane(jj)) * W8 + w);
      out |= ((word >> (4 * r)) & 0xFu) << (4 * jj);
    }
  }
  packed[i] = out;
}

static int device_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  std::call_once(g_dev_once[dev], [dev] {
    cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    set_smem_attr<16>();
    set_smem_attr<32>();
    set_smem_attr<48>();
    set_smem_attr<64>();
    cudaGetLastError();
  });
  return g_sms[dev];
}

constexpr int kMaxChunk = 64;

static int mpad_for(int m) { return (m + 15) / 16 * 16; }

struct Plan {
  int tiles, groups, grid;
  long long units;
};
static Plan make_plan(int sms, int K, int N) {
  Plan pl;
  pl.tiles = (N + kTileCols - 1) / kTileCols;
  pl.groups = K / kGroupRows;
  pl.units = (long long)pl.tiles * pl.groups;
  pl.grid = (int)std::min<long long>(sms, pl.units);
  return pl;
}

}  // namespace tc_verify

bool verify_tc_supported(const void* x, const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                         int M, int K, int N, int G) {
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  return M >= 1 && G == tc_verify::kGroupRows && K % tc_verify::kGroupRows == 0 && N % 32 == 0 && a16(x) &&
         a16(qweight) && a16(qzeros) && a16(scales) && tc_verify::encode_fn() != nullptr &&
         tc_verify::device_sms() > 0;
}

size_t verify_tc_workspace_bytes(int M, int K, int N) {
  using namespace tc_verify;
  const int sms = device_sms();
  if (sms <= 0 || K < kGroupRows) return 0;
  const Plan pl = make_plan(sms, K, N);
  const int mpad = mpad_for(std::min(M, kMaxChunk));
  return ANVILQ_WORKSPACE_COUNTER_BYTES + (size_t)pl.grid * 2 * mpad * kTileCols * sizeof(float);
}

size_t tc_pack_bytes(int K, int N) {
  using namespace tc_verify;
  if (K < kGroupRows || K % kGroupRows || N < 32 || N % 32) return 0;
  return (size_t)((N + kTileCols - 1) / kTileCols) * (K / kGroupRows) * kQBytes;
}

int launch_tc_pack(const int32_t* qweight, int32_t* packed, int K, int N, cudaStream_t stream) {
  using namespace tc_verify;
  const size_t bytes = tc_pack_bytes(K, N);
  if (!bytes) return ANVILQ_ESHAPE;
  const long long words = (long long)(bytes / 4);
  tc_pack_kernel<<<(unsigned)((words + 255) / 256), 256, 0, stream>>>(qweight, reinterpret_cast<uint32_t*>(packed),
                                                                    N / 8, K / kGroupRows, words);
  return cudaGetLastError() == cudaSuccess ? ANVILQ_OK : ANVILQ_ECUDA;
}

int launch_verify_tc(const uint16_t* x, const int32_t* qweight, const int32_t* packed, const int32_t* qzeros,
                     const uint16_t* scales, const uint16_t* bias, uint16_t* y, int M, int K, int N,
                     void* workspace, size_t workspace_bytes, int* dev_err, cudaStream_t stream,
                     bool overlap_prior) {
  using namespace tc_verify;
  const int sms = device_sms();
  auto encode = encode_fn();
  if (sms <= 0 || !encode) return ANVILQ_ECUDA;
  const Plan pl = make_plan(sms, K, N);
  if (pl.units < 1) return ANVILQ_ESHAPE;
  if ((size_t)pl.tiles * kEpiWarps * sizeof(int) > ANVILQ_WORKSPACE_COUNTER_BYTES) return ANVILQ_ESHAPE;
  if (!workspace || workspace_bytes < verify_tc_workspace_bytes(M, K, N)) return ANVILQ_EWORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) return ANVILQ_EALIGN;
  const int W8 = N / 8;

  // qweight [K][W8] int32; one box = 128 rows x 16 words (64 B) of a 128-column
  // tile, 64-byte swizzled (unused with packed weights)
  CUtensorMap mq;
  if (!packed) {
    const cuuint64_t dims[2] = {(cuuint64_t)W8, (cuuint64_t)K};
    const cuuint64_t strides[1] = {(cuuint64_t)W8 * 4};
    const cuuint32_t box[2] = {(cuuint32_t)kTileWords, (cuuint32_t)kGroupRows};
    const cuuint32_t estr[2] = {1, 1};
    if (encode(&mq, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(qweight), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return ANVILQ_EALIGN;
  }
  Params p;
  p.packed = packed;
  p.qzeros = qzeros;
  p.scales = reinterpret_cast<const __half*>(scales);
  p.bias = reinterpret_cast<const __half*>(bias);
  p.tickets = reinterpret_cast<int*>(workspace);
  p.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + ANVILQ_WORKSPACE_COUNTER_BYTES);
  p.dev_err = dev_err;
  p.K = K;
  p.N = N;
  p.W8 = W8;
  p.tiles = pl.tiles;
  p.groups = pl.groups;
  p.units = pl.units;

  for (int m0 = 0; m0 < M; m0 += kMaxChunk) {
    const int mc = std::min(kMaxChunk, M - m0);
    const int mpad = mpad_for(mc);
    CUtensorMap mx;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)mc};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)mpad};
    const cuuint32_t estr[2] = {1, 1};
    if (encode(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(x + (size_t)m0 * K), dims, strides,
               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return ANVILQ_EALIGN;
    p.M = mc;
    p.y = reinterpret_cast<__half*>(y) + (size_t)m0 * N;
    if (packed) mq = mx;   // not read by the packed kernel
    auto launch = [&](auto kernel, int smem) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(pl.grid, 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = overlap_prior ? 1 : 0;
      cudaLaunchKernelEx(&cfg, kernel, mq, mx, p);
    };
    switch (mpad) {
      case 16:
        packed ? launch(verify_tc_kernel<16, true>, Cfg<16>::kSmem) : launch(verify_tc_kernel<16, false>, Cfg<16>::kSmem);
        break;
      case 32:
        packed ? launch(verify_tc_kernel<32, true>, Cfg<32>::kSmem) : launch(verify_tc_kernel<32, false>, Cfg<32>::kSmem);
        break;
      case 48:
        packed ? launch(verify_tc_kernel<48, true>, Cfg<48>::kSmem) : launch(verify_tc_kernel<48, false>, Cfg<48>::kSmem);
        break;
      default:
        packed ? launch(verify_tc_kernel<64, true>, Cfg<64>::kSmem) : launch(verify_tc_kernel<64, false>, Cfg<64>::kSmem);
        break;
    }
    if (cudaGetLastError() != cudaSuccess) return ANVILQ_ECUDA;
  }
  return ANVILQ_OK;
}

}  // namespace anvilq
