/*
 * awq_oracle.c -- CPU restatement of the reference's golden models for the
 * W4A16 AWQ decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: the parity tests,
 * the smoke check and the CPU-baseline / reference arm of the benchmark call
 * it.  The product path (the CUDA kernels behind include/anvilq.h) never
 * links, loads or calls anything here.
 *
 * Every function follows a reference function line by line in meaning
 * (not in code); the citation is given above each one.  Paths are relative
 * to the reference project root (aHappend/anvil-q).
 *
 * Build: see oracle/Makefile.  It must be compiled WITHOUT floating-point
 * contraction (-ffp-contract=off) and without -ffast-math: the reference
 * rounds every multiply and every add separately to IEEE binary32, and the
 * restatement is only bit-exact when the compiler does the same.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <pthread.h>
#include <stdlib.h>
#include <unistd.h>

/* anvil-q1/tests/verify.py:38 and anvil-q1/tests/official_weights.py:20:
 * logical output lane i of a packed int32 sits at bit shift SHIFTS[i]. */
static const int kShift[8] = {0, 16, 4, 20, 8, 24, 12, 28};

#define ORACLE_OK 0
#define ORACLE_EINVAL (-1)
#define ORACLE_ESCALE (-2)    /* negative-nonzero or nonfinite AWQ scale */
#define ORACLE_ENONFINITE (-3) /* FP32 overflow / nonfinite result */

/* Exact binary16 -> binary32 decode.  Every binary16 value is exactly
 * representable in binary32, so this is the value struct.unpack("<e") gives
 * (official_weights.py:327) widened by f32() (official_weights.py:383-390). */
static float half_bits_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) & 1u;
    uint32_t exponent = (uint32_t)(h >> 10) & 31u;
    uint32_t mantissa = (uint32_t)h & 1023u;
    float magnitude;
    if (exponent == 0) {
        magnitude = ldexpf((float)mantissa, -24);
    } else if (exponent == 31) {
        magnitude = mantissa ? NAN : INFINITY;
    } else {
        magnitude = ldexpf((float)(mantissa + 1024u), (int)exponent - 25);
    }
    return sign ? -magnitude : magnitude;
}

/* anvil-q1/design/SPEC.md:175-177 and verify.py:241-248: a scale is invalid
 * when it is nonfinite (exponent 31) or negative and nonzero.  Negative zero
 * is zero and valid. */
static int scale_invalid(uint16_t h) {
    if (((h >> 10) & 31u) == 31u) return 1;
    if ((h & 0x8000u) && (h & 0x7fffu)) return 1;
    return 0;
}

static inline int nibble(uint32_t word, int lane) {
    return (int)((word >> kShift[lane]) & 15u);
}

/* verify.py:252-253 pack(values) -> int: value i goes to shift SHIFTS[i]. */
uint32_t anvilq_oracle_pack8(const uint8_t values[8]) {
    uint32_t word = 0;
    for (int i = 0; i < 8; ++i) word |= (uint32_t)(values[i] & 15u) << kShift[i];
    return word;
}

/* anvil-q1-fp/tests/awq_prepare.py:84-99 restated on a row-major code matrix:
 * codes[K][N] (uint8, 0..15) <-> packed[K][N/8] (uint32). */
int anvilq_oracle_pack(const uint8_t* codes, uint32_t* packed, int rows, int n) {
    if (!codes || !packed || rows < 0 || n < 0 || n % 8) return ORACLE_EINVAL;
    const int words = n / 8;
    for (int r = 0; r < rows; ++r)
        for (int w = 0; w < words; ++w)
            packed[(size_t)r * words + w] = anvilq_oracle_pack8(codes + (size_t)r * n + 8 * w);
    return ORACLE_OK;
}

int anvilq_oracle_unpack(const uint32_t* packed, uint8_t* codes, int rows, int n) {
    if (!codes || !packed || rows < 0 || n < 0 || n % 8) return ORACLE_EINVAL;
    const int words = n / 8;
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < n; ++c)
            codes[(size_t)r * n + c] = (uint8_t)nibble(packed[(size_t)r * words + c / 8], c % 8);
    return ORACLE_OK;
}

/* Exact rational decode of binary16 used by the integer golden:
 * verify.py:216-224 half_fraction -> numerator / 2^den_log2. */
static int half_fraction(uint16_t raw, int64_t* num, int* den_log2) {
    int sign = (raw & 0x8000u) ? -1 : 1;
    int exponent = (raw >> 10) & 31, mantissa = raw & 1023;
    if (exponent == 31) return -1;
    int64_t significand = exponent == 0 ? mantissa : mantissa + 1024;
    int power = exponent == 0 ? -24 : exponent - 25;
    if (power >= 0) {
        *num = sign * (significand << power);
        *den_log2 = 0;
    } else {
        *num = sign * significand;
        *den_log2 = -power;
    }
    return 0;
}

/* verify.py:227-229 rounded(n, d): round half away from zero, d = 2^dl. */
static __int128 round_away_pow2(__int128 n, int dl) {
    if (dl == 0) return n;
    __int128 d = (__int128)1 << dl;
    __int128 mag = n < 0 ? -n : n;
    __int128 r = (2 * mag + d) / (2 * d);
    return n < 0 ? -r : r;
}

/* verify.py:236-238 half_fixed(raw, 16): round_away(value * 2^16). */
static int half_fixed16(uint16_t raw, int64_t* out) {
    int64_t num;
    int dl;
    if (half_fraction(raw, &num, &dl)) return -1;
    *out = (int64_t)round_away_pow2((__int128)num << 16, dl);
    return 0;
}

static int64_t sat32(__int128 v) {
    if (v > 2147483647) return 2147483647;
    if (v < -2147483648LL) return -2147483648LL;
    return (int64_t)v;
}

/* Dequantise a [K, N] AWQ matrix element by element.
 *   delta  = u4 q - u4 z                 (verify.py:248, official_weights.py:428)
 *   w_f32  = f32(delta * scale)          (official_weights.py:429-431)
 *   w_q16  = delta * round_away(scale * 2^16)  (verify.py:241-250)
 *   invalid: verify.py:242-247 (0 on success; the element's outputs are 0).
 * Any output pointer may be NULL.  Returns the number of invalid elements. */
int64_t anvilq_oracle_dequant(const uint32_t* qweight, const uint32_t* qzeros,
                              const uint16_t* scales, int K, int N, int G,
                              int8_t* delta_out, float* w_out, int64_t* q16_out,
                              uint8_t* invalid_out) {
    if (!qweight || !qzeros || !scales || K < 0 || N < 0 || N % 8 || G <= 0) return ORACLE_EINVAL;
    const int words = N / 8;
    int64_t bad = 0;
    for (int k = 0; k < K; ++k) {
        const int g = k / G;
        for (int c = 0; c < N; ++c) {
            const size_t at = (size_t)k * N + c;
            const uint32_t qw = qweight[(size_t)k * words + c / 8];
            const uint32_t qz = qzeros[(size_t)g * words + c / 8];
            const uint16_t h = scales[(size_t)g * N + c];
            const int delta = nibble(qw, c % 8) - nibble(qz, c % 8);
            const int invalid = scale_invalid(h);
            bad += invalid;
            if (delta_out) delta_out[at] = (int8_t)delta;
            if (invalid_out) invalid_out[at] = (uint8_t)invalid;
            if (w_out) w_out[at] = invalid ? 0.0f : (float)delta * half_bits_to_float(h);
            if (q16_out) {
                int64_t s16 = 0;
                if (!invalid) half_fixed16(h, &s16);
                q16_out[at] = invalid ? 0 : (int64_t)delta * s16;
            }
        }
    }
    return bad;
}

/* FP32 golden GEMV / small-M GEMM, restating FP32Model.linear
 * (anvil-q1/tests/official_weights.py:418-437) for M independent rows:
 *   for each output column c:
 *     total = +0.0f
 *     for k in increasing order:
 *        weight = f32(delta * scale);  product = f32(x[k] * weight)
 *        total  = f32(total + product)          (fp_sum, :393-397)
 *     if bias: total = f32(total + bias[c])     (:434-435, Q/K/V only)
 * x is binary32 [M][K]; scales/bias are binary16 bit patterns; y is [M][N].
 * Columns [n_begin, n_end) only (pass 0, N for all).  `threads` > 1 splits
 * columns across POSIX threads; each column is still summed in the
 * reference order, so the result does not depend on the thread count. */
typedef struct {
    const float* x; const uint32_t* qweight; const uint32_t* qzeros;
    const uint16_t* scales; const uint16_t* bias; float* y;
    int M, K, N, G, c0, c1, status;
} Fp32Job;

static void* gemv_fp32_columns(void* arg) {
    Fp32Job* j = (Fp32Job*)arg;
    const int words = j->N / 8;
    for (int c = j->c0; c < j->c1; ++c) {
        const int lane = c % 8, word = c / 8;
        for (int m = 0; m < j->M; ++m) {
            const float* xm = j->x + (size_t)m * j->K;
            int local = ORACLE_OK;
            float total = 0.0f;
            for (int k = 0; k < j->K; ++k) {
                const int g = k / j->G;
                const uint16_t h = j->scales[(size_t)g * j->N + c];
                if (scale_invalid(h)) { local = ORACLE_ESCALE; break; }
                const int delta = nibble(j->qweight[(size_t)k * words + word], lane) -
                                  nibble(j->qzeros[(size_t)g * words + word], lane);
                const float weight = (float)delta * half_bits_to_float(h);
                const float product = xm[k] * weight;
                total = total + product;
            }
            if (local == ORACLE_OK && j->bias) {
                const uint16_t hb = j->bias[c];
                if (((hb >> 10) & 31u) == 31u) local = ORACLE_ENONFINITE;
                else total = total + half_bits_to_float(hb);
            }
            if (local == ORACLE_OK && !isfinite(total)) local = ORACLE_ENONFINITE;
            j->y[(size_t)m * j->N + c] = local == ORACLE_OK ? total : 0.0f;
            if (local != ORACLE_OK) j->status = local;
        }
    }
    return NULL;
}

/* Runs fn over `threads` contiguous column slices of [c0, c1); returns the
 * first nonzero slice status.  Each column is computed by exactly one
 * thread in the reference order, so results do not depend on `threads`. */
#define MAX_THREADS 256
static int split_columns(void* (*fn)(void*), void* jobs, size_t job_size,
                         int* (*status_of)(void*), void (*set_range)(void*, int, int),
                         int c0, int c1, int threads) {
    if (threads < 1) threads = 1;
    if (threads > MAX_THREADS) threads = MAX_THREADS;
    if (threads > c1 - c0) threads = c1 - c0 > 0 ? c1 - c0 : 1;
    pthread_t tids[MAX_THREADS];
    int started[MAX_THREADS];
    for (int t = 0; t < threads; ++t) {
        void* job = (char*)jobs + (size_t)t * job_size;
        const long span = (long)(c1 - c0);
        set_range(job, c0 + (int)(span * t / threads), c0 + (int)(span * (t + 1) / threads));
        started[t] = threads > 1 && pthread_create(&tids[t], NULL, fn, job) == 0;
        if (!started[t]) fn(job);
    }
    int status = ORACLE_OK;
    for (int t = 0; t < threads; ++t) {
        void* job = (char*)jobs + (size_t)t * job_size;
        if (started[t]) pthread_join(tids[t], NULL);
        if (*status_of(job) != ORACLE_OK && status == ORACLE_OK) status = *status_of(job);
    }
    return status;
}

static int* fp32_status(void* j) { return &((Fp32Job*)j)->status; }
static void fp32_range(void* j, int a, int b) { ((Fp32Job*)j)->c0 = a; ((Fp32Job*)j)->c1 = b; }

int anvilq_oracle_gemv_fp32(const float* x, const uint32_t* qweight, const uint32_t* qzeros,
                            const uint16_t* scales, const uint16_t* bias, float* y,
                            int M, int K, int N, int G, int n_begin, int n_end, int threads) {
    if (!x || !qweight || !qzeros || !scales || !y) return ORACLE_EINVAL;
    if (M < 0 || K < 0 || N < 0 || N % 8 || G <= 0) return ORACLE_EINVAL;
    if (n_begin < 0 || n_end > N || n_begin > n_end) return ORACLE_EINVAL;
    Fp32Job jobs[MAX_THREADS];
    for (int t = 0; t < MAX_THREADS; ++t) {
        Fp32Job j = {x, qweight, qzeros, scales, bias, y, M, K, N, G, 0, 0, ORACLE_OK};
        jobs[t] = j;
    }
    return split_columns(gemv_fp32_columns, jobs, sizeof(Fp32Job), fp32_status, fp32_range,
                         n_begin, n_end, threads);
}

/* Integer Q16.16 golden GEMV, restating FixedModel.linear
 * (anvil-q1/tests/official_weights.py:592-612) with the dequantiser of
 * verify.py:241-250 and the rounding of verify.py:227-233:
 *   total = sum_k x_q16[k] * delta * round_away(scale * 2^16)  (signed 128-bit)
 *   total += sat32(half_fixed(bias)) * 65536                    (Q/K/V only)
 *   y = sat32(round_away(total / 65536))
 * x_q16 is signed Q16.16 [M][K]; y is signed Q16.16 [M][N]. */
typedef struct {
    const int32_t* x; const uint32_t* qweight; const uint32_t* qzeros;
    const uint16_t* scales; const uint16_t* bias; int32_t* y;
    int M, K, N, G, c0, c1, status;
} Q16Job;

static void* gemv_q16_columns(void* arg) {
    Q16Job* j = (Q16Job*)arg;
    const int words = j->N / 8;
    for (int c = j->c0; c < j->c1; ++c) {
        const int lane = c % 8, word = c / 8;
        for (int m = 0; m < j->M; ++m) {
            int local = ORACLE_OK;
            __int128 total = 0;
            for (int k = 0; k < j->K; ++k) {
                const int g = k / j->G;
                const uint16_t h = j->scales[(size_t)g * j->N + c];
                int64_t s16;
                if (scale_invalid(h) || half_fixed16(h, &s16)) { local = ORACLE_ESCALE; break; }
                const int delta = nibble(j->qweight[(size_t)k * words + word], lane) -
                                  nibble(j->qzeros[(size_t)g * words + word], lane);
                total += (__int128)j->x[(size_t)m * j->K + k] * ((__int128)delta * s16);
            }
            if (local == ORACLE_OK && j->bias) {
                int64_t b16;
                if (half_fixed16(j->bias[c], &b16)) local = ORACLE_ENONFINITE;
                else total += (__int128)sat32(b16) * 65536;
            }
            j->y[(size_t)m * j->N + c] =
                local == ORACLE_OK ? (int32_t)sat32(round_away_pow2(total, 16)) : 0;
            if (local != ORACLE_OK) j->status = local;
        }
    }
    return NULL;
}

static int* q16_status(void* j) { return &((Q16Job*)j)->status; }
static void q16_range(void* j, int a, int b) { ((Q16Job*)j)->c0 = a; ((Q16Job*)j)->c1 = b; }

int anvilq_oracle_gemv_q16(const int32_t* x_q16, const uint32_t* qweight, const uint32_t* qzeros,
                           const uint16_t* scales, const uint16_t* bias, int32_t* y,
                           int M, int K, int N, int G, int threads) {
    if (!x_q16 || !qweight || !qzeros || !scales || !y) return ORACLE_EINVAL;
    if (M < 0 || K < 0 || N < 0 || N % 8 || G <= 0) return ORACLE_EINVAL;
    Q16Job jobs[MAX_THREADS];
    for (int t = 0; t < MAX_THREADS; ++t) {
        Q16Job j = {x_q16, qweight, qzeros, scales, bias, y, M, K, N, G, 0, 0, ORACLE_OK};
        jobs[t] = j;
    }
    return split_columns(gemv_q16_columns, jobs, sizeof(Q16Job), q16_status, q16_range,
                         0, N, threads);
}

/* FP32 sequential GQA decode attention, restating the inline attention of
 * FP32Model.token (anvil-q1/tests/official_weights.py:471-486) for one
 * sequence: causal over positions [0, T), kv head = head / (Hq / Hkv).
 *   score_t = f32(fp_sum_c f32(q*k) / f32(sqrt(D)))   (here: times `scale`
 *             when scale > 0 is given instead of the sqrt(D) divide)
 *   p_t = f32(exp(f32(s_t - max)) / sum)   out_c = fp_sum_t f32(p_t * v_tc)
 * q [Hq][D], k/v [T][Hkv][D] binary16 bit patterns, out [Hq][D] binary32.
 * scratch must hold T floats.  `threads` is accepted for interface symmetry
 * and ignored (one sequence is computed on the calling thread). */
int anvilq_oracle_attention_fp32(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                 float* out, int Hq, int Hkv, int D, int T,
                                 float* scratch, int threads) {
    if (!q || !k || !v || !out || !scratch) return ORACLE_EINVAL;
    if (Hq <= 0 || Hkv <= 0 || D <= 0 || T <= 0 || Hq % Hkv) return ORACLE_EINVAL;
    const float denominator = (float)sqrt((double)D);
    const int group = Hq / Hkv;
    (void)threads;
    for (int head = 0; head < Hq; ++head) {
        float* scores = scratch;
        const int kh = head / group;
        float maximum = -INFINITY;
        for (int t = 0; t < T; ++t) {
            float dot = 0.0f;
            for (int c = 0; c < D; ++c) {
                const float a = half_bits_to_float(q[(size_t)head * D + c]);
                const float b = half_bits_to_float(k[((size_t)t * Hkv + kh) * D + c]);
                dot = dot + a * b;
            }
            scores[t] = dot / denominator;
            if (scores[t] > maximum) maximum = scores[t];
        }
        float total = 0.0f;
        for (int t = 0; t < T; ++t) {
            scores[t] = (float)exp((double)(scores[t] - maximum));
            total = total + scores[t];
        }
        for (int t = 0; t < T; ++t) scores[t] = scores[t] / total;
        for (int c = 0; c < D; ++c) {
            float acc = 0.0f;
            for (int t = 0; t < T; ++t)
                acc = acc + scores[t] * half_bits_to_float(v[((size_t)t * Hkv + kh) * D + c]);
            out[(size_t)head * D + c] = acc;
        }
    }
    return ORACLE_OK;
}

int anvilq_oracle_max_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}
