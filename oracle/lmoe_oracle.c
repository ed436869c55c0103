/*
 * lmoe_oracle.c -- CPU oracle for the MoE-layer hot path (TEST INFRASTRUCTURE ONLY).
 *
 * This file is the checker, never the product: only the tests, the smoke check and the
 * CPU-baseline leg of bench.py load it.  The CUDA library must never call it.
 *
 * It restates, in plain C with explicitly rounded IEEE-754 operations, the integer and
 * floating-point steps whose results the CUDA kernels must reproduce bit for bit:
 *
 *   - routing from fp32 gate logits: softmax -> top-k (ties to the lower expert id) ->
 *     renormalisation.  Follows light-moe csrc/fused_moe_ops.cu:49-134 (max-reduce,
 *     exp, sum, reciprocal-multiply, insertion top-k with strict '>', renormalise by
 *     reciprocal-multiply) and python/light_moe/ops/moe_gate.py:39-77 (same semantics).
 *   - per-expert counts, exclusive offsets and a STABLE permutation of the flattened
 *     [T, k] assignment list.  Follows python/light_moe/ops/grouped_gemm.py:202-247 and
 *     csrc/fused_moe_ops.cu:214-225; the reference argsort is unstable, this restatement
 *     pins the order to (expert, token, slot).
 *   - symmetric per-group int4 weight quantisation along K with fp16 scales, and its
 *     dequantisation to bf16.  The reference has no int4 code (only the unused flag at
 *     python/light_moe/engine/executor.py:44-48); the format is defined here.
 *
 * Arithmetic rules (identical on the GPU side, which uses the __*_rn intrinsics):
 *   - every float operation is a single IEEE round-to-nearest-even operation; the file is
 *     compiled with -ffp-contract=off so the compiler fuses nothing on its own;
 *   - exp(x) for x <= 0 is lmoe_ref_expf below (Cody-Waite reduction + Taylor polynomial).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* ------------------------------------------------------------------------------------ */
/* bit-level conversions                                                                  */
/* ------------------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* fp32 -> bf16, round to nearest even (NaN kept quiet). */
uint16_t lmoe_ref_f32_to_bf16(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float lmoe_ref_bf16_to_f32(uint16_t h) { return u2f(((uint32_t)h) << 16); }

/* fp32 -> fp16, round to nearest even, with subnormals, overflow to inf, NaN kept. */
uint16_t lmoe_ref_f32_to_f16(float f) {
    uint32_t u = f2u(f);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);           /* NaN */
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);          /* >= 65520: inf */
    if (a < 0x38800000u) {                                            /* < 2^-14: subnormal */
        /* value = a_float; subnormal half unit = 2^-24.  Compute round(a / 2^-24). */
        if (a < 0x33000000u) return (uint16_t)sign;                   /* < 2^-25: rounds to 0 */
        uint32_t mant = (a & 0x7fffffu) | 0x800000u;
        int exp = (int)(a >> 23);                                     /* biased, 102..112 */
        int shift = 126 - exp;                                        /* 14..24 */
        uint32_t q = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q += 1u;
        return (uint16_t)(sign | q);
    }
    /* normal range: rebias exponent 127 -> 15 and round 23 -> 10 mantissa bits */
    uint32_t r = a - 0x38000000u;                                     /* exponent rebias */
    uint32_t q = r >> 13;
    uint32_t rem = r & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q += 1u;
    return (uint16_t)(sign | q);
}

float lmoe_ref_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    if (e == 0) {
        /* subnormal: m * 2^-24, exact in fp32 */
        float v = (float)m * u2f(0x33800000u);
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* ------------------------------------------------------------------------------------ */
/* exp for x <= 0                                                                         */
/* ------------------------------------------------------------------------------------ */
/*
 * Method (Cody & Waite, "Software Manual for the Elementary Functions", 1980): write
 * x = n*ln2 + r with n = rint(x*log2(e)) and |r| <= ln2/2, where ln2 = LN2_HI + LN2_LO and
 * LN2_HI has 12 trailing zero mantissa bits so n*LN2_HI is exact; then exp(x) = 2^n * P(r)
 * with P the degree-7 Taylor polynomial of exp (coefficients 1/j!, rounded to fp32),
 * evaluated by Horner's rule with fused multiply-adds.  Truncation error r^8/8! < 6e-9;
 * the result is within 2 ulp of exp(x) (checked against double-precision exp in tests).
 * Results below the fp32 subnormal range flush to +0.
 */
#define LMOE_LOG2E   0x3fb8aa3bu  /* fp32(1/ln 2)                     */
#define LMOE_LN2_HI  0x3f317000u  /* ln 2 with the low 12 bits cleared */
#define LMOE_LN2_LO  0x3805fdf4u  /* fp32(ln 2 - LN2_HI)               */
#define LMOE_C2      0x3f000000u  /* 1/2!  */
#define LMOE_C3      0x3e2aaaabu  /* 1/3!  */
#define LMOE_C4      0x3d2aaaabu  /* 1/4!  */
#define LMOE_C5      0x3c088889u  /* 1/5!  */
#define LMOE_C6      0x3ab60b61u  /* 1/6!  */
#define LMOE_C7      0x39500d01u  /* 1/7!  */

float lmoe_ref_expf(float x) {
    if (!(x > -104.0f)) return 0.0f;          /* also maps NaN to 0 */
    if (x > 0.0f) x = 0.0f;                   /* softmax arguments are <= 0 */
    float t = x * u2f(LMOE_LOG2E);
    float n = rintf(t);
    float r = fmaf(-n, u2f(LMOE_LN2_HI), x);
    r = fmaf(-n, u2f(LMOE_LN2_LO), r);
    float p = u2f(LMOE_C7);
    p = fmaf(p, r, u2f(LMOE_C6));
    p = fmaf(p, r, u2f(LMOE_C5));
    p = fmaf(p, r, u2f(LMOE_C4));
    p = fmaf(p, r, u2f(LMOE_C3));
    p = fmaf(p, r, u2f(LMOE_C2));
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;                          /* -151 .. 0 */
    if (ni >= -126) return p * u2f((uint32_t)(ni + 127) << 23);
    /* two-step scaling so the only rounding happens in the final (subnormal) product */
    float p2 = p * u2f((uint32_t)(ni + 64 + 127) << 23);
    return p2 * u2f((uint32_t)(127 - 64) << 23);
}

/* ------------------------------------------------------------------------------------ */
/* routing                                                                                */
/* ------------------------------------------------------------------------------------ */
/*
 * logits: [T, E] fp32 (gate bias already added).  Writes ids [T, k] int32 in descending
 * probability order (ties: lower expert id first) and weights [T, k] fp32.
 * Returns 0, or -1 on bad arguments (k > E, k > 64).
 */
int lmoe_ref_route(const float* logits, int T, int E, int k, int32_t* ids, float* weights) {
    if (T < 0 || E <= 0 || k <= 0 || k > E || k > 64 || E > 1024) return -1;
    float p[1024];
    for (int t = 0; t < T; ++t) {
        const float* l = logits + (size_t)t * E;
        float m = l[0];
        for (int e = 1; e < E; ++e) m = fmaxf(m, l[e]);
        float sum = 0.0f;
        for (int e = 0; e < E; ++e) {
            p[e] = lmoe_ref_expf(l[e] - m);
            sum = sum + p[e];
        }
        float inv = 1.0f / sum;
        for (int e = 0; e < E; ++e) p[e] = p[e] * inv;
        /* insertion top-k with strict '>' : an equal later expert never displaces an
           earlier (lower-id) one, as in csrc/fused_moe_ops.cu:106-118 */
        int32_t ti[64];
        float tv[64];
        for (int j = 0; j < k; ++j) { ti[j] = 0; tv[j] = -INFINITY; }
        for (int e = 0; e < E; ++e) {
            float v = p[e];
            if (v > tv[k - 1]) {
                int pos = k - 1;
                while (pos > 0 && v > tv[pos - 1]) {
                    tv[pos] = tv[pos - 1];
                    ti[pos] = ti[pos - 1];
                    --pos;
                }
                tv[pos] = v;
                ti[pos] = e;
            }
        }
        float s = 0.0f;
        for (int j = 0; j < k; ++j) s = s + tv[j];
        float invs = 1.0f / s;
        for (int j = 0; j < k; ++j) {
            ids[(size_t)t * k + j] = ti[j];
            weights[(size_t)t * k + j] = tv[j] * invs;
        }
    }
    return 0;
}

/*
 * The full softmax probabilities of the routing above (router_probs of
 * python/light_moe/ops/moe_gate.py:20-36, computed by top_k_routing at :66-67): the same
 * max, exponentials, sequential sum and reciprocal-multiply as lmoe_ref_route.
 */
int lmoe_ref_softmax(const float* logits, int T, int E, float* probs) {
    if (T < 0 || E <= 0) return -1;
    for (int t = 0; t < T; ++t) {
        const float* l = logits + (size_t)t * E;
        float* p = probs + (size_t)t * E;
        float m = l[0];
        for (int e = 1; e < E; ++e) m = fmaxf(m, l[e]);
        float sum = 0.0f;
        for (int e = 0; e < E; ++e) {
            p[e] = lmoe_ref_expf(l[e] - m);
            sum = sum + p[e];
        }
        float inv = 1.0f / sum;
        for (int e = 0; e < E; ++e) p[e] = p[e] * inv;
    }
    return 0;
}

/*
 * Histogram, exclusive scan and stable permutation of the flattened assignment list.
 * ids: [T, k].  counts: [E], offsets: [E+1], sorted_idx: [T*k] with
 * sorted_idx[offsets[e] + r] = the r-th flat index t*k+j (in increasing order) whose
 * expert is e.  Returns 0, or -1 if an id is out of range.
 */
int lmoe_ref_counts_offsets(const int32_t* ids, int T, int k, int E,
                            int32_t* counts, int32_t* offsets, int32_t* sorted_idx) {
    for (int e = 0; e < E; ++e) counts[e] = 0;
    size_t n = (size_t)T * k;
    for (size_t i = 0; i < n; ++i) {
        int32_t e = ids[i];
        if (e < 0 || e >= E) return -1;
        counts[e] += 1;
    }
    offsets[0] = 0;
    for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
    if (sorted_idx) {
        int32_t cursor[4096];
        if (E > 4096) return -1;
        for (int e = 0; e < E; ++e) cursor[e] = offsets[e];
        for (size_t i = 0; i < n; ++i) sorted_idx[cursor[ids[i]]++] = (int32_t)i;
    }
    return 0;
}

/* ------------------------------------------------------------------------------------ */
/* W4 quantisation (format defined by this project)                                       */
/* ------------------------------------------------------------------------------------ */
/*
 * w: [rows, K] fp32 (bf16 inputs are widened exactly before the call).  Group size g
 * divides K, K even.  For each (row, group):
 *     s  = fp16_rn( max|w| / 7 )             (fp32 division, then one fp16 rounding)
 *     q  = s == 0 ? 0 : clamp( rint( w / float(s) ), -8, 7 )
 * packed: [rows, K/2] uint8, byte b of a row holds k = 2b in the low nibble and
 * k = 2b+1 in the high nibble, each as q + 8.  scales: [rows, K/g] fp16 bits.
 */
int lmoe_ref_quantize_w4(const float* w, int64_t rows, int K, int g,
                         uint8_t* packed, uint16_t* scales) {
    if (rows < 0 || K <= 0 || g <= 0 || (K % g) != 0 || (K & 1) || (g & 1)) return -1;
    int G = K / g;
    for (int64_t r = 0; r < rows; ++r) {
        const float* wr = w + r * K;
        for (int gi = 0; gi < G; ++gi) {
            float m = 0.0f;
            for (int i = 0; i < g; ++i) m = fmaxf(m, fabsf(wr[gi * g + i]));
            uint16_t s16 = lmoe_ref_f32_to_f16(m / 7.0f);
            scales[r * G + gi] = s16;
            float sf = lmoe_ref_f16_to_f32(s16);
            for (int i = 0; i < g; i += 2) {
                int q[2];
                for (int h = 0; h < 2; ++h) {
                    float v = wr[gi * g + i + h];
                    int qq = 0;
                    if (sf != 0.0f && isfinite(sf)) {
                        float x = rintf(v / sf);
                        qq = x > 7.0f ? 7 : (x < -8.0f ? -8 : (int)x);
                    }
                    q[h] = qq;
                }
                packed[r * (K / 2) + (gi * g + i) / 2] =
                    (uint8_t)(((q[0] + 8) & 0xf) | (((q[1] + 8) & 0xf) << 4));
            }
        }
    }
    return 0;
}

/* out: [rows, K] bf16 bits, out = bf16_rn( float(q) * float(s) ). */
int lmoe_ref_dequantize_w4(const uint8_t* packed, const uint16_t* scales, int64_t rows, int K,
                           int g, uint16_t* out) {
    if (rows < 0 || K <= 0 || g <= 0 || (K % g) != 0 || (K & 1)) return -1;
    int G = K / g;
    for (int64_t r = 0; r < rows; ++r) {
        for (int kk = 0; kk < K; ++kk) {
            uint8_t b = packed[r * (K / 2) + kk / 2];
            int q = (int)((kk & 1) ? (b >> 4) : (b & 0xf)) - 8;
            float sf = lmoe_ref_f16_to_f32(scales[r * G + kk / g]);
            out[r * K + kk] = lmoe_ref_f32_to_bf16((float)q * sf);
        }
    }
    return 0;
}

/* Batch helpers used by the Python side to check conversions against numpy. */
void lmoe_ref_f32_to_f16_array(const float* x, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = lmoe_ref_f32_to_f16(x[i]);
}
void lmoe_ref_f32_to_bf16_array(const float* x, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = lmoe_ref_f32_to_bf16(x[i]);
}
void lmoe_ref_expf_array(const float* x, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = lmoe_ref_expf(x[i]);
}
