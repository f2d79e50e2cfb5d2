/*
 * bfp8_oracle.c -- CPU restatement of the reference decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA kernels
 * are compared against.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it; the product library never links
 * or calls it.
 *
 * What it restates (reference = ideal1128/qwen35-ax7020-edge-llm):
 *   - EXP_SCALE table           04-板载脚本与工具/qwen_kernels_opt.c:104,128-135
 *   - quant_x_blocks            04-板载脚本与工具/qwen_kernels_opt.c:182-205
 *   - bfp8_gemv, NEON int16 path (lane classes, non-fused per-block combine,
 *     final pairing, odd last row on scalar VFP)
 *                               04-板载脚本与工具/qwen_kernels_opt.c:213-308
 *   - bfp8_gemv scalar fallback 04-板载脚本与工具/qwen_kernels_opt.c:311-325
 *   - lm_head_argmax NEON order 04-板载脚本与工具/qwen_kernels_opt.c:401-488
 *     (and its scalar build     :489-505)
 *   - lm_head_topk selection    04-板载脚本与工具/qwen_sampling.c:110-155,160-353
 *   - gemv_core dequant mode    02-RTL与仿真/gemv_core.v:40-69,299-534
 *   - rmsnorm, NEON and scalar  04-板载脚本与工具/qwen_kernels_opt.c:140-172
 *   - add_residual              04-板载脚本与工具/qwen_kernels_opt.c:388-396
 *
 * Floating point model.  The reference board runs the vector parts on ARMv7
 * Advanced SIMD, which always flushes subnormal inputs and results to a zero
 * of the same sign and always rounds to nearest even; multiply-accumulate
 * (VMLA) is not fused.  The scalar parts run on VFP with IEEE subnormals.
 * Every vector-path operation below goes through neon_mul/neon_add, which
 * model that flush explicitly; scalar-path operations use plain C float
 * arithmetic.  Build with -ffp-contract=off so no multiply-add is fused.
 */
#include <math.h>
#include <float.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------- helpers */

static float ftz(float x) {
    return (fpclassify(x) == FP_SUBNORMAL) ? copysignf(0.0f, x) : x;
}
static float neon_mul(float a, float b) { return ftz(ftz(a) * ftz(b)); }
static float neon_add(float a, float b) { return ftz(ftz(a) + ftz(b)); }

static float bf16_bits_to_f32(uint16_t u) {
    uint32_t w = ((uint32_t)u) << 16;
    float f;
    memcpy(&f, &w, 4);
    return f;
}

/* ---------------------------------------------------------------- rmsnorm */
/* rmsnorm (qwen_kernels_opt.c:140-172), NEON build: four lane sums of x*x
 * over i = 4j + l (VMLA, not fused, flushed), combined as (s0 + s2) + (s1 + s3);
 * any n % 4 tail added on VFP; r = 1 / sqrtf(sum / n + eps) on VFP; then
 * y = x * (r * (1 + w)) on the vector unit (tail: (x * r) * (1 + w) on VFP). */
ORC_API void orc_rmsnorm_neon(float* y, const float* x, const float* w, int n, float eps) {
    float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int i = 0;
    for (; i + 4 <= n; i += 4)
        for (int l = 0; l < 4; l++) s4[l] = neon_add(s4[l], neon_mul(x[i + l], x[i + l]));
    float sum = neon_add(neon_add(s4[0], s4[2]), neon_add(s4[1], s4[3]));
    for (; i < n; i++) sum += x[i] * x[i];
    const float r = 1.0f / sqrtf((sum / (float)n) + eps);
    for (i = 0; i + 4 <= n; i += 4)
        for (int l = 0; l < 4; l++) y[i + l] = neon_mul(x[i + l], neon_mul(r, neon_add(1.0f, w[i + l])));
    for (; i < n; i++) y[i] = x[i] * r * (1.0f + w[i]);
}

/* add_residual (qwen_kernels_opt.c:388-396): x += res, four lanes at a time on
 * the vector unit (flushed), any n % 4 tail on VFP.  neon = 0: the portable
 * build (every element on VFP). */
ORC_API void orc_add_residual(float* x, const float* res, int n, int neon) {
    int i = 0;
    if (neon)
        for (; i + 4 <= n; i += 4)
            for (int l = 0; l < 4; l++) x[i + l] = neon_add(x[i + l], res[i + l]);
    for (; i < n; i++) x[i] += res[i];
}

/* ------------------------------------------------------------------ swiglu */
static float neon_sub(float a, float b) { return ftz(ftz(a) - ftz(b)); }

/* VMAX / VMIN against a constant (ARMv7 Advanced SIMD, flush-to-zero): a NaN
 * operand gives NaN, else the larger / smaller of the flushed operands. */
static float neon_max_c(float a, float c) { a = ftz(a); return (a != a) ? a : (a > c ? a : c); }
static float neon_min_c(float a, float c) { a = ftz(a); return (a != a) ? a : (a < c ? a : c); }

/* exp_neon (qwen_kernels_opt.c:332-351), one lane: x clamped to [-87, 88];
 * fx = x * RN(1/ln 2); n = fx rounded to an integer by adding and
 * subtracting 1.5 * 2^23; f = fx - n; p = the degree-6 Taylor polynomial of
 * 2^f, coefficients RN((ln 2)^k / k!), by Horner steps that round the product
 * before the add (VMLA); times 2^n built from exponent bits (VCVT rounds
 * toward zero, a NaN converts to 0).  Every step flushed like the vector
 * unit. */
static const float kLog2e = 0x1.715476p+0f;                  /* RN(1/ln 2) */
static const float kRoundMagic = 0x1.8p+23f;                 /* 1.5 * 2^23 */
static const float kExp2Taylor[7] = {                        /* RN((ln 2)^k / k!), k = 0..6 */
    0x1p+0f, 0x1.62e430p-1f, 0x1.ebfbe0p-3f, 0x1.c6b08ep-5f, 0x1.3b2ab6p-7f, 0x1.5d87fep-10f, 0x1.430912p-13f};

static float exp_neon_lane(float x) {
    x = neon_min_c(neon_max_c(x, -87.0f), 88.0f);
    const float fx = neon_mul(x, kLog2e);
    const float n = neon_sub(neon_add(fx, kRoundMagic), kRoundMagic);
    const float f = neon_sub(fx, n);
    float p = kExp2Taylor[6];
    for (int k = 5; k >= 0; k--) p = neon_add(kExp2Taylor[k], neon_mul(p, f));
    const int e = ((n != n) ? 0 : (int)n) + 127;
    const uint32_t bits = (uint32_t)e << 23;
    float sc;
    memcpy(&sc, &bits, 4);
    return neon_mul(p, sc);
}

/* swiglu (qwen_kernels_opt.c:365-386), NEON build: per lane
 * y = (g / (1 + exp_neon(-g))) * up, the add and the final product on the
 * vector unit (flushed), the division on VFP (IEEE, unflushed g); elements
 * past the last multiple of 4 on VFP with the C library's expf.  neon = 0:
 * the portable build, every element (g / (1 + expf(-g))) * up on VFP. */
ORC_API void orc_swiglu(float* y, const float* gate, const float* up, int n, int neon) {
    int i = 0;
    if (neon)
        for (; i < (n & ~3); i++) {
            const float g = gate[i];
            const float d = neon_add(1.0f, exp_neon_lane(-g));
            y[i] = neon_mul(g / d, up[i]);
        }
    for (; i < n; i++) {
        const float g = gate[i];
        y[i] = (g / (1.0f + expf(-g))) * up[i];
    }
}

/* The same routine's portable build: one running sum, y = (x * r) * (1 + w). */
ORC_API void orc_rmsnorm_scalar(float* y, const float* x, const float* w, int n, float eps) {
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum += x[i] * x[i];
    const float r = 1.0f / sqrtf((sum / (float)n) + eps);
    for (int i = 0; i < n; i++) y[i] = x[i] * r * (1.0f + w[i]);
}

/* EXP_SCALE[e] = 2^(e-134); subnormal for e < 8 (qwen_kernels_opt.c:131). */
ORC_API void orc_exp_scale(float* out256) {
    for (int e = 0; e < 256; e++) out256[e] = ldexpf(1.0f, e - 134);
}

/* ------------------------------------------------------------- quantizer */
/* Block-64 activation quantizer (qwen_kernels_opt.c:182-205):
 *   amax = max |x| over the block, NaN never wins the compare;
 *   amax > 1e-20: q = 16384/amax, xs = amax/16384, xq = lrintf(x*q)
 *   otherwise xs = 0 and xq = 0.
 * Runs on scalar VFP in the reference: IEEE division, round-half-even. */
ORC_API void orc_quant_x(const float* x, int K, int16_t* xq, float* xs) {
    int nb = K / 64;
    for (int b = 0; b < nb; b++) {
        const float* xb = x + 64 * b;
        float amax = 0.0f;
        for (int i = 0; i < 64; i++) {
            float v = fabsf(xb[i]);
            if (v > amax) amax = v;
        }
        if (amax > 1e-20f) {
            float q = 16384.0f / amax;
            xs[b] = amax / 16384.0f;
            for (int i = 0; i < 64; i++) {
                float p = xb[i] * q;
                long r = lrintf(p);
                xq[64 * b + i] = (int16_t)r;
            }
        } else {
            xs[b] = 0.0f;
            for (int i = 0; i < 64; i++) xq[64 * b + i] = 0;
        }
    }
}

/* ------------------------------------------------------------ block dots */
/* Per (row, block) lane-class sums L_j = sum_{i = j mod 4} m*xq, the int32
 * partials the NEON loop holds in a0+a1 (qwen_kernels_opt.c:231-257,265). */
ORC_API void orc_lane_dots(const int8_t* mant, const int16_t* xq, int M, int K,
                           int32_t* lanes /* [M][K/64][4] */) {
    int nb = K / 64;
    for (int m = 0; m < M; m++) {
        for (int b = 0; b < nb; b++) {
            int32_t L[4] = {0, 0, 0, 0};
            const int8_t* w = mant + (size_t)m * K + 64 * b;
            const int16_t* xv = xq + 64 * b;
            for (int i = 0; i < 64; i++) L[i & 3] += (int32_t)w[i] * (int32_t)xv[i];
            for (int j = 0; j < 4; j++) lanes[((size_t)m * nb + b) * 4 + j] = L[j];
        }
    }
}

/* Whole-block int32 dot products (the value gemv_core legacy mode emits,
 * 02-RTL与仿真/gemv_core.v:36-38,498). */
ORC_API void orc_block_dots(const int8_t* mant, const int16_t* xq, int M, int K,
                            int32_t* dots /* [M][K/64] */) {
    int nb = K / 64;
    for (int m = 0; m < M; m++)
        for (int b = 0; b < nb; b++) {
            int32_t s = 0;
            const int8_t* w = mant + (size_t)m * K + 64 * b;
            const int16_t* xv = xq + 64 * b;
            for (int i = 0; i < 64; i++) s += (int32_t)w[i] * (int32_t)xv[i];
            dots[(size_t)m * nb + b] = s;
        }
}

/* ------------------------------------------------ GEMV, NEON int16 path */
/* One row on the vector unit (qwen_kernels_opt.c:223-277):
 *   f_j = 0; for b: f_j = f_j + ((float(L_j) * S(e_b)) * xs_b)   [VMUL, VMLA]
 *   y = (f_0 + f_2) + (f_1 + f_3)                                [VADD, VPADD]  */
static float row_neon(const int8_t* w, const uint8_t* e, const int16_t* xq,
                      const float* xs, const float* S, int nb) {
    float f[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int b = 0; b < nb; b++) {
        int32_t L[4] = {0, 0, 0, 0};
        for (int i = 0; i < 64; i++)
            L[i & 3] += (int32_t)w[64 * b + i] * (int32_t)xq[64 * b + i];
        for (int j = 0; j < 4; j++) {
            float t = neon_mul(neon_mul((float)L[j], S[e[b]]), xs[b]);
            f[j] = neon_add(f[j], t);
        }
    }
    return neon_add(neon_add(f[0], f[2]), neon_add(f[1], f[3]));
}

/* Odd last row on scalar VFP (qwen_kernels_opt.c:279-305):
 *   sum = sum + (float)D * S(e_b) * xs_b, left to right, IEEE subnormals. */
static float row_scalar_q(const int8_t* w, const uint8_t* e, const int16_t* xq,
                          const float* xs, const float* S, int nb) {
    float sum = 0.0f;
    for (int b = 0; b < nb; b++) {
        int32_t s = 0;
        for (int i = 0; i < 64; i++) s += (int32_t)w[64 * b + i] * (int32_t)xq[64 * b + i];
        float t = (float)s * S[e[b]];
        t = t * xs[b];
        sum = sum + t;
    }
    return sum;
}

/* bfp8_gemv from an already quantized activation (xq, xs). */
ORC_API void orc_bfp8_gemv_q(float* y, const int16_t* xq, const float* xs,
                             const int8_t* mant, const uint8_t* exps, int M, int K) {
    float S[256];
    orc_exp_scale(S);
    int nb = K / 64;
    for (int m = 0; m < (M & ~1); m++)
        y[m] = row_neon(mant + (size_t)m * K, exps + (size_t)m * nb, xq, xs, S, nb);
    if (M & 1) {
        int m = M - 1;
        y[m] = row_scalar_q(mant + (size_t)m * K, exps + (size_t)m * nb, xq, xs, S, nb);
    }
}

/* bfp8_gemv, NEON int16 path generalised to any K multiple of 64. */
ORC_API void orc_bfp8_gemv_neon(float* y, const float* x, const int8_t* mant,
                                const uint8_t* exps, int M, int K) {
    int16_t* xq = (int16_t*)malloc(sizeof(int16_t) * (size_t)K);
    float* xs = (float*)malloc(sizeof(float) * (size_t)(K / 64 + 1));
    orc_quant_x(x, K, xq, xs);
    orc_bfp8_gemv_q(y, xq, xs, mant, exps, M, K);
    free(xq);
    free(xs);
}

/* Batched form: x [B][K] -> y [B][M], each row of x quantized on its own. */
ORC_API void orc_bfp8_gemv_neon_batch(float* y, const float* x, const int8_t* mant,
                                      const uint8_t* exps, int B, int M, int K) {
    for (int r = 0; r < B; r++)
        orc_bfp8_gemv_neon(y + (size_t)r * M, x + (size_t)r * K, mant, exps, M, K);
}

/* Scalar float fallback (qwen_kernels_opt.c:311-325): no activation quant,
 * sequential float block dot, sum += block_dot * S. */
ORC_API void orc_bfp8_gemv_scalar(float* y, const float* x, const int8_t* mant,
                                  const uint8_t* exps, int M, int K) {
    float S[256];
    orc_exp_scale(S);
    int nb = K / 64;
    for (int m = 0; m < M; m++) {
        const int8_t* w = mant + (size_t)m * K;
        const uint8_t* e = exps + (size_t)m * nb;
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            float d = 0.0f;
            for (int i = 0; i < 64; i++) d += (float)w[64 * b + i] * x[64 * b + i];
            sum += d * S[e[b]];
        }
        y[m] = sum;
    }
}

/* --------------------------------------------------- gemv_core dequant mode */
/* Row word of the RTL dequant datapath (02-RTL与仿真/gemv_core.v:299-534):
 *   xs float bits -> 17-bit mantissa 1.f[22:7] (truncated) and exponent Ex;
 *   zero/subnormal/inf/NaN xs -> mantissa 0;
 *   sh = Ex + e - 110 clamped to [-63, 63] (sh > 63 flags overflow);
 *   prod = D * mant; contrib = prod << sh or prod >>> -sh (arithmetic),
 *   shifted in two stages (:374-428): the low three bits of the amount come
 *   from the clamped shift, the high three from the unclamped one (sh_q2),
 *   so a shift below -63 moves right by 7 + 8*((-sh >> 3) & 7), not 63;
 *   left-shift overflow (|prod| >> (63-sh) != 0 for sh >= 16) or a clamped
 *   shift saturates the contribution to +-(2^63-1) by the sign of prod;
 *   64-bit saturating row sum; output clamp(acc, -(2^31)<<20, (2^31-1)<<20)
 *   bits [51:20] = floor(y * 2^20).  Returns the sticky flags in *flags:
 *   bit0 = arithmetic saturation, bit1 = output clamp. */
#define ACC_MAX64 ((int64_t)0x7FFFFFFFFFFFFFFFLL)
#define ACC_MIN64 (-(int64_t)0x7FFFFFFFFFFFFFFFLL)
#define OUT_MAX64 ((int64_t)2251799812636672LL)
#define OUT_MIN64 ((int64_t)-2251799813685248LL)

static int32_t rtl_row(const int8_t* w, const uint8_t* e, const int16_t* xq,
                       const uint32_t* xs_bits, int nb, int* flags) {
    int64_t acc = 0;
    for (int b = 0; b < nb; b++) {
        int32_t D = 0;
        for (int i = 0; i < 64; i++) D += (int32_t)w[64 * b + i] * (int32_t)xq[64 * b + i];
        uint32_t xb = xs_bits[b];
        int eb = (int)((xb >> 23) & 0xFF);
        int norm = (eb != 0) && (eb != 255);
        int64_t mant = norm ? (int64_t)((1u << 16) | ((xb >> 7) & 0xFFFFu)) : 0;
        int ex = norm ? eb - 127 : 0;
        int sh = ex + ((int)e[b] - 134) + 24;
        int clamped = sh > 63;
        int shc = sh > 63 ? 63 : (sh < -63 ? -63 : sh);
        int64_t prod = (int64_t)D * mant;
        uint64_t pabs = (uint64_t)(D < 0 ? -(int64_t)D : (int64_t)D) * (uint64_t)mant;
        int ovf_sh = (shc >= 16) ? (63 - shc) : 63;
        int ovf = ((pabs >> ovf_sh) != 0) || clamped;
        int64_t contrib;
        if (ovf) {
            contrib = (prod < 0) ? ACC_MIN64 : ACC_MAX64;
            *flags |= 1;
        } else if (shc >= 0) {
            contrib = (int64_t)((uint64_t)prod << shc);
        } else {
            contrib = (prod >> ((-shc) & 7)) >> (8 * (((-sh) >> 3) & 7));
        }
        int64_t sum;
        if (__builtin_add_overflow(acc, contrib, &sum)) {
            acc = (acc < 0) ? ACC_MIN64 : ACC_MAX64;
            *flags |= 1;
        } else {
            acc = sum;
        }
    }
    int64_t o = acc;
    if (o > OUT_MAX64) { o = OUT_MAX64; *flags |= 2; }
    if (o < OUT_MIN64) { o = OUT_MIN64; *flags |= 2; }
    return (int32_t)(o >> 20);
}

ORC_API int orc_bfp8_gemv_rtl20(int32_t* yw, const int16_t* xq, const float* xs,
                                const int8_t* mant, const uint8_t* exps, int M, int K) {
    int nb = K / 64;
    int flags = 0;
    uint32_t* bits = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(nb + 1));
    memcpy(bits, xs, sizeof(float) * (size_t)nb);
    for (int m = 0; m < M; m++)
        yw[m] = rtl_row(mant + (size_t)m * K, exps + (size_t)m * nb, xq, bits, nb, &flags);
    free(bits);
    return flags;
}

/* ----------------------------------------------------------- lm_head scores */
/* NEON order (qwen_kernels_opt.c:427-456; qwen_sampling.c:171-208): eight
 * fp32 chains c = i mod 8, acc_c = acc_c + E*h (VMLA, not fused), then
 * s = ((c0+c4) + (c2+c6)) + ((c1+c5) + (c3+c7)).  with_tail != 0 adds the
 * elements past the last multiple of 8 on scalar VFP (lm_head_topk,
 * qwen_sampling.c:205-208); with_tail == 0 drops them (lm_head_argmax,
 * qwen_kernels_opt.c:430). */
ORC_API void orc_lm_scores_neon(float* scores, const float* h, const uint16_t* E,
                                int vocab, int hidden, int with_tail) {
    for (int t = 0; t < vocab; t++) {
        const uint16_t* row = E + (size_t)t * hidden;
        float c[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int i = 0;
        for (; i + 8 <= hidden; i += 8)
            for (int j = 0; j < 8; j++)
                c[j] = neon_add(c[j], neon_mul(bf16_bits_to_f32(row[i + j]), h[i + j]));
        float a0 = neon_add(c[0], c[4]), a1 = neon_add(c[1], c[5]);
        float a2 = neon_add(c[2], c[6]), a3 = neon_add(c[3], c[7]);
        float s = neon_add(neon_add(a0, a2), neon_add(a1, a3));
        if (with_tail)
            for (; i < hidden; i++) s += h[i] * bf16_bits_to_f32(row[i]);
        scores[t] = s;
    }
}

/* Scalar build of both lm_head routines (qwen_kernels_opt.c:490-503,
 * qwen_sampling.c:250-266): score += h[i] * E[t][i], left to right. */
ORC_API void orc_lm_scores_scalar(float* scores, const float* h, const uint16_t* E,
                                  int vocab, int hidden) {
    for (int t = 0; t < vocab; t++) {
        const uint16_t* row = E + (size_t)t * hidden;
        float s = 0.0f;
        for (int i = 0; i < hidden; i++) s += h[i] * bf16_bits_to_f32(row[i]);
        scores[t] = s;
    }
}

/* Greedy pick (qwen_kernels_opt.c:402-403,450-487): best starts at -1e30 /
 * id 0, strict '>' in ascending id order, so ties go to the lowest id and a
 * NaN score never wins.  The 2-thread split merges with '>=' and gives the
 * same winner as one ascending scan. */
ORC_API int orc_argmax(const float* scores, int n) {
    float best = -1e30f;
    int id = 0;
    for (int t = 0; t < n; t++)
        if (scores[t] > best) { best = scores[t]; id = t; }
    return id;
}

/* Sorted top-k (qwen_sampling.c:117-155,209-215,283-353): only scores
 * strictly above -FLT_MAX are offered (NaN never is); the table keeps the k
 * best, score descending, equal scores in ascending id.  Returns min(k, n)
 * entries, fewer if fewer scores qualify; 0 on bad arguments. */
ORC_API int orc_topk(const float* scores, int n, int k, int* ids, float* out) {
    if (!scores || !ids || !out || n <= 0 || k <= 0) return 0;
    int kk = k < n ? k : n;
    int cnt = 0;
    for (int t = 0; t < n; t++) {
        float s = scores[t];
        if (!(s > -FLT_MAX)) continue;
        if (cnt == kk && !(s > out[kk - 1])) continue;
        int pos = (cnt < kk) ? cnt : kk - 1;
        while (pos > 0 && out[pos - 1] < s) {
            out[pos] = out[pos - 1];
            ids[pos] = ids[pos - 1];
            pos--;
        }
        out[pos] = s;
        ids[pos] = t;
        if (cnt < kk) cnt++;
    }
    return cnt;
}

/* The greedy and sampled lm_head entry points over a bf16 table. */
ORC_API int orc_lm_head_argmax(const float* h, const uint16_t* E, int vocab, int hidden) {
    float* s = (float*)malloc(sizeof(float) * (size_t)vocab);
    orc_lm_scores_neon(s, h, E, vocab, hidden, 0);
    int id = orc_argmax(s, vocab);
    free(s);
    return id;
}

ORC_API int orc_lm_head_topk(const float* h, const uint16_t* E, int vocab, int hidden,
                             int k, int* ids, float* out) {
    if (!h || !E || !ids || !out || vocab <= 0 || hidden <= 0 || k <= 0) return 0;
    float* s = (float*)malloc(sizeof(float) * (size_t)vocab);
    orc_lm_scores_neon(s, h, E, vocab, hidden, 1);
    int n = orc_topk(s, vocab, k, ids, out);
    free(s);
    return n;
}

/* BFP8 lm_head (new variant, no reference routine): bfp8_gemv NEON-path
 * scores, then the argmax and top-k rules above. */
ORC_API int orc_bfp8_lm_head(const float* h, const int8_t* mant, const uint8_t* exps,
                             int vocab, int hidden, int k, int* ids, float* out,
                             int* argmax_id) {
    float* s = (float*)malloc(sizeof(float) * (size_t)vocab);
    orc_bfp8_gemv_neon(s, h, mant, exps, vocab, hidden);
    *argmax_id = orc_argmax(s, vocab);
    int n = orc_topk(s, vocab, k, ids, out);
    free(s);
    return n;
}

/* ------------------------------------------------------------ generators */
/* Marsaglia xorshift32 (13, 17, 5), zero state remapped to 0x9E3779B9 -- the
 * generator the reference sampler and its self-test use
 * (04-板载脚本与工具/qwen_sampling.c:360-368, 536-561). */
ORC_API void orc_xorshift32(uint32_t* state, uint32_t* out, size_t n) {
    uint32_t x = *state;
    for (size_t i = 0; i < n; i++) {
        if (x == 0u) x = 0x9E3779B9u;
        x ^= x << 13;
        x ^= x >> 17;
        x ^= x << 5;
        out[i] = x;
    }
    *state = x;
}

/* The self-test fill rule (qwen_sampling.c:544-561): v = ((r >> 16) & 0xFFFF)
 * - 32768, f = v / 16384; tables keep the top 16 bits of f (bf16 truncation). */
ORC_API void orc_selftest_fill(uint32_t* state, uint16_t* tab, size_t n_tab, float* h, size_t n_h) {
    for (size_t i = 0; i < n_tab; i++) {
        uint32_t r;
        orc_xorshift32(state, &r, 1);
        int v = (int)((r >> 16) & 0xFFFFu) - 32768;
        float f = (float)v * (1.0f / 16384.0f);
        uint32_t bits;
        memcpy(&bits, &f, 4);
        tab[i] = (uint16_t)(bits >> 16);
    }
    for (size_t i = 0; i < n_h; i++) {
        uint32_t r;
        orc_xorshift32(state, &r, 1);
        int v = (int)((r >> 16) & 0xFFFFu) - 32768;
        h[i] = (float)v * (1.0f / 16384.0f);
    }
}
