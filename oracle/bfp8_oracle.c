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

/* ============================================ Gated-DeltaNet layer and token loop
 * The glue forward_linear_layer / forward_token_c run around the GEMVs
 * (qwen_kernels_opt.c:507-858, 938-1049).  Every routine takes `neon`: 1 is
 * the board build (Advanced SIMD lanes, flushed, VMLA not fused; scalar VFP
 * where the reference leaves the vector unit), 0 the portable build the
 * reference compiles to on x86 (plain C float arithmetic, the C library's
 * expf/log1pf). */

/* causal_conv1d_update_silu (qwen_kernels_opt.c:511-545): channel c has the
 * weights w[4c..4c+3] and the state s0/s1/s2 (three rows of C floats):
 * d = w0*s0 + w1*s1 + w2*s2 + w3*x, y = d / (1 + exp(-d)), then the state
 * shifts (s0 <- s1 <- s2 <- x).  NEON build, channels in groups of four:
 * the multiply and the three multiply-adds (product rounded first), the
 * exp_neon of -d and 1 + e on the vector unit, the division on VFP.
 * The portable build has no scalar loop for those groups: its loop starts at
 * C & ~3 (the vector loop that would cover channels below it is compiled
 * out), so it computes only a C % 4 tail and leaves every other channel's
 * output and state untouched -- restated as such for neon = 0. */
ORC_API void orc_conv1d_silu(float* y, const float* x, float* st, const float* w, int C, int neon) {
    float* s0 = st;
    float* s1 = st + C;
    float* s2 = st + 2 * C;
    int c = neon ? 0 : (C & ~3);
    if (neon)
        for (; c < (C & ~3); c++) {
            const float xc = x[c], t0 = s0[c], t1 = s1[c], t2 = s2[c];
            float d = neon_mul(w[4 * c], t0);
            d = neon_add(d, neon_mul(w[4 * c + 1], t1));
            d = neon_add(d, neon_mul(w[4 * c + 2], t2));
            d = neon_add(d, neon_mul(w[4 * c + 3], xc));
            y[c] = d / neon_add(1.0f, exp_neon_lane(-d));
            s0[c] = t1;
            s1[c] = t2;
            s2[c] = xc;
        }
    for (; c < C; c++) {
        const float xc = x[c];
        const float dot = w[4 * c] * s0[c] + w[4 * c + 1] * s1[c] + w[4 * c + 2] * s2[c] + w[4 * c + 3] * xc;
        y[c] = dot / (1.0f + expf(-dot));
        s0[c] = s1[c];
        s1[c] = s2[c];
        s2[c] = xc;
    }
}

/* Four flushed lane sums of a[i]*b[i] over i = 4j + l, combined as
 * (s0 + s2) + (s1 + s3) -- the VMLA accumulator, vadd(low, high), vpadd
 * reduction the reference uses for every vector dot (returns the number of
 * elements consumed: n rounded down to a multiple of 4). */
static int neon_dot4(const float* a, const float* b, int n, float* out) {
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int i = 0;
    for (; i + 4 <= n; i += 4)
        for (int l = 0; l < 4; l++) s[l] = neon_add(s[l], neon_mul(a[i + l], b[i + l]));
    *out = neon_add(neon_add(s[0], s[2]), neon_add(s[1], s[3]));
    return i;
}

/* qk_l2norm (qwen_kernels_opt.c:548-591): per head, k *= 1/sqrt(|k|^2 + 1e-6),
 * q *= (1/sqrt(D)) / sqrt(|q|^2 + 1e-6).  NEON build: the squared norms by
 * neon_dot4 (any tail on VFP), the scales on VFP, the products on the
 * vector unit (which leaves a D % 4 tail unscaled, as the reference does). */
ORC_API void orc_qk_l2norm(float* q, float* k, int H, int D, int neon) {
    const float q_scale = 1.0f / sqrtf((float)D);
    const float eps = 1e-6f;
    for (int h = 0; h < H; h++) {
        float* kh = k + (size_t)h * D;
        float* qh = q + (size_t)h * D;
        float k_sq = 0.0f, q_sq = 0.0f;
        int i = 0;
        if (neon) {
            neon_dot4(kh, kh, D, &k_sq);
            i = neon_dot4(qh, qh, D, &q_sq);
        }
        for (; i < D; i++) {
            k_sq += kh[i] * kh[i];
            q_sq += qh[i] * qh[i];
        }
        const float k_r = 1.0f / sqrtf(k_sq + eps);
        const float q_r = q_scale / sqrtf(q_sq + eps);
        if (neon) {
            for (i = 0; i < (D & ~3); i++) {
                kh[i] = neon_mul(kh[i], k_r);
                qh[i] = neon_mul(qh[i], q_r);
            }
        } else {
            for (i = 0; i < D; i++) {
                kh[i] *= k_r;
                qh[i] *= q_r;
            }
        }
    }
}

/* gdn_gates (qwen_kernels_opt.c:593-625): per head h, av = wa[h].x and
 * bv = wb[h].x (neon_dot4 on the NEON build, any tail on VFP);
 * beta = 1 / (1 + expf(-bv)); alpha = expf(nea[h] * log1pf(expf(av + dt[h])))
 * on VFP with the C library's expf / log1pf. */
ORC_API void orc_gdn_gates(float* alpha, float* beta, const float* x, const float* wa, const float* wb,
                           const float* nea, const float* dt, int H, int K, int neon) {
    for (int h = 0; h < H; h++) {
        const float* ra = wa + (size_t)h * K;
        const float* rb = wb + (size_t)h * K;
        float av = 0.0f, bv = 0.0f;
        int i = 0;
        if (neon) {
            neon_dot4(ra, x, K, &av);
            i = neon_dot4(rb, x, K, &bv);
        }
        for (; i < K; i++) {
            av += ra[i] * x[i];
            bv += rb[i] * x[i];
        }
        beta[h] = 1.0f / (1.0f + expf(-bv));
        const float z = av + dt[h];
        alpha[h] = expf(nea[h] * log1pf(expf(z)));
    }
}

/* gdn_recurrent_step (qwen_kernels_opt.c:664-829).  State of head h: D x D
 * floats, blocked so that S[i][j] sits at ((j/4 * D/4 + i/4) * 4 + j%4) * 4 +
 * i%4.  Per head: qk = q.k (neon_dot4 on the NEON build, one running sum on
 * the portable one); per column j: kv = sum_i S[i][j] k[i] and
 * qs = sum_i S[i][j] q[i] in ascending i (product rounded, then added);
 * d = (v - kv*a) * b; out = qs*a + qk*d; then S[i][j] = S*a + d*k[i].  Both
 * builds use that order; the NEON one flushes every step. */
ORC_API void orc_gdn_step(float* out, float* state, const float* q, const float* k, const float* v,
                          const float* alpha, const float* beta, int H, int D, int neon) {
    for (int h = 0; h < H; h++) {
        const float* qh = q + (size_t)h * D;
        const float* kh = k + (size_t)h * D;
        const float* vh = v + (size_t)h * D;
        float* oh = out + (size_t)h * D;
        const float a = alpha[h], b = beta[h];
        float* S = state + (size_t)h * D * D;
        float qk = 0.0f;
        if (neon)
            neon_dot4(qh, kh, D, &qk);
        else
            for (int i = 0; i < D; i++) qk += qh[i] * kh[i];
        for (int j0 = 0; j0 < D; j0 += 4) {
            float* B = S + (size_t)(j0 >> 2) * D * 4;
            float kv[4] = {0.0f, 0.0f, 0.0f, 0.0f}, qs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int i = 0; i < D; i++) {
                const int blk = (i >> 2) * 16 + (i & 3);
                for (int l = 0; l < 4; l++) {
                    const float t = B[blk + l * 4];
                    if (neon) {
                        kv[l] = neon_add(kv[l], neon_mul(t, kh[i]));
                        qs[l] = neon_add(qs[l], neon_mul(t, qh[i]));
                    } else {
                        kv[l] += kh[i] * t;
                        qs[l] += qh[i] * t;
                    }
                }
            }
            float dd[4];
            for (int l = 0; l < 4; l++) {
                if (neon) {
                    dd[l] = neon_mul(neon_sub(vh[j0 + l], neon_mul(kv[l], a)), b);
                    oh[j0 + l] = neon_add(neon_mul(qs[l], a), neon_mul(qk, dd[l]));
                } else {
                    dd[l] = b * (vh[j0 + l] - a * kv[l]);
                    oh[j0 + l] = a * qs[l] + qk * dd[l];
                }
            }
            for (int i = 0; i < D; i++) {
                const int blk = (i >> 2) * 16 + (i & 3);
                for (int l = 0; l < 4; l++) {
                    float* t = &B[blk + l * 4];
                    *t = neon ? neon_add(neon_mul(*t, a), neon_mul(dd[l], kh[i])) : a * *t + kh[i] * dd[l];
                }
            }
        }
    }
}

/* rmsnorm_gated (qwen_kernels_opt.c:832-858): per head, r = 1 / sqrtf(|x|^2 / D
 * + eps) (the squared norm by neon_dot4 on the NEON build); then on VFP
 * y = ((x * r) * w[i]) * (z / (1 + expf(-z))). */
ORC_API void orc_rmsnorm_gated(float* y, const float* x, const float* z, const float* w, int H, int D, float eps,
                               int neon) {
    for (int h = 0; h < H; h++) {
        const float* xh = x + (size_t)h * D;
        const float* zh = z + (size_t)h * D;
        float* yh = y + (size_t)h * D;
        float ss = 0.0f;
        int i = 0;
        if (neon) i = neon_dot4(xh, xh, D, &ss);
        for (; i < D; i++) ss += xh[i] * xh[i];
        const float r = 1.0f / sqrtf((ss / (float)D) + eps);
        for (i = 0; i < D; i++) {
            const float zi = zh[i];
            yh[i] = xh[i] * r * w[i] * (zi / (1.0f + expf(-zi)));
        }
    }
}

/* The plans of the token loop, field for field the reference's
 * (qwen_kernels_opt.c:866-917). */
typedef struct {
    const float* in_ln_w;
    const int8_t* mant_qkv;
    const uint8_t* exp_qkv;
    int M_qkv, K_qkv;
    const float* conv_w;
    float* conv_s;
    const float* wa;
    const float* wb;
    const float* nea;
    const float* dt;
    float* state;
    const int8_t* mant_z;
    const uint8_t* exp_z;
    int M_z, K_z;
    const float* norm_w;
    const int8_t* mant_o;
    const uint8_t* exp_o;
    int M_o, K_o;
    const float* post_ln_w;
    const int8_t* mant_gate;
    const uint8_t* exp_gate;
    int M_gate, K_gate;
    const int8_t* mant_up;
    const uint8_t* exp_up;
    int M_up, K_up;
    const int8_t* mant_down;
    const uint8_t* exp_down;
    int M_down, K_down;
} OrcLinearPlan;

typedef struct {
    const float* post_ln_w;
    const int8_t* mant_gate;
    const uint8_t* exp_gate;
    int M_gate, K_gate;
    const int8_t* mant_up;
    const uint8_t* exp_up;
    int M_up, K_up;
    const int8_t* mant_down;
    const uint8_t* exp_down;
    int M_down, K_down;
} OrcMlpPlan;

enum { kOrcHidden = 1024, kOrcHeads = 16, kOrcHeadDim = 128, kOrcVocab = 65536, kOrcLayers = 24 };

static void orc_gemv(float* y, const float* x, const int8_t* m, const uint8_t* e, int M, int K, int neon) {
    if (neon)
        orc_bfp8_gemv_neon(y, x, m, e, M, K);
    else
        orc_bfp8_gemv_scalar(y, x, m, e, M, K);
}
static void orc_rmsnorm(float* y, const float* x, const float* w, int n, int neon) {
    if (neon)
        orc_rmsnorm_neon(y, x, w, n, 1e-6f);
    else
        orc_rmsnorm_scalar(y, x, w, n, 1e-6f);
}

/* forward_mlp (qwen_kernels_opt.c:994-1004): h += down(swiglu(gate(n), up(n))),
 * n = rmsnorm(h, post_ln_w). */
ORC_API void orc_forward_mlp(const OrcMlpPlan* p, float* h, int neon) {
    const int H = p->K_gate, F = p->M_gate;   /* the reference hard-codes 1024 / 3584 */
    float* n = (float*)malloc(sizeof(float) * H);
    float* g = (float*)malloc(sizeof(float) * F);
    float* u = (float*)malloc(sizeof(float) * F);
    float* a = (float*)malloc(sizeof(float) * F);
    float* d = (float*)malloc(sizeof(float) * H);
    orc_rmsnorm(n, h, p->post_ln_w, H, neon);
    orc_gemv(g, n, p->mant_gate, p->exp_gate, p->M_gate, p->K_gate, neon);
    orc_gemv(u, n, p->mant_up, p->exp_up, p->M_up, p->K_up, neon);
    orc_swiglu(a, g, u, F, neon);
    orc_gemv(d, a, p->mant_down, p->exp_down, p->M_down, p->K_down, neon);
    orc_add_residual(h, d, H, neon);
    free(n); free(g); free(u); free(a); free(d);
}

/* forward_linear_layer (qwen_kernels_opt.c:938-992), the Gated-DeltaNet layer:
 * n = rmsnorm(h, in_ln); qkv GEMV; conv1d + SiLU over the 3*heads*D channels;
 * q, k = the first two thirds, l2-normalised; gates from n; the recurrent
 * step; z GEMV; rmsnorm_gated; o GEMV; h += o; then forward_mlp's steps. */
ORC_API void orc_forward_linear_layer(const OrcLinearPlan* p, float* h, int neon) {
    /* shapes from the plan (the reference hard-codes 1024 / 16 heads x 128) */
    const int H = p->K_qkv, D = kOrcHeadDim, V = p->M_z, NH = V / D;
    float* n = (float*)malloc(sizeof(float) * H);
    float* qkv = (float*)malloc(sizeof(float) * p->M_qkv);
    /* zeroed: the reference's workspace is a zero-initialised static, and its
     * portable build's conv never writes the channels below C & ~3 */
    float* mixed = (float*)calloc((size_t)p->M_qkv, sizeof(float));
    float* alpha = (float*)malloc(sizeof(float) * NH);
    float* beta = (float*)malloc(sizeof(float) * NH);
    float* attn = (float*)malloc(sizeof(float) * V);
    float* z = (float*)malloc(sizeof(float) * p->M_z);
    float* gated = (float*)malloc(sizeof(float) * V);
    float* o = (float*)malloc(sizeof(float) * p->M_o);
    orc_rmsnorm(n, h, p->in_ln_w, H, neon);
    orc_gemv(qkv, n, p->mant_qkv, p->exp_qkv, p->M_qkv, p->K_qkv, neon);
    orc_conv1d_silu(mixed, qkv, p->conv_s, p->conv_w, 3 * V, neon);
    orc_qk_l2norm(mixed, mixed + V, NH, D, neon);
    orc_gdn_gates(alpha, beta, n, p->wa, p->wb, p->nea, p->dt, NH, H, neon);
    orc_gdn_step(attn, p->state, mixed, mixed + V, mixed + 2 * V, alpha, beta, NH, D, neon);
    orc_gemv(z, n, p->mant_z, p->exp_z, p->M_z, p->K_z, neon);
    orc_rmsnorm_gated(gated, attn, z, p->norm_w, NH, D, 1e-6f, neon);
    orc_gemv(o, gated, p->mant_o, p->exp_o, p->M_o, p->K_o, neon);
    orc_add_residual(h, o, H, neon);
    OrcMlpPlan m = {p->post_ln_w, p->mant_gate, p->exp_gate, p->M_gate, p->K_gate, p->mant_up, p->exp_up,
                    p->M_up, p->K_up, p->mant_down, p->exp_down, p->M_down, p->K_down};
    orc_forward_mlp(&m, h, neon);
    free(n); free(qkv); free(mixed); free(attn); free(z); free(gated); free(o); free(alpha); free(beta);
}

typedef void (*OrcFullAttnCallback)(int layer, float* h, void* ctx);

/* forward_token_c (qwen_kernels_opt.c:1008-1049): h = the bf16 embedding row
 * of token_id % 65536; 24 layers (full-attention layers: the callback, then
 * forward_mlp; the others forward_linear_layer with the next linear plan);
 * the final rmsnorm; the lm_head argmax over 65536 rows (h keeps the last
 * residual stream). */
ORC_API int orc_forward_token(int token_id, float* h, const OrcLinearPlan* lps, const OrcMlpPlan* mps,
                              const int* is_full, const float* final_w, const uint16_t* E,
                              OrcFullAttnCallback cb, void* ctx, int neon) {
    const uint16_t* row = E + (size_t)(token_id % kOrcVocab) * kOrcHidden;
    for (int i = 0; i < kOrcHidden; i++) h[i] = bf16_bits_to_f32(row[i]);
    int li = 0;
    for (int l = 0; l < kOrcLayers; l++) {
        if (is_full[l]) {
            if (cb) cb(l, h, ctx);
            orc_forward_mlp(&mps[l], h, neon);
        } else {
            orc_forward_linear_layer(&lps[li++], h, neon);
        }
    }
    float* n = (float*)malloc(sizeof(float) * kOrcHidden);
    orc_rmsnorm(n, h, final_w, kOrcHidden, neon);
    float* s = (float*)malloc(sizeof(float) * kOrcVocab);
    if (neon)
        orc_lm_scores_neon(s, n, E, kOrcVocab, kOrcHidden, 0);
    else
        orc_lm_scores_scalar(s, n, E, kOrcVocab, kOrcHidden);
    const int id = orc_argmax(s, kOrcVocab);
    free(n);
    free(s);
    return id;
}
