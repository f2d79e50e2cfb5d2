// bfp8_gemv.cu -- exact-order BFP8 block-64 GEMV for sm_100a.
//
// Semantics (reference 04-板载脚本与工具/qwen_kernels_opt.c):
//   quant_x_blocks :182-205   x fp32 -> xq int16 = rint(x * (16384/amax)),
//                             xs = amax/16384 per 64-block
//   bfp8_gemv      :213-308   per row m and block b the int32 lane-class sums
//                             L_j = sum_{i = j mod 4} m*xq (j = 0..3); per lane
//                             f_j = f_j + ((float(L_j) * 2^(e-134)) * xs_b) in
//                             block order with flush-to-zero and no fused
//                             multiply-add; y = (f_0 + f_2) + (f_1 + f_3).
//                             An odd last row uses the scalar VFP form
//                             sum = sum + (float(D) * 2^(e-134)) * xs_b with
//                             D the whole block dot and IEEE subnormals.
// The result is bit-identical to the reference's NEON build.
//
// Two kernels per launch:
//  1. act_prep: every activation of the launch is quantized once into a
//     paired int16 layout (block b, group g = elements 8g..8g+7, word j =
//     the pair (xq[64b+8g+j], xq[64b+8g+4+j]), the operand order of __dp2a)
//     plus its block scales.  It releases the dependent launch at once.
//  2. gemv_warp (programmatic dependent launch): warp-autonomous streaming.
//     A work unit is 32 consecutive rows of one GEMV; a warp owns a unit
//     from its first byte to its output (lane = row), streaming it through a
//     private 3-stage ring: per stage two TMA boxes of 32 rows x 128 bytes
//     (SWIZZLE_128B, 4 blocks of every row) plus one bulk copy of those 4
//     blocks' activation pairs and scales, all on one mbarrier, while each
//     lane copies its row's four exponent bytes with cp.async.  Each lane
//     forms the four lane-class sums of a block with __dp2a (int16 pairs
//     against weight bytes paired by prmt) and keeps the four fp32 chains in
//     registers, so the float order is the reference's with no cross-thread
//     exchange and no CTA barrier.  Weight loads are issued before the kernel
//     waits on act_prep.  Units are handed out by an atomic counter (largest
//     K first) in grouped launches and round-robin for a single GEMV.
#include "bfp8_gemv.cuh"
#include "common.cuh"
#include "tma.cuh"
#include "topk.cuh"

#include <algorithm>
#include <cmath>
#include <numeric>
#include <vector>

namespace qb {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRows = 32;            // rows per unit (lane = row)
constexpr int kStage = 8192;         // bytes per stage: 32 rows x 256 bytes (4 blocks)
constexpr int kBox = 4096;           // one TMA box: 32 rows x 128 bytes
constexpr int kRing = 3;             // stages per warp
constexpr int kXp = 528;             // activation bytes per stage: 4 blocks x 128 B pairs + 4 scales
constexpr int kMaxSDesc = 160;       // GEMVs per grouped launch

size_t gemv_act_words(int K) { return (size_t)K / 2 + (size_t)K / 64; }

// ---------------------------------------------------------------- act_prep
struct PrepArgs {
    GemvDesc single;
    const GemvDesc* list;
    int n;
    const unsigned int* wait_flags;   // row-sharded stacks: inputs complete once every rank's flag
    unsigned int wait_epoch;          // reaches wait_epoch (0: no wait)
    const unsigned int* epoch_base;   // nullptr, or the counter wait_epoch is an offset from
    int world;
    unsigned int* err;
};

__device__ __forceinline__ const GemvDesc& prep_desc(const PrepArgs& A, int d) {
    return A.list ? A.list[d] : A.single;
}

// The reference block-64 quantizer on one block, lane l holding elements 2l
// and 2l+1 in `v`: q = 16384/amax, xq = rint(x*q) half-even, xs = amax/16384;
// a zero block when amax <= 1e-20 (quant_x_blocks, qwen_kernels_opt.c:182-205).
__device__ __forceinline__ void block_quant(float2 v, int& q0, int& q1, float& xs) {
    float a = fmaxf(fabsf(v.x), fabsf(v.y));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (a > 1e-20f) {
        const float q = __fdiv_rn(16384.0f, a);
        xs = __fdiv_rn(a, 16384.0f);
        q0 = __float2int_rn(__fmul_rn(v.x, q));
        q1 = __float2int_rn(__fmul_rn(v.y, q));
    } else {
        xs = 0.0f;
        q0 = q1 = 0;
    }
}

// swiglu (qwen_kernels_opt.c:365-386), NEON build, one lane:
// (g / (1 + exp_neon(-g))) * up, the add and the product flushed, the
// division on VFP (IEEE, g unflushed).
__device__ __forceinline__ float swiglu_lane(float g, float up) {
    const float d = add_ftz(1.0f, exp_neon_lane(-g));
    return mul_ftz(__fdiv_rn(g, d), up);
}

// Block b of the paired activation layout the GEMV consumes (global or
// shared memory) from lane l's int16 elements 2l, 2l+1 and the block scale.
__device__ __forceinline__ void block_store(uint32_t* xpairs, float* xscale, int b, int lane, int q0, int q1,
                                            float xs) {
    const uint32_t mine = ((uint32_t)q0 & 0xFFFFu) | ((uint32_t)q1 << 16);
    const uint32_t part = __shfl_down_sync(0xffffffffu, mine, 2);
    if ((lane & 3) < 2) {
        const int g = lane >> 2, p = 2 * (lane & 3);
        const uint32_t w0 = (mine & 0xFFFFu) | (part << 16);
        const uint32_t w1 = (mine >> 16) | (part & 0xFFFF0000u);
        *reinterpret_cast<uint2*>(xpairs + b * 32 + g * 4 + p) = make_uint2(w0, w1);
    }
    if (lane == 0) xscale[b] = xs;
}

// grid (n, chunks), kPrepThreads threads: CTA (d, c) prepares blocks
// [kPrepChunk*c, kPrepChunk*(c+1)) of GEMV d, each warp kPrepPerWarp blocks
// with all their loads in flight at once.  Small CTAs (64 threads, <= 32
// registers) fit beside a resident gemv_warp CTA, so the PDL-launched GEMV
// starts streaming weights while the activations are still being prepared.
constexpr int kPrepThreads = 64;
constexpr int kPrepPerWarp = 4;
constexpr int kPrepChunk = kPrepThreads / 32 * kPrepPerWarp;

__global__ void __launch_bounds__(kPrepThreads) act_prep_kernel(const __grid_constant__ PrepArgs A) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // the descriptor is immutable: its fields are read before the wait below
    const GemvDesc& D = prep_desc(A, blockIdx.x);
    const int nb = D.K >> 6;
    const float* x = D.x;
    const int16_t* xq = D.xq;
    const float* xsrc = D.xs;
    uint32_t* xpairs = D.xpairs;
    float* xscale = D.xscale;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b0 = blockIdx.y * kPrepChunk + warp * kPrepPerWarp;
    // warps without blocks leave at once (a CTA that waits for peers keeps
    // them for the block-wide wait)
    if (!A.wait_epoch && b0 >= nb) return;
    // launched as a programmatic dependent of the stream's previous kernel:
    // x (possibly its output) and this plan's scratch (which it may still
    // read) are touched, and peer flags polled, only once that grid has
    // completed -- so a row-sharded wait never spins beside the kernel on
    // this GPU that raises this rank's own flag (a no-op for a plain launch)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (A.wait_epoch) {
        wait_peer_flags(A.wait_flags, A.world, A.wait_epoch, A.epoch_base, A.err);
        if (b0 >= nb) return;
    }
    float2 v[kPrepPerWarp];
    if (x) {
#pragma unroll
        for (int j = 0; j < kPrepPerWarp; j++)
            if (b0 + j < nb) v[j] = reinterpret_cast<const float2*>(x + 64 * (b0 + j))[lane];
    }
#pragma unroll
    for (int j = 0; j < kPrepPerWarp; j++) {
        const int b = b0 + j;
        if (b >= nb) break;
        int q0, q1;
        float xs;
        if (x) {
            block_quant(v[j], q0, q1, xs);
        } else {
            const short2 w = reinterpret_cast<const short2*>(xq + 64 * b)[lane];
            q0 = w.x;
            q1 = w.y;
            xs = xsrc[b];
        }
        block_store(xpairs, xscale, b, lane, q0, q1, xs);
    }
}

// ---------------------------------------------------------------- gemv_warp
struct WArgs {
    GemvDesc single;
    const GemvDesc* list;   // nullptr -> `single`
    int n;
    int total_units;
    unsigned int* ctr;      // [0] next unit, [1] exhausted warps; nullptr -> round-robin
    unsigned int* err;
    // lm_head epilogue
    LmScratch* sc;
    int kk;
    int* out_id;
    int* out_ids;
    float* out_scores;
    int* out_n;
    int lm_warp_lists;      // top-k in per-warp register lists (k <= 64 and too many rows per CTA to buffer)
    int res_act;            // single GEMV, small K: every CTA quantizes the whole activation into its own
                            // shared memory (no act_prep kernel, no activation copies per stage)
    const float* norm_w;    // res_act only: x is first rmsnorm-ed with these weights (nullptr: not)
    float norm_eps;
    const float* norm_res;  // with norm_w: x + norm_res is normalized (nullptr: x) ...
    float* norm_xout;       // ... and CTA 0 stores x + norm_res there (the updated residual stream)
    float* norm_out;        // with norm_w: CTA 0 also stores the normalized vector there (nullptr: not)
    unsigned int* rtl_flags;   // RTL mode: sticky flags word (may be null)
    const float* glu_up;    // res_act only: the activation is swiglu(x, glu_up) (nullptr: x)
    SyncArgs sync;          // row-sharded stacks: completion signal (sig_epoch 0: none)
    // split kernel only: units [second_begin, total_units) run `second`, a
    // GEMV of the same activation (same x and K) -- two projections of one
    // normalized vector in one launch (second_begin 0: none)
    int second_begin;
    GemvDesc second;
    // split kernel only: y is the residual stream, updated in place with the
    // reference's add_residual arithmetic (y[i] += result: flushed lane adds
    // for i below M & ~3, IEEE adds for the tail)
    int res_epi;
};

__device__ __forceinline__ const GemvDesc& wdesc(const WArgs& A, int d) {
    return A.list ? A.list[d] : A.single;
}

// What a warp needs to know about a GEMV, copied to shared memory at start
// so that mapping a claimed unit to its GEMV never touches global memory.
struct SDesc {
    int unit_begin, M, K, nseg;
    int seg_stages, pad0, pad1, pad2;
    const uint8_t* exps;
    const uint32_t* xp;
    const float* xs;
    const void* tmap;
    float* y;
    float* partial;
    unsigned int* tickets;
    const PeerOut* peer;
};

struct Unit {
    bool valid;
    int d, r0, M, K, nb, g, s, st0, st1;   // row group g, K segment s = stages [st0, st1)
    const uint8_t* exps;
    const uint32_t* xp;
    const float* xs;
};

__device__ __forceinline__ Unit load_unit(const SDesc* T, int n, int total_units, int u) {
    Unit U;
    U.valid = u < total_units;
    if (!U.valid) return U;
    int lo = 0, hi = n - 1;
    while (lo < hi) {   // largest d with unit_begin <= u
        const int mid = (lo + hi + 1) >> 1;
        if (T[mid].unit_begin <= u) lo = mid;
        else hi = mid - 1;
    }
    const SDesc& D = T[lo];
    const int local = u - D.unit_begin;
    U.d = lo;
    U.g = local / D.nseg;
    U.s = local - U.g * D.nseg;
    U.r0 = U.g * kRows;
    U.M = D.M;
    U.K = D.K;
    U.nb = D.K >> 6;
    U.st0 = U.s * D.seg_stages;
    U.st1 = min(D.K >> 8, U.st0 + D.seg_stages);
    U.exps = D.exps;
    U.xp = D.xp;
    U.xs = D.xs;
    return U;
}

struct LmState {
    unsigned long long best;
    unsigned long long* cand;
    int* cand_count;
    // k <= 64: every warp keeps its best 64 keys in registers (element
    // i = r*32 + lane in r_r, descending); thr is the 64th of them
    bool wl;
    unsigned long long r0, r1, thr;
};

// A row-sharded GEMV's output row into every rank's full vector.
__device__ __forceinline__ void store_peers(const PeerOut* P, int row, float v) {
    const int n = P->n, g = P->row_base + row;
    for (int r = 0; r < n; r++) P->y[r][g] = v;
}

// A whole-K unit's row results (split segments are published by the caller).
template <bool LM>
__device__ __forceinline__ void unit_result(const WArgs& A, const SDesc* T, const Unit& U, int lane, float yv,
                                            LmState& lm) {
    const int row = U.r0 + lane;
    if (LM) {
        const bool ok = row < U.M;
        if (ok && yv > -1e30f) {
            const unsigned long long k = cand_key(yv, row);
            lm.best = k > lm.best ? k : lm.best;
        }
        if (A.kk > 0) {
            if (lm.wl) {   // whole warp: fold the unit's 32 scores into the warp's top-64
                const unsigned long long key = (ok && yv > -3.402823466e38f) ? cand_key(yv, row) : 0ull;
                if (__any_sync(0xffffffffu, key > lm.thr)) {
                    warp_fold64(lm.r0, lm.r1, key, 0ull);
                    lm.thr = __shfl_sync(0xffffffffu, lm.r1, 31);
                }
            } else {   // append the unit's keys to the CTA's buffer (one atomic per warp)
                const bool take = ok && yv > -3.402823466e38f;
                const unsigned int bal = __ballot_sync(0xffffffffu, take);
                int base = 0;
                if (lane == 0 && bal) base = atomicAdd(lm.cand_count, __popc(bal));
                base = __shfl_sync(0xffffffffu, base, 0);
                const int p = base + __popc(bal & ((1u << lane) - 1u));
                if (take && p < kCandCap) lm.cand[p] = cand_key(yv, row);
            }
        }
        return;
    }
    if (row >= U.M) return;
    T[U.d].y[row] = yv;
    if (T[U.d].peer) store_peers(T[U.d].peer, row, yv);
}

// ---------------------------------------------------------- RTL dequant mode
// The FPGA dequant datapath (02-RTL与仿真/gemv_core.v:299-534), integer only:
// the block scale xs decodes to a 17-bit mantissa 1.f[22:7] (truncated) and
// exponent Ex (zero / subnormal / inf / NaN xs -> mantissa 0, Ex 0); with
// sh = Ex + e - 110 the block adds D * mant * 2^sh to a 64-bit accumulator
// carrying 40 fraction bits.  sh is clamped to [-63, 63]; a clamped positive
// shift, or a left shift that loses bits of |D * mant|, saturates the term to
// +-(2^63 - 1) by the sign of the product; the row sum saturates the same way.
// The shifter works in two stages (:374-428): the low three bits of the
// amount come from the clamped shift, the high three from the unclamped one,
// so a shift below -63 moves right by 7 + 8 * ((-sh >> 3) & 7), as the
// hardware does.
// The row's word is clamp(acc, -2^31 << 20, (2^31 - 1) << 20) bits [51:20],
// i.e. floor(y * 2^20).  Flags: bit 0 a term or the sum saturated, bit 1 the
// output was clamped (the RTL's sticky saturation bit).
constexpr long long kRtlAccMax = 0x7FFFFFFFFFFFFFFFll;
constexpr long long kRtlAccMin = -0x7FFFFFFFFFFFFFFFll;
constexpr long long kRtlOutMax = 2251799812636672ll;    // (2^31 - 1) << 20
constexpr long long kRtlOutMin = -2251799813685248ll;   // -2^31 << 20

__device__ __forceinline__ void rtl_block(long long& acc, unsigned int& flags, int D, uint32_t xsb, uint32_t e) {
    const uint32_t eb = (xsb >> 23) & 0xFFu;
    const bool norm = eb != 0u && eb != 255u;
    const unsigned long long mant = norm ? (unsigned long long)((1u << 16) | ((xsb >> 7) & 0xFFFFu)) : 0ull;
    const int sh = (norm ? (int)eb - 127 : 0) + (int)e - 110;
    const int shc = sh > 63 ? 63 : (sh < -63 ? -63 : sh);
    const long long prod = (long long)D * (long long)mant;                   // |prod| < 2^45
    const unsigned long long pabs = (unsigned long long)(D < 0 ? -(long long)D : (long long)D) * mant;
    const int ovf_sh = shc >= 16 ? 63 - shc : 63;
    long long term;
    if (sh > 63 || (pabs >> ovf_sh) != 0ull) {
        term = prod < 0 ? kRtlAccMin : kRtlAccMax;
        flags |= 1u;
    } else if (shc >= 0) {
        term = (long long)((unsigned long long)prod << shc);
    } else {
        term = (prod >> ((-shc) & 7)) >> (8 * (((-sh) >> 3) & 7));   // arithmetic: floors
    }
    const long long sum = (long long)((unsigned long long)acc + (unsigned long long)term);
    if (((acc ^ sum) & (term ^ sum)) < 0) {   // signed overflow: acc and term share the sign sum lost
        acc = acc < 0 ? kRtlAccMin : kRtlAccMax;
        flags |= 1u;
    } else {
        acc = sum;
    }
}

__device__ __forceinline__ int rtl_word(long long acc, unsigned int& flags) {
    if (acc > kRtlOutMax) {
        acc = kRtlOutMax;
        flags |= 2u;
    } else if (acc < kRtlOutMin) {
        acc = kRtlOutMin;
        flags |= 2u;
    }
    return (int)(acc >> 20);
}

// Lane-class sums L_j = sum over i = j mod 4 of m*xq for block jb of a
// stage (four 16-byte chunks of this lane's swizzled row, the paired int16
// activation of the block), with __dp2a.
__device__ __forceinline__ void lane_sums(const unsigned char* st, const uint4* xst, int sw, int jb, int& L0,
                                          int& L1, int& L2, int& L3) {
    const unsigned char* rowp = st + (jb >> 1) * kBox;
    const int cb = (jb & 1) * 4;
    const uint4* xb = xst + jb * 8;
    int A0 = 0, A1 = 0, A2 = 0, A3 = 0, B0 = 0, B1 = 0, B2 = 0, B3 = 0;
#pragma unroll
    for (int cc = 0; cc < 4; cc++) {
        const uint4 w = *reinterpret_cast<const uint4*>(rowp + (((cb + cc) ^ sw) << 4));
        const uint4 xa = xb[2 * cc], xc = xb[2 * cc + 1];
        const int p01 = (int)__byte_perm(w.x, w.y, 0x5140), p23 = (int)__byte_perm(w.x, w.y, 0x7362);
        A0 = __dp2a_lo((int)xa.x, p01, A0);
        A1 = __dp2a_hi((int)xa.y, p01, A1);
        A2 = __dp2a_lo((int)xa.z, p23, A2);
        A3 = __dp2a_hi((int)xa.w, p23, A3);
        const int q01 = (int)__byte_perm(w.z, w.w, 0x5140), q23 = (int)__byte_perm(w.z, w.w, 0x7362);
        B0 = __dp2a_lo((int)xc.x, q01, B0);
        B1 = __dp2a_hi((int)xc.y, q01, B1);
        B2 = __dp2a_lo((int)xc.z, q23, B2);
        B3 = __dp2a_hi((int)xc.w, q23, B3);
    }
    L0 = A0 + B0;
    L1 = A1 + B1;
    L2 = A2 + B2;
    L3 = A3 + B3;
}

// The 4 blocks of one stage for this lane's row: lane-class sums, then the
// reference float steps into the four chains (or, for the odd last row, the
// scalar form into fo).
template <bool ODD, bool FAST>
__device__ __forceinline__ void stage_blocks(const unsigned char* st, const uint4* xst, const float* xsst,
                                             uint32_t ew, int sw, bool odd, float& f0, float& f1, float& f2,
                                             float& f3, float& fo) {
#pragma unroll
    for (int jb = 0; jb < 4; jb++) {
        int L0, L1, L2, L3;
        lane_sums(st, xst, sw, jb, L0, L1, L2, L3);
        const uint32_t e = (ew >> (8 * jb)) & 0xFFu;
        const float xsb = xsst[jb];
        if (FAST) {
            // one int32 dot per block, one fused multiply-add per block
            f0 = __fmaf_rn(i2f_rn((L0 + L1) + (L2 + L3)), __fmul_rn(exp_scale_ieee(e), xsb), f0);
        } else if (!ODD || !odd) {
            const float S = exp_scale_ftz(e);
            f0 = add_ftz(f0, mul_ftz(mul_ftz(i2f_rn(L0), S), xsb));
            f1 = add_ftz(f1, mul_ftz(mul_ftz(i2f_rn(L1), S), xsb));
            f2 = add_ftz(f2, mul_ftz(mul_ftz(i2f_rn(L2), S), xsb));
            f3 = add_ftz(f3, mul_ftz(mul_ftz(i2f_rn(L3), S), xsb));
        } else {
            fo = add_rn(fo, mul_rn(mul_rn(i2f_rn(L0 + L1 + L2 + L3), exp_scale_ieee(e)), xsb));
        }
    }
}

// The 4 blocks of one stage in the RTL dequant mode: one int32 dot per block
// into the row's 64-bit fixed-point accumulator.
__device__ __forceinline__ void stage_blocks_rtl(const unsigned char* st, const uint4* xst, const float* xsst,
                                                 uint32_t ew, int sw, long long& acc, unsigned int& flags) {
#pragma unroll
    for (int jb = 0; jb < 4; jb++) {
        int L0, L1, L2, L3;
        lane_sums(st, xst, sw, jb, L0, L1, L2, L3);
        rtl_block(acc, flags, (L0 + L1) + (L2 + L3), __float_as_uint(xsst[jb]), (ew >> (8 * jb)) & 0xFFu);
    }
}

// Resident activation of a single GEMV: every CTA quantizes all K/64 blocks
// of the activation into its own shared memory at `xact` (paired int16 words,
// 2K bytes, then the K/64 fp32 scales), applying first -- as the flags of A
// say -- the reference's swiglu (NEON build) or its add_residual + rmsnorm
// (NEON order; CTA 0 also stores the updated residual stream).  Every thread
// of the CTA calls it; it ends with a CTA barrier.
__device__ __forceinline__ void quantize_resident(const WArgs& A, const GemvDesc& D, unsigned char* xact, int warp,
                                                  int lane, float* stage = nullptr) {
    const int nb = D.K >> 6;
    uint32_t* xp = reinterpret_cast<uint32_t*>(xact);
    float* xsc = reinterpret_cast<float*>(xact + (size_t)D.K * 2);
    float nr = 0.0f;   // rmsnorm scale
    if (A.norm_w) {
        // rmsnorm, the reference's NEON build (qwen_kernels_opt.c:140-172):
        // four lane sums of x*x over i = 4j + l (multiply, then add, both
        // flushed), combined as (s0 + s2) + (s1 + s3); then, in IEEE
        // single precision, r = 1 / sqrt(sum / K + eps)
        __shared__ float s_nr;
        if (stage) {
            // the whole CTA first brings x (+ res: add_residual, qwen_kernels_opt.c:
            // 388-396, flushed lane adds) into shared memory with coalesced
            // 8-byte loads, so the four sequential chains below read shared
            // memory and the quantizer reads the same values
            for (int i = threadIdx.x; i < (D.K >> 1); i += blockDim.x) {
                float2 v = reinterpret_cast<const float2*>(D.x)[i];
                if (A.norm_res) {
                    const float2 r = reinterpret_cast<const float2*>(A.norm_res)[i];
                    v = make_float2(add_ftz(v.x, r.x), add_ftz(v.y, r.y));
                }
                reinterpret_cast<float2*>(stage)[i] = v;
            }
            __syncthreads();
        }
        if (warp == 0) {
            float acc = 0.0f;
            if (lane < 4) {
                if (stage) {
#pragma unroll 8
                    for (int i = lane; i < D.K; i += 4) acc = add_ftz(acc, mul_ftz(stage[i], stage[i]));
                } else {
                    for (int i = lane; i < D.K; i += 4) {
                        // add_residual (qwen_kernels_opt.c:388-396): flushed lane adds
                        const float v = A.norm_res ? add_ftz(D.x[i], A.norm_res[i]) : D.x[i];
                        acc = add_ftz(acc, mul_ftz(v, v));
                    }
                }
            }
            const float pair = add_ftz(acc, __shfl_down_sync(0xffffffffu, acc, 2));   // s0+s2, s1+s3
            const float other = __shfl_down_sync(0xffffffffu, pair, 1);
            if (lane == 0) {
                const float sum = add_ftz(pair, other);
                s_nr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)D.K), A.norm_eps)));
            }
        }
        __syncthreads();
        nr = s_nr;
    }
    for (int b0 = warp; b0 < nb; b0 += 4 * kWarps) {
        float2 v[4];
        if (D.x) {
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (b0 + j * kWarps < nb)
                    v[j] = reinterpret_cast<const float2*>((stage ? stage : D.x) + 64 * (b0 + j * kWarps))[lane];
            if (A.glu_up) {   // x holds the gate projection: swiglu(gate, up)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (b0 + j * kWarps < nb) {
                        const float2 u = reinterpret_cast<const float2*>(A.glu_up + 64 * (b0 + j * kWarps))[lane];
                        v[j].x = swiglu_lane(v[j].x, u.x);
                        v[j].y = swiglu_lane(v[j].y, u.y);
                    }
            }
            if (A.norm_w) {   // y = x * (r * (1 + w)), flushed like the vector unit
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (b0 + j * kWarps < nb) {
                        if (A.norm_res) {
                            if (!stage) {   // staged values already hold x + res
                                const float2 rr =
                                    reinterpret_cast<const float2*>(A.norm_res + 64 * (b0 + j * kWarps))[lane];
                                v[j].x = add_ftz(v[j].x, rr.x);
                                v[j].y = add_ftz(v[j].y, rr.y);
                            }
                            if (blockIdx.x == 0)
                                reinterpret_cast<float2*>(A.norm_xout + 64 * (b0 + j * kWarps))[lane] = v[j];
                        }
                        const float2 w =
                            reinterpret_cast<const float2*>(A.norm_w + 64 * (b0 + j * kWarps))[lane];
                        v[j].x = mul_ftz(v[j].x, mul_ftz(nr, add_ftz(1.0f, w.x)));
                        v[j].y = mul_ftz(v[j].y, mul_ftz(nr, add_ftz(1.0f, w.y)));
                        if (A.norm_out && blockIdx.x == 0)
                            reinterpret_cast<float2*>(A.norm_out + 64 * (b0 + j * kWarps))[lane] = v[j];
                    }
            }
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int b = b0 + j * kWarps;
            if (b >= nb) break;
            int q0, q1;
            float xs;
            if (D.x) {
                block_quant(v[j], q0, q1, xs);
            } else {
                short2 w = reinterpret_cast<const short2*>(D.xq + 64 * b)[lane];
                q0 = w.x;
                q1 = w.y;
                xs = D.xs[b];
            }
            block_store(xp, xsc, b, lane, q0, q1, xs);
        }
    }
    __syncthreads();
}

// LM: lm_head epilogue (argmax / top-k instead of stores).  FAST: fast-mode
// arithmetic.  RTL: the RTL dequant mode (one int32 word per row, stored in
// y's bits, sticky flags ORed into A.rtl_flags).
template <bool LM, bool FAST, bool RTL>
// <= 128 registers (no spills): half of the SM's 65536 stay free, so the next
// launch's input quantizer CTAs (64 threads, <= 32 registers) run many at a
// time beside a resident GEMV CTA -- at a 248-register cap only one fit, and
// the quantizer's waves between the steps of a stack cost 6% of a token
__global__ void __maxnreg__(128) gemv_warp_kernel(const __grid_constant__ WArgs A) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                           ~uintptr_t(1023));
    unsigned char* rings = smem;                                            // [warp][slot] 8 KB
    unsigned char* xrings = smem + kWarps * kRing * kStage;                 // [warp][slot] 528 B
    unsigned char* erings = xrings + kWarps * kRing * kXp;                  // [warp][slot][lane] 4 B
    uint64_t* bars = reinterpret_cast<uint64_t*>(erings + kWarps * kRing * 128);   // [warp][slot]
    SDesc* sdesc = reinterpret_cast<SDesc*>(bars + kWarps * kRing);                  // [n]
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(sdesc + A.n);
    __shared__ int s_cand_count;
    __shared__ unsigned long long s_red[kWarps];

    // a following act_prep launched as this grid's programmatic dependent
    // may start now (it waits for this grid's completion before it touches
    // memory), and so may the next GEMV behind it: its CTAs take the SMs of
    // this grid's finished CTAs and prefetch their first weight stages
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned char* ring = rings + warp * kRing * kStage;
    unsigned char* xring = xrings + warp * kRing * kXp;
    unsigned char* ering = erings + warp * kRing * 128;
    uint64_t* bar = bars + warp * kRing;
    if (threadIdx.x == 0) s_cand_count = 0;
    if (lane == 0) {
        for (int s = 0; s < kRing; s++) mbar_init(&bar[s], 1);
        fence_barrier_init();
    }
    for (int d = threadIdx.x; d < A.n; d += kThreads) {
        const GemvDesc& D = wdesc(A, d);
        SDesc t;
        t.unit_begin = D.unit_begin;
        t.M = D.M;
        t.K = D.K;
        t.nseg = D.nseg;
        t.seg_stages = D.seg_stages;
        t.pad0 = t.pad1 = t.pad2 = 0;
        t.partial = D.partial;
        t.tickets = D.tickets;
        t.exps = D.exps;
        t.xp = D.xpairs;
        t.xs = D.xscale;
        t.tmap = &D.tmap;
        t.y = D.y;
        t.peer = D.peer;
        sdesc[d] = t;
    }
    __syncthreads();
    const int nd = A.n, nu_total = A.total_units;

    LmState lm;
    lm.best = 0ull;
    lm.cand = cand;
    lm.cand_count = &s_cand_count;
    lm.wl = A.kk > 0 && A.lm_warp_lists;
    lm.r0 = lm.r1 = lm.thr = 0ull;

    const int W = gridDim.x * kWarps;
    // static schedule: CTA c owns the contiguous units [U*c/G, U*(c+1)/G)
    // (13 or 14 of 2048 on 148 SMs rather than 8 or 16), its warps take
    // them in turn
    const int cta_end = (int)(((long long)nu_total * (blockIdx.x + 1)) / gridDim.x);
    int rr_next = (int)(((long long)nu_total * blockIdx.x) / gridDim.x) + warp;
    bool exhausted = false;
    auto claim = [&]() -> int {
        if (exhausted) return nu_total;
        int u;
        if (A.ctr) {
            // units [0, W) go to the warps statically (warp gw starts on unit
            // gw), the counter hands out the rest
            unsigned int v = 0;
            if (lane == 0) v = atomicAdd(&A.ctr[0], 1u) + (unsigned int)W;
            u = (int)__shfl_sync(0xffffffffu, v, 0);
            if (u >= nu_total) {
                exhausted = true;
                __threadfence();
                if (lane == 0 && atomicAdd(&A.ctr[1], 1u) == (unsigned int)W - 1u) {
                    // every warp has seen the end: leave the counters zero
                    A.ctr[0] = 0u;
                    A.ctr[1] = 0u;
                }
            }
        } else {
            u = rr_next < cta_end ? rr_next : nu_total;
            rr_next += kWarps;
            if (u >= nu_total) exhausted = true;
        }
        return u < nu_total ? u : nu_total;
    };

    // producer: claimed units in a two-entry ring (it runs at most one unit
    // ahead of the consumer); the claim after the producer's current unit is
    // requested as soon as that unit starts, so the atomic's round trip
    // overlaps the unit's streaming
    int claimed0, claimed1;          // claim sequence entries 2j and 2j+1
    int kp = 0;                      // index of the producer's unit in the claim sequence
    const int gw = blockIdx.x * kWarps + warp;
    claimed0 = A.ctr ? (gw < nu_total ? gw : nu_total) : claim();
    claimed1 = nu_total;
    int ahead = nu_total;            // claimed once the activations are ready (its round trip overlaps their copies)
    Unit pu = load_unit(sdesc, nd, nu_total, claimed0);
    int ps = pu.valid ? pu.st0 : 0;
    if (lane == 0 && pu.valid) tma_prefetch_desc(sdesc[pu.d].tmap);

    // One stage: both weight boxes and the stage's activation slice (pairs +
    // scales of its 4 blocks) land on bar[slot].  The activation slice comes
    // from act_prep, so the stages issued before griddepcontrol.wait defer
    // their activation copies (the barrier already expects those bytes).
    static_assert(kRing == 3, "two deferred activation copies are tracked");
    const uint32_t* pend_xp0 = nullptr;
    const uint32_t* pend_xp1 = nullptr;
    const float* pend_xs0 = nullptr;
    const float* pend_xs1 = nullptr;
    const bool res = A.res_act != 0;
    auto issue = [&](int slot, bool xp_ready) {
        if (pu.valid) {
            if (lane == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive_expect_tx(&bar[slot], res ? kStage : kStage + kXp);
                const void* tm = sdesc[pu.d].tmap;
                tma_load_2d(ring + slot * kStage, tm, ps * 256, pu.r0, &bar[slot]);
                tma_load_2d(ring + slot * kStage + kBox, tm, ps * 256 + 128, pu.r0, &bar[slot]);
                if (xp_ready && !res) {
                    bulk_load(xring + slot * kXp, pu.xp + ps * 128, 512, &bar[slot]);
                    bulk_load(xring + slot * kXp + 512, pu.xs + ps * 4, 16, &bar[slot]);
                }
            }
            if (!xp_ready && !res) {
                if (slot == 0) {
                    pend_xp0 = pu.xp + ps * 128;
                    pend_xs0 = pu.xs + ps * 4;
                } else {
                    pend_xp1 = pu.xp + ps * 128;
                    pend_xs1 = pu.xs + ps * 4;
                }
            }
            if (pu.r0 + lane < pu.M)
                cp_async4(ering + slot * 128 + lane * 4, pu.exps + (size_t)(pu.r0 + lane) * pu.nb + ps * 4);
            if (++ps == pu.st1) {
                kp++;
                const int nu = ahead;
                if (kp & 1) claimed1 = nu;
                else claimed0 = nu;
                pu = load_unit(sdesc, nd, nu_total, nu);
                ps = pu.valid ? pu.st0 : 0;
                ahead = claim();
            }
        }
        cp_async_commit();
    };

    // a unit has >= 2 stages, so the first issue never needs the next claim;
    // the second goes out now unless it could finish the unit
    issue(0, false);
    bool issued1 = false;
    if (!pu.valid || pu.st1 - ps >= 2) {
        issue(1, false);
        issued1 = true;
    }

    if (res) {
        // launched as a programmatic dependent of the stream's previous
        // kernel: its weight stages are already in flight; the activation
        // (maybe that kernel's output) is read, and anything written, only now
        asm volatile("griddepcontrol.wait;" ::: "memory");
        quantize_resident(A, wdesc(A, 0), xrings, warp, lane);
    } else {
        // the activations come from act_prep (programmatic dependent launch)
        asm volatile("griddepcontrol.wait;" ::: "memory");
    }
    if (lane == 0 && !res) {
        if (pend_xp0) {
            bulk_load(xring, pend_xp0, 512, &bar[0]);
            bulk_load(xring + 512, pend_xs0, 16, &bar[0]);
        }
        if (pend_xp1) {
            bulk_load(xring + kXp, pend_xp1, 512, &bar[1]);
            bulk_load(xring + kXp + 512, pend_xs1, 16, &bar[1]);
        }
    }
    ahead = claim();
    if (!issued1) issue(1, true);

    int kc = 0;
    Unit cu = load_unit(sdesc, nd, nu_total, claimed0);
    int cs = cu.valid ? cu.st0 : 0;
    float f0 = 0.f, f1 = 0.f, f2 = 0.f, f3 = 0.f, fo = 0.f;
    long long racc = 0;          // RTL: the row's fixed-point accumulator
    unsigned int rfl = 0u;       // RTL: flags of the current unit
    unsigned int rflags = 0u;    // RTL: sticky flags of this lane's rows
    const int sw = lane & 7;
    // fast mode (the only one that splits row groups): a finished segment's
    // sums are stored at once; the fence and the group ticket follow one
    // stage later and the ticket's answer one more stage later, so neither
    // round trip stalls the stream.  The warp holding the group's last
    // ticket adds the segments in order.
    int pub = 0;                     // 0: none; 1: sums stored; 2: ticket requested
    int pub_d = 0, pub_g = 0;        // the pending segment's GEMV and row group
    unsigned int pub_raw = 0u;       // lane 0: the ticket's answer
    auto pub_ticket = [&]() {
        __threadfence();
        __syncwarp();
        if (lane == 0) pub_raw = atomicAdd(&sdesc[pub_d].tickets[pub_g], 1u);
        pub = 2;
    };
    auto pub_finish = [&]() {
        const SDesc& D = sdesc[pub_d];
        const unsigned int t = __shfl_sync(0xffffffffu, pub_raw, 0);
        pub = 0;
        if (t != (unsigned int)D.nseg - 1u) return;
        __threadfence();
        const int row = pub_g * kRows + lane;
        if (row < D.M) {
            float sum = 0.0f;
            // eight segment loads in flight at a time, added in segment order
            for (int s0 = 0; s0 < D.nseg; s0 += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; j++)
                    v[j] = s0 + j < D.nseg ? __ldcg(D.partial + (size_t)(s0 + j) * D.M + row) : 0.0f;
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (s0 + j < D.nseg) sum = __fadd_rn(sum, v[j]);
            }
            D.y[row] = sum;
            if (D.peer) store_peers(D.peer, row, sum);
        }
        if (lane == 0) D.tickets[pub_g] = 0u;
    };
    auto pub_flush = [&]() {
        if (pub == 1) pub_ticket();
        if (pub == 2) pub_finish();
    };
    int i = 0;
#pragma unroll 1
    while (cu.valid) {
        const int slot = i % kRing;
        mbar_wait(&bar[slot], (uint32_t)(i / kRing) & 1u, A.err);
        cp_async_wait<kRing - 2>();
        __syncwarp();
        issue((i + kRing - 1) % kRing, true);

        const bool odd_unit = !FAST && !RTL && (cu.M & 1) && (cu.r0 + kRows > cu.M - 1);   // holds the odd last row
        const bool odd = odd_unit && (cu.r0 + lane == cu.M - 1);
        const uint32_t ew = *reinterpret_cast<const uint32_t*>(ering + slot * 128 + lane * 4);
        const unsigned char* st = ring + slot * kStage + lane * 128;
        const uint4* xst = res ? reinterpret_cast<const uint4*>(xrings + cs * 512)
                               : reinterpret_cast<const uint4*>(xring + slot * kXp);
        const float* xsst = res ? reinterpret_cast<const float*>(xrings + (size_t)cu.K * 2) + cs * 4
                                : reinterpret_cast<const float*>(xring + slot * kXp + 512);
        if (RTL)
            stage_blocks_rtl(st, xst, xsst, ew, sw, racc, rfl);
        else if (FAST)
            stage_blocks<false, true>(st, xst, xsst, ew, sw, false, f0, f1, f2, f3, fo);
        else if (!odd_unit)
            stage_blocks<false, false>(st, xst, xsst, ew, sw, false, f0, f1, f2, f3, fo);
        else
            stage_blocks<true, false>(st, xst, xsst, ew, sw, odd, f0, f1, f2, f3, fo);
        if (FAST && !LM && pub) {
            if (pub == 2) pub_finish();
            else pub_ticket();
        }
        if (++cs == cu.st1) {
            float yv;
            if (RTL) {
                yv = __int_as_float(rtl_word(racc, rfl));
                if (cu.r0 + lane < cu.M) rflags |= rfl;   // lanes past M hold no row
                racc = 0;
                rfl = 0u;
            } else {
                yv = FAST ? f0 : (odd ? fo : add_ftz(add_ftz(f0, f2), add_ftz(f1, f3)));
            }
            if (FAST && !LM && sdesc[cu.d].nseg > 1) {
                pub_flush();
                const int row = cu.r0 + lane;
                if (row < cu.M) sdesc[cu.d].partial[(size_t)cu.s * cu.M + row] = yv;
                pub_d = cu.d;
                pub_g = cu.g;
                pub = 1;
            } else {
                unit_result<LM>(A, sdesc, cu, lane, yv, lm);
            }
            f0 = f1 = f2 = f3 = fo = 0.f;
            kc++;
            cu = load_unit(sdesc, nd, nu_total, (kc & 1) ? claimed1 : claimed0);
            cs = cu.valid ? cu.st0 : 0;
        }
        i++;
    }
    if (FAST && !LM) pub_flush();
    cp_async_wait<0>();
    if (RTL && A.rtl_flags) {
        const unsigned int f = __reduce_or_sync(0xffffffffu, rflags);
        if (lane == 0 && f) atomicOr(A.rtl_flags, f);
    }
    // row-sharded stacks: the last CTA publishes the epoch to every rank
    if (!LM) signal_peers(A.sync);
    if (LM) {
        __syncthreads();
        if (lm.wl) {
            cand[warp * 64 + lane] = lm.r0;
            cand[warp * 64 + 32 + lane] = lm.r1;
            merge_warp_lists64(cand, &s_cand_count, A.kk);
        }
        unsigned long long* work = reinterpret_cast<unsigned long long*>(rings);
        lm_finish(A.sc, cand, kCandCap, &s_cand_count, work, (kWarps * kRing * kStage) / 8, lm.best, A.kk, A.out_id,
                  A.out_ids, A.out_scores, A.out_n, s_red, lm.wl);
    }
}

// ---------------------------------------------------- single GEMV, split K
// A single exact GEMV whose activation fits shared memory (K <= 6144): one
// CTA per 32-row group, its 8 warps splitting the group's 256-byte K stages
// (warp w takes stages w, w + 8, w + 16), so every weight byte of the group
// is requested at once -- a short GEMV then costs about one memory round
// trip, not one per stage.  A warp turns each block's four lane-class sums
// into the operands of the reference's chain, (float(L_j) * 2^(e-134)) *
// xs (flushed multiplies; for the odd last row the scalar VFP term of the
// whole block dot), and keeps them in registers; when every warp is done they
// meet in shared memory over the drained stage buffers and warp 0 adds them
// lane by lane in block order -- the float order of the reference, bit for
// bit.  Weight and exponent loads go out before griddepcontrol.wait, so as a
// programmatic dependent launch the kernel streams its weights during the
// previous kernel's tail; it reads the activation and writes only after it.

// Split kernels with K <= kStageMaxK stage an rmsnorm's input in shared
// memory (4K bytes more); deeper ones read it from global memory.
constexpr int kStageMaxK = 4096;

static size_t split_smem_bytes(int K, bool stage) {
    const int nst = K >> 8, spw = (nst + kWarps - 1) / kWarps;
    return 1024 + (size_t)kWarps * spw * kStage + ((2 * (size_t)K + (size_t)K / 16 + 127) & ~size_t(127)) +
           (size_t)kWarps * spw * (128 + 8) + (stage ? 4 * (size_t)K : 0);
}

// SPW: the most stages one warp takes (K <= SPW * 2048); its terms stay in registers.
template <int SPW>
__global__ void __launch_bounds__(kThreads, SPW == 1 ? 2 : 1) gemv_split_kernel(const __grid_constant__ WArgs A) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                           ~uintptr_t(1023));
    // one unit per CTA: the CTAs past second_begin serve the second GEMV
    const bool sec = A.second_begin > 0 && (int)blockIdx.x >= A.second_begin;
    const GemvDesc& D = sec ? A.second : A.single;
    const int ubase = sec ? A.second_begin : 0;
    const int uend = A.second_begin > 0 && !sec ? A.second_begin : A.total_units;
    const int K = D.K, M = D.M, nb = K >> 6, nst = K >> 8;
    const int spw = (nst + kWarps - 1) / kWarps;
    unsigned char* rings = smem;                                                  // [warp][spw] stages
    unsigned char* xact = rings + (size_t)kWarps * spw * kStage;                  // resident activation
    unsigned char* erings = xact + ((2 * (size_t)K + (size_t)K / 16 + 127) & ~size_t(127));   // [warp][spw][lane]
    uint64_t* bars = reinterpret_cast<uint64_t*>(erings + (size_t)kWarps * spw * 128);         // [warp][spw]
    float* stage = (A.norm_w && K <= kStageMaxK) ? reinterpret_cast<float*>(bars + kWarps * spw) : nullptr;

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned char* ring = rings + (size_t)warp * spw * kStage;
    unsigned char* ering = erings + (size_t)warp * spw * 128;
    uint64_t* bar = bars + warp * spw;
    if (lane == 0) {
        for (int k = 0; k < spw; k++) mbar_init(&bar[k], 1);
        fence_barrier_init();
    }
    __syncwarp();
    const int sw = lane & 7;
    uint32_t phase = 0;
    bool first = true;
    for (int u = blockIdx.x; u < uend; u += gridDim.x, phase ^= 1u) {
        const int r0 = (u - ubase) * kRows;
        const bool row_ok = r0 + lane < M;
        // every stage of this warp's share goes out at once (weights are immutable)
#pragma unroll
        for (int k = 0; k < SPW; k++) {
            const int st = warp + k * kWarps;
            if (st >= nst) break;
            if (lane == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive_expect_tx(&bar[k], kStage);
                tma_load_2d(ring + k * kStage, &D.tmap, st * 256, r0, &bar[k]);
                tma_load_2d(ring + k * kStage + kBox, &D.tmap, st * 256 + 128, r0, &bar[k]);
            }
            if (row_ok) cp_async4(ering + k * 128 + lane * 4, D.exps + (size_t)(r0 + lane) * nb + st * 4);
        }
        cp_async_commit();
        if (first) {
            // the activation may be the previous kernel's output: read only now
            asm volatile("griddepcontrol.wait;" ::: "memory");
            quantize_resident(A, D, xact, warp, lane, stage);
            first = false;
        }
        cp_async_wait<0>();
        __syncwarp();
        const bool odd = (M & 1) && r0 + lane == M - 1;   // the odd last row: scalar VFP arithmetic
        float t[SPW][4][4];
#pragma unroll
        for (int k = 0; k < SPW; k++) {
            const int st = warp + k * kWarps;
            if (st >= nst) break;
            mbar_wait(&bar[k], phase, A.err);
            const uint32_t ew = *reinterpret_cast<const uint32_t*>(ering + k * 128 + lane * 4);
            const unsigned char* stp = ring + k * kStage + lane * 128;
            const uint4* xst = reinterpret_cast<const uint4*>(xact + st * 512);
            const float* xsst = reinterpret_cast<const float*>(xact + (size_t)K * 2) + st * 4;
#pragma unroll
            for (int jb = 0; jb < 4; jb++) {
                int L0, L1, L2, L3;
                lane_sums(stp, xst, sw, jb, L0, L1, L2, L3);
                const uint32_t e = (ew >> (8 * jb)) & 0xFFu;
                const float xsb = xsst[jb];
                if (!odd) {
                    const float S = exp_scale_ftz(e);
                    t[k][jb][0] = mul_ftz(mul_ftz(i2f_rn(L0), S), xsb);
                    t[k][jb][1] = mul_ftz(mul_ftz(i2f_rn(L1), S), xsb);
                    t[k][jb][2] = mul_ftz(mul_ftz(i2f_rn(L2), S), xsb);
                    t[k][jb][3] = mul_ftz(mul_ftz(i2f_rn(L3), S), xsb);
                } else {
                    t[k][jb][0] = mul_rn(mul_rn(i2f_rn(L0 + L1 + L2 + L3), exp_scale_ieee(e)), xsb);
                    t[k][jb][1] = t[k][jb][2] = t[k][jb][3] = 0.0f;
                }
            }
        }
        __syncthreads();   // every warp is done with the stage buffers
        float* T = reinterpret_cast<float*>(rings);   // [block][lane class][lane]
#pragma unroll
        for (int k = 0; k < SPW; k++) {
            const int st = warp + k * kWarps;
            if (st >= nst) break;
#pragma unroll
            for (int jb = 0; jb < 4; jb++)
#pragma unroll
                for (int j = 0; j < 4; j++) T[((st * 4 + jb) * 4 + j) * 32 + lane] = t[k][jb][j];
        }
        __syncthreads();
        if (warp == 0) {
            float f0 = 0.f, f1 = 0.f, f2 = 0.f, f3 = 0.f, fo = 0.f;
            if (!odd) {
                for (int b = 0; b < nb; b++) {
                    const float* tb = T + b * 128 + lane;
                    f0 = add_ftz(f0, tb[0]);
                    f1 = add_ftz(f1, tb[32]);
                    f2 = add_ftz(f2, tb[64]);
                    f3 = add_ftz(f3, tb[96]);
                }
            } else {
                for (int b = 0; b < nb; b++) fo = add_rn(fo, T[b * 128 + lane]);
            }
            if (row_ok) {
                const float v = odd ? fo : add_ftz(add_ftz(f0, f2), add_ftz(f1, f3));
                const int i = r0 + lane;
                // add_residual (qwen_kernels_opt.c:388-396) folded into the store
                D.y[i] = !A.res_epi ? v : (i < (M & ~3) ? add_ftz(D.y[i], v) : __fadd_rn(D.y[i], v));
            }
        }
        __syncthreads();   // the next unit's stages overwrite the terms
    }
}

// ---------------------------------------------------------------- generic
// Any K multiple of 64, any alignment: one thread per row, same arithmetic
// (RTL: the dequant datapath's words, sticky flags ORed into *rtl_flags).
template <bool RTL>
__global__ void __launch_bounds__(kThreads) gemv_generic_kernel(const __grid_constant__ GemvDesc D,
                                                                unsigned int* rtl_flags) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int nb = D.K >> 6;
    int16_t* xq = reinterpret_cast<int16_t*>(smem);
    float* xs = reinterpret_cast<float*>(smem + ((2 * D.K + 15) & ~15));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < nb; b += kThreads / 32) {
        int q0, q1;
        float s;
        if (D.x) {
            float v0 = D.x[64 * b + 2 * lane], v1 = D.x[64 * b + 2 * lane + 1];
            float a = fmaxf(fabsf(v0), fabsf(v1));
            for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
            if (a > 1e-20f) {
                float q = __fdiv_rn(16384.0f, a);
                s = __fdiv_rn(a, 16384.0f);
                q0 = __float2int_rn(__fmul_rn(v0, q));
                q1 = __float2int_rn(__fmul_rn(v1, q));
            } else {
                s = 0.0f;
                q0 = q1 = 0;
            }
        } else {
            q0 = D.xq[64 * b + 2 * lane];
            q1 = D.xq[64 * b + 2 * lane + 1];
            s = D.xs[b];
        }
        xq[64 * b + 2 * lane] = (int16_t)q0;
        xq[64 * b + 2 * lane + 1] = (int16_t)q1;
        if (lane == 0) xs[b] = s;
    }
    __syncthreads();
    const int m = blockIdx.x * kThreads + threadIdx.x;
    if (m >= D.M) return;
    const int8_t* w = D.mant + (size_t)m * D.K;
    const uint8_t* e = D.exps + (size_t)m * nb;
    const bool odd = (D.M & 1) && m == D.M - 1;
    float f0 = 0.f, f1 = 0.f, f2 = 0.f, f3 = 0.f, sum = 0.f;
    long long racc = 0;
    unsigned int rfl = 0u;
    for (int b = 0; b < nb; b++) {
        int L[4] = {0, 0, 0, 0};
        for (int i2 = 0; i2 < 64; i2++) L[i2 & 3] += (int)w[64 * b + i2] * (int)xq[64 * b + i2];
        const uint32_t eb = e[b];
        if (RTL) {
            rtl_block(racc, rfl, (L[0] + L[1]) + (L[2] + L[3]), __float_as_uint(xs[b]), eb);
        } else if (odd) {
            float t = mul_rn(mul_rn(i2f_rn(L[0] + L[1] + L[2] + L[3]), exp_scale_ieee(eb)), xs[b]);
            sum = add_rn(sum, t);
        } else {
            const float S = exp_scale_ftz(eb);
            f0 = add_ftz(f0, mul_ftz(mul_ftz(i2f_rn(L[0]), S), xs[b]));
            f1 = add_ftz(f1, mul_ftz(mul_ftz(i2f_rn(L[1]), S), xs[b]));
            f2 = add_ftz(f2, mul_ftz(mul_ftz(i2f_rn(L[2]), S), xs[b]));
            f3 = add_ftz(f3, mul_ftz(mul_ftz(i2f_rn(L[3]), S), xs[b]));
        }
    }
    if (RTL) {
        D.y[m] = __int_as_float(rtl_word(racc, rfl));
        if (rfl && rtl_flags) atomicOr(rtl_flags, rfl);
        return;
    }
    D.y[m] = odd ? sum : add_ftz(add_ftz(f0, f2), add_ftz(f1, f3));
}

// ---------------------------------------------------------------- residual
// add_residual (qwen_kernels_opt.c:388-396), NEON build: x += res with the
// vector unit's flushed adds over whole groups of four, the scalar (IEEE)
// add on the tail.
__global__ void __launch_bounds__(kThreads) add_residual_kernel(float* x, const float* res, int n) {
    const int body = n & ~3;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        x[i] = i < body ? add_ftz(x[i], res[i]) : add_rn(x[i], res[i]);
}

cudaError_t launch_add_residual(float* x, const float* res, int n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    add_residual_kernel<<<std::min((n + kThreads - 1) / kThreads, num_sms()), kThreads, 0, stream>>>(x, res, n);
    return cudaGetLastError();
}

// ---------------------------------------------------------------- quantizer
__global__ void __launch_bounds__(kThreads) quant_block64_kernel(const float* x, int B, int K,
                                                                 int16_t* xq, float* xs) {
    const int nb = K >> 6;
    const long long total = (long long)B * nb;
    const int lane = threadIdx.x & 31;
    for (long long blk = (long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); blk < total;
         blk += (long long)gridDim.x * (kThreads / 32)) {
        const float* xb = x + blk * 64;
        float v0 = xb[2 * lane], v1 = xb[2 * lane + 1];
        float a = fmaxf(fabsf(v0), fabsf(v1));
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        int q0 = 0, q1 = 0;
        float s = 0.0f;
        if (a > 1e-20f) {
            float q = __fdiv_rn(16384.0f, a);
            s = __fdiv_rn(a, 16384.0f);
            q0 = __float2int_rn(__fmul_rn(v0, q));
            q1 = __float2int_rn(__fmul_rn(v1, q));
        }
        xq[blk * 64 + 2 * lane] = (int16_t)q0;
        xq[blk * 64 + 2 * lane + 1] = (int16_t)q1;
        if (lane == 0) xs[blk] = s;
    }
}

// ------------------------------------------------------- shard-local SwiGLU
// The MLP activation of a row-sharded layer: this rank holds elements
// [col0, col0 + n) of the gate and up projections of every batch row; it
// applies swiglu (the reference's NEON build, as in the fused down
// projection), quantizes each 64-block by the reference rule -- blocks lie
// wholly inside one rank's slice, so the bits are those of the unsharded
// activation -- and stores the quantized slice into its own copy of the
// down projection's input and into every other rank's, so only int16 values
// and block scales cross NVLink.  With a signal epoch, the last CTA then
// publishes it to every rank and waits (bounded) until every rank has
// published it: the down projection launched after this kernel reads a
// complete input.
struct SqArgs {
    const float* gate;
    const float* up;
    int B, n, ld_in, col0, K, ldxs, planar, ndst;
    unsigned char* dst[kMaxRanks];   // dst[0] this GPU's input, then the other ranks'
    SyncArgs sync;
    unsigned int* err;
};

__global__ void __launch_bounds__(256) swiglu_quant_kernel(const __grid_constant__ SqArgs A) {
    // a programmatic dependent of the gate / up GEMV: its outputs are read
    // once that grid has completed; the next launch may start its prologue
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int nbl = A.n >> 6;
    const long long total = (long long)A.B * nbl;
    for (long long t = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); t < total; t += (long long)gridDim.x * 8) {
        const int b = (int)(t / nbl), j = (int)(t - (long long)b * nbl);
        const size_t src = (size_t)b * A.ld_in + (size_t)j * 64;
        const float2 g = reinterpret_cast<const float2*>(A.gate + src)[lane];
        const float2 u = reinterpret_cast<const float2*>(A.up + src)[lane];
        const float2 v = make_float2(swiglu_lane(g.x, u.x), swiglu_lane(g.y, u.y));
        int q0, q1;
        float xs;
        block_quant(v, q0, q1, xs);
        const int col = A.col0 + 64 * j + 2 * lane, kb = (A.col0 >> 6) + j;
        if (!A.planar) {   // quantized record: xq int16 [K], then xs fp32 [K/64]
            const uint32_t w = ((uint32_t)q0 & 0xFFFFu) | ((uint32_t)q1 << 16);
            for (int d = 0; d < A.ndst; d++) {
                reinterpret_cast<uint32_t*>(A.dst[d])[col >> 1] = w;
                if (lane == 0) reinterpret_cast<float*>(A.dst[d] + 2 * (size_t)A.K)[kb] = xs;
            }
        } else {           // planes [2][B][K] (xq = 256 * hi + lo), then xs_t [K/64][ldxs]
            const int l0 = (int)(int8_t)(q0 & 0xFF), l1 = (int)(int8_t)(q1 & 0xFF);
            const uint16_t hi =
                (uint16_t)(((uint32_t)((q0 - l0) >> 8) & 0xFFu) | (((uint32_t)((q1 - l1) >> 8) & 0xFFu) << 8));
            const uint16_t lo = (uint16_t)(((uint32_t)q0 & 0xFFu) | (((uint32_t)q1 & 0xFFu) << 8));
            const size_t off = (size_t)b * A.K + col, plane = (size_t)A.B * A.K;
            for (int d = 0; d < A.ndst; d++) {
                *reinterpret_cast<uint16_t*>(A.dst[d] + off) = hi;
                *reinterpret_cast<uint16_t*>(A.dst[d] + plane + off) = lo;
                if (lane == 0) reinterpret_cast<float*>(A.dst[d] + 2 * plane)[(size_t)kb * A.ldxs + b] = xs;
            }
        }
    }
    if (!A.sync.sig_epoch) return;
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned int tk = atomicAdd(A.sync.sig_ticket, 1u);
        s_last = tk == gridDim.x - 1;
        if (s_last) {
            __threadfence_system();
            const unsigned int e = epoch_of(A.sync.sig_epoch, A.sync.epoch_base);
            for (int r = 0; r < A.sync.world; r++) st_relaxed_sys(A.sync.sig_flags[r] + A.sync.rank, e);
            *A.sync.sig_ticket = 0u;   // the next launch using this ticket is stream-ordered after this one
        }
    }
    __syncthreads();
    if (s_last) wait_peer_flags(A.sync.wait_flags, A.sync.world, A.sync.sig_epoch, A.sync.epoch_base, A.err);
}

__global__ void epoch_advance_kernel(unsigned int* base, unsigned int n) { *base += n; }

// ---------------------------------------------------------------- host side
cudaError_t launch_epoch_advance(unsigned int* base, unsigned int n, cudaStream_t stream) {
    if (!base || (reinterpret_cast<uintptr_t>(base) & 3)) return cudaErrorInvalidValue;
    epoch_advance_kernel<<<1, 1, 0, stream>>>(base, n);
    return cudaGetLastError();
}

cudaError_t launch_swiglu_quant(const float* gate, const float* up, int B, int n, int ld_in, int col0, int K,
                                int planar, int ldxs, void* const* dst, int ndst, const SyncArgs* sync,
                                unsigned int* err, cudaStream_t stream) {
    if (!gate || !up || !dst || B < 1 || n < 0 || n % 64 || col0 < 0 || col0 % 64 || K % 64 || col0 + n > K ||
        ndst < 1 || ndst > kMaxRanks || (B > 1 && !planar) || ld_in < n || (ld_in & 1) ||
        (planar && ldxs < B) || (reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up)) & 7)
        return cudaErrorInvalidValue;
    if (sync && (!sync_args_ok(*sync) || (sync->sig_epoch && !sync->wait_flags))) return cudaErrorInvalidValue;
    SqArgs A{};
    A.gate = gate;
    A.up = up;
    A.B = B;
    A.n = n;
    A.ld_in = ld_in;
    A.col0 = col0;
    A.K = K;
    A.ldxs = ldxs;
    A.planar = planar;
    A.ndst = ndst;
    for (int d = 0; d < ndst; d++) {
        if (!dst[d] || reinterpret_cast<uintptr_t>(dst[d]) & 15) return cudaErrorInvalidValue;
        A.dst[d] = static_cast<unsigned char*>(dst[d]);
    }
    if (sync) A.sync = *sync;
    A.err = err;
    const long long total = (long long)B * (n / 64);
    const int grid = (int)std::max<long long>(1, std::min<long long>((total + 7) / 8, (long long)num_sms() * 8));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, swiglu_quant_kernel, A);
}

int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

static size_t warp_smem_bytes(bool lm, int n) {
    return 1024 + (size_t)kWarps * kRing * (kStage + kXp + 128) + (size_t)kWarps * kRing * 8 +
           (size_t)n * sizeof(SDesc) + (lm ? (size_t)kCandCap * 8 : 0);
}

static bool fast_shape_ok(const GemvDesc& d) {
    if (d.M <= 0 || d.K <= 0 || d.K % 512) return false;
    if (reinterpret_cast<uintptr_t>(d.mant) % 16 || reinterpret_cast<uintptr_t>(d.exps) % 4) return false;
    if (d.x ? (reinterpret_cast<uintptr_t>(d.x) % 8) : (reinterpret_cast<uintptr_t>(d.xq) % 4)) return false;
    return true;
}

bool gemv_plan(GemvDesc* descs, int n, uint32_t* act, GemvPlan* plan, int mode, size_t act_cap_words,
               unsigned int* tickets, size_t tickets_cap, int fixed_seg_stages) {
    if (n <= 0 || n > kMaxSDesc) return false;
    const bool fast = mode == kFast;
    // largest K first: the counter then hands out the biggest units first
    std::vector<int> order(n);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return descs[a].K > descs[b].K; });
    std::vector<GemvDesc> sorted;
    sorted.reserve(n);
    for (int i : order) sorted.push_back(descs[i]);
    // fast mode: split row groups into K segments so that every GEMV gets
    // about its byte share of 2 units per warp slot
    const double slots = 2.0 * num_sms() * kWarps;
    double total_bytes = 0;
    for (const GemvDesc& d : sorted) total_bytes += (double)d.M * d.K;
    size_t pair_words = 0, part_words = 0, ticket_words = 0;
    for (GemvDesc& d : sorted) {
        const int groups = (d.M + kRows - 1) / kRows, nst = d.K >> 8;
        int nseg = 1;
        if (fast && fixed_seg_stages > 0) {
            // segments of a fixed length: where a row's K is cut depends on K
            // alone, not on how many rows this GPU holds, so a row-sharded
            // plan gives every row the bits of the unsharded plan
            nseg = std::max(1, (nst + fixed_seg_stages - 1) / fixed_seg_stages);
        } else if (fast) {
            // segments of >= 2 stages: the per-warp claim ring assumes its
            // producer never runs more than one unit ahead
            nseg = (int)std::ceil(slots * ((double)d.M * d.K / total_bytes) / groups);
            nseg = std::max(1, std::min(nseg, nst / 2));
        }
        d.seg_stages = (nst + nseg - 1) / nseg;
        d.nseg = (nst + d.seg_stages - 1) / d.seg_stages;
        // every segment, the last one included, has >= 2 stages: the kernel
        // issues a unit's first stage before it claims the next unit
        while (d.nseg > 1 && nst - (d.nseg - 1) * d.seg_stages < 2) {
            d.seg_stages++;
            d.nseg = (nst + d.seg_stages - 1) / d.seg_stages;
        }
        pair_words += (gemv_act_words(d.K) + 3) & ~size_t(3);
        if (d.nseg > 1) {
            part_words += (size_t)d.nseg * d.M;
            ticket_words += (size_t)groups;
        }
    }
    if (tickets) {   // counters live in the caller's separate zeroed buffer
        if (ticket_words > tickets_cap) part_words = ticket_words = (size_t)-1 / 4;
        else ticket_words = 0;
    }
    if (act_cap_words && pair_words + part_words + ticket_words > act_cap_words) {
        // not enough scratch for the segment sums: whole rows
        part_words = ticket_words = 0;
        for (GemvDesc& d : sorted) {
            d.nseg = 1;
            d.seg_stages = d.K >> 8;
        }
    }
    int units = 0, kmax = 0;
    size_t words = 0, pw = pair_words, tw = pair_words + part_words;
    for (int i = 0; i < n; i++) {
        GemvDesc& d = sorted[i];
        if (!fast_shape_ok(d)) return false;
        if (!encode_tmap_2d(&d.tmap, d.mant, 1, (uint64_t)d.M, (uint64_t)d.K, (uint32_t)kRows)) return false;
        d.unit_begin = units;
        d.xpairs = act ? act + words : nullptr;
        d.xscale = act ? reinterpret_cast<float*>(act + words + d.K / 2) : nullptr;
        words += (gemv_act_words(d.K) + 3) & ~size_t(3);   // keep every pair block 16-byte aligned
        const int groups = (d.M + kRows - 1) / kRows;
        d.partial = nullptr;
        d.tickets = nullptr;
        if (d.nseg > 1) {
            d.partial = act ? reinterpret_cast<float*>(act + pw) : nullptr;
            d.tickets = tickets ? tickets + (tw - pair_words - part_words) : (act ? act + tw : nullptr);
            pw += (size_t)d.nseg * d.M;
            tw += (size_t)groups;
        }
        units += groups * d.nseg;
        kmax = std::max(kmax, d.K);
    }
    for (int i = 0; i < n; i++) descs[i] = sorted[i];
    plan->n = n;
    plan->total_units = units;
    plan->kmax = kmax;
    plan->fast = fast;
    plan->act_words = pair_words + part_words + ticket_words;
    return true;
}

// A single GEMV whose whole paired activation (2K bytes + K/16 scale bytes)
// fits the activation-ring space quantizes it in every CTA (res_act).
static bool res_fits(int K) { return 2 * (size_t)K + (size_t)K / 16 <= (size_t)kWarps * kRing * kXp; }

// pdl: launch as a programmatic dependent of the stream's previous kernel
// (the kernel waits for that grid before it reads or writes memory).
static cudaError_t launch_prep(const PrepArgs& P, int kmax, cudaStream_t stream, bool pdl = false) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P.n, (kmax / 64 + kPrepChunk - 1) / kPrepChunk);
    cfg.blockDim = dim3(kPrepThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, act_prep_kernel, P);
}

template <bool LM, bool FAST, bool RTL = false>
static cudaError_t launch_warp(const WArgs& A, int grid, cudaStream_t stream) {
    const size_t smem = warp_smem_bytes(LM, A.n);
    cudaError_t err = raise_smem_limit(reinterpret_cast<const void*>(gemv_warp_kernel<LM, FAST, RTL>), smem);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;   // a programmatic dependent of act_prep, or (resident activation) of whatever ran before
    return cudaLaunchKernelEx(&cfg, gemv_warp_kernel<LM, FAST, RTL>, A);
}

cudaError_t launch_gemv_list(const GemvDesc* dev_descs, const GemvPlan& plan, unsigned int* ctr,
                             unsigned int* err, cudaStream_t stream, const SyncArgs* sync) {
    if (plan.n <= 0 || plan.total_units <= 0) return cudaSuccess;
    if (sync && !sync_args_ok(*sync)) return cudaErrorInvalidValue;
    PrepArgs P{};
    P.list = dev_descs;
    P.n = plan.n;
    P.err = err;
    if (sync) {
        P.wait_flags = sync->wait_flags;
        P.wait_epoch = sync->wait_epoch;
        P.epoch_base = sync->epoch_base;
        P.world = sync->world;
    }
    // back-to-back steps overlap: this step's GEMV CTAs start (descriptor
    // table, first weight stages) while the previous kernel's last CTAs
    // finish (act_prep waits for that kernel before it reads, writes or
    // polls peer flags)
    cudaError_t e = launch_prep(P, plan.kmax, stream, true);
    if (e != cudaSuccess) return e;
    WArgs A{};
    A.list = dev_descs;
    A.n = plan.n;
    A.total_units = plan.total_units;
    A.ctr = ctr;
    A.err = err;
    if (sync) A.sync = *sync;
    const int grid = std::min(num_sms(), (plan.total_units + kWarps - 1) / kWarps);
    return plan.fast ? launch_warp<false, true>(A, grid, stream) : launch_warp<false, false>(A, grid, stream);
}

cudaError_t launch_gemv_fast(const GemvDesc& d0, uint32_t* act, size_t act_cap_words, unsigned int* tickets,
                             size_t tickets_cap, unsigned int* err, cudaStream_t stream) {
    if (d0.M <= 0) return cudaSuccess;
    GemvDesc d = d0;
    GemvPlan plan;
    if (!act || !tickets || !gemv_plan(&d, 1, act, &plan, kFast, act_cap_words, tickets, tickets_cap))
        return cudaErrorInvalidValue;
    const bool res = res_fits(d.K);
    if (!res) {
        PrepArgs P{};
        P.single = d;
        P.n = 1;
        cudaError_t e = launch_prep(P, d.K, stream);
        if (e != cudaSuccess) return e;
    }
    WArgs A{};
    A.res_act = res ? 1 : 0;
    A.single = d;
    A.n = 1;
    A.total_units = plan.total_units;
    A.ctr = nullptr;
    A.err = err;
    const int grid = std::min(num_sms(), (plan.total_units + kWarps - 1) / kWarps);
    return launch_warp<false, true>(A, grid, stream);
}

// One exact single GEMV (K <= 6144, K % 512 == 0) on the split-K kernel, a
// programmatic dependent of the stream's previous kernel.
static cudaError_t launch_split(const WArgs& A, cudaStream_t stream) {
    const size_t smem = split_smem_bytes(A.single.K, A.norm_w && A.single.K <= kStageMaxK);
    const int spw = ((A.single.K >> 8) + kWarps - 1) / kWarps;
    auto kern = spw <= 1 ? gemv_split_kernel<1> : spw == 2 ? gemv_split_kernel<2> : gemv_split_kernel<3>;
    cudaError_t err = raise_smem_limit(reinterpret_cast<const void*>(kern), smem);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(A.total_units);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, A);
}

template <bool RTL>
static cudaError_t launch_generic(const GemvDesc& d, unsigned int* rtl_flags, cudaStream_t stream) {
    const size_t smem = (((size_t)2 * d.K + 15) & ~size_t(15)) + 4 * (size_t)(d.K / 64);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(gemv_generic_kernel<RTL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    gemv_generic_kernel<RTL><<<(d.M + kThreads - 1) / kThreads, kThreads, smem, stream>>>(d, rtl_flags);
    return cudaGetLastError();
}

cudaError_t launch_gemv(const GemvDesc& d0, uint32_t* act, unsigned int* err, cudaStream_t stream, int mode,
                        unsigned int* rtl_flags) {
    if (d0.M <= 0) return cudaSuccess;
    if (d0.K <= 0 || d0.K % 64 || (mode != kExact && mode != kRtl20)) return cudaErrorInvalidValue;
    const bool rtl = mode == kRtl20;
    GemvDesc d = d0;
    GemvPlan plan;
    if (!fast_shape_ok(d) || !act || !gemv_plan(&d, 1, act, &plan))
        return rtl ? launch_generic<true>(d, rtl_flags, stream) : launch_generic<false>(d, nullptr, stream);
    const bool res = res_fits(d.K);
    if (!res) {
        PrepArgs P{};
        P.single = d;
        P.n = 1;
        cudaError_t e = launch_prep(P, d.K, stream);
        if (e != cudaSuccess) return e;
    }
    WArgs A{};
    A.res_act = res ? 1 : 0;
    A.single = d;
    A.n = 1;
    A.total_units = plan.total_units;
    A.ctr = nullptr;
    A.err = err;
    A.rtl_flags = rtl_flags;
    if (res && !rtl) return launch_split(A, stream);
    const int grid = std::min(num_sms(), (plan.total_units + kWarps - 1) / kWarps);
    return rtl ? launch_warp<false, false, true>(A, grid, stream) : launch_warp<false, false>(A, grid, stream);
}

cudaError_t launch_rmsnorm_gemv(const GemvDesc& d0, const float* norm_w, float eps, uint32_t* act, unsigned int* err,
                               cudaStream_t stream, const float* res, float* x_out) {
    if (d0.M <= 0) return cudaSuccess;
    GemvDesc d = d0;
    GemvPlan plan;
    if (!d.x || !norm_w || (reinterpret_cast<uintptr_t>(norm_w) & 7) || !res_fits(d.K) || !fast_shape_ok(d) ||
        !act || !gemv_plan(&d, 1, act, &plan))
        return cudaErrorInvalidValue;
    if ((res == nullptr) != (x_out == nullptr)) return cudaErrorInvalidValue;
    if (res) {
        // x_out is written while every CTA still reads x and res: no overlap
        const uintptr_t o0 = reinterpret_cast<uintptr_t>(x_out), o1 = o0 + 4 * (size_t)d.K;
        auto overlaps = [&](const float* p) {
            const uintptr_t p0 = reinterpret_cast<uintptr_t>(p), p1 = p0 + 4 * (size_t)d.K;
            return p0 < o1 && o0 < p1;
        };
        if (((reinterpret_cast<uintptr_t>(res) | o0) & 7) || overlaps(d.x) || overlaps(res))
            return cudaErrorInvalidValue;
    }
    WArgs A{};
    A.res_act = 1;
    A.norm_w = norm_w;
    A.norm_eps = eps;
    A.norm_res = res;
    A.norm_xout = x_out;
    A.single = d;
    A.n = 1;
    A.total_units = plan.total_units;
    A.ctr = nullptr;
    A.err = err;
    return launch_split(A, stream);
}

cudaError_t launch_rmsnorm_gemv2(const GemvDesc& d0, const GemvDesc& d1, const float* norm_w, float eps,
                                uint32_t* act, unsigned int* err, cudaStream_t stream, const float* res,
                                float* x_out, float* norm_out) {
    if (d0.M <= 0 || d1.M <= 0 || d0.K != d1.K || d0.x != d1.x) return cudaErrorInvalidValue;
    GemvDesc e1 = d1;
    GemvPlan p1;
    if (!fast_shape_ok(e1) || !act || !gemv_plan(&e1, 1, act, &p1)) return cudaErrorInvalidValue;
    // the first GEMV's checks and plan, then the second's units appended
    GemvDesc e0 = d0;
    GemvPlan p0;
    if (!e0.x || !norm_w || (reinterpret_cast<uintptr_t>(norm_w) & 7) || !res_fits(e0.K) || !fast_shape_ok(e0) ||
        !gemv_plan(&e0, 1, act, &p0))
        return cudaErrorInvalidValue;
    if ((res == nullptr) != (x_out == nullptr)) return cudaErrorInvalidValue;
    if (res) {
        const uintptr_t o0 = reinterpret_cast<uintptr_t>(x_out), o1 = o0 + 4 * (size_t)e0.K;
        auto overlaps = [&](const float* p) {
            const uintptr_t q0 = reinterpret_cast<uintptr_t>(p), q1 = q0 + 4 * (size_t)e0.K;
            return q0 < o1 && o0 < q1;
        };
        if (((reinterpret_cast<uintptr_t>(res) | o0) & 7) || overlaps(e0.x) || overlaps(res))
            return cudaErrorInvalidValue;
    }
    WArgs A{};
    A.res_act = 1;
    A.norm_w = norm_w;
    A.norm_eps = eps;
    A.norm_res = res;
    A.norm_xout = x_out;
    A.norm_out = norm_out;
    A.single = e0;
    A.n = 1;
    A.second = e1;
    A.second_begin = p0.total_units;
    A.total_units = p0.total_units + p1.total_units;
    A.ctr = nullptr;
    A.err = err;
    return launch_split(A, stream);
}

cudaError_t launch_swiglu_gemv(const GemvDesc& d0, const float* up, uint32_t* act, unsigned int* err,
                               cudaStream_t stream, bool residual) {
    if (d0.M <= 0) return cudaSuccess;
    GemvDesc d = d0;
    GemvPlan plan;
    if (!d.x || !up || (reinterpret_cast<uintptr_t>(up) & 7) || !res_fits(d.K) || !fast_shape_ok(d) || !act ||
        !gemv_plan(&d, 1, act, &plan))
        return cudaErrorInvalidValue;
    WArgs A{};
    A.res_act = 1;
    A.res_epi = residual ? 1 : 0;
    A.glu_up = up;
    A.single = d;
    A.n = 1;
    A.total_units = plan.total_units;
    A.ctr = nullptr;
    A.err = err;
    return launch_split(A, stream);
}

cudaError_t launch_bfp8_lm_head(const float* h, const int8_t* mant, const uint8_t* exps, int vocab,
                                int hidden, int k, LmScratch* scratch, uint32_t* act, unsigned int* ctr,
                                unsigned int* err, int* out_id, int* out_ids, float* out_scores, int* out_n,
                                cudaStream_t stream) {
    GemvDesc d{};
    d.mant = mant;
    d.exps = exps;
    d.x = h;
    d.M = vocab;
    d.K = hidden;
    if (vocab <= 0 || hidden <= 0 || k < 0 || std::min(k, vocab) > kTopkMax || !act) return cudaErrorInvalidValue;
    GemvPlan plan;
    if (!fast_shape_ok(d) || !gemv_plan(&d, 1, act, &plan)) return cudaErrorInvalidValue;
    const int grid = std::min(std::min(num_sms(), (plan.total_units + kWarps - 1) / kWarps), kMaxGrid);
    const int kk = std::min(k, vocab);
    // Every scored row is appended to the CTA's shared buffer and the CTA
    // selects its top-k once at its end; when its rows do not fit the buffer,
    // k <= 64 keeps running per-warp top-64 lists in registers instead (a
    // bitonic fold per unit, which stalls that warp's weight stream).
    const long long rows_per_cta =
        (long long)((plan.total_units + grid * kWarps - 1) / (grid * kWarps)) * kWarps * kRows;
    const bool warp_lists = rows_per_cta > kCandCap;
    if (warp_lists && kk > 64) return cudaErrorInvalidValue;
    const bool res = res_fits(d.K);
    if (!res) {
        PrepArgs P{};
        P.single = d;
        P.n = 1;
        cudaError_t e = launch_prep(P, d.K, stream);
        if (e != cudaSuccess) return e;
    }
    WArgs A{};
    A.res_act = res ? 1 : 0;
    A.single = d;
    A.n = 1;
    A.total_units = plan.total_units;
    A.ctr = nullptr;   // round-robin: with ~2 units per warp a claim round trip costs more than it balances
    (void)ctr;
    A.err = err;
    A.sc = scratch;
    A.kk = kk;
    A.out_id = out_id;
    A.out_ids = out_ids;
    A.out_scores = out_scores;
    A.out_n = out_n;
    A.lm_warp_lists = warp_lists ? 1 : 0;
    return launch_warp<true, false>(A, grid, stream);
}

cudaError_t launch_quant_block64(const float* x, int B, int K, int16_t* xq, float* xs,
                                 cudaStream_t stream) {
    if (B <= 0) return cudaSuccess;
    if (K <= 0 || K % 64) return cudaErrorInvalidValue;
    const long long blocks = (long long)B * (K / 64);
    const int grid = (int)std::min<long long>((blocks + 7) / 8, (long long)num_sms() * 8);
    quant_block64_kernel<<<grid, kThreads, 0, stream>>>(x, B, K, xq, xs);
    return cudaGetLastError();
}

}  // namespace qb
