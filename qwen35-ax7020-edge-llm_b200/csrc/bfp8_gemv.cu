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
// Kernel shape.  A work unit is RG consecutive rows of one GEMV; a CTA owns a
// contiguous run of units (balanced by bytes across all GEMVs of a grouped
// launch) and streams each unit through a P-stage cp.async ring in 16 KB
// slices of RG rows x (16384/RG) bytes.  Inside a slice, lane = row and warp
// = 64-byte block: a thread forms the four lane-class sums of one (row, block)
// with __dp2a (int16 activation pairs (k, k+4) against weight bytes paired by
// prmt), turns them into the four fp32 block terms and stores them; the
// per-row float chains then run sequentially over blocks in 4*RG "chain"
// threads (row, lane class), one slice behind.  Weight tiles are laid out in
// shared memory as 128-byte rows with the 16-byte chunk index XORed by
// (row & 7), the TMA SWIZZLE_128B pattern, so the per-row reads of a warp are
// bank-conflict free.
#include "bfp8_gemv.cuh"
#include "common.cuh"
#include "tma.cuh"
#include "topk.cuh"

#include <algorithm>

namespace qb {

constexpr int kThreads = 256;
constexpr int kStageMant = 16384;   // mantissa bytes per stage (TMA boxes)
constexpr int kStages = 5;          // ring depth; two CTAs fit one SM for K <= 4096

template <int RG>
struct Geo {
    static constexpr int SB = 256 / RG;          // 64-byte blocks per slice row
    static constexpr int RS = 64 * SB;           // bytes per slice row
    static constexpr int BOXES = RS / 128;       // TMA boxes (RG rows x 128 B) per slice
    static constexpr int EXB = RG * SB;          // exponent bytes per stage (256)
};

struct GemvArgs {
    GemvDesc single;
    const GemvDesc* list;   // nullptr -> `single`
    int n;
    int total_units;
    long long total_cost;
    int kmax;
    unsigned int* err;
    // lm_head epilogue
    LmScratch* sc;
    int kk;
    int* out_id;
    int* out_ids;
    float* out_scores;
    int* out_n;
};

__device__ __forceinline__ const GemvDesc& desc_ref(const GemvArgs& A, int d) {
    return A.list ? A.list[d] : A.single;
}

template <int RG>
struct Cursor {
    int d, u, s, ns, M, K, nb, ub, ue;
    const uint8_t* exps;
    bool valid;

    __device__ void set_desc(const GemvArgs& A, int dd) {
        const GemvDesc& D = desc_ref(A, dd);
        d = dd;
        M = D.M;
        K = D.K;
        nb = K >> 6;
        ns = (nb + Geo<RG>::SB - 1) / Geo<RG>::SB;
        ub = D.unit_begin;
        ue = D.unit_begin + (M + RG - 1) / RG;
        exps = D.exps;
    }
    __device__ void advance(const GemvArgs& A, int u_end) {
        if (++s < ns) return;
        s = 0;
        if (++u >= u_end) {
            valid = false;
            return;
        }
        while (u >= ue) set_desc(A, d + 1);
    }
};

// First unit whose cost start is >= pos (units ordered GEMV by GEMV).
template <int RG>
__device__ int unit_at_cost(const GemvArgs& A, long long pos, int* d_out) {
    if (pos >= A.total_cost) {
        *d_out = A.n;
        return A.total_units;
    }
    int lo = 0, hi = A.n - 1;
    while (lo < hi) {  // largest d with cost_begin <= pos
        int mid = (lo + hi + 1) >> 1;
        if (desc_ref(A, mid).cost_begin <= pos) lo = mid;
        else hi = mid - 1;
    }
    const GemvDesc& D = desc_ref(A, lo);
    int ns = ((D.K >> 6) + Geo<RG>::SB - 1) / Geo<RG>::SB;
    int units = (D.M + RG - 1) / RG;
    long long off = pos - D.cost_begin;
    long long uo = (off + ns - 1) / ns;
    if (uo >= units) {
        *d_out = lo + 1;
        return D.unit_begin + units;
    }
    *d_out = lo;
    return D.unit_begin + (int)uo;
}

// Quantize (or load) one activation into the paired shared layout:
// block b, group g (elements 8g..8g+7), word j holds the int16 pair
// (xq[64b+8g+j], xq[64b+8g+4+j]) -- the operand order of __dp2a below.
__device__ void stage_activation(const GemvDesc& D, uint32_t* xp, float* xss) {
    const int nb = D.K >> 6;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < nb; b += kThreads / 32) {
        int q0, q1;
        float xs;
        if (D.x) {
            float2 v = reinterpret_cast<const float2*>(D.x + 64 * b)[lane];
            float a = fmaxf(fabsf(v.x), fabsf(v.y));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
            if (a > 1e-20f) {
                float q = __fdiv_rn(16384.0f, a);
                xs = __fdiv_rn(a, 16384.0f);
                q0 = __float2int_rn(__fmul_rn(v.x, q));
                q1 = __float2int_rn(__fmul_rn(v.y, q));
            } else {
                xs = 0.0f;
                q0 = q1 = 0;
            }
        } else {
            short2 v = reinterpret_cast<const short2*>(D.xq + 64 * b)[lane];
            q0 = v.x;
            q1 = v.y;
            xs = D.xs[b];
        }
        uint32_t mine = ((uint32_t)q0 & 0xFFFFu) | ((uint32_t)q1 << 16);
        uint32_t part = __shfl_down_sync(0xffffffffu, mine, 2);
        if ((lane & 3) < 2) {
            int g = lane >> 2, p = 2 * (lane & 3);
            uint32_t w0 = (mine & 0xFFFFu) | (part << 16);
            uint32_t w1 = (mine >> 16) | (part & 0xFFFF0000u);
            *reinterpret_cast<uint2*>(xp + b * 32 + g * 4 + p) = make_uint2(w0, w1);
        }
        if (lane == 0) xss[b] = xs;
    }
}

// Start one slice: thread 0 arms the stage barrier and issues the TMA boxes
// of the mantissa tile; warp 1 copies the slice's exponent bytes (8-byte
// pieces, cp.async, one commit group per slice issued by every thread).
template <int RG>
__device__ __forceinline__ void issue_slice(const GemvArgs& A, const Cursor<RG>& c, unsigned char* mant_st,
                                            unsigned char* exps_st, uint64_t* bar) {
    using G = Geo<RG>;
    const int r0 = (c.u - c.ub) * RG;
    const int b0 = c.s * G::SB;
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(bar, kStageMant);
        const void* tm = &desc_ref(A, c.d).tmap;
#pragma unroll
        for (int j = 0; j < G::BOXES; j++) tma_load_2d(mant_st + j * (RG * 128), tm, b0 * 64 + j * 128, r0, bar);
    } else if ((threadIdx.x >> 5) == 1) {
        const int lane = threadIdx.x & 31;
        const int rv = min(RG, c.M - r0);
        const int vb = min(G::SB, c.nb - b0);
        const int ppr = vb >> 3;
        const uint8_t* esrc = c.exps + (size_t)r0 * c.nb + b0;
        for (int idx = lane; idx < rv * ppr; idx += 32) {
            int r = idx / ppr, p = idx - r * ppr;
            cp_async8(exps_st + r * G::SB + p * 8, esrc + (size_t)r * c.nb + p * 8);
        }
    }
}

// Block terms of one slice: thread (row r = lane % RG, block bs) -> tb[bs][r][0..3].
template <int RG>
__device__ __forceinline__ void compute_slice(const Cursor<RG>& c, const unsigned char* mant_st,
                                              const unsigned char* exps_st, float* tb, const uint32_t* xp,
                                              const float* xss) {
    using G = Geo<RG>;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = lane % RG;
    const int bs = warp * (32 / RG) + lane / RG;
    const int b0 = c.s * G::SB;
    const int vb = min(G::SB, c.nb - b0);
    if (bs >= vb) return;
    const int b = b0 + bs;
    const unsigned char* rowp = mant_st + (bs >> 1) * (RG * 128) + r * 128;
    const int sw = r & 7;
    const int cbase = (bs & 1) * 4;
    const uint4* xb = reinterpret_cast<const uint4*>(xp) + b * 8;
    // two accumulators per lane class: dependent dp2a chains of 4, not 8
    int A0 = 0, A1 = 0, A2 = 0, A3 = 0, B0 = 0, B1 = 0, B2 = 0, B3 = 0;
#pragma unroll
    for (int cc = 0; cc < 4; cc++) {
        uint4 w = *reinterpret_cast<const uint4*>(rowp + (((cbase + cc) ^ sw) << 4));
        uint4 xa = xb[2 * cc], xc = xb[2 * cc + 1];
        int p01 = (int)__byte_perm(w.x, w.y, 0x5140), p23 = (int)__byte_perm(w.x, w.y, 0x7362);
        A0 = __dp2a_lo((int)xa.x, p01, A0);
        A1 = __dp2a_hi((int)xa.y, p01, A1);
        A2 = __dp2a_lo((int)xa.z, p23, A2);
        A3 = __dp2a_hi((int)xa.w, p23, A3);
        int q01 = (int)__byte_perm(w.z, w.w, 0x5140), q23 = (int)__byte_perm(w.z, w.w, 0x7362);
        B0 = __dp2a_lo((int)xc.x, q01, B0);
        B1 = __dp2a_hi((int)xc.y, q01, B1);
        B2 = __dp2a_lo((int)xc.z, q23, B2);
        B3 = __dp2a_hi((int)xc.w, q23, B3);
    }
    const int L0 = A0 + B0, L1 = A1 + B1, L2 = A2 + B2, L3 = A3 + B3;
    const uint32_t e = exps_st[r * G::SB + bs];
    const float xsb = xss[b];
    const int grow = (c.u - c.ub) * RG + r;
    float4 T;
    if ((c.M & 1) && grow == c.M - 1) {
        const float S = exp_scale_ieee(e);
        T.x = mul_rn(mul_rn(i2f_rn(L0 + L1 + L2 + L3), S), xsb);
        T.y = T.z = T.w = 0.0f;
    } else {
        const float S = exp_scale_ftz(e);
        T.x = mul_ftz(mul_ftz(i2f_rn(L0), S), xsb);
        T.y = mul_ftz(mul_ftz(i2f_rn(L1), S), xsb);
        T.z = mul_ftz(mul_ftz(i2f_rn(L2), S), xsb);
        T.w = mul_ftz(mul_ftz(i2f_rn(L3), S), xsb);
    }
    reinterpret_cast<float4*>(tb)[bs * RG + r] = T;
}

struct SliceInfo {
    int vb, row0, M, rv, d;
    bool last;
};

template <int RG>
__device__ __forceinline__ SliceInfo slice_info(const Cursor<RG>& c) {
    SliceInfo s;
    s.vb = min(Geo<RG>::SB, c.nb - c.s * Geo<RG>::SB);
    s.row0 = (c.u - c.ub) * RG;
    s.M = c.M;
    s.rv = min(RG, c.M - s.row0);
    s.d = c.d;
    s.last = (c.s == c.ns - 1);
    return s;
}

struct LmState {
    unsigned long long best;
    unsigned long long* cand;
    int* cand_count;
};

// Sequential float chain of one slice, run by the 4*RG threads of the LAST
// warps of the CTA (warps 0 and 1 also issue the TMA and exponent copies):
// chain thread c = row*4 + class.  The slice's terms are loaded first (they
// do not depend on the chain), then added in block order.
template <int RG, bool LM>
__device__ __forceinline__ void chain_slice(const GemvArgs& A, const SliceInfo& s, const float* tb,
                                            float& f, LmState& lm) {
    constexpr int SB = Geo<RG>::SB;
    const int ct = threadIdx.x - (kThreads - 4 * RG);
    if (ct < 0) return;
    const int r = ct >> 2, j = ct & 3;
    const int grow = s.row0 + r;
    const bool odd = (s.M & 1) && grow == s.M - 1;
    float t[SB];
#pragma unroll
    for (int bs = 0; bs < SB; bs++) t[bs] = (bs < s.vb) ? tb[bs * RG * 4 + ct] : 0.0f;
    if (odd) {
#pragma unroll
        for (int bs = 0; bs < SB; bs++)
            if (bs < s.vb) f = add_rn(f, t[bs]);
    } else {
#pragma unroll
        for (int bs = 0; bs < SB; bs++)
            if (bs < s.vb) f = add_ftz(f, t[bs]);
    }
    if (s.last) {
        float a = add_ftz(f, __shfl_xor_sync(0xffffffffu, f, 2));
        float yv = add_ftz(a, __shfl_xor_sync(0xffffffffu, a, 1));
        if (odd) yv = f;
        if (j == 0 && r < s.rv) {
            if (LM) {
                if (yv > -1e30f) {
                    unsigned long long k = cand_key(yv, grow);
                    lm.best = k > lm.best ? k : lm.best;
                }
                if (A.kk > 0 && yv > -3.402823466e38f) {
                    int p = atomicAdd(lm.cand_count, 1);
                    lm.cand[p] = cand_key(yv, grow);
                }
            } else {
                desc_ref(A, s.d).y[grow] = yv;
            }
        }
        f = 0.0f;
    }
}

struct SmemLayout {
    size_t exps, bars, terms, xp, xss, cand, total;
};
__host__ __device__ inline SmemLayout smem_layout(int kmax, bool lm) {
    SmemLayout L;
    L.exps = (size_t)kStages * kStageMant;
    L.bars = L.exps + (size_t)kStages * 256;
    L.terms = (L.bars + kStages * 8 + 15) & ~size_t(15);
    L.xp = L.terms + 2 * 1024 * sizeof(float);
    L.xss = L.xp + 2 * (size_t)kmax;
    L.cand = (L.xss + 4 * (size_t)(kmax / 64) + 15) & ~size_t(15);
    L.total = L.cand + (lm ? (size_t)kCandCap * 8 : 0);
    return L;
}

template <int RG, bool LM>
__global__ void __launch_bounds__(kThreads, 2) gemv_exact_kernel(const __grid_constant__ GemvArgs A) {
    using G = Geo<RG>;
    constexpr int P = kStages;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // TMA 128-byte swizzle needs 1024-byte aligned destinations
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                           ~uintptr_t(1023));
    const SmemLayout Ly = smem_layout(A.kmax, LM);
    unsigned char* mant_st = smem;
    unsigned char* exps_st = smem + Ly.exps;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Ly.bars);
    float* terms = reinterpret_cast<float*>(smem + Ly.terms);
    uint32_t* xp = reinterpret_cast<uint32_t*>(smem + Ly.xp);
    float* xss = reinterpret_cast<float*>(smem + Ly.xss);
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem + Ly.cand);
    __shared__ int s_cand_count;
    __shared__ unsigned long long s_red[kThreads / 32];

    LmState lm;
    lm.best = 0ull;
    lm.cand = cand;
    lm.cand_count = &s_cand_count;
    if (threadIdx.x == 0) {
        s_cand_count = 0;
        for (int s = 0; s < P; s++) mbar_init(&bars[s], 1);
        fence_barrier_init();
    }
    __syncthreads();

    const long long T = A.total_cost;
    int d0, d1;
    const int u_begin = unit_at_cost<RG>(A, (T * blockIdx.x) / gridDim.x, &d0);
    const int u_end = unit_at_cost<RG>(A, (T * (blockIdx.x + 1)) / gridDim.x, &d1);

    Cursor<RG> ic;
    ic.valid = u_begin < u_end;
    ic.u = u_begin;
    ic.s = 0;
    if (ic.valid) {
        ic.set_desc(A, d0);
        if (threadIdx.x == 0) tma_prefetch_desc(&desc_ref(A, d0).tmap);
    }
    Cursor<RG> cc = ic;

#pragma unroll 1
    for (int p = 0; p < P - 1; p++) {
        if (ic.valid) {
            issue_slice<RG>(A, ic, mant_st + p * kStageMant, exps_st + p * G::EXB, &bars[p]);
            ic.advance(A, u_end);
        }
        cp_async_commit();
    }

    int loaded_d = -1;
    float f = 0.0f;
    SliceInfo prev;
    bool have_prev = false;
    int i = 0;
#pragma unroll 1
    for (; cc.valid; i++) {
        const int st = i % P;
        mbar_wait(&bars[st], (uint32_t)(i / P) & 1u, A.err);
        cp_async_wait<P - 2>();
        __syncthreads();
        if (ic.valid) {
            const int ns = (i + P - 1) % P;
            issue_slice<RG>(A, ic, mant_st + ns * kStageMant, exps_st + ns * G::EXB, &bars[ns]);
            ic.advance(A, u_end);
        }
        cp_async_commit();
        if (cc.d != loaded_d) {
            stage_activation(desc_ref(A, cc.d), xp, xss);
            __syncthreads();
            loaded_d = cc.d;
        }
        if (LM && s_cand_count > kCandCap - 2 * RG) cand_compact(cand, &s_cand_count, A.kk);
        if (have_prev) chain_slice<RG, LM>(A, prev, terms + ((i - 1) & 1) * 1024, f, lm);
        compute_slice<RG>(cc, mant_st + st * kStageMant, exps_st + st * G::EXB, terms + (i & 1) * 1024, xp, xss);
        prev = slice_info<RG>(cc);
        have_prev = true;
        cc.advance(A, u_end);
    }
    cp_async_wait<0>();
    __syncthreads();
    if (have_prev) chain_slice<RG, LM>(A, prev, terms + ((i - 1) & 1) * 1024, f, lm);
    if (LM) {
        __syncthreads();
        unsigned long long* work = reinterpret_cast<unsigned long long*>(mant_st);
        const int work_cap = (P * kStageMant) / 8;
        lm_finish(A.sc, cand, &s_cand_count, work, work_cap, lm.best, A.kk, A.out_id, A.out_ids,
                  A.out_scores, A.out_n, s_red);
    }
}

// ---------------------------------------------------------------- generic
// Any K multiple of 64, any alignment: one thread per row, same arithmetic.
__global__ void __launch_bounds__(kThreads) gemv_generic_kernel(const __grid_constant__ GemvDesc D) {
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
    for (int b = 0; b < nb; b++) {
        int L[4] = {0, 0, 0, 0};
        for (int i2 = 0; i2 < 64; i2++) L[i2 & 3] += (int)w[64 * b + i2] * (int)xq[64 * b + i2];
        const uint32_t eb = e[b];
        if (odd) {
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
    D.y[m] = odd ? sum : add_ftz(add_ftz(f0, f2), add_ftz(f1, f3));
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

// ---------------------------------------------------------------- host side
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

static bool fast_shape_ok(const GemvDesc& d) {
    if (d.M <= 0 || d.K <= 0 || d.K % 512) return false;
    if (reinterpret_cast<uintptr_t>(d.mant) % 16 || reinterpret_cast<uintptr_t>(d.exps) % 8) return false;
    if (d.x ? (reinterpret_cast<uintptr_t>(d.x) % 8) : (reinterpret_cast<uintptr_t>(d.xq) % 4)) return false;
    return true;
}

bool gemv_plan(GemvDesc* descs, int n, int rows_per_unit, GemvPlan* plan) {
    const int sb = 256 / rows_per_unit;
    int units = 0, kmax = 0;
    long long cost = 0;
    for (int i = 0; i < n; i++) {
        GemvDesc& d = descs[i];
        if (!fast_shape_ok(d)) return false;
        if (!encode_tmap_2d(&d.tmap, d.mant, 1, (uint64_t)d.M, (uint64_t)d.K, (uint32_t)rows_per_unit)) return false;
        d.unit_begin = units;
        d.cost_begin = cost;
        const int u = (d.M + rows_per_unit - 1) / rows_per_unit;
        const int ns = ((d.K >> 6) + sb - 1) / sb;
        units += u;
        cost += (long long)u * ns;
        kmax = std::max(kmax, d.K);
    }
    plan->rows_per_unit = rows_per_unit;
    plan->n = n;
    plan->total_units = units;
    plan->total_cost = cost;
    plan->kmax = kmax;
    return true;
}

template <int RG, bool LM>
static cudaError_t launch_exact(const GemvArgs& A, int max_grid, cudaStream_t stream) {
    const size_t smem = smem_layout(A.kmax, LM).total + 1024;
    auto kern = gemv_exact_kernel<RG, LM>;
    static size_t configured = 0;   // largest dynamic smem size set so far
    if (smem > configured) {
        cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (err != cudaSuccess) return err;
        configured = smem;
    }
    int occ = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem) != cudaSuccess || occ < 1)
        occ = 1;
    const int grid = std::max(1, std::min(max_grid, num_sms() * occ));
    kern<<<grid, kThreads, smem, stream>>>(A);
    return cudaGetLastError();
}

static int pick_rows_per_unit(int M) {
    // enough units to give every CTA slot work; 32-row units read the most
    // bytes per shared-memory access
    const int slots = num_sms() * 2;
    if ((M + 31) / 32 >= slots) return 32;
    if ((M + 15) / 16 >= slots) return 16;
    return 8;
}

static cudaError_t dispatch_exact(GemvArgs& A, int rg, bool lm, int max_grid, cudaStream_t stream) {
    if (lm) {
        switch (rg) {
            case 32: return launch_exact<32, true>(A, max_grid, stream);
            case 16: return launch_exact<16, true>(A, max_grid, stream);
            default: return launch_exact<8, true>(A, max_grid, stream);
        }
    }
    switch (rg) {
        case 32: return launch_exact<32, false>(A, max_grid, stream);
        case 16: return launch_exact<16, false>(A, max_grid, stream);
        default: return launch_exact<8, false>(A, max_grid, stream);
    }
}

cudaError_t launch_gemv_list(const GemvDesc* dev_descs, const GemvPlan& plan, unsigned int* err,
                             cudaStream_t stream) {
    if (plan.n <= 0 || plan.total_units <= 0) return cudaSuccess;
    GemvArgs A{};
    A.list = dev_descs;
    A.n = plan.n;
    A.total_units = plan.total_units;
    A.total_cost = plan.total_cost;
    A.kmax = plan.kmax;
    A.err = err;
    return dispatch_exact(A, plan.rows_per_unit, false, plan.total_units, stream);
}

cudaError_t launch_gemv(const GemvDesc& d0, unsigned int* err, cudaStream_t stream) {
    if (d0.M <= 0) return cudaSuccess;
    if (d0.K <= 0 || d0.K % 64) return cudaErrorInvalidValue;
    GemvDesc d = d0;
    const int rg = pick_rows_per_unit(d.M);
    GemvPlan plan;
    if (!fast_shape_ok(d) || !gemv_plan(&d, 1, rg, &plan)) {
        const size_t smem = (((size_t)2 * d.K + 15) & ~size_t(15)) + 4 * (size_t)(d.K / 64);
        if (smem > 200 * 1024) return cudaErrorInvalidValue;
        cudaError_t e = cudaFuncSetAttribute(gemv_generic_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        gemv_generic_kernel<<<(d.M + kThreads - 1) / kThreads, kThreads, smem, stream>>>(d);
        return cudaGetLastError();
    }
    GemvArgs A{};
    A.single = d;
    A.list = nullptr;
    A.n = 1;
    A.total_units = plan.total_units;
    A.total_cost = plan.total_cost;
    A.kmax = plan.kmax;
    A.err = err;
    return dispatch_exact(A, rg, false, plan.total_units, stream);
}

cudaError_t launch_bfp8_lm_head(const float* h, const int8_t* mant, const uint8_t* exps, int vocab,
                                int hidden, int k, LmScratch* scratch, unsigned int* err, int* out_id,
                                int* out_ids, float* out_scores, int* out_n, cudaStream_t stream) {
    GemvDesc d{};
    d.mant = mant;
    d.exps = exps;
    d.x = h;
    d.M = vocab;
    d.K = hidden;
    if (vocab <= 0 || hidden <= 0 || k < 0 || std::min(k, vocab) > kTopkMax) return cudaErrorInvalidValue;
    const int rg = pick_rows_per_unit(vocab);
    GemvPlan plan;
    if (!fast_shape_ok(d) || !gemv_plan(&d, 1, rg, &plan)) return cudaErrorInvalidValue;
    GemvArgs A{};
    A.single = d;
    A.n = 1;
    A.total_units = plan.total_units;
    A.total_cost = plan.total_cost;
    A.kmax = plan.kmax;
    A.err = err;
    A.sc = scratch;
    A.kk = std::min(k, vocab);
    A.out_id = out_id;
    A.out_ids = out_ids;
    A.out_scores = out_scores;
    A.out_n = out_n;
    return dispatch_exact(A, rg, true, std::min(plan.total_units, kMaxGrid), stream);
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
