// gdn.cu -- the Gated-DeltaNet glue of a linear-attention layer and the
// token loop's small kernels.
//
// gdn_layer_kernel: one CTA per head.  Four column warps -- thread j owns
// channel j of the head's q, k and v and column j of its 128 x 128 state --
// and one gate warp, which computes the head's alpha and beta (two
// hidden-long dot products of the layer's normalized input in the
// reference's four-lane order, the longest dependent chains of the step)
// beside the column work.  Float semantics are
// the reference's NEON build (qwen_kernels_opt.c:507-858): vector steps
// flushed (mul/add/sub_ftz), multiply-accumulate not fused, every vector dot
// product four lane chains over i = 4m + l combined as (s0 + s2) + (s1 + s3),
// scalar VFP steps in IEEE single precision.
#include "common.cuh"
#include "gdn.cuh"

namespace qb {
namespace {

constexpr int kD = kGdnHeadDim;
constexpr int kColThreads = kD;              // four column warps
constexpr int kThreads = kColThreads + 32;   // and the gate warp

// Named barrier of the column warps only (the gate warp never joins it).
__device__ __forceinline__ void col_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kColThreads) : "memory"); }

// Two four-lane dot products in one warp, the reference's vector order:
// lanes 0..3 run the chains of a0 . b0 (lane l over i = 4m + l, product
// rounded then added, both flushed), lanes 4..7 those of a1 . b1; the result
// (s0 + s2) + (s1 + s3) lands in lane 0 (first dot) and lane 4 (second).
// Every lane of the warp calls it; n % 4 == 0.
__device__ __forceinline__ float dot4_pair(const float* a0, const float* b0, const float* a1, const float* b1, int n,
                                           int lane) {
    float acc = 0.0f;
    if (lane < 8) {
        const float* a = lane < 4 ? a0 : a1;
        const float* b = lane < 4 ? b0 : b1;
#pragma unroll 8
        for (int i = lane & 3; i < n; i += 4) acc = add_ftz(acc, mul_ftz(a[i], b[i]));
    }
    const float pair = add_ftz(acc, __shfl_down_sync(0xffffffffu, acc, 2));   // s0 + s2, s1 + s3
    return add_ftz(pair, __shfl_down_sync(0xffffffffu, pair, 1));
}

// 1 / sqrtf(x) as the reference's scalar code evaluates it (IEEE divide and
// square root).
__device__ __forceinline__ float recip_sqrt_ieee(float x) { return __fdiv_rn(1.0f, __fsqrt_rn(x)); }

__global__ void __launch_bounds__(kThreads) gdn_layer_kernel(const GdnArgs a) {
    extern __shared__ float gdn_smem[];   // normed | wa row | wb row (hidden floats each)
    __shared__ float sq[kD], sk[kD], sv[kD], so[kD];
    __shared__ float s_kr, s_qr, s_qk, s_rg, s_alpha, s_beta;
    const int hd = blockIdx.x, t = threadIdx.x;
    const int HD = a.heads * kD, C = 3 * HD;

    if (t < kColThreads) {
        // column t of the head's state, S[4g+u][t] = B[16g+u]: all 32 float4
        // loads go out first and land while the conv and the norms run
        float* B = a.state + (size_t)hd * kD * kD + (size_t)(t >> 2) * (kD * 4) + (t & 3) * 4;
        float4 col[kD / 4];
#pragma unroll
        for (int g = 0; g < kD / 4; g++) col[g] = *reinterpret_cast<const float4*>(B + 16 * g);
        const float zt = a.z[hd * kD + t], nw = a.norm_w[t];   // for the gated norm at the end
        // ---- causal_conv1d_update_silu (qwen_kernels_opt.c:511-545), channels
        // hd*128 + t of q, k and v: d = w0*s0 + w1*s1 + w2*s2 + w3*x (multiply,
        // then three multiply-adds), y = d / (1 + exp_neon(-d)) with the
        // division on VFP; the state shifts
#pragma unroll
        for (int part = 0; part < 3; part++) {
            const int c = part * HD + hd * kD + t;
            const float xc = a.qkv[c];
            const float t0 = a.conv_s[c], t1 = a.conv_s[C + c], t2 = a.conv_s[2 * C + c];
            const float* w = a.conv_w + 4 * (size_t)c;
            float d = mul_ftz(w[0], t0);
            d = add_ftz(d, mul_ftz(w[1], t1));
            d = add_ftz(d, mul_ftz(w[2], t2));
            d = add_ftz(d, mul_ftz(w[3], xc));
            const float y = __fdiv_rn(d, add_ftz(1.0f, exp_neon_lane(-d)));
            a.conv_s[c] = t1;
            a.conv_s[C + c] = t2;
            a.conv_s[2 * C + c] = xc;
            (part == 0 ? sq : part == 1 ? sk : sv)[t] = y;
        }
        col_sync();
        // ---- qk_l2norm (qwen_kernels_opt.c:548-591): |k|^2 and |q|^2 in the
        // vector order, the scales on VFP, the products on the vector unit
        if (t < 32) {
            const float s = dot4_pair(sk, sk, sq, sq, kD, t);
            if (t == 0) s_kr = recip_sqrt_ieee(__fadd_rn(s, 1e-6f));
            if (t == 4) s_qr = __fdiv_rn(recip_sqrt_ieee((float)kD), __fsqrt_rn(__fadd_rn(s, 1e-6f)));
        }
        col_sync();
        sk[t] = mul_ftz(sk[t], s_kr);
        sq[t] = mul_ftz(sq[t], s_qr);
        col_sync();
        // ---- gdn_recurrent_step (qwen_kernels_opt.c:664-829): qk = q . k;
        // column t: kv = sum_i S[i][t] k[i], qs = sum_i S[i][t] q[i], ascending i
        if (t < 32) {
            const float s = dot4_pair(sq, sk, sq, sk, kD, t);
            if (t == 0) s_qk = s;
        }
        float kv = 0.0f, qs = 0.0f;
#pragma unroll
        for (int g = 0; g < kD / 4; g++) {
            const float4 s4 = col[g];
            kv = add_ftz(kv, mul_ftz(s4.x, sk[4 * g]));
            qs = add_ftz(qs, mul_ftz(s4.x, sq[4 * g]));
            kv = add_ftz(kv, mul_ftz(s4.y, sk[4 * g + 1]));
            qs = add_ftz(qs, mul_ftz(s4.y, sq[4 * g + 1]));
            kv = add_ftz(kv, mul_ftz(s4.z, sk[4 * g + 2]));
            qs = add_ftz(qs, mul_ftz(s4.z, sq[4 * g + 2]));
            kv = add_ftz(kv, mul_ftz(s4.w, sk[4 * g + 3]));
            qs = add_ftz(qs, mul_ftz(s4.w, sq[4 * g + 3]));
        }
        __syncthreads();   // the gate warp's alpha and beta
        const float al = s_alpha, be = s_beta;
        // d = (v - kv*a) * b; out = qs*a + qk*d; S = S*a + d*k[i]
        const float d = mul_ftz(sub_ftz(sv[t], mul_ftz(kv, al)), be);
        so[t] = add_ftz(mul_ftz(qs, al), mul_ftz(s_qk, d));
#pragma unroll
        for (int g = 0; g < kD / 4; g++) {
            float4 s4 = col[g];
            s4.x = add_ftz(mul_ftz(s4.x, al), mul_ftz(d, sk[4 * g]));
            s4.y = add_ftz(mul_ftz(s4.y, al), mul_ftz(d, sk[4 * g + 1]));
            s4.z = add_ftz(mul_ftz(s4.z, al), mul_ftz(d, sk[4 * g + 2]));
            s4.w = add_ftz(mul_ftz(s4.w, al), mul_ftz(d, sk[4 * g + 3]));
            *reinterpret_cast<float4*>(B + 16 * g) = s4;
        }
        col_sync();
        // ---- rmsnorm_gated (qwen_kernels_opt.c:832-858): r from |out|^2 in the
        // vector order; then on VFP y = ((out * r) * w) * (z / (1 + expf(-z)))
        if (t < 32) {
            const float s = dot4_pair(so, so, so, so, kD, t);
            if (t == 0) s_rg = recip_sqrt_ieee(__fadd_rn(__fdiv_rn(s, (float)kD), 1e-6f));
        }
        col_sync();
        const float silu = __fdiv_rn(zt, __fadd_rn(1.0f, expf(-zt)));
        a.out[hd * kD + t] = __fmul_rn(__fmul_rn(__fmul_rn(so[t], s_rg), nw), silu);
    } else {
        // ---- gate warp: gdn_gates (qwen_kernels_opt.c:593-625) for this head
        // from n = the layer's rmsnorm(h, in_ln_w): av = wa . n, bv = wb . n;
        // beta = 1 / (1 + expf(-bv)); alpha = expf(nea * log1pf(expf(av + dt)))
        const int lane = t - kColThreads, H = a.hidden;
        float* sx = gdn_smem;
        float* swa = gdn_smem + H;
        float* swb = gdn_smem + 2 * H;
        const float* wa = a.wa + (size_t)hd * H;
        const float* wb = a.wb + (size_t)hd * H;
        // stage n and the head's wa / wb rows; every load of a lane goes out
        // before the first store (16-byte loads where all three allow them)
        if (((reinterpret_cast<uintptr_t>(a.normed) | reinterpret_cast<uintptr_t>(wa) |
              reinterpret_cast<uintptr_t>(wb)) & 15) == 0) {
            for (int i0 = lane; i0 < H / 4; i0 += 32 * 4) {
                float4 v[4][3];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int i = i0 + 32 * u;
                    if (i < H / 4) {
                        v[u][0] = reinterpret_cast<const float4*>(a.normed)[i];
                        v[u][1] = reinterpret_cast<const float4*>(wa)[i];
                        v[u][2] = reinterpret_cast<const float4*>(wb)[i];
                    }
                }
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int i = i0 + 32 * u;
                    if (i < H / 4) {
                        reinterpret_cast<float4*>(sx)[i] = v[u][0];
                        reinterpret_cast<float4*>(swa)[i] = v[u][1];
                        reinterpret_cast<float4*>(swb)[i] = v[u][2];
                    }
                }
            }
        } else {
#pragma unroll 8
            for (int i = lane; i < H; i += 32) {
                const float x = a.normed[i], ya = wa[i], yb = wb[i];
                sx[i] = x;
                swa[i] = ya;
                swb[i] = yb;
            }
        }
        __syncwarp();
        const float g = dot4_pair(swa, sx, swb, sx, H, lane);   // lane 0: av, lane 4: bv
        const float bv = __shfl_sync(0xffffffffu, g, 4);
        if (lane == 0) {
            s_beta = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-bv)));
            s_alpha = expf(__fmul_rn(a.nea[hd], log1pf(expf(__fadd_rn(g, a.dt[hd])))));
        }
        __syncthreads();
    }
}

__global__ void embed_row_kernel(float* h, const uint16_t* E, long long row, int hidden) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
        h[i] = __uint_as_float((uint32_t)E[row * hidden + i] << 16);
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(float* y, const float* x, const float* w, int n, float eps) {
    extern __shared__ float rms_smem[];
    __shared__ float s_r;
    for (int i = threadIdx.x; i < n; i += blockDim.x) rms_smem[i] = x[i];
    __syncthreads();
    if (threadIdx.x < 32) {
        const float ss = dot4_pair(rms_smem, rms_smem, rms_smem, rms_smem, n, threadIdx.x);
        if (threadIdx.x == 0) s_r = recip_sqrt_ieee(__fadd_rn(__fdiv_rn(ss, (float)n), eps));
    }
    __syncthreads();
    const float r = s_r;
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = mul_ftz(rms_smem[i], mul_ftz(r, add_ftz(1.0f, w[i])));
}

}  // namespace

cudaError_t launch_gdn_layer(const GdnArgs& a, cudaStream_t stream) {
    if (a.heads <= 0 || a.hidden <= 0 || a.hidden % 4 || a.hidden > kGdnMaxHidden || !a.qkv || !a.z || !a.normed ||
        !a.conv_w || !a.conv_s || !a.wa || !a.wb || !a.nea || !a.dt || !a.state || !a.norm_w || !a.out)
        return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(a.state) % 16) return cudaErrorInvalidValue;
    const size_t smem = 3 * (size_t)a.hidden * sizeof(float);
    if (cudaError_t e = raise_smem_limit(reinterpret_cast<const void*>(gdn_layer_kernel), smem)) return e;
    gdn_layer_kernel<<<a.heads, kThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_embed_row(float* h, const uint16_t* E, long long row, int hidden, cudaStream_t stream) {
    if (!h || !E || row < 0 || hidden <= 0) return cudaErrorInvalidValue;
    embed_row_kernel<<<(hidden + 255) / 256, 256, 0, stream>>>(h, E, row, hidden);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(float* y, const float* x, const float* w, int n, float eps, cudaStream_t stream) {
    if (!y || !x || !w || n <= 0 || n % 4 || n > kGdnMaxHidden) return cudaErrorInvalidValue;
    const size_t smem = (size_t)n * sizeof(float);
    if (cudaError_t e = raise_smem_limit(reinterpret_cast<const void*>(rmsnorm_kernel), smem)) return e;
    rmsnorm_kernel<<<1, 256, smem, stream>>>(y, x, w, n, eps);
    return cudaGetLastError();
}

}  // namespace qb
