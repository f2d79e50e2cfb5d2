// bfp8_gemm_tc.cu -- batched BFP8 GEMM: tcgen05 kind::i8 with TMEM
// accumulators, TMA-fed shared-memory pipeline, warp-specialised CTA.
//
// Work unit: a tile of 128 weight rows x N batch columns over the whole K of
// one GEMM.  A persistent CTA (one per SM) walks its units in a fixed
// round-robin order; its warps split the work:
//   warp 0      TMA producer: per 128-byte K stage one weight box
//               (128 rows x 128 B), one activation box (both planes, N rows)
//               and one scale box (N columns x 2 blocks) on one mbarrier;
//   warp 1      allocates TMEM and issues the MMAs from one thread: per
//               64-block two K=32 steps into a hi accumulator and two into
//               a lo accumulator (N columns each), then tcgen05.commit;
//   warps 2..9  epilogue: each thread owns one weight row (its TMEM lane)
//               and N/2 batch columns; per block it reads Dhi/Dlo from
//               TMEM, frees the slot, and accumulates
//               float(256*Dhi + Dlo) * 2^(e-134) * xs in f32 registers.
// TMEM holds kSlots accumulator pairs so the tensor cores run ahead of the
// epilogue by up to kSlots blocks; shared memory holds kStages K stages.
// Every mbarrier wait is bounded (error word + early exit), and TMEM is
// released only after a final commit shows no MMA in flight.
#include "bfp8_gemm_tc.cuh"
#include "bfp8_gemv.cuh"
#include "common.cuh"
#include "tma.cuh"

#include <algorithm>

namespace qb {
namespace {

constexpr int kTcThreads = 320;
constexpr int kEpiWarps = 8;
constexpr int kTileRows = 128;
constexpr int kStageK = 128;   // K bytes per pipeline stage (two 64-blocks)

template <int N>
struct TcCfg {
    static constexpr int kStages = N >= 128 ? 4 : (N >= 64 ? 6 : 8);
    static constexpr int kSlots = (256 / N) < 8 ? (256 / N) : 8;
    static constexpr int kTmemCols = kSlots * 2 * N;   // 128..512, a power of two
    static constexpr int kWBytes = kTileRows * kStageK;
    static constexpr int kXBytes = 2 * N * kStageK;
    static constexpr int kStageBytes = kWBytes + kXBytes;
    static constexpr int kSBox = 2 * N * 4;                          // scale bytes per stage
    static constexpr int kSBytes = kSBox < 128 ? 128 : kSBox;        // 128-byte aligned slots
    static constexpr int kTxBytes = kStageBytes + kSBox;
    static constexpr int kCols = N / 2;                              // columns per epilogue thread
    static constexpr int kChunk = kCols < 16 ? kCols : 16;
    static constexpr size_t kSmem =
        1024 + (size_t)kStages * (kStageBytes + kSBytes) + (size_t)(2 * kStages + 2 * kSlots + 1) * 8 + 16;
};

struct TcLaunch {
    const TcDesc* descs;   // device array, or null: use `one`
    int n, total_units;
    unsigned int* err;
    TcDesc one;
};

// ------------------------------------------------------------ tcgen05 PTX
// Shared-memory matrix descriptor of a K-major tile written by TMA with
// SWIZZLE_128B: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO),
// descriptor version 1, layout code 2 (128-byte swizzle).  Advancing along K
// inside the 128-byte row adds (bytes >> 4) to the start-address field.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: int32 accumulator, A signed int8 K-major, B int8
// (signed or unsigned) K-major, M = 128, N columns.
template <int N>
__host__ __device__ constexpr uint32_t idesc_i8(bool b_signed) {
    return (2u << 4) | (1u << 7) | ((b_signed ? 1u : 0u) << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(kTileRows >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accum));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 lanes x C consecutive 32-bit columns: thread i gets lane (base + i).
template <int C>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&v)[C]);
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, uint32_t (&v)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

__device__ __forceinline__ const TcDesc* desc_for(const TcLaunch& p, int u, int& di) {
    if (!p.descs) return &p.one;
    while (di + 1 < p.n && u >= p.descs[di + 1].unit_begin) di++;
    return p.descs + di;
}

// Warp-uniform bounded wait (every lane polls; the warp agrees on the result).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
    const bool ok = mbar_wait(bar, parity, err);
    return __all_sync(0xffffffffu, ok);
}

template <int N, bool DOTS>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const __grid_constant__ TcLaunch p) {
    using C = TcCfg<N>;
    extern __shared__ unsigned char tc_smem_raw[];
    unsigned char* base =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* stages = base;
    unsigned char* sxs = base + (size_t)C::kStages * C::kStageBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(sxs + (size_t)C::kStages * C::kSBytes);
    uint64_t* empty = full + C::kStages;
    uint64_t* tfull = empty + C::kStages;
    uint64_t* tempty = tfull + C::kSlots;
    uint64_t* done = tempty + C::kSlots;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + kEpiWarps);   // MMA commit + every epilogue warp (scales read)
        }
        for (int t = 0; t < C::kSlots; t++) {
            mbar_init(&tfull[t], 1);
            mbar_init(&tempty[t], kEpiWarps);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, C::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t gs = 0;
            int di = 0;
            bool bad = false;
            for (int u = blockIdx.x; u < p.total_units && !bad; u += gridDim.x) {
                const TcDesc* d = desc_for(p, u, di);
                const int local = u - d->unit_begin, rt = local / d->n_nt, nt = local - rt * d->n_nt;
                const int nst = (d->nb + 1) >> 1;
                for (int st = 0; st < nst; st++, gs++) {
                    const int s = gs % C::kStages;
                    if (!mbar_wait(&empty[s], ((gs / C::kStages) & 1) ^ 1, p.err)) {
                        bad = true;
                        break;
                    }
                    unsigned char* sm = stages + (size_t)s * C::kStageBytes;
                    mbar_arrive_expect_tx(&full[s], C::kTxBytes);
                    tma_load_2d(sm, &d->tm_w, st * kStageK, rt * kTileRows, &full[s]);
                    tma_load_3d(sm + C::kWBytes, &d->tm_x, st * kStageK, nt * N, 0, &full[s]);
                    tma_load_2d(sxs + (size_t)s * C::kSBytes, &d->tm_s, nt * N, st * 2, &full[s]);
                }
            }
            // the last loads of every slot have landed unless a consumer quit early
            for (uint32_t i = gs > (uint32_t)C::kStages ? gs - C::kStages : 0; i < gs; i++)
                mbar_wait(&full[i % C::kStages], (i / C::kStages) & 1, nullptr);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t kIdHi = idesc_i8<N>(true), kIdLo = idesc_i8<N>(false);
            uint32_t gs = 0, gb = 0;
            int di = 0;
            bool bad = false;
            for (int u = blockIdx.x; u < p.total_units && !bad; u += gridDim.x) {
                const TcDesc* d = desc_for(p, u, di);
                const int nb = d->nb, nst = (nb + 1) >> 1;
                for (int st = 0; st < nst && !bad; st++, gs++) {
                    const int s = gs % C::kStages;
                    if (!mbar_wait(&full[s], (gs / C::kStages) & 1, p.err)) {
                        bad = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(stages + (size_t)s * C::kStageBytes);
                    const uint64_t da = desc_sw128(a0), dh = desc_sw128(a0 + C::kWBytes),
                                   dl = desc_sw128(a0 + C::kWBytes + N * kStageK);
                    for (int h = 0; h < 2 && 2 * st + h < nb; h++, gb++) {
                        const int t = gb % C::kSlots;
                        if (!mbar_wait(&tempty[t], ((gb / C::kSlots) & 1) ^ 1, p.err)) {
                            bad = true;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t dhi = tmem + (uint32_t)(t * 2 * N), dlo = dhi + N;
#pragma unroll
                        for (int kk = 0; kk < 2; kk++) {
                            const uint64_t off = (uint64_t)((h * 64 + kk * 32) >> 4);
                            mma_i8(dhi, da + off, dh + off, kIdHi, kk);
                            mma_i8(dlo, da + off, dl + off, kIdLo, kk);
                        }
                        mma_commit(&tfull[t]);
                    }
                    mma_commit(&empty[s]);
                }
            }
            // no MMA may still be writing TMEM when it is released
            mma_commit(done);
            mbar_wait(done, 0, nullptr);
        }
    } else {
        // ---------------------------------------------------- epilogue
        const int ew = warp - 2, q = warp & 3, chalf = ew >> 2;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        uint32_t gs = 0, gb = 0;
        int di = 0;
        bool bad = false;
        for (int u = blockIdx.x; u < p.total_units && !bad; u += gridDim.x) {
            const TcDesc* d = desc_for(p, u, di);
            const int M = d->M, nb = d->nb, B = d->B;
            const int local = u - d->unit_begin, rt = local / d->n_nt, nt = local - rt * d->n_nt;
            const int m = rt * kTileRows + q * 32 + lane;
            const bool row_ok = m < M;
            const uint8_t* erow = d->exps + (size_t)(row_ok ? m : 0) * nb;
            int32_t* dots = d->dots;
            float acc[C::kCols];
#pragma unroll
            for (int i = 0; i < C::kCols; i++) acc[i] = 0.0f;
            uint32_t e_next = __ldg(erow);
            for (int j = 0; j < nb; j++, gb++) {
                const int h = j & 1;
                const int s = (gs + (j >> 1)) % C::kStages;
                const uint32_t e = e_next;
                if (j + 1 < nb) e_next = __ldg(erow + j + 1);
                const int t = gb % C::kSlots;
                if (!warp_wait(&tfull[t], (gb / C::kSlots) & 1, p.err)) {
                    bad = true;
                    break;
                }
                tc_fence_after();
                const float sm = exp_scale_ieee(e);
                const float* xsv =
                    reinterpret_cast<const float*>(sxs + (size_t)s * C::kSBytes) + h * N + chalf * C::kCols;
                const uint32_t tcol = tmem + lane_base + (uint32_t)(t * 2 * N + chalf * C::kCols);
#pragma unroll
                for (int c = 0; c < C::kCols; c += C::kChunk) {
                    uint32_t hv[C::kChunk], lv[C::kChunk];
                    tmem_ld<C::kChunk>(tcol + c, hv);
                    tmem_ld<C::kChunk>(tcol + N + c, lv);
                    tmem_wait_ld();
                    if (c + C::kChunk >= C::kCols) {   // slot drained: hand it back to the MMA warp
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[t]);
                    }
#pragma unroll
                    for (int i = 0; i < C::kChunk; i++) {
                        const int D = (int)hv[i] * 256 + (int)lv[i];
                        acc[c + i] = fmaf(i2f_rn(D), sm * xsv[c + i], acc[c + i]);
                        if constexpr (DOTS) {
                            const int b = nt * N + chalf * C::kCols + c + i;
                            if (row_ok && b < B) dots[((size_t)b * M + m) * nb + j] = D;
                        }
                    }
                }
                if (h == 1 || j == nb - 1) {   // this warp is done with the stage's scales
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[s]);
                }
            }
            gs += (nb + 1) >> 1;
            if (bad) break;
            if (row_ok) {
                float* y = d->y;
#pragma unroll
                for (int i = 0; i < C::kCols; i++) {
                    const int b = nt * N + chalf * C::kCols + i;
                    if (b < B) y[(size_t)b * M + m] = acc[i];
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

// ------------------------------------------------------------ quantizer
// One warp per (row, 64-block); lane l quantizes elements 2l and 2l+1 with
// the reference's arithmetic: amax, q = 16384/amax (IEEE division), xq =
// rint(x*q) half-even, xs = amax/16384; zero block when amax <= 1e-20.
__global__ void __launch_bounds__(256) quant_planes_kernel(const float* x, int B, int K, uint8_t* planes,
                                                           float* xs_t, int ldxs) {
    const int nb = K >> 6;
    const long long total = (long long)B * nb;
    const int lane = threadIdx.x & 31;
    for (long long g = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); g < total; g += (long long)gridDim.x * 8) {
        const int b = (int)(g / nb), kb = (int)(g - (long long)b * nb);
        const size_t off = (size_t)b * K + (size_t)kb * 64 + 2 * lane;
        const float2 v = *reinterpret_cast<const float2*>(x + off);
        float a = fmaxf(fabsf(v.x), fabsf(v.y));
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        int q0 = 0, q1 = 0;
        float s = 0.0f;
        if (a > 1e-20f) {
            const float q = __fdiv_rn(16384.0f, a);
            s = __fdiv_rn(a, 16384.0f);
            q0 = __float2int_rn(__fmul_rn(v.x, q));
            q1 = __float2int_rn(__fmul_rn(v.y, q));
        }
        const uint32_t hi = ((uint32_t)(q0 >> 8) & 0xFFu) | (((uint32_t)(q1 >> 8) & 0xFFu) << 8);
        const uint32_t lo = ((uint32_t)q0 & 0xFFu) | (((uint32_t)q1 & 0xFFu) << 8);
        *reinterpret_cast<uint16_t*>(planes + off) = (uint16_t)hi;
        *reinterpret_cast<uint16_t*>(planes + (size_t)B * K + off) = (uint16_t)lo;
        if (lane == 0) xs_t[(size_t)kb * ldxs + b] = s;
    }
}

template <int N, bool DOTS>
cudaError_t launch_n(const TcDesc* dev_descs, const TcDesc* one, int n, int total_units, unsigned int* err,
                     cudaStream_t stream) {
    using C = TcCfg<N>;
    static unsigned long long attr_set = 0;   // one bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!(attr_set >> dev & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<N, DOTS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)C::kSmem);
        if (e != cudaSuccess) return e;
        attr_set |= 1ull << dev;
    }
    TcLaunch p{};
    p.descs = dev_descs;
    p.n = n;
    p.total_units = total_units;
    p.err = err;
    if (one) p.one = *one;
    const int grid = std::max(1, std::min(total_units, num_sms()));
    gemm_tc_kernel<N, DOTS><<<grid, kTcThreads, C::kSmem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

int tc_tile_n(int B) {
    if (B <= 8) return 8;
    if (B <= 16) return 16;
    if (B <= 32) return 32;
    if (B <= 64) return 64;
    return 128;
}

bool tc_make_desc(TcDesc* d, float* y, const void* planes, const float* xs_t, int ldxs, const int8_t* mant,
                  const uint8_t* exps, int M, int K, int B, int32_t* dots) {
    if (!d || !y || !planes || !xs_t || !mant || !exps || M <= 0 || K <= 0 || K % 64 || B <= 0) return false;
    if (ldxs < B || ldxs % 4) return false;
    if ((reinterpret_cast<uintptr_t>(planes) | reinterpret_cast<uintptr_t>(xs_t) |
         reinterpret_cast<uintptr_t>(mant)) & 15)
        return false;
    const int N = tc_tile_n(B);
    *d = TcDesc{};
    {   // weights: [M][K] bytes, box 128 B x 128 rows
        const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
        const uint64_t str[1] = {(uint64_t)K};
        const uint32_t box[2] = {(uint32_t)kStageK, (uint32_t)kTileRows};
        if (!encode_tmap(&d->tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, mant, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
            return false;
    }
    {   // activation planes: [2][B][K] bytes, box 128 B x N rows x 2 planes
        const uint64_t dims[3] = {(uint64_t)K, (uint64_t)B, 2};
        const uint64_t str[2] = {(uint64_t)K, (uint64_t)B * (uint64_t)K};
        const uint32_t box[3] = {(uint32_t)kStageK, (uint32_t)N, 2};
        if (!encode_tmap(&d->tm_x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, planes, dims, str, box,
                         CU_TENSOR_MAP_SWIZZLE_128B))
            return false;
    }
    {   // scales: [nb][ldxs] f32, box N columns x 2 blocks
        const uint64_t dims[2] = {(uint64_t)B, (uint64_t)(K / 64)};
        const uint64_t str[1] = {(uint64_t)ldxs * 4};
        const uint32_t box[2] = {(uint32_t)N, 2};
        if (!encode_tmap(&d->tm_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, xs_t, dims, str, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE))
            return false;
    }
    d->exps = exps;
    d->y = y;
    d->dots = dots;
    d->M = M;
    d->K = K;
    d->B = B;
    d->nb = K / 64;
    d->unit_begin = 0;
    d->n_nt = (B + N - 1) / N;
    return true;
}

int tc_units(const TcDesc& d) { return ((d.M + kTileRows - 1) / kTileRows) * d.n_nt; }

template <bool DOTS>
static cudaError_t launch_b(const TcDesc* dev_descs, const TcDesc* one, int n, int total_units, int B, unsigned int* err,
                     cudaStream_t stream) {
    switch (tc_tile_n(B)) {
        case 8: return launch_n<8, DOTS>(dev_descs, one, n, total_units, err, stream);
        case 16: return launch_n<16, DOTS>(dev_descs, one, n, total_units, err, stream);
        case 32: return launch_n<32, DOTS>(dev_descs, one, n, total_units, err, stream);
        case 64: return launch_n<64, DOTS>(dev_descs, one, n, total_units, err, stream);
        default: return launch_n<128, DOTS>(dev_descs, one, n, total_units, err, stream);
    }
}

cudaError_t launch_gemm_tc(const TcDesc* dev_descs, const TcDesc* one, int n, int total_units, int B, bool dots,
                           unsigned int* err, cudaStream_t stream) {
    if (total_units <= 0) return cudaSuccess;
    return dots ? launch_b<true>(dev_descs, one, n, total_units, B, err, stream)
                : launch_b<false>(dev_descs, one, n, total_units, B, err, stream);
}

cudaError_t launch_quant_planes(const float* x, int B, int K, void* planes, float* xs_t, int ldxs,
                                cudaStream_t stream) {
    const long long total = (long long)B * (K / 64);
    if (total <= 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((total + 7) / 8, (long long)num_sms() * 16);
    quant_planes_kernel<<<grid, 256, 0, stream>>>(x, B, K, static_cast<uint8_t*>(planes), xs_t, ldxs);
    return cudaGetLastError();
}

}  // namespace qb
