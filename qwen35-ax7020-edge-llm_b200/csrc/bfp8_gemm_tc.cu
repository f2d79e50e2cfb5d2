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
//               64-block two K=32 steps of one M=128, N=2*N_tile MMA whose
//               B operand is the hi plane rows followed by the lo plane rows
//               (both signed int8), so the accumulator holds the hi dots in
//               columns [0, N) and the lo dots in [N, 2N); then
//               tcgen05.commit;
//   warps 2..   epilogue (8 or 16 warps): each thread owns one weight row
//               (its TMEM lane) and a slice of the batch columns; per block
//               it reads Dhi/Dlo from TMEM, frees the slot, and accumulates
//               float(256*Dhi + Dlo) * 2^(e-134) * xs in f32 registers.
// TMEM holds kSlots accumulator pairs so the tensor cores run ahead of the
// epilogue by up to kSlots blocks; shared memory holds kStages K stages.
// The producer resolves each unit (descriptor, tile, exponent tile) once and
// publishes it through a two-entry unit ring in shared memory, so the MMA and
// epilogue warps never wait on descriptor loads at unit boundaries.
// Every mbarrier wait is bounded (error word + early exit), and TMEM is
// released only after a final commit shows no MMA in flight.
#include "bfp8_gemm_tc.cuh"
#include "bfp8_gemv.cuh"
#include "common.cuh"
#include "tma.cuh"

#include <algorithm>

namespace qb {
namespace {

constexpr int kTileRows = 128;
static_assert(kTileRows == kTcTileRowsPublic, "partial slots are laid out for 128-row tiles");
constexpr int kBoxK = 128;     // K bytes of one TMA box (one 128-byte swizzled row per matrix row)

// 64-blocks per pipeline stage: four for narrow tiles (so the single TMA and
// MMA threads pay their per-stage barrier work once per 32 KB of weights),
// two for wide ones (shared memory holds fewer, larger stages).
__host__ __device__ constexpr int tc_blocks_per_stage(int N) { return N <= 32 ? 4 : 2; }

constexpr int kExpsMax = 56;   // block exponents per row staged in shared memory (K <= 3584)
constexpr int kMaxTable = kTcMaxDescs;   // GEMMs per launch (their scalar fields are kept in shared memory)
constexpr int kEBytes = kTileRows * kExpsMax;

// Block dot recombination: each block's hi and lo accumulators hold the
// exact int32 dots Dhi and Dlo; 256 * Dhi + Dlo is the exact int32 block dot
// D (|D| < 2^31), formed with one integer multiply-add and converted to fp32
// with one rounding (the conversion runs on the integer pipe, beside the
// fp32 scale-and-accumulate on the FMA pipe).

// Scalar fields of one GEMM, copied to shared memory at kernel start so that
// unit lookups never wait on global loads.
struct DescRow {
    int unit_begin, n_nt, nb, M, B, ldy, tile_begin, pad_;
    const uint8_t* exps;
    float* y;
    int32_t* dots;
    const PeerOut* peer;
};

// One unit as the producer publishes it to the MMA and epilogue warps.
struct UnitInfo {
    const uint8_t* exps;   // exponent rows of the tile (shared-memory copy when ebulk)
    float* y;
    int32_t* dots;
    const PeerOut* peer;
    unsigned int* tickets;  // pieces of a cut tile: the tile's counters
    int M, nb, B, rt, nt, ebulk, ldy;
    int j0, nbs;            // the unit covers blocks [j0, j0 + nbs) of the tile; nbs == 0 ends the sequence
    int npieces, cfirst, pslot;   // a tile cut between CTAs: its piece count, first CTA, this piece's slot
};

template <int N>
struct TcCfg {
    static constexpr int kBPS = tc_blocks_per_stage(N);
    static constexpr int kStageK = 64 * kBPS;                        // K bytes per stage
    static constexpr int kBoxes = kStageK / kBoxK;                   // TMA boxes per operand per stage
    static constexpr int kStages = N >= 128 ? 4 : (N >= 64 ? 6 : (N >= 32 ? 4 : 5));
    static constexpr int kSlots = (256 / N) < 8 ? (256 / N) : 8;
    static constexpr int kTmemCols = kSlots * 2 * N;   // 128..512, a power of two
    static constexpr int kWBytes = kTileRows * kStageK;
    static constexpr int kXBytes = 2 * N * kStageK;
    static constexpr int kStageBytes = kWBytes + kXBytes;
    static constexpr int kSBox = kBPS * N * 4;                       // scale bytes per stage
    static constexpr int kSBytes = kSBox < 128 ? 128 : kSBox;        // 128-byte aligned slots
    static constexpr int kTxBytes = kStageBytes + kSBox;
    // Epilogue warps: four per 32-lane TMEM quarter for wide tiles (each warp
    // a quarter of the columns), two for narrow ones.
    static constexpr int kEpiWarps = N >= 64 ? 16 : 8;
    static constexpr int kColSplit = kEpiWarps / 4;
    static constexpr int kThreads = 64 + 32 * kEpiWarps;
    static constexpr int kCols = N / kColSplit;                      // columns per epilogue thread
    // Small tiles: the epilogue takes kGroup blocks per round (one barrier
    // wait and one TMEM load wait for all of them).  Large tiles: one block
    // per round, read whole and its slot freed before the arithmetic.
    static constexpr int kGroup = N <= 16 ? 4 : (N <= 32 ? 2 : 1);
    static constexpr int kGroupsInFlight = kSlots / kGroup;
    // blocks whose TMEM slots the MMA thread claims with one wait (whole
    // epilogue groups, at most half of the slots)
    static constexpr int kWaitSpan = kGroup > kSlots / 2 ? kGroup : kSlots / 2 < 4 ? kSlots / 2 : 4;
    static constexpr size_t kSmem = 1024 + (size_t)kStages * (kStageBytes + kSBytes) + 2 * (size_t)kEBytes +
                                    2 * sizeof(UnitInfo) + (size_t)kMaxTable * sizeof(DescRow) +
                                    (size_t)(2 * kStages + kGroupsInFlight + kSlots + 5) * 8 + 16;
};

struct TcLaunch {
    const TcDesc* descs;   // device array, or null: use `one`
    int n, total_units;
    unsigned int* err;
    SyncArgs sync;         // row-sharded plans: completion signal (sig_epoch 0: none)
    float* partial;        // stream-K (nullptr: one whole tile per unit, CTA c takes units c, c + G, ...)
    unsigned int* tickets;
    long long total_stages;
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

// Instruction descriptor: int32 accumulator, A and B signed int8, both
// K-major, M = 128, N columns.
template <int N>
__host__ __device__ constexpr uint32_t idesc_i8() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kTileRows >> 4) << 24);
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



// tcgen05.wait::ld, then tie the loaded registers to it so that no use of
// them can be scheduled before the wait.
template <int C>
__device__ __forceinline__ void tmem_wait_ld_dep(uint32_t (&a)[C], uint32_t (&b)[C]) {
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < C; i++) asm volatile("" : "+r"(a[i]), "+r"(b[i]));
}

// Block exponents of a unit's 128-row tile reach shared memory in one bulk
// copy when its rows are contiguous whole 16-byte multiples; otherwise the
// epilogue reads them from global memory.

// Index of the GEMM that owns unit u (units are numbered GEMM by GEMM, and
// every role walks its units in increasing order, so the index only grows).
__device__ __forceinline__ int desc_index(const DescRow* tab, int n, int u, int di) {
    while (di + 1 < n && u >= tab[di + 1].unit_begin) di++;
    return di;
}

// Warp-uniform bounded wait (every lane polls; the warp agrees on the result).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
    const bool ok = mbar_wait_sleep(bar, parity, err);
    return __all_sync(0xffffffffu, ok);
}

template <int N, bool DOTS>
__global__ void __launch_bounds__(TcCfg<N>::kThreads, 1) gemm_tc_kernel(const __grid_constant__ TcLaunch p) {
    using C = TcCfg<N>;
    extern __shared__ unsigned char tc_smem_raw[];
    unsigned char* base =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* stages = base;
    unsigned char* sxs = base + (size_t)C::kStages * C::kStageBytes;
    unsigned char* ebuf = sxs + (size_t)C::kStages * C::kSBytes;
    UnitInfo* uring = reinterpret_cast<UnitInfo*>(ebuf + 2 * kEBytes);
    DescRow* tab = reinterpret_cast<DescRow*>(uring + 2);
    uint64_t* full = reinterpret_cast<uint64_t*>(tab + kMaxTable);
    uint64_t* empty = full + C::kStages;
    uint64_t* tfull = empty + C::kStages;          // one per group of blocks in flight
    uint64_t* tempty = tfull + C::kGroupsInFlight;  // one per TMEM slot
    uint64_t* ufull = tempty + C::kSlots;   // unit ring entry published (and its exponent tile landed)
    uint64_t* uempty = ufull + 2;           // unit ring entry consumed by the epilogue
    uint64_t* done = uempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    // the next launch on the stream (a programmatic dependent) may start its
    // CTAs' prologues on the SMs this grid's finished CTAs leave
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // the warp index broadcast from lane 0: the compiler then knows it (and the
    // TMEM addresses built from it) to be warp-uniform
    const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0), lane = threadIdx.x & 31;
    const int n = p.descs ? p.n : 1;
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        const TcDesc* d = p.descs ? p.descs + k : &p.one;
        DescRow r;
        r.unit_begin = d->unit_begin;
        r.n_nt = d->n_nt;
        r.nb = d->nb;
        r.M = d->M;
        r.B = d->B;
        r.ldy = d->ldy;
        r.tile_begin = d->tile_begin;
        r.pad_ = 0;
        r.exps = d->exps;
        r.y = d->y;
        r.dots = d->dots;
        r.peer = d->peer;
        tab[k] = r;
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], C::kEpiWarps * 32);   // every epilogue thread, after the stage's MMAs completed
        }
        for (int g = 0; g < C::kGroupsInFlight; g++) mbar_init(&tfull[g], 1);
        for (int t = 0; t < C::kSlots; t++) mbar_init(&tempty[t], C::kEpiWarps * 32);
        for (int b = 0; b < 2; b++) {
            mbar_init(&ufull[b], 1);
            mbar_init(&uempty[b], C::kEpiWarps);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, C::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int q = warp & 3, chalf = (warp - 2) >> 2;   // TMEM lane quarter, column slice
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Up to here only the (immutable) descriptor table was read; activation
    // planes, outputs and stream-K scratch are touched only once the
    // previous grid on the stream has completed (a no-op for a plain launch).
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t gs = 0;
            int di = 0, i = 0, prefetched = -1;   // prefetched: last GEMM whose successor's maps were warmed
            bool bad = false;
            // Publish unit i (tile `tile` of GEMM di, stages [st0, st1) of its
            // K) to the MMA and epilogue warps, then stream its stages.
            auto unit = [&](int tile, int st0, int st1, int npieces, int cfirst) {
                const DescRow& r = tab[di];
                const TcDesc* d = p.descs ? p.descs + di : &p.one;
                if (p.partial && di != prefetched && p.descs && di + 1 < n) {
                    // stream-K walks the GEMMs in order: warm the next one's TMA maps
                    tma_prefetch_desc(&p.descs[di + 1].tm_w);
                    tma_prefetch_desc(&p.descs[di + 1].tm_x);
                    tma_prefetch_desc(&p.descs[di + 1].tm_s);
                    prefetched = di;
                }
                const int rt = tile / r.n_nt, nt = tile - rt * r.n_nt;
                const int nb = r.nb, j0 = st0 * C::kBPS, nbs = min(nb, st1 * C::kBPS) - j0;
                const int eb = i & 1;
                const int rows = min(kTileRows, r.M - rt * kTileRows);
                const uint32_t ebytes = (uint32_t)rows * (uint32_t)nb;
                const uint8_t* esrc = r.exps + (size_t)rt * kTileRows * nb;
                const bool ebulk = nb <= kExpsMax && (ebytes & 15u) == 0 && (reinterpret_cast<uintptr_t>(esrc) & 15u) == 0;
                UnitInfo info;
                info.exps = ebulk ? ebuf + eb * kEBytes : esrc;
                info.y = r.y;
                info.dots = r.dots;
                info.peer = r.peer;
                info.ldy = r.ldy;
                info.M = r.M;
                info.nb = nb;
                info.B = r.B;
                info.rt = rt;
                info.nt = nt;
                info.ebulk = ebulk;
                info.j0 = j0;
                info.nbs = nbs;
                info.npieces = npieces;
                info.cfirst = cfirst;
                info.pslot = 2 * (int)blockIdx.x + ((int)blockIdx.x == cfirst ? 1 : 0);
                info.tickets = npieces > 1 ? p.tickets + (size_t)(r.tile_begin + tile) * kTcTicketsPerTile : nullptr;
                if (!mbar_wait_sleep(&uempty[eb], ((i >> 1) & 1) ^ 1, p.err)) {
                    bad = true;
                    return;
                }
                uring[eb] = info;   // published by the arrive below (release)
                if (ebulk) {
                    mbar_arrive_expect_tx(&ufull[eb], ebytes);
                    bulk_load(ebuf + eb * kEBytes, esrc, ebytes, &ufull[eb]);
                } else {
                    mbar_arrive_expect_tx(&ufull[eb], 0);
                }
                i++;
                for (int sg = st0; sg < st1; sg++, gs++) {   // sg: stage index along the tile's K
                    const int s = gs % C::kStages;
                    if (!mbar_wait_sleep(&empty[s], ((gs / C::kStages) & 1) ^ 1, p.err)) {
                        bad = true;
                        return;
                    }
                    unsigned char* sm = stages + (size_t)s * C::kStageBytes;
                    mbar_arrive_expect_tx(&full[s], C::kTxBytes);
#pragma unroll
                    for (int bx = 0; bx < C::kBoxes; bx++) {
                        const int x = sg * C::kStageK + bx * kBoxK;
                        tma_load_2d(sm + bx * (kTileRows * kBoxK), &d->tm_w, x, rt * kTileRows, &full[s]);
                        tma_load_3d(sm + C::kWBytes + bx * (2 * N * kBoxK), &d->tm_x, x, nt * N, 0, &full[s]);
                    }
                    tma_load_2d(sxs + (size_t)s * C::kSBytes, &d->tm_s, nt * N, sg * C::kBPS, &full[s]);
                }
            };
            if (p.partial) {
                // stream-K: this CTA's share [sa, sb) of the launch's stages
                const long long S = p.total_stages, G = gridDim.x;
                const long long sa = S * blockIdx.x / G, sb = S * (blockIdx.x + 1) / G;
                auto cta_of = [&](long long x) -> int {   // the CTA whose share holds stage x
                    long long c = x * G / S;
                    while (c + 1 < G && S * (c + 1) / G <= x) c++;
                    while (c > 0 && S * c / G > x) c--;
                    return (int)c;
                };
                long long pos = sa;
                while (pos < sb && !bad) {
                    di = desc_index(tab, n, (int)pos, di);
                    const DescRow& r = tab[di];
                    const int nstt = (r.nb + C::kBPS - 1) / C::kBPS;
                    const int local = (int)(pos - r.unit_begin), tile = local / nstt, st0 = local - tile * nstt;
                    const int st1 = (int)min((long long)nstt, (long long)st0 + (sb - pos));
                    const long long tb = (long long)r.unit_begin + (long long)tile * nstt;
                    const int cf = cta_of(tb), cl = cta_of(tb + nstt - 1);
                    unit(tile, st0, st1, cl - cf + 1, cf);
                    pos += st1 - st0;
                }
            } else {
                for (int u = blockIdx.x; u < p.total_units && !bad; u += gridDim.x) {
                    di = desc_index(tab, n, u, di);
                    const DescRow& r = tab[di];
                    if (u + (int)gridDim.x < p.total_units) {   // warm the TMA maps of this CTA's next unit
                        const int dj = desc_index(tab, n, u + gridDim.x, di);
                        const TcDesc* dn = p.descs ? p.descs + dj : &p.one;
                        tma_prefetch_desc(&dn->tm_w);
                        tma_prefetch_desc(&dn->tm_x);
                        tma_prefetch_desc(&dn->tm_s);
                    }
                    unit(u - r.unit_begin, 0, (r.nb + C::kBPS - 1) / C::kBPS, 1, (int)blockIdx.x);
                }
            }
            if (!bad) {   // end of the sequence: an entry with no blocks
                const int eb = i & 1;
                if (mbar_wait_sleep(&uempty[eb], ((i >> 1) & 1) ^ 1, p.err)) {
                    uring[eb].nbs = 0;
                    mbar_arrive_expect_tx(&ufull[eb], 0);
                }
            }
            // the last loads of every slot have landed unless a consumer quit early
            for (uint32_t k = gs > (uint32_t)C::kStages ? gs - C::kStages : 0; k < gs; k++)
                mbar_wait_sleep(&full[k % C::kStages], (k / C::kStages) & 1, nullptr);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t kId = idesc_i8<2 * N>();
            constexpr int G = C::kGroup;
            uint32_t gs = 0, gb = 0, gg = 0;
            bool bad = false;
            for (int i = 0; !bad; i++) {
                if (!mbar_wait_sleep(&ufull[i & 1], (i >> 1) & 1, p.err)) break;
                const int nb = uring[i & 1].nbs, nst = (nb + C::kBPS - 1) / C::kBPS;   // this unit's blocks
                if (nb == 0) break;   // end of the sequence
                for (int st = 0; st < nst && !bad; st++, gs++) {
                    const int s = gs % C::kStages;
                    if (!mbar_wait_sleep(&full[s], (gs / C::kStages) & 1, p.err)) {
                        bad = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(stages + (size_t)s * C::kStageBytes);
                    for (int h = 0; h < C::kBPS && st * C::kBPS + h < nb; h++, gb++) {
                        const int t = gb % C::kSlots, j = st * C::kBPS + h;
                        if (j % C::kWaitSpan == 0) {   // slots free in order: wait for the span's last one
                            const uint32_t gl = gb + (uint32_t)(min(C::kWaitSpan, nb - j) - 1);
                            if (!mbar_wait_sleep(&tempty[gl % C::kSlots], ((gl / C::kSlots) & 1) ^ 1, p.err)) {
                                bad = true;
                                break;
                            }
                            tc_fence_after();
                        }
                        const int bx = h >> 1;   // which 128-byte box of the stage holds block j
                        const uint64_t da = desc_sw128(a0 + bx * (kTileRows * kBoxK)),
                                       dx = desc_sw128(a0 + C::kWBytes + bx * (2 * N * kBoxK));
#pragma unroll
                        for (int kk = 0; kk < 2; kk++) {
                            const uint64_t off = (uint64_t)(((h & 1) * 64 + kk * 32) >> 4);
                            mma_i8(tmem + (uint32_t)(t * 2 * N), da + off, dx + off, kId,
                                   (uint32_t)kk);   // a block's first step overwrites its slot
                        }
                        if (j % G == G - 1 || j == nb - 1) {   // a group of blocks is complete
                            mma_commit(&tfull[gg % C::kGroupsInFlight]);
                            gg++;
                        }
                    }
                }
            }
            // no MMA may still be writing TMEM when it is released
            mma_commit(done);
            mbar_wait_sleep(done, 0, nullptr);
        }
    } else {
        // ---------------------------------------------------- epilogue
        constexpr int G = C::kGroup;
        uint32_t gs = 0, gb = 0, gg = 0;
        bool bad = false;
        for (int i = 0; !bad; i++) {
            const int eb = i & 1;
            if (!warp_wait(&ufull[eb], (i >> 1) & 1, p.err)) break;
            if (uring[eb].nbs == 0) break;   // end of the sequence
            const UnitInfo info = uring[eb];
            const int M = info.M, nb = info.nbs, B = info.B, nt = info.nt;   // nb: this unit's blocks
            const int r = q * 32 + lane, m = info.rt * kTileRows + r;
            const bool row_ok = m < M;
            const uint8_t* erow = info.exps + (size_t)(row_ok ? r : 0) * info.nb + info.j0;
            const int col0 = chalf * C::kCols;
            float2 acc[C::kCols / 2];
#pragma unroll
            for (int k = 0; k < C::kCols / 2; k++) acc[k] = make_float2(0.0f, 0.0f);

            // Per block: the shared-state address of this thread's first scale
            // (plain shared loads, not generic ones) and the weight scale pair.
            auto scale_base = [&](int j) -> uint32_t {
                const int s = (gs + j / C::kBPS) % C::kStages;
                return smem_u32(sxs) + (uint32_t)(s * C::kSBytes + ((j % C::kBPS) * N + col0) * 4);
            };
            // acc += float(D) * 2^(e-134) * xs over the kCh columns starting at
            // column c; dv holds the exact int32 block dots of block j.
            auto scale_add = [&](const int* dv, int c, int kCh, uint32_t xsb, float2 sm2, int j) {
                float4 x4;   // one 16-byte load serves four columns (two pairs)
#pragma unroll
                for (int k = 0; k < kCh; k += 2) {
                    if ((k & 2) == 0)
                        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                     : "=f"(x4.x), "=f"(x4.y), "=f"(x4.z), "=f"(x4.w)
                                     : "r"(xsb + 4 * (c + k)));
                    const float2 xs2 = (k & 2) ? make_float2(x4.z, x4.w) : make_float2(x4.x, x4.y);
                    const float2 fd = make_float2(__int2float_rn(dv[k]), __int2float_rn(dv[k + 1]));
                    acc[(c + k) / 2] = __ffma2_rn(fd, __fmul2_rn(sm2, xs2), acc[(c + k) / 2]);
                    if constexpr (DOTS) {
#pragma unroll
                        for (int w = 0; w < 2; w++) {
                            const int b = nt * N + col0 + c + k + w;
                            if (row_ok && b < B) info.dots[((size_t)b * M + m) * info.nb + info.j0 + j] = dv[k + w];
                        }
                    }
                }
            };
            auto accumulate = [&](const int* dv, int c, int kCh, int j, uint32_t e) {
                const float sm = exp_scale_ieee(e);
                scale_add(dv, c, kCh, scale_base(j), make_float2(sm, sm), j);
            };
            // this thread is done with a stage's scales after the stage's last
            // block (every epilogue thread arrives: no divergent branch)
            auto release_stage = [&](int j) {
                if (j % C::kBPS == C::kBPS - 1 || j == nb - 1) mbar_arrive(&empty[(gs + j / C::kBPS) % C::kStages]);
            };

            for (int j0 = 0; j0 < nb; j0 += G) {
                const int ng = min(G, nb - j0);
                uint32_t ev[G];
#pragma unroll
                for (int g = 0; g < G; g++) ev[g] = g < ng ? (uint32_t)erow[j0 + g] : 0u;
                // the group's commit covers all of its MMAs (and every earlier one)
                if (!warp_wait(&tfull[gg % C::kGroupsInFlight], (gg / C::kGroupsInFlight) & 1, p.err)) {
                    bad = true;
                    break;
                }
                gg++;
                tc_fence_after();
                if constexpr (G > 1) {
                    uint32_t hv[G][C::kCols], lv[G][C::kCols];
#pragma unroll
                    for (int g = 0; g < G; g++)
                        if (g < ng) {
                            const uint32_t tcol = tmem + lane_base + (uint32_t)(((gb + g) % C::kSlots) * 2 * N + col0);
                            tmem_ld<C::kCols>(tcol, hv[g]);
                            tmem_ld<C::kCols>(tcol + N, lv[g]);
                        }
                    tmem_wait_ld();
#pragma unroll
                    for (int g = 0; g < G; g++)
#pragma unroll
                        for (int k = 0; k < C::kCols; k++) asm volatile("" : "+r"(hv[g][k]), "+r"(lv[g][k]));
                    int dv[G][C::kCols];
#pragma unroll
                    for (int g = 0; g < G; g++)
#pragma unroll
                        for (int k = 0; k < C::kCols; k++) dv[g][k] = (int)hv[g][k] * 256 + (int)lv[g][k];
                    // the group's slots are free once their dots are in registers
                    tc_fence_before();
                    for (int g = 0; g < ng; g++) mbar_arrive(&tempty[(gb + g) % C::kSlots]);
#pragma unroll
                    for (int g = 0; g < G; g++)
                        if (g < ng) {
                            accumulate(dv[g], 0, C::kCols, j0 + g, ev[g]);
                            release_stage(j0 + g);
                        }
                } else {
                    // Wide tiles: the slot slice is read in pieces (one TMEM load
                    // per plane, then one wait): the whole 16 columns of a thread,
                    // or 8 at a time of 32 (the 96-register budget of an 18-warp
                    // CTA); each piece is reduced to the exact block dots
                    // 256 * Dhi + Dlo and scaled.  Every thread frees the slot as
                    // soon as the last piece is in registers, so the MMAs of a
                    // later block overlap that piece's arithmetic.
                    const uint32_t tcol = tmem + lane_base + (uint32_t)((gb % C::kSlots) * 2 * N + col0);
                    const float sm = exp_scale_ieee(ev[0]);
                    const float2 sm2 = make_float2(sm, sm);
                    const uint32_t xsb = scale_base(j0);
                    constexpr int kPiece = C::kCols <= 16 ? C::kCols : 8;
#pragma unroll
                    for (int c = 0; c < C::kCols; c += kPiece) {
                        int dv[kPiece];
                        {
                            uint32_t hv[kPiece], lv[kPiece];
                            tmem_ld<kPiece>(tcol + c, hv);
                            tmem_ld<kPiece>(tcol + N + c, lv);
                            tmem_wait_ld_dep<kPiece>(hv, lv);
#pragma unroll
                            for (int k = 0; k < kPiece; k++) dv[k] = (int)hv[k] * 256 + (int)lv[k];
                        }
                        if (c + kPiece == C::kCols) {
                            tc_fence_before();
                            mbar_arrive(&tempty[gb % C::kSlots]);
                        }
                        scale_add(dv, c, kPiece, xsb, sm2, j0);
                    }
                    release_stage(j0);
                }
                gb += ng;
            }
            gs += (nb + C::kBPS - 1) / C::kBPS;
            // output stride, peer list and K split, read from the ring entry
            // after the block loop (not held in registers through it)
            const int ldy = uring[eb].ldy;
            const PeerOut* peer = uring[eb].peer;
            const int npieces = uring[eb].npieces, cfirst = uring[eb].cfirst, pslot = uring[eb].pslot;
            unsigned int* tick = uring[eb].tickets;
            __syncwarp();
            if (lane == 0) mbar_arrive(&uempty[eb]);   // unit entry and exponent tile consumed
            if (bad) break;
            if (npieces > 1) {
                // a tile cut between CTAs: publish this piece's sums ([slot][b][row]);
                // the warp that completes the tile's column slice adds the
                // pieces in K order (CTA order)
                const int b0 = nt * N + col0;
                if (row_ok) {
                    float* dst = p.partial + ((size_t)pslot * B + b0) * kTileRows + r;
#pragma unroll
                    for (int k = 0; k < C::kCols; k += 2) {
                        if (b0 + k < B) dst[(size_t)k * kTileRows] = acc[k / 2].x;
                        if (b0 + k + 1 < B) dst[(size_t)(k + 1) * kTileRows] = acc[k / 2].y;
                    }
                }
                __threadfence();
                __syncwarp();
                unsigned int t = 0;
                if (lane == 0) t = atomicAdd(tick + (warp - 2), 1u);
                t = __shfl_sync(0xffffffffu, t, 0);
                if (t != (unsigned int)npieces - 1u) continue;
                __threadfence();
                if (row_ok) {
#pragma unroll
                    for (int k = 0; k < C::kCols; k += 2) {
                        float2 sum = make_float2(0.0f, 0.0f);
                        for (int c2 = 0; c2 < npieces; c2++) {
                            const int slot = 2 * (cfirst + c2) + (c2 == 0 ? 1 : 0);
                            float2 v = acc[k / 2];
                            if (slot != pslot) {
                                const float* src = p.partial + ((size_t)slot * B + b0 + k) * kTileRows + r;
                                v.x = b0 + k < B ? __ldcg(src) : 0.0f;
                                v.y = b0 + k + 1 < B ? __ldcg(src + kTileRows) : 0.0f;
                            }
                            sum = c2 == 0 ? v : __fadd2_rn(sum, v);
                        }
                        acc[k / 2] = sum;
                    }
                }
                if (lane == 0) tick[warp - 2] = 0u;   // the next launch is stream-ordered after this one
            }
            if (row_ok) {
                // destination 0: this GPU's output; then every other rank's
                // copy of the full output (row-sharded plans)
                const int np = peer ? peer->n : 0;
                const int b0 = nt * N + col0;
                for (int q2 = -1; q2 < np; q2++) {
                    float* dst = q2 < 0 ? info.y + m : peer->y[q2] + peer->row_base + m;
                    dst += (size_t)b0 * ldy;
#pragma unroll
                    for (int k = 0; k < C::kCols; k += 2) {
                        if (b0 + k < B) dst[k * ldy] = acc[k / 2].x;
                        if (b0 + k + 1 < B) dst[(k + 1) * ldy] = acc[k / 2].y;
                    }
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
    signal_peers(p.sync);   // row-sharded plans: the last CTA publishes the epoch
}

// ------------------------------------------------------------ quantizer
// One warp per (row, 64-block); lane l quantizes elements 2l and 2l+1 with
// the reference's arithmetic: amax, q = 16384/amax (IEEE division), xq =
// rint(x*q) half-even, xs = amax/16384; zero block when amax <= 1e-20.
__global__ void __launch_bounds__(256) quant_planes_kernel(const float* x, int B, int K, uint8_t* planes,
                                                           float* xs_t, int ldxs, const unsigned int* wait_flags,
                                                           unsigned int wait_epoch, const unsigned int* epoch_base,
                                                           int world, unsigned int* err) {
    // row-sharded: inputs from all ranks
    if (wait_epoch) wait_peer_flags(wait_flags, world, wait_epoch, epoch_base, err);
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
        // xq = 256*hi + lo with lo the low byte read as a signed int8 and
        // hi = (xq - lo) / 256 in [-64, 64]: both planes are signed int8
        const int l0 = (int)(int8_t)(q0 & 0xFF), l1 = (int)(int8_t)(q1 & 0xFF);
        const uint32_t hi = ((uint32_t)((q0 - l0) >> 8) & 0xFFu) | (((uint32_t)((q1 - l1) >> 8) & 0xFFu) << 8);
        const uint32_t lo = ((uint32_t)q0 & 0xFFu) | (((uint32_t)q1 & 0xFFu) << 8);
        *reinterpret_cast<uint16_t*>(planes + off) = (uint16_t)hi;
        *reinterpret_cast<uint16_t*>(planes + (size_t)B * K + off) = (uint16_t)lo;
        if (lane == 0) xs_t[(size_t)kb * ldxs + b] = s;
    }
}

template <int N, bool DOTS>
cudaError_t launch_n(const TcDesc* dev_descs, const TcDesc* one, int n, int total_units, unsigned int* err,
                     cudaStream_t stream, const SyncArgs* sync, const TcStreamK* sk) {
    using C = TcCfg<N>;
    static_assert(C::kSmem <= 232448, "shared memory plan exceeds 227 KB");
    if (cudaError_t e = raise_smem_limit(reinterpret_cast<const void*>(gemm_tc_kernel<N, DOTS>), C::kSmem))
        return e;
    TcLaunch p{};
    p.descs = dev_descs;
    p.n = n;
    p.total_units = total_units;
    p.err = err;
    if (sync) p.sync = *sync;
    if (one) p.one = *one;
    int grid = std::max(1, std::min(total_units, num_sms()));
    if (sk) {
        p.partial = sk->partial;
        p.tickets = sk->tickets;
        p.total_stages = sk->total_stages;
        grid = tc_streamk_grid(sk->total_stages);
    }
    // a programmatic dependent of the previous kernel (its prologue overlaps
    // that grid's tail), except under stream capture
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) return cudaGetLastError();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(C::kThreads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cap == cudaStreamCaptureStatusNone ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<N, DOTS>, p);
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
                  const uint8_t* exps, int M, int K, int B, int32_t* dots, int ldy) {
    if (!d || !y || !planes || !xs_t || !mant || !exps || M <= 0 || K <= 0 || K % 64 || B <= 0) return false;
    if (ldy == 0) ldy = M;
    if (ldy < M) return false;
    if (ldxs < B || ldxs % 4) return false;
    if ((reinterpret_cast<uintptr_t>(planes) | reinterpret_cast<uintptr_t>(xs_t) |
         reinterpret_cast<uintptr_t>(mant)) & 15)
        return false;
    const int N = tc_tile_n(B);
    *d = TcDesc{};
    {   // weights: [M][K] bytes, box 128 B x 128 rows
        const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
        const uint64_t str[1] = {(uint64_t)K};
        const uint32_t box[2] = {(uint32_t)kBoxK, (uint32_t)kTileRows};
        if (!encode_tmap(&d->tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, mant, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
            return false;
    }
    {   // activation planes: [2][B][K] bytes, box 128 B x N rows x 2 planes
        const uint64_t dims[3] = {(uint64_t)K, (uint64_t)B, 2};
        const uint64_t str[2] = {(uint64_t)K, (uint64_t)B * (uint64_t)K};
        const uint32_t box[3] = {(uint32_t)kBoxK, (uint32_t)N, 2};
        if (!encode_tmap(&d->tm_x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, planes, dims, str, box,
                         CU_TENSOR_MAP_SWIZZLE_128B))
            return false;
    }
    {   // scales: [nb][ldxs] f32, box N columns x (blocks per stage)
        const uint64_t dims[2] = {(uint64_t)B, (uint64_t)(K / 64)};
        const uint64_t str[1] = {(uint64_t)ldxs * 4};
        const uint32_t box[2] = {(uint32_t)N, (uint32_t)tc_blocks_per_stage(N)};
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
    d->ldy = ldy;
    return true;
}

int tc_units(const TcDesc& d) { return ((d.M + kTileRows - 1) / kTileRows) * d.n_nt; }

int tc_stages(const TcDesc& d) {
    const int bps = tc_blocks_per_stage(tc_tile_n(d.B));
    return tc_units(d) * ((d.nb + bps - 1) / bps);
}

int tc_streamk_grid(int total_stages) { return std::max(1, std::min(total_stages, num_sms())); }

bool tc_prefer_streamk(int tiles) { return tiles < 8 * num_sms(); }

template <bool DOTS>
static cudaError_t launch_b(const TcDesc* dev_descs, const TcDesc* one, int n, int total_units, int B, unsigned int* err,
                     cudaStream_t stream, const SyncArgs* sync, const TcStreamK* sk) {
    switch (tc_tile_n(B)) {
        case 8: return launch_n<8, DOTS>(dev_descs, one, n, total_units, err, stream, sync, sk);
        case 16: return launch_n<16, DOTS>(dev_descs, one, n, total_units, err, stream, sync, sk);
        case 32: return launch_n<32, DOTS>(dev_descs, one, n, total_units, err, stream, sync, sk);
        case 64: return launch_n<64, DOTS>(dev_descs, one, n, total_units, err, stream, sync, sk);
        default: return launch_n<128, DOTS>(dev_descs, one, n, total_units, err, stream, sync, sk);
    }
}

cudaError_t launch_gemm_tc(const TcDesc* dev_descs, const TcDesc* one, int n, int total_units, int B, bool dots,
                           unsigned int* err, cudaStream_t stream, const SyncArgs* sync, const TcStreamK* sk) {
    if (sync && !sync_args_ok(*sync)) return cudaErrorInvalidValue;
    if (total_units <= 0) return cudaSuccess;
    if (n < 1 || n > kTcMaxDescs || (!dev_descs && !one)) return cudaErrorInvalidValue;
    if (sk && (!sk->partial || !sk->tickets || sk->total_stages <= 0)) return cudaErrorInvalidValue;
    return dots ? launch_b<true>(dev_descs, one, n, total_units, B, err, stream, sync, sk)
                : launch_b<false>(dev_descs, one, n, total_units, B, err, stream, sync, sk);
}

cudaError_t launch_quant_planes(const float* x, int B, int K, void* planes, float* xs_t, int ldxs,
                                cudaStream_t stream, const SyncArgs* sync, unsigned int* err) {
    if (sync && !sync_args_ok(*sync)) return cudaErrorInvalidValue;
    const long long total = (long long)B * (K / 64);
    if (total <= 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((total + 7) / 8, (long long)num_sms() * 16);
    quant_planes_kernel<<<grid, 256, 0, stream>>>(x, B, K, static_cast<uint8_t*>(planes), xs_t, ldxs,
                                                  sync ? sync->wait_flags : nullptr, sync ? sync->wait_epoch : 0u,
                                                  sync ? sync->epoch_base : nullptr, sync ? sync->world : 1, err);
    return cudaGetLastError();
}

}  // namespace qb
