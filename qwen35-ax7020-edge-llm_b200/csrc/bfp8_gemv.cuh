// bfp8_gemv.cuh -- host-visible declarations of the BFP8 GEMV launchers.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "peer.cuh"

namespace qb {

// One BFP8 GEMV.  Weights use the reference's SoA layout: mantissas int8
// [M][K] row-major, then exponents uint8 [M][K/64]
// (05-主机侧源码/bfp8_packer.py:53-86).  The activation is either fp32 `x`
// (quantized by the reference block-64 rule) or, when x == nullptr, an
// already quantized int16 `xq` [K] with scales `xs` [K/64].
struct alignas(64) GemvDesc {
    CUtensorMap tmap;       // planner: 2D map of `mant` (M rows x K bytes, 32 x 128-byte boxes)
    const int8_t* mant;
    const uint8_t* exps;
    const float* x;
    const int16_t* xq;
    const float* xs;
    float* y;
    uint32_t* xpairs;       // planner: where the paired int16 activation goes (K/2 words)
    float* xscale;          // planner: its block scales (K/64)
    float* partial;         // planner (fast mode): nseg x M fp32 segment sums
    unsigned int* tickets;  // planner (fast mode): one zero-initialised counter per 32-row group
    int M;
    int K;
    int unit_begin;         // planner: first work unit of this GEMV
    int nseg;               // planner: K segments per row group (1 = whole rows)
    int seg_stages;         // planner: 256-byte columns per segment
    int pad_;
    const PeerOut* peer;    // optional (device memory): also store rows into every rank's vector
};

struct LmScratch;

// Work plan of a grouped launch.
struct GemvPlan {
    int n;
    int total_units;
    int kmax;
    bool fast;
    size_t act_words;       // 32-bit words of scratch the plan needs (zeroed once before first use)
};

// Arithmetic of a launch.
//   exact: the reference NEON float order, bit for bit (one warp streams
//          each 32-row group end to end).
//   fast:  per block one int32 dot, acc = fma(float(dot), 2^(e-134)*xs, acc)
//          within a K segment, segments summed in order; rows may be split
//          into K segments so that short, deep matrices fill the GPU.
//          Deterministic; |y - exact| <= 1e-5 * sum_b |term_b|.
//   rtl20: the FPGA dequant datapath (02-RTL与仿真/gemv_core.v:299-534):
//          per row one int32 word floor(y * 2^20) from a saturating 64-bit
//          fixed-point sum (stored in y's 32 bits), sticky flags (bit 0 a
//          term or sum saturated, bit 1 the output clamped) ORed into a
//          device word.  Integer only, bit-exact.
enum GemvMode { kExact = 0, kFast = 1, kRtl20 = 2 };

// Activation scratch (32-bit words) one GEMV of depth K needs.
size_t gemv_act_words(int K);

// Fill tmap / xpairs / xscale / unit_begin of `descs` (host array) for a
// grouped launch, placing every activation in `act` (device buffer of
// plan->act_words words; may be null to only size the plan).  Descriptors
// are reordered largest K first (they are independent, and the scheduler
// hands out the biggest units first).  Descriptors with M == 0 must not be
// passed; at most 160 descriptors.  Returns false if a shape is not served
// by the fast kernel (K % 512 != 0 or misaligned pointers) or a tensor map
// cannot be encoded.
// Fast mode keeps one counter per split row group: in `act` after the
// segment sums, or, when `tickets` is given, in that separate zeroed buffer
// of tickets_cap words (for scratch that other launches also write).
// fixed_seg_stages > 0 (fast mode): cut every row's K into segments of that
// many 256-byte stages, independent of the rows this GPU holds.
bool gemv_plan(GemvDesc* descs, int n, uint32_t* act, GemvPlan* plan, int mode = kExact,
               size_t act_cap_words = 0, unsigned int* tickets = nullptr, size_t tickets_cap = 0,
               int fixed_seg_stages = 0);

// Grouped exact GEMV over a planned, device-resident descriptor array.
// `ctr` is a 2-word device counter pair owned by the plan (zero before the
// first launch; every launch leaves it zero).  `err` (device word, may be
// null) collects kernel error bits.
cudaError_t launch_gemv_list(const GemvDesc* dev_descs, const GemvPlan& plan, unsigned int* ctr,
                             unsigned int* err, cudaStream_t stream,
                             const SyncArgs* sync = nullptr);

// One exact (or, mode kRtl20, RTL dequant) GEMV: any M >= 1, K a positive
// multiple of 64, any alignment.  `act` is device scratch of
// gemv_act_words(K) words; `rtl_flags` (device word, may be null) collects
// the kRtl20 flags.
cudaError_t launch_gemv(const GemvDesc& d, uint32_t* act, unsigned int* err, cudaStream_t stream,
                        int mode = kExact, unsigned int* rtl_flags = nullptr);

// One exact GEMV of rmsnorm(x, norm_w, eps) (the reference's NEON-order
// rmsnorm, then its quantizer and GEMV), in one launch: every CTA normalizes
// and quantizes x itself.  K <= 6144, a multiple of 512; aligned pointers.
// With `res`, x + res (the reference's add_residual) is normalized instead
// and also stored to x_out, which must not overlap x or res.
cudaError_t launch_rmsnorm_gemv(const GemvDesc& d, const float* norm_w, float eps, uint32_t* act, unsigned int* err,
                               cudaStream_t stream, const float* res = nullptr, float* x_out = nullptr);

// Two exact GEMVs of the same rmsnorm(x) (or of x + res, stored to x_out) in
// one launch -- d0 and d1 share x and K (a layer's qkv and z projections, an
// MLP's gate and up); the same conditions as launch_rmsnorm_gemv.  With
// norm_out, the normalized vector itself (the reference's rmsnorm output) is
// stored there too, 8-byte aligned.
cudaError_t launch_rmsnorm_gemv2(const GemvDesc& d0, const GemvDesc& d1, const float* norm_w, float eps,
                                uint32_t* act, unsigned int* err, cudaStream_t stream, const float* res = nullptr,
                                float* x_out = nullptr, float* norm_out = nullptr);

// One exact GEMV of swiglu(gate, up) (the reference's NEON swiglu, then its
// quantizer and GEMV; d.x holds the gate projection) in one launch: every
// CTA applies swiglu and quantizes itself.  K <= 6144, a multiple of 512;
// aligned pointers (up 8-byte).  With `residual`, d.y is the residual stream
// and receives y += result (the reference's add_residual after the down
// projection), in place, instead of the result.
cudaError_t launch_swiglu_gemv(const GemvDesc& d, const float* up, uint32_t* act, unsigned int* err,
                               cudaStream_t stream, bool residual = false);

// Fast-mode single GEMV (K % 512 == 0, aligned pointers); `act` holds
// act_cap_words words of scratch, `tickets` tickets_cap zeroed counters
// (every launch leaves them zero).
cudaError_t launch_gemv_fast(const GemvDesc& d, uint32_t* act, size_t act_cap_words, unsigned int* tickets,
                             size_t tickets_cap, unsigned int* err, cudaStream_t stream);

// BFP8 lm_head: scores = bfp8_gemv(h), fused argmax (ties -> lowest id, best
// must beat -1e30) and top-k (k <= 1024; score desc, ties ascending id).
// Results land in device memory: out_id[0], out_ids/out_scores[0..n), *out_n.
// `ctr` is a zeroed pair of counters the launch may use for dynamic unit
// claims (k <= 64); the kernel leaves it zero.
cudaError_t launch_bfp8_lm_head(const float* h, const int8_t* mant, const uint8_t* exps, int vocab,
                                int hidden, int k, LmScratch* scratch, uint32_t* act, unsigned int* ctr,
                                unsigned int* err, int* out_id, int* out_ids, float* out_scores, int* out_n,
                                cudaStream_t stream);

// Standalone block-64 quantizer: x [B][K] -> xq [B][K] (natural order), xs [B][K/64].
cudaError_t launch_quant_block64(const float* x, int B, int K, int16_t* xq, float* xs,
                                 cudaStream_t stream);

// Shard-local SwiGLU + quantizer of a row-sharded MLP layer: elements
// [col0, col0 + n) of every batch row b of gate / up (row stride ld_in) ->
// swiglu (the reference's NEON build) -> block-64 quantization, stored into
// each dst: planar == 0 (B == 1): the quantized record xq int16 [K] followed
// by xs fp32 [K/64]; planar == 1: planes int8 [2][B][K] (hi, lo) followed by
// xs_t fp32 [K/64][ldxs].  With sync->sig_epoch the last CTA publishes it to
// every rank and waits for every rank's (sync->wait_flags, bounded).
cudaError_t launch_swiglu_quant(const float* gate, const float* up, int B, int n, int ld_in, int col0, int K,
                                int planar, int ldxs, void* const* dst, int ndst, const SyncArgs* sync,
                                unsigned int* err, cudaStream_t stream);

// Enqueue *base += n (mod 2^32): moves the epoch counter of row-sharded
// launches (SyncArgs::epoch_base) past one step's epochs.
cudaError_t launch_epoch_advance(unsigned int* base, unsigned int n, cudaStream_t stream);

// add_residual (NEON build): x[i] += res[i], flushed over groups of four.
cudaError_t launch_add_residual(float* x, const float* res, int n, cudaStream_t stream);

int num_sms();

}  // namespace qb
