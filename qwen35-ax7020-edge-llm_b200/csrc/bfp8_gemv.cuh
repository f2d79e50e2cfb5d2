// bfp8_gemv.cuh -- host-visible declarations of the BFP8 GEMV launchers.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

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
    int M;
    int K;
    int unit_begin;         // planner: first 32-row work unit of this GEMV
    int pad_;
};

struct LmScratch;

// Work plan of a grouped launch.
struct GemvPlan {
    int n;
    int total_units;
    int kmax;
    size_t act_words;       // 32-bit words of activation scratch the plan needs
};

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
bool gemv_plan(GemvDesc* descs, int n, uint32_t* act, GemvPlan* plan);

// Grouped exact GEMV over a planned, device-resident descriptor array.
// `ctr` is a 2-word device counter pair owned by the plan (zero before the
// first launch; every launch leaves it zero).  `err` (device word, may be
// null) collects kernel error bits.
cudaError_t launch_gemv_list(const GemvDesc* dev_descs, const GemvPlan& plan, unsigned int* ctr,
                             unsigned int* err, cudaStream_t stream);

// One exact GEMV (any M >= 1, K a positive multiple of 64, any alignment).
// `act` is device scratch of gemv_act_words(K) words.
cudaError_t launch_gemv(const GemvDesc& d, uint32_t* act, unsigned int* err, cudaStream_t stream);

// BFP8 lm_head: scores = bfp8_gemv(h), fused argmax (ties -> lowest id, best
// must beat -1e30) and top-k (k <= 1024; score desc, ties ascending id).
// Results land in device memory: out_id[0], out_ids/out_scores[0..n), *out_n.
cudaError_t launch_bfp8_lm_head(const float* h, const int8_t* mant, const uint8_t* exps, int vocab,
                                int hidden, int k, LmScratch* scratch, uint32_t* act, unsigned int* err,
                                int* out_id, int* out_ids, float* out_scores, int* out_n,
                                cudaStream_t stream);

// Standalone block-64 quantizer: x [B][K] -> xq [B][K] (natural order), xs [B][K/64].
cudaError_t launch_quant_block64(const float* x, int B, int K, int16_t* xq, float* xs,
                                 cudaStream_t stream);

int num_sms();

}  // namespace qb
