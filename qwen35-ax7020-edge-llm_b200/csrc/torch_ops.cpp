// torch_ops.cpp -- the device-level API as PyTorch operators (torch.ops.qwen_b200.*).
//
// Each operator takes CUDA tensors, runs on the tensor's device and the
// current CUDA stream, and raises a c10::Error carrying
// qwen_b200_last_error() when the kernel library refuses or fails.  It is a
// thin layer over the C ABI of libqwen_kernels_b200.so (include/qwen_b200.h):
// every operator calls one entry point, so the arithmetic is exactly that of
// the drop-in exports -- the reference NEON build's for the exact GEMV
// (04-板载脚本与工具/qwen_kernels_opt.c:182-308), its lm_head order and
// selection rules (:401-506, qwen_sampling.c:283-353) and its sampler
// (qwen_sampling.c:411-529).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <string>
#include <tuple>

#include "qwen_b200.h"

namespace {

void* stream_of(const at::Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

void ok(int rc, const char* what) {
    TORCH_CHECK(rc == QB_OK, "qwen_b200.", what, " failed (", rc, "): ", qwen_b200_last_error());
}

at::Tensor need(const at::Tensor& t, at::ScalarType dt, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.scalar_type() == dt, name, " must be ", dt, ", got ", t.scalar_type());
    return t.contiguous();
}

// (mant int8 [M, K], exps uint8 [M, K/64]) -> M, K
std::pair<int, int> weight_shape(const at::Tensor& mant, const at::Tensor& exps) {
    TORCH_CHECK(mant.dim() == 2, "mant must be [M, K]");
    const int64_t M = mant.size(0), K = mant.size(1);
    TORCH_CHECK(K > 0 && K % 64 == 0, "K must be a positive multiple of 64");
    TORCH_CHECK(exps.numel() >= M * (K / 64), "exps must hold M * K / 64 block exponents");
    TORCH_CHECK(mant.device() == exps.device(), "mant and exps must be on one device");
    return {(int)M, (int)K};
}

enum Mode { kExact, kFast, kRtl };

Mode parse_mode(const std::string& mode) {
    if (mode == "exact") return kExact;
    if (mode == "fast") return kFast;
    if (mode == "rtl20") return kRtl;
    TORCH_CHECK(false, "mode must be 'exact', 'fast' or 'rtl20', got '", mode, "'");
    return kExact;
}

// quant_x_blocks (qwen_kernels_opt.c:182-205): x [..., K] -> (xq int16, xs fp32 [..., K/64]).
std::tuple<at::Tensor, at::Tensor> op_quant_block64(const at::Tensor& x_) {
    const at::Tensor x = need(x_, at::kFloat, "x");
    c10::cuda::CUDAGuard g(x.device());
    const int64_t K = x.size(-1);
    TORCH_CHECK(K > 0 && K % 64 == 0, "K must be a positive multiple of 64");
    const int64_t B = x.numel() / K;
    at::Tensor xq = at::empty(x.sizes(), x.options().dtype(at::kShort));
    auto s = x.sizes().vec();
    s.back() = K / 64;
    at::Tensor xs = at::empty(s, x.options());
    ok(qwen_b200_quant_dev(x.data_ptr<float>(), (int)B, (int)K, xq.data_ptr<int16_t>(), xs.data_ptr<float>(),
                           stream_of(x)),
       "quant_block64");
    return {xq, xs};
}

// bfp8_gemv (qwen_kernels_opt.c:207-326) of x [K] or [B, K]: fp32 y [.., M]
// (exact, fast) or int32 floor(y * 2^20) words (rtl20, the gemv_core
// dequant mode, 02-RTL与仿真/gemv_core.v:299-534).
at::Tensor op_bfp8_gemv(const at::Tensor& x_, const at::Tensor& mant_, const at::Tensor& exps_, const std::string& mode) {
    const Mode md = parse_mode(mode);
    const at::Tensor x = need(x_, at::kFloat, "x");
    const at::Tensor mant = need(mant_, at::kChar, "mant");
    const at::Tensor exps = need(exps_, at::kByte, "exps");
    c10::cuda::CUDAGuard g(x.device());
    auto [M, K] = weight_shape(mant, exps);
    TORCH_CHECK(x.size(-1) == K, "x must end in K = ", K);
    TORCH_CHECK(md != kFast || x.dim() == 1, "mode 'fast' takes one activation vector");
    const int64_t B = x.numel() / K;
    auto shape = x.sizes().vec();
    shape.back() = M;
    at::Tensor y = at::empty(shape, x.options().dtype(md == kRtl ? at::kInt : at::kFloat));
    void* st = stream_of(x);
    for (int64_t b = 0; b < B; b++) {
        const float* xb = x.data_ptr<float>() + b * K;
        if (md == kRtl) {
            ok(qwen_b200_gemv_rtl20_dev(y.data_ptr<int32_t>() + b * M, xb, nullptr, nullptr, mant.data_ptr<int8_t>(),
                                        exps.data_ptr<uint8_t>(), M, K, nullptr, st),
               "bfp8_gemv");
        } else if (md == kFast) {
            ok(qwen_b200_gemv_fast_dev(y.data_ptr<float>(), xb, mant.data_ptr<int8_t>(), exps.data_ptr<uint8_t>(), M,
                                       K, st),
               "bfp8_gemv");
        } else {
            ok(qwen_b200_gemv_dev(y.data_ptr<float>() + b * M, xb, mant.data_ptr<int8_t>(), exps.data_ptr<uint8_t>(),
                                  M, K, st),
               "bfp8_gemv");
        }
    }
    return y;
}

// The same from an already quantized activation xq int16 [K], xs fp32 [K/64]
// (mode exact or rtl20).
at::Tensor op_bfp8_gemv_q(const at::Tensor& xq_, const at::Tensor& xs_, const at::Tensor& mant_, const at::Tensor& exps_,
                       const std::string& mode) {
    const Mode md = parse_mode(mode);
    TORCH_CHECK(md != kFast, "bfp8_gemv_q: mode 'exact' or 'rtl20'");
    const at::Tensor xq = need(xq_, at::kShort, "xq");
    const at::Tensor xs = need(xs_, at::kFloat, "xs");
    const at::Tensor mant = need(mant_, at::kChar, "mant");
    const at::Tensor exps = need(exps_, at::kByte, "exps");
    c10::cuda::CUDAGuard g(xq.device());
    auto [M, K] = weight_shape(mant, exps);
    TORCH_CHECK(xq.numel() == K && xs.numel() == K / 64, "xq must hold K and xs K / 64 values");
    at::Tensor y = at::empty({M}, xq.options().dtype(md == kRtl ? at::kInt : at::kFloat));
    if (md == kRtl)
        ok(qwen_b200_gemv_rtl20_dev(y.data_ptr<int32_t>(), nullptr, xq.data_ptr<int16_t>(), xs.data_ptr<float>(),
                                    mant.data_ptr<int8_t>(), exps.data_ptr<uint8_t>(), M, K, nullptr, stream_of(xq)),
           "bfp8_gemv_q");
    else
        ok(qwen_b200_gemv_q_dev(y.data_ptr<float>(), xq.data_ptr<int16_t>(), xs.data_ptr<float>(),
                                mant.data_ptr<int8_t>(), exps.data_ptr<uint8_t>(), M, K, stream_of(xq)),
           "bfp8_gemv_q");
    return y;
}

using LmOut = std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor>;

LmOut lm_outputs(const at::Tensor& like, int64_t kk) {
    auto i = like.options().dtype(at::kInt);
    return {at::zeros({1}, i), at::zeros({std::max<int64_t>(kk, 1)}, i),
            at::zeros({std::max<int64_t>(kk, 1)}, like.options().dtype(at::kFloat)), at::zeros({1}, i)};
}

// lm_head_argmax / lm_head_topk over a bf16 table (qwen_kernels_opt.c:401-506,
// qwen_sampling.c:283-353): (argmax id [1], ids [k], scores [k], n [1]).
LmOut op_lm_head_bf16(const at::Tensor& h_, const at::Tensor& E_, int64_t k) {
    const at::Tensor h = need(h_, at::kFloat, "h");
    at::Tensor E = E_;
    if (E.scalar_type() == at::kBFloat16) E = E.view(at::kShort);
    TORCH_CHECK(E.is_cuda() && E.scalar_type() == at::kShort && E.dim() == 2,
                "E must be a CUDA [vocab, hidden] table of bf16 bits");
    E = E.contiguous();
    c10::cuda::CUDAGuard g(h.device());
    const int64_t V = E.size(0), H = E.size(1);
    TORCH_CHECK(h.numel() == H, "h must hold hidden = ", H, " values");
    LmOut r = lm_outputs(h, std::min(k, V));
    ok(qwen_b200_lm_head_bf16_dev(h.data_ptr<float>(), reinterpret_cast<const uint16_t*>(E.data_ptr<int16_t>()),
                                  (int)V, (int)H, (int)k, std::get<0>(r).data_ptr<int>(), std::get<1>(r).data_ptr<int>(),
                                  std::get<2>(r).data_ptr<float>(), std::get<3>(r).data_ptr<int>(), stream_of(h)),
       "lm_head_bf16");
    return r;
}

// The BFP8 lm_head: exact bfp8_gemv scores fused with argmax and top-k.
LmOut op_lm_head_bfp8(const at::Tensor& h_, const at::Tensor& mant_, const at::Tensor& exps_, int64_t k) {
    const at::Tensor h = need(h_, at::kFloat, "h");
    const at::Tensor mant = need(mant_, at::kChar, "mant");
    const at::Tensor exps = need(exps_, at::kByte, "exps");
    c10::cuda::CUDAGuard g(h.device());
    auto [V, H] = weight_shape(mant, exps);
    TORCH_CHECK(h.numel() == H, "h must hold hidden = ", H, " values");
    LmOut r = lm_outputs(h, std::min<int64_t>(k, V));
    ok(qwen_b200_lm_head_bfp8_dev(h.data_ptr<float>(), mant.data_ptr<int8_t>(), exps.data_ptr<uint8_t>(), V, H,
                                  (int)k, std::get<0>(r).data_ptr<int>(), std::get<1>(r).data_ptr<int>(),
                                  std::get<2>(r).data_ptr<float>(), std::get<3>(r).data_ptr<int>(), stream_of(h)),
       "lm_head_bfp8");
    return r;
}

// x [B, K] fp32 -> (planes int8 [2, B, K], xs_t fp32 [K/64, ldxs]): the
// batched path's activation (xq = 256 * hi + lo, the reference quantizer).
std::tuple<at::Tensor, at::Tensor> op_quant_planes(const at::Tensor& x_) {
    const at::Tensor x = need(x_, at::kFloat, "x");
    TORCH_CHECK(x.dim() == 2, "x must be [B, K]");
    c10::cuda::CUDAGuard g(x.device());
    const int64_t B = x.size(0), K = x.size(1);
    TORCH_CHECK(K > 0 && K % 64 == 0, "K must be a positive multiple of 64");
    const int64_t ldxs = (B + 3) / 4 * 4;
    at::Tensor planes = at::empty({2, B, K}, x.options().dtype(at::kChar));
    at::Tensor xs_t = at::zeros({K / 64, ldxs}, x.options());
    ok(qwen_b200_quant_planes_dev(x.data_ptr<float>(), (int)B, (int)K, planes.data_ptr<int8_t>(),
                                  xs_t.data_ptr<float>(), (int)ldxs, stream_of(x)),
       "quant_planes");
    return {planes, xs_t};
}

// Batched decode on tcgen05: y fp32 [B, M] from planar activations.
at::Tensor op_bfp8_gemm_tc(const at::Tensor& planes_, const at::Tensor& xs_t_, const at::Tensor& mant_,
                        const at::Tensor& exps_) {
    const at::Tensor planes = need(planes_, at::kChar, "planes");
    const at::Tensor xs_t = need(xs_t_, at::kFloat, "xs_t");
    const at::Tensor mant = need(mant_, at::kChar, "mant");
    const at::Tensor exps = need(exps_, at::kByte, "exps");
    c10::cuda::CUDAGuard g(planes.device());
    auto [M, K] = weight_shape(mant, exps);
    TORCH_CHECK(planes.dim() == 3 && planes.size(0) == 2 && planes.size(2) == K, "planes must be [2, B, K]");
    const int64_t B = planes.size(1);
    TORCH_CHECK(xs_t.dim() == 2 && xs_t.size(0) == K / 64 && xs_t.size(1) >= B, "xs_t must be [K/64, ldxs >= B]");
    at::Tensor y = at::empty({B, M}, planes.options().dtype(at::kFloat));
    ok(qwen_b200_gemm_tc_dev(y.data_ptr<float>(), planes.data_ptr<int8_t>(), xs_t.data_ptr<float>(),
                             (int)xs_t.size(1), mant.data_ptr<int8_t>(), exps.data_ptr<uint8_t>(), M, K, (int)B, nullptr,
                             stream_of(planes)),
       "bfp8_gemm_tc");
    return y;
}

// sample_from_topk (qwen_sampling.c:411-529) on the device over a device
// candidate list of length min(ids.numel(), n[0]); rng_state (int32 [1])
// is updated in place; returns the chosen id (int32 [1]).
at::Tensor op_sample_topk(const at::Tensor& ids_, const at::Tensor& scores_, const at::Tensor& n_, double temperature,
                       int64_t top_k, double top_p, at::Tensor rng_state) {
    const at::Tensor ids = need(ids_, at::kInt, "ids");
    const at::Tensor scores = need(scores_, at::kFloat, "scores");
    const at::Tensor n = need(n_, at::kInt, "n");
    TORCH_CHECK(rng_state.is_cuda() && rng_state.scalar_type() == at::kInt && rng_state.is_contiguous(),
                "rng_state must be a contiguous int32 CUDA tensor (updated in place)");
    c10::cuda::CUDAGuard g(ids.device());
    at::Tensor out = at::empty({1}, ids.options());
    ok(qwen_b200_sample_topk_dev(ids.data_ptr<int>(), scores.data_ptr<float>(), n.data_ptr<int>(), (int)ids.numel(),
                                 (float)temperature, (int)top_k, (float)top_p,
                                 reinterpret_cast<unsigned int*>(rng_state.data_ptr<int>()), out.data_ptr<int>(),
                                 stream_of(ids)),
       "sample_topk");
    return out;
}

// The reference packer's rule on the device (05-主机侧源码/bfp8_packer.py:53-86).
std::tuple<at::Tensor, at::Tensor> op_pack_bfp8(const at::Tensor& w_) {
    const at::Tensor w = need(w_, at::kFloat, "w");
    TORCH_CHECK(w.dim() == 2 && w.size(1) % 64 == 0, "w must be [M, K] with K a multiple of 64");
    c10::cuda::CUDAGuard g(w.device());
    const int64_t M = w.size(0), K = w.size(1);
    at::Tensor mant = at::empty({M, K}, w.options().dtype(at::kChar));
    at::Tensor exps = at::empty({M, K / 64}, w.options().dtype(at::kByte));
    ok(qwen_b200_pack_bfp8_dev(w.data_ptr<float>(), (int)M, (int)K, mant.data_ptr<int8_t>(), exps.data_ptr<uint8_t>(),
                               stream_of(w)),
       "pack_bfp8");
    return {mant, exps};
}

}  // namespace

TORCH_LIBRARY(qwen_b200, m) {
    m.def("quant_block64(Tensor x) -> (Tensor, Tensor)");
    m.def("bfp8_gemv(Tensor x, Tensor mant, Tensor exps, str mode='exact') -> Tensor");
    m.def("bfp8_gemv_q(Tensor xq, Tensor xs, Tensor mant, Tensor exps, str mode='exact') -> Tensor");
    m.def("lm_head_bf16(Tensor h, Tensor E, int k) -> (Tensor, Tensor, Tensor, Tensor)");
    m.def("lm_head_bfp8(Tensor h, Tensor mant, Tensor exps, int k) -> (Tensor, Tensor, Tensor, Tensor)");
    m.def("quant_planes(Tensor x) -> (Tensor, Tensor)");
    m.def("bfp8_gemm_tc(Tensor planes, Tensor xs_t, Tensor mant, Tensor exps) -> Tensor");
    m.def("sample_topk(Tensor ids, Tensor scores, Tensor n, float temperature, int top_k, float top_p, "
          "Tensor(a!) rng_state) -> Tensor");
    m.def("pack_bfp8(Tensor w) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(qwen_b200, CUDA, m) {
    m.impl("quant_block64", &op_quant_block64);
    m.impl("bfp8_gemv", &op_bfp8_gemv);
    m.impl("bfp8_gemv_q", &op_bfp8_gemv_q);
    m.impl("lm_head_bf16", &op_lm_head_bf16);
    m.impl("lm_head_bfp8", &op_lm_head_bfp8);
    m.impl("quant_planes", &op_quant_planes);
    m.impl("bfp8_gemm_tc", &op_bfp8_gemm_tc);
    m.impl("sample_topk", &op_sample_topk);
    m.impl("pack_bfp8", &op_pack_bfp8);
}
