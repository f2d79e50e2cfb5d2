// capi.cu -- C ABI of libqwen_kernels_b200.so (declared in include/qwen_b200.h).
//
// The drop-in entry points keep the reference's signatures and host-pointer
// conventions (04-板载脚本与工具/qwen_kernels_opt.c, qwen_sampling.c) and run
// the work on the device; the _dev entry points take device pointers and a
// stream and are what the PyTorch operators and the benchmarks call.
#include "api_error.cuh"
#include "bfp8_gemm_tc.cuh"
#include "bfp8_gemv.cuh"
#include "common.cuh"
#include "gdn.cuh"
#include "lm_head.cuh"
#include "sample.cuh"
#include "topk.cuh"

#include "qwen_b200.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include <unistd.h>

namespace {
thread_local std::string g_err;
}  // namespace

namespace qb {
int api_fail(int code, const char* what, cudaError_t e) {
    char buf[256];
    if (e != cudaSuccess)
        snprintf(buf, sizeof buf, "%s: %s", what, cudaGetErrorString(e));
    else
        snprintf(buf, sizeof buf, "%s", what);
    g_err = buf;
    return code;
}
}  // namespace qb

namespace {

int fail(int code, const char* what, cudaError_t e = cudaSuccess) { return qb::api_fail(code, what, e); }

// ---------------------------------------------------------------- profiler
enum { PF_GEMV = 0, PF_ARGMAX, PF_TOPK, PF_SAMPLE, PF_UPLOAD, PF_MLP, PF_LINEAR, PF_TOKEN, PF_CALLBACK, PF_N };
const char* kProfNames[PF_N] = {"bfp8_gemv",   "lm_head_argmax",       "lm_head_topk",    "sample_from_topk",
                                "weight_upload", "forward_mlp",        "forward_linear_layer", "forward_token_c",
                                "full_attn_callback"};
int g_prof_on = 0;
double g_prof_ms[PF_N];

struct ProfScope {
    int slot;
    std::chrono::steady_clock::time_point t0;
    explicit ProfScope(int s) : slot(s), t0(std::chrono::steady_clock::now()) {}
    ~ProfScope() {
        if (g_prof_on)
            g_prof_ms[slot] +=
                std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    }
};

// ---------------------------------------------------------------- device context
struct Ctx {
    bool ready = false;
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaStream_t copy = nullptr;   // state copies of the layer loop, beside the compute stream
    qb::LmScratch* scratch = nullptr;
    // pinned host staging + device buffers for the drop-in calls
    void* h_in = nullptr;
    size_t h_in_cap = 0;
    void* h_out = nullptr;
    size_t h_out_cap = 0;
    void* d_in = nullptr;
    size_t d_in_cap = 0;
    void* d_out = nullptr;
    size_t d_out_cap = 0;
    int* d_res = nullptr;   // [0] id, [1] n
    float* d_scores = nullptr;
    size_t d_scores_cap = 0;
};
Ctx g_ctx;
std::mutex g_mu;   // serialises the drop-in entry points

int ensure_ctx() {
    if (g_ctx.ready) return QB_OK;
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess || ndev <= 0) return fail(QB_ENODEV, "no CUDA device", e);
    int dev = 0;
    if (const char* s = getenv("QWEN_B200_DEVICE")) dev = atoi(s);
    if (dev < 0 || dev >= ndev) dev = 0;
    if ((e = cudaSetDevice(dev)) != cudaSuccess) return fail(QB_ECUDA, "cudaSetDevice", e);
    if ((e = cudaStreamCreateWithFlags(&g_ctx.stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaStreamCreateWithFlags(&g_ctx.copy, cudaStreamNonBlocking)) != cudaSuccess)
        return fail(QB_ECUDA, "cudaStreamCreate", e);
    if ((e = cudaMalloc(&g_ctx.scratch, sizeof(qb::LmScratch))) != cudaSuccess)
        return fail(QB_ENOMEM, "scratch alloc", e);
    if ((e = cudaMemset(g_ctx.scratch, 0, sizeof(qb::LmScratch))) != cudaSuccess)
        return fail(QB_ECUDA, "scratch clear", e);
    if ((e = cudaMalloc(&g_ctx.d_res, 4 * sizeof(int))) != cudaSuccess)
        return fail(QB_ENOMEM, "result alloc", e);
    g_ctx.device = dev;
    g_ctx.ready = true;
    return QB_OK;
}

int grow_pinned(void** p, size_t* cap, size_t need) {
    if (*cap >= need) return QB_OK;
    if (*p) cudaFreeHost(*p);
    *p = nullptr;
    *cap = 0;
    cudaError_t e = cudaMallocHost(p, need);
    if (e != cudaSuccess) return fail(QB_ENOMEM, "pinned alloc", e);
    *cap = need;
    return QB_OK;
}
int grow_dev(void** p, size_t* cap, size_t need) {
    if (*cap >= need) return QB_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    cudaError_t e = cudaMalloc(p, need);
    if (e != cudaSuccess) return fail(QB_ENOMEM, "device alloc", e);
    *cap = need;
    return QB_OK;
}

// ---------------------------------------------------------------- weight registry
struct Range {
    const unsigned char* host;
    size_t bytes;
    unsigned char* dev;
};
std::vector<Range> g_ranges;

const void* lookup(const void* p, size_t bytes) {
    const unsigned char* h = static_cast<const unsigned char*>(p);
    for (const Range& r : g_ranges)
        if (h >= r.host && h + bytes <= r.host + r.bytes) return r.dev + (h - r.host);
    return nullptr;
}

int upload_range(const void* host, size_t bytes) {
    ProfScope ps(PF_UPLOAD);
    unsigned char* d = nullptr;
    cudaError_t e = cudaMalloc(&d, bytes ? bytes : 1);
    if (e != cudaSuccess) return fail(QB_ENOMEM, "weight upload alloc", e);
    e = cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(d);
        return fail(QB_ECUDA, "weight upload copy", e);
    }
    g_ranges.push_back({static_cast<const unsigned char*>(host), bytes, d});
    return QB_OK;
}

// Device address of [p, p + bytes), uploading it on first sight.
const void* device_of(const void* p, size_t bytes, int* rc) {
    if (const void* d = lookup(p, bytes)) return d;
    *rc = upload_range(p, bytes);
    return *rc == QB_OK ? lookup(p, bytes) : nullptr;
}

// ---------------------------------------------------------------- stack plans
struct StackPlan {
    qb::GemvPlan plan;
    qb::GemvDesc* dev_descs = nullptr;
    uint32_t* act = nullptr;          // paired activations of every GEMV
    unsigned int* ctr = nullptr;      // unit counter pair of the dynamic scheduler
    qb::PeerOut* peers = nullptr;     // row-sharded plans: where each GEMV's rows also go
    unsigned int* sig_ticket = nullptr;   // row-sharded plans: grid ticket of the completion signal
    bool live = false;
};
std::vector<StackPlan> g_plans;

// Grouped batched tensor-core plans: launches of at most qb::kTcMaxDescs
// GEMMs each (deepest first), their descriptors in one device array.
struct TcLaunchPart {
    int first, n, total_units;
    int total_stages;   // stream-K launches (0: whole-tile units): unit_begin of their descriptors = first stage
};
struct TcPlan {
    qb::TcDesc* dev_descs = nullptr;
    std::vector<TcLaunchPart> parts;
    int B = 0;
    float* partial = nullptr;           // stream-K piece sums (2 slots per CTA)
    unsigned int* sk_tickets = nullptr; // stream-K counters (kTcTicketsPerTile per tile, left zero)
    qb::PeerOut* peers = nullptr;         // row-sharded plans: where each GEMM's rows also go
    unsigned int* sig_ticket = nullptr;   // row-sharded plans: grid ticket of the completion signal
    bool live = false;
};
std::vector<TcPlan> g_tc_plans;

int check_gemv_args(const void* y, const void* x, const void* mant, const void* exps, int M, int K) {
    if (!y || !x || !mant || !exps) return fail(QB_EINVAL, "null pointer");
    if (M < 0 || K <= 0 || K % 64) return fail(QB_EINVAL, "M must be >= 0 and K a positive multiple of 64");
    return QB_OK;
}

// ---------------------------------------------------------------- sampler
// xorshift32 (Marsaglia 13/17/5) with the zero state remapped to 0x9E3779B9,
// the generator the reference sampler uses (qwen_sampling.c:360-373).
unsigned int xs32_next(unsigned int* st) {
    unsigned int x = *st;
    if (x == 0u) x = 0x9E3779B9u;
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    *st = x;
    return x;
}

struct Cand {
    int id;
    float score;
};

// Per-device state of the _dev entry points: lm_head scratch and the
// device error word the kernels report bounded-wait timeouts into.
struct DevState {
    qb::LmScratch* scratch = nullptr;
    unsigned int* err = nullptr;
    uint32_t* act = nullptr;       // paired-activation scratch of single-GEMV launches
    unsigned int* tickets = nullptr;   // zeroed split-K counters of fast single-GEMV launches
    unsigned int* lm_ctr = nullptr;    // zeroed unit-claim counters of the BFP8 lm_head
    const unsigned int* epoch_base = nullptr;   // row-sharded launches: epoch counter (nullptr: absolute epochs)
};
constexpr int kMaxDevices = 64;
constexpr size_t kTicketWords = 16384;
constexpr size_t kActScratchWords = 128 * 1024;   // serves K <= 253952

int dev_state(DevState** out) {
    static std::mutex mu;
    static DevState per_dev[kMaxDevices];   // fixed: the pointers handed out stay valid
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(QB_ECUDA, "cudaGetDevice", e);
    if (dev < 0 || dev >= kMaxDevices) return fail(QB_ENODEV, "device index beyond 63");
    std::lock_guard<std::mutex> lk(mu);
    DevState& st = per_dev[dev];
    if (!st.scratch) {
        qb::LmScratch* p = nullptr;
        if ((e = cudaMalloc(&p, sizeof(qb::LmScratch))) != cudaSuccess) return fail(QB_ENOMEM, "scratch alloc", e);
        if ((e = cudaMemset(p, 0, sizeof(qb::LmScratch))) != cudaSuccess) return fail(QB_ECUDA, "scratch clear", e);
        unsigned int* w = nullptr;
        if ((e = cudaMalloc(&w, sizeof(unsigned int))) != cudaSuccess) return fail(QB_ENOMEM, "error word alloc", e);
        if ((e = cudaMemset(w, 0, sizeof(unsigned int))) != cudaSuccess) return fail(QB_ECUDA, "error word clear", e);
        uint32_t* a = nullptr;
        if ((e = cudaMalloc(&a, kActScratchWords * 4)) != cudaSuccess) return fail(QB_ENOMEM, "act scratch alloc", e);
        if ((e = cudaMemset(a, 0, kActScratchWords * 4)) != cudaSuccess) return fail(QB_ECUDA, "act scratch clear", e);
        unsigned int* tk = nullptr;
        if ((e = cudaMalloc(&tk, kTicketWords * 4)) != cudaSuccess) return fail(QB_ENOMEM, "ticket alloc", e);
        if ((e = cudaMemset(tk, 0, kTicketWords * 4)) != cudaSuccess) return fail(QB_ECUDA, "ticket clear", e);
        unsigned int* lc = nullptr;
        if ((e = cudaMalloc(&lc, 2 * sizeof(unsigned int))) != cudaSuccess) return fail(QB_ENOMEM, "lm counter alloc", e);
        if ((e = cudaMemset(lc, 0, 2 * sizeof(unsigned int))) != cudaSuccess) return fail(QB_ECUDA, "lm counter clear", e);
        st.scratch = p;
        st.err = w;
        st.act = a;
        st.tickets = tk;
        st.lm_ctr = lc;
    }
    *out = &st;
    return QB_OK;
}

// ---------------------------------------------------------------- layer loop
// The reference's per-token C loop (qwen_kernels_opt.c:938-1049) on the
// device.  Plans carry host pointers; weights and fp32 vectors resolve like
// bfp8_gemv's (a registered range, or an upload on first sight, kept), the
// two mutable Gated-DeltaNet states through StateSlot below.

constexpr int kLoopLayers = 24;      // forward_token_c's layer count (qwen_kernels_opt.c:1028)
constexpr int kLoopVocab = 65536;    // its embedding / lm_head rows (:1020, :1046)
constexpr int kLoopHidden = 1024;    // its hidden size (:1021, :1043)

struct DevGemv {
    const int8_t* m = nullptr;
    const uint8_t* e = nullptr;
    int M = 0, K = 0;
};
struct DevMlp {
    const float* post_ln = nullptr;
    DevGemv gate, up, down;
};
struct DevLinear {
    const float* in_ln = nullptr;
    DevGemv qkv, z, o;
    const float *conv_w = nullptr, *wa = nullptr, *wb = nullptr, *nea = nullptr, *dt = nullptr, *norm_w = nullptr;
    float* conv_s = nullptr;   // host state arrays (mutable)
    float* state = nullptr;
    int heads = 0;
    DevMlp mlp;
};

// Device address of a BFP8 matrix's mantissas and exponents (contiguous SoA
// tensors resolve as one range).
bool resolve_gemv(const int8_t* m, const uint8_t* e, int M, int K, DevGemv* out, int* rc) {
    if (!m || !e || M <= 0 || K <= 0 || K % 64) {
        *rc = fail(QB_EINVAL, "layer plan: null or misshaped BFP8 matrix");
        return false;
    }
    const size_t wb = (size_t)M * K, eb = (size_t)M * (K / 64);
    if (e == reinterpret_cast<const uint8_t*>(m) + wb) {
        const void* d = device_of(m, wb + eb, rc);
        if (!d) return false;
        out->m = static_cast<const int8_t*>(d);
        out->e = static_cast<const uint8_t*>(d) + wb;
    } else {
        out->m = static_cast<const int8_t*>(device_of(m, wb, rc));
        out->e = out->m ? static_cast<const uint8_t*>(device_of(e, eb, rc)) : nullptr;
    }
    out->M = M;
    out->K = K;
    return out->m && out->e;
}

const float* resolve_vec(const float* p, size_t n, int* rc) {
    if (!p) {
        *rc = fail(QB_EINVAL, "layer plan: null vector");
        return nullptr;
    }
    return static_cast<const float*>(device_of(p, n * sizeof(float), rc));
}

// forward_mlp's shapes: hidden H = K_gate = K_up = M_down, F = M_gate = M_up =
// K_down, both multiples of 512 and <= 6144 (the fused rmsnorm / swiglu GEMVs).
int resolve_mlp(const float* post_ln, const int8_t* mg, const uint8_t* eg, int Mg, int Kg, const int8_t* mu,
                const uint8_t* eu, int Mu, int Ku, const int8_t* md, const uint8_t* ed, int Md, int Kd, DevMlp* out) {
    const int H = Kg, F = Mg;
    if (H <= 0 || H % 512 || H > 6144 || Ku != H || Mu != F || Kd != F || Md != H || F <= 0 || F % 512 || F > 6144)
        return fail(QB_EINVAL, "MLP plan: K_gate == K_up == M_down and M_gate == M_up == K_down, multiples of 512, "
                               "<= 6144");
    int rc = QB_OK;
    if (!resolve_gemv(mg, eg, Mg, Kg, &out->gate, &rc) || !resolve_gemv(mu, eu, Mu, Ku, &out->up, &rc) ||
        !resolve_gemv(md, ed, Md, Kd, &out->down, &rc))
        return rc ? rc : fail(QB_EINVAL, "MLP plan: weights");
    if (!(out->post_ln = resolve_vec(post_ln, (size_t)H, &rc))) return rc;
    return QB_OK;
}

int resolve_mlp_plan(const MlpPlanC* p, DevMlp* out) {
    if (!p) return fail(QB_EINVAL, "null MLP plan");
    return resolve_mlp(p->post_ln_w, p->mant_gate, p->exp_gate, p->M_gate, p->K_gate, p->mant_up, p->exp_up, p->M_up,
                       p->K_up, p->mant_down, p->exp_down, p->M_down, p->K_down, out);
}

// forward_linear_layer's shapes (the reference hard-codes 1024 / 6144 / 16 x
// 128): hidden H = K_qkv = K_z = M_o; value width V = M_z = K_o = heads * 128;
// M_qkv = 3 V (q | k | v); the MLP as above.
int resolve_linear_plan(const LinearLayerPlanC* p, DevLinear* out) {
    if (!p) return fail(QB_EINVAL, "null linear-layer plan");
    const int H = p->K_qkv, V = p->M_z;
    if (V <= 0 || V % qb::kGdnHeadDim || p->M_qkv != 3 * V || p->K_z != H || p->K_o != V || p->M_o != H ||
        p->K_gate != H)
        return fail(QB_EINVAL, "linear-layer plan: K_qkv == K_z == M_o == K_gate, M_qkv == 3 M_z, K_o == M_z, "
                               "M_z a multiple of 128");
    if (int rc = resolve_mlp(p->post_ln_w, p->mant_gate, p->exp_gate, p->M_gate, p->K_gate, p->mant_up, p->exp_up,
                             p->M_up, p->K_up, p->mant_down, p->exp_down, p->M_down, p->K_down, &out->mlp))
        return rc;
    int rc = QB_OK;
    const int heads = V / qb::kGdnHeadDim;
    if (!resolve_gemv(p->mant_qkv, p->exp_qkv, p->M_qkv, p->K_qkv, &out->qkv, &rc) ||
        !resolve_gemv(p->mant_z, p->exp_z, p->M_z, p->K_z, &out->z, &rc) ||
        !resolve_gemv(p->mant_o, p->exp_o, p->M_o, p->K_o, &out->o, &rc))
        return rc ? rc : fail(QB_EINVAL, "linear-layer plan: weights");
    if (!(out->in_ln = resolve_vec(p->in_ln_w, (size_t)H, &rc)) ||
        !(out->conv_w = resolve_vec(p->conv_w, 4 * (size_t)p->M_qkv, &rc)) ||
        !(out->wa = resolve_vec(p->wa, (size_t)heads * H, &rc)) ||
        !(out->wb = resolve_vec(p->wb, (size_t)heads * H, &rc)) ||
        !(out->nea = resolve_vec(p->nea, (size_t)heads, &rc)) || !(out->dt = resolve_vec(p->dt, (size_t)heads, &rc)) ||
        !(out->norm_w = resolve_vec(p->norm_w, (size_t)qb::kGdnHeadDim, &rc)))
        return rc;
    if (!p->conv_s || !p->state) return fail(QB_EINVAL, "linear-layer plan: null conv_s or state");
    out->conv_s = p->conv_s;
    out->state = p->state;
    out->heads = heads;
    return QB_OK;
}

// Device copies of the engine's mutable Gated-DeltaNet state arrays, keyed
// by host address.  Modes (qwen_b200_gdn_state_mode):
//   0 mirror         the host array is copied in before every layer call and
//                    back after it (the reference's contract): pageable
//                    copies, or, in forward_token_c, through the staging
//                    buffer below;
//   1 resident       copied in once, then the device copy is the state until
//                    qwen_b200_gdn_state_sync() copies it back or _drop()
//                    forgets it;
//   2 pinned mirror  mode 0 with the host arrays page-locked in place on first
//                    sight (cudaHostRegister), so the copies are asynchronous
//                    DMA -- for callers whose arrays live until _drop() (a
//                    registration outlives a freed array and makes later
//                    copies over an overlapping range fail).
enum { kStateMirror = 0, kStateResident = 1, kStatePinned = 2 };
struct StateSlot {
    float* dev = nullptr;
    size_t n = 0;
    bool pinned = false;
};
std::unordered_map<const float*, StateSlot> g_state_slots;
int g_state_mode = kStateMirror;

void slot_release(const float* host, StateSlot& s) {
    if (s.pinned) cudaHostUnregister(const_cast<float*>(host));
    if (s.dev) cudaFree(s.dev);
    s = StateSlot{};
}

void slots_clear() {
    for (auto& kv : g_state_slots) slot_release(kv.first, kv.second);
    g_state_slots.clear();
}

float* state_slot(float* host, size_t n, bool* fresh, int* rc) {
    *fresh = false;
    auto it = g_state_slots.find(host);
    if (it != g_state_slots.end() && it->second.n != n) {   // a different-sized array at the same address
        slot_release(it->first, it->second);
        g_state_slots.erase(it);
        it = g_state_slots.end();
    }
    if (it == g_state_slots.end()) {
        // two live arrays never overlap: a slot whose range meets this one
        // belongs to an array that is gone
        const char* lo = reinterpret_cast<const char*>(host);
        const char* hi = lo + n * sizeof(float);
        for (auto o = g_state_slots.begin(); o != g_state_slots.end();) {
            const char* olo = reinterpret_cast<const char*>(o->first);
            if (olo < hi && lo < olo + o->second.n * sizeof(float)) {
                slot_release(o->first, o->second);
                o = g_state_slots.erase(o);
            } else {
                ++o;
            }
        }
        StateSlot sl;
        cudaError_t e = cudaMalloc(&sl.dev, n * sizeof(float));
        if (e != cudaSuccess) {
            *rc = fail(QB_ENOMEM, "state alloc", e);
            return nullptr;
        }
        sl.n = n;
        if (g_state_mode == kStatePinned) {
            sl.pinned = cudaHostRegister(host, n * sizeof(float), cudaHostRegisterDefault) == cudaSuccess;
            if (!sl.pinned) cudaGetLastError();   // not an error: the copies stay pageable
        }
        it = g_state_slots.emplace(host, sl).first;
        *fresh = true;
    }
    return it->second.dev;
}

// Floats of a layer's conv state and recurrent state.
size_t conv_floats(const DevLinear& w) { return 3 * (size_t)w.qkv.M; }
size_t state_floats(const DevLinear& w) { return (size_t)w.heads * qb::kGdnHeadDim * qb::kGdnHeadDim; }

// Bring a layer's states onto the device on stream s (per the mode);
// dev_conv / dev_state receive the device copies.  With `stage` (mirror
// mode in forward_token_c) the host side of the copies is the layer's
// page-locked staging area -- conv state, then recurrent state -- instead of
// the caller's arrays.
int states_in(const DevLinear& w, float** dev_conv, float** dev_state, cudaStream_t s, const float* stage = nullptr) {
    int rc = QB_OK;
    const size_t nc = conv_floats(w), ns = state_floats(w);
    bool fc = false, fs = false;
    if (!(*dev_conv = state_slot(w.conv_s, nc, &fc, &rc)) || !(*dev_state = state_slot(w.state, ns, &fs, &rc)))
        return rc;
    cudaError_t e = cudaSuccess;
    const bool resident = g_state_mode == kStateResident;
    const float* hc = stage ? stage : w.conv_s;
    const float* hs = stage ? stage + nc : w.state;
    if (!resident || fc) e = cudaMemcpyAsync(*dev_conv, hc, nc * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && (!resident || fs)) e = cudaMemcpyAsync(*dev_state, hs, ns * 4, cudaMemcpyHostToDevice, s);
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "state copy in", e);
}
int states_out(const DevLinear& w, const float* dev_conv, const float* dev_state, cudaStream_t s,
               float* stage = nullptr) {
    if (g_state_mode == kStateResident) return QB_OK;
    const size_t nc = conv_floats(w), ns = state_floats(w);
    float* hc = stage ? stage : w.conv_s;
    float* hs = stage ? stage + nc : w.state;
    cudaError_t e = cudaMemcpyAsync(hc, dev_conv, nc * 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(hs, dev_state, ns * 4, cudaMemcpyDeviceToHost, s);
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "state copy out", e);
}

// Mirror mode's staging: the caller's pageable state arrays are copied into
// one page-locked buffer (and back) by several host threads at once, and
// the device copies are DMA from / to that buffer.  A pageable cudaMemcpy
// stages through the driver's own buffers on one thread (~8.6 GB/s here);
// the threads split the bytes evenly (QWEN_B200_COPY_THREADS, default
// min(4, hardware threads)).
void* g_stage = nullptr;
size_t g_stage_bytes = 0;

int stage_reserve(size_t bytes) {
    if (bytes <= g_stage_bytes) return QB_OK;
    if (g_stage) cudaFreeHost(g_stage);
    g_stage = nullptr;
    g_stage_bytes = 0;
    cudaError_t e = cudaHostAlloc(&g_stage, bytes, cudaHostAllocDefault);
    if (e != cudaSuccess) {
        g_stage = nullptr;
        return fail(QB_ENOMEM, "state staging buffer", e);
    }
    g_stage_bytes = bytes;
    return QB_OK;
}

struct CopyChunk {
    char* dst;
    const char* src;
    size_t n;
};

// The copy threads: created on first use, they wait for jobs and live until
// the process exits.  One job at a time (callers hold the library lock);
// the caller's own thread copies the first part.
class CopyPool {
  public:
    explicit CopyPool(int n) : n_(1), pid_(getpid()) {
        int i = 1;
        try {
            for (; i < n; i++) std::thread([this, i] { run(i); }).detach();
        } catch (...) {   // fewer threads than asked for
        }
        n_ = i;
    }
    void copy(const std::vector<CopyChunk>& v) {
        size_t total = 0;
        for (const CopyChunk& c : v) total += c.n;
        // a forked child has none of the parent's threads: it copies alone
        if (n_ == 1 || total < ((size_t)1 << 20) || getpid() != pid_) {
            part(v, 0, total);
            return;
        }
        {
            std::lock_guard<std::mutex> lk(mu_);
            job_ = &v;
            total_ = total;
            pending_ = n_ - 1;
            gen_++;
        }
        cv_.notify_all();
        part(v, 0, total / n_);
        std::unique_lock<std::mutex> lk(mu_);
        done_.wait(lk, [this] { return pending_ == 0; });
        job_ = nullptr;
    }

  private:
    // the bytes [b0, b1) of the chunks' concatenation
    static void part(const std::vector<CopyChunk>& v, size_t b0, size_t b1) {
        size_t base = 0;
        for (const CopyChunk& c : v) {
            const size_t lo = std::max(b0, base), hi = std::min(b1, base + c.n);
            if (lo < hi) memcpy(c.dst + (lo - base), c.src + (lo - base), hi - lo);
            base += c.n;
            if (base >= b1) break;
        }
    }
    void run(int i) {
        unsigned int seen = 0;
        for (;;) {
            const std::vector<CopyChunk>* job;
            size_t total;
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return gen_ != seen; });
                seen = gen_;
                job = job_;
                total = total_;
            }
            part(*job, total * i / n_, total * (i + 1) / n_);
            std::lock_guard<std::mutex> lk(mu_);
            if (--pending_ == 0) done_.notify_one();
        }
    }
    int n_;
    pid_t pid_;   // the process whose threads these are
    std::mutex mu_;
    std::condition_variable cv_, done_;
    const std::vector<CopyChunk>* job_ = nullptr;
    size_t total_ = 0;
    int pending_ = 0;
    unsigned int gen_ = 0;
};

// Every chunk copied, the concatenated bytes split evenly over the pool.
void parallel_copy(const std::vector<CopyChunk>& v) {
    static CopyPool* pool = [] {   // never destroyed: its threads outlive static destructors
        const char* e = getenv("QWEN_B200_COPY_THREADS");
        int t = e ? atoi(e) : 0;
        if (t <= 0) t = std::min(4, (int)std::max(1u, std::thread::hardware_concurrency()));
        return new CopyPool(std::min(t, 64));
    }();
    pool->copy(v);
}

// Event pool of the layer loop's copy / compute ordering (two per layer).
std::vector<cudaEvent_t> g_loop_events;
int loop_events(size_t n) {
    while (g_loop_events.size() < n) {
        cudaEvent_t ev = nullptr;
        cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        if (e != cudaSuccess) return fail(QB_ECUDA, "event create", e);
        g_loop_events.push_back(ev);
    }
    return QB_OK;
}

// Work buffers of the device layer loop (the entry points are serialised).
struct LoopBufs {
    float *h = nullptr, *h2 = nullptr, *qkv = nullptr, *z = nullptr, *gated = nullptr, *o = nullptr,
          *gate = nullptr, *up = nullptr, *norm = nullptr;
    int* res = nullptr;
    void* pin = nullptr;   // pinned staging of h and the token id
    size_t pin_cap = 0;
    void* block = nullptr;
    size_t cap = 0;
};
LoopBufs g_loop;
// Set while forward_token_c runs (its lock is released during the attention
// callback): the layer entry points share g_loop and refuse to run inside it.
bool g_token_busy = false;

// Sized for hidden H, value width V (3 V qkv channels) and MLP width F.
int loop_bufs(int H, int V, int F) {
    auto al = [](size_t n) { return (n * sizeof(float) + 255) & ~size_t(255); };
    const size_t need = 3 * al(H) + al(3 * (size_t)V) + 2 * al(V) + al(H) + 2 * al(F) + 256;
    if (int rc = grow_dev(&g_loop.block, &g_loop.cap, need)) return rc;
    if (int rc = grow_pinned(&g_loop.pin, &g_loop.pin_cap, (size_t)H * 4 + 64)) return rc;
    unsigned char* b = static_cast<unsigned char*>(g_loop.block);
    auto take = [&](size_t n) {
        float* p = reinterpret_cast<float*>(b);
        b += al(n);
        return p;
    };
    g_loop.h = take(H);
    g_loop.h2 = take(H);
    g_loop.o = take(H);
    g_loop.qkv = take(3 * (size_t)V);
    g_loop.z = take(V);
    g_loop.gated = take(V);
    g_loop.norm = take(H);
    g_loop.gate = take(F);
    g_loop.up = take(F);
    g_loop.res = reinterpret_cast<int*>(b);
    return QB_OK;
}

qb::GemvDesc gemv_desc(const DevGemv& g, const float* x, float* y) {
    qb::GemvDesc d{};
    d.mant = g.m;
    d.exps = g.e;
    d.x = x;
    d.y = y;
    d.M = g.M;
    d.K = g.K;
    return d;
}

// forward_mlp's steps on the device: h += down(swiglu(gate(n), up(n))),
// n = rmsnorm(h) -- gate and up in one launch with the rmsnorm in front,
// then down with swiglu in front and the residual add folded into its
// stores (two launches).  With `res`, the layer's
// pending residual h + res is formed in front of gate (h_out = h + res) and
// the MLP runs on h_out; h_out then holds the result.
cudaError_t mlp_launch(const DevMlp& w, float* h, const float* res, float* h_out, DevState* st, cudaStream_t s) {
    // gate and up projections of the same rmsnorm(h) (or of h + res) in one launch
    cudaError_t e = qb::launch_rmsnorm_gemv2(gemv_desc(w.gate, h, g_loop.gate), gemv_desc(w.up, h, g_loop.up),
                                             w.post_ln, 1e-6f, st->act, st->err, s, res, res ? h_out : nullptr);
    float* hh = res ? h_out : h;
    // down projection of swiglu(gate, up), its rows added into the residual stream as they are stored
    if (e == cudaSuccess)
        e = qb::launch_swiglu_gemv(gemv_desc(w.down, g_loop.gate, hh), g_loop.up, st->act, st->err, s, true);
    return e;
}

// forward_linear_layer's steps on the device (five launches): the qkv and z
// projections of rmsnorm(h) (one launch), the Gated-DeltaNet kernel, the out
// projection, then the MLP with h + o formed in front of its gate and up
// projections and the down rows added into it.  The result lands in g_loop.h2.
cudaError_t linear_launch(const DevLinear& w, float* h, float* dev_conv, float* dev_state, DevState* st,
                          cudaStream_t s) {
    // qkv and z projections of the same rmsnorm(h) in one launch, which also
    // leaves the normalized vector for the gates
    cudaError_t e = qb::launch_rmsnorm_gemv2(gemv_desc(w.qkv, h, g_loop.qkv), gemv_desc(w.z, h, g_loop.z), w.in_ln,
                                             1e-6f, st->act, st->err, s, nullptr, nullptr, g_loop.norm);
    if (e == cudaSuccess) {
        qb::GdnArgs a{};
        a.qkv = g_loop.qkv;
        a.z = g_loop.z;
        a.normed = g_loop.norm;
        a.conv_w = w.conv_w;
        a.conv_s = dev_conv;
        a.wa = w.wa;
        a.wb = w.wb;
        a.nea = w.nea;
        a.dt = w.dt;
        a.state = dev_state;
        a.norm_w = w.norm_w;
        a.out = g_loop.gated;
        a.heads = w.heads;
        a.hidden = w.qkv.K;
        e = qb::launch_gdn_layer(a, s);
    }
    if (e == cudaSuccess) e = qb::launch_gemv(gemv_desc(w.o, g_loop.gated, g_loop.o), st->act, st->err, s);
    if (e == cudaSuccess) e = mlp_launch(w.mlp, h, g_loop.o, g_loop.h2, st, s);
    return e;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorInvalidValue ? QB_EINVAL : QB_ECUDA, what, e);
}

// Prefix the pending error message with the failing entry point's name.
void name_error(const char* entry) {
    if (g_err.compare(0, strlen(entry), entry) != 0) g_err = std::string(entry) + ": " + g_err;
}

}  // namespace

extern "C" {

void init_kernels(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    ensure_ctx();
}

const char* qwen_b200_last_error(void) { return g_err.c_str(); }

void qwen_prof_enable(int on) { g_prof_on = on; }
void qwen_prof_reset(void) {
    for (double& v : g_prof_ms) v = 0.0;
}
int qwen_prof_count(void) { return PF_N; }
double qwen_prof_get(int i) { return (i >= 0 && i < PF_N) ? g_prof_ms[i] : 0.0; }
const char* qwen_prof_name(int i) { return (i >= 0 && i < PF_N) ? kProfNames[i] : "?"; }

int qwen_b200_register_weights(const void* host_base, size_t nbytes) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!host_base || !nbytes) return fail(QB_EINVAL, "empty range");
    int rc = ensure_ctx();
    if (rc) return rc;
    if (lookup(host_base, nbytes)) return QB_OK;
    return upload_range(host_base, nbytes);
}

int qwen_b200_forget_weights(const void* host_ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    const unsigned char* h = static_cast<const unsigned char*>(host_ptr);
    for (size_t i = 0; i < g_ranges.size();) {
        if (h >= g_ranges[i].host && h < g_ranges[i].host + g_ranges[i].bytes) {
            cudaFree(g_ranges[i].dev);
            g_ranges.erase(g_ranges.begin() + i);
        } else {
            i++;
        }
    }
    return QB_OK;
}

void qwen_b200_reset_weights(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (Range& r : g_ranges) cudaFree(r.dev);
    g_ranges.clear();
}

// ------------------------------------------------------------ drop-ins
void bfp8_gemv(float* y, const float* x, const int8_t* mant, const uint8_t* exps, int M, int K) {
    ProfScope ps(PF_GEMV);
    std::lock_guard<std::mutex> lk(g_mu);
    if (check_gemv_args(y, x, mant, exps, M, K) || M == 0) return;
    if (ensure_ctx()) return;
    const size_t wbytes = (size_t)M * K, ebytes = (size_t)M * (K / 64);
    int rc = QB_OK;
    const void* dm;
    const void* de;
    if (exps == reinterpret_cast<const uint8_t*>(mant) + wbytes) {
        dm = device_of(mant, wbytes + ebytes, &rc);
        de = dm ? static_cast<const unsigned char*>(dm) + wbytes : nullptr;
    } else {
        dm = device_of(mant, wbytes, &rc);
        de = dm ? device_of(exps, ebytes, &rc) : nullptr;
    }
    if (!dm || !de) return;
    if (grow_pinned(&g_ctx.h_in, &g_ctx.h_in_cap, 4 * (size_t)K) ||
        grow_pinned(&g_ctx.h_out, &g_ctx.h_out_cap, 4 * (size_t)M) ||
        grow_dev(&g_ctx.d_in, &g_ctx.d_in_cap, 4 * (size_t)K))
        return;
    cudaStream_t s = g_ctx.stream;
    memcpy(g_ctx.h_in, x, 4 * (size_t)K);
    cudaMemcpyAsync(g_ctx.d_in, g_ctx.h_in, 4 * (size_t)K, cudaMemcpyHostToDevice, s);
    qb::GemvDesc d{};
    d.mant = static_cast<const int8_t*>(dm);
    d.exps = static_cast<const uint8_t*>(de);
    d.x = static_cast<const float*>(g_ctx.d_in);
    // the kernel stores y straight into the pinned staging buffer (device-
    // addressable host memory): one copy-engine round trip fewer per call
    d.y = static_cast<float*>(g_ctx.h_out);
    d.M = M;
    d.K = K;
    DevState* dst = nullptr;
    if (dev_state(&dst)) return;
    if (qb::gemv_act_words(K) > kActScratchWords) {
        fail(QB_EINVAL, "bfp8_gemv: K too large");
        return;
    }
    cudaError_t e = qb::launch_gemv(d, dst->act, dst->err, s);
    if (e != cudaSuccess) {
        fail(QB_ECUDA, "bfp8_gemv launch", e);
        return;
    }
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        fail(QB_ECUDA, "bfp8_gemv", e);
        return;
    }
    memcpy(y, g_ctx.h_out, 4 * (size_t)M);
}

void forward_mlp(const MlpPlanC* p, float* h) {
    ProfScope ps(PF_MLP);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!h) {
        fail(QB_EINVAL, "forward_mlp: null h");
        return;
    }
    if (g_token_busy) {
        fail(QB_EINVAL, "forward_mlp: called from inside forward_token_c's callback");
        return;
    }
    DevMlp w;
    DevState* st = nullptr;
    if (ensure_ctx() || resolve_mlp_plan(p, &w) || dev_state(&st) || loop_bufs(w.gate.K, qb::kGdnHeadDim, w.gate.M))
        return name_error("forward_mlp");
    const size_t hb = 4 * (size_t)w.gate.K;
    cudaStream_t s = g_ctx.stream;
    memcpy(g_loop.pin, h, hb);
    cudaError_t e = cudaMemcpyAsync(g_loop.h, g_loop.pin, hb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = mlp_launch(w, g_loop.h, nullptr, nullptr, st, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(g_loop.pin, g_loop.h, hb, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        cuda_fail(e, "forward_mlp");
        return;
    }
    memcpy(h, g_loop.pin, hb);
}

void forward_linear_layer(const LinearLayerPlanC* p, float* h) {
    ProfScope ps(PF_LINEAR);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!h) {
        fail(QB_EINVAL, "forward_linear_layer: null h");
        return;
    }
    if (g_token_busy) {
        fail(QB_EINVAL, "forward_linear_layer: called from inside forward_token_c's callback");
        return;
    }
    DevLinear w;
    DevState* st = nullptr;
    if (ensure_ctx() || resolve_linear_plan(p, &w) || dev_state(&st) || loop_bufs(w.qkv.K, w.z.M, w.mlp.gate.M))
        return name_error("forward_linear_layer");
    const size_t hb = 4 * (size_t)w.qkv.K;
    cudaStream_t s = g_ctx.stream;
    float *dconv = nullptr, *dstate = nullptr;
    if (states_in(w, &dconv, &dstate, s)) return name_error("forward_linear_layer");
    memcpy(g_loop.pin, h, hb);
    cudaError_t e = cudaMemcpyAsync(g_loop.h, g_loop.pin, hb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = linear_launch(w, g_loop.h, dconv, dstate, st, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(g_loop.pin, g_loop.h2, hb, cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) {
        cuda_fail(e, "forward_linear_layer");
        return;
    }
    if (states_out(w, dconv, dstate, s)) return name_error("forward_linear_layer");
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) {
        cuda_fail(e, "forward_linear_layer");
        return;
    }
    memcpy(h, g_loop.pin, hb);
}

int forward_token_c(int token_id, float* h, const LinearLayerPlanC* linear_plans, const MlpPlanC* mlp_plans,
                    const int* layer_is_full, const float* final_norm_w, const uint16_t* embed_table,
                    QbFullAttnCallback full_attn_cb, void* py_context) {
    ProfScope ps(PF_TOKEN);
    std::unique_lock<std::mutex> lk(g_mu);
    if (!h || !linear_plans || !mlp_plans || !layer_is_full || !final_norm_w || !embed_table || token_id < 0)
        return fail(QB_EINVAL, "forward_token_c: null pointer or negative token id"), -1;
    if (g_token_busy) return fail(QB_EINVAL, "forward_token_c: called from inside its own callback"), -1;
    if (ensure_ctx()) return name_error("forward_token_c"), -1;
    // resolve every layer first: a bad plan changes nothing
    std::vector<DevLinear> lin;
    std::vector<DevMlp> mlp(kLoopLayers);
    int n_lin = 0, F = 0, V = qb::kGdnHeadDim;
    for (int l = 0; l < kLoopLayers; l++) {
        if (layer_is_full[l]) {
            if (resolve_mlp_plan(&mlp_plans[l], &mlp[l])) return name_error("forward_token_c"), -1;
            if (mlp[l].gate.K != kLoopHidden) return fail(QB_EINVAL, "forward_token_c: hidden must be 1024"), -1;
            F = std::max(F, mlp[l].gate.M);
        } else {
            lin.emplace_back();
            if (resolve_linear_plan(&linear_plans[n_lin++], &lin.back())) return name_error("forward_token_c"), -1;
            if (lin.back().qkv.K != kLoopHidden) return fail(QB_EINVAL, "forward_token_c: hidden must be 1024"), -1;
            F = std::max(F, lin.back().mlp.gate.M);
            V = std::max(V, lin.back().z.M);
        }
    }
    int rc = QB_OK;
    const uint16_t* dE =
        static_cast<const uint16_t*>(device_of(embed_table, (size_t)kLoopVocab * kLoopHidden * 2, &rc));
    const float* dfin = resolve_vec(final_norm_w, kLoopHidden, &rc);
    DevState* st = nullptr;
    if (!dE || !dfin || dev_state(&st) || loop_bufs(kLoopHidden, V, F)) return name_error("forward_token_c"), -1;
    cudaStream_t s = g_ctx.stream;
    const size_t hb = 4 * (size_t)kLoopHidden;
    // States move on the copy stream, interleaved with the layers: layer i's
    // states go in just before its work is queued and its compute waits for
    // them; they come back once layer i + 1 is queued.  The host side of
    // these copies is page-locked, so nothing waits: the staging buffer in
    // mirror mode, the registered arrays in mode 2.
    std::vector<float*> dconv(lin.size()), dstate(lin.size());
    // mirror mode: every layer's states are first copied into the staging
    // buffer by several host threads, and back into the caller's arrays
    // once their copies out have landed (while the host waits for the GPU
    // at a callback or at the end)
    std::vector<float*> stage(lin.size(), nullptr);
    std::vector<CopyChunk> back;   // staging -> the caller's arrays, after the last copy out
    if (g_state_mode == kStateMirror && !lin.empty()) {
        size_t total = 0;
        for (const DevLinear& w : lin) total += (conv_floats(w) + state_floats(w)) * 4;
        if (stage_reserve(total)) return name_error("forward_token_c"), -1;
        std::vector<CopyChunk> in;
        char* p = static_cast<char*>(g_stage);
        for (size_t i = 0; i < lin.size(); i++) {
            const size_t bc = conv_floats(lin[i]) * 4, bs = state_floats(lin[i]) * 4;
            stage[i] = reinterpret_cast<float*>(p);
            in.push_back({p, reinterpret_cast<const char*>(lin[i].conv_s), bc});
            in.push_back({p + bc, reinterpret_cast<const char*>(lin[i].state), bs});
            back.push_back({reinterpret_cast<char*>(lin[i].conv_s), p, bc});
            back.push_back({reinterpret_cast<char*>(lin[i].state), p + bc, bs});
            p += bc + bs;
        }
        parallel_copy(in);
    }
    cudaStream_t cs = g_ctx.copy;
    if (loop_events(3 * lin.size() + 1)) return name_error("forward_token_c"), -1;
    cudaEvent_t* ev_in = g_loop_events.data();
    cudaEvent_t* ev_done = ev_in + lin.size();
    cudaEvent_t* ev_out = ev_in + 2 * lin.size();   // a layer's copy out has landed in the staging buffer
    cudaEvent_t ev_start = ev_in[3 * lin.size()];
    size_t out_queued = 0, out_back = 0;   // mirror mode: layers whose copy out is queued / written back
    // mirror mode: while the GPU works through what is queued on s, the
    // layers whose states have landed are written back to the caller's arrays
    auto write_back_while_busy = [&]() {
        if (back.empty()) return;
        while (cudaStreamQuery(s) == cudaErrorNotReady) {
            if (out_back < out_queued && cudaEventQuery(ev_out[out_back]) == cudaSuccess) {
                parallel_copy({back[2 * out_back], back[2 * out_back + 1]});
                out_back++;
            } else {
                std::this_thread::yield();
            }
        }
        cudaGetLastError();   // "not ready" is no failure
    };
    if (cudaEventRecord(ev_start, s) != cudaSuccess || cudaStreamWaitEvent(cs, ev_start, 0) != cudaSuccess)
        return cuda_fail(cudaGetLastError(), "forward_token_c"), -1;   // the previous call's work is done first
    // 1. the bf16 embedding row of token_id % 65536
    cudaError_t e = qb::launch_embed_row(g_loop.h, dE, token_id % kLoopVocab, kLoopHidden, s);
    // 2. the layers: full-attention ones run the caller's callback on the host
    // h (the lock released: it calls back into bfp8_gemv), then the MLP
    size_t li = 0;
    for (int l = 0; l < kLoopLayers && e == cudaSuccess; l++) {
        if (layer_is_full[l]) {
            if (full_attn_cb) {
                e = cudaMemcpyAsync(g_loop.pin, g_loop.h, hb, cudaMemcpyDeviceToHost, s);
                if (e != cudaSuccess) break;
                write_back_while_busy();
                if ((e = cudaStreamSynchronize(s)) != cudaSuccess) break;
                memcpy(h, g_loop.pin, hb);
                g_token_busy = true;
                lk.unlock();
                {
                    ProfScope pc(PF_CALLBACK);
                    full_attn_cb(l, h, py_context);
                }
                lk.lock();
                g_token_busy = false;
                memcpy(g_loop.pin, h, hb);
                e = cudaMemcpyAsync(g_loop.h, g_loop.pin, hb, cudaMemcpyHostToDevice, s);
                if (e != cudaSuccess) break;
            }
            e = mlp_launch(mlp[l], g_loop.h, nullptr, nullptr, st, s);
        } else {
            if (states_in(lin[li], &dconv[li], &dstate[li], cs, stage[li])) return name_error("forward_token_c"), -1;
            e = cudaEventRecord(ev_in[li], cs);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ev_in[li], 0);
            if (e == cudaSuccess) e = linear_launch(lin[li], g_loop.h, dconv[li], dstate[li], st, s);
            if (e == cudaSuccess) e = cudaEventRecord(ev_done[li], s);
            if (e == cudaSuccess && li > 0) e = cudaStreamWaitEvent(cs, ev_done[li - 1], 0);
            if (e == cudaSuccess && li > 0 &&
                states_out(lin[li - 1], dconv[li - 1], dstate[li - 1], cs, stage[li - 1]))
                return name_error("forward_token_c"), -1;
            if (e == cudaSuccess && li > 0 && (e = cudaEventRecord(ev_out[li - 1], cs)) == cudaSuccess)
                out_queued = li;
            std::swap(g_loop.h, g_loop.h2);   // the layer's output is the next layer's h
            li++;
        }
    }
    // 3. final rmsnorm, 4. lm_head argmax over the 65536 embedding rows
    if (e == cudaSuccess) e = qb::launch_rmsnorm(g_loop.norm, g_loop.h, dfin, kLoopHidden, 1e-6f, s);
    if (e == cudaSuccess)
        e = qb::launch_lm_head_bf16(g_loop.norm, dE, kLoopVocab, kLoopHidden, 0, 0, g_ctx.scratch, st->err, nullptr,
                                    g_loop.res, nullptr, nullptr, g_loop.res + 1, s);
    int* pid = reinterpret_cast<int*>(static_cast<unsigned char*>(g_loop.pin) + hb);
    if (e == cudaSuccess) e = cudaMemcpyAsync(g_loop.pin, g_loop.h, hb, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(pid, g_loop.res, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && li > 0) e = cudaStreamWaitEvent(cs, ev_done[li - 1], 0);
    if (e != cudaSuccess) return cuda_fail(e, "forward_token_c"), -1;
    if (li > 0 && states_out(lin[li - 1], dconv[li - 1], dstate[li - 1], cs, stage[li - 1]))
        return name_error("forward_token_c"), -1;
    if (li > 0 && (e = cudaEventRecord(ev_out[li - 1], cs)) != cudaSuccess) return cuda_fail(e, "forward_token_c"), -1;
    out_queued = li;
    write_back_while_busy();
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess || (e = cudaStreamSynchronize(cs)) != cudaSuccess)
        return cuda_fail(e, "forward_token_c"), -1;
    if (!back.empty() && out_back < li)
        parallel_copy(std::vector<CopyChunk>(back.begin() + 2 * out_back, back.end()));
    memcpy(h, g_loop.pin, hb);
    return *pid;
}

int qwen_b200_gdn_state_mode(int mode) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (mode != kStateMirror && mode != kStateResident && mode != kStatePinned)
        return fail(QB_EINVAL, "qwen_b200_gdn_state_mode: 0 (mirror), 1 (resident) or 2 (pinned mirror)");
    if (mode == g_state_mode) return QB_OK;
    if (g_state_mode == kStateResident) {   // leaving resident mode: the host arrays catch up first
        for (auto& kv : g_state_slots) {
            cudaError_t e = cudaMemcpy(const_cast<float*>(kv.first), kv.second.dev, kv.second.n * 4,
                                       cudaMemcpyDeviceToHost);
            if (e != cudaSuccess) return fail(QB_ECUDA, "state sync", e);
        }
    }
    slots_clear();   // every mode starts from the host arrays (and holds no registration it did not make)
    g_state_mode = mode;
    return QB_OK;
}

int qwen_b200_gdn_state_sync(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto& kv : g_state_slots) {
        cudaError_t e =
            cudaMemcpy(const_cast<float*>(kv.first), kv.second.dev, kv.second.n * 4, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return fail(QB_ECUDA, "state sync", e);
    }
    return QB_OK;
}

void qwen_b200_gdn_state_drop(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    slots_clear();
}

static int lm_bf16_host(const float* h, const uint16_t* E, int vocab, int hidden, int k, int with_tail,
                        int* out_ids, float* out_scores, int* id_out) {
    if (ensure_ctx()) return QB_ENODEV;
    int rc = QB_OK;
    const void* dE = device_of(E, (size_t)vocab * hidden * 2, &rc);
    if (!dE) return rc;
    const size_t kk = (size_t)(k < vocab ? k : vocab);
    const size_t in_b = 4 * (size_t)hidden;
    const size_t out_b = kk * 8 + 16;
    if ((rc = grow_pinned(&g_ctx.h_in, &g_ctx.h_in_cap, in_b)) ||
        (rc = grow_pinned(&g_ctx.h_out, &g_ctx.h_out_cap, out_b)) ||
        (rc = grow_dev(&g_ctx.d_in, &g_ctx.d_in_cap, in_b + 16)) ||
        (rc = grow_dev(&g_ctx.d_out, &g_ctx.d_out_cap, out_b)))
        return rc;
    float* score_buf = nullptr;
    if (hidden % 8 || reinterpret_cast<uintptr_t>(dE) % 16) {
        if ((rc = grow_dev(reinterpret_cast<void**>(&g_ctx.d_scores), &g_ctx.d_scores_cap, 4 * (size_t)vocab)))
            return rc;
        score_buf = g_ctx.d_scores;
    }
    cudaStream_t s = g_ctx.stream;
    memcpy(g_ctx.h_in, h, in_b);
    cudaMemcpyAsync(g_ctx.d_in, g_ctx.h_in, in_b, cudaMemcpyHostToDevice, s);
    int* d_ids = static_cast<int*>(g_ctx.d_out);
    float* d_sc = reinterpret_cast<float*>(d_ids + kk);
    DevState* dst = nullptr;
    if (int rc2 = dev_state(&dst)) return rc2;
    cudaError_t e = qb::launch_lm_head_bf16(static_cast<const float*>(g_ctx.d_in), static_cast<const uint16_t*>(dE),
                                            vocab, hidden, (int)kk, with_tail, g_ctx.scratch, dst->err, score_buf,
                                            g_ctx.d_res, d_ids, d_sc, g_ctx.d_res + 1, s);
    if (e != cudaSuccess) return fail(QB_ECUDA, "lm_head launch", e);
    int res[2] = {0, 0};
    cudaMemcpyAsync(g_ctx.h_out, d_ids, kk * 8, cudaMemcpyDeviceToHost, s);
    cudaMemcpyAsync(res, g_ctx.d_res, 2 * sizeof(int), cudaMemcpyDeviceToHost, s);
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(QB_ECUDA, "lm_head", e);
    *id_out = res[0];
    if (kk > 0) {
        const int n = res[1];
        memcpy(out_ids, g_ctx.h_out, (size_t)n * 4);
        memcpy(out_scores, static_cast<char*>(g_ctx.h_out) + kk * 4, (size_t)n * 4);
        return n;
    }
    return 0;
}

// lm_head_topk for k above the fused kernels' 1024: the scores of every row
// in the lm_head_topk order, then one device radix sort of (score, ~id) keys.
static int lm_bf16_host_large(const float* h, const uint16_t* E, int vocab, int hidden, int k, int* out_ids,
                              float* out_scores) {
    if (ensure_ctx()) return QB_ENODEV;
    int rc = QB_OK;
    const void* dE = device_of(E, (size_t)vocab * hidden * 2, &rc);
    if (!dE) return rc;
    const int kk = k < vocab ? k : vocab;
    const size_t in_b = 4 * (size_t)hidden, out_b = (size_t)kk * 8 + 16;
    const size_t temp_b = qb::topk_large_temp_bytes(vocab);
    // device: scores, two key buffers, sort temp storage (one growable block)
    const size_t sc_b = (4 * (size_t)vocab + 255) & ~size_t(255), key_b = (8 * (size_t)vocab + 255) & ~size_t(255);
    if ((rc = grow_pinned(&g_ctx.h_in, &g_ctx.h_in_cap, in_b)) ||
        (rc = grow_pinned(&g_ctx.h_out, &g_ctx.h_out_cap, out_b)) ||
        (rc = grow_dev(&g_ctx.d_in, &g_ctx.d_in_cap, in_b + 16)) ||
        (rc = grow_dev(&g_ctx.d_out, &g_ctx.d_out_cap, out_b)) ||
        (rc = grow_dev(reinterpret_cast<void**>(&g_ctx.d_scores), &g_ctx.d_scores_cap, sc_b + 2 * key_b + temp_b)))
        return rc;
    unsigned char* blk = reinterpret_cast<unsigned char*>(g_ctx.d_scores);
    float* d_sc_all = reinterpret_cast<float*>(blk);
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(blk + sc_b);
    unsigned long long* keys_alt = reinterpret_cast<unsigned long long*>(blk + sc_b + key_b);
    void* temp = blk + sc_b + 2 * key_b;
    cudaStream_t s = g_ctx.stream;
    memcpy(g_ctx.h_in, h, in_b);
    cudaMemcpyAsync(g_ctx.d_in, g_ctx.h_in, in_b, cudaMemcpyHostToDevice, s);
    int* d_ids = static_cast<int*>(g_ctx.d_out);
    float* d_sc = reinterpret_cast<float*>(d_ids + kk);
    cudaError_t e = qb::launch_lm_scores_bf16(static_cast<const float*>(g_ctx.d_in), static_cast<const uint16_t*>(dE),
                                              vocab, hidden, 1, d_sc_all, s);
    if (e == cudaSuccess)
        e = qb::launch_topk_large(d_sc_all, vocab, kk, keys, keys_alt, temp, temp_b, d_ids, d_sc, g_ctx.d_res + 1,
                                  s);
    if (e != cudaSuccess) return fail(QB_ECUDA, "lm_head_topk launch", e);
    int n = 0;
    cudaMemcpyAsync(g_ctx.h_out, d_ids, (size_t)kk * 8, cudaMemcpyDeviceToHost, s);
    cudaMemcpyAsync(&n, g_ctx.d_res + 1, sizeof(int), cudaMemcpyDeviceToHost, s);
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return fail(QB_ECUDA, "lm_head_topk", e);
    memcpy(out_ids, g_ctx.h_out, (size_t)n * 4);
    memcpy(out_scores, static_cast<char*>(g_ctx.h_out) + (size_t)kk * 4, (size_t)n * 4);
    return n;
}

int lm_head_argmax(const float* h, const uint16_t* embed_table, int vocab_size, int hidden_dim) {
    ProfScope ps(PF_ARGMAX);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!h || !embed_table || vocab_size <= 0 || hidden_dim <= 0) {
        fail(QB_EINVAL, "lm_head_argmax: bad arguments");
        return -1;
    }
    int id = 0;
    int rc = lm_bf16_host(h, embed_table, vocab_size, hidden_dim, 0, 0, nullptr, nullptr, &id);
    return rc < 0 ? -1 : id;
}

int lm_head_topk(const float* h, const uint16_t* embed_table, int vocab_size, int hidden_dim, int k,
                 int* out_ids, float* out_scores) {
    ProfScope ps(PF_TOPK);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!h || !embed_table || !out_ids || !out_scores) return 0;
    if (vocab_size <= 0 || hidden_dim <= 0 || k <= 0) return 0;
    if ((k < vocab_size ? k : vocab_size) > qb::kTopkMax) {
        const int n = lm_bf16_host_large(h, embed_table, vocab_size, hidden_dim, k, out_ids, out_scores);
        return n < 0 ? 0 : n;
    }
    int id = 0;
    int n = lm_bf16_host(h, embed_table, vocab_size, hidden_dim, k, 1, out_ids, out_scores, &id);
    return n < 0 ? 0 : n;
}

int sample_from_topk(const int* ids, const float* scores, int n, float temperature, int top_k, float top_p,
                     unsigned int* rng_state) {
    ProfScope ps(PF_SAMPLE);
    // Draws equal qwen_sampling.c:411-529 bit for bit, so every rounding step below (float
    // exponent argument, double accumulation in candidate order, the 24-bit uniform) is fixed.
    if (!ids || !scores || n <= 0) return -1;
    if (!rng_state) return ids[0];

    // The candidates in descending score order (ties: lower id first). The fused lm_head top-k
    // already emits them that way, so the copy is only made for an unordered list.
    std::vector<Cand> reordered;
    bool descending = true;
    for (int i = 1; i < n && descending; i++) descending = !(scores[i] > scores[i - 1]);
    if (!descending) {
        reordered.resize(n);
        for (int i = 0; i < n; i++) reordered[i] = {ids[i], scores[i]};
        qsort(reordered.data(), (size_t)n, sizeof(Cand), [](const void* a, const void* b) -> int {
            const Cand& l = *static_cast<const Cand*>(a);
            const Cand& r = *static_cast<const Cand*>(b);
            if (l.score > r.score) return -1;  // two comparisons: unordered (NaN) scores fall
            if (l.score < r.score) return 1;   // through to the id order
            return l.id < r.id ? -1 : (l.id > r.id ? 1 : 0);
        });
    }
    auto token = [&](int i) { return descending ? ids[i] : reordered[i].id; };
    auto score = [&](int i) { return descending ? scores[i] : reordered[i].score; };

    if (!(temperature >= 1e-6f)) return token(0);  // greedy (also catches NaN)
    const int window = (top_k > 0 && top_k < n) ? top_k : n;
    float peak = score(0);  // first-wins scan: a NaN head stays the peak
    for (int i = 1; i < window; i++) peak = score(i) > peak ? score(i) : peak;
    const float inv_temp = 1.0f / temperature;
    // Unnormalised softmax weight of candidate i, exactly as the reference rounds it.
    auto weight = [&](int i) { return (double)expf((score(i) - peak) * inv_temp); };

    double z_window = 0.0;
    for (int i = 0; i < window; i++) z_window += weight(i);
    if (!(z_window > 0.0)) return token(0);

    // Nucleus: the shortest prefix whose probability mass passes clamp(top_p, 0, 1).
    const float mass = top_p > 1.0f ? 1.0f : (top_p > 0.0f ? top_p : 0.0f);
    int nucleus = window;
    double share = 0.0;
    for (int i = 0; i < window; i++) {
        share += weight(i) / z_window;
        if (share > (double)mass) {
            nucleus = i + 1;
            break;
        }
    }
    double z_nucleus = 0.0;
    for (int i = 0; i < nucleus; i++) z_nucleus += weight(i);
    if (!(z_nucleus > 0.0)) return token(0);

    // Inverse-CDF draw with a 24-bit uniform from the xorshift32 stream.
    const double u = (double)((float)(xs32_next(rng_state) >> 8) * (1.0f / 16777216.0f));
    const double target = u * z_nucleus;
    double below = 0.0;
    for (int i = 0; i < nucleus; i++) {
        below += weight(i);
        if (target < below) return token(i);
    }
    return token(nucleus - 1);
}

// ------------------------------------------------------------ device entry points
int qwen_b200_gemv_dev(float* y, const float* x, const int8_t* mant, const uint8_t* exps, int M, int K,
                       void* stream) {
    if (int rc = check_gemv_args(y, x, mant, exps, M, K)) return rc;
    qb::GemvDesc d{};
    d.mant = mant;
    d.exps = exps;
    d.x = x;
    d.y = y;
    d.M = M;
    d.K = K;
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    if (qb::gemv_act_words(K) > kActScratchWords) return fail(QB_EINVAL, "K too large");
    cudaError_t e = qb::launch_gemv(d, st->act, st->err, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_gemv_dev", e);
}

int qwen_b200_rmsnorm_gemv_dev(float* y, const float* x, const float* norm_w, float eps, const int8_t* mant,
                               const uint8_t* exps, int M, int K, void* stream) {
    if (int rc = check_gemv_args(y, x, mant, exps, M, K)) return rc;
    if (!norm_w) return fail(QB_EINVAL, "qwen_b200_rmsnorm_gemv_dev: null norm weights");
    qb::GemvDesc d{};
    d.mant = mant;
    d.exps = exps;
    d.x = x;
    d.y = y;
    d.M = M;
    d.K = K;
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    cudaError_t e = qb::launch_rmsnorm_gemv(d, norm_w, eps, st->act, st->err, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue)
        return fail(QB_EINVAL, "qwen_b200_rmsnorm_gemv_dev: K a multiple of 512 and <= 6144, mant/exps/x/norm_w "
                               "16/4/8/8-byte aligned");
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_rmsnorm_gemv_dev", e);
}

int qwen_b200_residual_rmsnorm_gemv_dev(float* y, float* x_out, const float* x, const float* res,
                                        const float* norm_w, float eps, const int8_t* mant, const uint8_t* exps,
                                        int M, int K, void* stream) {
    if (int rc = check_gemv_args(y, x, mant, exps, M, K)) return rc;
    if (!norm_w || !res || !x_out) return fail(QB_EINVAL, "qwen_b200_residual_rmsnorm_gemv_dev: null pointer");
    qb::GemvDesc d{};
    d.mant = mant;
    d.exps = exps;
    d.x = x;
    d.y = y;
    d.M = M;
    d.K = K;
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    cudaError_t e = qb::launch_rmsnorm_gemv(d, norm_w, eps, st->act, st->err, static_cast<cudaStream_t>(stream),
                                            res, x_out);
    if (e == cudaErrorInvalidValue)
        return fail(QB_EINVAL, "qwen_b200_residual_rmsnorm_gemv_dev: K a multiple of 512 and <= 6144, 8-byte aligned "
                               "vectors, x_out overlapping neither x nor res");
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_residual_rmsnorm_gemv_dev", e);
}

int qwen_b200_rmsnorm_gemv2_dev(float* y0, float* y1, float* x_out, const float* x, const float* res,
                                const float* norm_w, float eps, const int8_t* mant0, const uint8_t* exps0, int M0,
                                const int8_t* mant1, const uint8_t* exps1, int M1, int K, void* stream) {
    if (int rc = check_gemv_args(y0, x, mant0, exps0, M0, K)) return rc;
    if (int rc = check_gemv_args(y1, x, mant1, exps1, M1, K)) return rc;
    if (!norm_w || (res == nullptr) != (x_out == nullptr))
        return fail(QB_EINVAL, "qwen_b200_rmsnorm_gemv2_dev: null norm weights, or only one of res / x_out");
    qb::GemvDesc d0{}, d1{};
    d0.mant = mant0;
    d0.exps = exps0;
    d0.x = x;
    d0.y = y0;
    d0.M = M0;
    d0.K = K;
    d1 = d0;
    d1.mant = mant1;
    d1.exps = exps1;
    d1.y = y1;
    d1.M = M1;
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    cudaError_t e = qb::launch_rmsnorm_gemv2(d0, d1, norm_w, eps, st->act, st->err, static_cast<cudaStream_t>(stream),
                                             res, x_out);
    if (e == cudaErrorInvalidValue)
        return fail(QB_EINVAL, "qwen_b200_rmsnorm_gemv2_dev: M0, M1 >= 1, K a multiple of 512 and <= 6144, 8-byte "
                               "aligned vectors, x_out overlapping neither x nor res");
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_rmsnorm_gemv2_dev", e);
}

int qwen_b200_swiglu_gemv_dev(float* y, const float* gate, const float* up, const int8_t* mant,
                              const uint8_t* exps, int M, int K, void* stream) {
    if (int rc = check_gemv_args(y, gate, mant, exps, M, K)) return rc;
    if (!up) return fail(QB_EINVAL, "qwen_b200_swiglu_gemv_dev: null up projection");
    qb::GemvDesc d{};
    d.mant = mant;
    d.exps = exps;
    d.x = gate;
    d.y = y;
    d.M = M;
    d.K = K;
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    cudaError_t e = qb::launch_swiglu_gemv(d, up, st->act, st->err, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue)
        return fail(QB_EINVAL, "qwen_b200_swiglu_gemv_dev: K a multiple of 512 and <= 6144, mant/exps 16/4-byte, "
                               "gate/up 8-byte aligned");
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_swiglu_gemv_dev", e);
}

int qwen_b200_gemv_q_dev(float* y, const int16_t* xq, const float* xs, const int8_t* mant,
                         const uint8_t* exps, int M, int K, void* stream) {
    if (int rc = check_gemv_args(y, xq, mant, exps, M, K)) return rc;
    if (!xs) return fail(QB_EINVAL, "null xs");
    qb::GemvDesc d{};
    d.mant = mant;
    d.exps = exps;
    d.xq = xq;
    d.xs = xs;
    d.y = y;
    d.M = M;
    d.K = K;
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    if (qb::gemv_act_words(K) > kActScratchWords) return fail(QB_EINVAL, "K too large");
    cudaError_t e = qb::launch_gemv(d, st->act, st->err, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_gemv_q_dev", e);
}

int qwen_b200_gemv_rtl20_dev(int32_t* y_words, const float* x, const int16_t* xq, const float* xs,
                             const int8_t* mant, const uint8_t* exps, int M, int K, unsigned int* flags,
                             void* stream) {
    if ((x != nullptr) == (xq != nullptr) || (xq && !xs))
        return fail(QB_EINVAL, "qwen_b200_gemv_rtl20_dev: give x, or xq and xs");
    if (int rc = check_gemv_args(y_words, x ? (const void*)x : (const void*)xq, mant, exps, M, K)) return rc;
    qb::GemvDesc d{};
    d.mant = mant;
    d.exps = exps;
    d.x = x;
    d.xq = xq;
    d.xs = x ? nullptr : xs;
    d.y = reinterpret_cast<float*>(y_words);   // the kernels store each row's int32 word in these bits
    d.M = M;
    d.K = K;
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    if (qb::gemv_act_words(K) > kActScratchWords) return fail(QB_EINVAL, "K too large");
    cudaError_t e = qb::launch_gemv(d, st->act, st->err, static_cast<cudaStream_t>(stream), qb::kRtl20, flags);
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_gemv_rtl20_dev", e);
}

int qwen_b200_gemv_fast_dev(float* y, const float* x, const int8_t* mant, const uint8_t* exps, int M, int K,
                            void* stream) {
    if (int rc = check_gemv_args(y, x, mant, exps, M, K)) return rc;
    if (M == 0) return QB_OK;
    qb::GemvDesc d{};
    d.mant = mant;
    d.exps = exps;
    d.x = x;
    d.y = y;
    d.M = M;
    d.K = K;
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    cudaError_t e = qb::launch_gemv_fast(d, st->act, kActScratchWords, st->tickets, kTicketWords, st->err,
                                         static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue)
        return fail(QB_EINVAL, "gemv_fast: K must be a multiple of 512, mant/exps/x 16/4/8-byte aligned");
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_gemv_fast_dev", e);
}

int qwen_b200_quant_dev(const float* x, int B, int K, int16_t* xq, float* xs, void* stream) {
    if (!x || !xq || !xs || B < 0 || K <= 0 || K % 64) return fail(QB_EINVAL, "qwen_b200_quant_dev: bad arguments");
    cudaError_t e = qb::launch_quant_block64(x, B, K, xq, xs, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_quant_dev", e);
}

}  // extern "C"

namespace {

// QB_STACK_FIXED_SPLIT: K segments of 8 stages (2 KB of every row) -- short
// enough that the 1/8 shard of a deep matrix still fills the GPU, long
// enough that a whole matrix is not cut into needlessly many pieces.
constexpr int kFixedSegStages = 8;

struct PeerSpec {
    int world;
    const float* const* peer_y;   // n x (world - 1): the other ranks' full vectors per GEMV
    const int* row_base;          // n: global row of this rank's row 0
};

int stack_create_impl(int n, const int8_t* const* mant, const uint8_t* const* exps, const float* const* x,
                      float* const* y, const int* M, const int* K, int flags, const PeerSpec* ps) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (n <= 0 || !mant || !exps || !x || !y || !M || !K) return fail(QB_EINVAL, "stack: bad arguments");
    if (ps && (ps->world < 1 || ps->world > qb::kMaxRanks || (ps->world > 1 && !ps->peer_y) || !ps->row_base))
        return fail(QB_EINVAL, "stack: bad peer description");
    std::vector<qb::GemvDesc> v;
    std::vector<qb::PeerOut> peers;
    StackPlan sp;
    if (ps) {
        cudaError_t e = cudaMalloc(&sp.peers, sizeof(qb::PeerOut) * n);
        if (e != cudaSuccess) return fail(QB_ENOMEM, "stack peer alloc", e);
        if ((e = cudaMalloc(&sp.sig_ticket, sizeof(unsigned int))) != cudaSuccess)
            return fail(QB_ENOMEM, "stack ticket alloc", e);
        if ((e = cudaMemset(sp.sig_ticket, 0, sizeof(unsigned int))) != cudaSuccess)
            return fail(QB_ECUDA, "stack ticket clear", e);
    }
    for (int i = 0; i < n; i++) {
        if (M[i] < 0 || K[i] <= 0 || K[i] % 64 || !mant[i] || !exps[i] || !x[i] || !y[i])
            return fail(QB_EINVAL, "stack: bad descriptor");
        qb::PeerOut po{};
        if (ps) {
            po.n = ps->world - 1;
            po.row_base = ps->row_base[i];
            for (int r = 0; r + 1 < ps->world; r++) {
                po.y[r] = const_cast<float*>(ps->peer_y[(size_t)i * (ps->world - 1) + r]);
                if (!po.y[r]) return fail(QB_EINVAL, "stack: null peer vector");
            }
        }
        peers.push_back(po);
        if (M[i] == 0) continue;
        qb::GemvDesc d{};
        d.mant = mant[i];
        d.exps = exps[i];
        if (flags & QB_STACK_Q_INPUT) {   // x[i]: int16 xq [K], then fp32 xs [K/64]
            d.xq = reinterpret_cast<const int16_t*>(x[i]);
            d.xs = reinterpret_cast<const float*>(reinterpret_cast<const char*>(x[i]) + 2 * (size_t)K[i]);
        } else {
            d.x = x[i];
        }
        d.y = y[i];
        d.M = M[i];
        d.K = K[i];
        d.peer = ps ? sp.peers + i : nullptr;
        v.push_back(d);
    }
    const int mode = (flags & QB_STACK_FAST) ? qb::kFast : qb::kExact;
    const int fixed = (flags & QB_STACK_FIXED_SPLIT) ? kFixedSegStages : 0;
    if (!qb::gemv_plan(v.data(), (int)v.size(), nullptr, &sp.plan, mode, 0, nullptr, 0, fixed))
        return fail(QB_EINVAL, "stack: 1..160 GEMVs, every K a multiple of 512, mant/exps/x 16/4/8-byte aligned");
    cudaError_t e = cudaMalloc(&sp.act, sp.plan.act_words * 4 + 16);
    if (e != cudaSuccess) return fail(QB_ENOMEM, "stack act alloc", e);
    if ((e = cudaMalloc(&sp.ctr, 2 * sizeof(unsigned int))) != cudaSuccess) return fail(QB_ENOMEM, "stack ctr alloc", e);
    if ((e = cudaMemset(sp.ctr, 0, 2 * sizeof(unsigned int))) != cudaSuccess)
        return fail(QB_ECUDA, "stack ctr clear", e);
    if ((e = cudaMemset(sp.act, 0, sp.plan.act_words * 4 + 16)) != cudaSuccess)
        return fail(QB_ECUDA, "stack act clear", e);
    qb::gemv_plan(v.data(), (int)v.size(), sp.act, &sp.plan, mode, 0, nullptr, 0, fixed);
    if (ps && (e = cudaMemcpy(sp.peers, peers.data(), sizeof(qb::PeerOut) * n, cudaMemcpyHostToDevice)) != cudaSuccess)
        return fail(QB_ECUDA, "stack peer upload", e);
    e = cudaMalloc(&sp.dev_descs, sizeof(qb::GemvDesc) * (v.size() ? v.size() : 1));
    if (e != cudaSuccess) return fail(QB_ENOMEM, "stack alloc", e);
    e = cudaMemcpy(sp.dev_descs, v.data(), sizeof(qb::GemvDesc) * v.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return fail(QB_ECUDA, "stack upload", e);
    sp.live = true;
    g_plans.push_back(sp);
    return (int)g_plans.size();
}

}  // namespace

extern "C" {

int qwen_b200_stack_create_ex(int n, const int8_t* const* mant, const uint8_t* const* exps, const float* const* x,
                              float* const* y, const int* M, const int* K, int flags) {
    return stack_create_impl(n, mant, exps, x, y, M, K, flags, nullptr);
}

int qwen_b200_stack_create_sharded(int n, const int8_t* const* mant, const uint8_t* const* exps,
                                   const float* const* x, float* const* y, const int* M, const int* K, int flags,
                                   int world, const float* const* peer_y, const int* row_base) {
    PeerSpec ps{world, peer_y, row_base};
    return stack_create_impl(n, mant, exps, x, y, M, K, flags, &ps);
}

int qwen_b200_stack_run_sync(int plan, void* stream, const unsigned int* wait_flags, unsigned int wait_epoch,
                             unsigned int* const* sig_flags, unsigned int sig_epoch, int world, int rank) {
    if (plan < 1 || plan > (int)g_plans.size() || !g_plans[plan - 1].live) return fail(QB_EINVAL, "stack: bad handle");
    const StackPlan& sp = g_plans[plan - 1];
    if (world < 1 || world > qb::kMaxRanks || rank < 0 || rank >= world || (sig_epoch && (!sig_flags || !sp.sig_ticket)) ||
        (wait_epoch && !wait_flags))
        return fail(QB_EINVAL, "stack_run_sync: bad arguments (a plan from qwen_b200_stack_create_sharded, "
                               "1 <= world <= 8)");
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    qb::SyncArgs sy{};
    sy.wait_flags = wait_flags;
    sy.wait_epoch = wait_epoch;
    sy.sig_ticket = sp.sig_ticket;
    sy.sig_epoch = sig_epoch;
    sy.world = world;
    sy.rank = rank;
    sy.epoch_base = st->epoch_base;
    for (int r = 0; r < world && sig_flags; r++) sy.sig_flags[r] = sig_flags[r];
    cudaError_t e =
        qb::launch_gemv_list(sp.dev_descs, sp.plan, sp.ctr, st->err, static_cast<cudaStream_t>(stream), &sy);
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_stack_run_sync", e);
}

int qwen_b200_swiglu_quant_sharded_dev(const float* gate, const float* up, int B, int n, int ld_in, int col0, int K,
                                       int planar, int ldxs, void* const* dst, int ndst, unsigned int* const* sig_flags,
                                       unsigned int* sig_ticket, unsigned int sig_epoch, const unsigned int* wait_flags,
                                       int world, int rank, void* stream) {
    if (sig_epoch && (!sig_flags || !sig_ticket || !wait_flags || world < 1 || world > qb::kMaxRanks || rank < 0 ||
                      rank >= world))
        return fail(QB_EINVAL, "swiglu_quant_sharded: a signal needs every rank's flags, a ticket and this GPU's "
                               "flags (1 <= world <= 8)");
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    qb::SyncArgs sy{};
    if (sig_epoch) {
        sy.wait_flags = wait_flags;
        sy.sig_ticket = sig_ticket;
        sy.sig_epoch = sig_epoch;
        sy.world = world;
        sy.rank = rank;
        sy.epoch_base = st->epoch_base;
        for (int r = 0; r < world; r++) sy.sig_flags[r] = sig_flags[r];
    }
    cudaError_t e = qb::launch_swiglu_quant(gate, up, B, n, ld_in, col0, K, planar, ldxs, dst, ndst,
                                            sig_epoch ? &sy : nullptr, st->err, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue)
        return fail(QB_EINVAL, "swiglu_quant_sharded: n, col0 and K multiples of 64 with col0 + n <= K, B == 1 unless "
                               "planar, ldxs >= B, gate/up 8-byte and every dst 16-byte aligned, 1..8 destinations");
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_swiglu_quant_sharded_dev", e);
}

int qwen_b200_sync_epoch_base(const unsigned int* base) {
    if (reinterpret_cast<uintptr_t>(base) & 3)
        return fail(QB_EINVAL, "qwen_b200_sync_epoch_base: the counter must be 4-byte aligned");
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    st->epoch_base = base;
    return QB_OK;
}

int qwen_b200_sync_epoch_advance(unsigned int* base, unsigned int n, void* stream) {
    cudaError_t e = qb::launch_epoch_advance(base, n, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue)
        return fail(QB_EINVAL, "qwen_b200_sync_epoch_advance: a 4-byte aligned device counter is required");
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_sync_epoch_advance", e);
}

int qwen_b200_dev_alloc(size_t bytes, void** out) {
    if (!out || !bytes) return fail(QB_EINVAL, "qwen_b200_dev_alloc: bad arguments");
    cudaError_t e = cudaMalloc(out, bytes);
    if (e != cudaSuccess) return fail(QB_ENOMEM, "qwen_b200_dev_alloc", e);
    if ((e = cudaMemset(*out, 0, bytes)) != cudaSuccess) return fail(QB_ECUDA, "qwen_b200_dev_alloc clear", e);
    return QB_OK;
}

int qwen_b200_dev_free(void* p) {
    cudaError_t e = cudaFree(p);
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_dev_free", e);
}

int qwen_b200_ipc_handle(const void* base, void* handle_out) {
    if (!base || !handle_out) return fail(QB_EINVAL, "qwen_b200_ipc_handle: bad arguments");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(base));
    if (e != cudaSuccess) return fail(QB_ECUDA, "cudaIpcGetMemHandle", e);
    std::memcpy(handle_out, &h, sizeof h);
    return QB_OK;
}

int qwen_b200_ipc_open(const void* handle, void** out) {
    if (!handle || !out) return fail(QB_EINVAL, "qwen_b200_ipc_open: bad arguments");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    cudaError_t e = cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "cudaIpcOpenMemHandle", e);
}

int qwen_b200_ipc_close(void* p) {
    cudaError_t e = cudaIpcCloseMemHandle(p);
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "cudaIpcCloseMemHandle", e);
}

int qwen_b200_stack_create(int n, const int8_t* const* mant, const uint8_t* const* exps, const float* const* x,
                           float* const* y, const int* M, const int* K) {
    return qwen_b200_stack_create_ex(n, mant, exps, x, y, M, K, 0);
}

int qwen_b200_stack_run(int plan, void* stream) {
    if (plan < 1 || plan > (int)g_plans.size() || !g_plans[plan - 1].live) return fail(QB_EINVAL, "stack: bad handle");
    const StackPlan& sp = g_plans[plan - 1];
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    cudaError_t e = qb::launch_gemv_list(sp.dev_descs, sp.plan, sp.ctr, st->err, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_stack_run", e);
}

int qwen_b200_stack_destroy(int plan) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (plan < 1 || plan > (int)g_plans.size() || !g_plans[plan - 1].live) return fail(QB_EINVAL, "stack: bad handle");
    cudaFree(g_plans[plan - 1].dev_descs);
    cudaFree(g_plans[plan - 1].act);
    cudaFree(g_plans[plan - 1].ctr);
    cudaFree(g_plans[plan - 1].peers);
    cudaFree(g_plans[plan - 1].sig_ticket);
    g_plans[plan - 1].live = false;
    g_plans[plan - 1].dev_descs = nullptr;
    return QB_OK;
}

int qwen_b200_device_error(int clear) {
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    unsigned int v = 0;
    cudaError_t e = cudaMemcpy(&v, st->err, sizeof v, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail(QB_ECUDA, "device error read", e);
    if (clear) cudaMemset(st->err, 0, sizeof v);
    return (int)v;
}

int qwen_b200_lm_head_bf16_dev(const float* h, const uint16_t* E, int vocab, int hidden, int k, int* out_id,
                               int* out_ids, float* out_scores, int* out_n, void* stream) {
    if (!h || !E || !out_id || vocab <= 0 || hidden <= 0 || k < 0) return fail(QB_EINVAL, "lm_head_bf16: bad arguments");
    if (k > 0 && (!out_ids || !out_scores || !out_n)) return fail(QB_EINVAL, "lm_head_bf16: null outputs");
    if ((k < vocab ? k : vocab) > qb::kTopkMax) return fail(QB_EINVAL, "lm_head_bf16: k above 1024");
    if (hidden % 8 || reinterpret_cast<uintptr_t>(E) % 16 || reinterpret_cast<uintptr_t>(h) % 8)
        return fail(QB_EINVAL, "lm_head_bf16_dev: hidden must be a multiple of 8, E 16-byte and h 8-byte aligned");
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    cudaError_t e = qb::launch_lm_head_bf16(h, E, vocab, hidden, k, 1, st->scratch, st->err, nullptr, out_id,
                                            out_ids, out_scores, out_n, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_lm_head_bf16_dev", e);
}

int qwen_b200_sample_topk_dev(const int* ids, const float* scores, const int* n_dev, int n, float temperature,
                              int top_k, float top_p, unsigned int* rng_state, int* out_id, void* stream) {
    if (!ids || !scores || !out_id || n < 0 || n > qb::kSampleMax)
        return fail(QB_EINVAL, "qwen_b200_sample_topk_dev: null list or output, or n outside 0..1024");
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    qb::SampleArgs a{ids, scores, n_dev, n, temperature, top_k, top_p, rng_state, out_id};
    cudaError_t e = qb::launch_sample_topk(a, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_sample_topk_dev", e);
}

int qwen_b200_lm_head_bfp8_dev(const float* h, const int8_t* mant, const uint8_t* exps, int vocab, int hidden,
                               int k, int* out_id, int* out_ids, float* out_scores, int* out_n, void* stream) {
    if (!h || !mant || !exps || !out_id || vocab <= 0 || hidden <= 0 || k < 0)
        return fail(QB_EINVAL, "lm_head_bfp8: bad arguments");
    if (k > 0 && (!out_ids || !out_scores || !out_n)) return fail(QB_EINVAL, "lm_head_bfp8: null outputs");
    if ((k < vocab ? k : vocab) > qb::kTopkMax) return fail(QB_EINVAL, "lm_head_bfp8: k above 1024");
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    if (qb::gemv_act_words(hidden) > kActScratchWords) return fail(QB_EINVAL, "lm_head_bfp8: hidden too large");
    cudaError_t e = qb::launch_bfp8_lm_head(h, mant, exps, vocab, hidden, k, st->scratch, st->act, st->lm_ctr, st->err,
                                            out_id,
                                            out_ids, out_scores, out_n, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue)
        return fail(QB_EINVAL, "lm_head_bfp8: hidden must be a multiple of 512, mant/exps/h 16/4/8-byte aligned, "
                               "and at most 2048 vocab rows per SM");
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_lm_head_bfp8_dev", e);
}

int qwen_b200_quant_planes_dev(const float* x, int B, int K, int8_t* planes, float* xs_t, int ldxs, void* stream) {
    if (!x || !planes || !xs_t || B <= 0 || K <= 0 || K % 64 || ldxs < B)
        return fail(QB_EINVAL, "qwen_b200_quant_planes_dev: bad arguments");
    if ((reinterpret_cast<uintptr_t>(x) & 7) || (reinterpret_cast<uintptr_t>(planes) & 1))
        return fail(QB_EINVAL, "qwen_b200_quant_planes_dev: x must be 8-byte and planes 2-byte aligned");
    cudaError_t e = qb::launch_quant_planes(x, B, K, planes, xs_t, ldxs, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_quant_planes_dev", e);
}

int qwen_b200_gemm_tc_dev(float* y, const int8_t* planes, const float* xs_t, int ldxs, const int8_t* mant,
                          const uint8_t* exps, int M, int K, int B, int32_t* dots, void* stream) {
    if (M == 0 || B == 0) return QB_OK;
    qb::TcDesc d;
    if (M < 0 || B < 0 || !qb::tc_make_desc(&d, y, planes, xs_t, ldxs, mant, exps, M, K, B, dots))
        return fail(QB_EINVAL, "qwen_b200_gemm_tc_dev: K a positive multiple of 64, planes/xs_t/mant 16-byte "
                               "aligned, ldxs >= B and a multiple of 4");
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    cudaError_t e = qb::launch_gemm_tc(nullptr, &d, 1, qb::tc_units(d), B, dots != nullptr, st->err,
                                       static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_gemm_tc_dev", e);
}

}  // extern "C"

namespace {

int tc_stack_create_impl(int n, const int8_t* const* mant, const uint8_t* const* exps, const int8_t* const* planes,
                         const float* const* xs_t, float* const* y, const int* M, const int* K, const int* ldy, int B,
                         int ldxs, const PeerSpec* ps) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (n <= 0 || n > 4096 || !mant || !exps || !planes || !xs_t || !y || !M || !K || B <= 0)
        return fail(QB_EINVAL, "tc_stack: bad arguments");
    if (ps && (ps->world < 1 || ps->world > qb::kMaxRanks || (ps->world > 1 && !ps->peer_y) || !ps->row_base))
        return fail(QB_EINVAL, "tc_stack: bad peer description");
    TcPlan tp;
    std::vector<qb::PeerOut> peers(ps ? n : 0);
    if (ps) {
        cudaError_t e = cudaMalloc(&tp.peers, sizeof(qb::PeerOut) * n);
        if (e != cudaSuccess) return fail(QB_ENOMEM, "tc_stack peer alloc", e);
        if ((e = cudaMalloc(&tp.sig_ticket, sizeof(unsigned int))) != cudaSuccess)
            return fail(QB_ENOMEM, "tc_stack ticket alloc", e);
        if ((e = cudaMemset(tp.sig_ticket, 0, sizeof(unsigned int))) != cudaSuccess)
            return fail(QB_ECUDA, "tc_stack ticket clear", e);
    }
    std::vector<qb::TcDesc> v;
    for (int i = 0; i < n; i++) {
        if (ps) {
            qb::PeerOut& po = peers[i];
            po = qb::PeerOut{};
            po.n = ps->world - 1;
            po.row_base = ps->row_base[i];
            for (int r = 0; r + 1 < ps->world; r++) {
                po.y[r] = const_cast<float*>(ps->peer_y[(size_t)i * (ps->world - 1) + r]);
                if (!po.y[r]) return fail(QB_EINVAL, "tc_stack: null peer output");
            }
        }
        if (M[i] == 0) continue;
        qb::TcDesc d;
        if (M[i] < 0 || (ldy && ldy[i] < M[i]) ||
            !qb::tc_make_desc(&d, y[i], planes[i], xs_t[i], ldxs, mant[i], exps[i], M[i], K[i], B, nullptr,
                              ldy ? ldy[i] : 0))
            return fail(QB_EINVAL, "tc_stack: bad descriptor (K a multiple of 64, 16-byte aligned planes/xs_t/"
                                   "mant, ldxs >= B and a multiple of 4, ldy >= M)");
        d.peer = ps ? tp.peers + i : nullptr;
        v.push_back(d);
    }
    if (ps && (cudaMemcpy(tp.peers, peers.data(), sizeof(qb::PeerOut) * n, cudaMemcpyHostToDevice) != cudaSuccess))
        return fail(QB_ECUDA, "tc_stack peer upload");
    // deepest matrices first, so the round-robin tail is made of short units
    std::stable_sort(v.begin(), v.end(), [](const qb::TcDesc& a, const qb::TcDesc& b) { return a.K > b.K; });
    // stream-K launches: every CTA an equal share of the K stages
    int max_tiles = 0, max_grid = 0;
    for (int first = 0; first < (int)v.size(); first += qb::kTcMaxDescs) {
        TcLaunchPart part{first, std::min(qb::kTcMaxDescs, (int)v.size() - first), 0, 0};
        long long stages = 0;
        for (int k = first; k < first + part.n; k++) {
            v[k].unit_begin = part.total_units;
            v[k].tile_begin = part.total_units;
            stages += qb::tc_stages(v[k]);
            part.total_units += qb::tc_units(v[k]);
        }
        if (stages > (1ll << 30)) return fail(QB_EINVAL, "tc_stack: too much work for one launch");
        if (qb::tc_prefer_streamk(part.total_units)) {
            long long st = 0;
            for (int k = first; k < first + part.n; k++) {
                v[k].unit_begin = (int)st;
                st += qb::tc_stages(v[k]);
            }
            part.total_stages = (int)stages;
            max_tiles = std::max(max_tiles, part.total_units);
            max_grid = std::max(max_grid, qb::tc_streamk_grid(part.total_stages));
        }
        tp.parts.push_back(part);
    }
    tp.B = B;
    if (max_grid > 0) {
        cudaError_t e2 = cudaMalloc(&tp.partial, (size_t)2 * max_grid * B * qb::kTcTileRowsPublic * sizeof(float));
        if (e2 != cudaSuccess) return fail(QB_ENOMEM, "tc_stack partial alloc", e2);
        const size_t tb = (size_t)max_tiles * qb::kTcTicketsPerTile * sizeof(unsigned int);
        if ((e2 = cudaMalloc(&tp.sk_tickets, tb)) != cudaSuccess) return fail(QB_ENOMEM, "tc_stack ticket alloc", e2);
        if ((e2 = cudaMemset(tp.sk_tickets, 0, tb)) != cudaSuccess) return fail(QB_ECUDA, "tc_stack ticket clear", e2);
    }
    cudaError_t e = cudaMalloc(&tp.dev_descs, sizeof(qb::TcDesc) * (v.empty() ? 1 : v.size()));
    if (e != cudaSuccess) return fail(QB_ENOMEM, "tc_stack alloc", e);
    if (!v.empty() &&
        (e = cudaMemcpy(tp.dev_descs, v.data(), sizeof(qb::TcDesc) * v.size(), cudaMemcpyHostToDevice)) != cudaSuccess)
        return fail(QB_ECUDA, "tc_stack upload", e);
    tp.live = true;
    g_tc_plans.push_back(tp);
    return (int)g_tc_plans.size();
}

int tc_stack_launch(int plan, void* stream, const qb::SyncArgs* sync) {
    if (plan < 1 || plan > (int)g_tc_plans.size() || !g_tc_plans[plan - 1].live)
        return fail(QB_EINVAL, "tc_stack: bad handle");
    const TcPlan& tp = g_tc_plans[plan - 1];
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    for (size_t k = 0; k < tp.parts.size(); k++) {
        const TcLaunchPart& part = tp.parts[k];
        // the completion signal rides on the last launch (the others finish before it starts)
        const qb::SyncArgs* s = k + 1 == tp.parts.size() ? sync : nullptr;
        const qb::TcStreamK sk{tp.partial, tp.sk_tickets, part.total_stages};
        cudaError_t e = qb::launch_gemm_tc(tp.dev_descs + part.first, nullptr, part.n, part.total_units, tp.B, false,
                                           st->err, static_cast<cudaStream_t>(stream), s,
                                           part.total_stages ? &sk : nullptr);
        if (e != cudaSuccess) return fail(QB_ECUDA, "qwen_b200_tc_stack_run", e);
    }
    return QB_OK;
}

}  // namespace

extern "C" {

int qwen_b200_tc_stack_create(int n, const int8_t* const* mant, const uint8_t* const* exps,
                              const int8_t* const* planes, const float* const* xs_t, float* const* y, const int* M,
                              const int* K, int B, int ldxs) {
    return tc_stack_create_impl(n, mant, exps, planes, xs_t, y, M, K, nullptr, B, ldxs, nullptr);
}

int qwen_b200_tc_stack_create_sharded(int n, const int8_t* const* mant, const uint8_t* const* exps,
                                      const int8_t* const* planes, const float* const* xs_t, float* const* y,
                                      const int* M, const int* K, const int* ldy, int B, int ldxs, int world,
                                      const float* const* peer_y, const int* row_base) {
    if (!ldy) return fail(QB_EINVAL, "tc_stack_create_sharded: ldy is required");
    PeerSpec ps{world, peer_y, row_base};
    return tc_stack_create_impl(n, mant, exps, planes, xs_t, y, M, K, ldy, B, ldxs, &ps);
}

int qwen_b200_tc_stack_run_sync(int plan, void* stream, unsigned int* const* sig_flags, unsigned int sig_epoch,
                                int world, int rank) {
    if (plan < 1 || plan > (int)g_tc_plans.size() || !g_tc_plans[plan - 1].live)
        return fail(QB_EINVAL, "tc_stack: bad handle");
    const TcPlan& tp = g_tc_plans[plan - 1];
    if (world < 1 || world > qb::kMaxRanks || rank < 0 || rank >= world ||
        (sig_epoch && (!sig_flags || !tp.sig_ticket)))
        return fail(QB_EINVAL, "tc_stack_run_sync: bad arguments (a plan from qwen_b200_tc_stack_create_sharded, "
                               "1 <= world <= 8)");
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    qb::SyncArgs sy{};
    sy.sig_ticket = tp.sig_ticket;
    sy.sig_epoch = sig_epoch;
    sy.world = world;
    sy.rank = rank;
    sy.epoch_base = st->epoch_base;
    for (int r = 0; r < world && sig_flags; r++) sy.sig_flags[r] = sig_flags[r];
    return tc_stack_launch(plan, stream, &sy);
}

int qwen_b200_quant_planes_wait_dev(const float* x, int B, int K, int8_t* planes, float* xs_t, int ldxs,
                                    const unsigned int* wait_flags, unsigned int wait_epoch, int world,
                                    void* stream) {
    if (!x || !planes || !xs_t || B <= 0 || K <= 0 || K % 64 || ldxs < B || world < 1 || world > qb::kMaxRanks ||
        (wait_epoch && !wait_flags))
        return fail(QB_EINVAL, "qwen_b200_quant_planes_wait_dev: bad arguments");
    if ((reinterpret_cast<uintptr_t>(x) & 7) || (reinterpret_cast<uintptr_t>(planes) & 1))
        return fail(QB_EINVAL, "qwen_b200_quant_planes_wait_dev: x must be 8-byte and planes 2-byte aligned");
    DevState* st = nullptr;
    if (int rc = dev_state(&st)) return rc;
    qb::SyncArgs sy{};
    sy.wait_flags = wait_flags;
    sy.wait_epoch = wait_epoch;
    sy.world = world;
    sy.epoch_base = st->epoch_base;
    cudaError_t e = qb::launch_quant_planes(x, B, K, planes, xs_t, ldxs, static_cast<cudaStream_t>(stream), &sy,
                                            st->err);
    return e == cudaSuccess ? QB_OK : fail(QB_ECUDA, "qwen_b200_quant_planes_wait_dev", e);
}

int qwen_b200_tc_stack_run(int plan, void* stream) { return tc_stack_launch(plan, stream, nullptr); }

int qwen_b200_tc_stack_destroy(int plan) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (plan < 1 || plan > (int)g_tc_plans.size() || !g_tc_plans[plan - 1].live)
        return fail(QB_EINVAL, "tc_stack: bad handle");
    cudaFree(g_tc_plans[plan - 1].dev_descs);
    cudaFree(g_tc_plans[plan - 1].peers);
    cudaFree(g_tc_plans[plan - 1].sig_ticket);
    cudaFree(g_tc_plans[plan - 1].partial);
    cudaFree(g_tc_plans[plan - 1].sk_tickets);
    g_tc_plans[plan - 1].partial = nullptr;
    g_tc_plans[plan - 1].sk_tickets = nullptr;
    g_tc_plans[plan - 1].dev_descs = nullptr;
    g_tc_plans[plan - 1].peers = nullptr;
    g_tc_plans[plan - 1].sig_ticket = nullptr;
    g_tc_plans[plan - 1].live = false;
    return QB_OK;
}

}  // extern "C"
