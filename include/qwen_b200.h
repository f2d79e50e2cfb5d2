/*
 * qwen_b200.h -- C ABI of libqwen_kernels_b200.so, the B200 (sm_100a)
 * implementation of the BFP8 GEMV / lm_head decode hot path of
 * ideal1128/qwen35-ax7020-edge-llm.
 *
 * Two groups of entry points:
 *
 *  1. Drop-in replacements of the reference C kernels.  Same names, argument
 *     meaning and return conventions as the reference libraries the Python
 *     engine binds through ctypes; every pointer is a HOST pointer.  Weight
 *     and embedding pointers are translated to device copies: ranges
 *     registered with qwen_b200_register_weights() map by offset, any other
 *     pointer is uploaded on first use and cached by (address, size) -- a
 *     caller that rewrites a weight buffer in place must call
 *     qwen_b200_forget_weights() first.  Activations and outputs are copied
 *     in and out on every call, and the call returns after the result is on
 *     the host.
 *
 *  2. Device entry points (suffix _dev).  Every pointer is a device pointer
 *     on the current device, `stream` is a cudaStream_t (NULL = legacy
 *     default stream), nothing is synchronised.  They return 0 on success or
 *     a negative QB_E* code; qwen_b200_last_error() describes the last
 *     failure of the calling thread.
 *
 * Weight layout (both groups): block-64 BFP8 SoA as written by the reference
 * packer (05-主机侧源码/bfp8_packer.py:53-86): mantissas int8 [M][K]
 * row-major, then exponents uint8 [M][K/64]; a weight's value is
 * m * 2^(e-134).  K must be a positive multiple of 64.
 *
 * Numerics: every entry point reproduces the reference's NEON build
 * bit-for-bit (activation quantization 04-板载脚本与工具/qwen_kernels_opt.c:
 * 182-205, GEMV float order :213-308, lm_head order :401-488,
 * top-k order qwen_sampling.c:117-155,283-353), for any K.
 */
#ifndef QWEN_B200_H
#define QWEN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QB_API __attribute__((visibility("default")))
#else
#define QB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define QB_OK 0
#define QB_EINVAL (-1)   /* bad argument (shape, null pointer, k out of range) */
#define QB_ECUDA (-2)    /* CUDA runtime error */
#define QB_ENOMEM (-3)   /* device allocation failed */
#define QB_ENODEV (-4)   /* no usable CUDA device */

/* ------------------------------------------------ 1. reference drop-ins */

/* Replaces init_kernels() (04-板载脚本与工具/qwen_kernels_opt.c:128-135;
 * called from qwen_real_engine.py:667-668).  Idempotent: selects the device
 * (QWEN_B200_DEVICE, default 0), creates the stream and scratch.  Every other
 * entry point calls it on first use. */
QB_API void init_kernels(void);

/* Replaces bfp8_gemv() (qwen_kernels_opt.c:207-326; callers
 * qwen_kernels_opt.c:946-1001, qwen_real_engine.py:1073-1087,1108-1165,
 * 1226-1232).  y[M] = BFP8 GEMV of x[K]; y is fully overwritten.  Unlike the
 * reference it keeps no static activation cache, so it is reentrant across
 * threads and never returns a stale quantization.  On error y is left
 * unchanged and qwen_b200_last_error() says why (the reference has no error
 * channel). */
QB_API void bfp8_gemv(float* y, const float* x, const int8_t* mantissas, const uint8_t* exps, int M, int K);

/* Replaces lm_head_argmax() (qwen_kernels_opt.c:401-506; callers
 * qwen_kernels_opt.c:1046, qwen_real_engine.py:1301).  Returns the id with
 * the largest score h . bf16(embed[id]); ties -> lowest id; 0 if no score
 * exceeds -1e30.  Returns -1 on error. */
QB_API int lm_head_argmax(const float* h, const uint16_t* embed_table, int vocab_size, int hidden_dim);

/* Replaces lm_head_topk() (04-板载脚本与工具/qwen_sampling.c:283-353; caller
 * chat_v3.py:151-155,180-181).  Writes the min(k, vocab) best (id, score)
 * pairs sorted by score descending, ties by ascending id, and returns their
 * number; 0 on invalid arguments.  Any k: k <= 1024 runs the fused scan,
 * larger k scores every row on the device and sorts (score, id) keys there. */
QB_API int lm_head_topk(const float* h, const uint16_t* embed_table, int vocab_size, int hidden_dim, int k,
                 int* out_ids, float* out_scores);

/* Replaces sample_from_topk() (qwen_sampling.c:411-529; caller
 * chat_v3.py:156-160,184-187).  Host-side temperature / top-k / top-p
 * sampling with the reference's xorshift32 stream; same results as the
 * reference for the same arguments and rng_state. */
QB_API int sample_from_topk(const int* ids, const float* scores, int n, float temperature, int top_k,
                     float top_p, unsigned int* rng_state);

/* The per-layer plans the engine hands the reference's C token loop,
 * field for field and byte for byte its ctypes layouts
 * (04-板载脚本与工具/qwen_real_engine.py:20-57 LinearLayerPlanC, :59-74
 * MlpPlanC; qwen_kernels_opt.c:866-917).  All pointers are host pointers:
 * weight slices of the mapped weight file, fp32 norm vectors. */
typedef struct {
    const float* in_ln_w;
    const int8_t* mant_qkv;
    const uint8_t* exp_qkv;
    int M_qkv;
    int K_qkv;
    const float* conv_w;
    float* conv_s;
    const float* wa;
    const float* wb;
    const float* nea;
    const float* dt;
    float* state;
    const int8_t* mant_z;
    const uint8_t* exp_z;
    int M_z;
    int K_z;
    const float* norm_w;
    const int8_t* mant_o;
    const uint8_t* exp_o;
    int M_o;
    int K_o;
    const float* post_ln_w;
    const int8_t* mant_gate;
    const uint8_t* exp_gate;
    int M_gate;
    int K_gate;
    const int8_t* mant_up;
    const uint8_t* exp_up;
    int M_up;
    int K_up;
    const int8_t* mant_down;
    const uint8_t* exp_down;
    int M_down;
    int K_down;
} LinearLayerPlanC;

typedef struct {
    const float* post_ln_w;
    const int8_t* mant_gate;
    const uint8_t* exp_gate;
    int M_gate;
    int K_gate;
    const int8_t* mant_up;
    const uint8_t* exp_up;
    int M_up;
    int K_up;
    const int8_t* mant_down;
    const uint8_t* exp_down;
    int M_down;
    int K_down;
} MlpPlanC;

/* Replaces forward_mlp() (qwen_kernels_opt.c:994-1003; caller
 * qwen_real_engine.py:1152-1153): h += down(swiglu(gate(n), up(n))) with
 * n = rmsnorm(h, post_ln_w, 1e-6) -- the reference's NEON-build rmsnorm,
 * GEMVs, swiglu and add_residual, bit for bit -- as two launches on the
 * device (gate and up together with the rmsnorm in front; down with swiglu
 * in front and the residual add folded into its stores); h (host, K_gate floats) is copied in and back, weight and
 * norm pointers are translated like bfp8_gemv's.  K_gate == K_up <= 6144,
 * M_gate == M_up == K_down, M_down == K_gate, multiples of 512.  On error h
 * is unchanged and qwen_b200_last_error() says why. */
QB_API void forward_mlp(const MlpPlanC* p, float* h);

/* Replaces forward_linear_layer() (qwen_kernels_opt.c:938-992; caller
 * qwen_real_engine.py:1096): one Gated-DeltaNet layer on the device in
 * five launches -- the qkv and z projections of rmsnorm(h, in_ln_w)
 * (one launch), one kernel for conv1d + SiLU, q/k l2 norm, the gates, the
 * recurrent step and rmsnorm_gated (one CTA per head), the out projection,
 * then the MLP with h + o formed in front of its gate and up projections
 * and the down rows added into it as they are stored.  NEON-build
 * order throughout (the GEMVs bit for bit); the gates and the gated norm's
 * SiLU use CUDA's expf / log1pf where the reference calls the C library's.
 * Shapes: K_qkv == K_z == M_o == K_gate <= 6144 (a multiple of 512),
 * M_qkv == 3 * M_z, M_z == K_o a multiple of 128 (heads = M_z / 128), the
 * MLP as forward_mlp's.  conv_s (3 x M_qkv floats) and state (heads x 128 x
 * 128 floats, the reference's blocked layout) are the engine's host arrays
 * and are updated in place (state mode below).  fp32 vectors and weights
 * resolve like bfp8_gemv's pointers (uploaded on first sight and kept: a
 * vector rewritten in place needs qwen_b200_forget_weights()).  On error h
 * and the states are unchanged and qwen_b200_last_error() says why. */
QB_API void forward_linear_layer(const LinearLayerPlanC* p, float* h);

/* The callback forward_token_c runs for a full-attention layer
 * (qwen_kernels_opt.c:1006; qwen_real_engine.py:982): layer index, the
 * host h to update in place, the caller's context. */
typedef void (*QbFullAttnCallback)(int layer_idx, float* h, void* py_context);

/* Replaces forward_token_c() (qwen_kernels_opt.c:1008-1049; caller
 * qwen_real_engine.py:1262-1272): h = the bf16 embedding row of
 * token_id % 65536; 24 layers -- a full-attention layer (layer_is_full[l])
 * runs full_attn_cb on the host h (copied out; the callback may call
 * bfp8_gemv, the lm_head and sampler drop-ins -- forward_mlp,
 * forward_linear_layer and forward_token_c refuse to run inside it -- then
 * copied back in), then forward_mlp with
 * mlp_plans[l]; the others forward_linear_layer with the next of
 * linear_plans; then the final rmsnorm and the lm_head argmax over the
 * 65536 embedding rows.  h stays on the device between layers; on return it
 * holds the last residual stream.  Returns the token id, or -1 (h and the
 * states unchanged unless the failure came after a callback) with
 * qwen_b200_last_error().  Hidden size 1024, as the reference's loop.  Not
 * reentrant across threads (neither is the reference's static workspace). */
QB_API int forward_token_c(int token_id, float* h, const LinearLayerPlanC* linear_plans, const MlpPlanC* mlp_plans,
                           const int* layer_is_full, const float* final_norm_w, const uint16_t* embed_table,
                           QbFullAttnCallback full_attn_cb, void* py_context);

/* Gated-DeltaNet state handling (no reference counterpart).
 *   mode 0 (the default, the reference's contract): every
 *     forward_linear_layer / forward_token_c call copies each layer's conv_s
 *     and state host arrays to the device before its work and back after it
 *     (19.3 MB each way per token for the 0.8B model).  forward_token_c
 *     reads every layer's arrays into a page-locked staging buffer of its
 *     own (several host threads; QWEN_B200_COPY_THREADS, default up to 4)
 *     before the first layer, copies between that buffer and the device
 *     beside the layers, and writes each layer's arrays back once its copy
 *     out has landed (while it waits for the GPU; all before it returns);
 *     forward_linear_layer copies the arrays directly (pageable);
 *   mode 1 (resident): the device copy, made on first sight after entering
 *     the mode, is the state; the host arrays are written only by
 *     qwen_b200_gdn_state_sync() and when leaving the mode;
 *   mode 2 (pinned mirror): mode 0 with the host arrays page-locked in place
 *     on first sight, so the copies run as asynchronous DMA beside the
 *     layers.  The arrays stay registered until qwen_b200_gdn_state_drop() or
 *     a mode change: a caller that frees a state array calls _drop() first.
 * A caller that resets or rewrites its state arrays in mode 1 calls
 * qwen_b200_gdn_state_drop() first, so the next call re-reads them.  Every
 * mode change starts from the host arrays.  Return 0 or a QB_E* code. */
QB_API int qwen_b200_gdn_state_mode(int mode);
QB_API int qwen_b200_gdn_state_sync(void);
QB_API void qwen_b200_gdn_state_drop(void);

/* Replace the stage profiler (qwen_kernels_opt.c:71-91; read by
 * qwen_real_engine.py:1008-1047 when QWEN_PROFILE=1).  Slots accumulate
 * host wall milliseconds per entry point. */
QB_API void qwen_prof_enable(int on);
QB_API void qwen_prof_reset(void);
QB_API int qwen_prof_count(void);
QB_API double qwen_prof_get(int i);
QB_API const char* qwen_prof_name(int i);

/* ------------------------------------------------ weight registry */

/* Upload [host_base, host_base + nbytes) once (e.g. the whole mmap'd weight
 * file or the embedding file); later drop-in calls whose pointers fall inside
 * it use the device copy.  Returns 0 or a QB_E* code.  No reference
 * counterpart: the reference reads the mmap directly. */
QB_API int qwen_b200_register_weights(const void* host_base, size_t nbytes);
/* Drop every registration or cached upload that contains `host_ptr`. */
QB_API int qwen_b200_forget_weights(const void* host_ptr);
/* Drop everything. */
QB_API void qwen_b200_reset_weights(void);

/* ------------------------------------------------ 2. device entry points */

/* y[M] = exact BFP8 GEMV of fp32 x[K] (quantized in-kernel by the reference
 * rule).  Device form of bfp8_gemv(). */
QB_API int qwen_b200_gemv_dev(float* y, const float* x, const int8_t* mant, const uint8_t* exps, int M, int K,
                       void* stream);

/* y[M] = exact BFP8 GEMV of rmsnorm(x, norm_w, eps) in one launch: the
 * reference's rmsnorm (qwen_kernels_opt.c:140-172, NEON build order: four
 * flushed lane sums of x*x, r = 1/sqrtf(sum/K + eps), x * (r * (1 + w))),
 * then its quantizer and GEMV, bit for bit -- the rmsnorm -> bfp8_gemv pair
 * forward_token_c runs before the attention and MLP projections
 * (qwen_kernels_opt.c:946-1001), without the normalized vector leaving the
 * SM.  K a multiple of 512 and <= 6144; x and norm_w 8-byte aligned. */
QB_API int qwen_b200_rmsnorm_gemv_dev(float* y, const float* x, const float* norm_w, float eps, const int8_t* mant,
                                      const uint8_t* exps, int M, int K, void* stream);

/* The residual step in front of it as well: x_out = x + res (the reference's
 * add_residual, qwen_kernels_opt.c:388-396, flushed vector adds -- the
 * residual-stream update forward_token_c makes after each attention and MLP
 * block), then y = qwen_b200_rmsnorm_gemv_dev of x_out, in one launch.
 * x_out must not overlap x or res (the reference updates x in place; here
 * every CTA reads x while one writes x_out). */
QB_API int qwen_b200_residual_rmsnorm_gemv_dev(float* y, float* x_out, const float* x, const float* res,
                                               const float* norm_w, float eps, const int8_t* mant,
                                               const uint8_t* exps, int M, int K, void* stream);

/* Two projections of the same normalized vector in one launch: y0 = the
 * M0 x K GEMV and y1 = the M1 x K GEMV of rmsnorm(x, norm_w, eps) (or, with
 * res and x_out, of x + res, which is also stored to x_out) -- a
 * linear-attention layer's qkv and z projections, an MLP's gate and up
 * (qwen_kernels_opt.c:946,970,998-999); each bit for bit
 * qwen_b200_rmsnorm_gemv_dev / qwen_b200_residual_rmsnorm_gemv_dev of it.
 * Same conditions as those (K a multiple of 512 and <= 6144). */
QB_API int qwen_b200_rmsnorm_gemv2_dev(float* y0, float* y1, float* x_out, const float* x, const float* res,
                                       const float* norm_w, float eps, const int8_t* mant0, const uint8_t* exps0,
                                       int M0, const int8_t* mant1, const uint8_t* exps1, int M1, int K, void* stream);

/* The MLP's down projection with its SwiGLU in front, in one launch:
 * y = qwen_b200_gemv_dev of swiglu(gate, up), swiglu as the reference's NEON
 * build computes it (qwen_kernels_opt.c:332-386: exp_neon's clamp, range
 * reduction and degree-6 polynomial, flushed lanes, the division on VFP) --
 * the pair forward_linear_layer / forward_mlp run between the gate / up and
 * down GEMVs (:983-984, :1000-1001).  K a multiple of 512 and <= 6144;
 * mant 16-, exps 4-, gate / up 8-byte aligned. */
QB_API int qwen_b200_swiglu_gemv_dev(float* y, const float* gate, const float* up, const int8_t* mant,
                                     const uint8_t* exps, int M, int K, void* stream);

/* Same from an already quantized activation: xq int16 [K], xs fp32 [K/64]. */
QB_API int qwen_b200_gemv_q_dev(float* y, const int16_t* xq, const float* xs, const int8_t* mant,
                         const uint8_t* exps, int M, int K, void* stream);

/* Fast form of qwen_b200_gemv_dev(): per 64-block one exact int32 dot
 * product (the same int16 activation), then acc = fma(float(dot),
 * 2^(e-134)*xs, acc) over a K segment and the segments added in order, so a
 * matrix with few rows can be split along K across the whole GPU.
 * Deterministic; differs from the reference float order by at most
 * 1e-5 * sum_b |float(dot_b) * 2^(e_b-134) * xs_b| per row.  Needs K a
 * multiple of 512, mant 16-, exps 4-, x 8-byte aligned.  No reference
 * routine (the reference has only the NEON order). */
QB_API int qwen_b200_gemv_fast_dev(float* y, const float* x, const int8_t* mant, const uint8_t* exps, int M,
                                   int K, void* stream);

/* RTL dequant mode: the GEMV the FPGA gemv_core computes with dequant_en = 1
 * (02-RTL与仿真/gemv_core.v:299-534; the host side reads each word as
 * y * 2^-20).  Per row one int32 word floor(y * 2^20): every block's exact
 * int32 dot D times the 17-bit truncated mantissa of xs, shifted by
 * Ex + e - 110 (clamped to [-63, 63]) into a saturating 64-bit accumulator
 * with 40 fraction bits, clamped to the int32 range on output.  As in the
 * RTL's two-stage shifter, a shift below -63 moves right by
 * 7 + 8*((-sh >> 3) & 7) (its high stage reads the unclamped amount).  The
 * activation is fp32 x (quantized by quant_x_blocks) or, with x == NULL, an
 * already quantized xq int16 [K] / xs fp32 [K/64]; exactly one of the two.
 * `flags` (device word, may be NULL; the caller zeroes it) gets bit 0 when a
 * term or a row sum saturated and bit 1 when an output word was clamped
 * (the RTL's sticky saturation bit).  Integer arithmetic, bit-exact; any M,
 * K a positive multiple of 64. */
QB_API int qwen_b200_gemv_rtl20_dev(int32_t* y_words, const float* x, const int16_t* xq, const float* xs,
                                    const int8_t* mant, const uint8_t* exps, int M, int K, unsigned int* flags,
                                    void* stream);

/* Block-64 activation quantizer (quant_x_blocks, qwen_kernels_opt.c:182-205)
 * over B rows: x [B][K] -> xq int16 [B][K], xs [B][K/64]. */
QB_API int qwen_b200_quant_dev(const float* x, int B, int K, int16_t* xq, float* xs, void* stream);

/* Same GEMV as qwen_b200_gemv_dev(), for callers that cannot let a library
 * allocate device memory (a process whose allocator owns all of HBM, a
 * path that cannot afford cudaMalloc's device-wide synchronisation, a host
 * framework that only lends memory from its own pools).  Its scratch is a
 * fixed 33 KB array inside the library's device image, present on every GPU
 * that loads the library until the process exits; nothing is allocated or
 * freed.  K <= 16384 (QB_EINVAL beyond).  The first call on a device looks
 * up the array's device address; make that first call before any stream
 * capture.  All calls on a device share the array: calls that overlap on
 * the GPU (e.g. on two streams) race and must be serialised by the caller.
 * Bounded-wait timeouts are not recorded for qwen_b200_device_error().  No
 * counterpart in the reference. */
QB_API int qwen_b200_gemv_noalloc_dev(float* y, const float* x, const int8_t* mant, const uint8_t* exps, int M,
                                      int K, void* stream);

/* Grouped launch of n independent GEMVs (e.g. the per-token linear stack).
 * Arrays are HOST arrays of DEVICE pointers.  Returns a plan handle (>= 1)
 * or a QB_E* code; the plan owns its activation scratch and scheduler
 * counters, is reusable and can be launched inside CUDA graph capture.
 * 1 <= n <= 160; every mant pointer 16-byte aligned, every exps pointer
 * 4-byte aligned, every x 8-byte aligned, every K a multiple of 512.  Runs
 * of one plan must not overlap on the GPU (they share its scratch). */
QB_API int qwen_b200_stack_create(int n, const int8_t* const* mant, const uint8_t* const* exps,
                           const float* const* x, float* const* y, const int* M, const int* K);
/* Same with flags: QB_STACK_FAST selects the fast arithmetic of
 * qwen_b200_gemv_fast_dev() and lets rows of deep matrices be split into K
 * segments (for stacks with few rows per GPU, e.g. row-sharded ones). */
#define QB_STACK_FAST 1
/* With QB_STACK_FAST: cut every row's K into fixed 2 KB segments, so where a
 * row is split depends on K alone -- a row-sharded plan then gives every row
 * the same bits as the unsharded plan, on any number of GPUs. */
#define QB_STACK_FIXED_SPLIT 2
/* x[i] is an already quantized activation record: int16 xq [K] followed by
 * fp32 block scales xs [K/64] (16-byte aligned), as
 * qwen_b200_swiglu_quant_sharded_dev writes it. */
#define QB_STACK_Q_INPUT 4
QB_API int qwen_b200_stack_create_ex(int n, const int8_t* const* mant, const uint8_t* const* exps,
                              const float* const* x, float* const* y, const int* M, const int* K, int flags);
QB_API int qwen_b200_stack_run(int plan, void* stream);
QB_API int qwen_b200_stack_destroy(int plan);

/* ---- Row-sharded stacks over several GPUs of one node (one process per GPU).
 * Each rank owns rows [row_base[i], row_base[i] + M[i]) of GEMV i; y[i] points
 * at that row range inside this rank's full-length output vector, and
 * peer_y[i * (world - 1) + r] at the FULL output vector (row 0) of GEMV i on
 * the r-th other rank, mapped into this process (qwen_b200_ipc_open).  Every
 * row the kernel finishes is stored locally and into each peer vector, so no
 * separate all-gather runs.  Replaces the per-layer all-gather of the
 * distributed decode loop (layer outputs gathered across ranks before the
 * next layer's GEMVs read them). */
QB_API int qwen_b200_stack_create_sharded(int n, const int8_t* const* mant, const uint8_t* const* exps,
                                          const float* const* x, float* const* y, const int* M, const int* K,
                                          int flags, int world, const float* const* peer_y, const int* row_base);
/* One launch of a (sharded) plan with cross-GPU ordering.  With wait_epoch
 * != 0 the launch first spins (bounded; QB_ERR peer timeout in the error word)
 * until wait_flags[r] >= wait_epoch for every rank r < world (wrap-safe
 * compare), i.e. until every rank finished the launch its inputs come from.
 * With sig_epoch != 0 the last CTA of the launch stores sig_epoch into
 * sig_flags[r][rank] for every r < world (behind a system-scope fence) after all
 * rows reached every GPU.  sig_flags[r] is rank r's flag array (world uints),
 * wait_flags is this rank's own; epochs grow by one per launch on all ranks. */
QB_API int qwen_b200_stack_run_sync(int plan, void* stream, const unsigned int* wait_flags, unsigned int wait_epoch,
                                    unsigned int* const* sig_flags, unsigned int sig_epoch, int world, int rank);
/* The MLP activation of a row-sharded layer, computed shard-locally: this
 * rank holds elements [col0, col0 + n) of the gate and up projections of
 * each of B batch rows (row stride ld_in floats); every element gets the
 * reference's swiglu (NEON build, qwen_kernels_opt.c:332-386) and every
 * 64-block the reference quantizer (quant_x_blocks, :182-205) -- slices are
 * whole blocks, so the bits equal the unsharded activation's -- and the
 * quantized slice is stored into each of the ndst buffers (this GPU's input
 * of the down projection, then the other ranks' copies mapped with
 * qwen_b200_ipc_open): planar == 0 (B == 1) the record of QB_STACK_Q_INPUT
 * (xq int16 [K], xs fp32 [K/64]); planar == 1 the tcgen05 input, planes
 * int8 [2][B][K] then xs_t fp32 [K/64][ldxs].  Only int16 values and block
 * scales cross NVLink (2.06 bytes per element, not 2 x 4 for gate and up).
 * With sig_epoch != 0 the last CTA publishes sig_epoch into sig_flags[r][rank]
 * of every rank r (sig_ticket: a zeroed device word of this rank) and then
 * waits (bounded; error bit 2) until wait_flags[r] >= sig_epoch for every
 * rank, so a down projection launched after it on the stream reads a
 * complete input.  Replaces the reference's swiglu between the gate / up and
 * down GEMVs (qwen_kernels_opt.c:983-986) for a row-sharded layer. */
QB_API int qwen_b200_swiglu_quant_sharded_dev(const float* gate, const float* up, int B, int n, int ld_in, int col0,
                                              int K, int planar, int ldxs, void* const* dst, int ndst,
                                              unsigned int* const* sig_flags, unsigned int* sig_ticket,
                                              unsigned int sig_epoch, const unsigned int* wait_flags, int world,
                                              int rank, void* stream);
/* Epochs relative to a device counter, so that a CUDA graph capturing a
 * step of row-sharded launches can be replayed: after
 * qwen_b200_sync_epoch_base(base) (base: a 4-byte aligned device uint32 of
 * the current device; NULL restores absolute epochs), every nonzero wait /
 * signal epoch given to qwen_b200_stack_run_sync,
 * qwen_b200_swiglu_quant_sharded_dev, qwen_b200_tc_stack_run_sync and
 * qwen_b200_quant_planes_wait_dev on this device is an offset: the launch
 * reads *base when it runs and uses *base + offset (mod 2^32).  The setting
 * is per device and is taken when a launch is enqueued (a captured launch
 * keeps the counter it was captured with).  qwen_b200_sync_epoch_advance
 * enqueues *base += n on `stream` (one single-thread kernel): a step whose
 * launches use offsets 1..n ends with it, and the next step (or the next
 * replay of the step's graph) uses the same offsets.  No reference
 * counterpart (the reference runs on one device). */
QB_API int qwen_b200_sync_epoch_base(const unsigned int* base);
QB_API int qwen_b200_sync_epoch_advance(unsigned int* base, unsigned int n, void* stream);
/* Zeroed device memory that can be shared with qwen_b200_ipc_handle (plain
 * cudaMalloc: IPC needs the allocation's own base pointer). */
QB_API int qwen_b200_dev_alloc(size_t bytes, void** out);
QB_API int qwen_b200_dev_free(void* p);
/* 64-byte CUDA IPC handle of a qwen_b200_dev_alloc base; open it in another
 * process on the same node (peer access enabled lazily), close when done. */
QB_API int qwen_b200_ipc_handle(const void* base, void* handle_out);
QB_API int qwen_b200_ipc_open(const void* handle, void** out);
QB_API int qwen_b200_ipc_close(void* p);

/* ---- Batched decode on the tensor cores (B sequences share the weights).
 * Activations are int16 block-64 values stored as two signed int8 planes,
 * xq = 256*hi + lo (lo = low byte of xq as a signed int8, hi = (xq - lo)/256):
 * planes [2][B][K] bytes (plane 0 = hi, plane 1 = lo), 16-byte aligned, and
 * block scales xs_t [K/64][ldxs] fp32 (block-major, ldxs >= B, ldxs % 4 == 0).
 * The reference decodes one sequence at a time; these entry points have no
 * reference counterpart.  The block dots are exact; each output is the
 * exact sum_b dot_b * 2^(e_b-134) * xs_b up to one f32 rounding per block,
 * and agrees with bfp8_gemv() on that batch row to 1e-5 of the magnitude of
 * the reference's own lane-class terms, sum_{b,j} |L_j * 2^(e_b-134) * xs_b|. */

/* fp32 x [B][K] -> planes + xs_t with quant_x_blocks' arithmetic
 * (qwen_kernels_opt.c:182-205): 256*hi + lo equals its xq bit for bit. */
QB_API int qwen_b200_quant_planes_dev(const float* x, int B, int K, int8_t* planes, float* xs_t, int ldxs,
                                      void* stream);

/* y [B][M] = W (BFP8 [M][K], mant 16-byte aligned) x activations, on
 * tcgen05 kind::i8 (exact int32 block dots, hi and lo accumulators).  If
 * dots is not null the exact block dots are also written to it
 * ([B][M][K/64] int32, a verification aid; slower). */
QB_API int qwen_b200_gemm_tc_dev(float* y, const int8_t* planes, const float* xs_t, int ldxs, const int8_t* mant,
                                 const uint8_t* exps, int M, int K, int B, int32_t* dots, void* stream);

/* Grouped batched launch of n independent GEMMs with a common B and ldxs
 * (e.g. the per-step linear stack of B sequences).  HOST arrays of DEVICE
 * pointers; returns a plan handle (>= 1) or a QB_E* code.  1 <= n <= 4096; a run
 * is one launch per 160 GEMMs. */
QB_API int qwen_b200_tc_stack_create(int n, const int8_t* const* mant, const uint8_t* const* exps,
                                     const int8_t* const* planes, const float* const* xs_t, float* const* y,
                                     const int* M, const int* K, int B, int ldxs);
QB_API int qwen_b200_tc_stack_run(int plan, void* stream);
QB_API int qwen_b200_tc_stack_destroy(int plan);

/* Row-sharded batched stacks (one process per GPU, same protocol as
 * qwen_b200_stack_create_sharded): GEMM i writes rows [row_base[i],
 * row_base[i] + M[i]) of every batch row, y[i] + b * ldy[i] + r (y[i] already
 * offset to this rank's first row inside its full [B][ldy[i]] output), and
 * stores the same values at peer_y[i * (world - 1) + r] + b * ldy[i] +
 * row_base[i] + r on every other rank.  world 1 with peer_y NULL gives a
 * plain stack with strided outputs. */
QB_API int qwen_b200_tc_stack_create_sharded(int n, const int8_t* const* mant, const uint8_t* const* exps,
                                             const int8_t* const* planes, const float* const* xs_t,
                                             float* const* y, const int* M, const int* K, const int* ldy, int B,
                                             int ldxs, int world, const float* const* peer_y, const int* row_base);
/* One run of a sharded batched plan; with sig_epoch != 0 its last CTA
 * publishes sig_epoch into sig_flags[r][rank] for every rank r. */
QB_API int qwen_b200_tc_stack_run_sync(int plan, void* stream, unsigned int* const* sig_flags,
                                       unsigned int sig_epoch, int world, int rank);
/* qwen_b200_quant_planes_dev() that first waits (bounded; error bit 2) until
 * wait_flags[r] >= wait_epoch for every rank r < world: the quantizer of a
 * sharded batched layer reads the full outputs all ranks wrote. */
QB_API int qwen_b200_quant_planes_wait_dev(const float* x, int B, int K, int8_t* planes, float* xs_t, int ldxs,
                                           const unsigned int* wait_flags, unsigned int wait_epoch, int world,
                                           void* stream);

/* bf16 lm_head over E [vocab][hidden] (tied embedding).  Always writes the
 * greedy id to out_id[0]; for k > 0 also the top-k into out_ids/out_scores
 * and its length into out_n[0].  k <= 1024.  Device form of
 * lm_head_argmax() / lm_head_topk().  Calls on one device share a scratch
 * area: do not run two lm_head calls concurrently on different streams. */
QB_API int qwen_b200_lm_head_bf16_dev(const float* h, const uint16_t* E, int vocab, int hidden, int k,
                               int* out_id, int* out_ids, float* out_scores, int* out_n, void* stream);

/* Device form of sample_from_topk() (qwen_sampling.c:411-529): one warp on
 * `stream` samples from a DEVICE candidate list -- typically the ids /
 * scores / out_n a qwen_b200_lm_head_*_dev call just wrote -- and writes the
 * chosen id to out_id[0] (device), so the token never crosses to the host.
 * The list length is n, or min(n, *n_dev) when n_dev (device) is given;
 * n <= 1024.  rng_state is a DEVICE xorshift32 word updated in place (NULL:
 * ids[0], as the reference); an empty list writes -1.  Same procedure and
 * IEEE float / double operation order as the reference, with CUDA's expf in
 * place of the C library's: the token is the reference's except when a
 * draw lands within a few ulps of a bucket boundary; the rng state advances
 * identically. */
QB_API int qwen_b200_sample_topk_dev(const int* ids, const float* scores, const int* n_dev, int n,
                                     float temperature, int top_k, float top_p, unsigned int* rng_state,
                                     int* out_id, void* stream);

/* BFP8 lm_head (vocab x hidden BFP8 matrix): exact bfp8_gemv scores fused
 * with the same argmax / top-k rules; the scores never reach global memory.
 * No reference routine (the reference lm_head is bf16); same scratch rule. */
QB_API int qwen_b200_lm_head_bfp8_dev(const float* h, const int8_t* mant, const uint8_t* exps, int vocab,
                               int hidden, int k, int* out_id, int* out_ids, float* out_scores,
                               int* out_n, void* stream);

/* Block-64 BFP8 packer on the device: w fp32 [M][K] -> mant int8 [M][K],
 * exps uint8 [M][K/64], by the reference packer's rule
 * (05-主机侧源码/bfp8_packer.py:53-86) with ceil(log2(peak)) taken exactly
 * from the float's bits. */
QB_API int qwen_b200_pack_bfp8_dev(const float* w, int M, int K, int8_t* mant, uint8_t* exps, void* stream);

/* Error bits the kernels of the current device recorded (bounded waits that
 * timed out: 1 for a copy or pipeline barrier, 2 for a peer flag of
 * qwen_b200_stack_run_sync); 0 if none.  clear != 0 resets them.  No reference
 * counterpart. */
QB_API int qwen_b200_device_error(int clear);

/* Description of the calling thread's last failure ("" if none). */
QB_API const char* qwen_b200_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_B200_H */
