"""GPU parity of the quantizer and the exact BFP8 GEMV against the CPU oracle.

Bit-exact: int16 activations, block scales and every fp32 output (compared
as bit patterns), over the model's shapes, odd row counts, odd block counts,
extreme exponents and the grouped 150-GEMV stack.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def bits(a):
    """fp32 bit patterns; every NaN maps to one pattern (each platform has
    its own default NaN, so payloads are not compared)."""
    a = np.ascontiguousarray(a, np.float32)
    return np.where(np.isnan(a), np.uint32(0x7FC00000), a.view(np.uint32))


def rand_weights(rng, M, K, std=0.02, exp_range=None):
    w = rng.normal(0, std, (M, K)).astype(np.float32)
    mant, exps = O.pack_bfp8(w)
    if exp_range is not None:
        exps = rng.integers(exp_range[0], exp_range[1] + 1, exps.shape).astype(np.uint8)
        mant = rng.integers(-128, 128, mant.shape).astype(np.int8)
    return mant, exps


def to_dev(*arrs):
    import torch

    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]


# ------------------------------------------------------------------ quantizer
def test_quant_block64_bit_exact(cuda):
    from qwen_b200 import ops

    rng = np.random.default_rng(0)
    for K in (64, 1024, 3584, 64 * 37):
        x = rng.normal(0, 1, (3, K)).astype(np.float32)
        x[0, :64] = 0.0                           # zero block
        x[1, 64:128] = 1e-22                      # below the 1e-20 floor
        if K >= 256:
            x[2, 128:192] = rng.normal(0, 1e4, 64)   # large block
            x[2, 192:256] = np.arange(64, dtype=np.float32) * 0.5 - 16   # rounding ties
        xq, xs = ops.quant_block64(*to_dev(x))
        for r in range(3):
            q_ref, s_ref = O.quant_x(x[r])
            assert np.array_equal(xq[r].cpu().numpy(), q_ref), (K, r)
            assert np.array_equal(bits(xs[r].cpu().numpy()), bits(s_ref)), (K, r)


# ------------------------------------------------------------------ single GEMV
SHAPES = [(3584, 1024), (1024, 3584), (6144, 1024), (2048, 1024), (1024, 2048), (4096, 1024), (512, 1024),
          (1, 1024), (2, 512), (3, 512), (31, 1024), (33, 2048), (3583, 1024), (129, 4096), (64, 8192),
          (33, 6144), (100, 5632), (4737, 1536)]   # split kernel: 3 and 2 stages per warp; more groups than SMs


@pytest.mark.parametrize("M,K", SHAPES)
def test_gemv_exact_model_shapes(cuda, M, K):
    from qwen_b200 import ops

    rng = np.random.default_rng(M * 7919 + K)
    mant, exps = rand_weights(rng, M, K)
    x = rng.normal(0, 1, K).astype(np.float32)
    y = ops.bfp8_gemv(*to_dev(x, mant, exps)).cpu().numpy()
    assert np.array_equal(bits(y), bits(O.bfp8_gemv(x, mant, exps)))


@pytest.mark.parametrize("M,K", [(5, 64), (17, 192), (40, 64 * 23), (7, 64 * 9)])
def test_gemv_exact_generic_shapes(cuda, M, K):
    """K not a multiple of 512 runs the generic kernel; same bits."""
    from qwen_b200 import ops

    rng = np.random.default_rng(K + M)
    mant, exps = rand_weights(rng, M, K)
    x = rng.normal(0, 1, K).astype(np.float32)
    y = ops.bfp8_gemv(*to_dev(x, mant, exps)).cpu().numpy()
    assert np.array_equal(bits(y), bits(O.bfp8_gemv(x, mant, exps)))


@pytest.mark.parametrize("lo,hi", [(0, 12), (0, 255), (100, 140), (200, 255)])
def test_gemv_exact_extreme_exponents(cuda, lo, hi):
    """Subnormal block scales (e < 8, flushed on the vector path, kept on the
    odd row's scalar path), huge scales (inf), random mantissas incl. -128."""
    from qwen_b200 import ops

    rng = np.random.default_rng(lo * 256 + hi)
    for M, K in ((33, 1024), (64, 512)):
        mant, exps = rand_weights(rng, M, K, exp_range=(lo, hi))
        x = rng.normal(0, 1, K).astype(np.float32) * np.float32(10.0) ** rng.integers(-30, 30, K)
        y = ops.bfp8_gemv(*to_dev(x.astype(np.float32), mant, exps)).cpu().numpy()
        ref = O.bfp8_gemv(x.astype(np.float32), mant, exps)
        assert np.array_equal(bits(y), bits(ref)), (M, K)


def test_gemv_q_known_answer_constant_pattern(cuda):
    """01-系统概述/FINAL_REPORT.md:222-226: all-0x01 weights, all-0x1111 x ->
    every block sum 279616.  With unit block scales (e = 134, xs = 1) and one
    block per row the GEMV returns that sum exactly."""
    from qwen_b200 import ops

    M, K = 3584, 1024
    mant = np.ones((M, K), np.int8)
    exps = np.full((M, K // 64), 134, np.uint8)
    xq = np.full(K, 0x1111, np.int16)
    xs = np.ones(K // 64, np.float32)
    y = ops.bfp8_gemv_q(*to_dev(xq, xs, mant, exps)).cpu().numpy()
    assert (y == 279616.0 * (K // 64)).all()
    y1 = ops.bfp8_gemv_q(*to_dev(xq[:64], xs[:1], mant[:, :64].copy(), exps[:, :1].copy())).cpu().numpy()
    assert (y1 == 279616.0).all()


def test_gemv_q_tb_vectors(cuda, golden):
    """tb_gemv_core.v stimulus (LCG cases :401-419) through the quantized-input
    path: bit-exact against the oracle, and within the testbench tolerance
    of its double-precision model where the row does not saturate."""
    from qwen_b200 import ops

    g = golden("tb_gemv.npz")
    for i, (K, M, sd, dq, elo, ehi, xo, au, sat) in enumerate(g["cases"]):
        xq, xs, w, e = g[f"{i}_xq"], g[f"{i}_xs"], g[f"{i}_w"], g[f"{i}_e"]
        y = ops.bfp8_gemv_q(*to_dev(xq, xs, w, e)).cpu().numpy()
        assert np.array_equal(bits(y), bits(O.bfp8_gemv_q(xq, xs, w, e))), i


# ------------------------------------------------------------------ RTL dequant mode
def test_gemv_rtl20_tb_vectors(cuda, golden):
    """tb_gemv_core.v stimulus (:401-419) in the RTL dequant mode: words and
    sticky flags equal the oracle's (rails with the clamp flag on the
    saturation case, ~0 on the flush case)."""
    from qwen_b200 import ops

    g = golden("tb_gemv.npz")
    for i, (K, M, sd, dq, elo, ehi, xo, au, sat) in enumerate(g["cases"]):
        xq, xs, w, e = g[f"{i}_xq"], g[f"{i}_xs"], g[f"{i}_w"], g[f"{i}_e"]
        mant, exps, dq_, ds_ = to_dev(w, e, xq, xs)
        words, flags = ops.bfp8_gemv_rtl20(mant, exps, xq=dq_, xs=ds_)
        ref_w, ref_f = O.bfp8_gemv_rtl20(xq, xs, w, e)
        assert np.array_equal(words.cpu().numpy(), ref_w), i
        assert flags == ref_f, i


RTL_SHAPES = [(3584, 1024), (64, 8192), (33, 2048), (1, 512), (257, 6144), (5, 192), (40, 64 * 23)]


@pytest.mark.parametrize("M,K", RTL_SHAPES)
@pytest.mark.parametrize("sh_lo,sh_hi", [(-120, -50), (-30, 12), (20, 70)])
def test_gemv_rtl20_bit_exact(cuda, rtl_case, M, K, sh_lo, sh_hi):
    """Pre-quantized activations over flushing, normal and saturating shifts
    (and zero / subnormal / inf / NaN / negative block scales): words and
    flags bit-exact; warp kernel (K % 512 == 0, both activation paths) and
    generic kernel (other K)."""
    from qwen_b200 import ops

    rng = np.random.default_rng(M * 31 + K + sh_lo)
    mant, exps, xq, xs = rtl_case(rng, M, K, sh_lo, sh_hi, specials=True)
    dm, de, dq, ds = to_dev(mant, exps, xq, xs)
    words, flags = ops.bfp8_gemv_rtl20(dm, de, xq=dq, xs=ds)
    ref_w, ref_f = O.bfp8_gemv_rtl20(xq, xs, mant, exps)
    assert np.array_equal(words.cpu().numpy(), ref_w)
    assert flags == ref_f


@pytest.mark.parametrize("M,K", [(3584, 1024), (1024, 3584), (64, 8192), (17, 192)])
def test_gemv_rtl20_from_fp32(cuda, M, K):
    """fp32 activations quantized in the launch by the reference rule, then
    the dequant datapath: equal to the oracle's quantizer + dequant mode, and
    close to the float GEMV: the 17-bit truncated xs mantissa loses < 2^-16
    of each block term, the floors < 2^-19 in all."""
    from qwen_b200 import ops

    rng = np.random.default_rng(K + 3 * M)
    mant, exps = rand_weights(rng, M, K)
    x = rng.normal(0, 1, K).astype(np.float32)
    dx, dm, de = to_dev(x, mant, exps)
    words, flags = ops.bfp8_gemv_rtl20(dm, de, x=dx)
    xq, xs = O.quant_x(x)
    ref_w, ref_f = O.bfp8_gemv_rtl20(xq, xs, mant, exps)
    words = words.cpu().numpy()
    assert np.array_equal(words, ref_w) and flags == ref_f == 0
    y = O.bfp8_gemv(x, mant, exps).astype(np.float64)
    terms = np.abs(O.block_dots(mant, xq).astype(np.float64) * np.exp2(exps.astype(np.float64) - 134) * xs)
    assert (np.abs(words / 2.0**20 - y) <= 3e-5 * terms.sum(1) + 2.0**-19).all()


def test_gemv_rtl20_rejects_bad_activation_args(cuda):
    from qwen_b200 import ops

    mant, exps = to_dev(np.zeros((4, 64), np.int8), np.zeros((4, 1), np.uint8))
    with pytest.raises(ValueError):
        ops.bfp8_gemv_rtl20(mant, exps)


# ------------------------------------------------------------------ grouped stack
def test_linear_stack_full_token_bit_exact(cuda):
    """The 150 GEMVs of one Qwen3.5-0.8B token in one grouped launch."""
    import torch

    from qwen_b200 import model, ops

    st = model.DeviceStack(model.qwen35_08b_stack(), copies=1, seed=5)
    items = st.views(0)
    stack = ops.LinearStack(items)
    stack.run()
    torch.cuda.synchronize()
    for (x, mant, exps, y), t in zip(items, st.stack):
        ref = O.bfp8_gemv(x.cpu().numpy(), mant.cpu().numpy(), exps.cpu().numpy())
        assert np.array_equal(bits(y.cpu().numpy()), bits(ref)), t.name
    stack.close()


def test_linear_stack_in_cuda_graph(cuda):
    import torch

    from qwen_b200 import model, ops

    shapes = [model.Linear(f"t{i}", M, K) for i, (M, K) in enumerate([(3584, 1024), (1024, 3584), (512, 1024),
                                                                       (6144, 1024), (33, 2048)])]
    st = model.DeviceStack(shapes, copies=1, seed=9)
    items = st.views(0)
    stack = ops.LinearStack(items)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        stack.run()       # warm up (attribute setup) outside capture
    torch.cuda.synchronize()
    for _, _, _, y in items:
        y.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        stack.run()
    for rep in range(2):
        for x, _, _, y in items:
            x.normal_()
            y.zero_()
        g.replay()
        torch.cuda.synchronize()
        for x, mant, exps, y in items:
            ref = O.bfp8_gemv(x.cpu().numpy(), mant.cpu().numpy(), exps.cpu().numpy())
            assert np.array_equal(bits(y.cpu().numpy()), bits(ref))
    stack.close()


def test_scaled_layer_shape(cuda):
    """One gate and one down projection of the multi-GPU configuration
    (28672 x 8192 and 8192 x 28672), bit-exact."""
    import torch

    from qwen_b200 import model, ops

    st = model.DeviceStack(model.scaled_stack(layers=1)[1:], copies=1, seed=3)
    for x, mant, exps, y in st.views(0):
        ops.bfp8_gemv(x, mant, exps, out=y)
        torch.cuda.synchronize()
        ref = O.bfp8_gemv(x.cpu().numpy(), mant.cpu().numpy(), exps.cpu().numpy())
        assert np.array_equal(bits(y.cpu().numpy()), bits(ref))


def test_device_packer_matches_reference_rule(cuda, golden):
    """On-device packer == reference packer on the committed fixtures (those
    matrices have no block peak within an ulp above a power of two)."""
    from qwen_b200 import ops

    g = golden("packer.npz")
    for name in ("normal", "edges", "wide"):
        w = g[f"{name}_w"]
        mant, exps = ops.pack_bfp8(*to_dev(w))
        assert np.array_equal(mant.cpu().numpy(), g[f"{name}_mant"]), name
        e = g[f"{name}_exps_padded"][: exps.numel()]
        assert np.array_equal(exps.cpu().numpy().reshape(-1), e), name


# ------------------------------------------------------------------ fast mode
def term_magnitude(x, mant, exps):
    """sum_b |float(dot_b) * 2^(e_b-134) * xs_b| per row (float64)."""
    xq, xs = O.quant_x(x)
    d = O.block_dots(mant, xq).astype(np.float64)
    return (np.abs(d) * np.ldexp(1.0, exps.astype(np.int64) - 134) * xs.astype(np.float64)).sum(axis=1)


@pytest.mark.parametrize("M,K", [(3584, 1024), (1024, 3584), (8192, 28672 // 4), (33, 2048), (1, 512)])
def test_gemv_fast_within_tolerance_and_deterministic(cuda, M, K):
    from qwen_b200 import ops

    rng = np.random.default_rng(M + 3 * K)
    mant, exps = rand_weights(rng, M, K)
    x = rng.normal(0, 1, K).astype(np.float32)
    dx, dm, de = to_dev(x, mant, exps)
    y1 = ops.bfp8_gemv_fast(dx, dm, de).cpu().numpy()
    y2 = ops.bfp8_gemv_fast(dx, dm, de).cpu().numpy()
    assert np.array_equal(bits(y1), bits(y2))
    ref = O.bfp8_gemv(x, mant, exps).astype(np.float64)
    tol = 1e-5 * term_magnitude(x, mant, exps) + 1e-30
    assert (np.abs(y1 - ref) <= tol).all()


def test_linear_stack_fast_within_tolerance(cuda):
    import torch

    from qwen_b200 import model, ops

    shapes = [model.Linear(f"t{i}", M, K) for i, (M, K) in enumerate([(8192, 7168), (2048, 1024), (512, 3584)])]
    st = model.DeviceStack(shapes, copies=1, seed=12)
    items = st.views(0)
    stack = ops.LinearStack(items, fast=True)
    for _ in range(2):   # the second run starts from the first run's tickets
        stack.run()
    torch.cuda.synchronize()
    for x, mant, exps, y in items:
        xn, mn, en = x.cpu().numpy(), mant.cpu().numpy(), exps.cpu().numpy()
        ref = O.bfp8_gemv(xn, mn, en).astype(np.float64)
        tol = 1e-5 * term_magnitude(xn, mn, en) + 1e-30
        assert (np.abs(y.cpu().numpy() - ref) <= tol).all()
    stack.close()


# ---------------------------------------------------- swiglu -> GEMV, fused
@pytest.mark.parametrize("M,K", [(1024, 3584), (33, 2048), (257, 6144), (1024, 512)])
def test_swiglu_gemv_bit_exact(cuda, M, K):
    """y = GEMV(swiglu(gate, up)) in one launch == the oracle chaining the
    NEON-build swiglu and the GEMV, bit for bit; the gates include zeros,
    subnormals and values past exp_neon's clamps."""
    from qwen_b200 import ops

    rng = np.random.default_rng(M + 7 * K)
    mant, exps = rand_weights(rng, M, K)
    gate = rng.normal(0, 3, K).astype(np.float32)
    up = rng.normal(0, 1, K).astype(np.float32)
    gate[:10] = np.array([0.0, -0.0, 1e-39, -1e-39, 87.5, -87.5, 88.5, -88.5, 100.0, -100.0], np.float32)
    up[20:23] = np.array([1e-39, 0.0, -3e-40], np.float32)
    y = ops.swiglu_bfp8_gemv(*to_dev(gate, up, mant, exps)).cpu().numpy()
    ref = O.bfp8_gemv(O.swiglu(gate, up, neon=True), mant, exps)
    assert np.array_equal(bits(y), bits(ref))


def test_mlp_block_chain_bit_exact(cuda):
    """Two chained MLP blocks of the 0.8B shapes (gate / up 3584x1024, down
    1024x3584) through ops.mlp_block == the oracle chaining the NEON-build
    add_residual, rmsnorm, GEMVs and swiglu, bit for bit (the residual
    stream h and each block's down output)."""
    import torch

    from qwen_b200 import ops

    rng = np.random.default_rng(77)
    h = rng.normal(0, 1, 1024).astype(np.float32)
    res = rng.normal(0, 1, 1024).astype(np.float32)
    dh, dres = to_dev(h, res)
    for blk in range(2):
        w = rng.normal(0, 0.1, 1024).astype(np.float32)
        mg, eg = rand_weights(rng, 3584, 1024)
        mu, eu = rand_weights(rng, 3584, 1024)
        md, ed = rand_weights(rng, 1024, 3584)
        dw, dmg, deg, dmu, deu, dmd, ded = to_dev(w, mg, eg, mu, eu, md, ed)
        dh, dres = ops.mlp_block(dh, dres, dw, (dmg, deg), (dmu, deu), (dmd, ded))
        torch.cuda.synchronize()
        h = O.add_residual(h, res, neon=True)
        nrm = O.rmsnorm(h, w, 1e-6, neon=True)
        inter = O.swiglu(O.bfp8_gemv(nrm, mg, eg), O.bfp8_gemv(nrm, mu, eu), neon=True)
        res = O.bfp8_gemv(inter, md, ed)
        assert np.array_equal(bits(dh.cpu().numpy()), bits(h)), blk
        assert np.array_equal(bits(dres.cpu().numpy()), bits(res)), blk


def test_swiglu_gemv_rejects_large_k(cuda):
    from qwen_b200 import ops
    from qwen_b200._lib import KernelError

    mant, exps = rand_weights(np.random.default_rng(1), 8, 8192)
    g = np.ones(8192, np.float32)
    with pytest.raises(KernelError):
        ops.swiglu_bfp8_gemv(*to_dev(g, g, mant, exps))


# ---------------------------------------------------- rmsnorm -> GEMV, fused
@pytest.mark.parametrize("M,K,sx,eps", [(3584, 1024, 1.0, 1e-6), (33, 2048, 25.0, 1e-5), (257, 6144, 0.5, 1e-6),
                                        (1, 512, 1e-20, 1e-6), (1024, 3584, 3.0, 1e-6)])
def test_rmsnorm_gemv_bit_exact(cuda, M, K, sx, eps):
    """One launch = the reference's rmsnorm (NEON build order) followed by its
    quantizer and GEMV: every output bit-identical to the oracle chaining
    rmsnorm and bfp8_gemv, including an odd row count (the scalar last row)
    and an input whose squares are subnormal (flushed; eps sets the scale)."""
    import torch

    from qwen_b200 import ops

    rng = np.random.default_rng(M + K)
    mant, exps = rand_weights(rng, M, K)
    x = rng.normal(0, sx, K).astype(np.float32)
    w = rng.normal(0, 0.1, K).astype(np.float32)
    ref = O.bfp8_gemv(O.rmsnorm(x, w, eps, neon=True), mant, exps)
    dx, dw, dm, de = to_dev(x, w, mant, exps)
    y = ops.rmsnorm_bfp8_gemv(dx, dw, eps, dm, de)
    y2 = ops.rmsnorm_bfp8_gemv(dx, dw, eps, dm, de)
    torch.cuda.synchronize()
    assert np.array_equal(bits(y.cpu().numpy()), bits(ref))
    assert np.array_equal(bits(y2.cpu().numpy()), bits(ref))


def test_rmsnorm_gemv_rejects_large_k(cuda):
    """The fused prologue keeps the whole activation in each CTA's shared
    memory: K above 6144 (or not a multiple of 512) is refused with QB_EINVAL."""
    import torch

    from qwen_b200 import ops
    from qwen_b200._lib import KernelError

    for K in (6656, 1088):
        mant = torch.zeros((8, K), dtype=torch.int8, device="cuda")
        exps = torch.zeros((8, K // 64), dtype=torch.uint8, device="cuda")
        x = torch.ones(K, device="cuda")
        with pytest.raises(KernelError):
            ops.rmsnorm_bfp8_gemv(x, x, 1e-6, mant, exps)


@pytest.mark.parametrize("M,K,sx", [(3584, 1024, 1.0), (33, 2048, 40.0), (257, 6144, 1e-20)])
def test_residual_rmsnorm_gemv_bit_exact(cuda, M, K, sx):
    """x_out = x + res (the reference's flushed add_residual) and y = GEMV of
    rmsnorm(x_out) from one launch, both bit-identical to the oracle chain,
    including subnormal residual sums (flushed)."""
    import torch

    from qwen_b200 import ops

    rng = np.random.default_rng(M * 3 + K)
    mant, exps = rand_weights(rng, M, K)
    x = rng.normal(0, sx, K).astype(np.float32)
    res = rng.normal(0, sx, K).astype(np.float32)
    w = rng.normal(0, 0.1, K).astype(np.float32)
    xo = O.add_residual(x, res, neon=True)
    ref = O.bfp8_gemv(O.rmsnorm(xo, w, 1e-6, neon=True), mant, exps)
    dx, dr, dw, dm, de = to_dev(x, res, w, mant, exps)
    for _ in range(2):
        y, x_out = ops.residual_rmsnorm_bfp8_gemv(dx, dr, dw, 1e-6, dm, de)
        torch.cuda.synchronize()
        assert np.array_equal(bits(x_out.cpu().numpy()), bits(xo))
        assert np.array_equal(bits(y.cpu().numpy()), bits(ref))


@pytest.mark.parametrize("M0,M1,K,residual", [(6144, 2048, 1024, False), (3584, 3584, 1024, True),
                                               (33, 1, 2048, True), (257, 64, 6144, False)])
def test_rmsnorm_gemv2_bit_exact(cuda, M0, M1, K, residual):
    """Two projections of one normalized vector in one launch (qkv and z,
    gate and up): each output, and x + res when given, bit-identical to the
    oracle chain, twice in a row."""
    import torch

    from qwen_b200 import ops

    rng = np.random.default_rng(M0 * 7 + M1 + K)
    m0, e0 = rand_weights(rng, M0, K)
    m1, e1 = rand_weights(rng, M1, K)
    x = rng.normal(0, 2.0, K).astype(np.float32)
    res = rng.normal(0, 2.0, K).astype(np.float32)
    w = rng.normal(0, 0.1, K).astype(np.float32)
    xo = O.add_residual(x, res, neon=True) if residual else x
    n = O.rmsnorm(xo, w, 1e-6, neon=True)
    ref0, ref1 = O.bfp8_gemv(n, m0, e0), O.bfp8_gemv(n, m1, e1)
    dx, dr, dw, dm0, de0, dm1, de1 = to_dev(x, res, w, m0, e0, m1, e1)
    for _ in range(2):
        out = ops.rmsnorm_bfp8_gemv2(dx, dw, 1e-6, (dm0, de0), (dm1, de1), res=dr if residual else None)
        torch.cuda.synchronize()
        assert np.array_equal(bits(out[0].cpu().numpy()), bits(ref0))
        assert np.array_equal(bits(out[1].cpu().numpy()), bits(ref1))
        if residual:
            assert np.array_equal(bits(out[2].cpu().numpy()), bits(xo))


def test_residual_rmsnorm_gemv_rejects_aliasing(cuda):
    """x_out may not overlap x or res (every CTA reads them while one writes it)."""
    import torch

    from qwen_b200._lib import load

    K, M = 1024, 64
    mant = torch.zeros((M, K), dtype=torch.int8, device="cuda")
    exps = torch.zeros((M, K // 64), dtype=torch.uint8, device="cuda")
    x = torch.ones(K, device="cuda")
    r = torch.ones(K, device="cuda")
    y = torch.empty(M, device="cuda")
    rc = load().qwen_b200_residual_rmsnorm_gemv_dev(y.data_ptr(), x.data_ptr(), x.data_ptr(), r.data_ptr(),
                                                    r.data_ptr(), 1e-6, mant.data_ptr(), exps.data_ptr(), M, K, None)
    assert rc == -1
