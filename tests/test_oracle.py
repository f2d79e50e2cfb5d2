"""Pin the CPU oracle to the reference's own outputs and known answers.

Fixtures in tests/golden/ were produced by the reference's code (packer run
as Python, C kernels compiled from source, testbench recipe) -- see
tests/golden/make_golden.py.  These tests need no GPU.
"""
import ctypes
import os

import numpy as np
import pytest

from oracle import oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(REPO, "oracle", "_ref")


# ------------------------------------------------------------------ packer
@pytest.mark.parametrize("name", ["normal", "edges", "wide"])
def test_packer_matches_reference_packer(golden, name):
    g = golden("packer.npz")
    w = g[f"{name}_w"]
    mant, exps = O.pack_bfp8(w)
    assert np.array_equal(mant, g[f"{name}_mant"])
    assert O.soa_bytes(mant, exps)[mant.size:] == g[f"{name}_exps_padded"].tobytes()


def test_packer_selftest_snr():
    """05-主机侧源码/bfp8_packer.py:89-107: SNR > 30 dB with an outlier."""
    rng = np.random.default_rng(42)
    v = rng.normal(0, 1, 64).astype(np.float32)
    v[17] = 25.0
    m, e = O.pack_bfp8(v[None, :])
    rec = O.dequant(m, e)[0]
    snr = 10 * np.log10(np.sum(v ** 2) / np.sum((v - rec) ** 2))
    assert snr > 30.0


def test_packer_soa_sizes():
    m, e = O.pack_bfp8(np.random.default_rng(1).normal(0, 1, (128, 64)).astype(np.float32))
    b = O.soa_bytes(m, e)
    assert len(b) - m.size == 128 and (len(b) - m.size) % 8 == 0


# ------------------------------------------------------------------ quantizer
def test_quant_rule_by_hand():
    x = np.zeros(128, np.float32)
    x[:64] = np.linspace(-3, 5, 64, dtype=np.float32)
    x[64:] = 1e-21                      # amax <= 1e-20 -> zero block
    xq, xs = O.quant_x(x)
    amax = np.float32(5.0)
    q = np.float32(16384.0) / amax
    assert xs[0] == amax / np.float32(16384.0)
    assert np.array_equal(xq[:64], np.rint(x[:64] * q).astype(np.int16))
    assert xs[1] == 0 and not xq[64:].any()
    assert xq[63] == 16384


def test_exp_scale_table():
    s = O.exp_scale()
    for e in (0, 7, 8, 127, 134, 255):
        assert s[e] == np.ldexp(np.float32(1), e - 134)


# ------------------------------------------------------------------ known answers
def test_constant_pattern_block_sum():
    """01-系统概述/FINAL_REPORT.md:222-226: all-0x01 weights x all-0x1111 x ->
    every block sum 279616, on the 3584 x 1024 shape (57,344 blocks)."""
    mant = np.ones((3584, 1024), np.int8)
    xq = np.full(1024, 0x1111, np.int16)
    d = O.block_dots(mant, xq)
    assert d.size == 57344 and (d == 279616).all()
    lanes = O.lane_dots(mant[:2], xq)
    assert (lanes.sum(axis=2) == 279616).all() and (lanes == 69904).all()


def test_tb_gemv_core_block_dots(golden):
    """tb_gemv_core.v legacy cases (:401-402): raw int32 block dots bit-exact."""
    g = golden("tb_gemv.npz")
    for i, case in enumerate(g["cases"]):
        d = O.block_dots(g[f"{i}_w"], g[f"{i}_xq"])
        assert np.array_equal(d.astype(np.int64), g[f"{i}_dots"]), i


def test_tb_gemv_core_rtl20_tolerance(golden):
    """tb_gemv_core.v dequant cases (:404-419): the gemv_core word / 2^20 lies
    within 2e-6 + 3e-4|y| of the double model; huge exponents sit on a rail
    with the saturation flag set; tiny exponents flush to ~0."""
    g = golden("tb_gemv.npz")
    for i, (K, M, sd, dq, elo, ehi, xo, au, sat) in enumerate(g["cases"]):
        if not dq:
            continue
        words, flags = O.bfp8_gemv_rtl20(g[f"{i}_xq"], g[f"{i}_xs"], g[f"{i}_w"], g[f"{i}_e"])
        yref = g[f"{i}_yref"]
        if sat:
            assert all(w in (2**31 - 1, -2**31) for w in words), i
            assert flags & 2
        else:
            err = np.abs(words / 2.0**20 - yref)
            assert (err <= 2e-6 + 3e-4 * np.abs(yref)).all(), (i, err.max())
            assert flags == 0


def rtl_stage_model(xq, xs, mant, exps):
    """gemv_core.v dequant datapath (02-RTL与仿真/gemv_core.v:299-495) stage
    by stage with the RTL's register widths: S7 xs decode and the 10-bit
    shift sh_q, S8 clamp / overflow-test operand / 49-bit product, S9 the
    low three shift bits from the clamped amount, S10 the high three from
    the unclamped sh_q2, S11 the 65-bit saturating row sum, S12 the output
    clamp and bits [51:20].  Returns (words, flags) like the oracle."""
    M64 = (1 << 64) - 1
    AMAX, OMAX, OMIN = (1 << 63) - 1, (2**31 - 1) << 20, -(2**31) << 20

    def s64(v):
        v &= M64
        return v - (1 << 64) if v >> 63 else v

    def s10(v):
        v &= 1023
        return v - 1024 if v >> 9 else v

    M, K = mant.shape
    nb = K // 64
    xb = np.ascontiguousarray(xs, np.float32).view(np.uint32)
    dots = (mant.astype(np.int64).reshape(M, nb, 64) * xq.astype(np.int64).reshape(nb, 64)).sum(-1)
    words, flags = np.zeros(M, np.int32), 0
    for m in range(M):
        acc = 0
        for b in range(nb):
            bd, x = int(dots[m, b]), int(xb[b])
            eb = (x >> 23) & 0xFF
            norm = eb not in (0, 255)
            mant17 = ((1 << 16) | ((x >> 7) & 0xFFFF)) if norm else 0
            sh_q = s10((eb - 127 if norm else 0) + (int(exps[m, b]) - 134) + 24)
            sh_c = max(-63, min(63, sh_q))
            ovf_sh = 63 - (sh_c & 63) if sh_c >= 16 else 63
            prod = bd * mant17
            ovf = ((abs(bd) * mant17) >> ovf_sh) != 0 or sh_q > 63
            lo = (prod >> ((-sh_c) & 7)) if sh_c < 0 else s64(prod << (sh_c & 7))
            if sh_q < 0:
                shifted = lo >> (8 * ((((-sh_q) & 1023) >> 3) & 7))
            else:
                shifted = s64(lo << (8 * ((sh_q >> 3) & 7)))
            contrib = (-AMAX if prod < 0 else AMAX) if ovf else shifted
            flags |= int(ovf)
            total = acc + contrib
            if total > AMAX or total < -(1 << 63):
                acc = -AMAX if acc < 0 else AMAX
                flags |= 1
            else:
                acc = total
        if acc > OMAX or acc < OMIN:
            flags |= 2
        words[m] = max(OMIN, min(OMAX, acc)) >> 20
    return words, flags


@pytest.mark.parametrize("sh_lo,sh_hi", [(-120, -50), (-70, 10), (-20, 20), (0, 40), (30, 80)])
@pytest.mark.parametrize("K,specials", [(64, False), (384, True), (640, True)])
def test_rtl20_oracle_matches_stage_model(rtl_case, sh_lo, sh_hi, K, specials):
    """The C oracle's dequant mode == the stage-by-stage Verilog model, words
    and flags, over shifts from deep flushes (incl. the -103..-64 band the
    two-stage shifter does not flush) to saturation."""
    rng = np.random.default_rng(K * 1009 + sh_lo + 500)
    for _ in range(4):
        mant, exps, xq, xs = rtl_case(rng, 6, K, sh_lo, sh_hi, specials)
        words, flags = O.bfp8_gemv_rtl20(xq, xs, mant, exps)
        mw, mf = rtl_stage_model(xq, xs, mant, exps)
        assert np.array_equal(words, mw)
        assert flags == mf


def test_rtl20_short_right_shift_below_minus_63():
    """A shift of -64 moves right by 7 (low bits of the clamped -63, high
    bits of the unclamped -64), so one block of dot 2^20 with xs = 1.0
    adds floor(2^20 * 2^16 / 2^7) to the 40-fraction-bit accumulator:
    word = 2^29 >> 20 = 512.  A lossless clamp would give 0."""
    mant = np.zeros((1, 64), np.int8)
    xq = np.zeros(64, np.int16)
    mant[0, :64] = 64
    xq[:64] = 256                      # D = 64 * 64 * 256 = 2^20
    xs = np.array([1.0], np.float32)   # Ex 0, mantissa 2^16
    exps = np.array([[46]], np.uint8)  # sh = 0 + 46 - 110 = -64
    words, flags = O.bfp8_gemv_rtl20(xq, xs, mant, exps)
    assert words[0] == (((1 << 20) << 16) >> 7) >> 20 == 512
    assert flags == 0
    assert rtl_stage_model(xq, xs, mant, exps)[0][0] == 512


def test_neon_order_close_to_double_model(golden):
    """The NEON-order float result tracks the exact double sum of its terms."""
    g = golden("tb_gemv.npz")
    for i, (K, M, sd, dq, elo, ehi, xo, au, sat) in enumerate(g["cases"]):
        if not dq or sat:
            continue
        y = O.bfp8_gemv_q(g[f"{i}_xq"], g[f"{i}_xs"], g[f"{i}_w"], g[f"{i}_e"])
        yref = g[f"{i}_yref"]
        d = g[f"{i}_dots"].astype(np.float64)
        scale = (np.abs(d) * np.ldexp(1.0, g[f"{i}_e"].astype(np.int64) - 134) *
                 g[f"{i}_xs"].astype(np.float64)).sum(axis=1)
        assert (np.abs(y - yref) <= 1e-6 * scale + 1e-30).all(), i


# ------------------------------------------------------------------ compiled reference
def _ref():
    k = os.path.join(REF_DIR, "libref_kernels.so")
    s = os.path.join(REF_DIR, "libref_sampling.so")
    if not (os.path.exists(k) and os.path.exists(s)):
        pytest.skip("reference C not compiled (make -C oracle ref)")
    return ctypes.CDLL(k), ctypes.CDLL(s)


def test_scalar_gemv_matches_fixture(golden):
    """Oracle's scalar form == reference bfp8_gemv compiled for x86 (its
    scalar fallback, qwen_kernels_opt.c:311-325), bit for bit."""
    g = golden("ref_gemv.npz")
    for t in "abc":
        y = O.bfp8_gemv_scalar(g[f"{t}_x"], g[f"{t}_mant"], g[f"{t}_exps"])
        assert np.array_equal(y.view(np.uint32), g[f"{t}_y"].view(np.uint32)), t


def test_neon_gemv_close_to_scalar_reference(golden):
    """The int16 path differs from the float fallback only by activation
    quantization (relative ~1e-4 of the row's magnitude)."""
    g = golden("ref_gemv.npz")
    for t in "abc":
        y = O.bfp8_gemv(g[f"{t}_x"], g[f"{t}_mant"], g[f"{t}_exps"])
        ref = g[f"{t}_y"]
        w = O.dequant(g[f"{t}_mant"], g[f"{t}_exps"])
        mag = np.abs(w) @ np.abs(g[f"{t}_x"])
        assert (np.abs(y - ref) <= 2e-4 * mag).all(), t


def _selftest_tables():
    g = O.XorShift32(0x13579BDF)
    return {"c1": g.selftest_fill(1000, 64), "c2": g.selftest_fill(500, 67), "c3": g.selftest_fill(65536, 1024)}


@pytest.fixture(scope="module")
def selftest_tables():
    return _selftest_tables()


def test_lm_selection_matches_reference_scalar_build(golden, selftest_tables):
    """With the scalar score order the oracle's argmax / top-k reproduce the
    compiled reference exactly (ids and scores), for every k of the
    reference self-test including k > vocab."""
    g = golden("ref_lm.npz")
    for tag, (tab, h) in selftest_tables.items():
        s = O.lm_scores_scalar(h, tab)
        assert O.argmax(s) == int(g[f"{tag}_argmax"])
        for key in g.files:
            if key.startswith(tag + "_k") and key.endswith("_ids"):
                k = int(key[len(tag) + 2:-4])
                ids, sc = O.topk(s, k)
                assert np.array_equal(ids, g[key]), key
                assert np.array_equal(sc.view(np.uint32), g[key.replace("_ids", "_scores")].view(np.uint32))


def test_lm_neon_order_agrees_with_reference_ranking(golden, selftest_tables):
    """NEON-order scores (what the board and the GPU compute) against the
    reference self-test criterion: same ranking up to swaps of scores closer
    than the 1e-3 tolerance of check_topk_against_brute (qwen_sampling.c:585-631)."""
    g = golden("ref_lm.npz")
    for tag, (tab, h) in selftest_tables.items():
        s = O.lm_scores(h, tab, with_tail=True)
        ids, sc = O.topk(s, 64)
        ref_ids = g[f"{tag}_k{1 if tag != 'c2' else 7}_ids"]
        assert ids[0] == ref_ids[0] or abs(sc[0] - s[ref_ids[0]]) < 1e-3
        sref = O.lm_scores_scalar(h, tab)
        assert np.abs(s - sref).max() < 1e-3


def test_oracle_topk_rules():
    s = np.array([1.0, 3.0, 3.0, np.nan, -np.inf, 2.0, -3.4028235e38, 3.0], np.float32)
    ids, sc = O.topk(s, 10)
    assert ids.tolist() == [1, 2, 7, 5, 0]
    assert O.argmax(s) == 1
    assert O.argmax(np.full(5, -1e31, np.float32)) == 0
    assert O.topk(s, 0)[0].size == 0


def test_scalar_rmsnorm_matches_fixture(golden):
    """Oracle's portable-build rmsnorm == the reference's rmsnorm compiled for
    x86 (qwen_kernels_opt.c:140-172), bit for bit, including a vector whose
    squares are subnormal (the eps term then decides the scale)."""
    g = golden("ref_rmsnorm.npz")
    for t in "abcd":
        y = O.rmsnorm(g[f"{t}_x"], g[f"{t}_w"], float(g[f"{t}_eps"]), neon=False)
        assert np.array_equal(y.view(np.uint32), g[f"{t}_y"].view(np.uint32)), t


def test_neon_rmsnorm_close_to_scalar_reference(golden):
    """The NEON-order restatement (four flushed lane sums, x * (r * (1 + w)))
    differs from the portable build only by rounding order.  A float sum of n
    positive squares carries at most n * 2^-24 relative error, which the
    square root halves; plus a few roundings in the scale: every output within
    (n / 2 + 4) * 2^-24 of the reference, relatively."""
    g = golden("ref_rmsnorm.npz")
    for t in "abcd":
        x = g[f"{t}_x"]
        y = O.rmsnorm(x, g[f"{t}_w"], float(g[f"{t}_eps"]), neon=True)
        ref = g[f"{t}_y"]
        tol = (x.size / 2 + 4) * 2.0 ** -24
        assert np.all(np.abs(y - ref) <= tol * np.abs(ref)), t


def test_swiglu_matches_fixture(golden):
    """Oracle's portable-build swiglu == the compiled reference
    (qwen_kernels_opt.c:365-386 built for x86), bit for bit, incl. zeros,
    subnormals, values past exp_neon's clamps and a tail of 3 elements."""
    g = golden("ref_swiglu.npz")
    y = O.swiglu(g["gate"], g["up"], neon=False)
    same = (y.view(np.uint32) == g["y"].view(np.uint32)) | (np.isnan(y) & np.isnan(g["y"]))
    assert same.all()


def test_swiglu_neon_restatement_bound(golden):
    """The NEON build's swiglu stays within 2^-24 * (16 + 2|g|) relative of
    the portable build while exp_neon's argument is inside its [-87, 88]
    clamp and the result is normal.  exp_neon rounds fx = x * log2(e) to
    float before splitting off n (an absolute error up to |fx| * 2^-24, i.e.
    ~|x| * 2^-24 relative in 2^fx), then evaluates the degree-6 Taylor
    polynomial of 2^f (|f| <= 1/2, truncation (ln2/2)^7/7! < 2^-23) with
    seven roundings; the add, the division and the product add three more.
    The tail (n % 4) is computed alike by both builds."""
    g = golden("ref_swiglu.npz")
    yn = O.swiglu(g["gate"], g["up"], neon=True).astype(np.float64)
    ref = g["y"].astype(np.float64)
    ag = np.abs(g["gate"].astype(np.float64))
    inside = (ag <= 87.0) & (np.abs(ref) >= 2.0**-126)
    assert inside.sum() > 3500
    bound = 2.0**-24 * (16 + 2 * ag[inside]) * np.abs(ref[inside])
    assert (np.abs(yn - ref)[inside] <= bound).all()
    n = g["gate"].size
    assert np.array_equal(yn[n - n % 4:], ref[n - n % 4:])
    # exp_neon clamps -g at 88: g = -100 gives a tiny nonzero value where
    # expf overflows to inf and the portable build returns -0
    i = int(np.where(g["gate"] == -100.0)[0][0])
    assert ref[i] == 0.0 and yn[i] != 0.0


def neon_swiglu_model(gate, up):
    """The NEON build's swiglu (qwen_kernels_opt.c:332-386) as numpy float32
    arithmetic, independent of the C oracle: every vector-unit step is one
    IEEE float32 operation with subnormal operands and results flushed to a
    signed zero; the division is IEEE (VFP)."""
    f32 = np.float32
    tiny = f32(2.0**-126)

    def ftz(a):
        a = np.asarray(a, f32)
        return np.where(np.abs(a) < tiny, np.copysign(f32(0), a), a).astype(f32)

    def mul(a, b):
        return ftz(ftz(a) * ftz(b))

    def add(a, b):
        return ftz(ftz(a) + ftz(b))

    def sub(a, b):
        return ftz(ftz(a) - ftz(b))

    g = np.asarray(gate, f32)
    x = ftz(-g)
    with np.errstate(invalid="ignore"):
        x = np.where(np.isnan(x), x, np.maximum(x, f32(-87)))
        x = np.where(np.isnan(x), x, np.minimum(x, f32(88)))
    fx = mul(x, f32(1 / np.log(2)))
    n = sub(add(fx, f32(1.5 * 2**23)), f32(1.5 * 2**23))
    f = sub(fx, n)
    coef = [f32(np.log(2) ** k / np.prod(range(1, k + 1))) for k in range(7)]
    p = coef[6]
    for k in range(5, -1, -1):
        p = add(coef[k], mul(p, f))
    e = np.where(np.isnan(n), 0, np.trunc(np.nan_to_num(n))).astype(np.int64) + 127
    sc = (e.astype(np.uint32) << np.uint32(23)).view(f32)
    d = add(f32(1), mul(p, sc))
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        return mul((g / d).astype(f32), np.asarray(up, f32))


def test_swiglu_neon_oracle_matches_numpy_model(golden):
    """The C oracle's NEON-build swiglu == the independent numpy model, bit
    for bit, over the fixture and 10^6 gates spanning the clamps, zeros and
    subnormals (NaN payloads aside)."""
    g = golden("ref_swiglu.npz")
    rng = np.random.default_rng(8)
    gates = [g["gate"][: g["gate"].size & ~3], rng.uniform(-100, 100, 1 << 20).astype(np.float32),
             (rng.normal(0, 1, 4096) * 1e-38).astype(np.float32)]
    for gate in gates:
        up = rng.normal(0, 1, gate.size).astype(np.float32)
        a = O.swiglu(gate, up, neon=True)
        b = neon_swiglu_model(gate, up)
        same = (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))
        assert same.all(), np.where(~same)[0][:5]


def neon_gemv_model(xq, xs, mant, exps):
    """bfp8_gemv's NEON int16 path (qwen_kernels_opt.c:213-308) as numpy
    arithmetic, independent of the C oracle: lane-class sums L_j over
    i = j mod 4 in integers; per block f_j = f_j + ((float(L_j) * S) * xs)
    with every float32 step flushed like the vector unit (S = 2^(e-134) is a
    subnormal, hence flushed, for e < 8); y = (f0 + f2) + (f1 + f3).  An odd
    last row runs on VFP: sum = sum + (float(sum_j L_j) * S) * xs in IEEE."""
    f32 = np.float32
    tiny = f32(2.0**-126)

    def ftz(a):
        a = np.asarray(a, f32)
        return np.where(np.abs(a) < tiny, np.copysign(f32(0), a), a).astype(f32)

    def mul(a, b):
        return ftz(ftz(a) * ftz(b))

    def add(a, b):
        return ftz(ftz(a) + ftz(b))

    M, K = mant.shape
    nb = K // 64
    L = (mant.astype(np.int64).reshape(M, nb, 16, 4) * xq.astype(np.int64).reshape(nb, 16, 4)).sum(axis=2)
    S = np.ldexp(f32(1), exps.astype(np.int32) - 134).astype(f32)
    xs = np.asarray(xs, f32)
    Mv = M & ~1
    f = np.zeros((Mv, 4), f32)
    with np.errstate(over="ignore", invalid="ignore"):   # huge exponents overflow to inf / NaN
        for b in range(nb):
            f = add(f, mul(mul(L[:Mv, b, :].astype(f32), S[:Mv, b:b + 1]), xs[b]))
        y = np.zeros(M, f32)
        y[:Mv] = add(add(f[:, 0], f[:, 2]), add(f[:, 1], f[:, 3]))
        if M & 1:
            acc = f32(0)
            for b in range(nb):
                acc = f32(acc + f32(f32(f32(L[M - 1, b].sum()) * S[M - 1, b]) * xs[b]))
            y[M - 1] = acc
    return y


@pytest.mark.parametrize("M,K,elo,ehi", [(64, 1024, 100, 140), (33, 512, 0, 20), (17, 2048, 0, 255),
                                         (5, 192, 120, 134)])
def test_neon_gemv_oracle_matches_numpy_model(M, K, elo, ehi):
    """The C oracle's NEON-order GEMV == the independent numpy model, bit for
    bit, incl. odd row counts and exponents that make S or the terms
    subnormal (flushed on the vector unit, kept on VFP)."""
    rng = np.random.default_rng(M * K + elo)
    mant = rng.integers(-128, 128, (M, K)).astype(np.int8)
    exps = rng.integers(elo, ehi + 1, (M, K // 64)).astype(np.uint8)
    xq, xs = O.quant_x(rng.normal(0, 1, K).astype(np.float32) * np.float32(rng.choice([1e-3, 1.0, 1e3])))
    a = O.bfp8_gemv_q(xq, xs, mant, exps)
    b = neon_gemv_model(xq, xs, mant, exps)
    assert ((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))).all()


def _ftz32(a):
    a = np.asarray(a, np.float32)
    return np.where(np.abs(a) < np.float32(2.0**-126), np.copysign(np.float32(0), a), a).astype(np.float32)


def _nmul(a, b):
    return _ftz32(_ftz32(a) * _ftz32(b))


def _nadd(a, b):
    return _ftz32(_ftz32(a) + _ftz32(b))


def test_neon_rmsnorm_and_lm_scores_match_numpy_models():
    """Two more NEON-order restatements against independent numpy models,
    bit for bit: rmsnorm (qwen_kernels_opt.c:140-172: four flushed lane sums
    of x*x over i = 4j + l, (s0 + s2) + (s1 + s3), r = 1/sqrt(sum/n + eps) in
    IEEE, y = x * (r * (1 + w)) flushed) and the bf16 lm_head scores
    (:427-456: eight flushed chains c = i mod 8, then
    ((c0 + c4) + (c2 + c6)) + ((c1 + c5) + (c3 + c7)))."""
    f32 = np.float32
    rng = np.random.default_rng(31)
    for n, sx in ((1024, 1.0), (3584, 30.0), (512, 1e-20)):
        x = (rng.normal(0, 1, n) * sx).astype(f32)
        w = rng.normal(0, 0.1, n).astype(f32)
        s4 = np.zeros(4, f32)
        for i in range(0, n, 4):
            s4 = _nadd(s4, _nmul(x[i:i + 4], x[i:i + 4]))
        total = _nadd(_nadd(s4[0], s4[2]), _nadd(s4[1], s4[3]))
        r = f32(f32(1) / np.sqrt(f32(f32(total / f32(n)) + f32(1e-6)), dtype=f32))
        model = _nmul(x, _nmul(r, _nadd(f32(1), w)))
        got = O.rmsnorm(x, w, 1e-6, neon=True)
        assert np.array_equal(got.view(np.uint32), model.view(np.uint32)), n
    V, H = 257, 1024
    E = (rng.normal(0, 0.05, (V, H)).astype(f32).view(np.uint32) >> 16).astype(np.uint16)
    h = rng.normal(0, 1, H).astype(f32)
    Ef = (E.astype(np.uint32) << 16).view(f32)
    c = np.zeros((V, 8), f32)
    for i in range(0, H, 8):
        c = _nadd(c, _nmul(Ef[:, i:i + 8], h[i:i + 8]))
    model = _nadd(_nadd(_nadd(c[:, 0], c[:, 4]), _nadd(c[:, 2], c[:, 6])),
                  _nadd(_nadd(c[:, 1], c[:, 5]), _nadd(c[:, 3], c[:, 7])))
    got = O.lm_scores(h, E, with_tail=False)
    assert np.array_equal(got.view(np.uint32), model.view(np.uint32))


def test_add_residual_matches_fixture(golden):
    """Oracle's portable-build add_residual == the compiled reference, bit for
    bit; the NEON form flushes subnormal operands and sums (the vector unit),
    and equals it elsewhere."""
    g = golden("ref_residual.npz")
    y = O.add_residual(g["x"], g["r"], neon=False)
    assert np.array_equal(y.view(np.uint32), g["y"].view(np.uint32))
    yn = O.add_residual(g["x"], g["r"], neon=True)
    sub = (np.abs(g["x"]) < 1.18e-38) | (np.abs(g["r"]) < 1.18e-38) | (np.abs(g["y"]) < 1.18e-38)
    assert np.array_equal(yn[~sub].view(np.uint32), g["y"][~sub].view(np.uint32))
    assert yn[5] == 0.0


def test_numpy_fallback_gemv_matches_reference_engine(golden):
    """oracle.bfp8_gemv_numpy equals the reference engine's own numpy
    fallback (qwen_real_engine.py:1233-1239, run as the reference's method in
    make_golden.py) bit for bit, incl. a subnormal and a large block scale."""
    g = golden("ref_numpy_gemv.npz")
    for tag in ("a", "b", "c"):
        y = O.bfp8_gemv_numpy(g[f"{tag}_x"], g[f"{tag}_mant"], g[f"{tag}_exps"])
        assert np.array_equal(y.view(np.uint32), g[f"{tag}_y"].view(np.uint32)), tag
