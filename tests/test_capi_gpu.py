"""The reference drop-in entry points (host pointers, ctypes, as the engine
calls them) on a GPU: bfp8_gemv, lm_head_argmax, lm_head_topk."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def bits(a):
    a = np.ascontiguousarray(a, np.float32)
    return np.where(np.isnan(a), np.uint32(0x7FC00000), a.view(np.uint32))


@pytest.fixture(scope="module")
def lib(cuda):
    from qwen_b200 import _lib

    L = _lib.load()
    L.init_kernels()
    return L


def fake_weight_file(rng, shapes):
    """A weight 'file' in host memory with 64-byte aligned SoA tensors, like
    qwen35_weights_64k.bin, and the (offset, M, K) the engine slices out."""
    from qwen_b200 import model

    stack = [model.Linear(f"t{i}", M, K) for i, (M, K) in enumerate(shapes)]
    table, total = model.layout(stack)
    buf = np.zeros(total + 64, np.uint8)
    base = (-buf.ctypes.data) % 64
    buf = buf[base:base + total]
    ents = []
    for t in stack:
        off, _ = table[t.name]
        mant, exps = O.pack_bfp8(rng.normal(0, 0.02, (t.M, t.K)).astype(np.float32))
        blob = np.frombuffer(O.soa_bytes(mant, exps), np.uint8)
        buf[off:off + blob.size] = blob
        ents.append((off, t.M, t.K, mant, exps))
    return buf, ents


def test_bfp8_gemv_dropin_engine_style(lib):
    """Pointers into one mapped weight buffer, sliced the way
    qwen_real_engine._gemv_ent does (mant at the offset, exps right after)."""
    rng = np.random.default_rng(11)
    buf, ents = fake_weight_file(rng, [(3584, 1024), (1024, 3584), (6144, 1024), (33, 512)])
    assert lib.qwen_b200_register_weights(buf.ctypes.data, buf.nbytes) == 0
    try:
        for off, M, K, mant, exps in ents:
            x = rng.normal(0, 1, K).astype(np.float32)
            y = np.zeros(M, np.float32)
            lib.bfp8_gemv(y.ctypes.data, x.ctypes.data, buf.ctypes.data + off, buf.ctypes.data + off + M * K, M, K)
            assert np.array_equal(bits(y), bits(O.bfp8_gemv(x, mant, exps)))
    finally:
        lib.qwen_b200_forget_weights(buf.ctypes.data)


def test_bfp8_gemv_dropin_unregistered_pointers(lib):
    """Separate mantissa / exponent arrays never registered: uploaded on
    first use, and the same x pointer with new contents is requantized (the
    reference's pointer cache, qwen_kernels_opt.c:183, would not)."""
    rng = np.random.default_rng(12)
    M, K = 515, 2048
    mant, exps = O.pack_bfp8(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    x = rng.normal(0, 1, K).astype(np.float32)
    for _ in range(2):
        y = np.zeros(M, np.float32)
        lib.bfp8_gemv(y.ctypes.data, x.ctypes.data, mant.ctypes.data, exps.ctypes.data, M, K)
        assert np.array_equal(bits(y), bits(O.bfp8_gemv(x, mant, exps)))
        x[:] = rng.normal(0, 1, K)
    lib.qwen_b200_forget_weights(mant.ctypes.data)
    lib.qwen_b200_forget_weights(exps.ctypes.data)


def test_lm_head_dropins_selftest_data(lib, golden):
    g = O.XorShift32(0x13579BDF)
    cases = {"c1": g.selftest_fill(1000, 64), "c2": g.selftest_fill(500, 67)}
    for tag, (tab, h) in cases.items():
        V, H = tab.shape
        am = lib.lm_head_argmax(h.ctypes.data, tab.ctypes.data, V, H)
        assert am == O.lm_head_argmax(h, tab)
        for k in (1, 7, 20, V + 50):
            kk = min(k, V)
            ids = np.zeros(kk, np.int32)
            sc = np.zeros(kk, np.float32)
            n = lib.lm_head_topk(h.ctypes.data, tab.ctypes.data, V, H, k, ids.ctypes.data, sc.ctypes.data)
            rids, rsc = O.lm_head_topk(h, tab, k)
            assert n == len(rids)
            assert np.array_equal(ids[:n], rids)
            assert np.array_equal(bits(sc[:n]), bits(rsc))
        lib.qwen_b200_forget_weights(tab.ctypes.data)
    assert lib.lm_head_topk(None, None, 0, 0, 0, None, None) == 0


def test_profiler_counts_dropin_calls(lib):
    lib.qwen_prof_enable(1)
    lib.qwen_prof_reset()
    rng = np.random.default_rng(1)
    mant, exps = O.pack_bfp8(rng.normal(0, 0.02, (64, 512)).astype(np.float32))
    x = rng.normal(0, 1, 512).astype(np.float32)
    y = np.zeros(64, np.float32)
    lib.bfp8_gemv(y.ctypes.data, x.ctypes.data, mant.ctypes.data, exps.ctypes.data, 64, 512)
    assert lib.qwen_prof_get(0) > 0.0
    lib.qwen_prof_enable(0)
    lib.qwen_b200_forget_weights(mant.ctypes.data)
    lib.qwen_b200_forget_weights(exps.ctypes.data)


def test_lm_head_topk_dropin_serves_k_above_1024(lib):
    """The reference returns min(k, vocab) entries for every k
    (qwen_sampling.c:283-353); above 1024 the scores are sorted on the device.
    Duplicate rows give tied scores (ascending id first), a NaN row and a
    -inf row are never offered, and k past the vocabulary caps at its size."""
    g = O.XorShift32(0x2468ACE1)
    tab, h = g.selftest_fill(3000, 64)
    tab[100] = tab[7]                               # ties with id 7
    tab[2999] = tab[7]
    tab[50] = np.uint16(0x7FC0)                     # NaN row -> NaN score
    tab[51] = np.uint16(0)
    tab[51][0] = np.uint16(0xFF80)                  # -inf * h[0] ... -> +-inf or NaN
    V, H = tab.shape
    for k in (1025, 2048, V - 1, V, V + 50):
        kk = min(k, V)
        ids = np.full(kk, -7, np.int32)
        sc = np.zeros(kk, np.float32)
        n = lib.lm_head_topk(h.ctypes.data, tab.ctypes.data, V, H, k, ids.ctypes.data, sc.ctypes.data)
        rids, rsc = O.lm_head_topk(h, tab, k)
        assert n == len(rids), (k, n, len(rids))
        assert np.array_equal(ids[:n], rids), k
        assert np.array_equal(bits(sc[:n]), bits(rsc)), k
    lib.qwen_b200_forget_weights(tab.ctypes.data)


def test_weight_file_through_the_dropin_and_the_device_api(lib):
    """A weight-file image laid out by the reference manifest (layer 0's six
    BFP8 tensors filled): the engine's pointer pattern -- the whole mapping
    registered once, bfp8_gemv on the views' addresses -- and the device API
    on DeviceWeights both give the oracle's bits."""
    import torch

    from qwen_b200 import model, ops
    from test_manifest_cpu import ref_manifest, synthetic_file

    buf, names, sub = synthetic_file(ref_manifest())
    wf = model.WeightFile(sub, buffer=buf)
    wf.register()
    dw = wf.to_device("cuda:0")
    rng = np.random.default_rng(77)
    for n in names:
        mant, exps = wf.views(n)
        M, K = mant.shape
        x = rng.normal(0, 1, K).astype(np.float32)
        ref = bits(O.bfp8_gemv(x, mant, exps))
        y = np.zeros(M, np.float32)
        lib.bfp8_gemv(y.ctypes.data, x.ctypes.data, mant.ctypes.data, exps.ctypes.data, M, K)
        assert np.array_equal(bits(y), ref), n
        dm, de = dw.views(n)
        assert np.array_equal(bits(ops.bfp8_gemv(torch.from_numpy(x).cuda(), dm, de).cpu().numpy()), ref), n
    wf.forget()


class MlpPlanC(ctypes.Structure):
    """include/qwen_b200.h MlpPlanC (the engine's ctypes layout)."""
    _fields_ = [("post_ln_w", ctypes.c_void_p), ("mant_gate", ctypes.c_void_p), ("exp_gate", ctypes.c_void_p),
                ("M_gate", ctypes.c_int), ("K_gate", ctypes.c_int), ("mant_up", ctypes.c_void_p),
                ("exp_up", ctypes.c_void_p), ("M_up", ctypes.c_int), ("K_up", ctypes.c_int),
                ("mant_down", ctypes.c_void_p), ("exp_down", ctypes.c_void_p), ("M_down", ctypes.c_int),
                ("K_down", ctypes.c_int)]


def test_forward_mlp_dropin_matches_the_oracle_chain(lib):
    """forward_mlp (qwen_kernels_opt.c:994-1003) on a full-attention layer's
    MLP shapes, weights in one registered buffer as in the weight file:
    h + down(swiglu(gate(n), up(n))), n = rmsnorm(h), equals the oracle's
    NEON-build chain bit for bit, twice in a row (h updated in place)."""
    H, F = 1024, 3584
    rng = np.random.default_rng(994)
    parts, offs, off = [], {}, 0
    for name, (M, K) in (("gate", (F, H)), ("up", (F, H)), ("down", (H, F))):
        mant, exps = O.pack_bfp8(rng.normal(0, 0.02, (M, K)).astype(np.float32))
        offs[name] = (off, mant, exps)
        parts += [mant.view(np.uint8).ravel(), exps.ravel(), np.zeros((-(mant.size + exps.size)) % 64, np.uint8)]
        off += mant.size + exps.size + (-(mant.size + exps.size)) % 64
    buf = np.concatenate(parts)
    ln = (rng.normal(0, 0.1, H)).astype(np.float32)
    lib.qwen_b200_register_weights(buf.ctypes.data, buf.nbytes)
    p = MlpPlanC()
    p.post_ln_w = ln.ctypes.data
    for name in ("gate", "up", "down"):
        o, mant, exps = offs[name]
        setattr(p, f"mant_{name}", buf.ctypes.data + o)
        setattr(p, f"exp_{name}", buf.ctypes.data + o + mant.size)
        setattr(p, f"M_{name}", mant.shape[0])
        setattr(p, f"K_{name}", mant.shape[1])
    h = rng.normal(0, 1, H).astype(np.float32)
    ref = h.copy()
    for _ in range(2):
        lib.forward_mlp(ctypes.byref(p), h.ctypes.data)
        n = O.rmsnorm(ref, ln, 1e-6, neon=True)
        g = O.bfp8_gemv(n, offs["gate"][1], offs["gate"][2])
        u = O.bfp8_gemv(n, offs["up"][1], offs["up"][2])
        d = O.bfp8_gemv(O.swiglu(g, u, neon=True), offs["down"][1], offs["down"][2])
        ref = O.add_residual(ref, d, neon=True)
        assert np.array_equal(bits(h), bits(ref))
    bad = MlpPlanC()
    lib.forward_mlp(ctypes.byref(bad), h.ctypes.data)          # refused: null pointers
    assert b"forward_mlp" in lib.qwen_b200_last_error()
    assert np.array_equal(bits(h), bits(ref))                    # h untouched
    lib.qwen_b200_forget_weights(buf.ctypes.data)
    lib.qwen_b200_forget_weights(ln.ctypes.data)                 # uploaded on first use, cached by address
