"""Pins the oracle's restatement of the Gated-DeltaNet layer glue and the
token loop (oracle/bfp8_oracle.c, qwen_kernels_opt.c:507-1049).

The reference's portable build (oracle/_ref/libref_kernels.so: its own C
file compiled here, x86 has no NEON) must equal the oracle with neon=0 bit
for bit -- every small op, forward_linear_layer with its state updates,
forward_mlp and forward_token_c over 24 layers with a callback.  (That build
skips conv1d + SiLU for every channel below C & ~3 -- its scalar loop starts
there -- and the oracle's neon=0 form restates that too.)  The NEON
restatement (neon=1, the board build the GPU follows) differs from the
portable forms only in lane order, flush-to-zero and exp_neon."""
import ctypes
import os

import numpy as np
import pytest

import layer_fixtures as LF

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(REPO, "oracle", "_ref", "libref_kernels.so")
needs_ref = pytest.mark.skipif(not os.path.exists(REF_SO), reason="oracle/_ref not built (make -C oracle ref)")

_P, _I, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def _ref():
    L = ctypes.CDLL(REF_SO)
    sig = {
        "causal_conv1d_update_silu": [_P, _P, _P, _P, _I],
        "qk_l2norm": [_P, _P, _I, _I],
        "gdn_gates": [_P, _P, _P, _P, _P, _P, _P, _I, _I],
        "gdn_recurrent_step": [_P, _P, _P, _P, _P, _P, _P, _I, _I],
        "rmsnorm_gated": [_P, _P, _P, _P, _I, _I, _F],
        "forward_linear_layer": [_P, _P],
        "forward_mlp": [_P, _P],
        "forward_token_c": [_I, _P, _P, _P, _P, _P, _P, LF.CALLBACK, _P],
    }
    for name, args in sig.items():
        getattr(L, name).argtypes = args
        getattr(L, name).restype = _I if name == "forward_token_c" else None
    return L


def _orc():
    from oracle import oracle as O
    return O.lib()


def _eq(a, b):
    return np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


@needs_ref
def test_small_ops_portable_build_bit_exact():
    R, O = _ref(), _orc()
    rng = np.random.default_rng(11)
    C, H, D, K = 3 * LF.V, LF.HEADS, LF.HEAD_DIM, LF.HIDDEN
    # conv1d + SiLU and its state shift
    x = rng.normal(0, 1, C).astype(np.float32)
    w = rng.normal(0, 0.3, (C, 4)).astype(np.float32)
    st = rng.normal(0, 0.5, (3, C)).astype(np.float32)
    y1, y2, s1, s2 = np.zeros(C, np.float32), np.zeros(C, np.float32), st.copy(), st.copy()
    R.causal_conv1d_update_silu(y1.ctypes.data, x.ctypes.data, s1.ctypes.data, w.ctypes.data, C)
    O.orc_conv1d_silu(y2.ctypes.data, x.ctypes.data, s2.ctypes.data, w.ctypes.data, C, 0)
    assert _eq(y1, y2) and _eq(s1, s2)
    # q/k l2 norm
    q = rng.normal(0, 1, H * D).astype(np.float32)
    k = rng.normal(0, 1, H * D).astype(np.float32)
    q1, k1, q2, k2 = q.copy(), k.copy(), q.copy(), k.copy()
    R.qk_l2norm(q1.ctypes.data, k1.ctypes.data, H, D)
    O.orc_qk_l2norm(q2.ctypes.data, k2.ctypes.data, H, D, 0)
    assert _eq(q1, q2) and _eq(k1, k2)
    # gates
    xs = rng.normal(0, 1, K).astype(np.float32)
    wa = rng.normal(0, 0.03, (H, K)).astype(np.float32)
    wb = rng.normal(0, 0.03, (H, K)).astype(np.float32)
    nea = (-np.exp(rng.uniform(0, 1.5, H))).astype(np.float32)
    dt = rng.uniform(-1, 1, H).astype(np.float32)
    g = [np.zeros(H, np.float32) for _ in range(4)]
    R.gdn_gates(g[0].ctypes.data, g[1].ctypes.data, xs.ctypes.data, wa.ctypes.data, wb.ctypes.data,
                nea.ctypes.data, dt.ctypes.data, H, K)
    O.orc_gdn_gates(g[2].ctypes.data, g[3].ctypes.data, xs.ctypes.data, wa.ctypes.data, wb.ctypes.data,
                    nea.ctypes.data, dt.ctypes.data, H, K, 0)
    assert _eq(g[0], g[2]) and _eq(g[1], g[3])
    # recurrent step (state in the blocked layout) and gated norm
    v = rng.normal(0, 1, H * D).astype(np.float32)
    S = rng.normal(0, 0.05, (H, D * D)).astype(np.float32)
    o1, o2, S1, S2 = np.zeros(H * D, np.float32), np.zeros(H * D, np.float32), S.copy(), S.copy()
    R.gdn_recurrent_step(o1.ctypes.data, S1.ctypes.data, q2.ctypes.data, k2.ctypes.data, v.ctypes.data,
                         g[0].ctypes.data, g[1].ctypes.data, H, D)
    O.orc_gdn_step(o2.ctypes.data, S2.ctypes.data, q2.ctypes.data, k2.ctypes.data, v.ctypes.data,
                   g[0].ctypes.data, g[1].ctypes.data, H, D, 0)
    assert _eq(o1, o2) and _eq(S1, S2)
    z = rng.normal(0, 1, H * D).astype(np.float32)
    nw = rng.normal(1, 0.1, D).astype(np.float32)
    r1, r2 = np.zeros(H * D, np.float32), np.zeros(H * D, np.float32)
    R.rmsnorm_gated(r1.ctypes.data, o1.ctypes.data, z.ctypes.data, nw.ctypes.data, H, D, 1e-6)
    O.orc_rmsnorm_gated(r2.ctypes.data, o1.ctypes.data, z.ctypes.data, nw.ctypes.data, H, D, 1e-6, 0)
    assert _eq(r1, r2)


@needs_ref
def test_linear_layer_and_mlp_portable_build_bit_exact():
    """Two consecutive forward_linear_layer calls (the states carry over)
    and a forward_mlp: h and both states bit-identical to the reference's
    own build."""
    R, O = _ref(), _orc()
    rng = np.random.default_rng(5)
    L = LF.Linear(rng)
    c1, s1 = L.copy_states()
    c2, s2 = L.copy_states()
    p1, p2 = L.plan(c1, s1), L.plan(c2, s2)
    h = rng.normal(0, 1, LF.HIDDEN).astype(np.float32)
    h1, h2 = h.copy(), h.copy()
    for _ in range(2):
        R.forward_linear_layer(ctypes.byref(p1), h1.ctypes.data)
        O.orc_forward_linear_layer(ctypes.byref(p2), h2.ctypes.data, 0)
        assert _eq(h1, h2) and _eq(c1, c2) and _eq(s1, s2)
    assert not _eq(h1, h) and not _eq(s1, L.state)   # the layer did change them
    mw = LF.Mlp(rng)   # keeps the arrays the plan points into alive
    m = mw.plan()
    R.forward_mlp(ctypes.byref(m), h1.ctypes.data)
    O.orc_forward_mlp(ctypes.byref(m), h2.ctypes.data, 0)
    assert _eq(h1, h2)


@needs_ref
def test_token_loop_portable_build_bit_exact():
    """forward_token_c over the 24 layers with a full-attention callback:
    token id, final h and all 18 layers' states bit-identical."""
    R, O = _ref(), _orc()
    M = LF.TokenModel(seed=2)
    cb = LF.attention_stand_in()
    st1, st2 = M.fresh_states(), M.fresh_states()
    (l1, m1), (l2, m2) = M.plans(st1), M.plans(st2)
    h1 = np.zeros(LF.HIDDEN, np.float32)
    h2 = np.zeros(LF.HIDDEN, np.float32)
    for tok in (17, 40001):
        a = R.forward_token_c(tok, h1.ctypes.data, ctypes.byref(l1), ctypes.byref(m1), M.is_full.ctypes.data,
                              M.final_ln.ctypes.data, M.embed.ctypes.data, cb, None)
        b = O.orc_forward_token(tok, h2.ctypes.data, ctypes.byref(l2), ctypes.byref(m2), M.is_full.ctypes.data,
                                M.final_ln.ctypes.data, M.embed.ctypes.data, ctypes.cast(cb, ctypes.c_void_p),
                                None, 0)
        assert a == b
        assert _eq(h1, h2)
        assert all(_eq(x[0], y[0]) and _eq(x[1], y[1]) for x, y in zip(st1, st2))


def test_neon_restatement_close_to_portable_forms():
    """The NEON-order small ops (what the GPU implements) against the
    portable forms where the two builds compute the same maths (lane order,
    flush-to-zero and exp_neon move a few ulps), and the NEON conv1d + SiLU
    against a numpy statement of its formula (the portable build skips it)."""
    O = _orc()
    rng = np.random.default_rng(8)
    C, H, D, K = 3 * LF.V, LF.HEADS, LF.HEAD_DIM, LF.HIDDEN
    x = rng.normal(0, 1, C).astype(np.float32)
    w = rng.normal(0, 0.3, (C, 4)).astype(np.float32)
    st = rng.normal(0, 0.5, (3, C)).astype(np.float32)
    y, s = np.zeros(C, np.float32), st.copy()
    O.orc_conv1d_silu(y.ctypes.data, x.ctypes.data, s.ctypes.data, w.ctypes.data, C, 1)
    d = (w[:, 0].astype(np.float64) * st[0] + w[:, 1] * st[1] + w[:, 2] * st[2] + w[:, 3] * x)
    assert np.abs(y - d / (1 + np.exp(-d))).max() <= 1e-5 * np.abs(d).max()
    assert np.array_equal(s, np.stack([st[1], st[2], x]))

    def both(fn, *arrays, args=()):
        outs = []
        for neon in (1, 0):
            cp = [a.copy() for a in arrays]
            fn(*[a.ctypes.data for a in cp], *args, neon)
            outs.append(cp)
        return outs

    q = rng.normal(0, 1, H * D).astype(np.float32)
    k = rng.normal(0, 1, H * D).astype(np.float32)
    (qa, ka), (qb, kb) = both(O.orc_qk_l2norm, q, k, args=(H, D))
    assert np.abs(qa - qb).max() <= 1e-6 * np.abs(qb).max() and np.abs(ka - kb).max() <= 1e-6 * np.abs(kb).max()
    xs = rng.normal(0, 1, K).astype(np.float32)
    wa = rng.normal(0, 0.03, (H, K)).astype(np.float32)
    wb = rng.normal(0, 0.03, (H, K)).astype(np.float32)
    nea = (-np.exp(rng.uniform(0, 1.5, H))).astype(np.float32)
    dt = rng.uniform(-1, 1, H).astype(np.float32)
    g = [np.zeros(H, np.float32) for _ in range(4)]
    for neon, (al, be) in ((1, g[:2]), (0, g[2:])):
        O.orc_gdn_gates(al.ctypes.data, be.ctypes.data, xs.ctypes.data, wa.ctypes.data, wb.ctypes.data,
                        nea.ctypes.data, dt.ctypes.data, H, K, neon)
    assert np.allclose(g[0], g[2], rtol=1e-5) and np.allclose(g[1], g[3], rtol=1e-5)
    v = rng.normal(0, 1, H * D).astype(np.float32)
    S = rng.normal(0, 0.05, (H, D * D)).astype(np.float32)
    o = [np.zeros(H * D, np.float32) for _ in range(2)]
    Ss = [S.copy(), S.copy()]
    for i, neon in enumerate((1, 0)):
        O.orc_gdn_step(o[i].ctypes.data, Ss[i].ctypes.data, qb.ctypes.data, kb.ctypes.data, v.ctypes.data,
                       g[2].ctypes.data, g[3].ctypes.data, H, D, neon)
    assert np.abs(o[0] - o[1]).max() <= 1e-6 * np.abs(o[1]).max()
    assert np.array_equal(Ss[0], Ss[1])   # same order, values far from the flush range
    z = rng.normal(0, 1, H * D).astype(np.float32)
    nw = rng.normal(1, 0.1, D).astype(np.float32)
    r = [np.zeros(H * D, np.float32) for _ in range(2)]
    for i, neon in enumerate((1, 0)):
        O.orc_rmsnorm_gated(r[i].ctypes.data, o[1].ctypes.data, z.ctypes.data, nw.ctypes.data, H, D, 1e-6, neon)
    assert np.abs(r[0] - r[1]).max() <= 1e-6 * np.abs(r[1]).max()
