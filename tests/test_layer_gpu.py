"""The device token loop -- forward_linear_layer and forward_token_c through
the C ABI -- against the oracle's NEON-build restatement
(oracle/bfp8_oracle.c; qwen_kernels_opt.c:507-1049).

The GEMVs, rmsnorms, swiglu, residual adds, conv1d + SiLU (exp_neon) and
the recurrent step follow the NEON order bit for bit; the gates and the
gated norm's SiLU call expf / log1pf, which CUDA and the C library round
differently in the last place.  So: with gates that need no libm (nea = 0
gives alpha = expf(0) = 1, wb = 0 gives beta = 1 / (1 + expf(0)) = 0.5) the
conv and recurrent states are compared bit for bit; in general the states
and h are compared to 1e-4 of their scale after one layer call (a
last-place change of an activation can flip one int16 rounding in the next
GEMV's quantizer, and such differences compound from call to call: 3e-4
after three calls, 1e-3 after forward_token_c's 24 layers, whose token ids
must be equal)."""
import ctypes

import numpy as np
import pytest

import layer_fixtures as LF

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def libs():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from oracle import oracle as O
    from qwen_b200 import _lib

    lib = _lib.load()
    assert lib.qwen_b200_gdn_state_mode(0) == 0
    return lib, O.lib()


@pytest.fixture(autouse=True)
def fresh_registry(libs):
    """Uploads are cached by host address and numpy reuses freed addresses:
    every test starts with an empty registry."""
    libs[0].qwen_b200_reset_weights()
    yield


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _run_layer(lib, orc, L, h, calls, first_call_check=None):
    c1, s1 = L.copy_states()
    c2, s2 = L.copy_states()
    p1, p2 = L.plan(c1, s1), L.plan(c2, s2)
    h1, h2 = h.copy(), h.copy()
    for i in range(calls):
        lib.forward_linear_layer(ctypes.byref(p1), h1.ctypes.data)
        orc.orc_forward_linear_layer(ctypes.byref(p2), h2.ctypes.data, 1)
        if i == 0 and first_call_check:
            first_call_check((h1, c1, s1), (h2, c2, s2))
    return (h1, c1, s1), (h2, c2, s2)


def test_linear_layer_states_bit_exact_with_libm_free_gates(libs):
    lib, orc = libs
    rng = np.random.default_rng(21)
    L = LF.Linear(rng)
    L.nea[:] = 0.0
    L.wb[:] = 0.0
    h = rng.normal(0, 1, LF.HIDDEN).astype(np.float32)
    (h1, c1, s1), (h2, c2, s2) = _run_layer(lib, orc, L, h, calls=1)
    assert not np.array_equal(h1, h)
    assert np.array_equal(c1, c2), "conv state"
    assert np.array_equal(s1.view(np.uint32), s2.view(np.uint32)), "recurrent state"
    print(f"h rel diff {_rel(h1, h2):.2e}")
    assert _rel(h1, h2) <= 1e-4


def test_linear_layer_matches_neon_oracle_over_calls(libs):
    """Three calls in a row: after the first, the conv state (inputs shifted
    in) is bit-exact and h and the state agree to 1e-4 of their scale; each
    later call starts from h values that differ in the last places, so the
    bound grows with the calls (3e-4 after three)."""
    lib, orc = libs
    rng = np.random.default_rng(22)
    L = LF.Linear(rng)
    h = rng.normal(0, 1, LF.HIDDEN).astype(np.float32)

    def first(a, b):
        assert np.array_equal(a[1], b[1]), "conv state after one call"
        print(f"first call: h {_rel(a[0], b[0]):.2e} state {_rel(a[2], b[2]):.2e}")
        assert _rel(a[0], b[0]) <= 1e-4 and _rel(a[2], b[2]) <= 1e-4

    (h1, c1, s1), (h2, c2, s2) = _run_layer(lib, orc, L, h, calls=3, first_call_check=first)
    print(f"third call: h {_rel(h1, h2):.2e} state {_rel(s1, s2):.2e} conv {_rel(c1, c2):.2e}")
    assert _rel(c1, c2) <= 3e-4
    assert _rel(s1, s2) <= 3e-4
    assert _rel(h1, h2) <= 3e-4
    assert not np.array_equal(s1, L.state)


def test_linear_layer_other_shape(libs):
    """A layer shape other than the 0.8B model's (the reference hard-codes
    1024 / 16 heads; this library takes the shape from the plan): hidden 2048,
    8 heads, ffn 2048 -- states bit-exact with libm-free gates, h to 1e-4."""
    lib, orc = libs
    rng = np.random.default_rng(24)
    L = LF.Linear(rng, hidden=2048, heads=8, ffn=2048)
    L.nea[:] = 0.0
    L.wb[:] = 0.0
    h = rng.normal(0, 1, 2048).astype(np.float32)
    (h1, c1, s1), (h2, c2, s2) = _run_layer(lib, orc, L, h, calls=1)
    assert not np.array_equal(h1, h), lib.qwen_b200_last_error()
    assert np.array_equal(c1, c2) and np.array_equal(s1.view(np.uint32), s2.view(np.uint32))
    assert _rel(h1, h2) <= 1e-4


def test_token_loop_matches_neon_oracle(libs):
    lib, orc = libs
    M = LF.TokenModel(seed=3)
    cb = LF.attention_stand_in()
    st1, st2 = M.fresh_states(), M.fresh_states()
    (l1, m1), (l2, m2) = M.plans(st1), M.plans(st2)
    h1 = np.zeros(LF.HIDDEN, np.float32)
    h2 = np.zeros(LF.HIDDEN, np.float32)
    for tok in (5, 65541, 30000):
        a = lib.forward_token_c(tok, h1.ctypes.data, ctypes.byref(l1), ctypes.byref(m1), M.is_full.ctypes.data,
                                M.final_ln.ctypes.data, M.embed.ctypes.data, cb, None)
        b = orc.orc_forward_token(tok, h2.ctypes.data, ctypes.byref(l2), ctypes.byref(m2), M.is_full.ctypes.data,
                                  M.final_ln.ctypes.data, M.embed.ctypes.data, ctypes.cast(cb, ctypes.c_void_p),
                                  None, 1)
        print(f"token {tok}: {a} vs {b}, h {_rel(h1, h2):.2e}")
        assert a == b
        assert _rel(h1, h2) <= 1e-3
    print(f"states {max(_rel(x[1], y[1]) for x, y in zip(st1, st2)):.2e} "
          f"conv {max(_rel(x[0], y[0]) for x, y in zip(st1, st2)):.2e}")
    assert max(_rel(x[1], y[1]) for x, y in zip(st1, st2)) <= 1e-3
    assert max(_rel(x[0], y[0]) for x, y in zip(st1, st2)) <= 1e-3


def test_token_loop_without_callback(libs):
    """A null callback skips attention, as the reference's loop does
    (qwen_kernels_opt.c:1031): still the oracle's token ids."""
    lib, orc = libs
    M = LF.TokenModel(seed=6)
    st1, st2 = M.fresh_states(), M.fresh_states()
    (l1, m1), (l2, m2) = M.plans(st1), M.plans(st2)
    h1 = np.zeros(LF.HIDDEN, np.float32)
    h2 = np.zeros(LF.HIDDEN, np.float32)
    for tok in (123, 4567):
        a = lib.forward_token_c(tok, h1.ctypes.data, ctypes.byref(l1), ctypes.byref(m1), M.is_full.ctypes.data,
                                M.final_ln.ctypes.data, M.embed.ctypes.data, LF.CALLBACK(), None)
        b = orc.orc_forward_token(tok, h2.ctypes.data, ctypes.byref(l2), ctypes.byref(m2), M.is_full.ctypes.data,
                                  M.final_ln.ctypes.data, M.embed.ctypes.data, None, None, 1)
        assert a == b and a >= 0
        assert _rel(h1, h2) <= 1e-3


def test_layer_calls_inside_the_callback_are_refused(libs):
    """The callback runs with the library unlocked; a forward_mlp call from
    inside it is refused (it would overwrite the loop's device buffers) and
    the token is still the oracle's."""
    lib, orc = libs
    M = LF.TokenModel(seed=7)
    st1, st2 = M.fresh_states(), M.fresh_states()
    (l1, m1), (l2, m2) = M.plans(st1), M.plans(st2)
    stand_in = LF.attention_stand_in()
    mp = M.mlp_w.plan()
    seen = []

    def cb(layer, h_ptr, ctx):
        lib.forward_mlp(ctypes.byref(mp), h_ptr)
        seen.append(lib.qwen_b200_last_error())
        stand_in(layer, h_ptr, ctx)

    ccb = LF.CALLBACK(cb)
    h1 = np.zeros(LF.HIDDEN, np.float32)
    h2 = np.zeros(LF.HIDDEN, np.float32)
    a = lib.forward_token_c(77, h1.ctypes.data, ctypes.byref(l1), ctypes.byref(m1), M.is_full.ctypes.data,
                            M.final_ln.ctypes.data, M.embed.ctypes.data, ccb, None)
    b = orc.orc_forward_token(77, h2.ctypes.data, ctypes.byref(l2), ctypes.byref(m2), M.is_full.ctypes.data,
                              M.final_ln.ctypes.data, M.embed.ctypes.data, ctypes.cast(stand_in, ctypes.c_void_p),
                              None, 1)
    assert len(seen) == 6 and all(b"inside forward_token_c" in e for e in seen)
    assert a == b and _rel(h1, h2) <= 1e-3


def test_state_modes_agree(libs):
    """Resident states (copied in once, synced back on request) and the
    page-locked mirror give the same tokens, h and states as the default
    mirror, bit for bit."""
    lib, _ = libs
    M = LF.TokenModel(seed=4)
    cb = LF.attention_stand_in()
    out = []
    for mode in (0, 1, 2):
        assert lib.qwen_b200_gdn_state_mode(mode) == 0
        st = M.fresh_states()
        lps, mps = M.plans(st)
        h = np.zeros(LF.HIDDEN, np.float32)
        ids = [lib.forward_token_c(t, h.ctypes.data, ctypes.byref(lps), ctypes.byref(mps), M.is_full.ctypes.data,
                                   M.final_ln.ctypes.data, M.embed.ctypes.data, cb, None) for t in (9, 99, 999)]
        assert min(ids) >= 0, lib.qwen_b200_last_error()
        if mode == 1:
            untouched = all(np.array_equal(s[1], s0[1]) for s, s0 in zip(st, M.states0))
            assert untouched, "resident mode wrote the host states before a sync"
            assert lib.qwen_b200_gdn_state_sync() == 0
        lib.qwen_b200_gdn_state_drop()
        out.append((ids, h, st))
    assert lib.qwen_b200_gdn_state_mode(0) == 0
    assert lib.qwen_b200_gdn_state_mode(3) != 0
    i0, h0, s0 = out[0]
    for i1, h1, s1 in out[1:]:
        assert i0 == i1
        assert np.array_equal(h0, h1)
        assert all(np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1]) for a, b in zip(s0, s1))


def test_bad_plan_leaves_h_and_states_unchanged(libs):
    lib, _ = libs
    rng = np.random.default_rng(23)
    L = LF.Linear(rng)
    c, s = L.copy_states()
    p = L.plan(c, s)
    p.M_qkv = 3 * LF.V - 64
    h = rng.normal(0, 1, LF.HIDDEN).astype(np.float32)
    h0 = h.copy()
    lib.forward_linear_layer(ctypes.byref(p), h.ctypes.data)
    assert np.array_equal(h, h0) and np.array_equal(c, L.conv_s) and np.array_equal(s, L.state)
    assert b"linear-layer plan" in lib.qwen_b200_last_error()
