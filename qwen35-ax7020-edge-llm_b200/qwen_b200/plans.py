"""The token loop's plan structures and a seeded synthetic Qwen3.5-0.8B
model for them.

LinearLayerPlanC / MlpPlanC are the engine's ctypes layouts
(qwen_real_engine.py:20-74), byte-identical to include/qwen_b200.h, so one
plan drives this library's forward_linear_layer / forward_token_c, the
reference's own C build and the test oracle alike.  TokenModel builds 24
layers over numpy arrays (random BFP8 weights, fp32 norm and gate vectors,
states, a bf16 embedding table) for the benchmark and the tests; its
attention_stand_in() replaces the engine's full-attention callback, whose
attention is not on this library's path."""
from __future__ import annotations

import ctypes

import numpy as np

_P = ctypes.c_void_p
_I = ctypes.c_int

HIDDEN, HEADS, HEAD_DIM, FFN, VOCAB, LAYERS = 1024, 16, 128, 3584, 65536, 24
V = HEADS * HEAD_DIM
FULL_LAYERS = (3, 7, 11, 15, 19, 23)   # the 0.8B model's full-attention layers (config.json)

CALLBACK = ctypes.CFUNCTYPE(None, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p)


class LinearLayerPlanC(ctypes.Structure):
    _fields_ = [("in_ln_w", _P), ("mant_qkv", _P), ("exp_qkv", _P), ("M_qkv", _I), ("K_qkv", _I),
                ("conv_w", _P), ("conv_s", _P), ("wa", _P), ("wb", _P), ("nea", _P), ("dt", _P), ("state", _P),
                ("mant_z", _P), ("exp_z", _P), ("M_z", _I), ("K_z", _I), ("norm_w", _P),
                ("mant_o", _P), ("exp_o", _P), ("M_o", _I), ("K_o", _I), ("post_ln_w", _P),
                ("mant_gate", _P), ("exp_gate", _P), ("M_gate", _I), ("K_gate", _I),
                ("mant_up", _P), ("exp_up", _P), ("M_up", _I), ("K_up", _I),
                ("mant_down", _P), ("exp_down", _P), ("M_down", _I), ("K_down", _I)]


class MlpPlanC(ctypes.Structure):
    _fields_ = [("post_ln_w", _P), ("mant_gate", _P), ("exp_gate", _P), ("M_gate", _I), ("K_gate", _I),
                ("mant_up", _P), ("exp_up", _P), ("M_up", _I), ("K_up", _I),
                ("mant_down", _P), ("exp_down", _P), ("M_down", _I), ("K_down", _I)]


def bfp8_matrix(rng, M, K):
    """One SoA tensor as the weight file holds it (mantissas, then the
    exponents right behind them): int8 mantissas in [-127, 127], exponents
    120..124, i.e. weights of a few hundredths."""
    buf = np.empty(M * K + M * (K // 64), dtype=np.uint8)
    buf[:M * K] = rng.integers(-127, 128, M * K, dtype=np.int64).astype(np.int8).view(np.uint8)
    buf[M * K:] = rng.integers(120, 125, M * (K // 64)).astype(np.uint8)
    return buf


class Mlp:
    def __init__(self, rng, hidden=HIDDEN, ffn=FFN):
        self.hidden, self.ffn = hidden, ffn
        self.post_ln = rng.normal(0, 0.1, hidden).astype(np.float32)
        self.gate = bfp8_matrix(rng, ffn, hidden)
        self.up = bfp8_matrix(rng, ffn, hidden)
        self.down = bfp8_matrix(rng, hidden, ffn)

    def plan(self) -> MlpPlanC:
        p = MlpPlanC()
        p.post_ln_w = self.post_ln.ctypes.data
        H, F = self.hidden, self.ffn
        for name, buf, M, K in (("gate", self.gate, F, H), ("up", self.up, F, H), ("down", self.down, H, F)):
            setattr(p, "mant_" + name, buf.ctypes.data)
            setattr(p, "exp_" + name, buf.ctypes.data + M * K)
            setattr(p, "M_" + name, M)
            setattr(p, "K_" + name, K)
        return p


class Linear:
    """Weights of one Gated-DeltaNet layer (plus its MLP) and a set of
    mutable states; copy_states() gives an independent set for another
    implementation."""

    def __init__(self, rng, mlp: Mlp | None = None, hidden=HIDDEN, heads=HEADS, ffn=FFN):
        self.hidden, self.heads = hidden, heads
        v = self.v = heads * HEAD_DIM
        self.in_ln = rng.normal(0, 0.1, hidden).astype(np.float32)
        self.qkv = bfp8_matrix(rng, 3 * v, hidden)
        self.z = bfp8_matrix(rng, v, hidden)
        self.o = bfp8_matrix(rng, hidden, v)
        self.conv_w = rng.normal(0, 0.3, (3 * v, 4)).astype(np.float32)
        self.wa = rng.normal(0, 0.03, (heads, hidden)).astype(np.float32)
        self.wb = rng.normal(0, 0.03, (heads, hidden)).astype(np.float32)
        self.nea = (-np.exp(rng.uniform(0.0, 1.5, heads))).astype(np.float32)
        self.dt = rng.uniform(-1.0, 1.0, heads).astype(np.float32)
        self.norm_w = rng.normal(1.0, 0.1, HEAD_DIM).astype(np.float32)
        self.mlp = mlp if mlp is not None else Mlp(rng, hidden, ffn)
        self.conv_s = rng.normal(0, 0.5, (3, 3 * v)).astype(np.float32)
        self.state = rng.normal(0, 0.05, (heads, HEAD_DIM * HEAD_DIM)).astype(np.float32)

    def copy_states(self):
        return self.conv_s.copy(), self.state.copy()

    def plan(self, conv_s=None, state=None) -> LinearLayerPlanC:
        conv_s = self.conv_s if conv_s is None else conv_s
        state = self.state if state is None else state
        p = LinearLayerPlanC()
        p.in_ln_w = self.in_ln.ctypes.data
        H, v = self.hidden, self.v
        for name, buf, M, K in (("qkv", self.qkv, 3 * v, H), ("z", self.z, v, H), ("o", self.o, H, v)):
            setattr(p, "mant_" + name, buf.ctypes.data)
            setattr(p, "exp_" + name, buf.ctypes.data + M * K)
            setattr(p, "M_" + name, M)
            setattr(p, "K_" + name, K)
        p.conv_w = self.conv_w.ctypes.data
        p.conv_s = conv_s.ctypes.data
        p.wa = self.wa.ctypes.data
        p.wb = self.wb.ctypes.data
        p.nea = self.nea.ctypes.data
        p.dt = self.dt.ctypes.data
        p.state = state.ctypes.data
        p.norm_w = self.norm_w.ctypes.data
        m = self.mlp.plan()
        for f, _ in MlpPlanC._fields_:
            setattr(p, f, getattr(m, f))
        return p


class TokenModel:
    """24 layers over two weight sets (every linear layer shares one set of
    weights but owns its states; every full-attention MLP shares another),
    a bf16 embedding table and the final norm -- enough for forward_token_c
    without 24 layers' worth of distinct weights."""

    def __init__(self, seed=0):
        rng = np.random.default_rng(seed)
        self.lin_w = Linear(rng)
        self.mlp_w = Mlp(rng)
        e = rng.normal(0, 0.05, (VOCAB, HIDDEN)).astype(np.float32)
        self.embed = (e.view(np.uint32) >> 16).astype(np.uint16)
        self.final_ln = rng.normal(0, 0.1, HIDDEN).astype(np.float32)
        self.is_full = np.array([1 if l in FULL_LAYERS else 0 for l in range(LAYERS)], dtype=np.int32)
        self.n_linear = LAYERS - len(FULL_LAYERS)
        self.states0 = [(rng.normal(0, 0.5, (3, 3 * V)).astype(np.float32),
                         rng.normal(0, 0.05, (HEADS, HEAD_DIM * HEAD_DIM)).astype(np.float32))
                        for _ in range(self.n_linear)]

    def fresh_states(self):
        return [(c.copy(), s.copy()) for c, s in self.states0]

    def plans(self, states):
        """Plan arrays over `states` (from fresh_states()); the model keeps
        the state arrays alive as long as it lives, since the plans hold
        only their addresses."""
        self._live = getattr(self, "_live", []) + [states]
        lps = (LinearLayerPlanC * self.n_linear)()
        for i, (c, s) in enumerate(states):
            lps[i] = self.lin_w.plan(c, s)
        mps = (MlpPlanC * LAYERS)()
        for l in range(LAYERS):
            if self.is_full[l]:
                mps[l] = self.mlp_w.plan()
        return lps, mps


def attention_stand_in():
    """A deterministic stand-in for the engine's full-attention callback:
    h += 0.05 * sin(l + i / 64) (the real callback runs attention on the host
    and adds its output the same way, qwen_real_engine.py:1088)."""
    idx = np.arange(HIDDEN, dtype=np.float32)

    def cb(layer, h_ptr, ctx):
        h = np.ctypeslib.as_array(ctypes.cast(h_ptr, ctypes.POINTER(ctypes.c_float)), shape=(HIDDEN,))
        h += (0.05 * np.sin(layer + idx / 64.0)).astype(np.float32)

    return CALLBACK(cb)
