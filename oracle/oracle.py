"""CPU oracle for the BFP8 GEMV / lm_head hot path -- TEST INFRASTRUCTURE ONLY.

numpy front end over ``oracle/_build/liboracle.so`` (the C restatement in
``bfp8_oracle.c``) plus a numpy restatement of the reference weight packer.
Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline leg use
this module, and only as the checker; the product never imports it.

Reference files restated here (paths inside ideal1128/qwen35-ax7020-edge-llm):
  * packer            05-主机侧源码/bfp8_packer.py:53-86
  * everything else   see the header of bfp8_oracle.c
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int


def build() -> str:
    """Compile liboracle.so (gcc, -ffp-contract=off) if it is missing or stale."""
    src = os.path.join(_HERE, "bfp8_oracle.c")
    if (not os.path.exists(_LIB_PATH)
            or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
        subprocess.run(["make", "-s", "-C", _HERE, "CC=gcc", "_build/liboracle.so"],
                       check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        sigs = {
            "orc_exp_scale": [_P],
            "orc_quant_x": [_P, _I, _P, _P],
            "orc_lane_dots": [_P, _P, _I, _I, _P],
            "orc_block_dots": [_P, _P, _I, _I, _P],
            "orc_bfp8_gemv_q": [_P, _P, _P, _P, _P, _I, _I],
            "orc_bfp8_gemv_neon": [_P, _P, _P, _P, _I, _I],
            "orc_bfp8_gemv_neon_batch": [_P, _P, _P, _P, _I, _I, _I],
            "orc_bfp8_gemv_scalar": [_P, _P, _P, _P, _I, _I],
            "orc_bfp8_gemv_rtl20": [_P, _P, _P, _P, _P, _I, _I],
            "orc_lm_scores_neon": [_P, _P, _P, _I, _I, _I],
            "orc_lm_scores_scalar": [_P, _P, _P, _I, _I],
            "orc_argmax": [_P, _I],
            "orc_topk": [_P, _I, _I, _P, _P],
            "orc_lm_head_argmax": [_P, _P, _I, _I],
            "orc_lm_head_topk": [_P, _P, _I, _I, _I, _P, _P],
            "orc_bfp8_lm_head": [_P, _P, _P, _I, _I, _I, _P, _P, _P],
            "orc_xorshift32": [_P, _P, ctypes.c_size_t],
            "orc_selftest_fill": [_P, _P, ctypes.c_size_t, _P, ctypes.c_size_t],
            "orc_rmsnorm_neon": [_P, _P, _P, _I, ctypes.c_float],
            "orc_rmsnorm_scalar": [_P, _P, _P, _I, ctypes.c_float],
            "orc_add_residual": [_P, _P, _I, _I],
            "orc_swiglu": [_P, _P, _P, _I, _I],
            "orc_conv1d_silu": [_P, _P, _P, _P, _I, _I],
            "orc_qk_l2norm": [_P, _P, _I, _I, _I],
            "orc_gdn_gates": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I],
            "orc_gdn_step": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I],
            "orc_rmsnorm_gated": [_P, _P, _P, _P, _I, _I, ctypes.c_float, _I],
            "orc_forward_mlp": [_P, _P, _I],
            "orc_forward_linear_layer": [_P, _P, _I],
            "orc_forward_token": [_I, _P, _P, _P, _P, _P, _P, _P, _P, _I],
        }
        for name, args in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _I if name in ("orc_argmax", "orc_topk", "orc_lm_head_argmax",
                                        "orc_lm_head_topk", "orc_bfp8_lm_head",
                                        "orc_bfp8_gemv_rtl20", "orc_forward_token") else None
        _lib = L
    return _lib


def _c(a, dtype):
    a = np.ascontiguousarray(a, dtype=dtype)
    return a, a.ctypes.data


# ----------------------------------------------------------------- packer
def pack_bfp8(w: np.ndarray):
    """Block-64 BFP8 SoA packing of a [M, K] float matrix.

    Restates 05-主机侧源码/bfp8_packer.py:53-86 in float32 numpy arithmetic:
    e = clip(ceil(log2(max|w|)) + 127, 0, 255) per 64-block (127 for blocks
    with max < 1e-12), m = clip(round_half_even(w * 2^(7 - (e - 127))),
    -128, 127).  Returns (mant int8 [M, K], exps uint8 [M, K/64]).
    """
    w = np.ascontiguousarray(w, dtype=np.float32)
    M, K = w.shape
    assert K % 64 == 0
    blk = w.reshape(M, K // 64, 64)
    peak = np.abs(blk).max(axis=2)
    lg = np.ceil(np.log2(np.maximum(peak, np.float32(1e-12))))
    e = np.clip(lg + np.float32(127), 0, 255).astype(np.uint8)
    zero = peak < np.float32(1e-12)
    e[zero] = 127
    step = np.float32(2.0) ** (np.float32(7.0) - (e.astype(np.float32) - np.float32(127)))
    q = np.round(blk * step[:, :, None])
    m = np.clip(q, -128, 127).astype(np.int8)
    m[zero] = 0
    return m.reshape(M, K), e


def soa_bytes(mant: np.ndarray, exps: np.ndarray) -> bytes:
    """Serialise one tensor the way the weight file stores it: mantissas then
    exponents padded with 127 to a multiple of 8 (bfp8_packer.py:80-86)."""
    e = exps.reshape(-1)
    pad = (-len(e)) % 8
    if pad:
        e = np.concatenate([e, np.full(pad, 127, np.uint8)])
    return mant.tobytes() + e.tobytes()


def dequant(mant: np.ndarray, exps: np.ndarray) -> np.ndarray:
    M, K = mant.shape
    s = np.ldexp(np.float32(1.0), exps.astype(np.int32) - 134).astype(np.float32)
    return (mant.reshape(M, K // 64, 64).astype(np.float32) * s[:, :, None]).reshape(M, K)


# -------------------------------------------------------------- wrappers
def exp_scale():
    out = np.zeros(256, np.float32)
    lib().orc_exp_scale(out.ctypes.data)
    return out


def quant_x(x):
    x, px = _c(x, np.float32)
    K = x.shape[-1]
    xq = np.zeros(K, np.int16)
    xs = np.zeros(K // 64, np.float32)
    lib().orc_quant_x(px, K, xq.ctypes.data, xs.ctypes.data)
    return xq, xs


def lane_dots(mant, xq):
    mant, pm = _c(mant, np.int8)
    xq, px = _c(xq, np.int16)
    M, K = mant.shape
    out = np.zeros((M, K // 64, 4), np.int32)
    lib().orc_lane_dots(pm, px, M, K, out.ctypes.data)
    return out


def block_dots(mant, xq):
    mant, pm = _c(mant, np.int8)
    xq, px = _c(xq, np.int16)
    M, K = mant.shape
    out = np.zeros((M, K // 64), np.int32)
    lib().orc_block_dots(pm, px, M, K, out.ctypes.data)
    return out


def bfp8_gemv(x, mant, exps):
    """Reference NEON int16 path: y fp32 [M] (or [B, M] for x [B, K])."""
    mant, pm = _c(mant, np.int8)
    exps, pe = _c(exps, np.uint8)
    M, K = mant.shape
    x = np.asarray(x, np.float32)
    if x.ndim == 2:
        B = x.shape[0]
        x, px = _c(x, np.float32)
        y = np.zeros((B, M), np.float32)
        lib().orc_bfp8_gemv_neon_batch(y.ctypes.data, px, pm, pe, B, M, K)
        return y
    x, px = _c(x, np.float32)
    y = np.zeros(M, np.float32)
    lib().orc_bfp8_gemv_neon(y.ctypes.data, px, pm, pe, M, K)
    return y


def rmsnorm(x, w, eps, neon=True):
    """rmsnorm (qwen_kernels_opt.c:140-172): the NEON build's order (what the
    board runs) or the portable build's."""
    x, px = _c(x, np.float32)
    w, pw = _c(w, np.float32)
    y = np.empty_like(x)
    fn = lib().orc_rmsnorm_neon if neon else lib().orc_rmsnorm_scalar
    fn(y.ctypes.data, px, pw, x.size, float(eps))
    return y


def add_residual(x, res, neon=True):
    """x + res as add_residual (qwen_kernels_opt.c:388-396) computes it in
    place: the NEON build's flushed lanes or the portable build."""
    y = np.array(x, dtype=np.float32, copy=True)
    r, pr = _c(res, np.float32)
    lib().orc_add_residual(y.ctypes.data, pr, y.size, 1 if neon else 0)
    return y


def swiglu(gate, up, neon=True):
    """(g / (1 + exp(-g))) * up as swiglu (qwen_kernels_opt.c:365-386)
    computes it: the NEON build (exp_neon, flushed lanes) or the portable
    build (expf on every element)."""
    g, pg = _c(gate, np.float32)
    u, pu = _c(up, np.float32)
    y = np.zeros(g.size, np.float32)
    lib().orc_swiglu(y.ctypes.data, pg, pu, g.size, 1 if neon else 0)
    return y


def bfp8_gemv_q(xq, xs, mant, exps):
    mant, pm = _c(mant, np.int8)
    exps, pe = _c(exps, np.uint8)
    xq, pq = _c(xq, np.int16)
    xs, ps = _c(xs, np.float32)
    M, K = mant.shape
    y = np.zeros(M, np.float32)
    lib().orc_bfp8_gemv_q(y.ctypes.data, pq, ps, pm, pe, M, K)
    return y


def bfp8_gemv_scalar(x, mant, exps):
    mant, pm = _c(mant, np.int8)
    exps, pe = _c(exps, np.uint8)
    x, px = _c(x, np.float32)
    M, K = mant.shape
    y = np.zeros(M, np.float32)
    lib().orc_bfp8_gemv_scalar(y.ctypes.data, px, pm, pe, M, K)
    return y


def bfp8_gemv_numpy(x, mant, exps):
    """The reference engine's numpy fallback GEMV, used when no C kernel
    library is loaded (04-板载脚本与工具/qwen_real_engine.py:1233-1239): no
    activation quantization; per row and 64-block the float32 sum of m * x
    (numpy's pairwise reduction over the block), times 2^(e - 134) computed
    in float32, then the float32 sum over the row's blocks."""
    mant = np.asarray(mant, np.int8)
    exps = np.asarray(exps, np.uint8)
    x = np.asarray(x, np.float32)
    M, K = mant.shape
    nb = K // 64
    scales = (2.0 ** (exps.astype(np.float32) - 134.0)).reshape(M, nb)
    dots = np.sum(mant.reshape(M, nb, 64).astype(np.float32) * x.reshape(nb, 64), axis=-1)
    return np.sum(dots * scales, axis=-1)


def bfp8_gemv_rtl20(xq, xs, mant, exps):
    """gemv_core dequant mode: (int32 words floor(y*2^20) [M], flags)."""
    mant, pm = _c(mant, np.int8)
    exps, pe = _c(exps, np.uint8)
    xq, pq = _c(xq, np.int16)
    xs, ps = _c(xs, np.float32)
    M, K = mant.shape
    y = np.zeros(M, np.int32)
    flags = lib().orc_bfp8_gemv_rtl20(y.ctypes.data, pq, ps, pm, pe, M, K)
    return y, flags


def lm_scores(h, E, with_tail=True):
    h, ph = _c(h, np.float32)
    E, pE = _c(E, np.uint16)
    V, H = E.shape
    s = np.zeros(V, np.float32)
    lib().orc_lm_scores_neon(s.ctypes.data, ph, pE, V, H, 1 if with_tail else 0)
    return s


def lm_scores_scalar(h, E):
    h, ph = _c(h, np.float32)
    E, pE = _c(E, np.uint16)
    V, H = E.shape
    s = np.zeros(V, np.float32)
    lib().orc_lm_scores_scalar(s.ctypes.data, ph, pE, V, H)
    return s


def argmax(scores):
    scores, p = _c(scores, np.float32)
    return int(lib().orc_argmax(p, scores.shape[0]))


def topk(scores, k):
    scores, p = _c(scores, np.float32)
    kk = max(0, min(k, scores.shape[0]))
    ids = np.zeros(max(kk, 1), np.int32)
    out = np.zeros(max(kk, 1), np.float32)
    n = lib().orc_topk(p, scores.shape[0], k, ids.ctypes.data, out.ctypes.data)
    return ids[:n].copy(), out[:n].copy()


def lm_head_argmax(h, E):
    h, ph = _c(h, np.float32)
    E, pE = _c(E, np.uint16)
    V, H = E.shape
    return int(lib().orc_lm_head_argmax(ph, pE, V, H))


def lm_head_topk(h, E, k):
    h, ph = _c(h, np.float32)
    E, pE = _c(E, np.uint16)
    V, H = E.shape
    kk = max(1, min(k, V))
    ids = np.zeros(kk, np.int32)
    out = np.zeros(kk, np.float32)
    n = lib().orc_lm_head_topk(ph, pE, V, H, k, ids.ctypes.data, out.ctypes.data)
    return ids[:n].copy(), out[:n].copy()


def bfp8_lm_head(h, mant, exps, k):
    """BFP8 lm_head: (argmax id, top-k ids, top-k scores)."""
    h, ph = _c(h, np.float32)
    mant, pm = _c(mant, np.int8)
    exps, pe = _c(exps, np.uint8)
    V, H = mant.shape
    kk = max(1, min(k, V))
    ids = np.zeros(kk, np.int32)
    out = np.zeros(kk, np.float32)
    am = ctypes.c_int(0)
    n = lib().orc_bfp8_lm_head(ph, pm, pe, V, H, k, ids.ctypes.data, out.ctypes.data,
                               ctypes.addressof(am))
    return am.value, ids[:n].copy(), out[:n].copy()


# ------------------------------------------------------------ generators
class XorShift32:
    """Marsaglia xorshift32 (13, 17, 5), zero state remapped to 0x9E3779B9 --
    the reference sampler's generator (qwen_sampling.c:360-368)."""

    def __init__(self, state: int):
        self.state = ctypes.c_uint32(state & 0xFFFFFFFF)

    def next(self, n: int) -> np.ndarray:
        out = np.empty(n, np.uint32)
        lib().orc_xorshift32(ctypes.addressof(self.state), out.ctypes.data, n)
        return out

    def selftest_fill(self, vocab: int, hidden: int):
        """(table uint16 [vocab, hidden], h fp32 [hidden]) drawn exactly like
        the reference self-test (qwen_sampling.c:544-561, 930-931)."""
        tab = np.empty((vocab, hidden), np.uint16)
        h = np.empty(hidden, np.float32)
        lib().orc_selftest_fill(ctypes.addressof(self.state), tab.ctypes.data, tab.size,
                                h.ctypes.data, h.size)
        return tab, h
