"""Device-tensor API of the hot path (PyTorch tensors in, PyTorch tensors out).

Every function runs on torch's current CUDA stream and raises on failure.
The arithmetic is the reference NEON build's, bit-for-bit (see
include/qwen_b200.h).  Calls that return fresh tensors go through the
PyTorch operators ``torch.ops.qwen_b200.*`` (csrc/torch_ops.cpp, errors as
RuntimeError); calls that write caller-provided buffers (``out=``), grouped
plans and the sharded launches call the C ABI directly (errors as
KernelError).  Both reach the same entry points of libqwen_kernels_b200.so.

Reference routines served (ideal1128/qwen35-ax7020-edge-llm):
  quant_block64   04-板载脚本与工具/qwen_kernels_opt.c:182-205 (quant_x_blocks)
  bfp8_gemv       04-板载脚本与工具/qwen_kernels_opt.c:207-326
  lm_head_bf16    04-板载脚本与工具/qwen_kernels_opt.c:401-506 (lm_head_argmax)
                  04-板载脚本与工具/qwen_sampling.c:283-353    (lm_head_topk)
  lm_head_bfp8    bfp8_gemv scores + the same selection rules (no reference routine)
  pack_bfp8       05-主机侧源码/bfp8_packer.py:53-86
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from ._lib import KernelError, check, load, torch_ops

T = torch_ops()   # torch.ops.qwen_b200: loading fails loudly without the built libraries

__all__ = [
    "KernelError", "quant_block64", "bfp8_gemv", "bfp8_gemv_fast", "bfp8_gemv_q", "lm_head_bf16", "lm_head_bfp8",
    "pack_bfp8", "LinearStack", "rmsnorm_bfp8_gemv", "residual_rmsnorm_bfp8_gemv", "LmResult", "Planes", "quant_planes", "bfp8_gemm_tc", "BatchedStack",
    "PeerRegion", "ShardedLinearStack", "quant_planes_wait", "ShardedBatchedStack", "swiglu_quant_sharded",
    "sync_epoch_base", "sync_epoch_advance",
    "quant_record_bytes", "planes_record_bytes", "planes_view", "STACK_FAST", "STACK_FIXED_SPLIT", "STACK_Q_INPUT",
]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _need(t: torch.Tensor, dtype: torch.dtype, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    return t.contiguous()


def quant_block64(x: torch.Tensor):
    """x fp32 [..., K] -> (xq int16 [..., K], xs fp32 [..., K/64])."""
    return T.quant_block64(_need(x, torch.float32, "x"))


def bfp8_gemv(x: torch.Tensor, mant: torch.Tensor, exps: torch.Tensor, out: torch.Tensor | None = None):
    """y = BFP8 GEMV.  x fp32 [K] or [B, K]; mant int8 [M, K]; exps uint8 [M, K/64]."""
    x = _need(x, torch.float32, "x")
    mant = _need(mant, torch.int8, "mant")
    exps = _need(exps, torch.uint8, "exps")
    M, K = mant.shape
    if x.shape[-1] != K or exps.numel() < M * (K // 64):
        raise ValueError("shape mismatch")
    if out is None:
        return T.bfp8_gemv(x, mant, exps, "exact")
    rows = x.reshape(-1, K)
    y = out
    yr = y.view(-1, M)
    L = load()
    for i in range(rows.shape[0]):
        check(L.qwen_b200_gemv_dev(_ptr(yr[i]), _ptr(rows[i]), _ptr(mant), _ptr(exps), M, K, _stream()),
              "bfp8_gemv")
    return y


def bfp8_gemv_fast(x: torch.Tensor, mant: torch.Tensor, exps: torch.Tensor, out: torch.Tensor | None = None):
    """Fast-mode GEMV (split-K, fused multiply-add per block); within
    1e-5 * sum|terms| of bfp8_gemv.  x fp32 [K]; K a multiple of 512."""
    x = _need(x, torch.float32, "x")
    mant = _need(mant, torch.int8, "mant")
    exps = _need(exps, torch.uint8, "exps")
    M, K = mant.shape
    if out is None:
        return T.bfp8_gemv(x, mant, exps, "fast")
    y = out
    check(load().qwen_b200_gemv_fast_dev(_ptr(y), _ptr(x), _ptr(mant), _ptr(exps), M, K, _stream()), "bfp8_gemv_fast")
    return y


def rmsnorm_bfp8_gemv(x: torch.Tensor, norm_w: torch.Tensor, eps: float, mant: torch.Tensor, exps: torch.Tensor,
                      out: torch.Tensor | None = None):
    """y [M] = bfp8_gemv(rmsnorm(x, norm_w, eps)) in one launch, bit for bit
    the reference's rmsnorm (NEON order) followed by its quantizer and GEMV.
    K a multiple of 512 and <= 6144."""
    x = _need(x, torch.float32, "x")
    norm_w = _need(norm_w, torch.float32, "norm_w")
    mant = _need(mant, torch.int8, "mant")
    exps = _need(exps, torch.uint8, "exps")
    M, K = mant.shape
    if x.numel() != K or norm_w.numel() != K:
        raise ValueError("shape mismatch")
    y = out if out is not None else torch.empty(M, dtype=torch.float32, device=mant.device)
    check(load().qwen_b200_rmsnorm_gemv_dev(_ptr(y), _ptr(x), _ptr(norm_w), float(eps), _ptr(mant), _ptr(exps), M, K,
                                            _stream()), "rmsnorm_bfp8_gemv")
    return y


def residual_rmsnorm_bfp8_gemv(x: torch.Tensor, res: torch.Tensor, norm_w: torch.Tensor, eps: float,
                               mant: torch.Tensor, exps: torch.Tensor):
    """(x + res, bfp8_gemv(rmsnorm(x + res, norm_w, eps))) in one launch, bit
    for bit the reference's add_residual, rmsnorm, quantizer and GEMV.
    K a multiple of 512 and <= 6144.  Returns (y [M], x_out [K])."""
    x = _need(x, torch.float32, "x")
    res = _need(res, torch.float32, "res")
    norm_w = _need(norm_w, torch.float32, "norm_w")
    mant = _need(mant, torch.int8, "mant")
    exps = _need(exps, torch.uint8, "exps")
    M, K = mant.shape
    if x.numel() != K or res.numel() != K or norm_w.numel() != K:
        raise ValueError("shape mismatch")
    y = torch.empty(M, dtype=torch.float32, device=mant.device)
    x_out = torch.empty(K, dtype=torch.float32, device=mant.device)
    check(load().qwen_b200_residual_rmsnorm_gemv_dev(_ptr(y), _ptr(x_out), _ptr(x), _ptr(res), _ptr(norm_w),
                                                     float(eps), _ptr(mant), _ptr(exps), M, K, _stream()),
          "residual_rmsnorm_bfp8_gemv")
    return y, x_out


def rmsnorm_bfp8_gemv2(x: torch.Tensor, norm_w: torch.Tensor, eps: float, w0, w1, res: torch.Tensor | None = None):
    """Two projections of one normalized vector in one launch (a layer's qkv
    and z, an MLP's gate and up): (y0, y1) = the GEMVs of w0 = (mant0, exps0)
    and w1 = (mant1, exps1) of rmsnorm(x) -- or, with res, of x + res, which
    is returned as a third element.  Bit for bit rmsnorm_bfp8_gemv /
    residual_rmsnorm_bfp8_gemv of each.  K a multiple of 512 and <= 6144."""
    x = _need(x, torch.float32, "x")
    norm_w = _need(norm_w, torch.float32, "norm_w")
    m0, e0 = _need(w0[0], torch.int8, "mant0"), _need(w0[1], torch.uint8, "exps0")
    m1, e1 = _need(w1[0], torch.int8, "mant1"), _need(w1[1], torch.uint8, "exps1")
    M0, K = m0.shape
    M1, K1 = m1.shape
    if K1 != K or x.numel() != K or norm_w.numel() != K:
        raise ValueError("shape mismatch")
    y0 = torch.empty(M0, dtype=torch.float32, device=m0.device)
    y1 = torch.empty(M1, dtype=torch.float32, device=m0.device)
    x_out = None
    if res is not None:
        res = _need(res, torch.float32, "res")
        if res.numel() != K:
            raise ValueError("shape mismatch")
        x_out = torch.empty(K, dtype=torch.float32, device=m0.device)
    check(load().qwen_b200_rmsnorm_gemv2_dev(_ptr(y0), _ptr(y1), _ptr(x_out) if x_out is not None else None, _ptr(x),
                                             _ptr(res) if res is not None else None, _ptr(norm_w), float(eps),
                                             _ptr(m0), _ptr(e0), M0, _ptr(m1), _ptr(e1), M1, K, _stream()),
          "rmsnorm_bfp8_gemv2")
    return (y0, y1) if res is None else (y0, y1, x_out)


def bfp8_gemv_q(xq: torch.Tensor, xs: torch.Tensor, mant: torch.Tensor, exps: torch.Tensor):
    """y = BFP8 GEMV of an already quantized activation (xq int16 [K], xs fp32 [K/64])."""
    return T.bfp8_gemv_q(_need(xq, torch.int16, "xq"), _need(xs, torch.float32, "xs"),
                         _need(mant, torch.int8, "mant"), _need(exps, torch.uint8, "exps"), "exact")


def swiglu_bfp8_gemv(gate: torch.Tensor, up: torch.Tensor, mant: torch.Tensor, exps: torch.Tensor):
    """y = BFP8 GEMV of swiglu(gate, up) in one launch, swiglu as the
    reference's NEON build computes it (qwen_kernels_opt.c:332-386): the MLP's
    down projection with its activation fused in front.  K <= 6144."""
    gate = _need(gate, torch.float32, "gate")
    up = _need(up, torch.float32, "up")
    mant = _need(mant, torch.int8, "mant")
    exps = _need(exps, torch.uint8, "exps")
    M, K = mant.shape
    y = torch.empty(M, dtype=torch.float32, device=mant.device)
    check(load().qwen_b200_swiglu_gemv_dev(_ptr(y), _ptr(gate), _ptr(up), _ptr(mant), _ptr(exps), M, K,
                                           _stream()), "swiglu_bfp8_gemv")
    return y


def mlp_block(h: torch.Tensor, res: torch.Tensor, post_ln_w: torch.Tensor, gate, up, down, eps: float = 1e-6):
    """forward_mlp (qwen_kernels_opt.c:994-1003) on the device in three
    launches, with the residual add of the block before it folded in front:
    h1 = h + res (add_residual), g / u = the gate / up GEMVs of rmsnorm(h1),
    d = the down GEMV of swiglu(g, u); returns (h1, d), and the next block
    adds d (the reference's closing add_residual(h, down_buf)).  ``gate``,
    ``up``, ``down`` are (mant, exps) pairs.  Every step is the reference's
    NEON-build arithmetic, so h1 and d equal its values bit for bit."""
    g, h1 = residual_rmsnorm_bfp8_gemv(h, res, post_ln_w, eps, *gate)
    u = rmsnorm_bfp8_gemv(h1, post_ln_w, eps, *up)
    return h1, swiglu_bfp8_gemv(g, u, *down)


def bfp8_gemv_rtl20(mant: torch.Tensor, exps: torch.Tensor, x: torch.Tensor | None = None,
                    xq: torch.Tensor | None = None, xs: torch.Tensor | None = None):
    """The FPGA gemv_core dequant mode (02-RTL与仿真/gemv_core.v:299-534):
    returns (words int32 [M], flags) with words = floor(y * 2^20) from the
    RTL's saturating 64-bit fixed-point sum and flags bit 0 = a term or row
    sum saturated, bit 1 = an output word clamped.  The activation is fp32
    ``x`` (quantized by the reference rule) or ``xq`` int16 / ``xs`` fp32."""
    mant = _need(mant, torch.int8, "mant")
    exps = _need(exps, torch.uint8, "exps")
    if (x is None) == (xq is None) or (xq is not None and xs is None):
        raise ValueError("bfp8_gemv_rtl20: give x, or xq and xs")
    M, K = mant.shape
    words = torch.empty(M, dtype=torch.int32, device=mant.device)
    flags = torch.zeros(1, dtype=torch.int32, device=mant.device)
    if x is not None:
        x = _need(x, torch.float32, "x")
        args = (_ptr(x), None, None)
    else:
        xq = _need(xq, torch.int16, "xq")
        xs = _need(xs, torch.float32, "xs")
        args = (None, _ptr(xq), _ptr(xs))
    check(load().qwen_b200_gemv_rtl20_dev(_ptr(words), *args, _ptr(mant), _ptr(exps), M, K, _ptr(flags),
                                          _stream()), "bfp8_gemv_rtl20")
    return words, int(flags.item())


@dataclass
class Planes:
    """Batched int16 block-64 activations as two signed int8 planes
    (xq = 256*hi + lo, lo the low byte of xq as a signed int8):
    ``planes`` int8 [2, B, K] (plane 0 = hi, plane 1 = lo) and
    block scales ``xs_t`` fp32 [K/64, ldxs] (block-major, first B columns used)."""
    planes: torch.Tensor
    xs_t: torch.Tensor
    B: int
    K: int

    @property
    def ldxs(self) -> int:
        return self.xs_t.shape[1]

    def xq(self) -> torch.Tensor:
        """The int16 activations [B, K] these planes encode."""
        hi = self.planes[0].to(torch.int32)
        lo = self.planes[1].to(torch.int32)
        return (hi * 256 + lo).to(torch.int16)

    def xs(self) -> torch.Tensor:
        """Block scales [B, K/64]."""
        return self.xs_t[:, :self.B].t().contiguous()


def planes_empty(B: int, K: int, device) -> Planes:
    ldxs = (B + 3) // 4 * 4
    return Planes(torch.empty((2, B, K), dtype=torch.int8, device=device),
                  torch.zeros((K // 64, ldxs), dtype=torch.float32, device=device), B, K)


def quant_planes(x: torch.Tensor, out: Planes | None = None) -> Planes:
    """x fp32 [B, K] -> Planes, with the reference quantizer's arithmetic
    (256*hi + lo equals quant_block64's xq bit for bit)."""
    x = _need(x, torch.float32, "x")
    B, K = x.shape
    if out is None:
        planes, xs_t = T.quant_planes(x)
        return Planes(planes, xs_t, B, K)
    p = out
    check(load().qwen_b200_quant_planes_dev(_ptr(x), B, K, _ptr(p.planes), _ptr(p.xs_t), p.ldxs, _stream()),
          "quant_planes")
    return p


def bfp8_gemm_tc(p: Planes, mant: torch.Tensor, exps: torch.Tensor, out: torch.Tensor | None = None,
                 dots: bool = False):
    """y fp32 [B, M] = BFP8 W [M, K] x planar activations, on tcgen05 kind::i8.
    With ``dots=True`` also returns the exact int32 block dots [B, M, K/64]."""
    mant = _need(mant, torch.int8, "mant")
    exps = _need(exps, torch.uint8, "exps")
    M, K = mant.shape
    if K != p.K or exps.numel() < M * (K // 64):
        raise ValueError("shape mismatch")
    if out is None and not dots:
        return T.bfp8_gemm_tc(p.planes, p.xs_t, mant, exps)
    y = out if out is not None else torch.empty((p.B, M), dtype=torch.float32, device=mant.device)
    d = torch.empty((p.B, M, K // 64), dtype=torch.int32, device=mant.device) if dots else None
    check(load().qwen_b200_gemm_tc_dev(_ptr(y), _ptr(p.planes), _ptr(p.xs_t), p.ldxs, _ptr(mant), _ptr(exps), M, K,
                                       p.B, _ptr(d) if d is not None else None, _stream()), "bfp8_gemm_tc")
    return (y, d) if dots else y


class BatchedStack:
    """A reusable grouped launch of independent batched BFP8 GEMMs (one
    kernel): ``items`` is a list of (Planes, mant, exps, y fp32 [B, M]) with a
    common B and ldxs."""

    def __init__(self, items):
        n = len(items)
        P = ctypes.c_void_p * n
        I = ctypes.c_int * n
        self._keep = items
        B = items[0][0].B
        ldxs = items[0][0].ldxs
        h = load().qwen_b200_tc_stack_create(
            n, P(*[_ptr(m) for (_, m, _, _) in items]), P(*[_ptr(e) for (_, _, e, _) in items]),
            P(*[_ptr(p.planes) for (p, _, _, _) in items]), P(*[_ptr(p.xs_t) for (p, _, _, _) in items]),
            P(*[_ptr(y) for (_, _, _, y) in items]), I(*[m.shape[0] for (_, m, _, _) in items]),
            I(*[m.shape[1] for (_, m, _, _) in items]), B, ldxs)
        if h <= 0:
            check(h, "BatchedStack")
        self.handle = h

    def run(self, stream: int | None = None) -> None:
        check(load().qwen_b200_tc_stack_run(self.handle, _stream() if stream is None else stream),
              "BatchedStack.run")

    def close(self) -> None:
        if getattr(self, "handle", 0) > 0:
            load().qwen_b200_tc_stack_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class LmResult:
    argmax: torch.Tensor      # int32 [1] (device)
    ids: torch.Tensor         # int32 [k] (device), first n valid
    scores: torch.Tensor      # fp32 [k] (device), first n valid
    n: torch.Tensor           # int32 [1] (device)

    def host(self):
        """(argmax id, ids list, scores list) on the host."""
        n = int(self.n.item())
        return int(self.argmax.item()), self.ids[:n].cpu().tolist(), self.scores[:n].cpu().tolist()


def _lm_outputs(device, k: int) -> LmResult:
    kk = max(k, 1)
    return LmResult(torch.zeros(1, dtype=torch.int32, device=device),
                    torch.zeros(kk, dtype=torch.int32, device=device),
                    torch.zeros(kk, dtype=torch.float32, device=device),
                    torch.zeros(1, dtype=torch.int32, device=device))


def lm_outputs(device, k: int) -> LmResult:
    """Preallocated outputs for repeated lm_head calls (``out=``): the kernels
    overwrite them with plain stores, so one set serves every call."""
    return _lm_outputs(torch.device(device), k)


def _lm_check_out(out: LmResult, device, k: int) -> LmResult:
    kk = max(k, 1)
    for t, dt, n, name in ((out.argmax, torch.int32, 1, "argmax"), (out.ids, torch.int32, kk, "ids"),
                           (out.scores, torch.float32, kk, "scores"), (out.n, torch.int32, 1, "n")):
        if t.device != device or t.dtype != dt or not t.is_contiguous() or t.numel() < n:
            raise ValueError(f"lm_head out.{name}: {dt} contiguous on {device} with >= {n} elements")
    return out


def lm_head_bf16(h: torch.Tensor, E: torch.Tensor, k: int = 0, out: LmResult | None = None) -> LmResult:
    """Tied-embedding lm_head over E bf16 bits [vocab, hidden] (uint16 or bfloat16);
    ``out`` (from lm_outputs) is written instead of fresh outputs."""
    h = _need(h, torch.float32, "h")
    if E.dtype == torch.bfloat16:
        E = E.view(torch.int16)
    if E.dtype not in (torch.int16, torch.uint16):
        raise TypeError("E must hold bf16 bit patterns (bfloat16/int16/uint16)")
    E = E.contiguous()
    V, H = E.shape
    if out is None:
        return LmResult(*T.lm_head_bf16(h, E.view(torch.int16), k))
    r = _lm_check_out(out, h.device, min(k, V))
    check(load().qwen_b200_lm_head_bf16_dev(_ptr(h), _ptr(E), V, H, k, _ptr(r.argmax), _ptr(r.ids),
                                            _ptr(r.scores), _ptr(r.n), _stream()), "lm_head_bf16")
    return r


def lm_head_bfp8(h: torch.Tensor, mant: torch.Tensor, exps: torch.Tensor, k: int = 40,
                 out: LmResult | None = None) -> LmResult:
    """BFP8 lm_head [vocab, hidden] with fused argmax and top-k; ``out`` (from
    lm_outputs) is written instead of fresh outputs."""
    h = _need(h, torch.float32, "h")
    mant = _need(mant, torch.int8, "mant")
    exps = _need(exps, torch.uint8, "exps")
    V, H = mant.shape
    if out is None:
        return LmResult(*T.lm_head_bfp8(h, mant, exps, k))
    r = _lm_check_out(out, h.device, min(k, V))
    check(load().qwen_b200_lm_head_bfp8_dev(_ptr(h), _ptr(mant), _ptr(exps), V, H, k, _ptr(r.argmax),
                                            _ptr(r.ids), _ptr(r.scores), _ptr(r.n), _stream()),
          "lm_head_bfp8")
    return r


def sample_topk(ids: torch.Tensor, scores: torch.Tensor, temperature: float, top_k: int, top_p: float,
                rng_state: torch.Tensor | None, n: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """sample_from_topk on the device (qwen_sampling.c:411-529) over a device
    candidate list, e.g. ``r = lm_head_bfp8(...); sample_topk(r.ids, r.scores,
    T, top_k, top_p, state, n=r.n)``.  ``rng_state`` is an int32 [1] device
    tensor holding the xorshift32 state, updated in place (None: the first
    id).  Returns the chosen id as an int32 [1] device tensor (no sync)."""
    ids = _need(ids, torch.int32, "ids")
    scores = _need(scores, torch.float32, "scores")
    if out is None and n is not None and rng_state is not None and rng_state.is_contiguous():
        return T.sample_topk(ids, scores, _need(n, torch.int32, "n"), float(temperature), int(top_k), float(top_p),
                             _need(rng_state, torch.int32, "rng_state"))
    if out is None:
        out = torch.empty(1, dtype=torch.int32, device=ids.device)
    for t, name in ((rng_state, "rng_state"), (out, "out")):
        # updated in place: a contiguous copy would take the update instead
        if t is not None and not t.is_contiguous():
            raise ValueError(f"sample_topk: {name} must be contiguous")
    st = None if rng_state is None else _ptr(_need(rng_state, torch.int32, "rng_state"))
    _need(out, torch.int32, "out")
    nd = None if n is None else _ptr(_need(n, torch.int32, "n"))
    check(load().qwen_b200_sample_topk_dev(_ptr(ids), _ptr(scores), nd, ids.numel(), float(temperature),
                                           int(top_k), float(top_p), st, _ptr(out), _stream()), "sample_topk")
    return out


def pack_bfp8(w: torch.Tensor, out_mant: torch.Tensor | None = None, out_exps: torch.Tensor | None = None):
    """Pack fp32 [M, K] weights into (mant int8 [M, K], exps uint8 [M, K/64]) on the device."""
    w = _need(w, torch.float32, "w")
    M, K = w.shape
    if out_mant is None and out_exps is None:
        return T.pack_bfp8(w)
    mant = out_mant if out_mant is not None else torch.empty((M, K), dtype=torch.int8, device=w.device)
    exps = out_exps if out_exps is not None else torch.empty((M, K // 64), dtype=torch.uint8, device=w.device)
    rc = load().qwen_b200_pack_bfp8_dev(_ptr(w), M, K, _ptr(mant), _ptr(exps), _stream())
    check(rc, "pack_bfp8")
    return mant, exps


# Plan flags of the grouped launches (include/qwen_b200.h QB_STACK_*).
STACK_FAST = 1          # split-K arithmetic (fused multiply-add per block)
STACK_FIXED_SPLIT = 2   # with STACK_FAST: K cut at fixed 2 KB steps (same bits on any number of GPUs)
STACK_Q_INPUT = 4       # x is a quantized record: int16 xq [K], then fp32 xs [K/64]


class LinearStack:
    """A reusable grouped launch of independent BFP8 GEMVs (one kernel).

    ``items`` is a list of (x fp32 [K], mant int8 [M, K], exps uint8 [M, K/64],
    y fp32 [M]) device tensors; the tensors must stay alive and in place while
    the stack is used.  ``run()`` enqueues every GEMV on the current stream and
    is safe inside CUDA graph capture.  ``flags`` (STACK_*) overrides ``fast``;
    with STACK_Q_INPUT every x is a quantized record (``quant_record``).
    """

    def __init__(self, items, fast: bool = False, flags: int | None = None):
        n = len(items)
        P = ctypes.c_void_p * n
        I = ctypes.c_int * n
        self._keep = items
        mant = P(*[_ptr(m) for (_, m, _, _) in items])
        exps = P(*[_ptr(e) for (_, _, e, _) in items])
        xs = P(*[_ptr(x) for (x, _, _, _) in items])
        ys = P(*[_ptr(y) for (_, _, _, y) in items])
        Ms = I(*[m.shape[0] for (_, m, _, _) in items])
        Ks = I(*[m.shape[1] for (_, m, _, _) in items])
        fl = flags if flags is not None else (STACK_FAST if fast else 0)
        h = load().qwen_b200_stack_create_ex(n, mant, exps, xs, ys, Ms, Ks, fl)
        if h <= 0:
            check(h, "LinearStack")
        self.handle = h

    def run(self, stream: int | None = None) -> None:
        check(load().qwen_b200_stack_run(self.handle, _stream() if stream is None else stream), "LinearStack.run")

    def run_wait(self, wait_flags: int, wait_epoch: int, world: int, stream: int | None = None) -> None:
        """run() whose input quantizer first waits (bounded) until every one
        of `world` ranks published ``wait_epoch`` into the flag array at
        ``wait_flags`` (row-sharded layers whose input other GPUs write)."""
        check(load().qwen_b200_stack_run_sync(self.handle, _stream() if stream is None else stream, wait_flags,
                                              wait_epoch, None, 0, world, 0), "LinearStack.run_wait")

    def close(self) -> None:
        if getattr(self, "handle", 0) > 0:
            load().qwen_b200_stack_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _DevArray:
    """A raw device range seen as a 1-D tensor (no ownership)."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


class PeerRegion:
    """Zeroed device memory shared with the other processes of one node over
    CUDA IPC: ``handle()`` gives 64 bytes to send to them, ``PeerRegion.open``
    maps another process's region into this one.  Tensors made by ``floats``
    and ``uints`` alias the memory and must not outlive ``close()``."""

    def __init__(self, nbytes: int = 0, _ptr: int = 0, _owned: bool = True):
        if _ptr:
            self.ptr = _ptr
        else:
            p = ctypes.c_void_p()
            check(load().qwen_b200_dev_alloc(max(nbytes, 256), ctypes.byref(p)), "PeerRegion")
            self.ptr = p.value
        self.nbytes = nbytes
        self._owned = _owned

    def handle(self) -> bytes:
        buf = ctypes.create_string_buffer(64)
        check(load().qwen_b200_ipc_handle(self.ptr, buf), "PeerRegion.handle")
        return buf.raw

    @classmethod
    def open(cls, handle: bytes, nbytes: int) -> "PeerRegion":
        p = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(handle), 64)
        check(load().qwen_b200_ipc_open(buf, ctypes.byref(p)), "PeerRegion.open")
        return cls(nbytes, _ptr=p.value, _owned=False)

    def floats(self, offset: int, n: int) -> torch.Tensor:
        return torch.as_tensor(_DevArray(self.ptr + offset, n, "<f4"))

    def uints(self, offset: int, n: int) -> torch.Tensor:
        return torch.as_tensor(_DevArray(self.ptr + offset, n, "<i4"))

    def bytes(self, offset: int, n: int) -> torch.Tensor:
        return torch.as_tensor(_DevArray(self.ptr + offset, n, "|u1"))

    def close(self) -> None:
        if self.ptr:
            if self._owned:
                load().qwen_b200_dev_free(self.ptr)
            else:
                load().qwen_b200_ipc_close(self.ptr)
            self.ptr = 0


class ShardedLinearStack:
    """A grouped launch of the row slices one rank owns of several GEMVs,
    storing every finished row into this rank's full output vector AND into
    the other ranks' (mapped) full vectors, then raising the ranks'
    completion flags.

    ``items``: (x fp32 [K], mant int8 [m, K], exps uint8 [m, K/64], y fp32 [m])
    where y is this rank's row range [r0, r0 + m) of its full vector;
    ``peer_ptrs[i]``: device addresses of GEMV i's full vector on every other
    rank (world - 1 of them); ``row_base[i]`` = r0.  ``run(wait, sig, ...)``
    waits for epoch ``wait`` on this rank's flags (0: no wait) and publishes
    epoch ``sig`` into every rank's flags.  Absolute epochs are baked into
    the launch; for a captured graph make them offsets from a device counter
    (``sync_epoch_base`` / ``sync_epoch_advance``).
    """

    def __init__(self, items, peer_ptrs, row_base, world: int, fast: bool = False, flags: int | None = None):
        n = len(items)
        P = ctypes.c_void_p * n
        I = ctypes.c_int * n
        self._keep = items
        self.world = world
        mant = P(*[_ptr(m) for (_, m, _, _) in items])
        exps = P(*[_ptr(e) for (_, _, e, _) in items])
        xs = P(*[_ptr(x) for (x, _, _, _) in items])
        ys = P(*[_ptr(y) for (_, _, _, y) in items])
        Ms = I(*[m.shape[0] for (_, m, _, _) in items])
        Ks = I(*[m.shape[1] for (_, m, _, _) in items])
        flat = [p for ps in peer_ptrs for p in ps]
        if len(flat) != n * (world - 1):
            raise ValueError("ShardedLinearStack: need world - 1 peer vectors per GEMV")
        peers = (ctypes.c_void_p * max(1, len(flat)))(*flat)
        rb = I(*row_base)
        fl = flags if flags is not None else (STACK_FAST if fast else 0)
        h = load().qwen_b200_stack_create_sharded(n, mant, exps, xs, ys, Ms, Ks, fl, world, peers, rb)
        if h <= 0:
            check(h, "ShardedLinearStack")
        self.handle = h

    def run(self, wait_flags: int, wait_epoch: int, sig_flags, sig_epoch: int, rank: int,
            stream: int | None = None) -> None:
        sf = (ctypes.c_void_p * self.world)(*sig_flags)
        check(load().qwen_b200_stack_run_sync(self.handle, _stream() if stream is None else stream, wait_flags,
                                              wait_epoch, sf, sig_epoch, self.world, rank),
              "ShardedLinearStack.run")

    def close(self) -> None:
        if getattr(self, "handle", 0) > 0:
            load().qwen_b200_stack_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def quant_record_bytes(K: int) -> int:
    """Bytes of a quantized activation record: int16 xq [K], fp32 xs [K/64]."""
    return 2 * K + 4 * (K // 64)


def planes_record_bytes(B: int, K: int, ldxs: int) -> int:
    """Bytes of a planar record: int8 planes [2, B, K], then fp32 xs_t [K/64, ldxs]."""
    return 2 * B * K + 4 * (K // 64) * ldxs


def planes_view(buf: torch.Tensor, B: int, K: int, ldxs: int) -> Planes:
    """The Planes stored in a planar record (a uint8 or int8 device tensor)."""
    b = buf.view(torch.int8)
    return Planes(b[:2 * B * K].view(2, B, K), b[2 * B * K:planes_record_bytes(B, K, ldxs)].view(torch.float32)
                  .view(K // 64, ldxs), B, K)


def swiglu_quant_sharded(gate_ptr: int, up_ptr: int, B: int, n: int, ld_in: int, col0: int, K: int, planar: bool,
                         ldxs: int, dst_ptrs, sig_flags=None, sig_ticket: int = 0, sig_epoch: int = 0,
                         wait_flags: int = 0, world: int = 1, rank: int = 0) -> None:
    """The shard-local MLP activation of a row-sharded layer
    (qwen_b200_swiglu_quant_sharded_dev): elements [col0, col0 + n) of every
    batch row of gate / up -> swiglu -> block-64 quantization -> each
    destination record (a quantized record, or a planar record when
    ``planar``).  With ``sig_epoch`` the last CTA publishes the epoch and
    waits for every rank's."""
    dst = (ctypes.c_void_p * len(dst_ptrs))(*dst_ptrs)
    sf = (ctypes.c_void_p * world)(*sig_flags) if sig_flags else None
    check(load().qwen_b200_swiglu_quant_sharded_dev(gate_ptr, up_ptr, B, n, ld_in, col0, K, 1 if planar else 0, ldxs,
                                                    dst, len(dst_ptrs), sf, sig_ticket, sig_epoch, wait_flags, world,
                                                    rank, _stream()), "swiglu_quant_sharded")


def sync_epoch_base(base_ptr: int | None) -> None:
    """Make the epochs of this device's row-sharded launches offsets from the
    device uint32 at ``base_ptr`` (None: absolute epochs again); the
    launches enqueued from now on read the counter when they run, so a CUDA
    graph of a step replays with fresh epochs (qwen_b200_sync_epoch_base)."""
    check(load().qwen_b200_sync_epoch_base(base_ptr or None), "sync_epoch_base")


def sync_epoch_advance(base_ptr: int, n: int) -> None:
    """Enqueue counter += n on the current stream (the end of a step whose
    launches used epoch offsets 1..n)."""
    check(load().qwen_b200_sync_epoch_advance(base_ptr, n & 0xFFFFFFFF, _stream()), "sync_epoch_advance")


def quant_planes_wait(x: torch.Tensor, out: Planes, wait_flags: int, wait_epoch: int, world: int) -> Planes:
    """quant_planes() that first waits (bounded) until every rank published
    ``wait_epoch`` into this GPU's flag array at ``wait_flags``."""
    x = _need(x, torch.float32, "x")
    B, K = x.shape
    check(load().qwen_b200_quant_planes_wait_dev(_ptr(x), B, K, _ptr(out.planes), _ptr(out.xs_t), out.ldxs,
                                                 wait_flags, wait_epoch, world, _stream()), "quant_planes_wait")
    return out


class ShardedBatchedStack:
    """A grouped tcgen05 launch over the row slices one rank owns of several
    batched GEMMs.  ``items``: (Planes, mant int8 [m, K], exps, y) where ``y``
    is the device address of this rank's first column inside its full
    [B][ldy] output; ``ldy[i]`` the full row length; ``peer_ptrs[i]`` the
    full outputs of GEMM i on the other ranks (world - 1, may be empty for
    world 1); ``row_base[i]`` this rank's first row.  ``run(sig_flags,
    sig_epoch, rank)`` publishes the epoch when every row reached every GPU."""

    def __init__(self, items, ldy, peer_ptrs, row_base, world: int):
        n = len(items)
        P = ctypes.c_void_p * n
        I = ctypes.c_int * n
        self._keep = items
        self.world = world
        B = items[0][0].B
        ldxs = items[0][0].ldxs
        flat = [p for ps in peer_ptrs for p in ps]
        if len(flat) != n * (world - 1):
            raise ValueError("ShardedBatchedStack: need world - 1 peer outputs per GEMM")
        peers = (ctypes.c_void_p * max(1, len(flat)))(*flat) if flat else None
        h = load().qwen_b200_tc_stack_create_sharded(
            n, P(*[_ptr(m) for (_, m, _, _) in items]), P(*[_ptr(e) for (_, _, e, _) in items]),
            P(*[_ptr(p.planes) for (p, _, _, _) in items]), P(*[_ptr(p.xs_t) for (p, _, _, _) in items]),
            P(*[int(y) for (_, _, _, y) in items]), I(*[m.shape[0] for (_, m, _, _) in items]),
            I(*[m.shape[1] for (_, m, _, _) in items]), I(*ldy), B, ldxs, world, peers, I(*row_base))
        if h <= 0:
            check(h, "ShardedBatchedStack")
        self.handle = h

    def run(self, sig_flags=None, sig_epoch: int = 0, rank: int = 0, stream: int | None = None) -> None:
        sf = (ctypes.c_void_p * self.world)(*sig_flags) if sig_flags else None
        check(load().qwen_b200_tc_stack_run_sync(self.handle, _stream() if stream is None else stream, sf, sig_epoch,
                                                 self.world, rank), "ShardedBatchedStack.run")

    def close(self) -> None:
        if getattr(self, "handle", 0) > 0:
            load().qwen_b200_tc_stack_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
