"""Linear-stack shapes of the served model and synthetic BFP8 weight stacks.

The per-token linear stack of Qwen3.5-0.8B as the reference engine runs it
(04-板载脚本与工具/qwen_real_engine.py:848-999, 1060-1166; shapes from
06-模型与权重/config.json and qwen35_weights_64k_manifest.json): 24 layers,
layers 3, 7, 11, 15, 19, 23 full attention (q+gate 4096x1024, k 512x1024,
v 512x1024, o 1024x2048), the other 18 Gated-DeltaNet (in_proj_qkv
6144x1024, in_proj_z 2048x1024, out_proj 1024x2048), every layer an MLP
(gate 3584x1024, up 3584x1024, down 1024x3584): 150 BFP8 tensors,
504,791,040 bytes.
"""
from __future__ import annotations

import json
from dataclasses import dataclass

HIDDEN = 1024
FFN = 3584
LAYERS = 24
FULL_ATTN = (3, 7, 11, 15, 19, 23)
VOCAB = 65536


@dataclass(frozen=True)
class Linear:
    name: str
    M: int
    K: int

    @property
    def mant_bytes(self) -> int:
        return self.M * self.K

    @property
    def exp_bytes(self) -> int:
        return self.M * self.K // 64

    @property
    def soa_bytes(self) -> int:
        e = self.exp_bytes
        return self.mant_bytes + e + ((-e) % 8)


def qwen35_08b_stack() -> list[Linear]:
    """The 150 BFP8 GEMVs of one token, in the order the engine issues them."""
    out = []
    for l in range(LAYERS):
        p = f"model.language_model.layers.{l}."
        if l in FULL_ATTN:
            out += [Linear(p + "self_attn.q_proj.weight", 4096, HIDDEN),
                    Linear(p + "self_attn.k_proj.weight", 512, HIDDEN),
                    Linear(p + "self_attn.v_proj.weight", 512, HIDDEN),
                    Linear(p + "self_attn.o_proj.weight", HIDDEN, 2048)]
        else:
            out += [Linear(p + "linear_attn.in_proj_qkv.weight", 6144, HIDDEN),
                    Linear(p + "linear_attn.in_proj_z.weight", 2048, HIDDEN),
                    Linear(p + "linear_attn.out_proj.weight", HIDDEN, 2048)]
        out += [Linear(p + "mlp.gate_proj.weight", FFN, HIDDEN),
                Linear(p + "mlp.up_proj.weight", FFN, HIDDEN),
                Linear(p + "mlp.down_proj.weight", HIDDEN, FFN)]
    return out


def scaled_stack(layers: int = 8, hidden: int = 8192, ffn: int = 28672) -> list[Linear]:
    """The multi-GPU configuration: `layers` x (gate, up ffn x hidden, down hidden x ffn)."""
    out = []
    for l in range(layers):
        p = f"layers.{l}.mlp."
        out += [Linear(p + "gate_proj", ffn, hidden), Linear(p + "up_proj", ffn, hidden),
                Linear(p + "down_proj", hidden, ffn)]
    return out


def stack_bytes(stack) -> dict:
    """Algorithmic bytes of one pass: weights (mantissas + exponents) and the
    fp32 activation in / output out of every GEMV."""
    w = sum(t.mant_bytes + t.exp_bytes for t in stack)
    io = sum(4 * t.K + 4 * t.M for t in stack)
    macs = sum(t.M * t.K for t in stack)
    return {"weights": w, "io": io, "total": w + io, "macs": macs}


def align64(n: int) -> int:
    return (n + 63) & ~63


def layout(stack) -> tuple[dict, int]:
    """Offsets of each tensor in one contiguous buffer, 64-byte aligned like the
    reference weight file (05-主机侧源码/export_qwen35_weights_bfp8_64k.py:31,64-80)."""
    off = 0
    table = {}
    for t in stack:
        off = align64(off)
        table[t.name] = (off, t)
        off += t.soa_bytes
    return table, align64(off)


def manifest_for(stack, model_name="synthetic") -> dict:
    """A manifest with the reference's keys for the BFP8 tensors of `stack`
    (06-模型与权重/qwen35_weights_64k_manifest.json)."""
    table, total = layout(stack)
    tensors = {}
    for name, (off, t) in table.items():
        tensors[name] = {
            "dtype": "bfp8_soa", "shape": [t.M, t.K], "type": "block64_bfp8",
            "mantissa_bytes": t.mant_bytes, "exponent_bytes": t.exp_bytes + ((-t.exp_bytes) % 8),
            "file_offset": off, "byte_size": t.soa_bytes,
        }
    return {"model_name": model_name, "tensors": tensors, "total_binary_bytes": total,
            "total_tensors": len(tensors)}


def read_manifest(path: str) -> dict:
    with open(path, encoding="utf-8") as f:
        return json.load(f)


def bfp8_tensors(manifest: dict) -> list[tuple[str, int, int, int]]:
    """(name, file_offset, M, K) of every BFP8 tensor of a reference manifest,
    sliced the way the engine does (qwen_real_engine.py:834-846)."""
    out = []
    for name, info in manifest["tensors"].items():
        if info.get("dtype") == "bfp8_soa":
            M, K = info["shape"]
            out.append((name, info["file_offset"], M, K))
    return out


def file_layout(entries) -> tuple[dict, int]:
    """File offsets of (name, byte_size) entries written in order with every
    tensor starting on a 64-byte boundary -- the reference exporter's rule
    (05-主机侧源码/export_qwen35_weights_bfp8_64k.py:31,64-80), which gives
    every file_offset of qwen35_weights_64k_manifest.json."""
    off, table = 0, {}
    for name, size in entries:
        off = align64(off)
        table[name] = off
        off += size
    return table, off


class WeightFile:
    """A BFP8 weight file and its manifest (the reference's
    qwen35_weights_64k.bin + qwen35_weights_64k_manifest.json), read the way
    the reference engine reads them: the file is mapped read-only
    (qwen_real_engine.py:741-756) -- or any host buffer holding its bytes is
    used -- and every BFP8 tensor is a zero-copy numpy view at its
    file_offset, mantissas int8 [M][K] then exponents uint8 [M][K/64]
    (:1188-1206, :834-846).  ``views`` pointers are what the engine passes to
    bfp8_gemv, so ``register()`` (the whole mapping, once) lets the drop-in
    C ABI find every tensor on the device; ``to_device`` uploads the tensors
    for the device API."""

    def __init__(self, manifest: dict, path: str | None = None, buffer=None):
        import mmap

        import numpy as np

        self.manifest = manifest
        if (path is None) == (buffer is None):
            raise ValueError("WeightFile: give a path or a buffer")
        self._f = self._mm = None
        if path is not None:
            self._f = open(path, "rb")
            self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
            self.buf = np.frombuffer(self._mm, dtype=np.uint8)
        else:
            self.buf = np.frombuffer(buffer, dtype=np.uint8)
        self.names = [n for n, _, _, _ in sorted(bfp8_tensors(manifest), key=lambda e: e[1])]
        for n in self.names:
            info = manifest["tensors"][n]
            if info["file_offset"] + info["byte_size"] > self.buf.nbytes:
                raise ValueError(f"WeightFile: {n} lies beyond the end of the file")

    def stack(self) -> list[Linear]:
        """The BFP8 tensors as GEMV shapes, in file order (the order the
        engine issues them in a token)."""
        return [Linear(n, *self.manifest["tensors"][n]["shape"]) for n in self.names]

    def views(self, name: str):
        """(mant int8 [M, K], exps uint8 [M, K/64]) zero-copy host views."""
        info = self.manifest["tensors"][name]
        M, K = info["shape"]
        off = info["file_offset"]
        mant = self.buf[off:off + M * K].view("int8").reshape(M, K)
        exps = self.buf[off + M * K:off + M * K + M * K // 64].reshape(M, K // 64)
        return mant, exps

    def register(self) -> None:
        """Upload the whole file once for the drop-in C ABI: later bfp8_gemv
        calls whose pointers fall inside it use the device copy."""
        from ._lib import check, load

        check(load().qwen_b200_register_weights(self.buf.ctypes.data, self.buf.nbytes), "WeightFile.register")

    def forget(self) -> None:
        from ._lib import load

        load().qwen_b200_forget_weights(self.buf.ctypes.data)

    def to_device(self, device="cuda", names=None) -> "DeviceWeights":
        return DeviceWeights(self, device, names)

    def close(self) -> None:
        self.buf = None
        if self._mm is not None:
            self._mm.close()
            self._f.close()
            self._mm = self._f = None


class DeviceWeights:
    """The BFP8 tensors of a WeightFile on one GPU: the file span from the
    first to the last of them copied in one transfer, so every tensor keeps
    its file_offset (relative to the span) and its SoA layout."""

    def __init__(self, wf: WeightFile, device="cuda", names=None):
        import torch

        self.names = list(names) if names is not None else list(wf.names)
        self.info = {n: wf.manifest["tensors"][n] for n in self.names}
        lo = min(i["file_offset"] for i in self.info.values())
        hi = max(i["file_offset"] + i["byte_size"] for i in self.info.values())
        self.base = lo
        self.buf = torch.from_numpy(wf.buf[lo:hi].copy()).to(device)

    def views(self, name: str):
        """(mant int8 [M, K], exps uint8 [M, K/64]) device views."""
        import torch

        info = self.info[name]
        M, K = info["shape"]
        o = info["file_offset"] - self.base
        mant = self.buf[o:o + M * K].view(torch.int8).view(M, K)
        exps = self.buf[o + M * K:o + M * K + M * K // 64].view(M, K // 64)
        return mant, exps


class DeviceStack:
    """One or more copies of a synthetic BFP8 stack resident on a CUDA device.

    Weights are fp32 N(0, std) drawn with a seeded torch generator on the
    device and packed by ``ops.pack_bfp8``; copy 0 is packed, further copies
    are byte-identical clones at distinct addresses (so a benchmark that
    rotates through them defeats the 126 MB L2).  Activations are fp32
    N(0, 1), one per GEMV, outputs one fp32 vector per GEMV.
    """

    def __init__(self, stack, copies=1, device="cuda", seed=0, std=0.02, host_bytes=None, host_x=None):
        import torch

        from . import ops

        self.stack = list(stack)
        self.table, self.nbytes = layout(self.stack)
        self.device = torch.device(device)
        if host_bytes is not None:
            # the packed weight file image (layout() offsets), e.g. an mmap
            if host_bytes.nbytes < self.nbytes:
                raise ValueError("host_bytes is shorter than the stack layout")
            base = torch.from_numpy(host_bytes[:self.nbytes]).to(self.device)
        else:
            g = torch.Generator(device=self.device)
            g.manual_seed(seed)
            base = torch.empty(self.nbytes, dtype=torch.uint8, device=self.device)
            for name, (off, t) in self.table.items():
                w = torch.randn((t.M, t.K), generator=g, device=self.device, dtype=torch.float32) * std
                mant = base[off:off + t.mant_bytes].view(torch.int8).view(t.M, t.K)
                exps = base[off + t.mant_bytes: off + t.mant_bytes + t.exp_bytes].view(t.M, t.K // 64)
                ops.pack_bfp8(w, mant, exps)
                del w
        self.buffers = [base] + [base.clone() for _ in range(copies - 1)]
        # activations and outputs live in two flat buffers (one copy each way
        # moves a whole token); each GEMV's slice starts on a 16-byte boundary
        xo, yo = [], []
        nx = ny = 0
        for t in self.stack:
            xo.append(nx)
            yo.append(ny)
            nx += (t.K + 3) & ~3
            ny += (t.M + 3) & ~3
        if host_x is not None:   # one fp32 activation per GEMV, concatenated in stack order
            xs = torch.zeros(nx, dtype=torch.float32)
            pos = 0
            for o, t in zip(xo, self.stack):
                xs[o:o + t.K] = torch.from_numpy(host_x[pos:pos + t.K])
                pos += t.K
            self.x_flat = xs.to(self.device)
        else:
            gx = torch.Generator(device=self.device)
            gx.manual_seed(seed + 1)
            self.x_flat = torch.randn(nx, generator=gx, device=self.device, dtype=torch.float32)
        self.y_flat = torch.zeros(ny, dtype=torch.float32, device=self.device)
        self.x_off, self.y_off = xo, yo   # each GEMV's slice of x_flat / y_flat
        self.x = [self.x_flat[o:o + t.K] for o, t in zip(xo, self.stack)]
        self.y = [self.y_flat[o:o + t.M] for o, t in zip(yo, self.stack)]

    def views(self, copy=0, x_flat=None, y_flat=None):
        """[(x, mant, exps, y)] of one copy, in stack order; x_flat / y_flat
        (same sizes as this stack's) substitute other activation / output
        buffers."""
        import torch

        buf = self.buffers[copy]
        out = []
        for i, t in enumerate(self.stack):
            off, _ = self.table[t.name]
            mant = buf[off:off + t.mant_bytes].view(torch.int8).view(t.M, t.K)
            exps = buf[off + t.mant_bytes: off + t.mant_bytes + t.exp_bytes].view(t.M, t.K // 64)
            x = self.x[i] if x_flat is None else x_flat[self.x_off[i]:self.x_off[i] + t.K]
            y = self.y[i] if y_flat is None else y_flat[self.y_off[i]:self.y_off[i] + t.M]
            out.append((x, mant, exps, y))
        return out


def batched_bytes(stack, B: int) -> dict:
    """Algorithmic bytes and work of one batched step (B sequences through
    every GEMM): weights once, planar int16 activations (2 B per element)
    and their block scales in, fp32 outputs out."""
    w = sum(t.mant_bytes + t.exp_bytes for t in stack)
    io = sum(B * (2 * t.K + 4 * (t.K // 64) + 4 * t.M) for t in stack)
    macs = sum(t.M * t.K for t in stack)
    return {"weights": w, "io": io, "total": w + io, "macs": macs, "int_ops": 2 * macs * B,
            "tensor_ops": 4 * macs * B}


class DeviceBatch:
    """Activations of B sequences for every GEMM of a stack, as planar int16
    (ops.Planes), plus the outputs, in three flat device buffers per set (so a
    step's inputs or outputs move in one copy).  Each set holds fresh fp32
    N(0, 1) rows quantized on the device; benchmarks pair set c with weight
    copy c."""

    def __init__(self, stack, B, sets=1, device="cuda", seed=0):
        import torch

        from . import ops

        self.stack = list(stack)
        self.B = B
        self.device = torch.device(device)
        ldxs = (B + 3) // 4 * 4
        self.ldxs = ldxs
        po, so, yo = [], [], []
        npl = nsc = ny = 0
        for t in self.stack:
            po.append(npl)
            so.append(nsc)
            yo.append(ny)
            npl += 2 * B * t.K
            nsc += (t.K // 64) * ldxs
            ny += (B * t.M + 3) & ~3
        self.sets = []
        g = torch.Generator(device=self.device)
        for s in range(sets):
            g.manual_seed(seed * 1000 + s)
            planes = torch.empty(npl, dtype=torch.int8, device=self.device)
            scales = torch.zeros(nsc, dtype=torch.float32, device=self.device)
            ys = torch.zeros(ny, dtype=torch.float32, device=self.device)
            items = []
            for i, t in enumerate(self.stack):
                nb = t.K // 64
                p = ops.Planes(planes[po[i]:po[i] + 2 * B * t.K].view(2, B, t.K),
                               scales[so[i]:so[i] + nb * ldxs].view(nb, ldxs), B, t.K)
                x = torch.randn((B, t.K), generator=g, device=self.device, dtype=torch.float32)
                ops.quant_planes(x, out=p)
                items.append((p, ys[yo[i]:yo[i] + B * t.M].view(B, t.M)))
            self.sets.append({"planes": planes, "scales": scales, "y": ys, "items": items})

    def items(self, weights, s=0):
        """[(Planes, mant, exps, y)] for ops.BatchedStack: set s against the
        (x, mant, exps, y) views of a DeviceStack copy."""
        return [(p, m, e, y) for (p, y), (_, m, e, _) in zip(self.sets[s]["items"], weights)]
