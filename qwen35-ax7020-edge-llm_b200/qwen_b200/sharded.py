"""Output-row-sharded BFP8 MLP stack over several GPUs (one process per GPU).

The multi-GPU configuration is `layers` x (gate, up: ffn x hidden; down:
hidden x ffn).  Every GEMV's rows are split into contiguous slices, one per
rank, with slice boundaries on multiples of 64 rows, and gate and up share
their boundaries.  Per layer, on every rank:

1. gate / up: this rank's rows of both, from the full layer input; the
   results stay on this GPU;
2. the MLP activation of those rows, shard-locally: swiglu (the reference's
   NEON build) and the block-64 quantizer -- slices are whole blocks, so the
   bits are the unsharded activation's -- and only the quantized slice (int16
   values + block scales, 2.06 bytes per element) is exchanged, once;
3. down: this rank's rows, from the complete quantized activation; its fp32
   rows reach every rank (the next layer's input -- in a real decoder the
   residual stream, which stays fp32).

Two exchanges:

* ``exchange="nccl"``: NCCL all-gathers of the quantized activation and of
  the down rows;
* ``exchange="peer"``: the kernels store into every rank's buffers over
  NVLink (CUDA IPC mappings of one region per rank): the activation kernel
  stores the quantized slice, publishes an epoch flag to every rank and
  waits (bounded) for everyone's; the down GEMV stores its rows into every
  rank's output and publishes the next epoch, which the next layer's input
  quantizer waits for.  No collective runs.  Epochs are offsets from a
  per-rank device counter that the step's last launch advances, so one step
  can be captured in a CUDA graph and replayed (``capture``).

Batch 1 runs the GEMV kernels, batch > 1 the tcgen05 GEMM (planar int16
activations).  With ``fast`` (batch 1) every row's K is cut into segments at
fixed 2 KB steps, so the outputs are the same bits on any number of GPUs.
"""
from __future__ import annotations

from dataclasses import dataclass

from . import model


def shard_rows(M: int, world: int, rank: int, align: int = 64) -> tuple[int, int]:
    """Rows [r0, r1) of an M-row matrix owned by `rank`: contiguous slices
    whose boundaries are multiples of `align` (the last rank takes the rest)."""
    blocks = (M + align - 1) // align
    b0 = blocks * rank // world
    b1 = blocks * (rank + 1) // world
    return min(M, b0 * align), min(M, b1 * align)


@dataclass(frozen=True)
class LayerPlan:
    """The three GEMVs of one scaled MLP layer."""
    gate: model.Linear
    up: model.Linear
    down: model.Linear


def scaled_layers(layers=8, hidden=8192, ffn=28672) -> list[LayerPlan]:
    s = model.scaled_stack(layers, hidden, ffn)
    return [LayerPlan(s[3 * i], s[3 * i + 1], s[3 * i + 2]) for i in range(layers)]


def run_layers(layers, x0, gemv, act_quant, gemv_q, all_gather, world, rank):
    """The data flow, independent of the device: ``gemv(name, x, r0, r1)``
    computes rows [r0, r1) of a GEMV from an fp32 input, ``act_quant(g, u)``
    the quantized swiglu (xq, xs) of a slice, ``gemv_q(name, xq, xs, r0, r1)``
    rows of a GEMV from a quantized input, ``all_gather(part)`` concatenates
    the ranks' parts.  Returns, per layer, the gathered activation (xq, xs)
    and the gathered down output."""
    outs = []
    x = x0
    for L in layers:
        g0, g1 = shard_rows(L.gate.M, world, rank)
        d0, d1 = shard_rows(L.down.M, world, rank)
        xq_s, xs_s = act_quant(gemv(L.gate.name, x, g0, g1), gemv(L.up.name, x, g0, g1))
        xq, xs = all_gather(xq_s), all_gather(xs_s)
        down = all_gather(gemv_q(L.down.name, xq, xs, d0, d1))
        outs += [xq, xs, down]
        x = down
    return outs


class ShardedDeviceStack:
    """This rank's weight slices of a scaled stack on its GPU, its buffers,
    and the launches of one step (one token, or ``batch`` sequences).

    Weights are fp32 N(0, 0.02) drawn per tensor from a seeded generator on
    the device (the same full matrix on every rank), packed, and sliced; only
    the slice is kept.  `copies` byte-identical copies of the slices rotate
    across steps so that timing never finds them in L2.
    """

    FLAGS_BYTES = 256   # region head: epoch flags (one uint per rank), the activation kernel's ticket,
    TICKET_OFFSET = 128   # and this rank's epoch counter
    COUNTER_OFFSET = 192

    def __init__(self, layers, world, rank, device, copies=1, seed=0, group=None, fast=False, exchange="nccl",
                 batch=1):
        import torch

        from . import ops

        if exchange not in ("nccl", "peer"):
            raise ValueError("exchange must be 'nccl' or 'peer'")
        if batch < 1:
            raise ValueError("batch must be >= 1")
        self.B = batch
        self.layers = list(layers)
        self.world, self.rank, self.group = world, rank, group
        self.fast = fast
        self.exchange = exchange
        self.region, self.peer_regions = None, []
        self.device = torch.device(device)
        self.ldxs = (batch + 3) // 4 * 4
        for L in self.layers:
            if L.gate.M != L.up.M or L.gate.K != L.up.K or L.down.K != L.gate.M:
                raise ValueError("a layer needs gate and up of one shape and down reading their activation")
        self.shards = {}   # name -> (r0, r1)
        slices = []        # (Linear, r0, r1)
        for L in self.layers:
            for t in (L.gate, L.up, L.down):
                r0, r1 = shard_rows(t.M, world, rank)
                self.shards[t.name] = (r0, r1)
                slices.append((t, r0, r1))
        if exchange == "peer" and world > 1 and any(r1 <= r0 for _, r0, r1 in slices):
            raise ValueError("exchange='peer' needs rows on every rank")
        # one buffer per copy holding every slice (SoA, 64-byte aligned)
        offs, off = {}, 0
        for t, r0, r1 in slices:
            off = model.align64(off)
            rows = r1 - r0
            offs[t.name] = off
            off += rows * t.K + model.align64(rows * t.K // 64)
        self.nbytes = model.align64(off)
        base = torch.empty(max(self.nbytes, 64), dtype=torch.uint8, device=self.device)
        g = torch.Generator(device=self.device)
        for i, (t, r0, r1) in enumerate(slices):
            g.manual_seed(seed * 1000 + i)
            w = torch.randn((t.M, t.K), generator=g, device=self.device, dtype=torch.float32) * 0.02
            mant, exps = ops.pack_bfp8(w)
            del w
            rows = r1 - r0
            o = offs[t.name]
            base[o:o + rows * t.K].view(torch.int8).view(rows, t.K).copy_(mant[r0:r1])
            base[o + rows * t.K:o + rows * t.K + rows * t.K // 64].view(rows, t.K // 64).copy_(exps[r0:r1])
            del mant, exps
        self.offs = offs
        self.buffers = [base] + [base.clone() for _ in range(copies - 1)]
        gx = torch.Generator(device=self.device)
        gx.manual_seed(seed + 7)
        L0 = self.layers[0]
        B = self.B
        xshape = (L0.gate.K,) if B == 1 else (B, L0.gate.K)
        self.x0 = torch.randn(xshape, generator=gx, device=self.device, dtype=torch.float32)
        # gate / up outputs: full-length, only this rank's slice is written
        self.gu = {t.name: torch.zeros(self._oshape(t.M), dtype=torch.float32, device=self.device)
                   for L in self.layers for t in (L.gate, L.up)}
        # the down projections' quantized inputs (records) and full outputs:
        # in the shared region (peer) or local (nccl)
        if exchange == "peer":
            self._map_regions()
        else:
            self.dq = [torch.zeros(self._rec_bytes(L.down.K), dtype=torch.uint8, device=self.device)
                       for L in self.layers]
            self.full = {L.down.name: torch.zeros(self._oshape(L.down.M), dtype=torch.float32, device=self.device)
                         for L in self.layers}
        if B > 1:   # planar activations of the layer inputs (local)
            self.planes_in = ops.planes_empty(B, L0.gate.K, self.device)
        if exchange == "nccl" and world > 1:
            self._gather_buffers()
        self.plans = [self._plans(c) for c in range(copies)]

    # ------------------------------------------------------------ buffers
    def _oshape(self, M):
        return (M,) if self.B == 1 else (self.B, M)

    def _rec_bytes(self, K):
        from . import ops

        if self.B == 1:
            return ops.quant_record_bytes(K)
        return ops.planes_record_bytes(self.B, K, self.ldxs)

    def _map_regions(self):
        """One IPC-shared region per rank: the flags and ticket, then per
        layer the down projection's quantized input and its full output
        (256-byte aligned).  Handles are exchanged with an all_gather_object;
        the other ranks' regions are mapped here."""
        import torch.distributed as dist

        from . import ops

        self.qoff, self.voff, off = [], {}, self.FLAGS_BYTES
        for L in self.layers:
            self.qoff.append(off)
            off += (self._rec_bytes(L.down.K) + 255) // 256 * 256
            self.voff[L.down.name] = off
            off += (4 * self.B * L.down.M + 255) // 256 * 256
        self.region = ops.PeerRegion(off)
        self.dq = [self.region.bytes(o, self._rec_bytes(L.down.K)) for o, L in zip(self.qoff, self.layers)]
        self.full = {L.down.name: self.region.floats(self.voff[L.down.name], self.B * L.down.M)
                     .view(self._oshape(L.down.M)) for L in self.layers}
        self.flags = self.region.uints(0, self.world)
        self.counter = self.region.uints(self.COUNTER_OFFSET, 1)
        self.peer_base = [0] * self.world   # every rank's region base, mapped into this process
        self.peer_base[self.rank] = self.region.ptr
        if self.world > 1:
            # epoch 1 stands for "before the first step" (the first layer's
            # wait); set before the handle exchange, so before any peer signals
            import torch

            self.flags.fill_(1)
            torch.cuda.synchronize(self.device)
            handles = [None] * self.world
            dist.all_gather_object(handles, self.region.handle(), group=self.group)
            for r in range(self.world):
                if r != self.rank:
                    reg = ops.PeerRegion.open(handles[r], off)
                    self.peer_regions.append(reg)
                    self.peer_base[r] = reg.ptr

    def _equal(self, M):
        """Every rank holds the same number of rows of an M-row matrix."""
        return self.padded_rows(M) * self.world == M

    def padded_rows(self, M):
        """Every rank contributes the same count to an all-gather: the
        largest slice."""
        return max(r1 - r0 for r0, r1 in (shard_rows(M, self.world, r) for r in range(self.world)))

    def _gather_buffers(self):
        import torch

        B, W = self.B, self.world
        self.part, self.gath = {}, {}
        for L in self.layers:
            P = self.padded_rows(L.down.M)
            self.part[L.down.name] = torch.zeros(B * P, dtype=torch.float32, device=self.device)
            self.gath[L.down.name] = torch.zeros(W * B * P, dtype=torch.float32, device=self.device)
            Q = self.padded_rows(L.gate.M)
            if B == 1:   # xq (int16) and xs (fp32) slices of the quantized record
                self.part[("q", L.down.name)] = torch.zeros(Q, dtype=torch.int16, device=self.device)
                self.gath[("q", L.down.name)] = torch.zeros(W * Q, dtype=torch.int16, device=self.device)
            else:        # the planes' columns of every (plane, row)
                self.part[("q", L.down.name)] = torch.zeros(2 * B * Q, dtype=torch.int8, device=self.device)
                self.gath[("q", L.down.name)] = torch.zeros(W * 2 * B * Q, dtype=torch.int8, device=self.device)
            nbq = Q // 64
            self.part[("s", L.down.name)] = torch.zeros(nbq * (1 if B == 1 else self.ldxs), dtype=torch.float32,
                                                        device=self.device)
            self.gath[("s", L.down.name)] = torch.zeros(W * nbq * (1 if B == 1 else self.ldxs),
                                                        dtype=torch.float32, device=self.device)

    def weight(self, copy, t):
        import torch

        r0, r1 = self.shards[t.name]
        rows = r1 - r0
        o = self.offs[t.name]
        buf = self.buffers[copy]
        mant = buf[o:o + rows * t.K].view(torch.int8).view(rows, t.K)
        exps = buf[o + rows * t.K:o + rows * t.K + rows * t.K // 64].view(rows, t.K // 64)
        return mant, exps

    # ------------------------------------------------------------ plans
    def _flags(self):
        from . import ops

        return (ops.STACK_FAST | ops.STACK_FIXED_SPLIT) if self.fast else 0

    def _plans(self, copy):
        """Per layer: one grouped launch for gate + up (same input, local
        outputs) and one for down (quantized input; rows to every rank)."""
        if self.B > 1:
            return self._batched_plans(copy)
        from . import ops

        others = [r for r in range(self.world) if r != self.rank]
        peer = self.exchange == "peer" and self.world > 1
        plans = []
        x = self.x0
        for i, L in enumerate(self.layers):
            g0, g1 = self.shards[L.gate.name]
            items = [(x, *self.weight(copy, t), self.gu[t.name][g0:g1]) for t in (L.gate, L.up) if g1 > g0]
            gu = ops.LinearStack(items, flags=self._flags()) if items else None
            d0, d1 = self.shards[L.down.name]
            fl = self._flags() | ops.STACK_Q_INPUT
            if d1 <= d0:
                dn = None
            elif peer:
                dn = ops.ShardedLinearStack([(self.dq[i], *self.weight(copy, L.down), self.full[L.down.name][d0:d1])],
                                            [[self.peer_base[r] + self.voff[L.down.name] for r in others]], [d0],
                                            self.world, flags=fl)
            else:
                # one rank, or equal slices (gathered in place): straight into the full output
                direct = self.world == 1 or self._equal(L.down.M)
                y = self.full[L.down.name][d0:d1] if direct else self.part[L.down.name][:d1 - d0]
                dn = ops.LinearStack([(self.dq[i], *self.weight(copy, L.down), y)], flags=fl)
            plans.append((gu, dn))
            x = self.full[L.down.name]
        return plans

    def _batched_plans(self, copy):
        """Per layer one grouped tcgen05 launch for gate + up (strided into
        the local [B][M] outputs) and one for down (into the full [B][M]
        outputs of every rank, or this rank's contiguous part for NCCL)."""
        from . import ops

        others = [r for r in range(self.world) if r != self.rank]
        peer = self.exchange == "peer" and self.world > 1
        plans = []
        for i, L in enumerate(self.layers):
            g0, g1 = self.shards[L.gate.name]
            items, ldy = [], []
            for t in (L.gate, L.up):
                if g1 > g0:
                    items.append((self.planes_in, *self.weight(copy, t), self.gu[t.name].data_ptr() + 4 * g0))
                    ldy.append(t.M)
            gu = ops.ShardedBatchedStack(items, ldy, [[] for _ in items], [0] * len(items), 1) if items else None
            d0, d1 = self.shards[L.down.name]
            planes = ops.planes_view(self.dq[i], self.B, L.down.K, self.ldxs)
            if d1 <= d0:
                dn = None
            elif peer:
                dn = ops.ShardedBatchedStack([(planes, *self.weight(copy, L.down),
                                               self.full[L.down.name].data_ptr() + 4 * d0)], [L.down.M],
                                             [[self.peer_base[r] + self.voff[L.down.name] for r in others]], [d0],
                                             self.world)
            elif self.world == 1:
                dn = ops.ShardedBatchedStack([(planes, *self.weight(copy, L.down), self.full[L.down.name].data_ptr())],
                                             [L.down.M], [[]], [0], 1)
            else:
                dn = ops.ShardedBatchedStack([(planes, *self.weight(copy, L.down), self.part[L.down.name].data_ptr())],
                                             [self.padded_rows(L.down.M)], [[]], [0], 1)
            plans.append((gu, dn))
        return plans

    # ------------------------------------------------------------ one step
    def _activation(self, i, L, sig=0):
        """The shard-local swiglu + quantizer of layer i into this rank's
        down input (and, peer exchange, every other rank's), with an optional
        epoch signal + wait."""
        from . import ops

        g0, g1 = self.shards[L.gate.name]
        if g1 <= g0:
            return
        gp, up = self.gu[L.gate.name].data_ptr() + 4 * g0, self.gu[L.up.name].data_ptr() + 4 * g0
        dst = [self.dq[i].data_ptr()]
        if self.exchange == "peer" and self.world > 1:
            dst += [self.peer_base[r] + self.qoff[i] for r in range(self.world) if r != self.rank]
        if sig:
            ops.swiglu_quant_sharded(gp, up, self.B, g1 - g0, L.gate.M, g0, L.down.K, self.B > 1, self.ldxs, dst,
                                     sig_flags=self.peer_base, sig_ticket=self.peer_base[self.rank] + self.TICKET_OFFSET,
                                     sig_epoch=sig, wait_flags=self.peer_base[self.rank], world=self.world,
                                     rank=self.rank)
        else:
            ops.swiglu_quant_sharded(gp, up, self.B, g1 - g0, L.gate.M, g0, L.down.K, self.B > 1, self.ldxs, dst)

    def step(self, copy=0):
        """One token (or batch) through every layer.  Peer exchange: layer
        i waits for epoch 2i+1, its activation kernel publishes 2i+2 and its
        down projection 2i+3, all offsets from this rank's device counter,
        which the step's last launch advances by 2 * layers (so the next
        step's first wait is this step's last signal)."""
        from . import ops

        peer = self.exchange == "peer" and self.world > 1
        if peer:
            ops.sync_epoch_base(self.region.ptr + self.COUNTER_OFFSET)
        try:
            self._step(copy, peer)
            if peer:
                ops.sync_epoch_advance(self.region.ptr + self.COUNTER_OFFSET, 2 * len(self.layers))
        finally:
            if peer:
                ops.sync_epoch_base(None)

    def capturable(self):
        """Whether a step launches only this library's kernels (peer
        exchange, or one rank), so that it can be captured in a CUDA graph."""
        return self.exchange == "peer" or self.world == 1

    def capture(self, copy=0):
        """A CUDA graph of one step on weight copy `copy`.  Every plan must
        have run once (step) before; every rank captures the same steps, and
        nothing runs while capturing.  Replays advance the epoch counter as
        step() does, so replays and steps may follow one another in any
        order (the same on every rank)."""
        import torch

        if not self.capturable():
            raise ValueError("a step with NCCL all-gathers is not captured")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step(copy)
        return g

    def _step(self, copy, peer):
        from . import ops

        x = self.x0
        for i, (L, (gu, dn)) in enumerate(zip(self.layers, self.plans[copy])):
            wait = 2 * i + 1
            if self.B > 1:
                if peer:
                    ops.quant_planes_wait(x, self.planes_in, self.peer_base[self.rank], wait, self.world)
                else:
                    ops.quant_planes(x, self.planes_in)
                if gu is not None:
                    gu.run()
            elif gu is not None:
                if peer:
                    gu.run_wait(self.peer_base[self.rank], wait, self.world)
                else:
                    gu.run()
            if peer:
                self._activation(i, L, 2 * i + 2)
                sig = 2 * i + 3
                if dn is not None:
                    if self.B > 1:
                        dn.run(self.peer_base, sig, self.rank)
                    else:
                        dn.run(self.peer_base[self.rank], 0, self.peer_base, sig, self.rank)
            else:
                self._activation(i, L)
                if self.world > 1:
                    self._gather_activation(i, L)
                if dn is not None:
                    dn.run()
                if self.world > 1:
                    self._gather_down(L.down)
            x = self.full[L.down.name]

    # ------------------------------------------------------------ NCCL gathers
    def _gather_activation(self, i, L):
        import torch.distributed as dist

        B, W, K = self.B, self.world, L.down.K
        g0, g1 = self.shards[L.gate.name]
        Q = self.padded_rows(L.gate.M)
        nbq = Q // 64
        rec = self.dq[i]
        qp, qg = self.part[("q", L.down.name)], self.gath[("q", L.down.name)]
        sp, sg = self.part[("s", L.down.name)], self.gath[("s", L.down.name)]
        if B == 1 and self._equal(L.gate.M):
            # equal slices: gather the int16 values and the scales in place
            # (NCCL has no int16: they travel as their bytes)
            dist.all_gather_into_tensor(rec[:2 * K], rec[2 * g0:2 * g1], group=self.group)
            xs = rec[2 * K:2 * K + 4 * (K // 64)]
            dist.all_gather_into_tensor(xs, xs[4 * (g0 // 64):4 * (g1 // 64)], group=self.group)
            return
        if B == 1:
            xq = rec[:2 * K].view(self._i16()).view(K)
            xs = rec[2 * K:].view(self._f32()).view(K // 64)
            qp[:g1 - g0].copy_(xq[g0:g1])
            sp[:(g1 - g0) // 64].copy_(xs[g0 // 64:g1 // 64])
            # NCCL has no int16: the int16 slices travel as their bytes
            dist.all_gather_into_tensor(qg.view(self._u8()), qp.view(self._u8()), group=self.group)
            dist.all_gather_into_tensor(sg, sp, group=self.group)
            for r in range(W):
                r0, r1 = shard_rows(L.gate.M, W, r)
                if r1 > r0:
                    xq[r0:r1].copy_(qg[r * Q:r * Q + r1 - r0])
                    xs[r0 // 64:r1 // 64].copy_(sg[r * nbq:r * nbq + (r1 - r0) // 64])
            return
        planes = rec[:2 * B * K].view(self._i8()).view(2, B, K)
        xs_t = rec[2 * B * K:].view(self._f32()).view(K // 64, self.ldxs)
        qp.view(2, B, Q)[:, :, :g1 - g0].copy_(planes[:, :, g0:g1])
        sp.view(nbq, self.ldxs)[:(g1 - g0) // 64].copy_(xs_t[g0 // 64:g1 // 64])
        dist.all_gather_into_tensor(qg, qp, group=self.group)
        dist.all_gather_into_tensor(sg, sp, group=self.group)
        qv, sv = qg.view(W, 2, B, Q), sg.view(W, nbq, self.ldxs)
        for r in range(W):
            r0, r1 = shard_rows(L.gate.M, W, r)
            if r1 > r0:
                planes[:, :, r0:r1].copy_(qv[r, :, :, :r1 - r0])
                xs_t[r0 // 64:r1 // 64].copy_(sv[r, :(r1 - r0) // 64])

    def _gather_down(self, t):
        import torch.distributed as dist

        part, gath, full = self.part[t.name], self.gath[t.name], self.full[t.name]
        B = self.B
        P = part.numel() // B
        if B == 1 and P * self.world == t.M:   # equal slices: the GEMV wrote its rows in place
            d0, d1 = self.shards[t.name]
            dist.all_gather_into_tensor(full, full[d0:d1], group=self.group)
            return
        dist.all_gather_into_tensor(gath, part, group=self.group)
        g = gath.view(self.world, B, P)
        f = full.view(B, t.M)
        for r in range(self.world):
            r0, r1 = shard_rows(t.M, self.world, r)
            if r1 > r0:
                f[:, r0:r1].copy_(g[r, :, :r1 - r0])

    @staticmethod
    def _i16():
        import torch

        return torch.int16

    @staticmethod
    def _u8():
        import torch

        return torch.uint8

    @staticmethod
    def _i8():
        import torch

        return torch.int8

    @staticmethod
    def _f32():
        import torch

        return torch.float32

    # ------------------------------------------------------------ results
    def outputs(self):
        """Every layer's complete quantized activation (as bytes) and down
        output, concatenated as uint32 words (the values to compare across
        runs bit for bit)."""
        import numpy as np

        parts = []
        for i, L in enumerate(self.layers):
            rec = self.dq[i].cpu().numpy()
            parts.append(np.frombuffer(rec.tobytes() + b"\0" * ((-len(rec)) % 4), np.uint32))
            parts.append(self.full[L.down.name].cpu().numpy().ravel().view(np.uint32))
        return np.concatenate(parts)

    def final_output(self):
        """The last layer's down output (full, every rank)."""
        return self.full[self.layers[-1].down.name]

    def bytes_per_step(self):
        """Algorithmic bytes of one step over ALL ranks: the full weights
        once; gate / up read the fp32 (batch 1) or planar (batch > 1) layer
        input and write fp32; down reads the quantized activation and writes
        fp32."""
        from . import ops

        tot = 0
        B = self.B
        for L in self.layers:
            for t in (L.gate, L.up, L.down):
                tot += t.M * t.K + t.M * t.K // 64 + 4 * B * t.M
            if B == 1:
                tot += 2 * 4 * L.gate.K + ops.quant_record_bytes(L.down.K)
            else:
                tot += 2 * B * (2 * L.gate.K + 4 * (L.gate.K // 64)) + B * (2 * L.down.K + 4 * (L.down.K // 64))
        return tot

    def exchange_bytes_per_step(self):
        """Bytes one rank sends to the others per step: its slice of every
        quantized activation and of every down output, to each other rank."""
        tot = 0
        B = self.B
        for L in self.layers:
            g0, g1 = self.shards[L.gate.name]
            d0, d1 = self.shards[L.down.name]
            tot += (self.world - 1) * (B * (2 * (g1 - g0) + 4 * ((g1 - g0) // 64)) + 4 * B * (d1 - d0))
        return tot

    def device_error(self) -> int:
        """The kernels' error word (2: a peer flag wait timed out), cleared."""
        from ._lib import load

        return load().qwen_b200_device_error(1)

    def close(self):
        """Release plans and mappings.  In peer mode every rank must call it
        (it synchronises the device and barriers before freeing its region,
        which the others map)."""
        import torch
        import torch.distributed as dist

        for gu, dn in (p for plans in self.plans for p in plans):
            for s in (gu, dn):
                if s is not None:
                    s.close()
        if self.region is not None:
            torch.cuda.synchronize(self.device)
            for reg in self.peer_regions:
                reg.close()
            self.peer_regions = []
            if self.world > 1:
                dist.barrier(group=self.group)
            self.full = {}
            self.dq = []
            self.flags = None
            self.region.close()
            self.region = None
