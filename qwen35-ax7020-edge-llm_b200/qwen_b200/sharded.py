"""Output-row-sharded BFP8 linear stack over several GPUs (one process per GPU).

Every GEMV's rows are split into contiguous slices, one per rank, with slice
boundaries on multiples of 64 rows.  Each rank streams only its slice of the
weights (rows bit-identical to an unsharded run of the same arithmetic) and
the full output vector is rebuilt in every rank's own memory before the next
GEMV reads it, in one of two ways:

* ``exchange="nccl"``: an NCCL all-gather after every grouped launch;
* ``exchange="peer"``: the GEMV kernel itself stores each finished row into
  every rank's full vector over NVLink (CUDA IPC mappings), and the last CTA
  of each launch raises a per-rank epoch flag on every GPU; the next launch
  waits (bounded) for all ranks' flags before it reads its input.  No
  collective runs, and the weight stream of a launch starts while it waits.  The data flow of one
scaled MLP layer (gate / up ffn x hidden, down hidden x ffn): gate and up
read the layer input; down reads the gathered gate output (the element-wise
SwiGLU between them is glue outside this path); the next layer reads the
gathered down output.
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


def run_layers(layers, x0, gemv, all_gather, world, rank):
    """Reference data flow, independent of the device: `gemv(name, x_full,
    r0, r1) -> y_shard` computes rows [r0, r1) of a GEMV, `all_gather(y_shard,
    M) -> y_full` concatenates the rank slices.  Returns every gathered
    output in order (gate, up, down per layer)."""
    outs = []
    x = x0
    for L in layers:
        g0, g1 = shard_rows(L.gate.M, world, rank)
        u0, u1 = shard_rows(L.up.M, world, rank)
        d0, d1 = shard_rows(L.down.M, world, rank)
        gate = all_gather(gemv(L.gate.name, x, g0, g1), L.gate.M)
        up = all_gather(gemv(L.up.name, x, u0, u1), L.up.M)
        down = all_gather(gemv(L.down.name, gate, d0, d1), L.down.M)
        outs += [gate, up, down]
        x = down
    return outs


class ShardedDeviceStack:
    """This rank's weight slices of a scaled stack on its GPU, plus the
    full outputs, driven by grouped launches and the chosen exchange.

    ``batch`` 1 runs the batch-1 GEMV kernels (one activation vector per
    token); ``batch`` B > 1 runs B sequences per step through the tcgen05
    kernels (each layer input quantized to planar int16, outputs [B][M]).

    `fast` selects the split-K arithmetic (see ops.bfp8_gemv_fast), which
    keeps every GPU busy when each holds few rows.  Weights are fp32 N(0, 0.02) drawn per tensor from a seeded generator on
    the device (the same full matrix on every rank), packed, and sliced; only
    the slice is kept.  `copies` byte-identical copies of the slices rotate
    across steps so that timing never finds them in L2.
    """

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
        self.epoch = 0
        self.device = torch.device(device)
        self.shards = {}   # name -> (r0, r1)
        slices = []        # (name, r0, r1, K)
        for L in self.layers:
            for t in (L.gate, L.up, L.down):
                r0, r1 = shard_rows(t.M, world, rank)
                self.shards[t.name] = (r0, r1)
                slices.append((t, r0, r1))
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
        # gathered outputs (full [M] vectors or [B][M] matrices, every rank)
        # and this rank's slices
        if exchange == "peer":
            self._map_regions()
        else:
            self.full = {t.name: torch.zeros(self._oshape(t.M), dtype=torch.float32, device=self.device)
                         for L in self.layers for t in (L.gate, L.up, L.down)}
        self.part = {t.name: torch.zeros(B * self.padded_rows(t.M), dtype=torch.float32, device=self.device)
                     for L in self.layers for t in (L.gate, L.up, L.down)}
        self.gath = {t.name: torch.zeros(B * self.padded_rows(t.M) * world, dtype=torch.float32, device=self.device)
                     for L in self.layers for t in (L.gate, L.up, L.down)}
        if B > 1:   # planar int16 activations, one set per input width (local only)
            self.planes = {}
            for L in self.layers:
                for K in (L.gate.K, L.down.K):
                    if K not in self.planes:
                        self.planes[K] = ops.planes_empty(B, K, self.device)
        self.plans = [self._plans(c) for c in range(copies)]

    def _oshape(self, M):
        return (M,) if self.B == 1 else (self.B, M)

    FLAGS_BYTES = 256   # epoch flags at the head of every region: one uint per rank

    def _map_regions(self):
        """One IPC-shared region per rank: the epoch flags, then every GEMV's
        full output vector (256-byte aligned).  Handles are exchanged with an
        all_gather_object; the other ranks' regions are mapped here."""
        import torch.distributed as dist

        from . import ops

        for L in self.layers:
            for t in (L.gate, L.up, L.down):
                r0, r1 = self.shards[t.name]
                if r1 <= r0:
                    raise ValueError(f"exchange='peer' needs rows on every rank ({t.name}: M={t.M})")
        self.voff, off = {}, self.FLAGS_BYTES
        for L in self.layers:
            for t in (L.gate, L.up, L.down):
                self.voff[t.name] = off
                off += (4 * self.B * t.M + 255) // 256 * 256
        self.region = ops.PeerRegion(off)
        self.full = {name: self.region.floats(o, self.B * t.M).view(self._oshape(t.M)) for name, o, t in
                     ((t.name, self.voff[t.name], t) for L in self.layers for t in (L.gate, L.up, L.down))}
        self.flags = self.region.uints(0, self.world)
        self.peer_base = [0] * self.world   # every rank's region base, mapped into this process
        self.peer_base[self.rank] = self.region.ptr
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, self.region.handle(), group=self.group)
            for r in range(self.world):
                if r != self.rank:
                    reg = ops.PeerRegion.open(handles[r], off)
                    self.peer_regions.append(reg)
                    self.peer_base[r] = reg.ptr

    def padded_rows(self, M):
        """Every rank contributes the same count to the all-gather: the
        largest slice, rounded up to 64."""
        return max(r1 - r0 for r0, r1 in (shard_rows(M, self.world, r) for r in range(self.world)))

    def weight(self, copy, t):
        import torch

        r0, r1 = self.shards[t.name]
        rows = r1 - r0
        o = self.offs[t.name]
        buf = self.buffers[copy]
        mant = buf[o:o + rows * t.K].view(torch.int8).view(rows, t.K)
        exps = buf[o + rows * t.K:o + rows * t.K + rows * t.K // 64].view(rows, t.K // 64)
        return mant, exps

    def _plans(self, copy):
        """Per layer: one grouped launch for gate+up (same input), one for down."""
        from . import ops

        plans = []
        x = self.x0

        def out(t, rows):   # a single rank writes straight into the full vector
            if self.exchange == "peer":
                r0, r1 = self.shards[t.name]
                return self.full[t.name][r0:r1]
            return self.full[t.name] if self.world == 1 else self.part[t.name][:rows]

        if self.B > 1:
            return self._batched_plans(copy)
        if self.exchange == "peer":
            return self._peer_plans(copy)
        for L in self.layers:
            gu = []
            for t in (L.gate, L.up):
                mant, exps = self.weight(copy, t)
                r0, r1 = self.shards[t.name]
                if r1 > r0:
                    gu.append((x, mant, exps, out(t, r1 - r0)))
            mant, exps = self.weight(copy, L.down)
            r0, r1 = self.shards[L.down.name]
            dn = [(self.full[L.gate.name], mant, exps, out(L.down, r1 - r0))] if r1 > r0 else []
            plans.append((ops.LinearStack(gu, fast=self.fast) if gu else None,
                          ops.LinearStack(dn, fast=self.fast) if dn else None))
            x = self.full[L.down.name]
        return plans

    def _peer_plans(self, copy):
        from . import ops

        others = [r for r in range(self.world) if r != self.rank]
        plans = []
        x = self.x0

        def stack(ts, xin):
            items, peers, bases = [], [], []
            for t in ts:
                mant, exps = self.weight(copy, t)
                r0, r1 = self.shards[t.name]
                items.append((xin, mant, exps, self.full[t.name][r0:r1]))
                peers.append([self.peer_base[r] + self.voff[t.name] for r in others])
                bases.append(r0)
            return ops.ShardedLinearStack(items, peers, bases, self.world, fast=self.fast)

        for L in self.layers:
            plans.append((stack((L.gate, L.up), x), stack((L.down,), self.full[L.gate.name])))
            x = self.full[L.down.name]
        return plans

    def _batched_plans(self, copy):
        """Per layer one grouped tcgen05 launch for gate+up and one for down.
        Outputs go straight into the full [B][M] matrices (one rank, or
        exchange="peer", which also stores into every other rank's), or into
        this rank's contiguous [B][slice] part for the NCCL all-gather."""
        from . import ops

        others = [r for r in range(self.world) if r != self.rank]
        peer = self.exchange == "peer" and self.world > 1
        plans = []

        def stack(ts, planes):
            items, ldy, peers, bases = [], [], [], []
            for t in ts:
                mant, exps = self.weight(copy, t)
                r0, r1 = self.shards[t.name]
                if self.world == 1 or peer:
                    y = self.full[t.name].data_ptr() + 4 * r0
                    ldy.append(t.M)
                else:
                    y = self.part[t.name].data_ptr()
                    ldy.append(self.padded_rows(t.M))
                items.append((planes, mant, exps, y))
                peers.append([self.peer_base[r] + self.voff[t.name] for r in others] if peer else [])
                bases.append(r0 if peer else 0)
            return ops.ShardedBatchedStack(items, ldy, peers, bases, self.world if peer else 1)

        for L in self.layers:
            plans.append((stack((L.gate, L.up), self.planes[L.gate.K]), stack((L.down,), self.planes[L.down.K])))
        return plans

    def _step_batched(self, copy):
        from . import ops

        peer = self.exchange == "peer" and self.world > 1
        x = self.x0
        for L, (gu, dn) in zip(self.layers, self.plans[copy]):
            for plan, xin, outs, K in ((gu, x, (L.gate, L.up), L.gate.K),
                                       (dn, self.full[L.gate.name], (L.down,), L.down.K)):
                if peer:
                    wait = self.epoch & 0xFFFFFFFF
                    self.epoch += 1
                    ops.quant_planes_wait(xin, self.planes[K], self.peer_base[self.rank], wait, self.world)
                    plan.run(self.peer_base, self.epoch & 0xFFFFFFFF, self.rank)
                else:
                    ops.quant_planes(xin, self.planes[K])
                    plan.run()
                    if self.world > 1:
                        for t in outs:
                            self._gather(t)
            x = self.full[L.down.name]

    def _launch_peer(self, plan):
        """Launch n waits for every rank's launch n - 1 and publishes n (one
        rank: stream order is enough, no flags)."""
        if self.world == 1:
            plan.run(self.peer_base[0], 0, self.peer_base, 0, 0)
            return
        wait = self.epoch & 0xFFFFFFFF
        self.epoch += 1
        sig = self.epoch & 0xFFFFFFFF
        plan.run(self.peer_base[self.rank], wait, [b for b in self.peer_base], sig, self.rank)

    def _gather(self, t):
        import torch.distributed as dist

        part, gath, full = self.part[t.name], self.gath[t.name], self.full[t.name]
        if self.world == 1:
            return
        B = self.B
        if B == 1 and part.numel() * self.world == t.M:   # equal slices: gather straight into place
            dist.all_gather_into_tensor(full, part, group=self.group)
            return
        dist.all_gather_into_tensor(gath, part, group=self.group)
        P = part.numel() // B
        g = gath.view(self.world, B, P)
        f = full.view(B, t.M)
        for r in range(self.world):
            r0, r1 = shard_rows(t.M, self.world, r)
            if r1 > r0:
                f[:, r0:r1].copy_(g[r, :, :r1 - r0])

    def step(self, copy=0):
        """One token through every layer (grouped GEMV launches + gathers)."""
        if self.B > 1:
            self._step_batched(copy)
            return
        if self.exchange == "peer":
            for gu, dn in self.plans[copy]:
                self._launch_peer(gu)
                self._launch_peer(dn)
            return
        for L, (gu, dn) in zip(self.layers, self.plans[copy]):
            if gu is not None:
                gu.run()
            self._gather(L.gate)
            self._gather(L.up)
            if dn is not None:
                dn.run()
            self._gather(L.down)

    def bytes_per_step(self):
        """Algorithmic bytes of one token over ALL ranks: the full weights
        once, plus the fp32 activation in and output out of every GEMV."""
        tot = 0
        for L in self.layers:
            for t in (L.gate, L.up, L.down):
                if self.B == 1:
                    tot += t.M * t.K + t.M * t.K // 64 + 4 * t.K + 4 * t.M
                else:   # planar int16 activations + block scales in, fp32 out
                    tot += t.M * t.K + t.M * t.K // 64 + self.B * (2 * t.K + 4 * (t.K // 64) + 4 * t.M)
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
            self.flags = None
            self.region.close()
            self.region = None
