#!/usr/bin/env python3
"""Benchmark of the BFP8 GEMV / lm_head decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload stack|gemv|lm_bf16|lm_bfp8|sharded|batched] [--batch B]

Default workload (the BASELINE metric's configuration): the full per-token
linear stack of Qwen3.5-0.8B at batch 1 -- 150 BFP8 GEMVs, 504,791,040 bytes
of weights, each GEMV on its own fp32 N(0,1) activation re-quantized inside
the kernel -- as ONE grouped kernel launch per token.  A step is one token.
Weights are random N(0, 0.02), packed on the device, and the timed steps
rotate through enough byte-identical copies (> 4 GB) that no step finds its
weights in the 126 MB L2.

One JSON line on rank 0.  `value` is algorithmic GB/s of the stack
(weights + fp32 activations in + fp32 outputs out, summed over ranks) with
everything resident in HBM; `e2e` is the same metric with every token's
activations copied in from pinned host memory and its outputs copied back
inside the timed region.  With --gpus N under torchrun every rank runs its
own token stream on its own GPU (independent decode replicas, weak scaling,
no collective on the data path).

--impl reference times the reference's own C bfp8_gemv (compiled from its
source for this host, scalar float path since the host has no NEON) on the
same workload with every host thread, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "qwen35-ax7020-edge-llm_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "BFP8 GEMV HBM GB/s (% of B200 peak); 0.8B-shape linear-stack ms/token, batch 1"
L2_DEFEAT_BYTES = 4.3e9


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["stack", "gemv", "lm_bf16", "lm_bfp8", "sharded", "batched", "rtl20"],
                    default="stack")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per step: --workload batched (default 256) or sharded (default 1)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="--workload sharded: rows stored into every GPU by the GEMV kernel, or NCCL all-gathers")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--copies", type=int, default=0,
                    help="weight copies to rotate (default: enough for > 4 GB; fewer only for profiling)")
    ap.add_argument("--cpu-sample", action="store_true", help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.batch is None:
        args.batch = 256 if args.workload == "batched" else 1
    return args


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def committed_traffic(kernel_key):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/traffic.json), or None."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            t = json.load(f)
        return t.get(kernel_key)
    except Exception:
        return None


# ------------------------------------------------------------------ workloads
def stack_shapes(workload):
    from qwen_b200 import model

    if workload == "stack":
        return model.qwen35_08b_stack(), "qwen35-0.8b linear stack (150 BFP8 GEMVs), batch 1"
    if workload == "gemv":
        return [model.Linear("mlp.up_proj", 3584, 1024)], "single BFP8 GEMV 3584x1024, batch 1"
    raise ValueError(workload)


class ClockSampler:
    """SM clock and throttle reasons of one GPU, polled through NVML from a
    thread every ~2 ms while the timed region runs (read-only queries)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, uuid, index):
        import threading

        self.samples, self.maxclk, self.err = [], None, None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            h = None
            want = (uuid or "").lower().replace("gpu-", "")
            for i in range(pynvml.nvmlDeviceGetCount()):
                hi = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(hi)
                u = (u.decode() if isinstance(u, bytes) else u).lower().replace("gpu-", "")
                if want and u == want:
                    h = hi
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.maxclk = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._nv, self._h = pynvml, h
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception as e:   # sampling must never break the benchmark
            self.err = str(e)[:120]
            self._t = None

    def _run(self):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                clk = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((clk, rs))
            except Exception:
                pass
            self._stop.wait(0.002)

    def stop(self):
        if self._t is None:
            return {"error": self.err}
        self._stop.set()
        self._t.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.maxclk, "reasons": [], "samples": 0}
        clks = [c for c, _ in self.samples]
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(clks), "sm_max_mhz": self.maxclk, "reasons": reasons,
                "samples": len(self.samples), "source": "nvml"}


def gpu_uuid(torch, dev):
    try:
        return str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        return None


def timed(torch, fn, steps, warmup, barrier):
    """Run warmup untimed steps, then time exactly `steps` steps with CUDA
    events on the current stream, barrier + synchronize on both sides."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(steps):
        fn(warmup + i)
    e.record()
    torch.cuda.synchronize()
    barrier()
    return s.elapsed_time(e) / 1e3


def run_b200(args):
    import torch
    import torch.distributed as dist

    from qwen_b200 import model, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    hbm_peak, peak_kind = peaks()
    line = {"metric": METRIC, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int16xint8->fp32",
            "data": "synthetic: weights N(0,0.02) packed BFP8 on device (seeded), activations N(0,1)"}

    if args.workload in ("stack", "gemv"):
        shapes, desc = stack_shapes(args.workload)
        nb = model.stack_bytes(shapes)
        wbytes = nb["weights"]
        copies = args.copies or max(2, math.ceil(L2_DEFEAT_BYTES / wbytes))
        ds = model.DeviceStack(shapes, copies=copies, device=dev, seed=1234 + rank)
        plans = [ops.LinearStack(ds.views(c)) for c in range(copies)]
        launches_per_step = 2   # act_prep + gemv_warp

        def step(i):
            plans[i % copies].run()

        # ------------------------------------------------ device-resident timing
        clk = ClockSampler(gpu_uuid(torch, dev), dev.index or 0)
        secs = timed(torch, step, args.steps, args.warmup, barrier)
        clocks = clk.stop()
        t = torch.tensor([secs], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        secs = float(t.item())
        per_step = secs / args.steps
        value = world * nb["total"] / per_step / 1e9
        kernel_gbs = nb["total"] / per_step / 1e9

        # ------------------------------------------------ end to end, host buffers
        e2e = None
        if not args.no_e2e:
            e2e = end_to_end(torch, dist, ds, plans, copies, nb, args, barrier, world, dev)
        line.update({
            "value": round(value, 2), "ms_per_step": round(per_step * 1e3, 4),
            "config": {"workload": desc, "gemvs_per_step": len(shapes), "weight_bytes": wbytes,
                       "algorithmic_bytes_per_step": nb["total"], "macs_per_step": nb["macs"],
                       "l2": f"rotates {copies} weight copies ({copies * wbytes / 1e9:.2f} GB) > 126 MB L2",
                       "launch": "act_prep + one grouped warp-autonomous kernel (PDL) per step", "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 2), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(kernel_gbs / hbm_peak, 4), "peak_kind": peak_kind,
                         "traffic": committed_traffic(args.workload),
                         "kernel": "gemv_warp_kernel (grouped)"},
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
        })
        for p in plans:
            p.close()
    elif args.workload == "sharded":
        line.update(run_sharded(args, torch, dist, dev, barrier, world, rank, local, hbm_peak, peak_kind))
    elif args.workload == "batched":
        line.update(run_batched(args, torch, dist, dev, barrier, world, rank, hbm_peak, peak_kind))
    elif args.workload == "rtl20":
        line.update(run_rtl20(args, torch, dev, barrier, world, hbm_peak, peak_kind))
    else:
        line.update(run_lm_head(args, torch, ops, dev, barrier, world, hbm_peak, peak_kind))

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload, args.batch)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def int8_peak_tops(torch, dev):
    """Dense int8 tensor throughput of this GPU, measured live: cuBLASLt
    through torch._int_mm on 8192^3 (2*N^3 ops), best of 10, CUDA events."""
    n = 8192
    a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device=dev).t()
    for _ in range(3):
        torch._int_mm(a, b)
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e) / 1e3)
    del a, b
    return 2 * n ** 3 / best / 1e12


def run_batched(args, torch, dist, dev, barrier, world, rank, hbm_peak, peak_kind):
    """B sequences x the 0.8B linear stack, one grouped
    tcgen05 kind::i8 launch per step (150 GEMMs).  Activations enter as
    planar int16 (hi/lo int8 planes + block scales, the quantizer's output);
    outputs leave as fp32 [B][M].  Weight copies and activation sets rotate
    together (> 4 GB), so no step finds its inputs in L2."""
    from qwen_b200 import model, ops

    B = args.batch
    shapes = model.qwen35_08b_stack()
    nb = model.batched_bytes(shapes, B)
    copies = args.copies or max(2, math.ceil(L2_DEFEAT_BYTES / nb["weights"]))
    ds = model.DeviceStack(shapes, copies=copies, device=dev, seed=1234 + rank)
    db = model.DeviceBatch(shapes, B, sets=copies, device=dev, seed=77 + rank)
    plans = [ops.BatchedStack(db.items(ds.views(c), c)) for c in range(copies)]
    p_int8 = int8_peak_tops(torch, dev)

    clk = ClockSampler(gpu_uuid(torch, dev), dev.index or 0)
    secs = timed(torch, lambda i: plans[i % copies].run(), args.steps, args.warmup, barrier)
    clocks = clk.stop()
    t = torch.tensor([secs], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    per_step = float(t.item()) / args.steps
    gbs = nb["total"] / per_step / 1e9
    tops = nb["tensor_ops"] / per_step / 1e12
    t_hbm = nb["total"] / (hbm_peak * 1e9)
    t_tc = nb["tensor_ops"] / (p_int8 * 1e12)
    if t_hbm >= t_tc:
        roof = {"bound": "hbm", "achieved": round(gbs, 2), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind}
    else:
        roof = {"bound": "tensor", "achieved": round(tops, 2), "peak": round(p_int8, 1), "unit": "TOPS (int8)",
                "frac": round(tops / p_int8, 4), "peak_kind": "measured live (cuBLASLt int8, torch._int_mm 8192^3)"}
    roof.update({"traffic": committed_traffic(f"batched_b{B}"), "kernel": "gemm_tc_kernel (grouped)",
                 "roofline_time_ms": round(max(t_hbm, t_tc) * 1e3, 4),
                 "frac_of_roofline_time": round(max(t_hbm, t_tc) / per_step, 4),
                 "hbm_frac": round(gbs / hbm_peak, 4), "tensor_frac": round(tops / p_int8, 4),
                 "int8_peak_tops": round(p_int8, 1)})

    e2e = None
    if not args.no_e2e:
        s0 = db.sets[0]
        hp = torch.empty(s0["planes"].numel(), dtype=torch.int8, pin_memory=True)
        hs = torch.empty(s0["scales"].numel(), dtype=torch.float32, pin_memory=True)
        hy = torch.empty(s0["y"].numel(), dtype=torch.float32, pin_memory=True)
        hp.copy_(s0["planes"].cpu())
        hs.copy_(s0["scales"].cpu())

        def e2e_step(i):
            st = db.sets[i % copies]
            st["planes"].copy_(hp, non_blocking=True)
            st["scales"].copy_(hs, non_blocking=True)
            plans[i % copies].run()
            hy.copy_(st["y"], non_blocking=True)

        esecs = timed(torch, e2e_step, args.steps, args.warmup, barrier)
        te = torch.tensor([esecs], device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        eper = float(te.item()) / args.steps
        e2e = {"value": round(world * nb["total"] / eper / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(eper * 1e3, 4), "tokens_per_s": round(world * B / eper, 1),
               "h2d_bytes_per_step": hp.numel() + hs.numel() * 4, "d2h_bytes_per_step": hy.numel() * 4}
    for p in plans:
        p.close()
    return {"value": round(world * gbs, 2), "ms_per_step": round(per_step * 1e3, 4), "dtype": "int8xint8->int32 (hi/lo planes)->fp32",
            "config": {"workload": f"batched decode: B={B} sequences x qwen35-0.8b linear stack (150 BFP8 GEMMs)",
                       "batch": B, "gemms_per_step": len(shapes), "weight_bytes": nb["weights"],
                       "algorithmic_bytes_per_step": nb["total"], "macs_per_step": nb["macs"] * B,
                       "tensor_int8_ops_per_step": nb["tensor_ops"], "tokens_per_s": round(world * B / per_step, 1),
                       "tops_issued_int8": round(tops, 2),
                       "l2": f"rotates {copies} weight copies + activation sets "
                             f"({copies * nb['weights'] / 1e9:.2f} GB weights) > 126 MB L2",
                       "launch": "one grouped tcgen05 kernel per step", "parallelism": f"replicas x{world}"},
            "roofline": roof, "e2e": e2e, "gpu_launches": args.steps, "clocks": clocks}


def run_sharded(args, torch, dist, dev, barrier, world, rank, local, hbm_peak, peak_kind):
    """8 layers x (gate, up 28672x8192; down 8192x28672),
    batch 1, output rows sharded over the ranks; the rows reach every GPU
    through the GEMV kernel's own peer stores (--exchange peer) or an NCCL
    all-gather after every projection.  Total work is fixed as N grows
    (strong scaling)."""
    from qwen_b200 import sharded

    layers = sharded.scaled_layers()
    full_w = sum(t.M * t.K + t.M * t.K // 64 for L in layers for t in (L.gate, L.up, L.down))
    copies = args.copies or max(1, math.ceil(L2_DEFEAT_BYTES / (full_w / world)))
    B = args.batch
    st = sharded.ShardedDeviceStack(layers, world, rank, dev, copies=copies, seed=11, fast=True,
                                    exchange=args.exchange, batch=B)
    clk = ClockSampler(gpu_uuid(torch, dev), local)
    secs = timed(torch, lambda i: st.step(i % copies), args.steps, args.warmup, barrier)
    clocks = clk.stop()
    t = torch.tensor([secs], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    per_step = float(t.item()) / args.steps
    nbytes = st.bytes_per_step()
    if args.exchange == "peer" and st.device_error():
        raise RuntimeError("sharded: a peer flag wait timed out")
    st.close()
    per_rank_gbs = nbytes / world / per_step / 1e9
    return {"value": round(nbytes / per_step / 1e9, 2), "ms_per_step": round(per_step * 1e3, 4), "scaling": "strong",
            "config": {"workload": f"scaled BFP8 stack: 8 x (gate/up 28672x8192, down 8192x28672), batch {B}",
                       "arithmetic": "fast (split-K, fma per block; within 1e-5 of the exact order)" if B == 1 else
                                     "tcgen05 kind::i8 over hi/lo int8 planes, exact int32 block dots",
                       "algorithmic_bytes_per_step": nbytes, "weight_bytes": full_w,
                       "parallelism": f"output rows sharded x{world}, " + (
                           "GEMV epilogue stores rows into every GPU over NVLink, epoch flags between launches"
                           if args.exchange == "peer" else "NCCL all-gather after each projection"),
                       "l2": f"rotates {copies} copies of this rank's {full_w / world / 1e9:.2f} GB"},
            "roofline": {"bound": "hbm", "achieved": round(per_rank_gbs, 2), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(per_rank_gbs / hbm_peak, 4), "peak_kind": peak_kind, "traffic": None,
                         "kernel": ("gemv_warp_kernel" if B == 1 else "gemm_tc_kernel") +
                                   " per rank (per-rank GB/s incl. the exchange)"},
            # 2 grouped launches per layer x (act_prep + gemv_warp, or quant_planes + gemm_tc); NCCL not counted
            "gpu_launches": args.steps * len(layers) * 4,
            "exchange": args.exchange,
            "clocks": clocks}


def end_to_end(torch, dist, ds, plans, copies, nb, args, barrier, world, dev):
    """The same token through the public API with host buffers: the step's
    activations copied in from pinned host memory, the stack run, its
    outputs copied back, all on the timed stream."""
    hx = torch.empty(ds.x_flat.numel(), dtype=torch.float32, pin_memory=True)
    hx.copy_(ds.x_flat.cpu())
    hy = torch.empty(ds.y_flat.numel(), dtype=torch.float32, pin_memory=True)

    def e2e_step(i):
        ds.x_flat.copy_(hx, non_blocking=True)
        plans[i % copies].run()
        hy.copy_(ds.y_flat, non_blocking=True)

    esecs = timed(torch, e2e_step, args.steps, args.warmup, barrier)
    te = torch.tensor([esecs], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    esecs = float(te.item())
    return {"value": round(world * nb["total"] / (esecs / args.steps) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(esecs / args.steps * 1e3, 4),
            "h2d_bytes_per_step": hx.numel() * 4, "d2h_bytes_per_step": hy.numel() * 4}


def graph_of(torch, fn, n):
    """CUDA graph of n calls fn(0..n-1) (warmed up on a side stream first)."""
    fn(0)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn(0)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n):
            fn(i)
    return g


def run_lm_head(args, torch, ops, dev, barrier, world, hbm_peak, peak_kind):
    """Secondary lines: the 65536 x 1024 lm_head (bf16 table or BFP8 matrix)
    fused with argmax and top-40.  `value` times the kernels alone: each
    step replays a CUDA graph of one call per table copy (no per-call host
    work); `e2e` calls the reference-facing host API (lm_head_topk with a
    host h and a registered host table for bf16; the BFP8 device call with
    h copied in and the ids and scores copied out otherwise)."""
    import ctypes

    import numpy as np

    from qwen_b200 import _lib

    V, H, k = 65536, 1024, 40
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    w = torch.randn((V, H), generator=g, device=dev) * 0.02
    h = torch.randn(H, generator=g, device=dev)
    if args.workload == "lm_bf16":
        tab = w.to(torch.bfloat16).view(torch.int16)
        per = V * H * 2
        copies = max(2, math.ceil(L2_DEFEAT_BYTES / per))
        tabs = [tab] + [tab.clone() for _ in range(copies - 1)]
        res = ops.lm_outputs(dev, k)   # preallocated: the timed graph holds only the lm_head kernels

        def call(i):
            ops.lm_head_bf16(h, tabs[i % copies], k, out=res)
        desc = "bf16 lm_head 65536x1024 + argmax + top-40"
    else:
        mant, exps = ops.pack_bfp8(w)
        per = V * H + V * H // 64
        copies = max(2, math.ceil(L2_DEFEAT_BYTES / per))
        mats = [(mant, exps)] + [(mant.clone(), exps.clone()) for _ in range(copies - 1)]
        res = ops.lm_outputs(dev, k)   # preallocated: the timed graph holds only the lm_head kernels

        def call(i):
            m, e = mats[i % copies]
            ops.lm_head_bfp8(h, m, e, k, out=res)
        desc = "BFP8 lm_head 65536x1024 + argmax + top-40"
    graph = graph_of(torch, call, copies)
    clk = ClockSampler(gpu_uuid(torch, dev), dev.index or 0)
    secs = timed(torch, lambda i: graph.replay(), args.steps, args.warmup, barrier)
    clocks = clk.stop()
    per_step = secs / args.steps / copies   # one lm_head per table copy in each replay
    nbytes = per + 4 * H
    gbs = nbytes / per_step / 1e9

    # end to end through the host API
    L = _lib.load()
    hh = h.cpu().numpy().astype(np.float32)
    ids = np.zeros(k, np.int32)
    scs = np.zeros(k, np.float32)
    if args.workload == "lm_bf16":
        host_tab = w[:].to(torch.bfloat16).view(torch.int16).cpu().numpy()
        L.qwen_b200_register_weights(host_tab.ctypes.data, host_tab.nbytes)

        def e2e_call(i):
            L.lm_head_topk(hh.ctypes.data, host_tab.ctypes.data, V, H, k, ids.ctypes.data, scs.ctypes.data)
    else:
        hx = torch.empty(H, dtype=torch.float32, pin_memory=True)
        hx.copy_(h.cpu())
        hi = torch.empty(k + 2, dtype=torch.int32, pin_memory=True)
        hs = torch.empty(k, dtype=torch.float32, pin_memory=True)
        dh = torch.empty(H, dtype=torch.float32, device=dev)

        def e2e_call(i):
            dh.copy_(hx, non_blocking=True)
            m, e = mats[i % copies]
            r = ops.lm_head_bfp8(dh, m, e, k, out=res)
            hi[:k].copy_(r.ids[:k], non_blocking=True)
            hs.copy_(r.scores[:k], non_blocking=True)
            hi[k:k + 1].copy_(r.argmax, non_blocking=True)
    for i in range(args.warmup):
        e2e_call(i)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_call(i)
    torch.cuda.synchronize()
    e2e_step = (time.perf_counter() - t0) / args.steps
    del w
    return {"value": round(world * gbs, 2), "ms_per_step": round(per_step * 1e3, 4),
            "config": {"workload": desc, "algorithmic_bytes_per_step": nbytes,
                       "l2": f"rotates {copies} copies", "launch": "CUDA graph of one call per copy"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind,
                         "traffic": committed_traffic(args.workload)},
            "e2e": {"value": round(world * nbytes / e2e_step / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_step * 1e3, 4), "h2d_bytes_per_step": 4 * H,
                    "d2h_bytes_per_step": 8 * k + 4},
            "gpu_launches": args.steps * copies, "clocks": clocks}


def run_rtl20(args, torch, dev, barrier, world, hbm_peak, peak_kind):
    """Secondary line: the RTL dequant mode (gemv_core's floor(y * 2^20)
    words) of the cfg-0 GEMV, 3584 x 1024, from fp32 x.  `value` times the
    kernel alone (a CUDA graph of one call per weight copy); `exact_ms`
    times the exact-mode single GEMV entry the same way; `e2e` copies x in
    and the words out around each call."""
    import numpy as np

    from qwen_b200 import _lib, model, ops

    L = _lib.load()
    M, K = 3584, 1024
    wbytes = M * K + M * K // 64
    nbytes = wbytes + 4 * K + 4 * M
    copies = args.copies or max(2, math.ceil(L2_DEFEAT_BYTES / wbytes))
    ds = model.DeviceStack([model.Linear("mlp.up_proj", M, K)], copies=copies, device=dev, seed=1234)
    views = [ds.views(c)[0] for c in range(copies)]
    words = torch.empty(M, dtype=torch.int32, device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    y = torch.empty(M, dtype=torch.float32, device=dev)

    def rtl(i, x=None):
        xx, m, e, _ = views[i % copies]
        xx = xx if x is None else x
        _lib.check(L.qwen_b200_gemv_rtl20_dev(words.data_ptr(), xx.data_ptr(), None, None, m.data_ptr(),
                                              e.data_ptr(), M, K, flags.data_ptr(), ops._stream()), "rtl20")

    def exact(i):
        xx, m, e, _ = views[i % copies]
        _lib.check(L.qwen_b200_gemv_dev(y.data_ptr(), xx.data_ptr(), m.data_ptr(), e.data_ptr(), M, K,
                                        ops._stream()), "gemv")

    per = {}
    clocks = None
    for name, fn in (("rtl20", rtl), ("exact", exact)):
        graph = graph_of(torch, fn, copies)
        clk = ClockSampler(gpu_uuid(torch, dev), dev.index or 0)
        per[name] = timed(torch, lambda i: graph.replay(), args.steps, args.warmup, barrier) / args.steps / copies
        sampled = clk.stop()
        if name == "rtl20":
            clocks = sampled
        del graph
    gbs = nbytes / per["rtl20"] / 1e9

    hx = torch.empty(K, dtype=torch.float32, pin_memory=True)
    hx.copy_(views[0][0].cpu())
    hw = torch.empty(M, dtype=torch.int32, pin_memory=True)
    dx = torch.empty(K, dtype=torch.float32, device=dev)

    def e2e_call(i):
        dx.copy_(hx, non_blocking=True)
        rtl(i, dx)
        hw.copy_(words, non_blocking=True)
    for i in range(args.warmup):
        e2e_call(i)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_call(i)
    torch.cuda.synchronize()
    e2e_step = (time.perf_counter() - t0) / args.steps
    if int(flags.item()) != 0:
        raise RuntimeError("rtl20 bench: unexpected saturation flags on N(0, 0.02) weights")
    return {"value": round(world * gbs, 2), "ms_per_step": round(per["rtl20"] * 1e3, 5),
            "dtype": "int16xint8->int64 fixed point",
            "config": {"workload": "RTL dequant mode (floor(y*2^20) words), single BFP8 GEMV 3584x1024",
                       "algorithmic_bytes_per_step": nbytes, "exact_ms": round(per["exact"] * 1e3, 5),
                       "l2": f"rotates {copies} weight copies ({copies * wbytes / 1e9:.2f} GB) > 126 MB L2",
                       "launch": "CUDA graph of one call per copy (one launch each: the CTAs quantize x)"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind, "traffic": None,
                         "kernel": "gemv_warp_kernel<RTL>"},
            "e2e": {"value": round(world * nbytes / e2e_step / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_step * 1e3, 4), "h2d_bytes_per_step": 4 * K,
                    "d2h_bytes_per_step": 4 * M},
            "gpu_launches": args.steps * copies, "clocks": clocks}


# ------------------------------------------------------------------ reference arm
def reference_stack_runner(workload, seed=7):
    """The reference's own bfp8_gemv (oracle/_ref/libref_kernels.so, built
    from 04-板载脚本与工具/qwen_kernels_opt.c) over the workload's GEMVs."""
    import ctypes

    import numpy as np

    lib = ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libref_kernels.so"))
    P, I = ctypes.c_void_p, ctypes.c_int
    lib.bfp8_gemv.argtypes = [P, P, P, P, I, I]
    lib.bfp8_gemv.restype = None
    lib.init_kernels()
    shapes, desc = stack_shapes("stack" if workload == "batched" else workload)
    rng = np.random.default_rng(seed)
    ents = []
    for t in shapes:
        mant = rng.integers(-128, 128, (t.M, t.K), dtype=np.int8)
        exps = rng.integers(118, 131, (t.M, t.K // 64), dtype=np.uint8)
        x = rng.standard_normal(t.K, dtype=np.float32)
        y = np.empty(t.M, np.float32)
        ents.append((y, x, mant, exps, t.M, t.K))

    def token():
        for y, x, m, e, M, K in ents:
            lib.bfp8_gemv(y.ctypes.data, x.ctypes.data, m.ctypes.data, e.ctypes.data, M, K)
    return token, shapes, desc


def cpu_baseline(workload, batch=1):
    """Bounded sample of the reference C on this host's cores, in a child
    process so OpenMP starts with every host thread."""
    if workload not in ("stack", "gemv", "batched"):
        return None
    env = dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count()))
    try:
        out = subprocess.run([sys.executable, os.path.abspath(__file__), "--impl", "reference", "--cpu-sample",
                              "--workload", workload, "--batch", str(batch)], env=env, capture_output=True, text=True,
                             timeout=300)
        return json.loads(out.stdout.strip().splitlines()[-1])
    except Exception as e:  # a baseline failure must not hide the GPU number
        return {"error": str(e)[:200]}


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    if args.workload == "rtl20":
        print(json.dumps({"impl": "reference", "unavailable": "the RTL dequant mode exists only as FPGA fabric "
                          "(gemv_core.v); the reference has no CPU implementation of it"}))
        return
    from qwen_b200 import model

    token, shapes, desc = reference_stack_runner(args.workload)
    nb = model.stack_bytes(shapes)
    # the reference has no batched path: B sequences cost B one-sequence passes
    seqs = args.batch if args.workload == "batched" else 1
    if seqs > 1:
        nb = model.batched_bytes(shapes, seqs)
        desc = f"batched decode: B={seqs} sequences x {desc}, one sequence at a time"
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count()))
    if args.cpu_sample:
        # bounded sample: whole tokens for ~10 s (at least 2)
        token()
        n, t0 = 0, time.perf_counter()
        while n < 2 or (time.perf_counter() - t0 < 10.0 and n < 1000):
            token()
            n += 1
        dt = (time.perf_counter() - t0) / n * seqs
        print(json.dumps({"value": round(nb["total"] / dt / 1e9, 4), "unit": "GB/s", "ms_per_step": round(dt * 1e3, 3),
                          "cores": cores, "kind": "reference",
                          "sample": f"{n} whole one-sequence passes of the stack after 1 warm-up pass, scaled by "
                                    f"{seqs} sequences per step ({desc}); reference C bfp8_gemv scalar build, "
                                    "OpenMP"}))
        return
    for _ in range(args.warmup):
        token()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(seqs):
            token()
    dt = (time.perf_counter() - t0) / args.steps
    v = nb["total"] / dt / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (reference scalar path)",
        "data": "synthetic: random int8 mantissas, exponents 118..130, activations N(0,1)",
        "config": {"workload": desc, "algorithmic_bytes_per_step": nb["total"]},
        "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": cores, "kind": "reference",
                         "sample": f"{args.steps} whole tokens after {args.warmup} warm-up tokens"},
        "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse()
    # the driver reads one JSON line from rank 0's stdout: keep NCCL's version
    # banner and informational lines off it unless the caller asked for them
    if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
        os.environ["NCCL_DEBUG"] = "WARN"
    if args.impl == "reference":
        os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count()))
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
