#!/usr/bin/env python3
"""Benchmark of the BFP8 GEMV / lm_head decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload stack|gemv|lm_bf16|lm_bfp8|sharded|batched|rtl20|token] [--batch B]
                    [--headline-only] [--no-sharded] [--no-cpu-baseline] [--no-e2e]

Default workload (the BASELINE metric's configuration): the full per-token
linear stack of Qwen3.5-0.8B at batch 1 -- 150 BFP8 GEMVs, 504,791,040 bytes
of weights, each GEMV on its own fp32 N(0,1) activation re-quantized inside
the kernel -- as ONE grouped kernel launch per token.  A step is one token.
The weights are the same packed bytes in both arms (``synthetic_stack``) and
the timed steps rotate through enough byte-identical device copies (> 4 GB)
that no step finds its weights in the 126 MB L2.

One JSON line on rank 0.  `value` is algorithmic GB/s of the stack
(weights + fp32 activations in + fp32 outputs out, summed over ranks) with
everything resident in HBM; `e2e` is the same metric with every token's
activations copied in from pinned host memory and its outputs copied back
inside the timed region (copies of one token overlap the neighbouring
tokens' kernels on two copy streams; `e2e.serial_*` has them in line).  With
--gpus N under torchrun every rank runs its own token stream on its own GPU
(independent decode replicas, weak scaling, no collective on the data path).

Beside the headline the default line carries, on one GPU, `configs`: the
other BASELINE configurations (the single 3584x1024 GEMV, the bf16 and BFP8
lm_heads with top-40, batched tcgen05 decode at B = 8/32/128/256), the same
150 GEMVs issued as a token issues them (`chain`), and the reference-facing
host-pointer bfp8_gemv per call (`abi`); and on every N, `sharded`: the
row-sharded multi-GPU configuration (8 x gate/up 28672x8192 + down
8192x28672) at batch 1 and 64, strong scaling over the ranks, with a parity
check against one GPU.  `cpu_baseline` times the reference on the host.

--impl reference times the reference's own C bfp8_gemv (compiled from its
source for this host, scalar float path since the host has no NEON) on the
same packed bytes with every host thread, rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "qwen35-ax7020-edge-llm_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "BFP8 GEMV HBM GB/s (% of B200 peak); 0.8B-shape linear-stack ms/token, batch 1"
L2_DEFEAT_BYTES = 4.3e9
STACK_SEED = 1234


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["stack", "gemv", "lm_bf16", "lm_bfp8", "sharded", "batched", "rtl20",
                                           "token"],
                    default="stack")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per step: --workload batched (default 256) or sharded (default 1)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="--workload sharded: stores into every GPU by the kernels, or NCCL all-gathers")
    ap.add_argument("--topk", type=int, default=40, help="--workload lm_bf16 / lm_bfp8: k of the fused top-k")
    ap.add_argument("--headline-only", action="store_true", help="skip the per-configuration sub-records")
    ap.add_argument("--no-sharded", action="store_true", help="skip the row-sharded multi-GPU record")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--copies", type=int, default=0,
                    help="weight copies to rotate (default: enough for > 4 GB; fewer only for profiling)")
    ap.add_argument("--cpu-sample", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--cpu-kind", default="ref", help=argparse.SUPPRESS)
    ap.add_argument("--cpu-data", default="", help=argparse.SUPPRESS)
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


def pack_rows(w):
    """Block-64 BFP8 SoA packing of fp32 rows [M, K] by the reference
    packer's rule (05-主机侧源码/bfp8_packer.py:53-86): e = ceil(log2(peak))
    + 127 per 64-block (127 and zero mantissas below 1e-12), m =
    clip(rint(w * 2^(134 - e)), -128, 127); ceil(log2) is taken exactly from
    the float's bits, as the device packer does."""
    import numpy as np

    M, K = w.shape
    blk = w.reshape(M, K // 64, 64)
    peak = np.abs(blk).max(axis=2)
    u = peak.view(np.uint32)
    lg = ((u >> 23) & 0xFF).astype(np.int32) - 127 + ((u & 0x7FFFFF) != 0)
    e = np.clip(lg + 127, 0, 255)
    zero = ~(peak >= np.float32(1e-12))
    e[zero] = 127
    scale = ((261 - e).astype(np.uint32) << 23).view(np.float32)
    m = np.clip(np.rint(blk * scale[:, :, None]), -128, 127).astype(np.int8)
    m[zero] = 0
    return m.reshape(M, K), e.astype(np.uint8)


def synthetic_stack(shapes, seed=STACK_SEED):
    """The packed weights (the weight-file image at model.layout offsets) and
    the fp32 activations (one per GEMV, concatenated in stack order) of a
    stack -- the SAME bytes in the B200 arm and the reference arm.  One
    N(0, 0.02) matrix per distinct shape is drawn (numpy, seeded) and packed;
    the i-th tensor of that shape is it with its rows rotated by 997 * i
    (packed rows are independent: every tensor is a packed N(0, 0.02) matrix
    and no two are equal).  Activations are N(0, 1)."""
    import numpy as np

    from qwen_b200 import model

    table, total = model.layout(shapes)
    buf = np.zeros(total, np.uint8)
    bases, seen = {}, {}
    for name, (off, t) in table.items():
        key = (t.M, t.K)
        if key not in bases:
            rng = np.random.default_rng([seed, t.M, t.K])
            w = rng.standard_normal((t.M, t.K), dtype=np.float32)
            w *= np.float32(0.02)
            bases[key] = pack_rows(w)
        i = seen.get(key, 0)
        seen[key] = i + 1
        mant, exps = bases[key]
        sh = (997 * i) % t.M
        buf[off:off + t.mant_bytes] = np.roll(mant, sh, axis=0).view(np.uint8).reshape(-1)
        buf[off + t.mant_bytes:off + t.mant_bytes + t.exp_bytes] = np.roll(exps, sh, axis=0).reshape(-1)
        buf[off + t.mant_bytes + t.exp_bytes:off + t.soa_bytes] = 127   # exponent padding of the file format
    x = np.random.default_rng([seed, 1]).standard_normal(sum(t.K for t in shapes), dtype=np.float32)
    return buf, x


def stack_views(buf, x, shapes):
    """(y, x, mant, exps, M, K) host arrays of every GEMV of a synthetic
    stack, sliced from the weight image as the engine slices its mmap
    (04-板载脚本与工具/qwen_real_engine.py:834-846)."""
    import numpy as np

    from qwen_b200 import model

    table, _ = model.layout(shapes)
    out, pos = [], 0
    for t in shapes:
        off, _ = table[t.name]
        mant = buf[off:off + t.mant_bytes].view(np.int8).reshape(t.M, t.K)
        exps = buf[off + t.mant_bytes:off + t.mant_bytes + t.exp_bytes].reshape(t.M, t.K // 64)
        out.append((np.empty(t.M, np.float32), x[pos:pos + t.K], mant, exps, t.M, t.K))
        pos += t.K
    return out


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


def max_over_ranks(torch, dist, secs, dev, world):
    t = torch.tensor([secs], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def guarded(fn, *a, **kw):
    """A sub-record must never take the headline down with it."""
    try:
        return fn(*a, **kw)
    except Exception as e:
        return {"error": f"{type(e).__name__}: {str(e)[:300]}"}


def run_b200(args):
    import torch
    import torch.distributed as dist

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
            "data": "synthetic: weights N(0,0.02) packed BFP8 (seeded), activations N(0,1)"}
    cpu_data = None
    if args.workload == "gemv":
        line.update(run_single_gemv(torch, dev, barrier, hbm_peak, peak_kind, args.steps, args.warmup))
    elif args.workload == "stack":
        rec, cpu_data = run_stack(args, torch, dist, dev, barrier, world, rank, hbm_peak, peak_kind)
        line.update(rec)
        if world == 1 and not args.headline_only:
            line["configs"] = run_configs(args, torch, dist, dev, barrier, world, rank, hbm_peak, peak_kind)
        if not args.headline_only and not args.no_sharded:
            line["sharded"] = run_sharded_records(args, torch, dist, dev, barrier, world, rank, local, hbm_peak,
                                                  peak_kind)
    elif args.workload == "sharded":
        line.update(run_sharded(args, torch, dist, dev, barrier, world, rank, local, hbm_peak, peak_kind,
                                args.batch, args.exchange, args.steps, args.warmup))
    elif args.workload == "batched":
        line.update(run_batched(args, torch, dist, dev, barrier, world, rank, hbm_peak, peak_kind, args.batch,
                                args.steps, args.warmup))
    elif args.workload == "rtl20":
        line.update(run_rtl20(args, torch, dev, barrier, world, hbm_peak, peak_kind))
    elif args.workload == "token":
        line.update(run_token(args, torch, dev, world, rank))
    else:
        line.update(run_lm_head(args, torch, dev, barrier, world, hbm_peak, peak_kind, args.workload, args.steps,
                                args.warmup))

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload, args.batch, cpu_data)
    if cpu_data:
        try:
            os.unlink(cpu_data)
        except OSError:
            pass
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ headline
def run_stack(args, torch, dist, dev, barrier, world, rank, hbm_peak, peak_kind):
    """The 0.8B linear stack as one grouped launch per token."""
    import numpy as np

    from qwen_b200 import model, ops

    shapes, desc = stack_shapes(args.workload)
    nb = model.stack_bytes(shapes)
    wbytes = nb["weights"]
    copies = args.copies or max(2, math.ceil(L2_DEFEAT_BYTES / wbytes))
    hbuf, hx = synthetic_stack(shapes)
    cpu_data = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the reference-arm children read the same bytes
        fd, cpu_data = tempfile.mkstemp(suffix=".npz", prefix="qwen_b200_bench_")
        os.close(fd)
        np.savez(cpu_data, buf=hbuf, x=hx)
    ds = model.DeviceStack(shapes, copies=copies, device=dev, host_bytes=hbuf, host_x=hx)
    del hbuf
    plans = [ops.LinearStack(ds.views(c)) for c in range(copies)]
    launches_per_step = 2   # act_prep + gemv_warp

    def step(i):
        plans[i % copies].run()

    clk = ClockSampler(gpu_uuid(torch, dev), dev.index or 0)
    secs = timed(torch, step, args.steps, args.warmup, barrier)
    clocks = clk.stop()
    per_step = max_over_ranks(torch, dist, secs, dev, world) / args.steps
    value = world * nb["total"] / per_step / 1e9
    kernel_gbs = nb["total"] / per_step / 1e9

    e2e = None
    if not args.no_e2e:
        e2e = end_to_end(torch, dist, ds, plans, copies, nb, args, barrier, world, dev)
    for p in plans:
        p.close()
    del ds, plans
    torch.cuda.empty_cache()
    return {
        "value": round(value, 2), "ms_per_step": round(per_step * 1e3, 4),
        "config": {"workload": desc, "gemvs_per_step": len(shapes), "weight_bytes": wbytes,
                   "algorithmic_bytes_per_step": nb["total"], "macs_per_step": nb["macs"],
                   "weights": "bench.synthetic_stack (the reference arm streams the same bytes)",
                   "l2": f"rotates {copies} weight copies ({copies * wbytes / 1e9:.2f} GB) > 126 MB L2",
                   "launch": "act_prep + one grouped warp-autonomous kernel (PDL) per step",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 2), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(kernel_gbs / hbm_peak, 4), "peak_kind": peak_kind,
                     "traffic": committed_traffic(args.workload), "kernel": "gemv_warp_kernel (grouped)"},
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }, cpu_data


def end_to_end(torch, dist, ds, plans, copies, nb, args, barrier, world, dev):
    """The same tokens through the public API with host buffers: every
    token's activations copied in from pinned host memory, the stack run, its
    outputs copied back.  Pipelined: two activation / output buffer sets, the
    input copies on one copy stream and the output copies on another, so a
    token's copies overlap the neighbouring tokens' kernels; the timed region
    runs from an event every stream waits on to the last output copy.  The
    serial figure has every copy in line with the kernels on one stream."""
    from qwen_b200 import ops

    hx = torch.empty(ds.x_flat.numel(), dtype=torch.float32, pin_memory=True)
    hx.copy_(ds.x_flat.cpu())
    hy = [torch.empty(ds.y_flat.numel(), dtype=torch.float32, pin_memory=True) for _ in range(2)]
    xb = [ds.x_flat, torch.empty_like(ds.x_flat)]
    yb = [ds.y_flat, torch.empty_like(ds.y_flat)]
    pl = [plans, [ops.LinearStack(ds.views(c, xb[1], yb[1])) for c in range(copies)]]
    cur = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    in_done = [torch.cuda.Event() for _ in range(2)]
    run_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]
    for k in range(2):
        for ev in (in_done[k], run_done[k], out_done[k]):
            ev.record(cur)

    def token(i):
        k = i % 2
        s_in.wait_event(run_done[k])            # the kernels two tokens back are done reading xb[k]
        with torch.cuda.stream(s_in):
            xb[k].copy_(hx, non_blocking=True)
            in_done[k].record(s_in)
        cur.wait_event(in_done[k])
        cur.wait_event(out_done[k])             # yb[k] was copied out
        pl[k][i % copies].run()
        run_done[k].record(cur)
        s_out.wait_event(run_done[k])
        with torch.cuda.stream(s_out):
            hy[k].copy_(yb[k], non_blocking=True)
            out_done[k].record(s_out)

    def run(n, base):
        for i in range(n):
            token(base + i)

    def barrier_():
        if world > 1:
            dist.barrier()

    run(args.warmup, 0)
    torch.cuda.synchronize()
    barrier_()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(cur)
    s_in.wait_event(start)
    s_out.wait_event(start)
    run(args.steps, args.warmup)
    cur.wait_event(out_done[0])
    cur.wait_event(out_done[1])
    end.record(cur)
    torch.cuda.synchronize()
    barrier_()
    per = max_over_ranks(torch, dist, start.elapsed_time(end) / 1e3, dev, world) / args.steps

    def serial_step(i):
        ds.x_flat.copy_(hx, non_blocking=True)
        plans[i % copies].run()
        hy[0].copy_(ds.y_flat, non_blocking=True)

    ser = max_over_ranks(torch, dist, timed(torch, serial_step, args.steps, args.warmup, barrier), dev, world)
    ser /= args.steps
    for p in pl[1]:
        p.close()
    return {"value": round(world * nb["total"] / per / 1e9, 2), "unit": "GB/s", "ms_per_step": round(per * 1e3, 4),
            "h2d_bytes_per_step": hx.numel() * 4, "d2h_bytes_per_step": hy[0].numel() * 4,
            "serial_value": round(world * nb["total"] / ser / 1e9, 2), "serial_ms_per_step": round(ser * 1e3, 4),
            "path": "ops.LinearStack.run on the timed stream; torch pinned-memory copies on two copy streams"}


# ------------------------------------------------------------------ sub-records (one GPU)
def run_configs(args, torch, dist, dev, barrier, world, rank, hbm_peak, peak_kind):
    """The other BASELINE configurations, each a bounded run with its own
    roofline (steps are kept short: these are reported beside the headline)."""
    steps, warm = 20, 3
    out = {}
    out["cfg0_gemv_3584x1024"] = guarded(run_single_gemv, torch, dev, barrier, hbm_peak, peak_kind, steps, warm)
    torch.cuda.empty_cache()
    for w in ("lm_bf16", "lm_bfp8"):
        out[f"cfg2_{w}"] = guarded(run_lm_head, args, torch, dev, barrier, world, hbm_peak, peak_kind, w, steps, warm)
        torch.cuda.empty_cache()
    for B in (8, 32, 128, 256):
        out[f"cfg3_b{B}"] = guarded(run_batched, args, torch, dist, dev, barrier, world, rank, hbm_peak, peak_kind, B,
                                    steps, warm, e2e=False)
        torch.cuda.empty_cache()
    out["chain"] = guarded(run_chain, torch, dev, barrier, hbm_peak, peak_kind, steps, warm)
    torch.cuda.empty_cache()
    out["abi"] = guarded(run_abi, torch, dev)
    torch.cuda.empty_cache()
    # the per-token C loop through forward_token_c, beside the reference's own loop on the host cores
    tok_args = argparse.Namespace(**vars(args))
    tok_args.steps, tok_args.warmup = steps, warm
    rec = guarded(run_token, tok_args, torch, dev, world, rank)
    if not args.no_cpu_baseline and "error" not in rec:
        rec["cpu_baseline"] = cpu_baseline("token")
    out["token"] = rec
    torch.cuda.empty_cache()
    return out


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


def run_single_gemv(torch, dev, barrier, hbm_peak, peak_kind, steps, warm):
    """one 3584 x 1024 GEMV per call through the device
    entry point (one launch: every CTA quantizes x), timed as a CUDA graph of
    one call per weight copy; `e2e` is the reference-facing bfp8_gemv with
    host pointers (registered weights), per call."""
    import numpy as np

    from qwen_b200 import _lib, model, ops

    L = _lib.load()
    M, K = 3584, 1024
    shapes = [model.Linear("mlp.up_proj", M, K)]
    wbytes = M * K + M * K // 64
    nbytes = wbytes + 4 * K + 4 * M
    copies = max(2, math.ceil(L2_DEFEAT_BYTES / wbytes))
    hbuf, hx = synthetic_stack(shapes)
    ds = model.DeviceStack(shapes, copies=copies, device=dev, host_bytes=hbuf, host_x=hx)
    views = [ds.views(c)[0] for c in range(copies)]
    y = torch.empty(M, dtype=torch.float32, device=dev)

    def call(i):
        xx, m, e, _ = views[i % copies]
        _lib.check(L.qwen_b200_gemv_dev(y.data_ptr(), xx.data_ptr(), m.data_ptr(), e.data_ptr(), M, K,
                                        ops._stream()), "gemv")

    graph = graph_of(torch, call, copies)
    clk = ClockSampler(gpu_uuid(torch, dev), dev.index or 0)
    per = timed(torch, lambda i: graph.replay(), steps, warm, barrier) / steps / copies
    clocks = clk.stop()
    del graph
    gbs = nbytes / per / 1e9
    # the drop-in: host x, host weights (registered once, like the engine's mmap), host y
    (yh, xh, mh, eh, _, _), = stack_views(hbuf, hx, shapes)
    L.qwen_b200_register_weights(hbuf.ctypes.data, hbuf.nbytes)
    for _ in range(20):
        L.bfp8_gemv(yh.ctypes.data, xh.ctypes.data, mh.ctypes.data, eh.ctypes.data, M, K)
    n, t0 = 0, time.perf_counter()
    while n < 200 or time.perf_counter() - t0 < 0.5:
        L.bfp8_gemv(yh.ctypes.data, xh.ctypes.data, mh.ctypes.data, eh.ctypes.data, M, K)
        n += 1
    call_s = (time.perf_counter() - t0) / n
    L.qwen_b200_forget_weights(hbuf.ctypes.data)
    ok = bool(np.array_equal(yh.view(np.uint32), y.cpu().numpy().view(np.uint32)))
    return {"value": round(gbs, 2), "unit": "GB/s", "us_per_call": round(per * 1e6, 3),
            "ms_per_step": round(per * 1e3, 5), "gpu_launches": steps * copies,
            "config": {"workload": "single BFP8 GEMV 3584x1024, batch 1 (BASELINE config 0)",
                       "algorithmic_bytes_per_step": nbytes, "launch": "CUDA graph of one call per copy",
                       "l2": f"rotates {copies} weight copies ({copies * wbytes / 1e9:.2f} GB)"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind,
                         "traffic": committed_traffic("gemv"), "kernel": "gemv_split_kernel"},
            "e2e": {"value": round(nbytes / call_s / 1e9, 2), "unit": "GB/s", "us_per_call": round(call_s * 1e6, 2),
                    "h2d_bytes_per_step": 4 * K, "d2h_bytes_per_step": 4 * M,
                    "path": "bfp8_gemv drop-in, host pointers, weights registered", "same_bits_as_device": ok},
            "clocks": clocks}


def run_chain(torch, dev, barrier, hbm_peak, peak_kind, steps, warm):
    """The 150 GEMVs of a token issued the way a decoder issues them, each a
    dependent launch: per layer the rmsnorm -> projection pairs of the
    attention / DeltaNet block (the first with the residual add in front),
    its output projection (its input, the attention / DeltaNet output, is a
    fixed vector: that glue is outside this path), then the MLP as residual
    add + rmsnorm -> gate, rmsnorm -> up, swiglu -> down.  The token is one
    CUDA graph per weight copy."""
    from qwen_b200 import _lib, model, ops

    L = _lib.load()
    shapes = model.qwen35_08b_stack()
    nb = model.stack_bytes(shapes)
    copies = max(2, math.ceil(L2_DEFEAT_BYTES / nb["weights"]))
    hbuf, hx = synthetic_stack(shapes)
    ds = model.DeviceStack(shapes, copies=copies, device=dev, host_bytes=hbuf, host_x=hx)
    del hbuf
    H = model.HIDDEN
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    h0 = torch.randn(H, generator=g, device=dev)
    ln = torch.randn(H, generator=g, device=dev) * 0.1
    glue = torch.randn(2048, generator=g, device=dev)
    hs = [torch.empty(H, device=dev) for _ in range(2)]
    ys = [torch.empty(t.M, device=dev) for t in shapes]
    st = lambda: ops._stream()   # noqa: E731
    eps = 1e-6

    def token(c):
        views = ds.views(c)
        h, nxt = h0, 0
        res = None
        i = 0
        for l in range(model.LAYERS):
            n_attn = 4 if l in model.FULL_ATTN else 3
            proj = list(range(i, i + n_attn - 1))        # q/k/v or qkv/z: from rmsnorm(h)
            o = i + n_attn - 1
            gate, up, down = o + 1, o + 2, o + 3
            for j, k in enumerate(proj):
                _, m, e, _ = views[k]
                t = shapes[k]
                if j == 0 and res is not None:          # h = h + previous down, then its rmsnorm
                    out = hs[nxt]
                    _lib.check(L.qwen_b200_residual_rmsnorm_gemv_dev(
                        ys[k].data_ptr(), out.data_ptr(), h.data_ptr(), res.data_ptr(), ln.data_ptr(), eps,
                        m.data_ptr(), e.data_ptr(), t.M, t.K, st()), "chain")
                    h, nxt = out, 1 - nxt
                else:
                    _lib.check(L.qwen_b200_rmsnorm_gemv_dev(ys[k].data_ptr(), h.data_ptr(), ln.data_ptr(), eps,
                                                            m.data_ptr(), e.data_ptr(), t.M, t.K, st()), "chain")
            _, m, e, _ = views[o]
            t = shapes[o]
            _lib.check(L.qwen_b200_gemv_dev(ys[o].data_ptr(), glue.data_ptr(), m.data_ptr(), e.data_ptr(), t.M, t.K,
                                            st()), "chain")
            out = hs[nxt]                                 # h = h + o, rmsnorm -> gate
            _, m, e, _ = views[gate]
            t = shapes[gate]
            _lib.check(L.qwen_b200_residual_rmsnorm_gemv_dev(
                ys[gate].data_ptr(), out.data_ptr(), h.data_ptr(), ys[o].data_ptr(), ln.data_ptr(), eps,
                m.data_ptr(), e.data_ptr(), t.M, t.K, st()), "chain")
            h, nxt = out, 1 - nxt
            _, m, e, _ = views[up]
            t = shapes[up]
            _lib.check(L.qwen_b200_rmsnorm_gemv_dev(ys[up].data_ptr(), h.data_ptr(), ln.data_ptr(), eps,
                                                    m.data_ptr(), e.data_ptr(), t.M, t.K, st()), "chain")
            _, m, e, _ = views[down]
            t = shapes[down]
            _lib.check(L.qwen_b200_swiglu_gemv_dev(ys[down].data_ptr(), ys[gate].data_ptr(), ys[up].data_ptr(),
                                                   m.data_ptr(), e.data_ptr(), t.M, t.K, st()), "chain")
            res = ys[down]
            i = down + 1
        assert i == len(shapes)

    graphs = [graph_of(torch, lambda _i, c=c: token(c), 1) for c in range(copies)]
    clk = ClockSampler(gpu_uuid(torch, dev), dev.index or 0)
    per = timed(torch, lambda i: graphs[i % copies].replay(), steps, warm, barrier) / steps
    clocks = clk.stop()
    del graphs
    gbs = nb["total"] / per / 1e9
    return {"value": round(gbs, 2), "unit": "GB/s", "ms_per_token": round(per * 1e3, 4),
            "config": {"workload": "qwen35-0.8b linear stack as a token issues it: 150 dependent GEMV launches "
                                   "(rmsnorm / residual / swiglu fused in front), one CUDA graph per token",
                       "algorithmic_bytes_per_step": nb["total"],
                       "l2": f"rotates {copies} weight copies"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind,
                         "kernel": "gemv_split_kernel (150 launches)"},
            "gpu_launches_per_token": len(shapes), "clocks": clocks}


# ------------------------------------------------------------------ token loop
TOKEN_METRIC = "forward_token_c ms/token: Qwen3.5-0.8B shape, 24 layers + lm_head argmax, drop-in C ABI"
TOKEN_LAUNCHES = 18 * 5 + 6 * 2 + 3   # per token: linear layers, full-attention MLPs, embed / rmsnorm / lm_head


def _token_loop(fwd, M, lps, mps, cb, h, first, n):
    """n autoregressive tokens through a forward_token_c-shaped function
    (each returned id is the next input); returns the last id."""
    tok = first
    for _ in range(n):
        tok = fwd(tok, h.ctypes.data, ctypes.byref(lps), ctypes.byref(mps), M.is_full.ctypes.data,
                  M.final_ln.ctypes.data, M.embed.ctypes.data, cb, None)
        if tok < 0:
            raise RuntimeError("forward_token_c failed")
    return tok


def run_token(args, torch, dev, world, rank):
    """The reference's per-token C loop as the engine calls it
    (qwen_real_engine.py:1262-1272): forward_token_c with host h, host plans,
    the engine's mutable states and a full-attention callback (a stand-in:
    attention is not on this library's path), timed by wall clock per token.
    Both state modes: mirror (the states copied in and out every token, the
    reference's contract) and resident (the states stay on the device)."""
    import numpy as np

    from qwen_b200 import _lib, plans

    L = _lib.load()
    M = plans.TokenModel(seed=0)
    cb = plans.attention_stand_in()
    out = {}
    for mode, name in ((0, "mirror"), (1, "resident"), (2, "pinned")):
        assert L.qwen_b200_gdn_state_mode(mode) == 0
        st = M.fresh_states()
        lps, mps = M.plans(st)
        h = np.zeros(plans.HIDDEN, np.float32)
        tok = _token_loop(L.forward_token_c, M, lps, mps, cb, h, 1, max(args.warmup, 3))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _token_loop(L.forward_token_c, M, lps, mps, cb, h, tok, args.steps)
        dt = (time.perf_counter() - t0) / args.steps
        if mode == 1:
            L.qwen_b200_gdn_state_sync()
        L.qwen_b200_gdn_state_drop()
        out[name] = dt
    L.qwen_b200_gdn_state_mode(0)
    L.qwen_b200_reset_weights()
    state_bytes = M.n_linear * (3 * 3 * plans.V + plans.HEADS * plans.HEAD_DIM ** 2) * 4
    return {"metric": TOKEN_METRIC, "unit": "ms/token", "higher_is_better": False, "scaling": "replicas",
            "value": round(out["mirror"] * 1e3, 3), "ms_per_step": round(out["mirror"] * 1e3, 3),
            "dtype": "int16xint8->fp32 GEMVs, fp32 layer glue (NEON-build order)",
            "data": "synthetic: plans.TokenModel(seed=0) -- random BFP8 weights (one linear-layer set, one MLP set "
                    "shared by the layers), per-layer states, random bf16 embedding table",
            "config": {"workload": "forward_token_c, 18 Gated-DeltaNet + 6 full-attention layers (attention: a "
                                   "host stand-in callback), final rmsnorm, lm_head argmax over 65536 rows",
                       "state_mode": "mirror (conv and recurrent states copied in and out every token)",
                       "resident_ms_per_token": round(out["resident"] * 1e3, 3),
                       "pinned_mirror_ms_per_token": round(out["pinned"] * 1e3, 3),
                       "launches_per_token": TOKEN_LAUNCHES,
                       "host_round_trips_per_token": 6},
            "e2e": {"value": round(out["mirror"] * 1e3, 3), "unit": "ms/token",
                    "h2d_bytes_per_step": 4 * plans.HIDDEN * 6 + state_bytes,
                    "d2h_bytes_per_step": 4 * plans.HIDDEN * 7 + 4 + state_bytes},
            "gpu_launches": TOKEN_LAUNCHES * args.steps}


def token_reference_sample(budget=10.0, steps=None, warmup=1):
    """The reference's own forward_token_c (oracle/_ref, its C file compiled
    here; portable build, OpenMP over every host thread) on the same
    synthetic model: (ms per token, tokens timed, threads)."""
    import numpy as np

    from qwen_b200 import plans

    cores = _omp_threads(os.cpu_count())
    lib = ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libref_kernels.so"))
    P, I = ctypes.c_void_p, ctypes.c_int
    lib.forward_token_c.argtypes = [I, P, P, P, P, P, P, plans.CALLBACK, P]
    lib.forward_token_c.restype = I
    lib.init_kernels()
    cores = _omp_threads(cores)
    M = plans.TokenModel(seed=0)
    cb = plans.attention_stand_in()
    states = M.fresh_states()
    lps, mps = M.plans(states)
    h = np.zeros(plans.HIDDEN, np.float32)
    tok = _token_loop(lib.forward_token_c, M, lps, mps, cb, h, 1, warmup)
    n, t0 = 0, time.perf_counter()
    while (steps is None and (n < 1 or time.perf_counter() - t0 < budget)) or (steps is not None and n < steps):
        tok = _token_loop(lib.forward_token_c, M, lps, mps, cb, h, tok, 1)
        n += 1
    return (time.perf_counter() - t0) / n * 1e3, n, cores


def run_abi(torch, dev):
    """The reference-facing drop-in as the engine calls it: 150 synchronous
    bfp8_gemv calls per token with host pointers into the (registered)
    weight image and host activations / outputs."""
    from qwen_b200 import _lib, model

    L = _lib.load()
    shapes = model.qwen35_08b_stack()
    nb = model.stack_bytes(shapes)
    hbuf, hx = synthetic_stack(shapes)
    ents = stack_views(hbuf, hx, shapes)
    L.qwen_b200_register_weights(hbuf.ctypes.data, hbuf.nbytes)

    def token():
        for y, x, m, e, M, K in ents:
            L.bfp8_gemv(y.ctypes.data, x.ctypes.data, m.ctypes.data, e.ctypes.data, M, K)

    token()
    n, t0 = 0, time.perf_counter()
    while n < 3 or (time.perf_counter() - t0 < 2.0 and n < 50):
        token()
        n += 1
    per = (time.perf_counter() - t0) / n
    L.qwen_b200_forget_weights(hbuf.ctypes.data)
    return {"value": round(nb["total"] / per / 1e9, 2), "unit": "GB/s", "ms_per_token": round(per * 1e3, 3),
            "us_per_call": round(per / len(shapes) * 1e6, 2), "tokens_timed": n,
            "config": {"workload": "150 bfp8_gemv drop-in calls per token, host pointers (the engine's ctypes "
                                   "loop, qwen_real_engine.py:1073-1087), weights registered once",
                       "algorithmic_bytes_per_step": nb["total"]},
            "h2d_bytes_per_step": 4 * sum(t.K for t in shapes), "d2h_bytes_per_step": 4 * sum(t.M for t in shapes)}


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


_INT8_PEAK = {}


def run_batched(args, torch, dist, dev, barrier, world, rank, hbm_peak, peak_kind, B, steps, warmup, e2e=True):
    """B sequences x the 0.8B linear stack, one grouped
    tcgen05 kind::i8 launch per step (150 GEMMs).  Activations enter as
    planar int16 (hi/lo int8 planes + block scales, the quantizer's output);
    outputs leave as fp32 [B][M].  Weight copies and activation sets rotate
    together (> 4 GB), so no step finds its inputs in L2."""
    from qwen_b200 import model, ops

    shapes = model.qwen35_08b_stack()
    nb = model.batched_bytes(shapes, B)
    copies = args.copies or max(2, math.ceil(L2_DEFEAT_BYTES / nb["weights"]))
    ds = model.DeviceStack(shapes, copies=copies, device=dev, seed=1234 + rank)
    db = model.DeviceBatch(shapes, B, sets=copies, device=dev, seed=77 + rank)
    plans = [ops.BatchedStack(db.items(ds.views(c), c)) for c in range(copies)]
    if dev.index not in _INT8_PEAK:
        _INT8_PEAK[dev.index] = int8_peak_tops(torch, dev)
    p_int8 = _INT8_PEAK[dev.index]

    clk = ClockSampler(gpu_uuid(torch, dev), dev.index or 0)
    secs = timed(torch, lambda i: plans[i % copies].run(), steps, warmup, barrier)
    clocks = clk.stop()
    per_step = max_over_ranks(torch, dist, secs, dev, world) / steps
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

    e2e_rec = None
    if e2e and not args.no_e2e:
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

        eper = max_over_ranks(torch, dist, timed(torch, e2e_step, steps, warmup, barrier), dev, world) / steps
        e2e_rec = {"value": round(world * nb["total"] / eper / 1e9, 2), "unit": "GB/s",
                   "ms_per_step": round(eper * 1e3, 4), "tokens_per_s": round(world * B / eper, 1),
                   "h2d_bytes_per_step": hp.numel() + hs.numel() * 4, "d2h_bytes_per_step": hy.numel() * 4}
    for p in plans:
        p.close()
    return {"value": round(world * gbs, 2), "ms_per_step": round(per_step * 1e3, 4),
            "dtype": "int8xint8->int32 (hi/lo planes)->fp32",
            "config": {"workload": f"batched decode: B={B} sequences x qwen35-0.8b linear stack (150 BFP8 GEMMs)",
                       "batch": B, "gemms_per_step": len(shapes), "weight_bytes": nb["weights"],
                       "algorithmic_bytes_per_step": nb["total"], "macs_per_step": nb["macs"] * B,
                       "tensor_int8_ops_per_step": nb["tensor_ops"], "tokens_per_s": round(world * B / per_step, 1),
                       "tops_issued_int8": round(tops, 2),
                       "l2": f"rotates {copies} weight copies + activation sets "
                             f"({copies * nb['weights'] / 1e9:.2f} GB weights) > 126 MB L2",
                       "launch": "one grouped tcgen05 kernel per step", "parallelism": f"replicas x{world}"},
            "roofline": roof, "e2e": e2e_rec, "gpu_launches": steps, "clocks": clocks}


# ------------------------------------------------------------------ multi-GPU (config 4)
def run_sharded_records(args, torch, dist, dev, barrier, world, rank, local, hbm_peak, peak_kind):
    """Config 4 beside the headline, on every N: batch 1 with the kernels'
    peer stores and with NCCL all-gathers, batch 64 with peer stores."""
    out = {}
    for key, B, ex in (("b1_peer", 1, "peer"), ("b1_nccl", 1, "nccl"), ("b64_peer", 64, "peer")):
        out[key] = run_sharded(args, torch, dist, dev, barrier, world, rank, local, hbm_peak, peak_kind, B, ex,
                               20, 3, check_parity=True)
        torch.cuda.empty_cache()
    return out


def run_sharded(args, torch, dist, dev, barrier, world, rank, local, hbm_peak, peak_kind, B, exchange, steps, warmup,
                check_parity=True):
    """8 layers x (gate, up 28672x8192; down 8192x28672),
    output rows sharded over the ranks; per layer the shard-local swiglu +
    quantizer's int16 activation and the down rows reach every GPU through
    the kernels' own peer stores (peer) or NCCL all-gathers.  Total work is
    fixed as N grows (strong scaling).  Parity: rank 0 runs the same steps
    on its own GPU alone and compares every layer's gathered activation and
    down output bit for bit (batch 1; the fast arithmetic cuts K at fixed
    steps, so the bits do not depend on N) or within 1e-4 of the output scale
    (batch 64: stream-K groups the fp32 sums by the total work)."""
    import numpy as np

    from qwen_b200 import sharded

    layers = sharded.scaled_layers()
    full_w = sum(t.M * t.K + t.M * t.K // 64 for L in layers for t in (L.gate, L.up, L.down))
    copies = args.copies or max(1, math.ceil(L2_DEFEAT_BYTES / (full_w / world)))
    st = sharded.ShardedDeviceStack(layers, world, rank, dev, copies=copies, seed=11, fast=True, exchange=exchange,
                                    batch=B)
    graphs = None
    if st.capturable():
        # every plan runs once eagerly, then every rank captures one graph
        # per weight copy (nothing runs while capturing: the barriers keep a
        # rank's replays from waiting on a peer that is still capturing)
        for c in range(copies):
            st.step(c)
        torch.cuda.synchronize()
        barrier()
        graphs = [st.capture(c) for c in range(copies)]
        torch.cuda.synchronize()
        barrier()
        step = lambda i: graphs[i % copies].replay()   # noqa: E731
    else:
        step = lambda i: st.step(i % copies)   # noqa: E731
    clk = ClockSampler(gpu_uuid(torch, dev), local)
    secs = timed(torch, step, steps, warmup, barrier)
    clocks = clk.stop()
    per_step = max_over_ranks(torch, dist, secs, dev, world) / steps
    nbytes = st.bytes_per_step()
    xbytes = st.exchange_bytes_per_step()
    err = st.device_error() if exchange == "peer" else 0
    parity = None
    if check_parity:
        torch.cuda.synchronize()
        mine = st.outputs() if B == 1 else st.final_output().cpu().numpy()
        if world == 1:
            parity = {"ok": True, "how": "one GPU: the run is its own reference"}
        elif rank == 0:
            ref = sharded.ShardedDeviceStack(layers, 1, 0, dev, copies=1, seed=11, fast=True, exchange="nccl",
                                             batch=B)
            ref.step()
            torch.cuda.synchronize()
            if B == 1:
                same = bool(np.array_equal(mine, ref.outputs()))
                parity = {"ok": same, "how": "every layer's gathered int16 activation + scales and down output "
                                             "vs one GPU, bit for bit"}
            else:
                r = ref.final_output().cpu().numpy()
                rel = float(np.max(np.abs(mine - r)) / max(np.max(np.abs(r)), 1e-30))
                parity = {"ok": rel <= 1e-4, "max_abs_diff_over_scale": rel,
                          "how": "last layer's down output vs one GPU, within 1e-4 of its scale (stream-K)"}
            ref.close()
            del ref
        barrier()
    launch_kind = ("one CUDA graph per weight copy (epochs offsets from a device counter)" if graphs is not None
                   else "eager launches from Python, NCCL between them")
    del graphs, step
    st.close()
    del st
    per_rank_gbs = nbytes / world / per_step / 1e9
    rec = {"value": round(nbytes / per_step / 1e9, 2), "unit": "GB/s", "ms_per_step": round(per_step * 1e3, 4),
           "scaling": "strong",
           "config": {"workload": f"scaled BFP8 stack: 8 x (gate/up 28672x8192, down 8192x28672), batch {B}",
                      "arithmetic": "fast (K cut at fixed 2 KB steps, fma per block; within 1e-5 of the exact order)"
                                    if B == 1 else "tcgen05 kind::i8 over hi/lo int8 planes, exact int32 block dots",
                      "algorithmic_bytes_per_step": nbytes, "weight_bytes": full_w,
                      "exchange_bytes_per_rank_per_step": xbytes,
                      "parallelism": f"output rows sharded x{world}; per layer gate/up local, swiglu + quantizer "
                                     "shard-local, int16 activation and fp32 down rows to every GPU by " + (
                                         "the kernels' NVLink stores, epoch flags between launches"
                                         if exchange == "peer" else "NCCL all-gathers"),
                      "l2": f"rotates {copies} copies of this rank's {full_w / world / 1e9:.2f} GB",
                      "launch": launch_kind},
           "roofline": {"bound": "hbm", "achieved": round(per_rank_gbs, 2), "peak": hbm_peak, "unit": "GB/s",
                        "frac": round(per_rank_gbs / hbm_peak, 4), "peak_kind": peak_kind, "traffic": None,
                        "kernel": ("gemv_warp_kernel" if B == 1 else "gemm_tc_kernel") +
                                  " per rank (per-rank GB/s incl. the exchange)"},
           # per layer: gate/up (quantizer + GEMV), activation, down (quantizer + GEMV / GEMM); NCCL not counted
           # (+ the epoch counter's advance per step with peer stores)
           "gpu_launches": steps * (len(layers) * (5 if B == 1 else 4) +
                                    (1 if exchange == "peer" and world > 1 else 0)),
           "exchange": exchange, "parity": parity, "clocks": clocks}
    if err:
        rec["device_error"] = err
    return rec


# ------------------------------------------------------------------ lm_head / rtl20
def run_lm_head(args, torch, dev, barrier, world, hbm_peak, peak_kind, workload, steps, warmup):
    """The 65536 x 1024 lm_head (bf16 table or BFP8 matrix) fused with
    argmax and top-40.  `value` times the kernels alone: each step replays a
    CUDA graph of one call per table copy (no per-call host work); `e2e`
    calls the reference-facing host API (lm_head_topk with a host h and a
    registered host table for bf16; the BFP8 device call with h copied in and
    the ids and scores copied out otherwise)."""
    import numpy as np

    from qwen_b200 import _lib, ops

    V, H, k = 65536, 1024, getattr(args, "topk", 40)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    w = torch.randn((V, H), generator=g, device=dev) * 0.02
    h = torch.randn(H, generator=g, device=dev)
    if workload == "lm_bf16":
        tab = w.to(torch.bfloat16).view(torch.int16)
        per = V * H * 2
        copies = max(2, math.ceil(L2_DEFEAT_BYTES / per))
        tabs = [tab] + [tab.clone() for _ in range(copies - 1)]
        res = ops.lm_outputs(dev, k)   # preallocated: the timed graph holds only the lm_head kernels

        def call(i):
            ops.lm_head_bf16(h, tabs[i % copies], k, out=res)
        desc = f"bf16 lm_head 65536x1024 + argmax + top-{k}"
    else:
        mant, exps = ops.pack_bfp8(w)
        per = V * H + V * H // 64
        copies = max(2, math.ceil(L2_DEFEAT_BYTES / per))
        mats = [(mant, exps)] + [(mant.clone(), exps.clone()) for _ in range(copies - 1)]
        res = ops.lm_outputs(dev, k)

        def call(i):
            m, e = mats[i % copies]
            ops.lm_head_bfp8(h, m, e, k, out=res)
        desc = f"BFP8 lm_head 65536x1024 + argmax + top-{k}"
    graph = graph_of(torch, call, copies)
    clk = ClockSampler(gpu_uuid(torch, dev), dev.index or 0)
    secs = timed(torch, lambda i: graph.replay(), steps, warmup, barrier)
    clocks = clk.stop()
    del graph
    per_step = secs / steps / copies   # one lm_head per table copy in each replay
    nbytes = per + 4 * H
    gbs = nbytes / per_step / 1e9

    L = _lib.load()
    hh = h.cpu().numpy().astype(np.float32)
    ids = np.zeros(k, np.int32)
    scs = np.zeros(k, np.float32)
    if workload == "lm_bf16":
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
    for i in range(warmup):
        e2e_call(i)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(steps):
        e2e_call(i)
    torch.cuda.synchronize()
    e2e_step = (time.perf_counter() - t0) / steps
    if workload == "lm_bf16":
        L.qwen_b200_forget_weights(host_tab.ctypes.data)
    del w
    return {"value": round(world * gbs, 2), "unit": "GB/s", "ms_per_step": round(per_step * 1e3, 4),
            "config": {"workload": desc, "algorithmic_bytes_per_step": nbytes,
                       "l2": f"rotates {copies} copies", "launch": "CUDA graph of one call per copy"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind,
                         "traffic": committed_traffic(workload)},
            "e2e": {"value": round(world * nbytes / e2e_step / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_step * 1e3, 4), "h2d_bytes_per_step": 4 * H,
                    "d2h_bytes_per_step": 8 * k + 4},
            "gpu_launches": steps * copies, "clocks": clocks}


def run_rtl20(args, torch, dev, barrier, world, hbm_peak, peak_kind):
    """Secondary line: the RTL dequant mode (gemv_core's floor(y * 2^20)
    words) of the cfg-0 GEMV, 3584 x 1024, from fp32 x.  `value` times the
    kernel alone (a CUDA graph of one call per weight copy); `exact_ms`
    times the exact-mode single GEMV entry the same way; `e2e` copies x in
    and the words out around each call."""
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


# ------------------------------------------------------------------ reference arm / CPU baseline
def _omp_threads(n):
    """Set the OpenMP team size of the reference library (libgomp reads
    OMP_NUM_THREADS once, when it loads; torchrun exports 1), and return the
    size OpenMP reports."""
    import ctypes

    try:
        gomp = ctypes.CDLL("libgomp.so.1")
        gomp.omp_set_num_threads(int(n))
        return int(gomp.omp_get_max_threads())
    except OSError:
        return int(n)


def cpu_runner(kind, workload, data_path=""):
    """(token function, shapes, description, cores) of one CPU row over the
    workload's GEMVs on the synthetic stack's bytes:
      ref       the reference's own C bfp8_gemv (oracle/_ref, built from
                04-板载脚本与工具/qwen_kernels_opt.c; x86 has no NEON, so its
                scalar float path), OpenMP with every host thread
      ref2      the same with 2 threads (the board's core count)
      numpy     the reference engine's numpy fallback (qwen_real_engine.py:
                1233-1239), restated in oracle/oracle.py and pinned to it
      oracle    the NEON-order int16 restatement (oracle/bfp8_oracle.c), one thread"""
    import ctypes

    import numpy as np

    shapes, desc = stack_shapes("stack" if workload in ("batched",) else workload)
    if data_path:
        d = np.load(data_path)
        buf, x = d["buf"], d["x"]
    else:
        buf, x = synthetic_stack(shapes)
    ents = stack_views(buf, x, shapes)
    if kind in ("ref", "ref2"):
        cores = _omp_threads(os.cpu_count() if kind == "ref" else 2)
        lib = ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libref_kernels.so"))
        P, I = ctypes.c_void_p, ctypes.c_int
        lib.bfp8_gemv.argtypes = [P, P, P, P, I, I]
        lib.bfp8_gemv.restype = None
        lib.init_kernels()
        cores = _omp_threads(cores)

        def token():
            for y, xx, m, e, M, K in ents:
                lib.bfp8_gemv(y.ctypes.data, xx.ctypes.data, m.ctypes.data, e.ctypes.data, M, K)
        label = (f"reference C bfp8_gemv (scalar build, OpenMP {cores} threads)")
        return token, shapes, desc, cores, label, buf
    from oracle import oracle as O

    if kind == "numpy":
        def token():
            for y, xx, m, e, M, K in ents:
                y[:] = O.bfp8_gemv_numpy(xx, m, e)
        return token, shapes, desc, 1, "reference engine numpy fallback (restated in oracle/)", buf

    def token():
        for y, xx, m, e, M, K in ents:
            y[:] = O.bfp8_gemv(xx, m, e)
    return token, shapes, desc, 1, "oracle: NEON-order int16 restatement, one thread", buf


def cpu_baseline(workload, batch=1, data_path=None):
    """Bounded samples of the CPU rows on this host, each in a child
    process (OpenMP starts with the thread count the row asks for)."""
    if workload == "token":
        env = dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count()))
        cmd = [sys.executable, os.path.abspath(__file__), "--impl", "reference", "--cpu-sample", "--workload", "token"]
        try:
            out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
            row = json.loads(out.stdout.strip().splitlines()[-1])
        except Exception as e:
            row = {"error": str(e)[:200]}
        row["host_cpu"] = _cpu_model()
        return row
    if workload not in ("stack", "gemv", "batched"):
        return None
    rows = []
    for kind in ("ref", "ref2", "numpy", "oracle"):
        env = dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count() if kind == "ref" else 2 if kind == "ref2" else 1))
        cmd = [sys.executable, os.path.abspath(__file__), "--impl", "reference", "--cpu-sample", "--cpu-kind", kind,
               "--workload", workload, "--batch", str(batch)]
        if data_path:
            cmd += ["--cpu-data", data_path]
        try:
            out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
            rows.append(json.loads(out.stdout.strip().splitlines()[-1]))
        except Exception as e:  # a baseline failure must not hide the GPU number
            rows.append({"kind": kind, "error": str(e)[:200]})
    main = dict(rows[0]) if rows and "value" in rows[0] else {"error": "reference row failed"}
    main["rows"] = rows
    main["host_cpu"] = _cpu_model()
    return main


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    if args.workload == "rtl20":
        print(json.dumps({"impl": "reference", "unavailable": "the RTL dequant mode exists only as FPGA fabric "
                          "(gemv_core.v); the reference has no CPU implementation of it"}))
        return
    if args.workload == "token":
        if args.cpu_sample:
            ms, n, cores = token_reference_sample(budget=10.0)
            print(json.dumps({"value": round(ms, 3), "unit": "ms/token", "cores": cores, "kind": "reference",
                              "sample": f"{n} autoregressive tokens after 1 warm-up token: the reference's "
                                        "forward_token_c (portable build, OpenMP) on plans.TokenModel(seed=0)"}))
            return
        ms, n, cores = token_reference_sample(steps=args.steps, warmup=args.warmup)
        print(json.dumps({
            "impl": "reference", "metric": TOKEN_METRIC, "value": round(ms, 3), "unit": "ms/token",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": False, "scaling": "replicas", "vs_baseline": None,
            "dtype": "fp32 (reference portable build)",
            "data": "synthetic: plans.TokenModel(seed=0), the B200 arm's model",
            "config": {"workload": "the reference's forward_token_c, 24 layers + lm_head argmax, stand-in "
                                   "attention callback"},
            "cpu_baseline": {"value": round(ms, 3), "unit": "ms/token", "cores": cores, "kind": "reference",
                             "sample": f"{n} autoregressive tokens after {args.warmup} warm-up tokens"},
            "e2e": {"value": round(ms, 3), "unit": "ms/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return
    from qwen_b200 import model

    kind = args.cpu_kind if args.cpu_sample else "ref"
    token, shapes, desc, cores, label, _buf = cpu_runner(kind, args.workload, args.cpu_data)
    nb = model.stack_bytes(shapes)
    # the reference has no batched path: B sequences cost B one-sequence passes
    seqs = args.batch if args.workload == "batched" else 1
    if seqs > 1:
        nb = model.batched_bytes(shapes, seqs)
        desc = f"batched decode: B={seqs} sequences x {desc}, one sequence at a time"
    ref_kind = "reference" if kind in ("ref", "ref2") else "port"
    if args.cpu_sample:
        # bounded sample: whole passes of the stack for ~6 s (at least 1)
        budget = 6.0
        token()
        n, t0 = 0, time.perf_counter()
        while n < 1 or (time.perf_counter() - t0 < budget and n < 1000):
            token()
            n += 1
        dt = (time.perf_counter() - t0) / n * seqs
        print(json.dumps({"value": round(nb["total"] / dt / 1e9, 4), "unit": "GB/s", "ms_per_step": round(dt * 1e3, 3),
                          "cores": cores, "kind": ref_kind, "row": kind,
                          "sample": f"{n} whole one-sequence passes of the stack after 1 warm-up pass, scaled by "
                                    f"{seqs} sequences per step ({desc}); {label}; the B200 arm's packed bytes"}))
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
        "data": "synthetic: the B200 arm's packed bytes (bench.synthetic_stack: N(0,0.02) weights, N(0,1) "
                "activations)",
        "config": {"workload": desc, "algorithmic_bytes_per_step": nb["total"]},
        "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": cores, "kind": "reference",
                         "sample": f"{args.steps} whole tokens after {args.warmup} warm-up tokens; {label}"},
        "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse()
    # the driver reads one JSON line from rank 0's stdout: keep NCCL's version
    # banner and informational lines off it unless the caller asked for them
    if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
        os.environ["NCCL_DEBUG"] = "WARN"
    if args.impl == "reference":
        if not args.cpu_sample:
            # every host thread, also under torchrun (which exports OMP_NUM_THREADS=1)
            os.environ["OMP_NUM_THREADS"] = str(os.cpu_count())
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
