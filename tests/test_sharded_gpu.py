"""Row-sharded MLP stack.  On two GPUs: at batch 1 every layer's complete
quantized activation and down output equal the single-GPU run bit for bit,
with NCCL all-gathers and with the in-kernel peer stores (exchange="peer"),
in the exact and the fast arithmetic (whose K segments are cut at fixed
steps, so they do not depend on the GPU count).  At batch 64 (tcgen05,
stream-K: where a tile is cut between CTAs depends on the total work, so the
fp32 sums group differently) both exchanges give the same bits and agree with
one GPU to 1e-4 of the output scale.  The two-GPU cases are skipped with fewer
GPUs; the shard-local activation kernel, its signal / wait and the bounded
flag wait are checked on one."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _layers():
    from qwen_b200 import sharded

    return sharded.scaled_layers(layers=2, hidden=1024, ffn=3584)


BATCH = 64   # the batched row of the multi-GPU configuration


def _outputs(st):
    return st.outputs()


def _worker(rank, world, port, path):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from qwen_b200 import sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    for exchange in ("nccl", "peer"):
        for fast in (False, True):
            st = sharded.ShardedDeviceStack(_layers(), world, rank, f"cuda:{rank}", copies=2, seed=4, fast=fast,
                                            exchange=exchange)
            for i in range(3):
                st.step(i % 2)
            torch.cuda.synchronize()
            np.save(path + f".{exchange}.{int(fast)}.{rank}.npy", _outputs(st))
            if exchange == "peer":
                assert st.device_error() == 0
                # epochs start at 1; 2 signals per layer and step, 3 steps
                assert st.flags.cpu().tolist() == [6 * len(st.layers) + 1] * world
                assert st.counter.cpu().tolist() == [6 * len(st.layers)]
                if fast:
                    # one CUDA graph per copy, replayed after the eager steps:
                    # the epochs come from the counter, so replays stay ordered
                    graphs = [st.capture(c) for c in range(2)]
                    torch.cuda.synchronize()
                    dist.barrier()
                    for i in range(3):
                        graphs[i % 2].replay()
                    torch.cuda.synchronize()
                    np.save(path + f".graph.{rank}.npy", _outputs(st))
                    assert st.device_error() == 0
                    assert st.flags.cpu().tolist() == [12 * len(st.layers) + 1] * world
                    del graphs
            st.close()
        st = sharded.ShardedDeviceStack(_layers(), world, rank, f"cuda:{rank}", copies=2, seed=4, exchange=exchange,
                                        batch=BATCH)
        for i in range(3):
            st.step(i % 2)
        torch.cuda.synchronize()
        np.save(path + f".{exchange}.b.{rank}.npy", _outputs(st))
        np.save(path + f".{exchange}.bf.{rank}.npy", st.final_output().cpu().numpy())
        if exchange == "peer":
            assert st.device_error() == 0
            assert st.flags.cpu().tolist() == [6 * len(st.layers) + 1] * world
        st.close()
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_sharded_stack_matches_single_gpu(cuda, tmp_path):
    import torch
    import torch.multiprocessing as mp

    from qwen_b200 import sharded

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ref = {}
    for fast in (False, True):
        single = sharded.ShardedDeviceStack(_layers(), 1, 0, "cuda:0", copies=1, seed=4, fast=fast)
        single.step()
        torch.cuda.synchronize()
        ref[fast] = _outputs(single)
        single.close()
    single = sharded.ShardedDeviceStack(_layers(), 1, 0, "cuda:0", copies=1, seed=4, batch=BATCH)
    single.step()
    torch.cuda.synchronize()
    ref_b = single.final_output().cpu().numpy()
    single.close()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    path = str(tmp_path / "out")
    mp.start_processes(_worker, args=(2, port, path), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        for exchange in ("nccl", "peer"):
            for fast in (False, True):
                got = np.load(path + f".{exchange}.{int(fast)}.{r}.npy")
                assert np.array_equal(got, ref[fast]), (exchange, fast, r)
            got = np.load(path + f".{exchange}.b.{r}.npy")
            assert np.array_equal(got, np.load(path + ".nccl.b.0.npy")), (exchange, "batched", r)
            fin = np.load(path + f".{exchange}.bf.{r}.npy")
            assert np.max(np.abs(fin - ref_b)) <= 1e-4 * np.max(np.abs(ref_b)), (exchange, "batched", r)
        assert np.array_equal(np.load(path + f".graph.{r}.npy"), ref[True]), ("graph replay", r)


def test_peer_mode_single_rank_matches_plain(cuda):
    """exchange="peer" on one rank (no mappings, no flags needed): the same
    bits as the plain stack."""
    import torch

    from qwen_b200 import sharded

    a = sharded.ShardedDeviceStack(_layers(), 1, 0, "cuda:0", copies=1, seed=4)
    b = sharded.ShardedDeviceStack(_layers(), 1, 0, "cuda:0", copies=1, seed=4, exchange="peer")
    a.step()
    b.step()
    b.step()
    torch.cuda.synchronize()
    assert np.array_equal(_outputs(a).view(np.uint32), _outputs(b).view(np.uint32))
    assert b.flags.cpu().tolist() == [0]
    assert b.device_error() == 0
    a.close()
    b.close()


def test_batched_single_rank_chains_layers(cuda):
    """batch > 1 on one rank: every layer's gate / up outputs match the
    tcgen05 GEMM of the layer input computed GEMM by GEMM through ops, its
    quantized activation equals the oracle's swiglu + quantizer of those
    outputs bit for bit, and its down output matches the GEMM of that
    activation (checks the layer chaining, the strided outputs, the planar
    record and the stream-K piece sums: the same exact block dots, fp32 sums
    grouped differently), for both exchanges."""
    import torch

    from oracle import oracle as O
    from qwen_b200 import ops, sharded

    for exchange in ("nccl", "peer"):
        st = sharded.ShardedDeviceStack(_layers(), 1, 0, "cuda:0", copies=1, seed=4, batch=12, exchange=exchange)
        st.step()
        torch.cuda.synchronize()
        x = st.x0
        for i, L in enumerate(st.layers):
            for t in (L.gate, L.up):
                y = ops.bfp8_gemm_tc(ops.quant_planes(x.contiguous()), *st.weight(0, t))
                err = (y - st.gu[t.name]).abs().max().item()
                assert err <= 1e-5 * y.abs().max().item(), (exchange, t.name, err)
            p = ops.planes_view(st.dq[i], st.B, L.down.K, st.ldxs)
            g, u = st.gu[L.gate.name].cpu().numpy(), st.gu[L.up.name].cpu().numpy()
            xq = p.xq().cpu().numpy()
            xs = p.xs().cpu().numpy()
            for b in range(st.B):
                rq, rs = O.quant_x(O.swiglu(g[b], u[b], neon=True))
                assert np.array_equal(xq[b], rq) and np.array_equal(xs[b].view(np.uint32), rs.view(np.uint32)), b
            y = ops.bfp8_gemm_tc(p, *st.weight(0, L.down))
            err = (y - st.full[L.down.name]).abs().max().item()
            assert err <= 1e-5 * y.abs().max().item(), (exchange, L.down.name, err)
            x = st.full[L.down.name]
        st.close()


def test_swiglu_quant_sharded_matches_oracle(cuda):
    """The shard-local activation kernel on one GPU: a slice [col0, col0 + n)
    of gate / up into two destination records (the local one and a stand-in
    for a peer's), in the quantized-record layout (batch 1) and the planar
    layout (batch 5): equal to the oracle's swiglu + quantizer of the slice,
    bytes outside the slice untouched; with a signal epoch on a one-rank
    world the kernel publishes it and its wait returns at once."""
    import torch

    from oracle import oracle as O
    from qwen_b200 import ops

    rng = np.random.default_rng(8)
    K, col0, n = 3584, 1024, 1536
    dev = torch.device("cuda:0")
    g = torch.from_numpy(rng.normal(0, 3, K).astype(np.float32)).to(dev)
    u = torch.from_numpy(rng.normal(0, 1, K).astype(np.float32)).to(dev)
    recs = [torch.full((ops.quant_record_bytes(K),), 0x5A, dtype=torch.uint8, device=dev) for _ in range(2)]
    flags = torch.zeros(64, dtype=torch.int32, device=dev)
    base = flags.data_ptr()
    ops.swiglu_quant_sharded(g.data_ptr() + 4 * col0, u.data_ptr() + 4 * col0, 1, n, K, col0, K, False, 1,
                             [r.data_ptr() for r in recs], sig_flags=[base], sig_ticket=base + 128, sig_epoch=3,
                             wait_flags=base, world=1, rank=0)
    torch.cuda.synchronize()
    rq, rs = O.quant_x(O.swiglu(g.cpu().numpy()[col0:col0 + n], u.cpu().numpy()[col0:col0 + n], neon=True))
    for r in recs:
        h = r.cpu().numpy()
        xq = h[:2 * K].view(np.int16)
        xs = h[2 * K:].view(np.float32)
        assert np.array_equal(xq[col0:col0 + n], rq)
        assert np.array_equal(xs[col0 // 64:(col0 + n) // 64].view(np.uint32), rs.view(np.uint32))
        assert (h[:2 * col0] == 0x5A).all() and (h[2 * (col0 + n):2 * K] == 0x5A).all()
    assert flags[0].item() == 3 and flags[32].item() == 0   # published; the ticket word left zero
    B, ldxs = 5, 8
    G = torch.from_numpy(rng.normal(0, 3, (B, K)).astype(np.float32)).to(dev)
    U = torch.from_numpy(rng.normal(0, 1, (B, K)).astype(np.float32)).to(dev)
    rec = torch.zeros(ops.planes_record_bytes(B, K, ldxs), dtype=torch.uint8, device=dev)
    ops.swiglu_quant_sharded(G.data_ptr() + 4 * col0, U.data_ptr() + 4 * col0, B, n, K, col0, K, True, ldxs,
                             [rec.data_ptr()])
    torch.cuda.synchronize()
    p = ops.planes_view(rec, B, K, ldxs)
    xq, xs = p.xq().cpu().numpy(), p.xs().cpu().numpy()
    for b in range(B):
        rq, rs = O.quant_x(O.swiglu(G[b].cpu().numpy()[col0:col0 + n], U[b].cpu().numpy()[col0:col0 + n], neon=True))
        assert np.array_equal(xq[b, col0:col0 + n], rq), b
        assert np.array_equal(xs[b, col0 // 64:(col0 + n) // 64].view(np.uint32), rs.view(np.uint32)), b
        assert (xq[b, :col0] == 0).all() and (xq[b, col0 + n:] == 0).all()
    from qwen_b200 import _lib

    assert _lib.load().qwen_b200_device_error(1) == 0


def test_peer_flag_wait_times_out_with_status(cuda):
    """A flag that nothing raises: the bounded wait gives up, the error word
    reports it (bit 2), the launch still completes and the context stays
    usable."""
    import torch

    from qwen_b200 import sharded

    st = sharded.ShardedDeviceStack(_layers(), 1, 0, "cuda:0", copies=1, seed=4, exchange="peer")
    st.device_error()
    gu, _ = st.plans[0][0]
    gu.run_wait(st.peer_base[0], 1000, 1)     # waits for epoch 1000, which never comes
    torch.cuda.synchronize()
    assert st.device_error() & 2
    assert st.flags.cpu().tolist() == [0]
    st.step()                                 # the context is still usable
    torch.cuda.synchronize()
    assert st.device_error() == 0
    st.close()


def test_epoch_counter_graph_replays(cuda):
    """Epochs as offsets from a device counter: a captured graph of (a
    GEMV that waits for offset 1 and publishes offset 2; counter += 1)
    publishes a fresh epoch on every replay, its rows equal the same GEMV
    in a plain stack, and with the counter unset the epochs are absolute
    again."""
    import torch

    from oracle import oracle as O
    from qwen_b200 import ops

    rng = np.random.default_rng(3)
    M, K = 256, 1024
    mant, exps = O.pack_bfp8(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    dev = torch.device("cuda:0")
    x = torch.from_numpy(rng.normal(0, 1, K).astype(np.float32)).to(dev)
    m, e = torch.from_numpy(mant).to(dev), torch.from_numpy(exps).to(dev)
    y = torch.zeros(M, dtype=torch.float32, device=dev)
    region = ops.PeerRegion(256)
    flags, counter = region.uints(0, 1), region.uints(192, 1)
    flags.fill_(1)
    stack = ops.ShardedLinearStack([(x, m, e, y)], [[]], [0], 1, fast=True)
    base = region.ptr + 192

    def step():
        ops.sync_epoch_base(base)
        try:
            stack.run(region.ptr, 1, [region.ptr], 2, 0)
            ops.sync_epoch_advance(base, 1)
        finally:
            ops.sync_epoch_base(None)

    lib = ops.load()
    lib.qwen_b200_device_error(1)
    step()                                    # eager: waits for 0 + 1, publishes 0 + 2
    torch.cuda.synchronize()
    assert flags.cpu().tolist() == [2] and counter.cpu().tolist() == [1]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for i in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert flags.cpu().tolist() == [5] and counter.cpu().tolist() == [4]
    assert lib.qwen_b200_device_error(1) == 0
    y2 = torch.zeros_like(y)
    plain = ops.LinearStack([(x, m, e, y2)], fast=True)
    plain.run()
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    plain.close()
    stack.run(region.ptr, 5, [region.ptr], 9, 0)   # counter unset: absolute epochs
    torch.cuda.synchronize()
    assert flags.cpu().tolist() == [9] and counter.cpu().tolist() == [4]
    assert lib.qwen_b200_device_error(1) == 0
    del g
    stack.close()
    region.close()
