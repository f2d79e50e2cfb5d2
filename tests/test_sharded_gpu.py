"""Row-sharded stack on two GPUs: at batch 1 every gathered output equals the
single-GPU run bit for bit, with the NCCL all-gather and with the in-kernel
peer stores (exchange="peer"); the fast arithmetic gives the same bits both
ways.  At batch 64 (tcgen05, stream-K: where a tile is cut between CTAs
depends on the total work, so the fp32 sums group differently) both exchanges
give the same bits and agree with one GPU to 1e-4 of the output scale.  The
two-GPU cases are skipped with fewer GPUs; the bounded flag wait runs on one."""
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
    return np.concatenate([st.full[t.name].cpu().numpy().ravel() for L in st.layers for t in (L.gate, L.up, L.down)])


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
                assert st.flags.cpu().tolist() == [6 * len(st.layers)] * world   # 2 launches x 3 steps
            st.close()
        st = sharded.ShardedDeviceStack(_layers(), world, rank, f"cuda:{rank}", copies=2, seed=4, exchange=exchange,
                                        batch=BATCH)
        for i in range(3):
            st.step(i % 2)
        torch.cuda.synchronize()
        np.save(path + f".{exchange}.b.{rank}.npy", _outputs(st))
        if exchange == "peer":
            assert st.device_error() == 0
            assert st.flags.cpu().tolist() == [6 * len(st.layers)] * world
        st.close()
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_sharded_stack_matches_single_gpu(cuda, tmp_path):
    import torch
    import torch.multiprocessing as mp

    from qwen_b200 import sharded

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    single = sharded.ShardedDeviceStack(_layers(), 1, 0, "cuda:0", copies=1, seed=4)
    single.step()
    torch.cuda.synchronize()
    ref = _outputs(single)
    single.close()
    single = sharded.ShardedDeviceStack(_layers(), 1, 0, "cuda:0", copies=1, seed=4, batch=BATCH)
    single.step()
    torch.cuda.synchronize()
    ref_b = _outputs(single)
    single.close()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    path = str(tmp_path / "out")
    mp.start_processes(_worker, args=(2, port, path), nprocs=2, join=True, start_method="spawn")
    fast_ref = np.load(path + ".nccl.1.0.npy")
    for r in range(2):
        for exchange in ("nccl", "peer"):
            got = np.load(path + f".{exchange}.0.{r}.npy")
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (exchange, r)
            got = np.load(path + f".{exchange}.1.{r}.npy")
            assert np.array_equal(got.view(np.uint32), fast_ref.view(np.uint32)), (exchange, r)
            got = np.load(path + f".{exchange}.b.{r}.npy")
            assert np.array_equal(got.view(np.uint32), np.load(path + ".nccl.b.0.npy").view(np.uint32)), \
                (exchange, "batched", r)
            assert np.max(np.abs(got - ref_b)) <= 1e-4 * np.max(np.abs(ref_b)), (exchange, "batched", r)
    np.testing.assert_allclose(fast_ref, ref, rtol=1e-4, atol=1e-4)


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
    """batch > 1 on one rank: every layer's outputs match the tcgen05 GEMM of
    the previous output computed GEMM by GEMM through ops (checks the layer
    chaining, the strided outputs and the stream-K piece sums: the same exact
    block dots, fp32 sums grouped differently), for both exchanges."""
    import torch

    from qwen_b200 import ops, sharded

    for exchange in ("nccl", "peer"):
        st = sharded.ShardedDeviceStack(_layers(), 1, 0, "cuda:0", copies=1, seed=4, batch=12, exchange=exchange)
        st.step()
        torch.cuda.synchronize()
        x = st.x0
        for L in st.layers:
            for t, xin in ((L.gate, x), (L.up, x), (L.down, None)):
                xin = xin if xin is not None else st.full[L.gate.name]
                mant, exps = st.weight(0, t)
                y = ops.bfp8_gemm_tc(ops.quant_planes(xin.contiguous()), mant, exps)
                err = (y - st.full[t.name]).abs().max().item()
                assert err <= 1e-5 * y.abs().max().item(), (exchange, t.name, err)
            x = st.full[L.down.name]
        st.close()


def test_peer_flag_wait_times_out_with_status(cuda):
    """A flag that nothing raises: the bounded wait gives up, the error word
    reports it (bit 2), the launch still completes and the context stays
    usable."""
    import torch

    from qwen_b200 import sharded

    st = sharded.ShardedDeviceStack(_layers(), 1, 0, "cuda:0", copies=1, seed=4, exchange="peer")
    st.device_error()
    gu, _ = st.plans[0][0]
    base = st.peer_base[0]
    gu.run(base, 1000, [base], 7, 0)     # waits for epoch 1000, which never comes
    torch.cuda.synchronize()
    assert st.device_error() & 2
    assert st.flags.cpu().tolist() == [7]
    st.close()
