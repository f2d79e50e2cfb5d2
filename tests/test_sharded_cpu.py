"""Host logic of the row-sharded multi-GPU stack, on CPU: shard planning and
the data flow (gate / up slices, shard-local swiglu + quantizer, gathered
int16 activation, down slices, gathered down rows), run as world_size-2 gloo
ranks with the oracle standing in for the kernels; results must equal a
single-rank run bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qwen_b200 import model, sharded


def test_shard_rows_cover_and_align():
    for M in (64, 512, 3584, 28672, 8192, 100, 1):
        for world in (1, 2, 3, 4, 8):
            prev = 0
            for r in range(world):
                r0, r1 = sharded.shard_rows(M, world, r)
                assert r0 == prev and r1 >= r0
                assert r0 % 64 == 0
                prev = r1
            assert prev == M


def small_layers():
    return sharded.scaled_layers(layers=2, hidden=512, ffn=1024)


def weights(layers):
    from oracle import oracle as O

    rng = np.random.default_rng(11)
    W = {}
    for L in layers:
        for t in (L.gate, L.up, L.down):
            W[t.name] = O.pack_bfp8(rng.normal(0, 0.02, (t.M, t.K)).astype(np.float32))
    return W


def flow(world, rank, gather):
    from oracle import oracle as O

    layers = small_layers()
    W = weights(layers)
    x0 = np.random.default_rng(3).normal(0, 1, layers[0].gate.K).astype(np.float32)

    def gemv(name, x, r0, r1):
        m, e = W[name]
        return O.bfp8_gemv(x, m[r0:r1], e[r0:r1])

    def act_quant(g, u):
        return O.quant_x(O.swiglu(g, u, neon=True))

    def gemv_q(name, xq, xs, r0, r1):
        m, e = W[name]
        return O.bfp8_gemv_q(xq, xs, m[r0:r1], e[r0:r1])

    return sharded.run_layers(layers, x0, gemv, act_quant, gemv_q, gather, world, rank)


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)

    def gather(part):
        parts = [None] * world
        dist.all_gather_object(parts, part)
        return np.concatenate(parts)

    outs = flow(world, rank, gather)
    np.save(out_path + f".{rank}.npy", np.concatenate([o.view(np.uint8) for o in outs]))
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_two_rank_gloo_flow_matches_single_rank(tmp_path):
    """The shard-local swiglu + quantizer, the gathered int16 activation and
    the down rows: every gathered value equals the single-rank flow's."""
    single = np.concatenate([o.view(np.uint8) for o in flow(1, 0, lambda part: part)])
    path = str(tmp_path / "out")
    mp.start_processes(_worker, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        got = np.load(path + f".{r}.npy")
        assert np.array_equal(got, single), r
