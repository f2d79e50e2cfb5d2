"""Row-sharded stack on two GPUs (NCCL): every gathered output equals the
single-GPU run bit for bit.  Needs two GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _layers():
    from qwen_b200 import sharded

    return sharded.scaled_layers(layers=2, hidden=1024, ffn=3584)


def _outputs(st):
    return np.concatenate([st.full[t.name].cpu().numpy() for L in st.layers for t in (L.gate, L.up, L.down)])


def _worker(rank, world, port, path):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from qwen_b200 import sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    st = sharded.ShardedDeviceStack(_layers(), world, rank, f"cuda:{rank}", copies=1, seed=4)
    for _ in range(2):
        st.step()
    torch.cuda.synchronize()
    np.save(path + f".{rank}.npy", _outputs(st))
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
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    path = str(tmp_path / "out")
    mp.start_processes(_worker, args=(2, port, path), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        got = np.load(path + f".{r}.npy")
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), r
