"""The GEMV entry point that allocates nothing (qwen_b200_gemv_noalloc_dev).

It exists for callers that must not have a library allocate device memory
behind their back -- e.g. a serving process whose allocator already owns
nearly all of HBM, or a loop that cannot take cudaMalloc's device-wide
synchronisation.  Its scratch is a fixed array compiled into the library,
shared by every call on a device.

Only GEMVs with 6144 < K <= 16384 (K a multiple of 512) route their
activation through that array: smaller K is quantized by every CTA into its
own shared memory.  The checks below therefore call the entry point through
the C ABI on scratch-path shapes back to back -- each call starting from the
previous call's leftover scratch, which held a different activation and, for
K = 8192 after K = 16384, more words than the call rewrites -- and require the
same bits as qwen_b200_gemv_dev and the CPU oracle.  A second check runs in a
fresh process and reads the device's free memory around the calls: it must
not move.  The file sorts last so that a run stopping at its first failure
has run everything else.
"""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def bits(a):
    a = np.ascontiguousarray(a, np.float32)
    return np.where(np.isnan(a), np.uint32(0x7FC00000), a.view(np.uint32))


def test_noalloc_gemv_matches_gemv_dev_on_consecutive_calls(cuda):
    import torch

    from qwen_b200 import _lib

    lib = _lib.load()
    rng = np.random.default_rng(2026)
    stream = torch.cuda.current_stream().cuda_stream
    # small K (shared-memory activation), then the scratch path: K = 8192, a
    # deeper K = 16384 that fills the whole array, and K = 8192 again on top of
    # its leftovers; odd M on two of them
    shapes = ((3584, 1024), (1025, 3584), (1025, 8192), (3584, 16384), (513, 8192))
    for M, K in shapes:
        mant, exps = O.pack_bfp8(rng.normal(0, 0.02, (M, K)).astype(np.float32))
        dm = torch.from_numpy(mant).cuda()
        de = torch.from_numpy(exps).cuda()
        x = torch.from_numpy(rng.normal(0, 1, K).astype(np.float32)).cuda()
        y_ref = torch.empty(M, dtype=torch.float32, device="cuda")
        y = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
        assert lib.qwen_b200_gemv_dev(y_ref.data_ptr(), x.data_ptr(), dm.data_ptr(), de.data_ptr(), M, K,
                                      stream) == 0
        assert lib.qwen_b200_gemv_noalloc_dev(y.data_ptr(), x.data_ptr(), dm.data_ptr(), de.data_ptr(), M, K,
                                              stream) == 0
        torch.cuda.synchronize()
        got = bits(y.cpu().numpy())
        assert np.array_equal(got, bits(y_ref.cpu().numpy())), (M, K)
        assert np.array_equal(got, bits(O.bfp8_gemv(x.cpu().numpy(), mant, exps))), (M, K)
    assert lib.qwen_b200_device_error(1) == 0


def test_noalloc_gemv_rejects_k_beyond_its_scratch(cuda):
    from qwen_b200 import _lib

    lib = _lib.load()
    # K = 16448 > 16384: refused before any device work (pointers are never touched)
    assert lib.qwen_b200_gemv_noalloc_dev(8, 8, 8, 8, 4, 16448, None) == -1
    assert b"16384" in lib.qwen_b200_last_error()
    assert lib.qwen_b200_gemv_noalloc_dev(8, 8, 8, 8, 4, 100, None) == -1
    assert b"multiple of 64" in lib.qwen_b200_last_error()


_CHILD = textwrap.dedent(r"""
    import sys
    import numpy as np
    import torch
    sys.path[:0] = [sys.argv[1], sys.argv[2]]
    from oracle import oracle as O
    from qwen_b200 import _lib

    lib = _lib.load()
    rng = np.random.default_rng(5)
    cases = []
    for M, K in ((1024, 8192), (2048, 16384)):
        mant, exps = O.pack_bfp8(rng.normal(0, 0.02, (M, K)).astype(np.float32))
        x = rng.normal(0, 1, K).astype(np.float32)
        cases.append((M, K, torch.from_numpy(mant).cuda(), torch.from_numpy(exps).cuda(),
                      torch.from_numpy(x).cuda(), torch.empty(M, dtype=torch.float32, device="cuda"),
                      O.bfp8_gemv(x, mant, exps)))
    # the library carries its own CUDA runtime: cudaFree(NULL) through it
    # initialises that runtime, which (eager loading) loads the library's
    # device image -- code and the fixed scratch array, about 2 MB -- before
    # the first reading; a torch kernel takes the context's first-launch
    # reservations
    assert lib.qwen_b200_dev_free(None) == 0
    warm = torch.ones(1024, device="cuda") * 2
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for rep in range(3):
        for M, K, dm, de, x, y, ref in cases:
            rc = lib.qwen_b200_gemv_noalloc_dev(y.data_ptr(), x.data_ptr(), dm.data_ptr(), de.data_ptr(), M, K, None)
            assert rc == 0, lib.qwen_b200_last_error()
        torch.cuda.synchronize()
        free = torch.cuda.mem_get_info()[0]
        assert free == free0, ("device memory moved", rep, free0, free)
        for M, K, dm, de, x, y, ref in cases:
            assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32)), (rep, M, K)
    print("noalloc child ok")
""")


def test_noalloc_gemv_allocates_nothing_in_a_fresh_process(cuda):
    """Only the no-alloc entry point of the library runs in the child, so
    nothing else can have created the library's per-device buffers first.
    The library's runtime is initialised first (cudaFree(NULL), loading its
    device image eagerly) and one torch kernel runs, so the reading before
    the first call already has the library image, its fixed array and the
    context's own reservations in place."""
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER")
    pkg = os.path.join(REPO, "qwen35-ax7020-edge-llm_b200")
    out = subprocess.run([sys.executable, "-c", _CHILD, REPO, pkg], env=env, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-2000:]
    assert "noalloc child ok" in out.stdout
