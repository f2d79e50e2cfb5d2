"""The GEMV entry point that allocates nothing (qwen_b200_gemv_noalloc_dev).

It exists for callers that must not have a library allocate device memory
behind their back -- e.g. a serving process whose allocator already owns
nearly all of HBM, or a loop that cannot take cudaMalloc's device-wide
synchronisation.  Its scratch is a fixed array compiled into the library,
shared by every call on a device.  These checks call it through the C ABI
twice in a row (so the second call starts from the first call's leftover
scratch) and require the same bits as qwen_b200_gemv_dev.  The file sorts
last so that a run stopping at its first failure has run everything else.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def bits(a):
    a = np.ascontiguousarray(a, np.float32)
    return np.where(np.isnan(a), np.uint32(0x7FC00000), a.view(np.uint32))


def test_noalloc_gemv_matches_gemv_dev_twice(cuda):
    import torch

    from qwen_b200 import _lib

    lib = _lib.load()
    rng = np.random.default_rng(2026)
    stream = torch.cuda.current_stream().cuda_stream
    for M, K in ((3584, 1024), (1025, 3584)):   # second call: other shape, odd M, more scratch
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
        assert np.array_equal(bits(y.cpu().numpy()), bits(y_ref.cpu().numpy())), (M, K)
        assert np.array_equal(bits(y.cpu().numpy()), bits(O.bfp8_gemv(x.cpu().numpy(), mant, exps))), (M, K)


def test_noalloc_gemv_rejects_k_beyond_its_scratch(cuda):
    from qwen_b200 import _lib

    lib = _lib.load()
    # K = 16448 > 16384: refused before any device work (pointers are never touched)
    assert lib.qwen_b200_gemv_noalloc_dev(8, 8, 8, 8, 4, 16448, None) == -1
    assert lib.qwen_b200_gemv_noalloc_dev(8, 8, 8, 8, 4, 100, None) == -1
