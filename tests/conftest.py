import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "qwen35-ax7020-edge-llm_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        return np.load(os.path.join(GOLDEN, name))

    return load


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwen_b200 import _lib

    _lib.load()   # the kernel library must load on a GPU box
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def rtl_case():
    """Inputs for the RTL dequant mode: random int8 mantissas and int16
    activations, block scales xs with exponents in [-30, 9] (plus, with
    specials, a zero, a subnormal, an inf, a NaN and a negative xs), and
    weight exponents chosen so that sh = Ex + e - 110 is uniform in
    [sh_lo, sh_hi] where e stays within 0..255."""
    import numpy as np

    def make(rng, M, K, sh_lo, sh_hi, specials=False):
        nb = K // 64
        mant = rng.integers(-128, 128, (M, K)).astype(np.int8)
        xq = rng.integers(-16384, 16385, K).astype(np.int16)
        ex = rng.integers(-30, 10, nb)
        bits = ((ex + 127) << 23) | rng.integers(0, 1 << 23, nb)
        ex_eff = ex.copy()
        if specials and nb >= 5:
            bits[0], ex_eff[0] = 0, 0                          # zero
            bits[1], ex_eff[1] = 0x00012345, 0                 # subnormal
            bits[2], ex_eff[2] = 0x7F800000, 0                 # inf
            bits[3], ex_eff[3] = 0x7FC00001, 0                 # NaN
            bits[4] |= 0x80000000                              # negative: the sign bit is ignored
        xs = bits.astype(np.uint32).view(np.float32)
        sh = rng.integers(sh_lo, sh_hi + 1, (M, nb))
        exps = np.clip(sh + 110 - ex_eff[None, :], 0, 255).astype(np.uint8)
        return mant, exps, xq, xs

    return make
