"""GPU parity of the device sampler (qwen_b200_sample_topk_dev).

The device sampler follows the reference sampler's procedure and IEEE
float / double operation order (qwen_sampling.c:411-529) with CUDA's expf in
place of the C library's.  Its draws must equal the reference's except where
a draw lands within a few ulps of a bucket boundary: such a draw may pick a
neighbouring candidate, so at most 1 in 1000 draws may differ and only by
one place in the sorted list.  The xorshift32 state must advance exactly.
The checkers are the compiled reference's recorded draws
(tests/golden/sampler.npz) and the library's host sample_from_topk, which
the CPU tests pin to those draws.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def to_dev(*arrs):
    import torch

    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]


def dev_state(st):
    import torch

    return torch.from_numpy(np.array([st], np.uint32).view(np.int32)).cuda()


def device_draws(ids, sc, t, tk, tp, st0, draws):
    """`draws` successive device samples from one list with a chained state."""
    import torch

    from qwen_b200 import ops

    d_ids, d_sc = to_dev(ids.astype(np.int32), sc.astype(np.float32))
    state = dev_state(st0)
    outs = torch.empty(draws, dtype=torch.int32, device=d_ids.device)
    for j in range(draws):
        ops.sample_topk(d_ids, d_sc, t, tk, tp, state, out=outs[j:j + 1])
    return outs.cpu().tolist(), int(state.cpu().numpy().view(np.uint32)[0])


def host_draws(ids, sc, t, tk, tp, st0, draws):
    from qwen_b200 import _lib

    lib = _lib.load()
    ids = np.ascontiguousarray(ids, np.int32)
    sc = np.ascontiguousarray(sc, np.float32)
    st = ctypes.c_uint(st0)
    out = [lib.sample_from_topk(ids.ctypes.data, sc.ctypes.data, len(ids), float(t), int(tk), float(tp),
                                ctypes.byref(st)) for _ in range(draws)]
    return out, st.value


def sorted_order(ids, sc):
    """Candidate ids in the sampler's order: score descending, id ascending."""
    return [int(ids[i]) for i in sorted(range(len(ids)), key=lambda i: (-float(sc[i]), int(ids[i])))]


class Tally:
    def __init__(self):
        self.draws = 0
        self.diffs = 0

    def check(self, ids, sc, got, want):
        order = sorted_order(ids, sc)
        for g, w in zip(got, want):
            self.draws += 1
            if g != w:
                self.diffs += 1
                assert abs(order.index(g) - order.index(w)) == 1, (g, w)

    def done(self):
        assert self.diffs <= self.draws // 1000, (self.diffs, self.draws)


def test_sampler_matches_reference_draws(cuda, golden):
    """The compiled reference's recorded draws and final rng states."""
    g = golden("sampler.npz")
    tally = Tally()
    for i in range(int(g["n_cases"])):
        ids, sc = g[f"{i}_ids"], g[f"{i}_scores"]
        t, tk, tp = g[f"{i}_args"]
        st0, st1 = (int(v) for v in g[f"{i}_state"])
        got, st = device_draws(ids, sc, float(t), int(tk), float(tp), st0, 25)
        tally.check(ids, sc, got, g[f"{i}_draws"].tolist())
        assert st == st1, i
    tally.done()


def test_sampler_sweep_against_host(cuda):
    """Lists of 1..1024 candidates (sorted, shuffled, with tied scores) over
    temperatures, top-k and top-p values incl. the clamped and NaN ones."""
    rng = np.random.default_rng(11)
    tally = Tally()
    for n in (1, 5, 40, 64, 1024):
        for case in range(3):
            sc = np.sort(rng.normal(0, 3, n).astype(np.float32))[::-1].copy()
            if case == 2 and n >= 5:
                sc[1:4] = sc[1]                               # tied scores: ids decide
            ids = rng.permutation(65536)[:n].astype(np.int32)
            if case == 1:                                     # unsorted input
                p = rng.permutation(n)
                ids, sc = ids[p], sc[p]
            for t in (0.0, 0.5, 1.0, 2.0):
                for tk in (0, 1, 10, 50):
                    for tp in (-1.0, 0.0, 0.3, 0.9, 1.0, 1.5, float("nan")):
                        st0 = int(rng.integers(0, 2**32))
                        got, st = device_draws(ids, sc, t, tk, tp, st0, 8)
                        want, st_h = host_draws(ids, sc, t, tk, tp, st0, 8)
                        tally.check(ids, sc, got, want)
                        assert st == st_h
    tally.done()


def test_sampler_edge_cases(cuda):
    import torch

    from qwen_b200 import ops

    ids = np.array([30, 10, 20], np.int32)
    sc = np.array([-1.0, 2.0, 0.5], np.float32)   # unsorted
    d_ids, d_sc = to_dev(ids, sc)
    # no rng state: the first id as given (before any sort), as the reference
    assert ops.sample_topk(d_ids, d_sc, 1.0, 0, 1.0, None).item() == 30
    # greedy: the best candidate of the sorted list; the state is not touched
    st = dev_state(0x1234)
    assert ops.sample_topk(d_ids, d_sc, 0.0, 0, 1.0, st).item() == 10
    assert int(st.cpu().numpy().view(np.uint32)[0]) == 0x1234
    # a zero state is remapped, not stuck
    st = dev_state(0)
    ops.sample_topk(d_ids, d_sc, 1.0, 0, 1.0, st)
    assert int(st.cpu().numpy().view(np.uint32)[0]) != 0
    # the device count limits the list; an empty list gives -1
    n0 = torch.zeros(1, dtype=torch.int32, device=d_ids.device)
    assert ops.sample_topk(d_ids, d_sc, 1.0, 0, 1.0, dev_state(5), n=n0).item() == -1
    n1 = torch.ones(1, dtype=torch.int32, device=d_ids.device)
    assert ops.sample_topk(d_ids, d_sc, 1.0, 0, 1.0, dev_state(5), n=n1).item() == 30


def test_lm_head_then_device_sampler(cuda):
    """The fused pipeline: BFP8 lm_head top-40 on the device, then the
    device sampler on its ids / scores / count, against the host sampler on
    the same list copied out."""
    import torch

    from qwen_b200 import ops

    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    w = torch.randn((8192, 1024), generator=g, device="cuda") * 0.02
    mant, exps = ops.pack_bfp8(w)
    tally = Tally()
    for seed in range(6):
        h = torch.randn(1024, generator=g, device="cuda")
        r = ops.lm_head_bfp8(h, mant, exps, 40)
        state = dev_state(0x9000 + seed)
        outs = [ops.sample_topk(r.ids, r.scores, 0.8, 40, 0.95, state, n=r.n).item() for _ in range(20)]
        _, hid, hsc = r.host()
        want, st_h = host_draws(np.array(hid), np.array(hsc), 0.8, 40, 0.95, 0x9000 + seed, 20)
        tally.check(np.array(hid), np.array(hsc, np.float32), outs, want)
        assert int(state.cpu().numpy().view(np.uint32)[0]) == st_h
    tally.done()
