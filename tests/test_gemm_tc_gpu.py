"""GPU parity of the batched tensor-core path (tcgen05 kind::i8) against the
CPU oracle.

* quant_planes: 256*hi + lo equals the reference quantizer's xq bit for bit,
  and the block scales match bit for bit.
* every per-block int32 dot product the tensor cores form (hi and lo planes
  recombined) equals the oracle's exact dot -- bit-exact;
* every fp32 output is within the rounding bound of its own arithmetic of
  the exact value sum_b dot_b * 2^(e_b-134) * xs_b (float64 from the exact
  dots): (nb + 1) * 2^-24 * sum_b |term_b|, one rounding per block;
* and within 1e-5 * sum_{b,j} |float(L_j) * 2^(e_b-134) * xs_b| of the
  reference's NEON-order result, where L_j are the reference's four
  lane-class partial dots: that sum scales the reference's own rounding
  (its lane partials can be far larger than the block dot they add up to);
  at least 97.5% of the outputs are also within 1e-5 * |reference| (the
  plain relative statistic, 98.3-99.7% measured: the rest are rows whose
  terms cancel, where a relative error says little);
* a grouped launch (stream-K: tiles may be cut between CTAs, the pieces'
  fp32 sums added in K order) stays within the same bounds with one more
  rounding per piece, and gives the same bits as single launches where no
  tile is cut.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def bits(a):
    a = np.ascontiguousarray(a, np.float32)
    return np.where(np.isnan(a), np.uint32(0x7FC00000), a.view(np.uint32))


def rand_weights(rng, M, K, std=0.02):
    return O.pack_bfp8(rng.normal(0, std, (M, K)).astype(np.float32))


class Rows:
    """Oracle view of a batch: reference outputs (NEON order), exact block
    dots, exact outputs and the two term magnitudes, per (row, output)."""

    def __init__(self, x, mant, exps):
        B = x.shape[0]
        M, K = mant.shape
        self.nb = K // 64
        self.ref = np.zeros((B, M), np.float32)
        self.dots = np.zeros((B, M, K // 64), np.int32)
        self.exact = np.zeros((B, M), np.float64)
        self.mag = np.zeros((B, M), np.float64)        # sum_b |dot_b * S * xs|
        self.mag_lane = np.zeros((B, M), np.float64)   # sum_{b,j} |L_j * S * xs|
        scale = np.ldexp(1.0, exps.astype(np.int64) - 134)
        for b in range(B):
            xq, xs = O.quant_x(x[b])
            lanes = O.lane_dots(mant, xq).astype(np.float64)
            d = O.block_dots(mant, xq)
            sx = scale * xs.astype(np.float64)
            self.dots[b] = d
            self.ref[b] = O.bfp8_gemv(x[b], mant, exps)
            self.exact[b] = (d.astype(np.float64) * sx).sum(axis=1)
            self.mag[b] = (np.abs(d.astype(np.float64)) * sx).sum(axis=1)
            self.mag_lane[b] = (np.abs(lanes).sum(axis=2) * sx).sum(axis=1)

    def check(self, y, what, extra_roundings=0):
        y = y.astype(np.float64)
        bound = (self.nb + 1 + extra_roundings) * 2.0 ** -24 * self.mag + 1e-30
        e1 = np.abs(y - self.exact)
        assert (e1 <= bound).all(), (what, "vs exact", float((e1 / bound).max()))
        tol = 1e-5 * self.mag_lane + 1e-30
        e2 = np.abs(y - self.ref.astype(np.float64))
        assert (e2 <= tol).all(), (what, "vs reference", float((e2 / tol).max()))
        # the plain relative statistic: the share of outputs within 1e-5 * |ref|
        # (outputs whose lane partials cancel to a tiny |ref| can miss it while
        # meeting the bound above) and the worst relative error
        rel = e2 / np.maximum(np.abs(self.ref.astype(np.float64)), 1e-30)
        share = float((rel <= 1e-5).mean())
        self.stats = {"share_within_1e-5_rel": share, "worst_rel": float(rel.max())}
        print("relative statistic", what, self.stats)   # shown with pytest -s
        assert share >= 0.975, (what, self.stats)
        return self.stats


def test_quant_planes_bit_exact(cuda):
    import torch

    from qwen_b200 import ops

    rng = np.random.default_rng(5)
    for B, K in ((1, 64), (5, 1024), (8, 3584), (33, 64 * 37)):
        x = rng.normal(0, 1, (B, K)).astype(np.float32)
        x[0, :64] = 0.0
        if B > 1:
            x[1, 64:128] = 1e-22
        if B > 2 and K >= 256:
            x[2, 128:192] = rng.normal(0, 1e4, 64)
            x[2, 192:256] = np.arange(64, dtype=np.float32) * 0.5 - 16
        p = ops.quant_planes(torch.from_numpy(x).cuda())
        xq = p.xq().cpu().numpy()
        xs = p.xs().cpu().numpy()
        for r in range(B):
            q_ref, s_ref = O.quant_x(x[r])
            assert np.array_equal(xq[r], q_ref), (B, K, r)
            assert np.array_equal(bits(xs[r]), bits(s_ref)), (B, K, r)
        hi = p.planes[0].cpu().numpy().astype(np.int32)
        assert hi.min() >= -64 and hi.max() <= 64


TC_SHAPES = [(128, 128, 8), (200, 1088, 5), (64, 512, 1), (1000, 1024, 16), (3584, 1024, 32), (512, 2048, 64),
             (1024, 3584, 128), (520, 2048, 256), (300, 640, 100)]


@pytest.mark.parametrize("M,K,B", TC_SHAPES)
def test_gemm_tc_dots_exact_and_outputs_within_tolerance(cuda, M, K, B):
    import torch

    from qwen_b200 import ops

    rng = np.random.default_rng(M * 7 + K + B)
    mant, exps = rand_weights(rng, M, K)
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    x[0, 64:128] = 0.0   # a zero block
    p = ops.quant_planes(torch.from_numpy(x).cuda())
    dm = torch.from_numpy(mant).cuda()
    de = torch.from_numpy(exps).cuda()
    y, d = ops.bfp8_gemm_tc(p, dm, de, dots=True)
    y2 = ops.bfp8_gemm_tc(p, dm, de)
    torch.cuda.synchronize()
    y, d, y2 = y.cpu().numpy(), d.cpu().numpy(), y2.cpu().numpy()
    rows = Rows(x, mant, exps)
    assert np.array_equal(d, rows.dots), (M, K, B)
    assert np.array_equal(bits(y), bits(y2))              # the dots variant computes the same floats
    rows.check(y, (M, K, B))


def test_gemm_tc_extreme_weights_exact_dots(cuda):
    """Full-range mantissas (-128..127 bytes, i.e. -127..127 plus -128) and
    activations at the +-16384 rails: the hi/lo split still gives exact dots."""
    import torch

    from qwen_b200 import ops

    rng = np.random.default_rng(99)
    M, K, B = 256, 1024, 32
    mant = rng.integers(-128, 128, (M, K)).astype(np.int8)
    mant[0, :] = -128
    mant[1, :] = 127
    exps = rng.integers(100, 140, (M, K // 64)).astype(np.uint8)
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    x[0] = np.sign(rng.normal(0, 1, K)).astype(np.float32)        # every element at +-amax -> xq = +-16384
    x[1] = -np.abs(x[1])
    p = ops.quant_planes(torch.from_numpy(x).cuda())
    _, d = ops.bfp8_gemm_tc(p, torch.from_numpy(mant).cuda(), torch.from_numpy(exps).cuda(), dots=True)
    assert np.array_equal(d.cpu().numpy(), Rows(x, mant, exps).dots)


def test_batched_stack_matches_single_launches(cuda):
    import torch

    from qwen_b200 import ops

    rng = np.random.default_rng(17)
    B = 32
    shapes = [(3584, 1024), (1024, 3584), (512, 1024), (6144, 1024), (1024, 2048)]
    items, host = [], []
    for M, K in shapes:
        mant, exps = rand_weights(rng, M, K)
        dm, de = torch.from_numpy(mant).cuda(), torch.from_numpy(exps).cuda()
        x = rng.normal(0, 1, (B, K)).astype(np.float32)
        p = ops.quant_planes(torch.from_numpy(x).cuda())
        y = torch.full((B, M), float("nan"), device="cuda")
        items.append((p, dm, de, y))
        host.append((x, mant, exps))
    st = ops.BatchedStack(items)
    st.run()
    first = [it[3].cpu().numpy().copy() for it in items]
    st.run()   # reusable, deterministic
    torch.cuda.synchronize()
    for (p, _, _, y), (x, mant, exps), y1 in zip(items, host, first):
        yh = y.cpu().numpy()
        assert np.array_equal(bits(yh), bits(y1))
        # stream-K pieces: at most one extra rounding per piece (<= one per block)
        Rows(x, mant, exps).check(yh, f"stack {mant.shape}", extra_roundings=mant.shape[1] // 64)
    st.close()
    from qwen_b200 import _lib

    assert _lib.load().qwen_b200_device_error(1) == 0


def test_batched_stack_split_over_launches(cuda):
    """More GEMMs than one launch takes (160): the plan runs as several
    launches and still matches single launches bit for bit (every tile here
    is a single K stage, so stream-K cuts none)."""
    import torch

    from qwen_b200 import ops

    rng = np.random.default_rng(23)
    B = 8
    items, singles = [], []
    for i in range(170):
        M, K = (128, 128) if i % 3 else (256, 192)
        mant, exps = rand_weights(rng, M, K)
        dm, de = torch.from_numpy(mant).cuda(), torch.from_numpy(exps).cuda()
        p = ops.quant_planes(torch.from_numpy(rng.normal(0, 1, (B, K)).astype(np.float32)).cuda())
        items.append((p, dm, de, torch.full((B, M), float("nan"), device="cuda")))
        singles.append(ops.bfp8_gemm_tc(p, dm, de))
    st = ops.BatchedStack(items)
    st.run()
    torch.cuda.synchronize()
    for (_, _, _, y), ys in zip(items, singles):
        assert np.array_equal(bits(y.cpu().numpy()), bits(ys.cpu().numpy()))
    st.close()


@pytest.mark.parametrize("M,K,B", [(256, 16384, 64), (130, 8192, 20), (128, 4096, 3)])
def test_batched_stack_stream_k_many_pieces(cuda, M, K, B):
    """A launch with far fewer tiles than SMs and a deep K: stream-K cuts every
    tile into dozens of pieces (one per CTA share), the last piece of each tile
    adds the others' sums in K order.  Outputs stay within the rounding bound
    (one extra rounding per piece, at most one per block), are the same bits on
    a second run, and the per-tile counters are left at zero (a third run with
    new activations is checked too)."""
    import torch

    from qwen_b200 import ops

    rng = np.random.default_rng(M + K + B)
    mant, exps = rand_weights(rng, M, K)
    dm, de = torch.from_numpy(mant).cuda(), torch.from_numpy(exps).cuda()
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    p = ops.quant_planes(torch.from_numpy(x).cuda())
    y = torch.full((B, M), float("nan"), device="cuda")
    st = ops.BatchedStack([(p, dm, de, y)])
    st.run()
    torch.cuda.synchronize()
    y1 = y.cpu().numpy().copy()
    Rows(x, mant, exps).check(y1, ("stream-K", M, K, B), extra_roundings=K // 64)
    st.run()
    torch.cuda.synchronize()
    assert np.array_equal(bits(y.cpu().numpy()), bits(y1))
    x2 = rng.normal(0, 1, (B, K)).astype(np.float32)
    ops.quant_planes(torch.from_numpy(x2).cuda(), out=p)
    st.run()
    torch.cuda.synchronize()
    Rows(x2, mant, exps).check(y.cpu().numpy(), ("stream-K second input", M, K, B), extra_roundings=K // 64)
    st.close()
    from qwen_b200 import _lib

    assert _lib.load().qwen_b200_device_error(1) == 0
