"""torch.ops.qwen_b200.* on the GPU against the CPU oracle: every operator of
the device-level API, on the current stream, bit-exact where the kernels are
(quantizer, exact GEMV, RTL words, lm_head ids and scores, packer, planes),
and within the stated bound for the tcgen05 floats; a bad argument raises
with the library's message."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def bits(a):
    a = np.ascontiguousarray(a, np.float32)
    return np.where(np.isnan(a), np.uint32(0x7FC00000), a.view(np.uint32))


@pytest.fixture(scope="module")
def T(cuda):
    from qwen_b200 import _lib

    return _lib.torch_ops()


def test_quant_gemv_modes(T):
    import torch

    rng = np.random.default_rng(31)
    M, K = 515, 2048
    mant, exps = O.pack_bfp8(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    x = rng.normal(0, 1, (3, K)).astype(np.float32)
    dm, de, dx = torch.from_numpy(mant).cuda(), torch.from_numpy(exps).cuda(), torch.from_numpy(x).cuda()
    xq, xs = T.quant_block64(dx)
    for b in range(3):
        rq, rs = O.quant_x(x[b])
        assert np.array_equal(xq[b].cpu().numpy(), rq) and np.array_equal(bits(xs[b].cpu().numpy()), bits(rs))
    y = T.bfp8_gemv(dx, dm, de, "exact").cpu().numpy()
    assert np.array_equal(bits(y), bits(O.bfp8_gemv(x, mant, exps)))
    yq = T.bfp8_gemv_q(xq[0], xs[0], dm, de, "exact").cpu().numpy()
    assert np.array_equal(bits(yq), bits(y[0]))
    words = T.bfp8_gemv(dx[0], dm, de, "rtl20").cpu().numpy()
    assert np.array_equal(words, O.bfp8_gemv_rtl20(xq[0].cpu().numpy(), xs[0].cpu().numpy(), mant, exps)[0])
    yf = T.bfp8_gemv(dx[0], dm, de, "fast").cpu().numpy()
    terms = np.abs(O.block_dots(mant, xq[0].cpu().numpy()).astype(np.float64)
                   * np.exp2(exps.astype(np.float64) - 134) * xs[0].cpu().numpy().astype(np.float64)).sum(1)
    assert np.all(np.abs(yf.astype(np.float64) - y[0]) <= 1e-5 * terms)
    with pytest.raises(RuntimeError, match="mode must be"):
        T.bfp8_gemv(dx[0], dm, de, "nope")


def test_lm_heads_and_sampler(T):
    import torch

    rng = np.random.default_rng(32)
    V, H, k = 4096, 1024, 40
    lm, le = O.pack_bfp8(rng.normal(0, 0.02, (V, H)).astype(np.float32))
    h = rng.normal(0, 1, H).astype(np.float32)
    dh = torch.from_numpy(h).cuda()
    am, ids, sc, n = T.lm_head_bfp8(dh, torch.from_numpy(lm).cuda(), torch.from_numpy(le).cuda(), k)
    ram, rids, rsc = O.bfp8_lm_head(h, lm, le, k)
    assert am.item() == ram and int(n.item()) == k
    assert np.array_equal(ids.cpu().numpy(), rids) and np.array_equal(bits(sc.cpu().numpy()), bits(rsc))
    tab = (rng.normal(0, 0.05, (V, H)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    am, ids, sc, n = T.lm_head_bf16(dh, torch.from_numpy(tab.view(np.int16)).cuda(), 64)
    rids, rsc = O.topk(O.lm_scores(h, tab), 64)
    assert am.item() == O.lm_head_argmax(h, tab) and np.array_equal(ids.cpu().numpy(), rids)
    st = torch.tensor([12345], dtype=torch.int32, device="cuda")
    tok = T.sample_topk(ids, sc, n, 0.8, 40, 0.9, st)
    assert 0 <= tok.item() < V and tok.item() in ids.cpu().tolist()
    assert st.item() != 12345                      # the xorshift32 state advanced in place


def test_planes_gemm_tc_and_packer(T):
    import torch

    rng = np.random.default_rng(33)
    M, K, B = 256, 1024, 8
    w = rng.normal(0, 0.02, (M, K)).astype(np.float32)
    dm, de = T.pack_bfp8(torch.from_numpy(w).cuda())
    mant, exps = O.pack_bfp8(w)
    assert np.array_equal(dm.cpu().numpy(), mant) and np.array_equal(de.cpu().numpy(), exps)
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    planes, xs_t = T.quant_planes(torch.from_numpy(x).cuda())
    xq = (planes[0].to(torch.int32) * 256 + planes[1].to(torch.int32)).cpu().numpy()
    for b in range(B):
        rq, rs = O.quant_x(x[b])
        assert np.array_equal(xq[b], rq) and np.array_equal(bits(xs_t[:, b].cpu().numpy()), bits(rs))
    y = T.bfp8_gemm_tc(planes, xs_t, dm, de).cpu().numpy()
    ref = O.bfp8_gemv(x, mant, exps)
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))
