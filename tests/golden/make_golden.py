"""Generate the committed golden fixtures in tests/golden/.

Run in a container that has the reference tree (read-only) and the
reference C files compiled by ``make -C oracle ref``:

    python tests/golden/make_golden.py REFERENCE_ROOT
    (or QWEN_REFERENCE_ROOT=... python tests/golden/make_golden.py)

Every fixture is produced by the reference's OWN code or recipe:
  packer.npz      05-主机侧源码/bfp8_packer.py pack_matrix_soa, imported and run
  ref_numpy_gemv.npz  04-板载脚本与工具/qwen_real_engine.py gemv_bfp8 (its numpy
                  fallback, :1233-1239), imported and run with no kernels
  manifest_64k.json   06-模型与权重/qwen35_weights_64k_manifest.json, every
                  tensor entry (board addresses dropped)
  plan_layouts.json   qwen_real_engine.py's ctypes LinearLayerPlanC / MlpPlanC:
                  field offsets and sizes
  ref_gemv.npz    04-板载脚本与工具/qwen_kernels_opt.c bfp8_gemv, compiled from
                  source for x86 (its scalar float path, :311-325)
  ref_lm.npz      qwen_kernels_opt.c lm_head_argmax and qwen_sampling.c
                  lm_head_topk (x86 scalar builds) on the sampling self-test
                  data (xorshift seed 0x13579BDF, qwen_sampling.c:536-561,
                  917-1010)
  sampler.npz     qwen_sampling.c sample_from_topk on a sweep of arguments
  tb_gemv.npz     the stimulus and golden model of 02-RTL与仿真/tb_gemv_core.v
                  (LCG seed*1103515245+12345, cases :399-419, exact block dots
                  :150-158, double-precision row model :161-170)
The GPU box never needs the reference tree: tests read only these files.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle import oracle as O  # noqa: E402

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QWEN_REFERENCE_ROOT", "")
if __name__ == "__main__" and not os.path.isdir(REF):
    sys.exit("make_golden.py: pass the reference checkout (or set QWEN_REFERENCE_ROOT)")
REF_DIR = os.path.join(REPO, "oracle", "_ref")


def ref_libs():
    k = ctypes.CDLL(os.path.join(REF_DIR, "libref_kernels.so"))
    s = ctypes.CDLL(os.path.join(REF_DIR, "libref_sampling.so"))
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    k.init_kernels.argtypes = []
    k.bfp8_gemv.argtypes = [P, P, P, P, I, I]
    k.bfp8_gemv.restype = None
    k.lm_head_argmax.argtypes = [P, P, I, I]
    k.lm_head_argmax.restype = I
    s.lm_head_topk.argtypes = [P, P, I, I, I, P, P]
    s.lm_head_topk.restype = I
    s.sample_from_topk.argtypes = [P, P, I, F, I, F, P]
    s.sample_from_topk.restype = I
    k.init_kernels()
    return k, s


# ------------------------------------------------------------------ packer
def make_packer():
    sys.path.insert(0, os.path.join(REF, "05-主机侧源码"))
    import bfp8_packer as R  # the reference packer itself

    rng = np.random.default_rng(20261201)
    mats = {}
    mats["normal"] = rng.normal(0, 0.02, (16, 1024)).astype(np.float32)
    w = rng.normal(0, 1, (8, 128)).astype(np.float32)
    w[0, 17] = 25.0                       # outlier (the packer self-test's case)
    w[1, :64] = 0.0                       # all-zero block -> e = 127
    w[2, :64] = 1e-13                     # below the 1e-12 floor -> zero block
    w[3, :64] = np.float32(2.0) ** -20    # exact power of two peak
    w[4, 64:] = -1.0                      # negative peak, -128 reachable
    w[5, :64] = np.linspace(-0.5, 0.5, 64, dtype=np.float32)
    mats["edges"] = w
    mats["wide"] = (rng.normal(0, 1, (4, 512)) * np.exp2(rng.integers(-30, 30, (4, 512)))).astype(np.float32)
    out = {}
    for name, m in mats.items():
        mb, eb = R.pack_matrix_soa(m)
        M, K = m.shape
        out[f"{name}_w"] = m
        out[f"{name}_mant"] = np.frombuffer(mb, np.int8).reshape(M, K)
        out[f"{name}_exps_padded"] = np.frombuffer(eb, np.uint8)
    np.savez_compressed(os.path.join(HERE, "packer.npz"), **out)


# ------------------------------------------------------------------ gemv
def make_ref_gemv(k):
    rng = np.random.default_rng(7)
    out = {}
    for tag, (M, K) in {"a": (33, 1024), "b": (64, 512), "c": (7, 4096)}.items():
        w = rng.normal(0, 0.02, (M, K)).astype(np.float32)
        mant, exps = O.pack_bfp8(w)
        x = rng.normal(0, 1, K).astype(np.float32)
        y = np.zeros(M, np.float32)
        k.bfp8_gemv(y.ctypes.data, x.ctypes.data, mant.ctypes.data, exps.ctypes.data, M, K)
        out[f"{tag}_mant"], out[f"{tag}_exps"], out[f"{tag}_x"], out[f"{tag}_y"] = mant, exps, x, y
    np.savez_compressed(os.path.join(HERE, "ref_gemv.npz"), **out)


def make_ref_numpy_gemv():
    """The reference engine's numpy fallback (qwen_real_engine.py:1233-1239),
    run as the reference's own method with no kernel library attached."""
    sys.path.insert(0, os.path.join(REF, "04-板载脚本与工具"))
    import qwen_real_engine as E  # the reference engine module itself

    class NoKernels:
        kernels = None

        def __init__(self, views):
            self.views = views

        def _tensor_views(self, name):
            return self.views[name]

        def _y_buf(self, name, M):
            return np.empty(M, np.float32)

    rng = np.random.default_rng(1233)
    out, views = {}, {}
    for tag, (M, K) in {"a": (40, 1024), "b": (16, 4096), "c": (3, 192)}.items():
        mant, exps = O.pack_bfp8(rng.normal(0, 0.02, (M, K)).astype(np.float32))
        if tag == "c":
            exps[0, 0] = 3      # a subnormal block scale 2^-131
            exps[1, 2] = 200    # a large one
        views[tag] = (mant.reshape(-1), exps.reshape(-1), M, K)
        x = rng.normal(0, 1, K).astype(np.float32)
        y = E.QwenRealEngine.gemv_bfp8(NoKernels(views), x, tag)
        out[f"{tag}_mant"], out[f"{tag}_exps"], out[f"{tag}_x"], out[f"{tag}_y"] = mant, exps, x, y
    np.savez_compressed(os.path.join(HERE, "ref_numpy_gemv.npz"), **out)


def make_manifest():
    """The reference weight manifest (06-模型与权重/qwen35_weights_64k_manifest.json):
    every tensor's dtype, shape, type, sizes and file_offset, in file order
    (the physical DDR addresses of the board are dropped)."""
    import json

    with open(os.path.join(REF, "06-模型与权重", "qwen35_weights_64k_manifest.json"), encoding="utf-8") as f:
        m = json.load(f)
    out = {k: v for k, v in m.items() if k not in ("tensors", "ddr3_base_addr")}
    out["tensors"] = {n: {k: v for k, v in t.items() if k != "phys_addr"} for n, t in m["tensors"].items()}
    with open(os.path.join(HERE, "manifest_64k.json"), "w", encoding="utf-8") as f:
        json.dump(out, f, indent=0, ensure_ascii=False)


def make_plan_layouts():
    """Field names, offsets and sizes of the reference engine's ctypes plan
    structures (qwen_real_engine.py:20-74), imported from the engine."""
    import json

    sys.path.insert(0, os.path.join(REF, "04-板载脚本与工具"))
    import qwen_real_engine as E

    out = {}
    for cls in (E.LinearLayerPlanC, E.MlpPlanC):
        out[cls.__name__] = {"size": ctypes.sizeof(cls),
                             "fields": [[n, getattr(cls, n).offset, getattr(cls, n).size] for n, _ in cls._fields_]}
    with open(os.path.join(HERE, "plan_layouts.json"), "w") as f:
        json.dump(out, f, indent=1)


# ------------------------------------------------------------------ lm_head
def make_ref_lm(k, s):
    g = O.XorShift32(0x13579BDF)
    out = {}
    cases = [("c1", 1000, 64, [1, 5, 20, 100, 1000, 1050]), ("c2", 500, 67, [7]),
             ("c3", 65536, 1024, [1, 20, 64])]
    for tag, V, H, ks in cases:
        tab, h = g.selftest_fill(V, H)
        out[f"{tag}_argmax"] = np.int32(k.lm_head_argmax(h.ctypes.data, tab.ctypes.data, V, H))
        for kk in ks:
            n_alloc = max(kk, 1)
            ids = np.zeros(n_alloc, np.int32)
            sc = np.zeros(n_alloc, np.float32)
            n = s.lm_head_topk(h.ctypes.data, tab.ctypes.data, V, H, kk, ids.ctypes.data, sc.ctypes.data)
            out[f"{tag}_k{kk}_ids"] = ids[:n].copy()
            out[f"{tag}_k{kk}_scores"] = sc[:n].copy()
        out[f"{tag}_shape"] = np.array([V, H], np.int32)
    np.savez_compressed(os.path.join(HERE, "ref_lm.npz"), **out)


# ------------------------------------------------------------------ sampler
def make_sampler(s):
    rng = np.random.default_rng(99)
    cases = []
    for ci in range(40):
        n = int(rng.integers(1, 65))
        scores = np.sort(rng.normal(0, 2, n).astype(np.float32))[::-1].copy()
        if ci % 5 == 0:
            rng.shuffle(scores)                           # unsorted input path
        if ci % 7 == 0 and n > 3:
            scores[1] = scores[2]                         # ties
        ids = rng.integers(0, 65536, n).astype(np.int32)
        temp = float([0.0, 1e-7, 0.3, 0.7, 1.0, 2.0][ci % 6])
        top_k = int([0, 1, 5, 40, 100][ci % 5])
        top_p = float([1.0, 0.9, 0.5, 1e-9, 0.0, 1.5][ci % 6])
        state = int(rng.integers(0, 2**32, dtype=np.uint64)) if ci % 9 else 0
        st = ctypes.c_uint(state)
        draws = [s.sample_from_topk(ids.ctypes.data, scores.ctypes.data, n, temp, top_k, top_p,
                                    ctypes.byref(st)) for _ in range(25)]
        cases.append((ids, scores, temp, top_k, top_p, state, np.array(draws, np.int32), st.value))
    out = {"n_cases": np.int32(len(cases))}
    for i, (ids, sc, t, tk, tp, st0, draws, st1) in enumerate(cases):
        out[f"{i}_ids"], out[f"{i}_scores"] = ids, sc
        out[f"{i}_args"] = np.array([t, tk, tp], np.float64)
        out[f"{i}_state"] = np.array([st0, st1], np.uint64)
        out[f"{i}_draws"] = draws
    np.savez_compressed(os.path.join(HERE, "sampler.npz"), **out)


# ------------------------------------------------------------------ tb_gemv_core
def lcg_case(k, mm, sd, e_lo, e_hi, xs_oct, auto_scale):
    """Stimulus of tb_gemv_core.v run_case (:202-249) with its golden model."""
    nb = k // 64
    NB_MAX = 16
    seed = sd & 0xFFFFFFFF

    def step():
        nonlocal seed
        seed = (seed * 1103515245 + 12345) & 0xFFFFFFFF
        return seed

    xq = np.zeros(k, np.int16)
    for i in range(k):
        v = step() & 0xFFFF
        v = v - 0x10000 if v & 0x8000 else v
        xq[i] = v >> 1
    wq = np.zeros(mm * k, np.int8)
    for i in range(mm * k):
        v = (step() >> 8) & 0xFF
        wq[i] = v - 256 if v & 0x80 else v
    we = np.zeros(mm * nb, np.uint8)
    for i in range(mm * nb):
        we[i] = e_lo + ((step() & 0xFF) % (e_hi - e_lo + 1))
    rel = np.ones(NB_MAX)
    for b in range(NB_MAX):
        sv = step()
        r = 1.0
        for i in range(xs_oct):
            if (sv >> i) & 1:
                r *= 2.0
        rel[b] = r
    W = wq.reshape(mm, k).astype(np.int64)
    dots = (W.reshape(mm, nb, 64) * xq.astype(np.int64).reshape(nb, 64)).sum(axis=2)
    expsc = np.ldexp(1.0, we.astype(np.int64) - 134).reshape(mm, nb)
    if auto_scale:
        ypk = np.abs((dots * expsc * rel[:nb]).sum(axis=1)).max()
        a0 = 1.2 * 16384.0 / ypk if ypk > 0 else 16384.0
    else:
        a0 = 16384.0
    if xs_oct:
        xs = np.array([np.float32(a0 * rel[b] / 16384.0) for b in range(nb)], np.float32)
    else:
        xs = np.ones(nb, np.float32)
    yref = (dots * expsc * xs.astype(np.float64)).sum(axis=1)
    return xq, wq.reshape(mm, k), we.reshape(mm, nb), xs, dots.astype(np.int64), yref


def make_tb():
    cases = [  # (K, M, seed, dequant, e_lo, e_hi, xs_octaves, auto_scale, exp_sat)  tb_gemv_core.v:401-419
        (128, 3, 0x12345678, 0, 118, 130, 0, 0, 0),
        (1024, 8, 0x0BADF00D, 0, 118, 130, 0, 0, 0),
        (128, 3, 0xA5A55A5A, 1, 118, 130, 4, 1, 0),
        (1024, 8, 0xCAFEBABE, 1, 118, 130, 4, 1, 0),
        (128, 8, 0x98765432, 1, 118, 130, 4, 1, 0),
        (1024, 4, 0x5EED1234, 1, 118, 130, 10, 1, 0),
        (512, 4, 0x2468ACE0, 1, 118, 130, 1, 1, 0),
        (512, 4, 0x13579BDF, 1, 104, 116, 0, 0, 0),
        (64, 2, 0xDEADBEEF, 1, 240, 250, 0, 0, 1),
        (64, 2, 0xF00D4321, 1, 40, 60, 0, 0, 0),
    ]
    out = {"cases": np.array(cases, np.int64)}
    for i, (K, M, sd, dq, elo, ehi, xo, au, sat) in enumerate(cases):
        xq, wq, we, xs, dots, yref = lcg_case(K, M, sd, elo, ehi, xo, au)
        out[f"{i}_xq"], out[f"{i}_w"], out[f"{i}_e"], out[f"{i}_xs"] = xq, wq, we, xs
        out[f"{i}_dots"], out[f"{i}_yref"] = dots, yref
    np.savez_compressed(os.path.join(HERE, "tb_gemv.npz"), **out)


def make_ref_rmsnorm(k):
    """rmsnorm of the reference compiled for x86 (its portable build,
    qwen_kernels_opt.c:140-172), on a few sizes, scales and eps values."""
    k.rmsnorm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_float]
    rng = np.random.default_rng(11)
    out = {}
    for tag, (n, sx, eps) in {"a": (1024, 1.0, 1e-6), "b": (3584, 20.0, 1e-5), "c": (1000, 1e-3, 1e-6),
                              "d": (4096, 1e-19, 1e-6)}.items():
        x = rng.normal(0, sx, n).astype(np.float32)
        w = rng.normal(0, 0.1, n).astype(np.float32)
        y = np.zeros(n, np.float32)
        k.rmsnorm(y.ctypes.data, x.ctypes.data, w.ctypes.data, n, eps)
        out[f"{tag}_x"], out[f"{tag}_w"], out[f"{tag}_y"] = x, w, y
        out[f"{tag}_eps"] = np.float32(eps)
    np.savez_compressed(os.path.join(HERE, "ref_rmsnorm.npz"), **out)


def make_ref_residual(k):
    """add_residual of the reference compiled for x86 (its portable build,
    qwen_kernels_opt.c:388-396), incl. subnormal operands."""
    k.add_residual.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    rng = np.random.default_rng(12)
    x = rng.normal(0, 1, 1003).astype(np.float32)
    r = rng.normal(0, 1, 1003).astype(np.float32)
    x[5], r[5], x[9], r[17] = 1e-39, 1e-39, -3e-40, 2e-41
    y = x.copy()
    k.add_residual(y.ctypes.data, r.ctypes.data, y.size)
    np.savez_compressed(os.path.join(HERE, "ref_residual.npz"), x=x, r=r, y=y)


def make_ref_swiglu(k):
    """swiglu of the reference compiled for x86 (its portable build,
    qwen_kernels_opt.c:365-386): g / (1 + expf(-g)) * up, over N(0, 3) gates
    plus zeros, subnormals, values past exp_neon's clamps (+-87, +-88) and
    large magnitudes; n = 3587 leaves a tail after the last multiple of 4."""
    k.swiglu.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    rng = np.random.default_rng(13)
    n = 3587
    g = rng.normal(0, 3, n).astype(np.float32)
    u = rng.normal(0, 1, n).astype(np.float32)
    special = [0.0, -0.0, 1e-39, -1e-39, 3e-41, 87.0, -87.0, 87.5, -87.5, 88.0, -88.0, 88.5, -88.5, 100.0,
               -100.0, 1e4, -1e4, 20.0, -20.0, 1e-6]
    g[:len(special)] = np.array(special, np.float32)
    u[40:44] = np.array([1e-39, -2e-40, 0.0, 1e30], np.float32)
    y = np.zeros(n, np.float32)
    k.swiglu(y.ctypes.data, g.ctypes.data, u.ctypes.data, n)
    np.savez_compressed(os.path.join(HERE, "ref_swiglu.npz"), gate=g, up=u, y=y)


def main():
    k, s = ref_libs()
    make_packer()
    make_ref_gemv(k)
    make_ref_numpy_gemv()
    make_manifest()
    make_plan_layouts()
    make_ref_rmsnorm(k)
    make_ref_residual(k)
    make_ref_swiglu(k)
    make_ref_lm(k, s)
    make_sampler(s)
    make_tb()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
