"""C ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and its host-side sampler reproduces the reference."""
import ctypes
import os
import re

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "qwen_b200.h")


def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^QB_API\s+[\w\s\*]+?\b(\w+)\(", text, re.M)))


def test_header_declares_reference_dropins():
    syms = header_symbols()
    for name in ("init_kernels", "bfp8_gemv", "lm_head_argmax", "lm_head_topk", "sample_from_topk",
                 "qwen_prof_enable", "qwen_prof_reset", "qwen_prof_count", "qwen_prof_get", "qwen_prof_name"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    from qwen_b200 import _lib

    lib = _lib.load()
    missing = [s for s in header_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    # and the Python binding covers the whole header
    assert set(header_symbols()) <= set(_lib.SIGNATURES)


def test_profiler_slots():
    from qwen_b200 import _lib

    lib = _lib.load()
    n = lib.qwen_prof_count()
    names = [lib.qwen_prof_name(i).decode() for i in range(n)]
    assert "bfp8_gemv" in names and "lm_head_argmax" in names
    assert lib.qwen_prof_name(n).decode() == "?"
    lib.qwen_prof_reset()
    assert lib.qwen_prof_get(0) == 0.0


def _sample(lib, ids, scores, t, tk, tp, state):
    st = ctypes.c_uint(state)
    return lib.sample_from_topk(ids.ctypes.data, scores.ctypes.data, len(ids), t, tk, tp, ctypes.byref(st)), st.value


def test_sampler_matches_reference(golden):
    """sample_from_topk reproduces the compiled reference draw for draw,
    including the rng state it leaves behind (qwen_sampling.c:411-529)."""
    from qwen_b200 import _lib

    lib = _lib.load()
    g = golden("sampler.npz")
    for i in range(int(g["n_cases"])):
        ids, sc = g[f"{i}_ids"], g[f"{i}_scores"]
        t, tk, tp = g[f"{i}_args"]
        st0, st1 = (int(v) for v in g[f"{i}_state"])
        st = ctypes.c_uint(st0)
        draws = [lib.sample_from_topk(ids.ctypes.data, sc.ctypes.data, len(ids), float(t), int(tk), float(tp),
                                      ctypes.byref(st)) for _ in range(25)]
        assert draws == g[f"{i}_draws"].tolist(), i
        assert st.value == st1, i


REF_SAMPLING = os.path.join(REPO, "oracle", "_ref", "libref_sampling.so")


@pytest.mark.skipif(not os.path.exists(REF_SAMPLING), reason="oracle/_ref not built (make -C oracle ref)")
def test_sampler_matches_compiled_reference_on_random_lists():
    """Draw for draw against the reference's own sample_from_topk compiled here
    (qwen_sampling.c:411-529): unordered lists, tied scores, NaN scores, and the
    temperature / top_k / top_p edges (0, negative, NaN, above 1)."""
    from qwen_b200 import _lib

    lib = _lib.load()
    ref = ctypes.CDLL(REF_SAMPLING)
    for f in (lib.sample_from_topk, ref.sample_from_topk):
        f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                      ctypes.c_float, ctypes.c_void_p]
        f.restype = ctypes.c_int
    rng = np.random.default_rng(7)
    temps = [0.0, 1e-7, 1e-6, 0.3, 0.8, 1.0, 2.5, -1.0, float("nan")]
    top_ps = [0.0, 0.05, 0.5, 0.9, 0.95, 1.0, 1.5, -0.2, float("nan")]
    for case in range(600):
        n = int(rng.integers(1, 70))
        ids = rng.permutation(200000)[:n].astype(np.int32)
        kind = case % 4
        if kind == 0:
            sc = np.sort(rng.normal(0, 3, n).astype(np.float32))[::-1].copy()
        elif kind == 1:
            sc = rng.normal(0, 3, n).astype(np.float32)
        elif kind == 2:
            sc = rng.integers(-3, 3, n).astype(np.float32)  # many ties
        else:
            sc = rng.normal(0, 3, n).astype(np.float32)
            sc[rng.integers(0, n, max(1, n // 8))] = np.nan
        t = temps[case % len(temps)]
        tp = top_ps[(case // len(temps)) % len(top_ps)]
        tk = int(rng.integers(-2, n + 3))
        s0 = int(rng.integers(1, 2**32))
        a, b = ctypes.c_uint(s0), ctypes.c_uint(s0)
        for _ in range(8):
            da = lib.sample_from_topk(ids.ctypes.data, sc.ctypes.data, n, t, tk, tp, ctypes.byref(a))
            db = ref.sample_from_topk(ids.ctypes.data, sc.ctypes.data, n, t, tk, tp, ctypes.byref(b))
            assert da == db, (case, n, t, tk, tp)
        assert a.value == b.value, case


def test_sampler_selftest_cases():
    """The reference self-test's sampling cases (qwen_sampling.c:682-898)."""
    from qwen_b200 import _lib

    lib = _lib.load()
    ids = np.array([7, 8, 9, 10], np.int32)
    sc = np.array([0.0, -0.5, -1.0, -1.5], np.float32)
    for t in (0.0, -1.0, 1e-7):
        assert _sample(lib, ids, sc, t, 0, 1.0, 0xDEADBEEF)[0] == 7
    st = ctypes.c_uint(0x11223344)
    assert all(lib.sample_from_topk(ids.ctypes.data, sc.ctypes.data, 4, 1.0, 1, 1.0, ctypes.byref(st)) == 7
               for _ in range(1000))
    ids2 = np.array([100, 101, 102, 103], np.int32)
    sc2 = np.array([0.0, 0.0, -1.0, -1.0], np.float32)
    st = ctypes.c_uint(0xC0FFEE01)
    counts = {i: 0 for i in ids2.tolist()}
    for _ in range(10000):
        counts[lib.sample_from_topk(ids2.ctypes.data, sc2.ctypes.data, 4, 1.0, 0, 1.0, ctypes.byref(st))] += 1
    p = np.exp(sc2.astype(np.float64))
    p /= p.sum()
    for j, i in enumerate(ids2.tolist()):
        if p[j] >= 0.2:
            assert abs(counts[i] / 10000 - p[j]) / p[j] <= 0.05
    st = ctypes.c_uint(0xABCD0002)
    assert all(lib.sample_from_topk(ids2.ctypes.data, sc2.ctypes.data, 4, 1.0, 0, 0.3, ctypes.byref(st)) == 100
               for _ in range(1000))
    # unsorted input, n = 0, NULL ids, n = 1
    ids3 = np.array([10, 11, 12], np.int32)
    sc3 = np.array([0.0, 2.0, 1.0], np.float32)
    assert _sample(lib, ids3, sc3, 0.0, 0, 1.0, 0x5555AAAA)[0] == 11
    assert lib.sample_from_topk(ids.ctypes.data, sc.ctypes.data, 0, 1.0, 0, 1.0, None) == -1
    assert lib.sample_from_topk(None, sc.ctypes.data, 4, 1.0, 0, 1.0, None) == -1
    assert lib.sample_from_topk(ids.ctypes.data, sc.ctypes.data, 1, 1.0, 0, 1.0, None) == 7


def test_invalid_arguments_are_rejected_without_a_device():
    from qwen_b200 import _lib

    lib = _lib.load()
    assert lib.lm_head_topk(None, None, 0, 0, 0, None, None) == 0
    assert lib.qwen_b200_quant_dev(None, 1, 64, None, None, None) == -1
    assert lib.qwen_b200_gemv_dev(None, None, None, None, 4, 64, None) == -1
    assert lib.qwen_b200_stack_run(12345, None) == -1
    assert b"bad handle" in lib.qwen_b200_last_error()


def test_sharded_entry_points_reject_bad_arguments_without_a_gpu():
    """The row-sharded and IPC entry points validate before touching a device:
    unknown plans, world sizes outside 1..8, missing flag arrays and null
    buffers return QB_EINVAL (-1) with a message."""
    from qwen_b200 import _lib

    lib = _lib.load()
    flags = (ctypes.c_void_p * 8)()
    assert lib.qwen_b200_stack_run_sync(0, None, None, 0, flags, 0, 1, 0) == -1
    assert lib.qwen_b200_stack_run_sync(12345, None, None, 0, flags, 0, 1, 0) == -1
    assert lib.qwen_b200_tc_stack_run_sync(0, None, flags, 1, 2, 0) == -1
    assert lib.qwen_b200_quant_planes_wait_dev(None, 1, 64, None, None, 4, None, 0, 1, None) == -1
    assert lib.qwen_b200_quant_planes_wait_dev(None, 1, 64, None, None, 4, None, 1, 9, None) == -1
    out = ctypes.c_void_p()
    assert lib.qwen_b200_dev_alloc(0, ctypes.byref(out)) == -1
    assert lib.qwen_b200_ipc_handle(None, None) == -1
    assert lib.qwen_b200_ipc_open(None, ctypes.byref(out)) == -1
    assert b"bad" in lib.qwen_b200_last_error() or b"qwen_b200" in lib.qwen_b200_last_error()
    one = (ctypes.c_void_p * 1)()
    ints = (ctypes.c_int * 1)(64)
    # world 9 is out of range
    assert lib.qwen_b200_stack_create_sharded(1, one, one, one, one, ints, ints, 0, 9, one, ints) == -1
    assert lib.qwen_b200_tc_stack_create_sharded(1, one, one, one, one, one, ints, ints, None, 8, 8, 1, None,
                                                 ints) == -1


def test_rtl20_and_device_sampler_reject_bad_arguments_without_a_gpu():
    """The RTL dequant GEMV wants exactly one activation form (fp32 x, or xq
    with xs) and K a positive multiple of 64; the device sampler wants a list,
    an output and 0 <= n <= 1024.  Both reject before touching a device."""
    from qwen_b200 import _lib

    lib = _lib.load()
    p = ctypes.c_void_p(64)   # never dereferenced: validation fails first
    assert lib.qwen_b200_gemv_rtl20_dev(p, None, None, None, p, p, 4, 64, None, None) == -1
    assert b"give x, or xq and xs" in lib.qwen_b200_last_error()
    assert lib.qwen_b200_gemv_rtl20_dev(p, p, p, p, p, p, 4, 64, None, None) == -1
    assert lib.qwen_b200_gemv_rtl20_dev(p, None, p, None, p, p, 4, 64, None, None) == -1
    assert lib.qwen_b200_gemv_rtl20_dev(p, p, None, None, p, p, 4, 96, None, None) == -1
    assert lib.qwen_b200_sample_topk_dev(p, p, None, 1025, 1.0, 0, 1.0, None, p, None) == -1
    assert lib.qwen_b200_sample_topk_dev(p, p, None, -1, 1.0, 0, 1.0, None, p, None) == -1
    assert lib.qwen_b200_sample_topk_dev(None, p, None, 4, 1.0, 0, 1.0, None, p, None) == -1
    assert b"outside 0..1024" in lib.qwen_b200_last_error()


def test_plan_structs_match_the_engine_ctypes_layouts(tmp_path):
    """LinearLayerPlanC / MlpPlanC in include/qwen_b200.h have, field by
    field, the offsets and sizes of the reference engine's ctypes structures
    (qwen_real_engine.py:20-74; tests/golden/plan_layouts.json), compiled
    here with gcc."""
    import json
    import shutil
    import subprocess

    if not shutil.which("gcc"):
        pytest.skip("no gcc")
    layouts = json.load(open(os.path.join(REPO, "tests", "golden", "plan_layouts.json")))
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "qwen_b200.h"', 'int main(void) {']
    for name, spec in layouts.items():
        lines.append(f'    printf("{name} size %zu\\n", sizeof({name}));')
        for field, _, _ in spec["fields"]:
            lines.append(f'    printf("{name} {field} %zu %zu\\n", offsetof({name}, {field}), '
                         f'sizeof((({name}*)0)->{field}));')
    lines.append("    return 0;\n}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)], check=True)
    got = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    want = []
    for name, spec in layouts.items():
        want.append(f"{name} size {spec['size']}")
        want += [f"{name} {f} {o} {s}" for f, o, s in spec["fields"]]
    assert [g for g in got if g] == want


def test_python_plan_structs_match_the_engine_layouts():
    """qwen_b200.plans' ctypes LinearLayerPlanC / MlpPlanC (what a Python
    host passes to forward_linear_layer / forward_token_c) have the engine's
    offsets and sizes (qwen_real_engine.py:20-74; tests/golden/plan_layouts.json)."""
    import ctypes
    import json

    from qwen_b200 import plans

    layouts = json.load(open(os.path.join(REPO, "tests", "golden", "plan_layouts.json")))
    for name, spec in layouts.items():
        cls = getattr(plans, name)
        assert ctypes.sizeof(cls) == spec["size"], name
        got = [(f, getattr(cls, f).offset, getattr(cls, f).size) for f, _ in cls._fields_]
        assert got == [tuple(x) for x in spec["fields"]], name


def test_token_loop_rejects_bad_arguments_without_a_gpu():
    """forward_token_c refuses a negative token id or a null pointer before
    any device work (returns -1 with a message); forward_linear_layer and
    forward_mlp refuse a null h; the state-mode call refuses unknown modes."""
    import ctypes

    import numpy as np

    from qwen_b200 import _lib, plans

    lib = _lib.load()
    h = np.zeros(plans.HIDDEN, np.float32)
    lps = (plans.LinearLayerPlanC * 18)()
    mps = (plans.MlpPlanC * 24)()
    full = np.zeros(24, np.int32)
    w = np.zeros(plans.HIDDEN, np.float32)
    emb = np.zeros(16, np.uint16)
    args = (h.ctypes.data, ctypes.byref(lps), ctypes.byref(mps), full.ctypes.data, w.ctypes.data, emb.ctypes.data,
            plans.CALLBACK(), None)   # CALLBACK(): a null function pointer
    assert lib.forward_token_c(-1, *args) == -1
    assert b"forward_token_c" in lib.qwen_b200_last_error()
    assert lib.forward_token_c(5, None, *args[1:]) == -1
    lib.forward_linear_layer(ctypes.byref(lps[0]), None)
    assert b"forward_linear_layer" in lib.qwen_b200_last_error()
    lib.forward_mlp(ctypes.byref(mps[0]), None)
    assert b"forward_mlp" in lib.qwen_b200_last_error()
    assert lib.qwen_b200_gdn_state_mode(7) != 0
