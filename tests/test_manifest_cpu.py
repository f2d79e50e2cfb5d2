"""The weight layout against the reference's own manifest
(06-模型与权重/qwen35_weights_64k_manifest.json, committed as
tests/golden/manifest_64k.json by make_golden.py): the 150 BFP8 GEMVs of a
token, their names, shapes and order, every per-tensor size key, the
exporter's 64-byte offset rule over all 320 tensors, and the zero-copy views
WeightFile gives the engine's pointers (qwen_real_engine.py:1188-1206)."""
import json
import os

import numpy as np

from qwen_b200 import model

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "manifest_64k.json")


def ref_manifest():
    with open(GOLDEN, encoding="utf-8") as f:
        return json.load(f)


def test_stack_is_the_manifest_bfp8_tensors_in_file_order():
    m = ref_manifest()
    bfp8 = sorted(model.bfp8_tensors(m), key=lambda e: e[1])
    stack = model.qwen35_08b_stack()
    assert len(bfp8) == len(stack) == 150
    assert [(n, M, K) for n, _, M, K in bfp8] == [(t.name, t.M, t.K) for t in stack]
    assert sum(m["tensors"][n]["byte_size"] for n, _, _, _ in bfp8) == 504791040
    assert model.stack_bytes(stack)["weights"] == 504791040


def test_manifest_for_gives_the_reference_entry_keys():
    ref = ref_manifest()["tensors"]
    mine = model.manifest_for(model.qwen35_08b_stack())["tensors"]
    for name, e in mine.items():
        r = ref[name]
        for key in ("dtype", "shape", "type", "mantissa_bytes", "exponent_bytes", "byte_size"):
            assert e[key] == r[key], (name, key)


def test_file_layout_reproduces_every_reference_offset():
    m = ref_manifest()
    table, total = model.file_layout([(n, t["byte_size"]) for n, t in m["tensors"].items()])
    assert total == m["total_binary_bytes"] == 643362048
    assert all(table[n] == t["file_offset"] for n, t in m["tensors"].items())
    # the stack-only layout keeps the same per-tensor alignment and sizes
    own, _ = model.layout(model.qwen35_08b_stack())
    assert all(off % 64 == 0 for off, _ in own.values())


def synthetic_file(m, upto_layer=0, seed=9):
    """A weight-file image of the reference layout up to the end of layer
    `upto_layer`'s BFP8 tensors, those filled with packed N(0, 0.02) rows,
    everything else zero."""
    from oracle import oracle as O

    names = [n for n, _, _, _ in sorted(model.bfp8_tensors(m), key=lambda e: e[1])
             if f".layers.{upto_layer}." in n or any(f".layers.{l}." in n for l in range(upto_layer))]
    end = max(m["tensors"][n]["file_offset"] + m["tensors"][n]["byte_size"] for n in names)
    buf = np.zeros(end, np.uint8)
    rng = np.random.default_rng(seed)
    for n in names:
        t = m["tensors"][n]
        M, K = t["shape"]
        mant, exps = O.pack_bfp8(rng.normal(0, 0.02, (M, K)).astype(np.float32))
        o = t["file_offset"]
        buf[o:o + M * K] = mant.view(np.uint8).ravel()
        buf[o + M * K:o + M * K + M * K // 64] = exps.ravel()
    # the manifest of the truncated file: the tensors it holds
    sub = dict(m, tensors={n: t for n, t in m["tensors"].items() if t["file_offset"] + t["byte_size"] <= end})
    return buf, names, sub


def test_weight_file_views_are_the_engine_slices():
    m = ref_manifest()
    buf, names, sub = synthetic_file(m)
    wf = model.WeightFile(sub, buffer=buf)
    assert [t.name for t in wf.stack()][:len(names)] == names
    for n in names:
        mant, exps = wf.views(n)
        info = m["tensors"][n]
        M, K = info["shape"]
        raw = np.frombuffer(buf, dtype=np.uint8, count=info["byte_size"], offset=info["file_offset"])
        assert mant.ctypes.data == raw[:M * K].ctypes.data and exps.ctypes.data == raw[M * K:].ctypes.data
        assert mant.shape == (M, K) and exps.shape == (M, K // 64)
