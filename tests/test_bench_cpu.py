"""bench.py's reference arm runs on the host cores (no GPU): its JSON line
keeps the contract the driver reads -- the metric, unit and config of the
default workload, a cpu_baseline block and an e2e block with no host/device
copies -- and a workload with no reference CPU implementation prints an
`unavailable` line and exits 0."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(REPO, "oracle", "_ref", "libref_kernels.so")


def run_bench(*args):
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], capture_output=True, text=True,
                         timeout=240, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference C not compiled (make -C oracle ref)")
def test_reference_arm_json_contract():
    d = run_bench("--impl", "reference", "--steps", "2", "--warmup", "1")
    assert d["impl"] == "reference"
    assert d["metric"].startswith("BFP8 GEMV HBM GB/s")
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 1 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"].startswith("qwen35-0.8b linear stack")
    assert d["config"]["algorithmic_bytes_per_step"] == 507346944
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_unavailable_for_the_rtl_mode():
    d = run_bench("--impl", "reference", "--workload", "rtl20")
    assert d["impl"] == "reference" and "FPGA" in d["unavailable"]
