"""bench.py --impl reference: one whole 32-layer forward of the reference's
own CPU forward_latent (compiled from its sources into oracle/_ref), printed
as one JSON line with the keys the benchmark contract names, from a process
that never loads the product library.

Here the arm runs on a small 8x10 token grid (the same code path; the
benchmark's 1080p grid takes minutes of CPU time)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SNIPPET = r"""
import json, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "5", "--warmup", "3"]
sys.path.insert(0, {root!r})
import bench
bench.GRIDS["1080p"] = (1, 8, 10)
rc = bench.main()
maps = open("/proc/self/maps").read()
print(json.dumps({{"rc": rc, "product_loaded": "libs2b.so" in maps,
                   "oracle_loaded": "libref_dit.so" in maps}}))
"""


def test_reference_arm_json_line_without_product_library():
    if not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libref_dit.so")):
        pytest.skip("reference library oracle/_ref/libref_dit.so not built here")
    out = subprocess.run([sys.executable, "-c", SNIPPET.format(root=ROOT)], capture_output=True, text=True,
                         timeout=900, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [json.loads(x) for x in out.stdout.strip().splitlines() if x.startswith("{")]
    line, status = lines[-2], lines[-1]
    assert status == {"rc": 0, "product_loaded": False, "oracle_loaded": True}
    assert line["impl"] == "reference"
    assert line["unit"] == "ms/frame" and line["higher_is_better"] is False
    assert line["steps"] == 1 and line["requested_steps"] == 5 and line["warmup"] == 0
    assert line["value"] > 0 and line["ms_per_step"] == line["value"]
    assert line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["cores"] >= 1
    assert "one whole 32-layer" in line["cpu_baseline"]["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "ms/frame", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["workload"].startswith("cfg3") and line["config"]["grid"] == [1, 8, 10]
