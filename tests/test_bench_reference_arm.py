"""bench.py's CPU reference arm (CPU only): it must time the oracle's restatement of the reference's CPU path
without importing the product package or mapping any of its native libraries, and print the same config dict
the GPU arm prints for the workload."""
from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROBE = r"""
import json, runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"]
runpy.run_path("bench.py", run_name="__main__")
maps = open("/proc/self/maps").read()
print("PROBE " + json.dumps({
    "product_modules": sorted(m for m in sys.modules if m.startswith("synthesize_cpp_b200")),
    "product_libs": sorted({l.split()[-1] for l in maps.splitlines() if "libb200q8" in l}),
    "oracle_lib": "libq8oracle" in maps,
}))
"""


def test_reference_arm_runs_the_oracle_only():
    out = subprocess.run([sys.executable, "-c", PROBE], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.splitlines()
    line = json.loads(next(l for l in lines if l.startswith("{")))
    probe = json.loads(next(l for l in lines if l.startswith("PROBE "))[6:])
    assert probe["product_modules"] == [] and probe["product_libs"] == [] and probe["oracle_lib"]
    assert line["impl"] == "reference" and line["unit"] == "tok/s" and line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["nproc"] >= 1 and "cpu_model" in cb
    assert set(cb["threads"]) == {"default", "all"}

    sys.path.insert(0, ROOT)
    import bench

    class Args:
        workload, batch, gpus = "talker", 1, 1

    shape = bench.talker_shape(Args)
    assert line["config"] == bench.talker_config(Args, shape, [1], 1)
    assert line["config"]["algorithmic_bytes_per_step"] == 470455360  # 467,927,040 B of Q8_0 weights + F32 activations + the GET_ROWS row


def test_default_thread_rule_matches_the_reference():
    sys.path.insert(0, ROOT)
    import bench

    # src/cpu-parallelism.cpp:93-99
    assert [bench.default_threads(n) for n in (1, 2, 3, 4, 8, 16, 20)] == [1, 1, 1, 2, 4, 8, 10]
