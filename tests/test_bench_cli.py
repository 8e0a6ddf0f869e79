"""bench.py's JSON contract on the CPU: the reference arm (the reference's
own host packers from oracle/_ref, else the oracle's restatement) prints
one line with the keys the driver reads, for the A and B packing workloads.
The GPU arms are exercised on the GPU box."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run_reference(workload):
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--workload", workload,
                          "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=300, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


@pytest.mark.parametrize("workload", ["pack", "packb"])
def test_reference_arm_line(workload):
    d = _run_reference(workload)
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling", "dtype",
                "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["unit"] == "GB/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["config"]["workload"].startswith(workload + ":")
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] == 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"]


def test_unknown_epilogue_is_rejected():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--epilogue", "nope"], capture_output=True,
                         text=True, timeout=120, cwd=REPO)
    assert out.returncode != 0 and "packed_b" in out.stderr


def test_reference_arm_decode_uses_only_the_oracle():
    """The default workload's reference arm: one JSON line whose config equals
    the repo arm's, computed without loading the product library."""
    code = ("import sys, runpy; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '3'];"
            "runpy.run_path('bench.py', run_name='__main__');"
            "maps = open('/proc/self/maps').read();"
            "assert 'libspmm24' not in maps, 'product library loaded';"
            "assert 'spmm24' not in sys.modules")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "TFLOPS" and d["value"] > 0
    sys.path.insert(0, REPO)
    import argparse

    import bench

    ours = bench.workload_config(argparse.Namespace(workload="decode", dtype="f16"), 1)
    assert d["config"] == ours
    assert d["cpu_baseline"]["kind"] == "port" and d["e2e"]["value"] == d["value"]


def test_help_lists_the_default_line_switches():
    """The switches that shape the default line and the profiler cases are
    accepted (argument parsing only; the GPU arms run on the GPU box)."""
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--help"], capture_output=True, text=True,
                         timeout=120, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    for flag in ("--no-comparators", "--no-secondary", "--no-config4", "--no-extras", "--gather-mc", "--single",
                 "--single-group", "--workload", "--dtype", "--epilogue", "--impl"):
        assert flag in out.stdout, flag
