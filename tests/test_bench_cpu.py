"""CPU checks of bench.py's contract: default workloads, the shared config
object of both arms, and a reference arm that runs the reference's restore on
host cores without loading any library of this repository."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _args(*argv: str):
    sys.path.insert(0, str(ROOT))
    import bench

    old = sys.argv
    sys.argv = ["bench.py", *argv]
    try:
        return bench, bench.parse_args()
    finally:
        sys.argv = old


def test_default_workloads_follow_the_gpu_count() -> None:
    _, one = _args()
    _, two = _args("--gpus", "2")
    _, moe = _args("--workload", "mixtral-8x7b")
    assert one.workload == "llama3-8b" and two.workload == "llama3-70b"
    assert moe.compare_full_copy  # config 4 times the pinned full copy beside the switch


def test_both_arms_name_the_workload_with_the_same_config() -> None:
    bench, args = _args("--gpus", "2")
    spec, desc = bench.workload_spec(args, 2, 0)
    cfg = bench.workload_config(args, desc, spec.nbytes)
    assert cfg == bench.workload_config(args, desc, spec.nbytes)
    assert set(cfg) == {"workload", "policy", "scale", "escapes", "split", "l2"}
    assert "tp=2" in cfg["workload"] and spec.tp == 2


def test_reference_arm_runs_on_host_cores_without_product_code() -> None:
    """A small run of --impl reference in a fresh process: one JSON line with the
    reference fields, and libwarpshift_b200.so never mapped into the process."""
    code = (
        "import runpy, sys\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'qwen2-0.5b', '--layers', '1',"
        " '--steps', '2', '--warmup', '1']\n"
        "try:\n"
        "    runpy.run_path('bench.py', run_name='__main__')\n"
        "finally:\n"
        "    maps = open('/proc/self/maps').read()\n"
        "    print('MAPPED_PRODUCT' if 'libwarpshift_b200' in maps else 'NO_PRODUCT_LIBRARY')\n"
    )
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0 and line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert set(line["config"]) == {"workload", "policy", "scale", "escapes", "split", "l2"}
    assert "NO_PRODUCT_LIBRARY" in out.stdout


if __name__ == "__main__":
    sys.exit(pytest.main([__file__, "-q"]))
