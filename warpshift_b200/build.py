"""Build the in-tree native library ``libwarpshift_b200.so`` with nvcc for sm_100a.

Run ``python -m warpshift_b200.build`` (or ``__graft_entry__.build()``). The
library is linked against the static CUDA runtime so it only needs the driver at
run time, and it is placed next to this file so it ships with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libwarpshift_b200.so"
SOURCES = ["ws_apply.cu", "ws_gpu_encoder.cu", "ws_hash.cu", "ws_encoder.cpp", "ws_plan.cpp", "ws_persist.cpp"]
HEADERS = ["ws_format.h", "ws_encoder.h", "ws_kernels.h", "ws_gpu_encoder.h", "ws_plan_internal.h", "ws_guard.h", "../../include/warpshift_b200.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the warpshift_b200 CUDA library cannot be built")
    return found


def is_stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    inputs = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [Path(__file__)]
    return any(p.stat().st_mtime > built for p in inputs)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not is_stale():
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [
        nvcc(),
        "-O3",
        "-std=c++17",
        *ARCH,
        "-lineinfo",
        "-Xcompiler",
        "-fPIC,-O3,-pthread,-fvisibility=hidden",
        "-Xptxas",
        "-v" if verbose else "-O3",
        "-shared",
        "-o",
        str(tmp),
        *[str(CSRC / s) for s in SOURCES],
    ]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    if verbose:
        sys.stderr.write(result.stderr)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
