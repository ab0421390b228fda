"""Builds the CUDA library ``duck_gym_b200/_lib/libduck_b200.so`` for sm_100a.

The library exports only the C ABI of ``include/duck_b200.h``; it does not
link against torch.  ``python -m duck_gym_b200.build`` rebuilds it.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
SOURCES = sorted((PACKAGE / "csrc").glob("*.cu")) + sorted((PACKAGE / "csrc").glob("*.cuh")) + sorted(
    (PACKAGE / "csrc").glob("*.hpp")) + [ROOT / "include" / "duck_b200.h"]
LIB_DIR = PACKAGE / "_lib"
LIB_PATH = LIB_DIR / "libduck_b200.so"


def nvcc():
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(home) / "bin" / "nvcc"
    return str(path) if path.exists() else shutil.which("nvcc") or "nvcc"


def flags(verbose=False):
    f = [
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-lineinfo", "-O3", "-std=c++17",
        "--expt-relaxed-constexpr",
        # Host code parses the model in double; keep its rounding identical to
        # the reference loader (no contraction).
        "-Xcompiler", "-fPIC,-ffp-contract=off",
        "-ccbin", "/usr/bin/g++",
    ]
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def up_to_date():
    if not LIB_PATH.exists():
        return False
    built = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in SOURCES + [Path(__file__)])


def build_library(force=False, verbose=False):
    """Compile the library if any source is newer than it; return its path."""
    if not force and up_to_date():
        return LIB_PATH
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), *flags(verbose), "-shared", str(PACKAGE / "csrc" / "duck_b200.cu"), "-o", str(tmp)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + result.stdout + result.stderr)
    if verbose:
        sys.stderr.write(result.stdout + result.stderr)
    tmp.replace(LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv))
