"""Build libqmesh_b200.so in-tree with nvcc for sm_100a (no GPU needed).

    python -m qmesh_b200.build          # from qmesh-afd-tp3_b200/ on sys.path
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

from ._lib import LIB_PATH, PKG_ROOT

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["csrc/qx_decode.cu", "csrc/qx_decode_tc.cu", "csrc/qx_nvf4_tile.cu", "csrc/qx_xchg.cu",
           "csrc/qx_prefill_tc.cu", "csrc/qx_front.cu"]
HEADERS = ["csrc/qx_ptx.cuh", "csrc/qx_tc.cuh"]
INCLUDE = PKG_ROOT.parent / "include"


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    if cand.is_file():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise FileNotFoundError("nvcc not found (set CUDA_HOME)")
    return found


def up_to_date(out: Path) -> bool:
    if not out.is_file():
        return False
    t = out.stat().st_mtime
    deps = [PKG_ROOT / s for s in SOURCES + HEADERS] + [INCLUDE / "qmesh_b200.h"]
    return all(d.stat().st_mtime <= t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    out = LIB_PATH
    if not force and up_to_date(out):
        return out
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           f"-I{INCLUDE}", "-o", str(out) + ".tmp", *[str(PKG_ROOT / s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(str(out) + ".tmp", out)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
