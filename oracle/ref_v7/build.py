"""Build oracle/_ref/libref_v7.so from the reference's own v7 kernel source.

    python oracle/ref_v7/build.py [/path/to/QMesh-AFD-TP3]

Test infrastructure only: the library is the reference's decode kernel, compiled
unmodified for sm_100a (its converts cvt.rn.f16x2.e2m1x2 / .e4m3x2 exist there),
used by tests/test_gpu_ref_v7.py to pin the CPU oracle to the reference's actual
arithmetic. Nothing under the product loads it. Skips quietly when the reference
tree is absent (the prebuilt file travels with the repository snapshot).
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE.parent / "_ref" / "libref_v7.so"
KERNEL = "gx/kernels/fp4_decode_moe_swz.cu"


def build(ref: str = "/root/reference") -> Path | None:
    src = Path(ref) / KERNEL
    if not src.is_file():
        return OUT if OUT.is_file() else None
    shim = HERE / "ref_v7_shim.cu"
    if OUT.is_file() and OUT.stat().st_mtime >= max(shim.stat().st_mtime, src.stat().st_mtime):
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
           "-Xcompiler", "-fPIC", "-shared", f'-DREF_KERNEL_FILE="{src}"', "-o", str(OUT), str(shim)]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else "/root/reference"))
