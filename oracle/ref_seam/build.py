"""Build oracle/_ref/libref_seam.so from the reference's own seam kernels.

    python oracle/ref_seam/build.py [REFERENCE_ROOT]     # or QX_REFERENCE_ROOT=...

Test infrastructure only: the library is the reference's FP8 post quantiser
(seam_amax_kernel + seam_finish + seam_pack_kernel) and ordered combine
(seam_combine_kernel, seam_combine_vec_kernel) from native/qmesh_afd_seam.cu,
compiled unmodified for sm_100a, used by tests/test_gpu_ref_seam.py to pin
qx_quant_fp8 and qx_combine_ordered to the reference's arithmetic. Nothing under
the product loads it. Without a reference tree the prebuilt file (which travels
with the repository snapshot) is used as it is.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE.parent / "_ref" / "libref_seam.so"
KERNEL = "native/qmesh_afd_seam.cu"


def build(ref: str | None = None) -> Path | None:
    ref = ref or os.environ.get("QX_REFERENCE_ROOT")
    src = Path(ref) / KERNEL if ref else None
    if src is None or not src.is_file():
        return OUT if OUT.is_file() else None
    shim = HERE / "ref_seam_shim.cu"
    if OUT.is_file() and OUT.stat().st_mtime >= max(shim.stat().st_mtime, src.stat().st_mtime):
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
           "-Xcompiler", "-fPIC", "-shared", f'-DREF_SEAM_FILE="{src}"', "-o", str(OUT), str(shim)]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None))
