"""qmesh_b200: the routed-expert NVFP4 SwiGLU slice of QMesh AFD-TP3, rebuilt for B200.

Host side of the C ABI in include/qmesh_b200.h (libqmesh_b200.so, sm_100a).
"""

from . import _lib, nvfp4, routing  # noqa: F401

__all__ = ["_lib", "nvfp4", "routing"]
