"""ctypes binding of libqmesh_b200.so (the C ABI declared in include/qmesh_b200.h).

The library is built in-tree by ``qmesh_b200.build``. There is no fallback: if
the shared object is missing or fails to load, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent      # qmesh-afd-tp3_b200/
LIB_NAME = "libqmesh_b200.so"
LIB_PATH = PKG_ROOT / LIB_NAME

QX_OK = 0
QX_ERR_ARG = 1
QX_ERR_SHAPE = 2
QX_ERR_ALIGN = 3
QX_ERR_WORKSPACE = 4
QX_ERR_LAUNCH = 5
QX_ERR_DEVICE = 6
ERR_NAMES = {
    QX_ERR_ARG: "bad argument",
    QX_ERR_SHAPE: "unsupported shape",
    QX_ERR_ALIGN: "misaligned pointer or stride",
    QX_ERR_WORKSPACE: "workspace too small",
    QX_ERR_LAUNCH: "CUDA launch failed",
    QX_ERR_DEVICE: "no sm_100 device",
}

QX_DEV_BAD_ID = 1
QX_DEV_TIMEOUT = 2
QX_DEV_OVERFLOW = 4

QX_LAYOUT_TC = 0x54430001
QX_LAYOUT_FRAG = 0x46520002

QX_X_E4M3 = 0
QX_X_E4M3_POST = 1
QX_X_BF16 = 2

HIDDEN = 5120
MAX_ROWS = 64
MAX_TOPK = 8
PREFILL_MAX_ROWS = 8192
STATIC_MAX_ROWS = 8
STATIC_MAX_TOPK = 8
STATIC_MAX_WIDTH = 2304


class QxArena(ctypes.Structure):
    _fields_ = [
        ("w13", ctypes.c_void_p),
        ("w2", ctypes.c_void_p),
        ("g13", ctypes.c_void_p),
        ("g2", ctypes.c_void_p),
        ("n_experts", ctypes.c_int32),
        ("a0", ctypes.c_int32),
        ("a1", ctypes.c_int32),
        ("layout", ctypes.c_int32),
    ]


class QxSliceArgs(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p),
        ("x_scale", ctypes.c_void_p),
        ("x_stride", ctypes.c_int64),
        ("x_fmt", ctypes.c_int32),
        ("ids", ctypes.c_void_p),
        ("ids_int64", ctypes.c_int32),
        ("tw", ctypes.c_void_p),
        ("rows", ctypes.c_int32),
        ("topk", ctypes.c_int32),
        ("c0", ctypes.c_int32),
        ("c1", ctypes.c_int32),
        ("swiglu_limit", ctypes.c_float),
        ("has_limit", ctypes.c_int32),
        ("out", ctypes.c_void_p),
        ("out_stride", ctypes.c_int64),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


XCHG_MAX_RANKS = 8
IPC_HANDLE_BYTES = 64


class QxXchgArgs(ctypes.Structure):
    _fields_ = [
        ("bufs", ctypes.c_void_p * XCHG_MAX_RANKS),
        ("part", ctypes.c_void_p),
        ("part_stride", ctypes.c_int64),
        ("shared", ctypes.c_void_p),
        ("shared_stride", ctypes.c_int64),
        ("out", ctypes.c_void_p),
        ("out_stride", ctypes.c_int64),
        ("status", ctypes.c_void_p),
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("dst", ctypes.c_int32),
        ("rows", ctypes.c_int32),
        ("rows_max", ctypes.c_int32),
    ]


# (name, restype, argtypes) of every exported entry point in include/qmesh_b200.h
SIGNATURES = [
    ("qx_arena_w13_bytes", ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32]),
    ("qx_arena_w2_bytes", ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32]),
    ("qx_slice_workspace_bytes", ctypes.c_size_t,
     [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    ("qx_slice_decode", ctypes.c_int,
     [ctypes.POINTER(QxArena), ctypes.POINTER(QxSliceArgs), ctypes.c_void_p]),
    ("qx_slice_decode_static", ctypes.c_int,
     [ctypes.POINTER(QxArena), ctypes.POINTER(QxSliceArgs), ctypes.c_void_p]),
    ("qx_slice_decode_static_status", ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), ctypes.c_void_p]),
    ("qx_combine_ordered", ctypes.c_int,
     [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p,
      ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]),
    ("qx_status_read", ctypes.c_int,
     [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32), ctypes.c_void_p]),
    ("qx_arena_tc_w13_bytes", ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32]),
    ("qx_arena_tc_w2_bytes", ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32]),
    ("qx_slice_workspace_tc_bytes", ctypes.c_size_t,
     [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    ("qx_slice_decode_tc", ctypes.c_int,
     [ctypes.POINTER(QxArena), ctypes.POINTER(QxSliceArgs), ctypes.c_void_p]),
    ("qx_diag_nvf4_tile", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
      ctypes.c_void_p, ctypes.c_void_p]),
    ("qx_prefill_workspace_bytes", ctypes.c_size_t,
     [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    ("qx_slice_prefill_tc", ctypes.c_int,
     [ctypes.POINTER(QxArena), ctypes.POINTER(QxSliceArgs), ctypes.c_void_p, ctypes.c_void_p]),
    ("qx_quant_fp8", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    ("qx_route_topk", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
      ctypes.c_void_p, ctypes.c_void_p]),
    ("qx_wait_cell", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]),
    ("qx_xchg_bytes", ctypes.c_size_t, [ctypes.c_int32]),
    ("qx_xchg_alloc", ctypes.c_int, [ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p)]),
    ("qx_xchg_free", ctypes.c_int, [ctypes.c_void_p]),
    ("qx_ipc_handle", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    ("qx_ipc_open", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    ("qx_ipc_close", ctypes.c_int, [ctypes.c_void_p]),
    ("qx_slice_decode_tc_xchg", ctypes.c_int,
     [ctypes.POINTER(QxArena), ctypes.POINTER(QxSliceArgs), ctypes.POINTER(QxXchgArgs), ctypes.c_void_p]),
    ("qx_slice_decode_tc_shared", ctypes.c_int,
     [ctypes.POINTER(QxArena), ctypes.POINTER(QxSliceArgs), ctypes.POINTER(QxArena), ctypes.POINTER(QxXchgArgs),
      ctypes.c_void_p]),
    ("qx_combine_p2p", ctypes.c_int, [ctypes.POINTER(QxXchgArgs), ctypes.c_void_p]),
    ("qx_version", ctypes.c_char_p, []),
]

_LIB = None


class QxError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""


def lib_path() -> Path:
    env = os.environ.get("QX_LIB")
    return Path(env) if env else LIB_PATH


def load() -> ctypes.CDLL:
    """Load the library once; raise (never fall back) if it is not built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = lib_path()
    if not path.is_file():
        raise ImportError(f"{path} is not built; run `python -m qmesh_b200.build` "
                          "(or __graft_entry__.build())")
    lib = ctypes.CDLL(str(path))
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != QX_OK:
        raise QxError(f"{what}: {ERR_NAMES.get(rc, 'error')} (status {rc})")
