"""Fixed-order combine of per-rank BF16 partials (the reference's seam combine,
native/qmesh_afd_seam.cu:310-484): out = bf16(p0 + p1 + ... ) summed in FP32 in
list order with one rounding, or kept in FP32 (out_f32)."""

from __future__ import annotations

import ctypes

import torch

from . import _lib


def combine_ordered(parts: list[torch.Tensor], out: torch.Tensor | None = None, out_f32: bool = False,
                    stream=None) -> torch.Tensor:
    if not parts:
        raise ValueError("no partials to combine")
    rows = parts[0].shape[0]
    for p in parts:
        if p.dtype != torch.bfloat16 or p.shape != parts[0].shape or p.stride(1) != 1:
            raise TypeError("partials must be bf16 [rows, 5120] with unit column stride, all the same shape")
        if p.stride(0) != parts[0].stride(0):
            raise ValueError("partials must share one row stride")
    dev = parts[0].device
    if out is None:
        out = torch.empty(rows, _lib.HIDDEN, dtype=torch.float32 if out_f32 else torch.bfloat16, device=dev)
    arr = (ctypes.c_void_p * len(parts))(*[p.data_ptr() for p in parts])
    if stream is None:
        stream = torch.cuda.current_stream(dev).cuda_stream
    rc = _lib.load().qx_combine_ordered(arr, len(parts), parts[0].stride(0), ctypes.c_void_p(out.data_ptr()),
                                        out.stride(0), 1 if out_f32 else 0, rows, ctypes.c_void_p(stream))
    _lib.check(rc, "qx_combine_ordered")
    return out
