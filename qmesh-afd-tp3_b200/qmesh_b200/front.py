"""Producer side of the slice on the device (qx_quant_fp8, qx_route_topk).

* ``quant_fp8(x)``: BF16 activations [rows, 5120] -> FP8 e4m3 bytes and the
  dequant scale, per row or, as the reference's seam does, per post
  (native/qmesh_afd_seam.cu:9-16, p7/afd_overlay/afd_session.py:106-107). Inside
  one box the slice also takes the BF16 rows directly (QX_X_BF16), so this is the
  transport form for activations that cross processes or machines.
* ``route_topk(logits, k)``: softmax, top-k experts, weights renormalised to 1.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def quant_fp8(x: torch.Tensor, per_post: bool = False, q: torch.Tensor | None = None,
              inv: torch.Tensor | None = None, status: torch.Tensor | None = None,
              work: torch.Tensor | None = None, stream=None) -> tuple[torch.Tensor, torch.Tensor]:
    """(q uint8 [rows, 5120], inv float32 [rows] or [1]); status (int32 [1], device)
    receives QX_DEV_NONFINITE for a non-finite maximum."""
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != _lib.HIDDEN or x.stride(1) != 1:
        raise TypeError("x must be bf16 [rows, 5120] with unit column stride")
    rows, dev = x.shape[0], x.device
    if q is None:
        q = torch.empty(rows, _lib.HIDDEN, dtype=torch.uint8, device=dev)
    if inv is None:
        inv = torch.empty(1 if per_post else rows, dtype=torch.float32, device=dev)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=dev)
    if per_post and work is None:
        work = torch.empty(1, dtype=torch.int32, device=dev)
    if stream is None:
        stream = torch.cuda.current_stream(dev).cuda_stream
    rc = _lib.load().qx_quant_fp8(_p(x), x.stride(0), rows, 1 if per_post else 0, _p(q), q.stride(0), _p(inv),
                                  _p(work), _p(status), ctypes.c_void_p(stream))
    _lib.check(rc, "qx_quant_fp8")
    return q, inv


def route_topk(logits: torch.Tensor, topk: int = 6, stream=None) -> tuple[torch.Tensor, torch.Tensor]:
    """(ids int32 [rows, k], tw float32 [rows, k]) from FP32 router logits [rows, E]."""
    if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
        raise TypeError("logits must be float32 [rows, E] with unit column stride")
    rows, e = logits.shape
    ids = torch.empty(rows, topk, dtype=torch.int32, device=logits.device)
    tw = torch.empty(rows, topk, dtype=torch.float32, device=logits.device)
    if stream is None:
        stream = torch.cuda.current_stream(logits.device).cuda_stream
    rc = _lib.load().qx_route_topk(_p(logits), logits.stride(0), rows, e, topk, _p(ids), _p(tw),
                                   ctypes.c_void_p(stream))
    _lib.check(rc, "qx_route_topk")
    return ids, tw
