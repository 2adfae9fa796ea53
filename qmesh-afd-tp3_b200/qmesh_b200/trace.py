"""NVTX ranges around the host-side phases of slice calls, off unless QX_NVTX=1
(the reference gates its worker's ranges the same way with GX_NVTX,
gx/gx_expert_worker.py:65-93), so an nsys or ncu range capture can pick out
staging, the slice, the exchange and the copies back."""

from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("QX_NVTX", "0") == "1"


@contextlib.contextmanager
def rng(name: str):
    if not ENABLED:
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
