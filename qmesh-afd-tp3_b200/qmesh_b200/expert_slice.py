"""The routed-expert slice call: the drop-in for the reference's decode body.

Two forms over the same C entry points (qx_slice_decode_tc for a tensor-core
layout arena, qx_slice_decode for a register-dequant layout arena):

* ``expert_slice(layer, x, ids, tw, c0=, c1=, x_scale=)`` -- the north-star form:
  FP8 e4m3 activations [rows, 5120] with an FP32 dequant scale per row (or one
  per post), top-k ids and weights, a column range [c0, c1); returns the BF16
  [rows, 5120] partial.
* ``make_body(arena, swiglu_limit)`` -> ``body(li, r, x, ids, tw, out, ws13, ws2, a1g)``
  with the signature, argument meaning and errors of gx/gx_decode_swz.py:148-179
  (x is the ingested BF16 activation; out is written in place).

Everything is launched on the current torch stream, allocates nothing once the
workspace exists, and never synchronises the host, so both forms can be captured
in a CUDA graph.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .arena import Arena
from .trace import rng

SWIGLU_LIMIT = 10.0


def workspace_bytes(rows: int, topk: int, c0: int, c1: int, layout: str = "tc") -> int:
    lib = _lib.load()
    fn = lib.qx_slice_workspace_tc_bytes if layout == "tc" else lib.qx_slice_workspace_bytes
    n = fn(rows, topk, c0, c1)
    if n == 0:
        raise ValueError(f"no workspace for rows={rows} topk={topk} columns [{c0}, {c1})")
    return n


def alloc_workspace(rows: int, topk: int, c0: int, c1: int, device, layout: str = "tc") -> torch.Tensor:
    """Workspace for calls of up to `rows` rows over `c1 - c0` columns."""
    return torch.empty(workspace_bytes(rows, topk, c0, c1, layout), dtype=torch.uint8, device=device)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _slice_args(x, ids, tw, out, c0, c1, workspace, x_scale, swiglu_limit, has_limit) -> _lib.QxSliceArgs:
    rows = x.shape[0]
    if x.dtype == torch.bfloat16:
        fmt = _lib.QX_X_BF16
        esz = 2
    elif x.dtype in (torch.float8_e4m3fn, torch.uint8):
        if x_scale is None:
            raise TypeError("FP8 activations need x_scale (per row [rows] or per post [1])")
        if x_scale.dtype != torch.float32:
            raise TypeError(f"x_scale must be float32, got {x_scale.dtype}")
        fmt = _lib.QX_X_E4M3 if x_scale.numel() == rows else _lib.QX_X_E4M3_POST
        if x_scale.numel() not in (1, rows):
            raise ValueError(f"x_scale has {x_scale.numel()} values for {rows} rows")
        esz = 1
    else:
        raise TypeError(f"x must be bf16 or e4m3, got {x.dtype}")
    if ids.dtype not in (torch.int32, torch.int64) or tw.dtype != torch.float32 or out.dtype != torch.bfloat16:
        raise TypeError(f"ids/tw/out must be int32|int64/f32/bf16, got {ids.dtype}/{tw.dtype}/{out.dtype}")
    if ids.shape != tw.shape or ids.shape[0] != rows or out.shape[0] < rows:
        raise ValueError(f"shape mismatch: x {tuple(x.shape)} ids {tuple(ids.shape)} tw {tuple(tw.shape)} "
                         f"out {tuple(out.shape)}")
    if x.shape[1] != _lib.HIDDEN or out.shape[1] != _lib.HIDDEN:
        raise ValueError(f"hidden size must be {_lib.HIDDEN}")
    if not (ids.is_contiguous() and tw.is_contiguous()) or x.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("ids/tw must be contiguous and x/out rows unit-stride")
    return _lib.QxSliceArgs(
        _ptr(x), _ptr(x_scale), x.stride(0) * esz, fmt,
        _ptr(ids), 1 if ids.dtype == torch.int64 else 0, _ptr(tw),
        rows, ids.shape[1], c0, c1, float(swiglu_limit), 1 if has_limit else 0,
        _ptr(out), out.stride(0), _ptr(workspace), workspace.numel())


def launch(view: _lib.QxArena, x: torch.Tensor, ids: torch.Tensor, tw: torch.Tensor, out: torch.Tensor,
           c0: int, c1: int, workspace: torch.Tensor, x_scale: torch.Tensor | None = None,
           swiglu_limit: float = SWIGLU_LIMIT, has_limit: bool = True, stream=None, layout: str = "tc",
           xchg: _lib.QxXchgArgs | None = None, shared: _lib.QxArena | None = None) -> None:
    """Validate and launch one slice call (no allocation, no host sync). `layout` is
    the arena's: "tc" runs qx_slice_decode_tc, "frag" qx_slice_decode. With `xchg`
    (tensor-core layout only) the call also combines the ranks' partials:
    qx_slice_decode_tc_xchg, see `shard.P2PExchange.slice_combine`. With
    `shared` (the view of a one-expert tensor-core arena) the same kernel also
    runs that shared expert over every row with weight 1 and adds its BF16
    output after the routed partials (qx_slice_decode_tc_shared)."""
    lib = _lib.load()
    args = _slice_args(x, ids, tw, out, c0, c1, workspace, x_scale, swiglu_limit, has_limit)
    if stream is None:
        stream = torch.cuda.current_stream(x.device).cuda_stream
    if shared is not None:
        if layout != "tc":
            raise ValueError("the shared expert runs on the tensor-core slice (layout 'tc')")
        with rng("qx.slice_shared"):
            rc = lib.qx_slice_decode_tc_shared(ctypes.byref(view), ctypes.byref(args), ctypes.byref(shared),
                                               ctypes.byref(xchg) if xchg is not None else None,
                                               ctypes.c_void_p(stream))
        _lib.check(rc, "qx_slice_decode_tc_shared")
        return
    if xchg is not None:
        if layout != "tc":
            raise ValueError("the fused rank combine runs on the tensor-core slice (layout 'tc')")
        with rng("qx.slice_xchg"):
            rc = lib.qx_slice_decode_tc_xchg(ctypes.byref(view), ctypes.byref(args), ctypes.byref(xchg),
                                             ctypes.c_void_p(stream))
        _lib.check(rc, "qx_slice_decode_tc_xchg")
        return
    name = "qx_slice_decode_tc" if layout == "tc" else "qx_slice_decode"
    with rng("qx.slice"):
        rc = getattr(lib, name)(ctypes.byref(view), ctypes.byref(args), ctypes.c_void_p(stream))
    _lib.check(rc, name)


def expert_slice(arena: Arena, li: int, x: torch.Tensor, ids: torch.Tensor, tw: torch.Tensor,
                 c0: int | None = None, c1: int | None = None, x_scale: torch.Tensor | None = None,
                 out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                 swiglu_limit: float = SWIGLU_LIMIT) -> torch.Tensor:
    """BF16 [rows, 5120] partial of the routed experts over columns [c0, c1)."""
    c0 = arena.a0 if c0 is None else c0
    c1 = arena.a1 if c1 is None else c1
    rows = x.shape[0]
    if out is None:
        out = torch.empty(rows, _lib.HIDDEN, dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        workspace = alloc_workspace(rows, ids.shape[1], c0, c1, x.device, arena.layout)
    launch(arena.view(li), x, ids, tw, out, c0, c1, workspace, x_scale=x_scale,
           swiglu_limit=max(swiglu_limit, 0.0), has_limit=swiglu_limit > 0, layout=arena.layout)
    return out


def device_status(workspace: torch.Tensor) -> int:
    """QX_DEV_* bits the last call on this workspace recorded (synchronises)."""
    st = ctypes.c_uint32(0)
    stream = torch.cuda.current_stream(workspace.device).cuda_stream
    _lib.check(_lib.load().qx_status_read(_ptr(workspace), ctypes.byref(st), ctypes.c_void_p(stream)),
               "qx_status_read")
    return int(st.value)


def make_body(arena: Arena, swiglu_limit: float, max_rows: int = 16, topk: int = 6):
    """``body(li, r, x, ids, tw, out, ws13, ws2, a1g)`` over the arena's own tensors.

    Mirrors gx/gx_decode_swz.py:148-179: x bf16 [r, 5120] (ingested), ids int32,
    tw f32, out bf16, all [r, ...]; ws13/ws2/a1g are accepted for signature
    compatibility. The kernel's scratch is this body's own workspace, sized once
    here for `max_rows`, so replays allocate nothing.
    """
    _lib.load()
    has_limit = bool(swiglu_limit > 0)
    limit = float(max(swiglu_limit, 0.0))
    ws = alloc_workspace(max_rows, topk, arena.a0, arena.a1, arena.dev, arena.layout)

    def body(li: int, r: int, x, ids, tw, out, ws13=None, ws2=None, a1g=None) -> None:
        if not arena.loaded(li):
            raise RuntimeError(f"layer {li} is not loaded in the arena")
        if (ids.dtype is not torch.int32 or tw.dtype is not torch.float32
                or x.dtype is not torch.bfloat16 or out.dtype is not torch.bfloat16):
            raise TypeError(
                f"decode body: ids/tw/x/out must be int32/f32/bf16/bf16, "
                f"got {ids.dtype}/{tw.dtype}/{x.dtype}/{out.dtype}")
        if not 1 <= r <= max_rows:
            raise ValueError(f"row count {r} outside 1..{max_rows}")
        launch(arena.view(li), x[:r], ids[:r], tw[:r], out[:r], arena.a0, arena.a1, ws,
               swiglu_limit=limit, has_limit=has_limit, layout=arena.layout)
    return body


# ---------------------------------------------------------------- prefill (W4A4)

def prefill_workspace_bytes(rows: int, topk: int, c0: int, c1: int, n_experts: int) -> int:
    n = _lib.load().qx_prefill_workspace_bytes(rows, topk, c0, c1, n_experts)
    if n == 0:
        raise ValueError(f"no prefill workspace for rows={rows} topk={topk} columns [{c0}, {c1}) E={n_experts}")
    return n


def alloc_prefill_workspace(rows: int, topk: int, c0: int, c1: int, n_experts: int, device) -> torch.Tensor:
    return torch.empty(prefill_workspace_bytes(rows, topk, c0, c1, n_experts), dtype=torch.uint8, device=device)


def launch_prefill(view: _lib.QxArena, x: torch.Tensor, ids: torch.Tensor, tw: torch.Tensor, a2: torch.Tensor,
                   out: torch.Tensor, c0: int, c1: int, workspace: torch.Tensor, x_scale: torch.Tensor | None = None,
                   swiglu_limit: float = SWIGLU_LIMIT, has_limit: bool = True, stream=None) -> None:
    """One W4A4 prefill slice call (qx_slice_prefill_tc): the reference's CUTLASS
    prefill body (gx/gx_ingest.py:190-246) on the tensor-core arena. `a2` is the
    layer's calibrated FP32 activation scale per expert ([n_experts], device)."""
    lib = _lib.load()
    if a2.dtype != torch.float32 or a2.dim() != 1 or a2.device != x.device:
        raise TypeError("a2 must be a float32 [n_experts] tensor on the activations' device")
    args = _slice_args(x, ids, tw, out, c0, c1, workspace, x_scale, swiglu_limit, has_limit)
    if stream is None:
        stream = torch.cuda.current_stream(x.device).cuda_stream
    with rng("qx.prefill"):
        rc = lib.qx_slice_prefill_tc(ctypes.byref(view), ctypes.byref(args), _ptr(a2), ctypes.c_void_p(stream))
    _lib.check(rc, "qx_slice_prefill_tc")


def prefill_slice(arena: Arena, li: int, x: torch.Tensor, ids: torch.Tensor, tw: torch.Tensor, a2: torch.Tensor,
                  c0: int | None = None, c1: int | None = None, x_scale: torch.Tensor | None = None,
                  out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                  swiglu_limit: float = SWIGLU_LIMIT) -> torch.Tensor:
    """BF16 [rows, 5120] partial of a prefill chunk over columns [c0, c1) (W4A4)."""
    if arena.layout != "tc":
        raise ValueError("the prefill slice needs a tensor-core layout arena")
    c0 = arena.a0 if c0 is None else c0
    c1 = arena.a1 if c1 is None else c1
    rows = x.shape[0]
    if out is None:
        out = torch.empty(rows, _lib.HIDDEN, dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        workspace = alloc_prefill_workspace(rows, ids.shape[1], c0, c1, arena.n_experts, x.device)
    launch_prefill(arena.view(li), x, ids, tw, a2, out, c0, c1, workspace, x_scale=x_scale,
                   swiglu_limit=max(swiglu_limit, 0.0), has_limit=swiglu_limit > 0)
    return out


# ---------------------------------------------------------------- host-buffer calls

def _al16(n: int) -> int:
    return (n + 15) & ~15


class HostSlice:
    """Slice calls whose inputs and output live in host memory.

    For a caller that receives a layer's activations and routing on the host (a
    transport that lands in host memory, or a test harness): each call packs
    x (FP8 e4m3 [rows, 5120]), its per-row FP32 scale, ids and tw into one pinned
    staging buffer, moves them with ONE host-to-device copy, runs the slice on
    views of the device copy and brings the BF16 output back with one
    device-to-host copy, without synchronising the host. The copies run on two
    side streams of their own, so call k+1's inputs move while call k computes
    and call k's output moves while call k+1 computes; the slice itself runs on
    the caller's current stream, after its inputs have landed. Two staging slots
    alternate, each guarded by events. Without `out`, the returned host tensor
    belongs to that call's slot and is overwritten by the call after next (a
    caller that keeps outputs passes `out`, or copies); with `out` (a host BF16
    tensor [rows, 5120], pinned for an asynchronous copy) the output lands there
    and is the caller's to keep. Either way, read it after `synchronize()`
    (host) or `join(stream)` (device ordering) or a device-wide synchronisation.

    With `xchg` (a `shard.P2PExchange`) every rank of the column split calls it
    once per step with the same inputs: each call runs the fused slice + rank
    combine, the output rank's call returns the combined output and the other
    ranks' calls return None (they copy nothing back). With `shared` (the view of
    a one-expert tensor-core arena) the output rank's kernel (or, without
    `xchg`, the one kernel) also runs config 2's shared expert and adds it last.
    """

    def __init__(self, arena: Arena, rows: int, topk: int = 6, c0: int | None = None, c1: int | None = None,
                 swiglu_limit: float = SWIGLU_LIMIT, slots: int = 2, xchg=None, shared: _lib.QxArena | None = None):
        if (xchg is not None or shared is not None) and arena.layout != "tc":
            raise ValueError("the fused combine and the shared expert run on the tensor-core arena")
        if xchg is not None and shared is not None and xchg.rank != xchg.dst:
            raise ValueError("only the output rank runs the shared expert")
        self.xchg, self.shared = xchg, shared
        self.arena = arena
        self.rows, self.topk = rows, topk
        self.c0 = arena.a0 if c0 is None else c0
        self.c1 = arena.a1 if c1 is None else c1
        self.limit = float(max(swiglu_limit, 0.0))
        self.has_limit = swiglu_limit > 0
        dev = arena.dev
        self.o_x = 0
        self.o_s = _al16(rows * _lib.HIDDEN)
        self.o_i = self.o_s + _al16(rows * 4)
        self.o_t = self.o_i + _al16(rows * topk * 4)
        self.nbytes = self.o_t + _al16(rows * topk * 4)
        self.host = [torch.empty(self.nbytes, dtype=torch.uint8).pin_memory() for _ in range(slots)]
        self.dev = [torch.empty(self.nbytes, dtype=torch.uint8, device=dev) for _ in range(slots)]
        self.out_d = [torch.empty(rows, _lib.HIDDEN, dtype=torch.bfloat16, device=dev) for _ in range(slots)]
        self.out_h = [torch.empty(rows, _lib.HIDDEN, dtype=torch.bfloat16).pin_memory() for _ in range(slots)]
        self.in_stream = torch.cuda.Stream(dev)
        self.out_stream = torch.cuda.Stream(dev)
        self.ev_in = [torch.cuda.Event() for _ in range(slots)]     # the slot's inputs have landed
        self.ev_done = [torch.cuda.Event() for _ in range(slots)]   # the slot's slice has run
        self.ev_out = [torch.cuda.Event() for _ in range(slots)]    # the slot's output has reached the host
        self.used = [False] * slots
        self.last: int | None = None
        self.ws = alloc_workspace(rows, topk, self.c0, self.c1, dev, arena.layout)
        self.k = 0

    def _views(self, buf: torch.Tensor, n: int):
        x = buf[self.o_x:self.o_x + n * _lib.HIDDEN].view(n, _lib.HIDDEN)
        s = buf[self.o_s:self.o_s + n * 4].view(torch.float32)
        i = buf[self.o_i:self.o_i + n * self.topk * 4].view(torch.int32).view(n, self.topk)
        t = buf[self.o_t:self.o_t + n * self.topk * 4].view(torch.float32).view(n, self.topk)
        return x, s, i, t

    def __call__(self, li: int, x: torch.Tensor, x_scale: torch.Tensor, ids: torch.Tensor,
                 tw: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor | None:
        n = x.shape[0]
        if not 1 <= n <= self.rows or ids.shape != (n, self.topk) or tw.shape != (n, self.topk):
            raise ValueError(f"call of {n} rows / ids {tuple(ids.shape)} outside this HostSlice ({self.rows} x {self.topk})")
        if out is not None and (out.device.type != "cpu" or out.dtype != torch.bfloat16
                                or tuple(out.shape) != (n, _lib.HIDDEN)):
            raise TypeError(f"out must be a host bf16 [{n}, {_lib.HIDDEN}] tensor")
        k = self.k
        self.k = (k + 1) % len(self.host)
        if self.used[k]:
            # The slot's previous call has left it: inputs consumed, output copied out
            # (so its host buffers and its device output may be reused).
            self.ev_out[k].synchronize()
        with rng("qx.host_stage"):
            hx, hs, hi, ht = self._views(self.host[k], n)
            hx.copy_(x.view(torch.uint8) if x.dtype != torch.uint8 else x)
            hs.copy_(x_scale.reshape(-1))
            hi.copy_(ids)
            ht.copy_(tw)
        stream = torch.cuda.current_stream(self.arena.dev)
        used = self.o_t + _al16(n * self.topk * 4) if n == self.rows else self.nbytes
        if self.used[k]:
            self.in_stream.wait_event(self.ev_done[k])     # the slot's previous slice has read its inputs
        with rng("qx.h2d"), torch.cuda.stream(self.in_stream):
            self.dev[k][:used].copy_(self.host[k][:used], non_blocking=True)
        self.ev_in[k].record(self.in_stream)
        stream.wait_event(self.ev_in[k])
        dx, ds, di, dt = self._views(self.dev[k], n)
        if self.xchg is not None:
            self.xchg.slice_combine(self.arena.view(li), dx.view(torch.float8_e4m3fn), di, dt, self.out_d[k][:n],
                                    self.c0, self.c1, self.ws, x_scale=ds, shared_expert=self.shared,
                                    stream=stream.cuda_stream, swiglu_limit=self.limit, has_limit=self.has_limit)
        else:
            launch(self.arena.view(li), dx.view(torch.float8_e4m3fn), di, dt, self.out_d[k][:n], self.c0, self.c1,
                   self.ws, x_scale=ds, swiglu_limit=self.limit, has_limit=self.has_limit,
                   stream=stream.cuda_stream, layout=self.arena.layout, shared=self.shared)
        self.ev_done[k].record(stream)
        if self.xchg is not None and self.xchg.rank != self.xchg.dst:
            # a sender: nothing comes back; the slot is free once its slice has run
            self.ev_out[k].record(stream)
            self.used[k] = True
            self.last = k
            return None
        self.out_stream.wait_event(self.ev_done[k])
        dst = self.out_h[k][:n] if out is None else out
        with rng("qx.d2h"), torch.cuda.stream(self.out_stream):
            dst.copy_(self.out_d[k][:n], non_blocking=True)
        self.ev_out[k].record(self.out_stream)
        self.used[k] = True
        self.last = k
        return dst

    def order_after(self, stream=None) -> None:
        """Order the next calls' input copies after the work queued so far on
        `stream` (default: the current stream), e.g. a timing event."""
        self.in_stream.wait_stream(stream or torch.cuda.current_stream(self.arena.dev))

    def join(self, stream=None) -> None:
        """Order `stream` (default: the current stream) after every call's output copy."""
        if self.last is not None:
            (stream or torch.cuda.current_stream(self.arena.dev)).wait_event(self.ev_out[self.last])

    def synchronize(self) -> None:
        """Block the host until every call's output is in host memory."""
        if self.last is not None:
            self.ev_out[self.last].synchronize()
