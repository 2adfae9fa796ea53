"""Graph-captured multi-layer driver for the slice.

The counterpart of the reference worker's `Layers` (gx/gx_ingest.py:282-466) and
its round-level spin (gx/gx_spin.py), over this library's tensor-core slice:

* per-(layer, width) CUDA graphs over ONE fixed buffer set of `graph_max` rows
  (16): a post of n rows replays the graph of width graph_rows(n) -- exactly 6
  for the decode post, the power-of-two bucket otherwise -- so a new width costs
  a graph per layer and no buffers; rows beyond `graph_max` run eagerly on a
  grow-only buffer set (doubling, as the reference caps retention);
* a round graph: every layer of a round in one graph, each layer first waiting
  (bounded, on the device) until the producer has published that layer's inputs
  by writing the round's sequence number into the layer's cell (device memory,
  written from the producer's own stream right after its input copies, so stream
  order puts the inputs in place first). A layer whose cell never arrives gives up after
  `spin_timeout_ms`, sets QX_DEV_TIMEOUT in `status` and the round completes
  anyway (its output for that layer is invalid), as the reference counts
  `round_timeouts`.

Padding rows of a graph width (n < width) carry ids -1 and contribute nothing.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .arena import Arena
from .expert_slice import SWIGLU_LIMIT, alloc_workspace, launch
from .routing import GRAPH_MAX, graph_rows

QX_DEV_TIMEOUT = 2


def _p(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


class _Buffers:
    """One input/output set of `cap` rows (FP8 x and its per-row scale, routing, out)."""

    def __init__(self, cap: int, topk: int, dev):
        self.cap = cap
        self.x = torch.zeros(cap, _lib.HIDDEN, dtype=torch.uint8, device=dev)
        self.inv = torch.ones(cap, dtype=torch.float32, device=dev)
        self.ids = torch.full((cap, topk), -1, dtype=torch.int32, device=dev)
        self.tw = torch.zeros(cap, topk, dtype=torch.float32, device=dev)
        self.out = torch.zeros(cap, _lib.HIDDEN, dtype=torch.bfloat16, device=dev)

    def stage(self, x: torch.Tensor, inv: torch.Tensor, ids: torch.Tensor, tw: torch.Tensor, width: int) -> None:
        n = x.shape[0]
        self.x[:n].copy_(x.view(torch.uint8) if x.dtype != torch.uint8 else x, non_blocking=True)
        self.inv[:n].copy_(inv.reshape(-1).expand(n) if inv.numel() == 1 else inv, non_blocking=True)
        self.ids[:n].copy_(ids, non_blocking=True)
        self.tw[:n].copy_(tw, non_blocking=True)
        if width > n:                      # padding rows: no expert, no contribution
            self.ids[n:width].fill_(-1)
            self.tw[n:width].zero_()
            self.inv[n:width].fill_(1.0)


class LayerDriver:
    """Per-(layer, width) graphs and a round graph of the slice over `arena`."""

    def __init__(self, arena: Arena, swiglu_limit: float = SWIGLU_LIMIT, topk: int = 6,
                 graph_max: int = GRAPH_MAX, spin_timeout_ms: float = 1000.0):
        if arena.layout != "tc":
            raise ValueError("the driver runs the tensor-core slice (arena layout 'tc')")
        self.arena = arena
        self.dev = arena.dev
        self.topk = topk
        self.graph_max = graph_max
        self.limit = float(max(swiglu_limit, 0.0))
        self.has_limit = swiglu_limit > 0
        self.spin_ns = int(spin_timeout_ms * 1e6)
        self.small = _Buffers(graph_max, topk, self.dev)
        self.ws = alloc_workspace(graph_max, topk, arena.a0, arena.a1, self.dev, "tc")
        self.graphs: dict[tuple[int, int], torch.cuda.CUDAGraph] = {}
        self.pool = torch.cuda.graph_pool_handle()
        self._big: tuple[_Buffers, torch.Tensor] | None = None
        # round state
        self.round_graph: torch.cuda.CUDAGraph | None = None
        self.round_rows = 0
        self.slots: list[_Buffers] = []
        self.cells = torch.zeros(arena.layers, dtype=torch.int32, device=self.dev)   # per layer: last published round
        self.seq = torch.zeros(1, dtype=torch.int32, device=self.dev)                # the round being served
        self.producer = torch.cuda.Stream(self.dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.dev)

    # -- per-(layer, width) graphs (gx_ingest.py:380-419) -------------------------
    def _run(self, li: int, r: int, buf: _Buffers, ws: torch.Tensor) -> None:
        launch(self.arena.view(li), buf.x[:r].view(torch.float8_e4m3fn), buf.ids[:r], buf.tw[:r], buf.out[:r],
               self.arena.a0, self.arena.a1, ws, x_scale=buf.inv[:r], swiglu_limit=self.limit,
               has_limit=self.has_limit, layout="tc")

    def capture(self, li: int, r: int) -> None:
        if r > self.graph_max:
            raise ValueError(f"graph width {r} > {self.graph_max}")
        saved = (self.small.ids[:r].clone(), self.small.tw[:r].clone())
        self.small.ids[:r].fill_(-1)          # warm up on neutral routing, not on whatever the buffers hold
        self.small.tw[:r].zero_()
        self._run(li, r, self.small, self.ws)
        torch.cuda.synchronize(self.dev)
        self.small.ids[:r].copy_(saved[0])
        self.small.tw[:r].copy_(saved[1])
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.pool):
            self._run(li, r, self.small, self.ws)
        self.graphs[(li, r)] = g

    def step(self, li: int, x: torch.Tensor, inv: torch.Tensor, ids: torch.Tensor, tw: torch.Tensor) -> torch.Tensor:
        """Serve layer `li` for a post of n = x.shape[0] rows; returns out [n, 5120]
        (a view of the driver's buffer, valid until the next step)."""
        n = x.shape[0]
        r = graph_rows(n)
        if r <= self.graph_max:
            self.small.stage(x, inv, ids, tw, r)
            if (li, r) not in self.graphs:
                self.capture(li, r)
            self.graphs[(li, r)].replay()
            return self.small.out[:n]
        cap = min(1 << max(0, (n - 1).bit_length()), _lib.MAX_ROWS)
        if n > cap:
            raise ValueError(f"post of {n} rows beyond the decode slice's {_lib.MAX_ROWS}; use the prefill slice")
        if self._big is None or self._big[0].cap < cap:
            self._big = (_Buffers(cap, self.topk, self.dev),
                         alloc_workspace(cap, self.topk, self.arena.a0, self.arena.a1, self.dev, "tc"))
        buf, ws = self._big
        buf.stage(x, inv, ids, tw, n)
        self._run(li, n, buf, ws)
        return buf.out[:n]

    # -- round graph (gx_ingest.py:421-466, gx_spin.py) ----------------------------
    def capture_round(self, rows: int) -> None:
        """One graph for a round of every layer at graph_rows(rows) rows; each layer
        waits for its cell, then runs on its own input slot."""
        r = graph_rows(rows)
        if r > self.graph_max:
            raise ValueError(f"round rows {rows} > {self.graph_max}")
        lib = _lib.load()
        self.round_rows = r
        self.slots = [_Buffers(r, self.topk, self.dev) for _ in range(self.arena.layers)]
        for li, buf in enumerate(self.slots):            # warm up outside the capture
            self._run(li, r, buf, self.ws)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.pool):
            st = torch.cuda.current_stream(self.dev).cuda_stream
            for li, buf in enumerate(self.slots):
                cell = ctypes.c_void_p(self.cells.data_ptr() + 4 * li)
                _lib.check(lib.qx_wait_cell(cell, _p(self.seq), self.spin_ns, _p(self.status), ctypes.c_void_p(st)),
                           "qx_wait_cell")
                self._run(li, r, buf, self.ws)
        self.round_graph = g

    def stage_layer(self, li: int, x, inv, ids, tw, seq: int) -> None:
        """Producer side (any time before or during the round): write layer li's
        inputs into its slot, then publish the round's sequence number in the
        layer's cell, both on the producer stream. The caller must not restage a
        layer while a round that reads it is still running."""
        self.producer.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(self.producer):
            self.slots[li].stage(x, inv, ids, tw, self.round_rows)
            self.cells[li:li + 1].fill_(seq)

    def replay_round(self, seq: int) -> None:
        """Serve one round: layer li runs once cells[li] == seq (published before or
        during the replay). Outputs: self.slots[li].out."""
        if self.round_graph is None:
            raise RuntimeError("capture_round() first")
        self.seq.fill_(seq)
        self.round_graph.replay()

    def round_timeouts(self) -> bool:
        """Whether a layer of the rounds since the last reset gave up waiting."""
        return bool(int(self.status.item()) & QX_DEV_TIMEOUT)

    def reset_status(self) -> None:
        self.status.zero_()
