"""Column-split tensor parallelism of the routed experts across the GPUs of one box.

The reference splits every expert's 2304 intermediate columns across machines
(NODE-A [0:576), NODE-B [576:1440), NODE-C [1440:2304); pack/build_packs.py:50)
and sums the BF16 partials on NODE-A in FP32 in a fixed order
(native/qmesh_afd_seam.cu:310-361, README.md:88-90). Inside one B200 box the
ranks are GPUs: rank r holds columns [r*2304/N, (r+1)*2304/N) of every expert,
computes its partial from replicated x/ids/tw, and the partials meet on the
output rank, summed in rank order with one BF16 rounding.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

INTER = 2304


def shard_range(rank: int, world: int, inter: int = INTER, align: int = 32) -> tuple[int, int]:
    """Contiguous equal column shard of `rank`; widths must stay `align`-aligned."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if inter % world or (inter // world) % align:
        raise ValueError(f"{inter} columns do not split into {world} {align}-aligned shards")
    w = inter // world
    return rank * w, (rank + 1) * w


def gather_partials(part: torch.Tensor, group=None, out_list: list[torch.Tensor] | None = None) -> list[torch.Tensor]:
    """All ranks' partials, in rank order (index i = rank i's partial)."""
    world = dist.get_world_size(group)
    if out_list is None:
        out_list = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(out_list, part, group=group)
    return out_list


def combine_across_ranks(part: torch.Tensor, group=None, dst: int = 0, shared: torch.Tensor | None = None,
                         out: torch.Tensor | None = None,
                         combine: Callable[..., torch.Tensor] | None = None,
                         gathered: list[torch.Tensor] | None = None) -> torch.Tensor | None:
    """Rank-ordered FP32 combine of every rank's BF16 partial on rank `dst`.

    All ranks take the same collective steps; only `dst` returns the combined
    BF16 output (bf16(p0 + p1 + ... [+ shared])), the others return None.
    `combine` defaults to the device kernel (qmesh_b200.combine.combine_ordered).
    """
    if combine is None:
        from .combine import combine_ordered as combine
    parts = gather_partials(part, group, gathered)
    if dist.get_rank(group) != dst:
        return None
    if shared is not None:
        parts = list(parts) + [shared]
    return combine(parts, out=out)


def row_bounds(rows: int, world: int) -> list[int]:
    """Row block boundaries of the row-split combine: rank k sums rows [b[k], b[k+1])."""
    return [k * rows // world for k in range(world + 1)]


def combine_rows_across_ranks(part: torch.Tensor, group=None, dst: int = 0, out: torch.Tensor | None = None,
                              combine: Callable[..., torch.Tensor] | None = None,
                              recv: torch.Tensor | None = None, mine: torch.Tensor | None = None,
                              spare: torch.Tensor | None = None) -> torch.Tensor | None:
    """The rank-ordered FP32 combine of `combine_across_ranks`, split by rows.

    For partials of many rows (a prefill chunk): an all-to-all hands rank k rows
    [b[k], b[k+1]) of every rank's partial (`row_bounds`), rank k sums them in
    rank order with one BF16 rounding, and the output rank `dst` collects the
    combined row blocks (an all-gather when the rows divide evenly, the other
    ranks receiving into `spare` ([rows, 5120]); else point-to-point). Every
    element is the same sum in the same order as in `combine_across_ranks`, so
    the bytes are identical; each rank moves (N-1)/N of one partial and the
    output rank receives (N-1)/N of one output, where the gather brings N-1
    whole partials to one rank. Needs at least one row per rank. `recv`
    ([N x rows of this rank's block, 5120]) and `mine` ([rows of this rank's
    block, 5120]) may be passed in to avoid allocating per call. Only `dst`
    returns the output.
    """
    if combine is None:
        from .combine import combine_ordered as combine
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    rows, hid = part.shape
    if rows < world:
        raise ValueError(f"{rows} rows cannot give each of {world} ranks a row block")
    b = row_bounds(rows, world)
    n_me = b[rank + 1] - b[rank]
    if recv is None:
        recv = torch.empty(world * n_me, hid, dtype=part.dtype, device=part.device)
    dist.all_to_all_single(recv, part.contiguous(), output_split_sizes=[n_me] * world,
                           input_split_sizes=[b[k + 1] - b[k] for k in range(world)], group=group)
    parts = [recv[j * n_me:(j + 1) * n_me] for j in range(world)]
    if rank == dst:
        if out is None:
            out = torch.empty(rows, hid, dtype=part.dtype, device=part.device)
        target = out[b[rank]:b[rank + 1]]
    else:
        target = mine if mine is not None else torch.empty(n_me, hid, dtype=part.dtype, device=part.device)
    res = combine(parts, out=target)
    if res is not None and res.data_ptr() != target.data_ptr():
        target.copy_(res)
    if rows % world == 0:
        # equal blocks: an all-gather (a collective, at NVLink bandwidth; the other
        # ranks receive into `spare`) lands them in `out` in rank order
        if rank != dst and spare is None:
            spare = torch.empty(rows, hid, dtype=part.dtype, device=part.device)
        dist.all_gather_into_tensor(out if rank == dst else spare, target, group=group)
        return out if rank == dst else None
    if rank == dst:
        ops = [dist.P2POp(dist.irecv, out[b[k]:b[k + 1]], k, group) for k in range(world) if k != dst]
    else:
        ops = [dist.P2POp(dist.isend, target, dst, group)]
    for w in dist.batch_isend_irecv(ops):
        w.wait()
    return out if rank == dst else None


class P2PExchange:
    """One-shot rank-ordered combine over NVLink peer memory (`qx_combine_p2p`,
    or fused into the slice kernel by `slice_combine`).

    The B200 replacement of the reference's RDMA seam between the column-split
    nodes (native/qmesh_afd_seam.cu:309-361): each rank's BF16 partial is stored
    straight into the output rank's receive slot, and the output rank sums the
    partials in FP32 in rank order (then `shared`) with one BF16 rounding, the
    same result as `combine_across_ranks`. Setup exchanges CUDA IPC handles
    through `torch.distributed` (one collective); each step is one kernel per
    rank and no collective. Every rank must call `combine` once per step, in
    the same order; `close` (collective) releases the mappings.
    """

    def __init__(self, rows_max: int, group=None, dst: int = 0, device: torch.device | None = None):
        import ctypes

        from . import _lib
        self._ct = ctypes
        self._lib = _lib.load()
        self._L = _lib
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.dst = dst
        self.rows_max = rows_max
        if self.world > _lib.XCHG_MAX_RANKS:
            raise ValueError(f"at most {_lib.XCHG_MAX_RANKS} ranks")
        if not 0 <= dst < self.world:
            raise ValueError(f"output rank {dst} outside world {self.world}")
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        own = ctypes.c_void_p()
        _lib.check(self._lib.qx_xchg_alloc(rows_max, ctypes.byref(own)), "qx_xchg_alloc")
        self._own = own.value
        handle = (ctypes.c_char * _lib.IPC_HANDLE_BYTES)()
        _lib.check(self._lib.qx_ipc_handle(ctypes.c_void_p(self._own), handle), "qx_ipc_handle")
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened: list[int] = []
        bufs = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                bufs.append(self._own)
                continue
            p = ctypes.c_void_p()
            _lib.check(self._lib.qx_ipc_open(hb, ctypes.byref(p)), "qx_ipc_open")
            bufs.append(p.value)
            self._opened.append(p.value)
        self._args = _lib.QxXchgArgs()
        for r, b in enumerate(bufs):
            self._args.bufs[r] = b
        self._args.rank, self._args.world, self._args.dst = self.rank, self.world, dst
        self._args.rows_max = rows_max
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._args.status = self.status.data_ptr()
        self._mode: str | None = None     # "chunk" (combine) or "fused" (slice_combine), fixed by the first call
        dist.barrier(group=group)   # every rank has mapped every buffer before the first step

    def _use(self, mode: str) -> None:
        # One buffer serves one protocol: the two keep separate call counters.
        if self._mode not in (None, mode):
            raise RuntimeError(f"this exchange already runs the {self._mode} protocol")
        self._mode = mode

    def slice_combine(self, view, x: torch.Tensor, ids: torch.Tensor, tw: torch.Tensor, out: torch.Tensor,
                      c0: int, c1: int, workspace: torch.Tensor, x_scale: torch.Tensor | None = None,
                      shared: torch.Tensor | None = None, shared_expert=None, stream=None,
                      **kw) -> torch.Tensor | None:
        """The slice of this rank's columns with the combine fused into its
        finalize (`qx_slice_decode_tc_xchg`): one kernel per rank and step. On
        the output rank `out` receives bf16(p0 + ... [+ shared]) and is returned;
        senders do not write `out` and get None. `shared` is a BF16 partial
        computed elsewhere; `shared_expert` (output rank only) is the view of a
        one-expert arena that the same kernel runs over every row with weight 1
        and adds last (`qx_slice_decode_tc_shared`). A wait that runs out sets
        QX_DEV_TIMEOUT in the workspace status (`expert_slice.device_status`)."""
        from .expert_slice import launch
        self._use("fused")
        rows = x.shape[0]
        if not 1 <= rows <= self.rows_max:
            raise ValueError(f"rows {rows} outside 1..{self.rows_max}")
        a = self._L.QxXchgArgs()
        for r in range(self.world):
            a.bufs[r] = self._args.bufs[r]
        a.rank, a.world, a.dst, a.rows, a.rows_max = self.rank, self.world, self.dst, rows, self.rows_max
        if shared is not None and self.rank == self.dst:
            if shared.dtype != torch.bfloat16 or tuple(shared.shape) != (rows, self._L.HIDDEN) or shared.stride(1) != 1:
                raise TypeError("shared partial must be bf16 [rows, 5120] with unit column stride")
            a.shared, a.shared_stride = shared.data_ptr(), shared.stride(0)
        if shared_expert is not None and (self.rank != self.dst or shared is not None):
            raise ValueError("only the output rank runs the shared expert, and not beside a shared partial")
        launch(view, x, ids, tw, out, c0, c1, workspace, x_scale=x_scale, stream=stream, layout="tc", xchg=a,
               shared=shared_expert, **kw)
        return out if self.rank == self.dst else None

    def combine(self, part: torch.Tensor, out: torch.Tensor | None = None, shared: torch.Tensor | None = None,
                stream=None) -> torch.Tensor | None:
        """Sends this rank's partial; on the output rank returns bf16(p0 + ... [+ shared])."""
        self._use("chunk")
        if part.dtype != torch.bfloat16 or part.dim() != 2 or part.shape[1] != self._L.HIDDEN or part.stride(1) != 1:
            raise TypeError("partial must be bf16 [rows, 5120] with unit column stride")
        rows = part.shape[0]
        if not 1 <= rows <= self.rows_max:
            raise ValueError(f"rows {rows} outside 1..{self.rows_max}")
        a = self._args
        a.part, a.part_stride, a.rows = part.data_ptr(), part.stride(0), rows
        a.shared, a.shared_stride, a.out, a.out_stride = None, 0, None, 0
        if self.rank == self.dst:
            if out is None:
                out = torch.empty(rows, self._L.HIDDEN, dtype=torch.bfloat16, device=part.device)
            a.out, a.out_stride = out.data_ptr(), out.stride(0)
            if shared is not None:
                if shared.dtype != torch.bfloat16 or shared.shape != part.shape or shared.stride(1) != 1:
                    raise TypeError("shared partial must be bf16 like the partial")
                a.shared, a.shared_stride = shared.data_ptr(), shared.stride(0)
        if stream is None:
            stream = torch.cuda.current_stream(part.device).cuda_stream
        from .trace import rng
        with rng("qx.combine_p2p"):
            self._L.check(self._lib.qx_combine_p2p(self._ct.byref(a), self._ct.c_void_p(stream)), "qx_combine_p2p")
        return out if self.rank == self.dst else None

    def close(self) -> None:
        """Collective: unmap the peers' buffers, then free this rank's own."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            self._L.check(self._lib.qx_ipc_close(self._ct.c_void_p(p)), "qx_ipc_close")
        self._opened = []
        dist.barrier(group=self.group)
        self._L.check(self._lib.qx_xchg_free(self._ct.c_void_p(self._own)), "qx_xchg_free")
        self._own = None
