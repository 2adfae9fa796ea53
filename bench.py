#!/usr/bin/env python3
"""Benchmark of the routed-expert NVFP4 slice (BASELINE.json metric: MoE-layer
decode µs for 6 rows, and NVFP4 weight GB/s against the measured HBM peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one MoE layer over one batch: the routed-expert slice of every rank's
column shard (N ranks split the 2304 intermediate columns contiguously), then the
fixed-order FP32 combine of the per-rank BF16 partials on rank 0. Weights are
seeded synthetic NVFP4 (BASELINE config 1/2 shapes: 384 experts, hidden 5120,
intermediate 2304), resident in HBM; each step routes a different seeded draw
over several resident layers, so the ~680 MB of expert weights a step reads
exceeds the 126 MB L2.

--impl reference times the reference's dequantize-and-matmul path restated on
the host cores (the oracle), on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qmesh-afd-tp3_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

HIDDEN = 5120
INTER = 2304
N_EXPERTS = 384
TOPK = 6
EXPERT_BYTES = 2 * INTER * (HIDDEN // 2 + HIDDEN // 16) + HIDDEN * (INTER // 2 + INTER // 16)  # 19,906,560
# DRAM bytes (read + write) per unique expert per launch of tc_decode_kernel, from the ncu capture in
# profiles/tc_decode_kernel_config1.md (543.85 MB over 27 unique experts, full 2304 columns). A shard
# streams whole 64-column tiles, so its traffic scales with its padded width.
DRAM_BYTES_PER_UNIQUE = 543.85e6 / 27
METRIC = "MoE-layer decode µs (6 rows) & NVFP4 weight GB/s vs HBM peak, 1/2/4/8 GPU"


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampler running during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        fd, name = tempfile.mkstemp(prefix=f"qx_clocks_{index}_", suffix=".csv")
        os.close(fd)
        self.path = Path(name)

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()
            self.rows = self.path.read_text().splitlines()
        self.path.unlink(missing_ok=True)

    def summary(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.rows:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        busy = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_inputs(n_draws: int, rows: int, seed: int, n_experts: int, zipf: float = 0.0):
    """Seeded routing (softmax top-6 of N(0,1) logits, plus a Zipf(s) per-expert
    bias -s ln(rank) over a seeded permutation when zipf > 0) and FP8 activations
    per draw."""
    from qmesh_b200.synth import make_activation, routing, zipf_bias
    gen = torch.Generator().manual_seed(seed)
    bias = zipf_bias(n_experts, zipf, gen) if zipf > 0 else None
    draws = []
    for _ in range(n_draws):
        logits = torch.randn(rows, n_experts, generator=gen)
        if bias is not None:
            logits = logits + bias
        ids, tw = routing(logits, TOPK)
        q, inv = make_activation(rows, gen)
        draws.append((q, inv, ids, tw))
    return draws


def workload_config(args, world: int) -> dict:
    """The workload a line is quoted on (the same keys in both arms)."""
    rows = args.rows
    if args.zipf > 0 or rows > 6:
        workload = f"config3-spec-decode-rows{rows}" + (f"-zipf{args.zipf}" if args.zipf > 0 else "")
    elif args.columns:
        workload = "config2-shard-columns-%s-on-one-gpu" % args.columns.replace(":", "-")
    else:
        workload = "config1-decode" if world == 1 else "config2-column-split"
    if args.columns:
        width = int(args.columns.split(":")[1]) - int(args.columns.split(":")[0])
    else:
        width = INTER // world
    return {"workload": workload, "experts": args.experts, "hidden": HIDDEN, "intermediate": INTER, "rows": rows,
            "topk": TOPK, "columns_per_rank": width, "routing_draws": args.draws, "zipf_s": args.zipf,
            "seed": args.seed, "parallelism": f"column-split tp{world}",
            "shared_expert": "dense NVFP4 SwiGLU, intermediate 2304, weight 1, on rank 0" if shared_on(args, world)
            else None}


L2_BYTES = 126e6
SHARED_SEED = 999


def shared_on(args, world: int) -> bool:
    """Config 2's shared-expert stand-in: on for the column split (N > 1, 6 rows,
    uniform routing) unless --shared off; --shared on forces it."""
    if args.shared != "auto":
        return args.shared == "on"
    return world > 1 and args.rows == 6 and args.zipf == 0 and not args.columns


def device_start(world: int, dev, stream, ev) -> None:
    """Records the start event of a timed region. With N > 1 a one-element NCCL
    all-reduce goes first on every rank, so each rank's clock starts when the
    ranks meet on the devices, not when its host thread got past the barrier
    (the host threads of N processes leave a barrier tens to hundreds of
    microseconds apart, which a few-millisecond loop would count per step)."""
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(torch.zeros(1, device=dev))
    ev.record(stream)


def gather_floats(v: float, world: int, dev) -> list[float]:
    """Every rank's value of v, in rank order (a collective: all ranks call it)."""
    import torch.distributed as dist
    parts = [torch.zeros(1, dtype=torch.float64, device=dev) for _ in range(world)]
    dist.all_gather(parts, torch.tensor([v], dtype=torch.float64, device=dev))
    return [float(t.item()) for t in parts]


def expected_unique(rows: int, n_experts: int) -> float:
    """Expected distinct experts among rows x top-6 uniform draws."""
    return n_experts * (1.0 - (1.0 - 1.0 / n_experts) ** (rows * TOPK))


def resident_layers(step_bytes: float) -> int:
    """Resident layers the device loop rotates through: a layer's weights are read
    again only after at least twice the L2 size of other layers' weights."""
    return max(2, 1 + math.ceil(2 * L2_BYTES / max(step_bytes, 1.0)))


def l2_note(step_bytes: float, layers: int) -> str:
    between = (layers - 1) * step_bytes
    return ("inputs larger than L2: %.0f MB of this rank's expert weights per step; a layer recurs every %d steps "
            "with %.0f MB of other layers' weights read in between (L2 126 MB)"
            % (step_bytes / 1e6, layers, between / 1e6))


def ulp_stats(out: torch.Tensor, ref: torch.Tensor, mag: torch.Tensor | None = None) -> dict:
    """Relative L2 and BF16 ulp errors of `out` against `ref` (CPU float): the ulp
    is the BF16 spacing at max(|ref|, 2^-10 rms(row)[, |mag|]) ("max_ulp") and
    at |ref| alone ("max_ulp_floorless"); counts of elements beyond 2 ulp."""
    out, ref = out.float().cpu(), ref.float().cpu()
    err = (out - ref).abs()

    def ulp(a):
        return torch.pow(2.0, torch.floor(torch.log2(a.clamp_min(2.0 ** -126))) - 7.0)
    rms = ref.pow(2).mean(dim=-1, keepdim=True).sqrt()
    m = torch.maximum(ref.abs(), (2.0 ** -10 * rms).expand_as(ref))
    if mag is not None:
        m = torch.maximum(m, mag.float().cpu().abs())
    u = err / ulp(m)
    u0 = err / ulp(ref.abs())
    return {"rel_l2": float(err.norm() / ref.norm().clamp_min(1e-30)), "max_ulp": float(u.max()),
            "max_ulp_floorless": float(u0.max()), "n_over_2ulp_floorless": int((u0 > 2).sum()),
            "n_over_2ulp": int((u > 2).sum()), "elements": ref.numel()}


def check_parity(args, world, rank, dev, dq, views, ws, part, out, a0, a1, last, slice_step, shv, sh_call,
                 layers, n_exp) -> dict:
    """Checks the timed path's results outside the timed region.

    N = 1: the output the timed loop left (step `last`) against the same step
    run again, bit for bit. N > 1: for the last timed step and two more, the
    output rank's combined output against the rank-ordered combine
    (qx_combine_ordered) of every rank's plain slice partial gathered with
    NCCL, followed by a separate shared-expert call when config 2's shared
    expert is on, bit for bit; and the last timed step against the full
    2304-column slice of the same layer (with the shared expert) on the output
    rank's GPU alone: relative L2 within 5e-3 and every element within
    N / 2 + 1 BF16 ulp, the ulp taken at the largest partial. The two are
    different roundings of one sum: the combine adds N partials that were each
    rounded to BF16 (at most half an ulp of the largest partial each), and both
    results are rounded once more (half an ulp each), so N / 2 + 1 bounds their
    distance; at N = 2 it is the north star's 2 ulp. Every rank takes the same
    collective steps; a mismatch ends the run with an error."""
    import torch.distributed as dist
    from qmesh_b200.arena import Arena
    from qmesh_b200.combine import combine_ordered
    from qmesh_b200.expert_slice import alloc_workspace, launch
    stream = torch.cuda.current_stream(dev).cuda_stream
    rows = args.rows

    def run(i: int) -> None:
        q, inv, ids, tw = dq[i % len(dq)]
        slice_step(views[i % layers], q, inv, ids, tw, stream)

    def plain(i: int, dst: torch.Tensor) -> None:
        q, inv, ids, tw = dq[i % len(dq)]
        launch(views[i % layers], q, ids, tw, dst, a0, a1, ws, x_scale=inv, stream=stream, layout=args.layout)

    res = {"checked": True, "steps": 0, "bit_exact": True}
    if world == 1:
        torch.cuda.synchronize()
        timed = part.clone()
        run(last)
        torch.cuda.synchronize()
        res.update(steps=1, bit_exact=bool(torch.equal(timed, part)),
                   what="timed-loop output vs the same step run again")
        if not res["bit_exact"]:
            raise SystemExit(f"parity: timed output differs from an eager call: {res}")
        return res
    gathered = [torch.empty_like(part) for _ in range(world)]
    mine = torch.empty_like(part)
    cmb = torch.empty_like(part)
    first_cmb, first_mag = None, None
    for k, i in enumerate((last, last + 1, last + 2)):
        if k > 0:   # a fresh step through the same exchange
            run(i)
        torch.cuda.synchronize()
        timed = out.clone()
        plain(i, mine)
        dist.all_gather(gathered, mine)
        ok = True
        if rank == 0:
            parts = list(gathered)
            if sh_call is not None:
                q, inv, _, _ = dq[i % len(dq)]
                parts.append(sh_call(q, inv, stream).clone())
            combine_ordered(parts, out=cmb)
            torch.cuda.synchronize()
            ok = bool(torch.equal(timed, cmb))
            if k == 0:
                first_cmb = cmb.clone()
                first_mag = torch.stack([g.float().abs() for g in parts]).amax(dim=0)
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        res["steps"] += 1
        res["bit_exact"] = res["bit_exact"] and bool(flag.item())
    res["what"] = ("combined output vs qx_combine_ordered of the ranks' plain slice partials (NCCL all-gather)"
                   + (" and a separate shared-expert call" if sh_call is not None else "")
                   + ", 3 steps; the last timed step vs the full-column slice on one GPU")
    ok = True
    if rank == 0:
        li = last % layers
        full = Arena(dev, li + 1, n_exp, 0, INTER, layout=args.layout)
        full.fill_synthetic(li, seed=1000 + li)
        wsf = alloc_workspace(rows, TOPK, 0, INTER, dev, args.layout)
        one = torch.empty_like(part)
        q, inv, ids, tw = dq[last % len(dq)]
        launch(full.view(li), q, ids, tw, one, 0, INTER, wsf, x_scale=inv, stream=stream, layout=args.layout,
               shared=shv)
        torch.cuda.synchronize()
        del full, wsf
        st = ulp_stats(first_cmb, one, first_mag)
        bound = world / 2 + 1
        ok = st["rel_l2"] <= 5e-3 and st["max_ulp"] <= bound
        res["vs_one_gpu"] = {k: (round(v, 7) if isinstance(v, float) else v) for k, v in st.items()}
        res["vs_one_gpu"]["bound_ulp"] = bound
        res["vs_one_gpu"]["within_tolerance"] = ok
    flag = torch.tensor([1 if (ok and res["bit_exact"]) else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if not flag.item():
        raise SystemExit(f"parity check failed on rank {rank}: {res}")
    return res


def run_ours(args) -> dict | None:
    import torch.distributed as dist
    from qmesh_b200 import build
    from qmesh_b200.arena import Arena
    from qmesh_b200.combine import combine_ordered
    from qmesh_b200.expert_slice import alloc_workspace, launch
    from qmesh_b200.shard import P2PExchange, combine_across_ranks, shard_range
    build.build()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    rows = args.rows
    a0, a1 = shard_range(rank, world)
    if args.columns:
        if world > 1:
            raise SystemExit("--columns times one rank's shard on one GPU (N = 1)")
        a0, a1 = (int(v) for v in args.columns.split(":"))
    width = a1 - a0
    n_exp = args.experts
    step_bytes = expected_unique(rows, n_exp) * EXPERT_BYTES * width / INTER
    layers = args.layers if args.layers > 0 else resident_layers(step_bytes)
    ar = Arena(dev, layers, n_exp, a0, a1, layout=args.layout)
    ar.check_memory()
    for li in range(layers):
        ar.fill_synthetic(li, seed=1000 + li)
    torch.cuda.synchronize()
    draws = make_inputs(args.draws, rows, seed=args.seed, n_experts=n_exp, zipf=args.zipf)
    dq = [(q.to(dev), inv.to(dev), ids.to(dev), tw.to(dev)) for q, inv, ids, tw in draws]
    uniq = [len(set(ids.flatten().tolist())) for _, _, ids, _ in draws]
    ws = alloc_workspace(rows, TOPK, a0, a1, dev, args.layout)
    part = torch.empty(rows, HIDDEN, dtype=torch.bfloat16, device=dev)
    gathered = [torch.empty_like(part) for _ in range(world)] if world > 1 and args.xchg == "nccl" else None
    xchg = P2PExchange(rows_max=rows, dst=0, device=dev) if world > 1 and args.xchg in ("p2p", "fused") else None
    fused = world > 1 and args.xchg == "fused"
    # config 2's shared-expert stand-in: one dense NVFP4 SwiGLU over all 2304
    # columns, every row with weight 1, on the output rank (rank 0), added after
    # the ranks' routed partials
    with_shared = shared_on(args, world)
    shv, sh_call = None, None
    if with_shared and rank == 0:
        if args.layout != "tc":
            raise SystemExit("the shared expert runs on the tensor-core slice (--layout tc)")
        sh_arena = Arena(dev, 1, 1, 0, INTER, layout="tc")
        sh_arena.fill_synthetic(0, seed=SHARED_SEED)
        shv = sh_arena.view(0)
        ws_s = alloc_workspace(rows, 1, 0, INTER, dev)
        sh_ids = torch.zeros(rows, 1, dtype=torch.int32, device=dev)
        sh_tw = torch.ones(rows, 1, dtype=torch.float32, device=dev)
        sh_out = torch.empty(rows, HIDDEN, dtype=torch.bfloat16, device=dev)

        def sh_call(q, inv, st) -> torch.Tensor:
            """The shared expert as a call of its own (ids 0, weight 1)."""
            launch(shv, q, sh_ids, sh_tw, sh_out, 0, INTER, ws_s, x_scale=inv, stream=st)
            return sh_out

    def exchange(p: torch.Tensor, shared: torch.Tensor | None = None, o: torch.Tensor | None = None):
        o = out if o is None else o
        if xchg is not None:
            return xchg.combine(p, out=o, shared=shared)
        return combine_across_ranks(p, dst=0, out=o, combine=combine_ordered, gathered=gathered, shared=shared)
    out = torch.empty(rows, HIDDEN, dtype=torch.bfloat16, device=dev)
    views = [ar.view(li) for li in range(layers)]
    stream = torch.cuda.current_stream(dev)

    def slice_step(view, q, inv, ids, tw, st, dst: torch.Tensor | None = None) -> None:
        """One step through the public calls: N = 1 the slice (with the shared
        expert in the same kernel when configured); N > 1 the fused slice +
        combine (the output rank runs the shared expert in its kernel), or the
        slice, a separate shared-expert call on the output rank and the combine.
        The result goes to `dst` when given (else `part` at N = 1, `out` at N > 1)."""
        if fused:
            xchg.slice_combine(view, q, ids, tw, out if dst is None else dst, a0, a1, ws, x_scale=inv, stream=st,
                               shared_expert=shv)
            return
        if world == 1:
            launch(view, q, ids, tw, part if dst is None else dst, a0, a1, ws, x_scale=inv, stream=st,
                   layout=args.layout, shared=shv)
            return
        launch(view, q, ids, tw, part, a0, a1, ws, x_scale=inv, stream=st, layout=args.layout)
        exchange(part, sh_call(q, inv, st) if sh_call is not None else None, dst)

    def step(i: int) -> None:
        q, inv, ids, tw = dq[i % len(dq)]
        st = torch.cuda.current_stream(dev).cuda_stream   # the capture stream while a graph is recorded
        slice_step(views[i % layers], q, inv, ids, tw, st)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    # The device-timed steps replay one CUDA graph per (draw, layer) pair, as a
    # serving loop replays its per-layer graphs: the host issues one graph launch
    # per step instead of the Python argument set-up of every call.
    graphs = None
    if not args.no_graphs and not (world > 1 and args.xchg == "nccl"):
        period = len(dq) * layers // math.gcd(len(dq), layers)
        graphs = []
        for j in range(period):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step(j)
            graphs.append(g)
        for i in range(args.warmup):
            graphs[(args.warmup + i) % period].replay()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    last = 2 * args.warmup + args.steps - 1       # the step whose output the timed loop leaves behind
    if graphs is not None:
        last %= len(graphs)
    with Clocks(local) as clk:
        torch.cuda.synchronize()
        device_start(world, dev, stream, ev0)
        for i in range(args.steps):
            if graphs is not None:
                graphs[(2 * args.warmup + i) % len(graphs)].replay()
            else:
                step(2 * args.warmup + i)
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    rank_loop_us = None
    if world > 1:
        rank_loop_us = [v * 1e3 / args.steps for v in gather_floats(ms, world, dev)]
        ms = max(rank_loop_us) * args.steps / 1e3
        dist.barrier()
    us_layer = ms * 1e3 / args.steps

    # ---- parity of the timed path (outside the timed region) ----
    par = check_parity(args, world, rank, dev, dq, views, ws, part, out, a0, a1, last, slice_step, shv, sh_call,
                       layers, n_exp)

    # ---- end to end through the public call with host buffers ----
    from qmesh_b200.expert_slice import expert_slice
    host = [(q.pin_memory(), inv.pin_memory(), ids.pin_memory(), tw.pin_memory()) for q, inv, ids, tw in draws]
    out_h = torch.empty(rows, HIDDEN, dtype=torch.bfloat16).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host[0])
    d2h = out_h.numel() * out_h.element_size()

    hslice = None
    if world == 1 and (shv is None or args.layout == "tc"):
        # the public host-buffer call: one packed host-to-device copy per step,
        # the copies on side streams overlapping the neighbouring steps' kernels.
        # (At N > 1 HostSlice's per-step host work outlasts a step: 130 us per step
        # at N = 2 against 113 us with the copies straight from the pinned inputs.)
        from qmesh_b200.expert_slice import HostSlice
        hslice = HostSlice(ar, rows, TOPK, a0, a1, shared=shv)
        h2d = hslice.nbytes

    # Without HostSlice: two slots of device inputs and outputs; step i's input
    # copies run on a copy stream while step i - 1 computes, and its output copy
    # (output rank) on a third stream while step i + 1 computes.
    slot_in = [[torch.empty_like(t, device=dev) for t in host[0]] for _ in range(2)]
    slot_out = [torch.empty(rows, HIDDEN, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    slot_host = [torch.empty(rows, HIDDEN, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    cp_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    slot_used = [False, False]

    def e2e_step(i: int) -> None:
        src = host[i % len(host)]
        if hslice is not None:
            hslice(i % layers, src[0], src[1], src[2], src[3])
            return
        k = i % 2
        if slot_used[k]:
            cp_stream.wait_event(ev_done[k])          # the slot's previous slice has read its inputs
        with torch.cuda.stream(cp_stream):
            for d, s in zip(slot_in[k], src):
                d.copy_(s, non_blocking=True)
        ev_in[k].record(cp_stream)
        stream.wait_event(ev_in[k])
        if slot_used[k] and rank == 0:
            stream.wait_event(ev_out[k])              # the slot's previous output has been copied out
        slice_step(views[i % layers], slot_in[k][0], slot_in[k][1], slot_in[k][2], slot_in[k][3],
                   stream.cuda_stream, dst=slot_out[k])
        ev_done[k].record(stream)
        if rank == 0:
            d2h_stream.wait_event(ev_done[k])
            with torch.cuda.stream(d2h_stream):
                slot_host[k].copy_(slot_out[k], non_blocking=True)
            ev_out[k].record(d2h_stream)
        slot_used[k] = True

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    device_start(world, dev, stream, ev0)
    if hslice is not None:
        hslice.order_after(stream)   # the first step's input copy starts inside the timed region
    else:
        cp_stream.wait_stream(stream)
        d2h_stream.wait_stream(stream)
    for i in range(args.steps):
        e2e_step(i)
    if hslice is not None:
        hslice.join(stream)   # the last step's output copy runs on the host-slice's copy stream
    else:
        stream.wait_stream(d2h_stream)
        stream.wait_stream(cp_stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    us_e2e = ms_e2e * 1e3 / args.steps

    # ---- kernel-only timing of the slice call (roofline) ----
    # The calls are queued behind a spin of the stream (1 ms + 60 us per call at
    # 2 GHz), so that they run back to back on the device however fast the host
    # issues them; the mean is the interval between the events around them over
    # their count.
    torch.cuda.synchronize()
    torch.cuda._sleep(int(2e6 + 1.2e5 * args.steps))
    ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ka.record(stream)
    for i in range(args.steps):
        q, inv, ids, tw = dq[i % len(dq)]
        launch(views[i % layers], q, ids, tw, part, a0, a1, ws, x_scale=inv, stream=stream.cuda_stream,
               layout=args.layout, shared=shv)
    kb.record(stream)
    torch.cuda.synchronize()
    k_mean = ka.elapsed_time(kb) * 1e3 / args.steps
    rank_kernel_us = gather_floats(k_mean, world, dev) if world > 1 else None
    mean_u = sum(uniq[i % len(uniq)] for i in range(args.steps)) / args.steps
    shared_bytes = EXPERT_BYTES if with_shared else 0     # on the output rank
    alg_bytes = (mean_u * EXPERT_BYTES * width / INTER + (shared_bytes if rank == 0 else 0)
                 + rows * HIDDEN * 1 + rows * HIDDEN * 2)
    gbs = alg_bytes / (k_mean * 1e-6) / 1e9
    peak, peak_kind = peaks()
    res = None
    if rank == 0:
        clocks = clk.summary()
        res = {
            "metric": METRIC,
            "value": round(us_layer, 3),
            "unit": "us/layer",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(us_layer / 1e3, 6),
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "nvfp4-w/fp8-x/fp32-acc",
            "data": "synthetic (seeded NVFP4 weights from N(0,0.02); FP8 activations from N(0,1))",
            "config": dict(workload_config(args, world), l2=l2_note(mean_u * EXPERT_BYTES * width / INTER, layers)),
            "ranks": None if world == 1 else {
                "step_us": [round(v, 2) for v in rank_loop_us],
                "slice_kernel_us": [round(v, 2) for v in rank_kernel_us],
                "note": "per rank: the timed loop's us per step (value is their max) and the slice "
                        "kernel alone (plain launch, no exchange; the output rank's with the shared expert)"},
            "setup": {"resident_layers": layers, "mean_unique_experts": round(mean_u, 2),
                      "shared_expert": ("in the output rank's slice kernel" if fused or world == 1
                                        else "a separate call on the output rank") if with_shared else None,
                      "timed_loop": "per-step CUDA graph replay" if graphs is not None else "eager calls",
                      "exchange": None if world == 1 else {
                          "fused": "in the slice kernel: NVLink stores of each finalize unit + rank-ordered FP32 sum",
                          "p2p": "one-shot NVLink store + rank-ordered FP32 sum kernel",
                          "nccl": "NCCL all-gather + rank-ordered FP32 sum kernel"}[args.xchg],
                      "kernel": "tcgen05 mxf4nvf4 (16-term e2m1 activations)" if args.layout == "tc"
                      else "register dequant + mma.sync"},
            "tokens_per_s": round(rows / (us_layer * 1e-6), 1),
            "weight_gbs": round(gbs, 1),   # per rank: its shard's bytes over its slice kernel time
            # whole step: every rank's weight bytes over the step time (the config-2 aggregate)
            "aggregate_weight_gbs": round((mean_u * EXPERT_BYTES * width * world / INTER + shared_bytes)
                                          / (us_layer * 1e-6) / 1e9, 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_kind": peak_kind,
                         "traffic": int(mean_u * DRAM_BYTES_PER_UNIQUE * (64 * math.ceil(width / 64)) / INTER),
                         "traffic_source": "ncu dram bytes per unique expert (small-arena capture) x mean unique "
                                           "experts x padded shard width / 2304",
                         "kernel_us": round(k_mean, 3), "alg_bytes_per_launch": int(alg_bytes)},
            "e2e": {"value": round(us_e2e, 3), "unit": "us/layer", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            # prep + decode (tc) or prologue + main + finalize (frag) per step, + a combine kernel for N > 1
            # unless the combine is fused into the decode kernel
            "gpu_launches": args.steps * ((2 if args.layout == "tc" else 3)
                                          + (1 if world > 1 and not fused else 0)
                                          + (2 if with_shared and world > 1 and not fused else 0)),
            "clocks": clocks,
            "parity": par,
        }
        if world == 1 and not args.no_cpu:
            res["cpu_baseline"] = cpu_baseline(args)
    if world > 1:
        if xchg is not None:
            xchg.close()
        dist.barrier()
        dist.destroy_process_group()
    return res


def cpu_sample(args, n_calls: int, warmup: int, world: int = 1) -> tuple[float, int, str]:
    """The reference's dequantize-and-matmul path of the slice, restated on the
    host cores (oracle.moe.slice_w4a16), all host threads: `n_calls` timed full
    2304-column layer calls (after `warmup` untimed ones) of the bench's own
    seeded routing draws over a resident random-code layer, plus config 2's
    shared expert (every row, weight 1) and the ordered combine when that is on.
    The CPU path's cost depends on the shapes only, so random codes stand in for
    the quantised weights. Returns (µs per call, threads, sample description)."""
    from oracle import moe, nvfp4 as oq
    n = moe.cpu_threads()
    rows = args.rows
    draws = make_inputs(max(args.draws, 1), rows, seed=args.seed, n_experts=args.experts, zipf=args.zipf)
    layer = moe.random_code_layer(rows * TOPK, torch.Generator().manual_seed(args.seed))
    with_shared = shared_on(args, world)
    sh_layer = moe.random_code_layer(1, torch.Generator().manual_seed(SHARED_SEED)) if with_shared else None
    sh_ids = torch.zeros(rows, 1, dtype=torch.int32)
    sh_tw = torch.ones(rows, 1)
    times = []
    for i in range(warmup + n_calls):
        q, inv, ids, tw = draws[i % len(draws)]
        experts = sorted(set(ids.flatten().tolist()))
        local = torch.tensor([experts.index(e) for e in ids.flatten().tolist()], dtype=torch.int32).view_as(ids)
        x = oq.fp8_ingest(q, inv)
        t0 = time.perf_counter()
        routed = moe.slice_w4a16(x, local, tw, layer, 0, INTER)
        if sh_layer is not None:
            moe.combine_ordered([routed], shared=moe.slice_w4a16(x, sh_ids, sh_tw, sh_layer, 0, INTER))
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    us = sum(times) / len(times) * 1e6
    what = "routed experts and the shared expert" if with_shared else "routed experts only"
    sample = (f"{n_calls} full-layer calls (all 2304 columns, {rows} rows, top-{TOPK}, {what}) of "
              f"the bench's seeded routing draws after {warmup} untimed, {n} threads")
    return us, n, sample


def cpu_baseline(args) -> dict:
    us, n, sample = cpu_sample(args, args.cpu_layers, 1)
    return {"value": round(us, 1), "unit": "us/layer", "cores": n, "kind": "port", "sample": sample}


def run_reference(args) -> dict | None:
    """The reference arm: the same CPU sampler as `cpu_baseline`, on rank 0 only,
    with the ours-arm config keys (the CPU path computes every column of the
    layer in one process)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    world = int(os.environ.get("WORLD_SIZE", "1"))
    us, n, sample = cpu_sample(args, args.steps, args.warmup, world)
    return {"impl": "reference", "metric": METRIC, "value": round(us, 1), "unit": "us/layer",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(us / 1e3, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp32 (W4A16 dequant)", "data": "synthetic",
            "config": workload_config(args, world),
            "cpu_baseline": {"value": round(us, 1), "unit": "us/layer", "cores": n, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(us, 1), "unit": "us/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


PREFILL_TOKENS = 2048
PREFILL_A2 = 0.25   # stands in for the reference's calibrated a2 (6 / (1.5 max|c2|) on this synthetic layer)
PREFILL_METRIC = "MoE-layer prefill µs (2048 tokens, W4A4) & NVFP4 weight GB/s, tensor TFLOP/s"


def run_prefill(args) -> dict | None:
    """Config 4: one prefill chunk of 2048 tokens through the W4A4 grouped tcgen05
    GEMM (qx_slice_prefill_tc), 384 experts, uniform top-6 routing, seed 4."""
    import torch.distributed as dist
    from qmesh_b200 import build
    from qmesh_b200.arena import Arena
    from qmesh_b200.combine import combine_ordered
    from qmesh_b200.expert_slice import alloc_prefill_workspace, launch_prefill
    from qmesh_b200.shard import combine_across_ranks, combine_rows_across_ranks, row_bounds, shard_range
    from qmesh_b200.synth import make_activation, routing
    build.build()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    T, E = args.tokens, args.experts
    a0, a1 = shard_range(rank, world)
    if args.columns:
        if world > 1:
            raise SystemExit("--columns times one rank's shard on one GPU (N = 1)")
        a0, a1 = (int(v) for v in args.columns.split(":"))
    width = a1 - a0
    ar = Arena(dev, 1, E, a0, a1, layout="tc")
    ar.fill_synthetic(0, 4)
    gen = torch.Generator().manual_seed(4)
    ids, tw = routing(torch.randn(T, E, generator=gen), TOPK)
    q, inv = make_activation(T, gen)
    a2 = torch.full((E,), PREFILL_A2, dtype=torch.float32, device=dev)
    dq, dinv, dids, dtw = q.to(dev), inv.to(dev), ids.to(dev), tw.to(dev)
    ws = alloc_prefill_workspace(T, TOPK, a0, a1, E, dev)
    part = torch.empty(T, HIDDEN, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(part)
    view = ar.view(0)
    stream = torch.cuda.current_stream(dev)
    # N > 1: the row-split combine (an all-to-all of row blocks, each rank sums its
    # block of every partial in rank order, the output rank collects the blocks)
    n_me = (row_bounds(T, world)[rank + 1] - row_bounds(T, world)[rank]) if world > 1 else 0
    recv = torch.empty(world * n_me, HIDDEN, dtype=torch.bfloat16, device=dev) if world > 1 else None
    mine = torch.empty(n_me, HIDDEN, dtype=torch.bfloat16, device=dev) if world > 1 else None
    spare = torch.empty(T, HIDDEN, dtype=torch.bfloat16, device=dev) if world > 1 and rank != 0 else None

    def step(x, xs, i_, t_, dst=None) -> None:
        """One prefill step; its output (N = 1 the slice, N > 1 the combined) goes
        to `dst` when given, else to `part` (N = 1) or `out` (N > 1)."""
        launch_prefill(view, x, i_, t_, a2, part if (world > 1 or dst is None) else dst, a0, a1, ws, x_scale=xs,
                       stream=stream.cuda_stream)
        if world > 1:
            combine_rows_across_ranks(part, dst=0, out=out if dst is None else dst, combine=combine_ordered,
                                      recv=recv, mine=mine, spare=spare)

    for _ in range(args.warmup):
        step(dq, dinv, dids, dtw)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.synchronize()
        device_start(world, dev, stream, ev0)
        for _ in range(args.steps):
            step(dq, dinv, dids, dtw)
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    us = ms * 1e3 / args.steps
    parity = None
    if world > 1:
        # the timed path's output against the gather combine of the same partials, bit for bit
        torch.cuda.synchronize()
        timed = out.clone()
        launch_prefill(view, dq, dids, dtw, a2, part, a0, a1, ws, x_scale=dinv, stream=stream.cuda_stream)
        want = combine_across_ranks(part, dst=0, combine=combine_ordered)
        torch.cuda.synchronize()
        ok = bool(torch.equal(timed, want)) if rank == 0 else True
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        parity = {"checked": True, "bit_exact": bool(flag.item()),
                  "what": "the row-split combine's output vs the gather combine (qx_combine_ordered of the "
                          "NCCL-gathered partials) of the same step"}
        if not flag.item():
            raise SystemExit(f"prefill parity failed: {parity}")
    # the slice alone, calls back to back behind a stream spin (per rank at N > 1)
    torch.cuda.synchronize()
    torch.cuda._sleep(int(2e6 + 1.2e5 * args.steps))
    ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ka.record(stream)
    for _ in range(args.steps):
        launch_prefill(view, dq, dids, dtw, a2, part, a0, a1, ws, x_scale=dinv, stream=stream.cuda_stream)
    kb.record(stream)
    torch.cuda.synchronize()
    k_us = ka.elapsed_time(kb) * 1e3 / args.steps
    rank_step_us = rank_kernel_us = None
    if world > 1:
        rank_step_us = [round(v, 1) for v in gather_floats(ms * 1e3 / args.steps, world, dev)]
        rank_kernel_us = [round(v, 1) for v in gather_floats(k_us, world, dev)]
    # end to end: H2D of the chunk's inputs from pinned memory, D2H of the output
    # (two slots of device inputs and outputs: a step's input copies run on a copy
    # stream while the previous step computes, its output copy on a third stream
    # while the next one computes)
    host = [t_.pin_memory() for t_ in (q, inv, ids, tw)]
    slot_in = [[torch.empty_like(t_, device=dev) for t_ in host] for _ in range(2)]
    slot_out = [torch.empty(T, HIDDEN, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    slot_host = [torch.empty(T, HIDDEN, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    h2d = sum(t_.numel() * t_.element_size() for t_ in host)
    d2h = slot_host[0].numel() * slot_host[0].element_size()
    cp_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    slot_used = [False, False]

    def e2e_step(i: int) -> None:
        k = i % 2
        if slot_used[k]:
            cp_stream.wait_event(ev_done[k])
        with torch.cuda.stream(cp_stream):
            for d_, h_ in zip(slot_in[k], host):
                d_.copy_(h_, non_blocking=True)
        ev_in[k].record(cp_stream)
        stream.wait_event(ev_in[k])
        if slot_used[k] and rank == 0:
            stream.wait_event(ev_out[k])
        step(slot_in[k][0], slot_in[k][1], slot_in[k][2], slot_in[k][3], dst=slot_out[k])
        ev_done[k].record(stream)
        if rank == 0:
            d2h_stream.wait_event(ev_done[k])
            with torch.cuda.stream(d2h_stream):
                slot_host[k].copy_(slot_out[k], non_blocking=True)
            ev_out[k].record(d2h_stream)
        slot_used[k] = True

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    device_start(world, dev, stream, ev0)
    cp_stream.wait_stream(stream)
    d2h_stream.wait_stream(stream)
    for i in range(args.steps):
        e2e_step(i)
    stream.wait_stream(d2h_stream)
    stream.wait_stream(cp_stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    us_e2e = ms_e2e * 1e3 / args.steps
    uniq = len(set(ids.flatten().tolist()))
    alg_bytes = uniq * EXPERT_BYTES * width / INTER + T * HIDDEN + T * HIDDEN * 2
    n_pairs = T * TOPK
    ka_gbs = alg_bytes / (k_us * 1e-6) / 1e9
    flops = 2.0 * n_pairs * (2 * width * HIDDEN + HIDDEN * width)
    peak, peak_kind = peaks()
    res = None
    if rank == 0:
        res = {
            "metric": PREFILL_METRIC, "value": round(us, 1), "unit": "us/layer", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 4),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "nvfp4-w/nvfp4-x (W4A4)/fp32-acc",
            "data": "synthetic (seeded NVFP4 weights from N(0,0.02); FP8 activations from N(0,1))",
            "config": {"workload": "config4-prefill" + ("-columns-%d-%d-on-one-gpu" % (a0, a1) if args.columns else ""),
                       "experts": E, "hidden": HIDDEN, "intermediate": INTER,
                       "tokens": T, "topk": TOPK, "columns_per_rank": width, "unique_experts": uniq,
                       "a2": PREFILL_A2, "l2": f"inputs larger than L2: {alg_bytes / 1e9:.2f} GB of expert weights per step",
                       "parallelism": f"column-split tp{world}",
                       "exchange": None if world == 1 else "row-split combine: NCCL all-to-all of row blocks, "
                                   "per-rank ordered FP32 sums (qx_combine_ordered), blocks all-gathered",
                       "kernel": "grouped tcgen05 mxf4nvf4 (NVFP4 x NVFP4, TMEM accumulators)"},
            "tokens_per_s": round(T / (us * 1e-6), 1),
            "weight_gbs": round(alg_bytes / (us * 1e-6) / 1e9, 1),
            "tensor_tflops": round(flops / (k_us * 1e-6) / 1e12, 2),
            "roofline": {"bound": "hbm", "achieved": round(ka_gbs, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(ka_gbs / peak, 4),
                         "peak_kind": peak_kind, "traffic": None, "kernel_us": round(k_us, 1),
                         "kernel_note": "the slice's six kernels per call, calls back to back",
                         "alg_bytes_per_launch": int(alg_bytes), "flops_per_launch": int(flops)},
            "parity": parity,
            "ranks": None if world == 1 else {"step_us": rank_step_us, "slice_kernel_us": rank_kernel_us},
            "e2e": {"value": round(us_e2e, 1), "unit": "us/layer", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps * 6 + (args.steps if world > 1 else 0),
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu:
            res["cpu_baseline"] = prefill_cpu_baseline(ar, q, inv, ids, tw, uniq)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


def prefill_cpu_baseline(ar, q, inv, ids, tw, uniq: int, n_experts: int = 3) -> dict:
    """The W4A4 prefill body restated on the host cores (oracle.prefill), timed on
    the pairs of a few experts and scaled by the unique experts of the chunk."""
    from oracle import moe, nvfp4 as oq, prefill as opf
    n = moe.cpu_threads()
    experts = sorted(set(ids.flatten().tolist()))[:n_experts]
    pack = ar.expert_pack(0, experts)
    remap = {e: i for i, e in enumerate(experts)}
    local = torch.tensor([remap.get(e, -1) for e in ids.flatten().tolist()], dtype=torch.int32).view_as(ids)
    x = oq.fp8_ingest(q, inv)
    t0 = time.perf_counter()
    opf.slice_w4a4(x, local, tw, pack, 0, ar.width, torch.full((len(experts),), PREFILL_A2))
    dt = time.perf_counter() - t0
    us = dt / len(experts) * uniq * 1e6
    return {"value": round(us, 1), "unit": "us/layer", "cores": n, "kind": "port",
            "sample": f"the pairs of {len(experts)} of the chunk's {uniq} experts ({dt:.1f} s), scaled by {uniq}/{len(experts)}"}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--rows", type=int, default=6)
    ap.add_argument("--experts", type=int, default=N_EXPERTS)
    ap.add_argument("--layers", type=int, default=0,
                    help="resident layers the device loop rotates through (0: enough that a layer's weights are "
                         "re-read only after twice the L2 size of other weights)")
    ap.add_argument("--draws", type=int, default=16)
    ap.add_argument("--cpu-layers", type=int, default=3)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--columns", default="",
                    help="A:B — time the slice of intermediate columns [A, B) on one GPU (one rank's shard)")
    ap.add_argument("--shared", default="auto", choices=["auto", "on", "off"],
                    help="config 2's shared expert on rank 0 (auto: on for N > 1 at 6 rows, uniform routing)")
    ap.add_argument("--no-graphs", action="store_true",
                    help="time the device loop with eager calls instead of per-step CUDA graph replays")
    ap.add_argument("--xchg", default="fused", choices=["fused", "p2p", "nccl"],
                    help="N>1 combine: fused into the slice kernel's finalize (fused), a separate one-shot "
                         "NVLink kernel (p2p), or NCCL all-gather + combine kernel (nccl)")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill"],
                    help="decode: BASELINE configs 1/2 (default); prefill: config 4 (2048-token W4A4 chunk)")
    ap.add_argument("--tokens", type=int, default=PREFILL_TOKENS)
    ap.add_argument("--zipf", type=float, default=0.0,
                    help="Zipf(s) expert bias of the routing logits (config 3: --rows 48 --zipf 1.1 --seed 3)")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--layout", default="tc", choices=["tc", "frag"],
                    help="arena layout / kernel: tc = tcgen05 block-scaled MMA, frag = register dequant + mma.sync")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "prefill":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the prefill reference arm is the CPU baseline "
                              "inside the ours line (cpu_baseline)"}), flush=True)
            return 0
        res = run_prefill(args)
    else:
        res = run_reference(args) if args.impl == "reference" else run_ours(args)
    if res is not None:
        print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
