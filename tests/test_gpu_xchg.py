"""The NVLink rank combines on 2+ GPUs, one process per GPU. The stand-alone
kernel (qx_combine_p2p): over several consecutive steps (both receive slots, the
acknowledgements) its output equals the oracle's rank-ordered FP32 sum with one
BF16 rounding, bit for bit, for either output rank and with a shared-expert
partial. The slice with the combine fused in (qx_slice_decode_tc_xchg): its
output equals the slice partials combined by qx_combine_p2p, bit for bit, also
when driven through HostSlice from host buffers. Both:
a rank that skips a step makes the output rank's bounded waits run out and
report, and the context keeps working. Skipped on a box with fewer than two
GPUs."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG, ROOT

pytestmark = pytest.mark.gpu

STEPS = 5


def _part(step, rank, rows):
    g = torch.Generator().manual_seed(1000 * step + rank)
    return (torch.randn(rows, 5120, generator=g) * (rank + 1)).to(torch.bfloat16)


def _worker(rank, world, port, rows, dst, q):
    import sys
    for p in (str(ROOT), str(PKG)):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from qmesh_b200 import shard
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=__import__("datetime").timedelta(seconds=60))
    xg = None
    try:
        xg = shard.P2PExchange(rows_max=8, dst=dst, device=dev)
        outs = []
        shared = torch.full((rows, 5120), 0.125, dtype=torch.bfloat16, device=dev)
        for step in range(STEPS):
            part = _part(step, rank, rows).to(dev)
            got = xg.combine(part, shared=shared if (rank == dst and step % 2) else None)
            if got is not None:
                outs.append(got.float().cpu().numpy())
        torch.cuda.synchronize()
        q.put((rank, outs, int(xg.status.item())))
    finally:
        if xg is not None:
            xg.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("rows,dst", [(6, 0), (1, 1)])
def test_p2p_combine_matches_oracle(rows, dst):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from oracle import moe
    world = min(torch.cuda.device_count(), 8)
    port = 29500 + os.getpid() % 400 + rows
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rows, dst, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, outs, status = q.get(timeout=180)
        res[r] = (outs, status)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r][1] == 0, f"rank {r} status {res[r][1]}"
        assert (len(res[r][0]) == STEPS) == (r == dst)
    for step in range(STEPS):
        parts = [_part(step, r, rows).float() for r in range(world)]
        shared = torch.full((rows, 5120), 0.125) if step % 2 else None
        want = moe.combine_ordered(parts, shared=shared).to(torch.bfloat16).float()
        assert torch.equal(torch.from_numpy(res[dst][0][step]), want), f"step {step}"


def _lost_worker(rank, world, port, q):
    import sys
    for p in (str(ROOT), str(PKG)):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["QX_TIMEOUT_MS"] = "400"
    from qmesh_b200 import shard
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=__import__("datetime").timedelta(seconds=60))
    xg = None
    try:
        xg = shard.P2PExchange(rows_max=8, dst=0, device=dev)
        part = _part(0, rank, 6).to(dev)
        got = xg.combine(part)                       # step 0: every rank takes part
        torch.cuda.synchronize()
        ok0 = int(xg.status.item())
        if rank != 0:
            pass                                     # step 1: this rank never sends (stays alive, between steps)
        else:
            xg.combine(part)                         # waits (bounded) for a partial that never comes
        torch.cuda.synchronize()
        st = int(xg.status.item())
        # the context stays usable: an ordinary device computation afterwards
        probe = float((torch.arange(1000, device=dev, dtype=torch.float32) * 2).sum().item())
        q.put((rank, ok0, st, probe, None if got is None else got.float().cpu().numpy()))
    finally:
        if xg is not None:
            xg.close()
        dist.destroy_process_group()


def test_p2p_combine_reports_a_missing_rank():
    """Rank 1 skips one step: rank 0's bounded wait runs out (QX_TIMEOUT_MS=400),
    QX_DEV_TIMEOUT is recorded and the GPU context goes on working."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from oracle import moe
    port = 29900 + os.getpid() % 90
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_lost_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, ok0, st, probe, got = q.get(timeout=180)
        res[r] = (ok0, st, probe, got)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0][0] == 0 and res[1][0] == 0                 # step 0 fine on both ranks
    assert res[0][1] == 2 and res[1][1] == 0                 # rank 0 timed out waiting for rank 1
    assert res[0][2] == res[1][2] == 999000.0
    want = moe.combine_ordered([_part(0, 0, 6).float(), _part(0, 1, 6).float()]).to(torch.bfloat16).float()
    assert torch.equal(torch.from_numpy(res[0][3]), want)


# ---- the slice with the combine fused into its finalize (qx_slice_decode_tc_xchg)

def _fused_case(step, rows, n_experts=16):
    from oracle import moe
    g = torch.Generator().manual_seed(500 + step)
    ids, tw = moe.routing(torch.randn(rows, n_experts, generator=g))
    _, q, inv = moe.make_activation(rows, g)
    return ids, tw, q, inv


def _fused_worker(rank, world, port, rows, dst, q):
    import sys
    for p in (str(ROOT), str(PKG)):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from qmesh_b200 import shard
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import alloc_workspace, device_status, expert_slice
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=__import__("datetime").timedelta(seconds=60))
    xf = xc = None
    try:
        a0, a1 = shard.shard_range(rank, world)
        ar = Arena(dev, 1, 16, a0, a1)
        ar.fill_synthetic(0, seed=7)
        xf = shard.P2PExchange(rows_max=8, dst=dst, device=dev)   # fused protocol
        xc = shard.P2PExchange(rows_max=8, dst=dst, device=dev)   # chunk protocol, for the comparison
        ws = alloc_workspace(rows, 6, a0, a1, dev)
        shared = torch.full((rows, 5120), 0.25, dtype=torch.bfloat16, device=dev)
        equal, statuses = [], []
        for step in range(STEPS):
            ids, tw, xq, inv = (t.to(dev) for t in _fused_case(step, rows))
            sh = shared if (rank == dst and step % 2) else None
            out = torch.full((rows, 5120), float("nan"), dtype=torch.bfloat16, device=dev)
            got = xf.slice_combine(ar.view(0), xq, ids, tw, out, a0, a1, ws, x_scale=inv, shared=sh)
            statuses.append(device_status(ws))
            part = expert_slice(ar, 0, xq, ids, tw, x_scale=inv)
            want = xc.combine(part, shared=sh)
            torch.cuda.synchronize()
            if rank == dst:
                equal.append(bool(torch.equal(got, want)))
        q.put((rank, equal, statuses, int(xc.status.item())))
    finally:
        for x in (xf, xc):
            if x is not None:
                x.close()
        dist.destroy_process_group()


def _host_worker(rank, world, port, rows, dst, q):
    import sys
    for p in (str(ROOT), str(PKG)):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from qmesh_b200 import shard
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import HostSlice, expert_slice
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=__import__("datetime").timedelta(seconds=60))
    xf = xc = None
    try:
        a0, a1 = shard.shard_range(rank, world)
        ar = Arena(dev, 1, 16, a0, a1)
        ar.fill_synthetic(0, seed=9)
        xf = shard.P2PExchange(rows_max=rows, dst=dst, device=dev)   # fused, through HostSlice
        xc = shard.P2PExchange(rows_max=rows, dst=dst, device=dev)   # chunk protocol, for the comparison
        hs = HostSlice(ar, rows, 6, a0, a1, xchg=xf)
        got, want = [], []
        for step in range(STEPS):
            ids, tw, xq, inv = _fused_case(step, rows)
            o = torch.empty(rows, 5120, dtype=torch.bfloat16).pin_memory() if rank == dst else None
            r_ = hs(0, xq, inv, ids, tw, out=o)
            got.append(r_ is not None)
            part = expert_slice(ar, 0, xq.to(dev), ids.to(dev), tw.to(dev), x_scale=inv.to(dev))
            w = xc.combine(part)
            if rank == dst:
                want.append((o, w.cpu()))
        hs.synchronize()
        torch.cuda.synchronize()
        equal = [bool(torch.equal(a, b)) for a, b in want] if rank == dst else []
        q.put((rank, got, equal, int(xf.status.item()), int(xc.status.item())))
    finally:
        for x in (xf, xc):
            if x is not None:
                x.close()
        dist.destroy_process_group()


def test_host_slice_fused_combine_equals_slice_then_combine():
    """HostSlice on every rank of the column split (host inputs, pipelined copies,
    the fused slice + combine): the output rank's host output equals the device
    slice partials combined by qx_combine_p2p, bit for bit, over consecutive
    steps; the other ranks' calls return None."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = min(torch.cuda.device_count(), 8)
    rows, dst = 6, 0
    port = 29400 + os.getpid() % 200
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_host_worker, args=(r, world, port, rows, dst, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, got, equal, s1, s2 = q.get(timeout=300)
        res[r] = (got, equal, s1, s2)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r][0] == [r == dst] * STEPS, f"rank {r}: {res[r][0]}"
        assert res[r][2] == 0 and res[r][3] == 0, f"rank {r}: status {res[r][2:]}"
    assert res[dst][1] == [True] * STEPS


@pytest.mark.parametrize("rows,dst", [(6, 0), (3, 1)])
def test_fused_slice_combine_equals_slice_then_combine(rows, dst):
    """Over consecutive steps (both receive slots, the acknowledgements) the fused
    kernel's output on the output rank equals the separate slice partials combined
    by qx_combine_p2p, bit for bit, with and without a shared-expert partial."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = min(torch.cuda.device_count(), 8)
    port = 29600 + os.getpid() % 200 + rows
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, rows, dst, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, equal, statuses, st = q.get(timeout=300)
        res[r] = (equal, statuses, st)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r][1] == [0] * STEPS and res[r][2] == 0, f"rank {r}: {res[r][1]} {res[r][2]}"
    assert res[dst][0] == [True] * STEPS


def _fused_lost_worker(rank, world, port, q):
    import sys
    for p in (str(ROOT), str(PKG)):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["QX_TIMEOUT_MS"] = "400"
    from qmesh_b200 import shard
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import alloc_workspace, device_status
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=__import__("datetime").timedelta(seconds=60))
    xf = None
    try:
        a0, a1 = shard.shard_range(rank, world)
        ar = Arena(dev, 1, 16, a0, a1)
        ar.fill_synthetic(0, seed=7)
        xf = shard.P2PExchange(rows_max=8, dst=0, device=dev)
        ws = alloc_workspace(6, 6, a0, a1, dev)
        ids, tw, xq, inv = (t.to(dev) for t in _fused_case(0, 6))
        out = torch.empty(6, 5120, dtype=torch.bfloat16, device=dev)
        xf.slice_combine(ar.view(0), xq, ids, tw, out, a0, a1, ws, x_scale=inv)   # step 0: every rank
        st0 = device_status(ws)
        if rank == 0:
            xf.slice_combine(ar.view(0), xq, ids, tw, out, a0, a1, ws, x_scale=inv)   # rank 1 never sends
        st1 = device_status(ws)
        probe = float((torch.arange(1000, device=dev, dtype=torch.float32) * 2).sum().item())
        q.put((rank, st0, st1, probe))
    finally:
        if xf is not None:
            xf.close()
        dist.destroy_process_group()


def test_fused_combine_reports_a_missing_rank():
    """Rank 1 skips a step of the fused kernel (between steps, nothing in flight):
    rank 0's bounded waits run out, QX_DEV_TIMEOUT lands in its workspace status
    and the GPU context goes on working."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    port = 29800 + os.getpid() % 90
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_fused_lost_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, st0, st1, probe = q.get(timeout=300)
        res[r] = (st0, st1, probe)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0][0] == 0 and res[1][0] == 0
    assert res[0][1] & 2 and res[1][1] == 0
    assert res[0][2] == res[1][2] == 999000.0


# ---- the shared expert inside the output rank's fused kernel (qx_slice_decode_tc_shared)

def _shared_worker(rank, world, port, rows, q):
    import sys
    for p in (str(ROOT), str(PKG)):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from qmesh_b200 import shard
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import alloc_workspace, device_status, expert_slice
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=__import__("datetime").timedelta(seconds=60))
    xf = xc = None
    try:
        a0, a1 = shard.shard_range(rank, world)
        ar = Arena(dev, 1, 16, a0, a1)
        ar.fill_synthetic(0, seed=7)
        sh = Arena(dev, 1, 1, 0, 2304)             # the shared expert, full width, on the output rank
        sh.fill_synthetic(0, seed=8)
        xf = shard.P2PExchange(rows_max=8, dst=0, device=dev)
        xc = shard.P2PExchange(rows_max=8, dst=0, device=dev)
        ws = alloc_workspace(rows, 6, a0, a1, dev)
        ws_s = alloc_workspace(rows, 1, 0, 2304, dev)
        zeros = torch.zeros(rows, 1, dtype=torch.int32, device=dev)
        ones = torch.ones(rows, 1, dtype=torch.float32, device=dev)
        equal, statuses = [], []
        for step in range(STEPS):
            ids, tw, xq, inv = (t.to(dev) for t in _fused_case(step, rows))
            out = torch.full((rows, 5120), float("nan"), dtype=torch.bfloat16, device=dev)
            got = xf.slice_combine(ar.view(0), xq, ids, tw, out, a0, a1, ws, x_scale=inv,
                                   shared_expert=sh.view(0) if rank == 0 else None)
            statuses.append(device_status(ws))
            part = expert_slice(ar, 0, xq, ids, tw, x_scale=inv)
            sh_out = expert_slice(sh, 0, xq, zeros, ones, x_scale=inv, workspace=ws_s) if rank == 0 else None
            want = xc.combine(part, shared=sh_out)
            torch.cuda.synchronize()
            if rank == 0:
                equal.append(bool(torch.equal(got, want)))
        q.put((rank, equal, statuses))
    finally:
        for x in (xf, xc):
            if x is not None:
                x.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("rows", [6, 2])
def test_fused_combine_with_shared_expert_kernel(rows):
    """The output rank runs the shared expert as extra items of its fused kernel:
    the combined output equals the routed partials plus a separate shared-expert
    call (ids 0, weight 1) combined by qx_combine_p2p, bit for bit, step after step."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = min(torch.cuda.device_count(), 8)
    port = 29700 + os.getpid() % 90 + rows
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_shared_worker, args=(r, world, port, rows, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, equal, statuses = q.get(timeout=300)
        res[r] = (equal, statuses)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r][1] == [0] * STEPS, f"rank {r}: {res[r][1]}"
    assert res[0][0] == [True] * STEPS
