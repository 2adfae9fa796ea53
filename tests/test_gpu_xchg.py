"""The one-shot NVLink combine (qx_combine_p2p) on 2+ GPUs, one process per GPU:
over several consecutive steps (both receive slots, the acknowledgements) its
output equals the oracle's rank-ordered FP32 sum with one BF16 rounding, bit for
bit, for either output rank and with a shared-expert partial. Skipped on a box
with fewer than two GPUs."""

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
