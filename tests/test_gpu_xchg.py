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
