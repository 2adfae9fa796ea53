"""Column-split host logic on two gloo ranks (CPU): shard assignment, rank-ordered
gather, and the combine on the output rank. The device combine kernel is
replaced by the oracle's FP32 rank-order sum (the kernel itself is checked
bit-exact against the same oracle on the GPU)."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG, ROOT


def _worker(rank, world, port, q):
    import sys
    for p in (str(ROOT), str(PKG)):
        sys.path.insert(0, p)
    from oracle import moe
    from qmesh_b200 import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a0, a1 = shard.shard_range(rank, world)
        # each rank's "partial": a rank-tagged BF16 tensor standing for its slice output
        g = torch.Generator().manual_seed(100 + rank)
        part = (torch.randn(3, 5120, generator=g) * (rank + 1)).to(torch.bfloat16)
        shared = torch.full((3, 5120), 0.125, dtype=torch.bfloat16)

        def cpu_combine(parts, out=None):
            return moe.combine_ordered([p.float() for p in parts]).to(torch.bfloat16)

        got = shard.combine_across_ranks(part, dst=0, shared=shared if rank == 0 else None, combine=cpu_combine)
        gathered = shard.gather_partials(part)
        q.put((rank, (a0, a1), None if got is None else got.float().numpy(),
               [t.float().numpy() for t in gathered]))
    finally:
        dist.destroy_process_group()


def test_column_split_two_ranks():
    world, port = 2, 29000 + os.getpid() % 1000
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, rng, got, gathered = q.get(timeout=120)
        res[r] = (rng, got, gathered)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][0] == (0, 1152) and res[1][0] == (1152, 2304)
    assert res[1][1] is None
    parts = []
    for r in range(world):
        g = torch.Generator().manual_seed(100 + r)
        parts.append((torch.randn(3, 5120, generator=g) * (r + 1)).to(torch.bfloat16).float())
    # gathered in rank order on every rank
    for r in range(world):
        for i in range(world):
            assert torch.equal(torch.from_numpy(res[r][2][i]), parts[i])
    want = (parts[0] + parts[1] + torch.full((3, 5120), 0.125)).to(torch.bfloat16).float()
    assert torch.equal(torch.from_numpy(res[0][1]), want)


def _rows_worker(rank, world, port, rows, q):
    import sys
    for p in (str(ROOT), str(PKG)):
        sys.path.insert(0, p)
    from oracle import moe
    from qmesh_b200 import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(300 + rank)
        part = (torch.randn(rows, 5120, generator=g) * (rank + 1)).to(torch.bfloat16)

        def cpu_combine(parts, out=None):
            r = moe.combine_ordered([p.float() for p in parts]).to(torch.bfloat16)
            if out is not None:
                out.copy_(r)
                return out
            return r

        by_rows = shard.combine_rows_across_ranks(part, dst=world - 1, combine=cpu_combine)
        by_gather = shard.combine_across_ranks(part, dst=world - 1, combine=cpu_combine)
        q.put((rank, None if by_rows is None else by_rows.float().numpy(),
               None if by_gather is None else by_gather.float().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,rows", [(2, 7), (3, 10), (2, 8)])
def test_row_split_combine_equals_gather_combine(world, rows):
    """The row-split combine (all-to-all of row blocks, per-rank ordered sums, the
    blocks collected on the output rank) gives the gather combine's bytes, with
    row counts that do not divide by the rank count (point-to-point collection)
    and that do (all-gather collection)."""
    port = 29100 + os.getpid() % 700 + world
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rows_worker, args=(r, world, port, rows, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, a, b = q.get(timeout=120)
        res[r] = (a, b)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world - 1):
        assert res[r] == (None, None)
    a, b = res[world - 1]
    assert a is not None and (a == b).all()


def test_row_bounds_cover_every_row_once():
    from qmesh_b200 import shard
    for rows, world in ((7, 2), (10, 3), (2048, 8), (8, 8)):
        b = shard.row_bounds(rows, world)
        assert b[0] == 0 and b[-1] == rows and len(b) == world + 1
        assert all(b[k + 1] - b[k] in (rows // world, rows // world + 1) for k in range(world))


def test_shard_range_rules():
    from qmesh_b200 import shard
    assert [shard.shard_range(r, 8) for r in range(8)][-1] == (2016, 2304)
    assert shard.shard_range(0, 1) == (0, 2304)
    assert shard.shard_range(2, 3) == (1536, 2304)
    with pytest.raises(ValueError):
        shard.shard_range(0, 5)       # 2304 does not divide by 5
    with pytest.raises(ValueError):
        shard.shard_range(0, 16)      # 144-column shards are not 32-aligned
    with pytest.raises(ValueError):
        shard.shard_range(2, 2)
