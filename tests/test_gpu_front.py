"""Producer side on the device: the FP8 activation quantiser (per row and per
post) bit for bit against the oracle's restatement of the seam arithmetic, its
non-finite path, and the routing front end against softmax/top-k/renormalise."""

import pytest
import torch

from oracle import moe
from oracle import nvfp4 as oq

pytestmark = pytest.mark.gpu


def _rows(rows, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, 5120, generator=g) * torch.exp(torch.randn(rows, 1, generator=g) * 3)
    x[0, :7] = torch.tensor([448.0, -1e-30, 0.0, -0.0, 3.0e5, 1e-7, -2.5])
    if rows > 2:
        x[2] = 0.0                                   # an all-zero row: mc = bf16(1e-6)
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("rows,seed", [(1, 1), (6, 2), (48, 3)])
def test_quant_rows_bit_exact(cuda_ready, rows, seed):
    from qmesh_b200.front import quant_fp8
    x = _rows(rows, seed)
    q, inv = quant_fp8(x.to(cuda_ready))
    wq, winv = oq.fp8_quant_rows(x.float())
    assert torch.equal(q.cpu(), wq)
    assert torch.equal(inv.cpu(), winv)


@pytest.mark.parametrize("rows,seed", [(1, 4), (6, 5), (37, 6)])
def test_quant_post_bit_exact(cuda_ready, rows, seed):
    from qmesh_b200.front import quant_fp8
    x = _rows(rows, seed)
    q, inv = quant_fp8(x.to(cuda_ready), per_post=True)
    wq, winv = oq.fp8_quant_post(x.float())
    assert torch.equal(q.cpu(), wq)
    assert torch.equal(inv.cpu(), winv)


def test_quant_nonfinite_row(cuda_ready):
    """A row with a NaN keeps its bytes, gets inv = 1 and raises the status bit;
    the other rows are quantised as usual."""
    from qmesh_b200.front import quant_fp8
    dev = cuda_ready
    x = _rows(4, 7)
    x[1, 100] = float("nan")
    q = torch.full((4, 5120), 0xAB, dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    q, inv = quant_fp8(x.to(dev), q=q, status=status)
    assert int(status.item()) == 8
    assert float(inv[1]) == 1.0 and (q[1] == 0xAB).all()
    wq, winv = oq.fp8_quant_rows(x[[0, 2, 3]].float())
    assert torch.equal(q.cpu()[[0, 2, 3]], wq) and torch.equal(inv.cpu()[[0, 2, 3]], winv)


@pytest.mark.parametrize("rows,experts,topk,seed", [(6, 384, 6, 1), (48, 384, 6, 2), (5, 16, 8, 3)])
def test_route_topk(cuda_ready, rows, experts, topk, seed):
    from qmesh_b200.front import route_topk
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(rows, experts, generator=g) * 2
    ids, tw = route_topk(logits.to(cuda_ready), topk)
    wids, wtw = moe.routing(logits, topk)
    assert torch.equal(ids.cpu(), wids)
    assert torch.allclose(tw.cpu(), wtw, rtol=2e-6, atol=0)
    assert torch.allclose(tw.sum(dim=1).cpu(), torch.ones(rows), rtol=1e-6)


def test_route_topk_ties_take_the_lower_id(cuda_ready):
    from qmesh_b200.front import route_topk
    logits = torch.zeros(2, 64)
    logits[0, [5, 9, 40]] = 3.0
    logits[1, [63, 1]] = 2.0
    ids, tw = route_topk(logits.to(cuda_ready), 4)
    assert ids.cpu()[0, :3].tolist() == [5, 9, 40] and ids.cpu()[1, :2].tolist() == [1, 63]
    assert ids.cpu()[0, 3] == 0 and ids.cpu()[1, 2:].tolist() == [0, 2]
