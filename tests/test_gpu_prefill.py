"""Prefill slice (W4A4 grouped tcgen05 block-scaled GEMM, qx_slice_prefill_tc)
against the W4A4 oracle (oracle/prefill.py) on seeded inputs: group sizes from
one pair to several groups of one expert, full and partial column ranges,
FP8 and BF16 activations. The north star's bar applies (relative L2 <= 5e-3,
max 2 BF16 ulp per element)."""

import pytest
import torch

import helpers as H
from oracle import prefill as pf

pytestmark = pytest.mark.gpu


def _calibrated_a2(x, ids, tw, layer, c0, c1, n_experts):
    """a2 = 6 / (1.5 max|c2|): the reference's calibration rule on this batch."""
    st = {}
    pf.slice_w4a4(x, ids, tw, layer, c0, c1, torch.ones(n_experts), stats=st)
    return torch.full((n_experts,), 6.0 / (1.5 * max(st["c2_amax"], 1e-6)))


@pytest.mark.parametrize("n_exp,inter,rows,topk,c0,c1,seed", [
    (8, 256, 32, 6, 0, 256, 1),        # ~24 pairs per expert, 4 column tiles
    (2, 128, 128, 2, 0, 128, 2),       # 128 pairs per expert: two groups each
    (16, 576, 40, 6, 256, 576, 3),     # column sub-range
    (10, 576, 16, 6, 0, 288, 5),       # 288 columns: the last tile is half padding
    (12, 2304, 24, 6, 0, 2304, 4),     # full width, ~12 pairs per expert
])
def test_prefill_matches_w4a4_oracle(cuda_ready, n_exp, inter, rows, topk, c0, c1, seed):
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import prefill_slice
    dev = cuda_ready
    layer = H.small_layer(seed, n_exp, inter=inter)
    ar = Arena(dev, 1, n_exp, 0, inter, layout="tc")
    ar.load_layer(0, layer)
    ids, tw = H.random_routing(rows, n_exp, seed, topk=topk)
    _, q, inv = H.activations(rows, seed)
    x = H.ingest(q, inv)
    a2 = _calibrated_a2(x, ids, tw, layer, c0, c1, n_exp)
    want = pf.slice_w4a4(x, ids, tw, layer, c0, c1, a2)
    out = prefill_slice(ar, 0, q.to(dev), ids.to(dev), tw.to(dev), a2.to(dev), c0=c0, c1=c1, x_scale=inv.to(dev))
    torch.cuda.synchronize()
    H.assert_parity(out, want, f"prefill E={n_exp} W=[{c0},{c1}) rows={rows}")


def test_prefill_bf16_input_and_padding_ids(cuda_ready):
    """BF16 activations (the reference body's own input) and -1 padding slots."""
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import prefill_slice
    dev = cuda_ready
    layer = H.small_layer(9, 6, inter=192)
    ar = Arena(dev, 1, 6, 0, 192, layout="tc")
    ar.load_layer(0, layer)
    ids, tw = H.random_routing(20, 6, 9, topk=4)
    ids[3, 1] = -1
    ids[7] = -1
    _, q, inv = H.activations(20, 9)
    x = H.ingest(q, inv)
    a2 = _calibrated_a2(x, ids, tw, layer, 0, 192, 6)
    want = pf.slice_w4a4(x, ids, tw, layer, 0, 192, a2)
    out = prefill_slice(ar, 0, x.to(torch.bfloat16).to(dev), ids.to(dev), tw.to(dev), a2.to(dev))
    torch.cuda.synchronize()
    H.assert_parity(out, want, "prefill bf16 x")
    assert (out[7].float() == 0).all()
