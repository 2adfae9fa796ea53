"""The shared expert inside the decode kernel (qx_slice_decode_tc_shared), one GPU.

BASELINE config 2 puts a dense NVFP4 SwiGLU (intermediate 2304, weight 1) on the
rank that writes the output, added after the routed partials (README.md:88-90;
native/qmesh_afd_seam.cu:309-361). The kernel runs it as extra work items; its
output must equal the routed partial and a separate shared-expert call (ids 0,
weights 1, one slot) combined in that order, bit for bit, and the oracle's
combine of the two within the north-star tolerance.
"""

import pytest
import torch

import helpers as H
from oracle import moe

pytestmark = pytest.mark.gpu


def _separate(ar, sh, q, inv, ids, tw, c0, c1):
    from qmesh_b200.combine import combine_ordered
    from qmesh_b200.expert_slice import expert_slice
    dev = ar.dev
    rows = q.shape[0]
    routed = expert_slice(ar, 0, q, ids, tw, c0=c0, c1=c1, x_scale=inv)
    zeros = torch.zeros(rows, 1, dtype=torch.int32, device=dev)
    ones = torch.ones(rows, 1, dtype=torch.float32, device=dev)
    shared = expert_slice(sh, 0, q, zeros, ones, x_scale=inv)
    return combine_ordered([routed, shared]), routed, shared


def _fused(ar, sh, q, inv, ids, tw, c0, c1):
    from qmesh_b200.expert_slice import alloc_workspace, device_status, launch
    dev = ar.dev
    rows = q.shape[0]
    ws = alloc_workspace(rows, ids.shape[1], c0, c1, dev)
    out = torch.full((rows, 5120), float("nan"), dtype=torch.bfloat16, device=dev)
    launch(ar.view(0), q, ids, tw, out, c0, c1, ws, x_scale=inv, shared=sh.view(0))
    torch.cuda.synchronize()
    assert device_status(ws) == 0
    return out


def test_shared_expert_small_layer_vs_oracle(cuda_ready):
    from qmesh_b200.arena import Arena
    dev = cuda_ready
    layer = H.small_layer(31, 16, inter=512)
    shl = H.small_layer(32, 1, inter=512)
    ar = Arena(dev, 1, 16, 0, 512)
    ar.load_layer(0, layer)
    sh = Arena(dev, 1, 1, 0, 512)
    sh.load_layer(0, shl)
    for rows, seed in ((6, 1), (1, 2), (13, 3)):
        ids, tw = H.random_routing(rows, 16, seed)
        _, q, inv = H.activations(rows, seed)
        dq, dinv, dids, dtw = q.to(dev), inv.to(dev), ids.to(dev), tw.to(dev)
        fused = _fused(ar, sh, dq, dinv, dids, dtw, 0, 512)
        sep, routed, shared = _separate(ar, sh, dq, dinv, dids, dtw, 0, 512)
        assert torch.equal(fused, sep), f"rows {rows}: fused differs from slice + shared + combine"
        x = H.ingest(q, inv)
        r_ref = H.oracle_out(x, ids, tw, layer, 0, 512)
        s_ref = H.oracle_out(x, torch.zeros(rows, 1, dtype=torch.int32), torch.ones(rows, 1), shl, 0, 512)
        want = moe.combine_ordered([r_ref], shared=s_ref)
        mag = torch.maximum(routed.float().abs().cpu(), shared.float().abs().cpu())
        H.assert_parity(fused, want, f"shared expert rows {rows}", mag=mag)


@pytest.mark.parametrize("c0,c1,rows", [(1152, 1440, 6), (0, 2304, 6), (2016, 2304, 48)])
def test_shared_expert_full_size_equals_separate_calls(cuda_ready, c0, c1, rows):
    """384 routed experts on one rank's shard (288 columns: split gate/up items) or
    all 2304 columns, the shared expert over its full 2304 columns (36 tiles of its
    own split), rows 6 and 48."""
    from qmesh_b200.arena import Arena
    dev = cuda_ready
    ar = Arena(dev, 1, 384, c0, c1)
    ar.fill_synthetic(0, seed=21)
    sh = Arena(dev, 1, 1, 0, 2304)
    sh.fill_synthetic(0, seed=22)
    g = torch.Generator().manual_seed(40 + rows)
    ids, tw = moe.routing(torch.randn(rows, 384, generator=g))
    _, q, inv = moe.make_activation(rows, g)
    dq, dinv, dids, dtw = q.to(dev), inv.to(dev), ids.to(dev), tw.to(dev)
    fused = _fused(ar, sh, dq, dinv, dids, dtw, c0, c1)
    sep, _, _ = _separate(ar, sh, dq, dinv, dids, dtw, c0, c1)
    assert torch.equal(fused, sep)
    again = _fused(ar, sh, dq, dinv, dids, dtw, c0, c1)
    assert torch.equal(fused, again)


def test_host_slice_with_shared_expert(cuda_ready):
    """HostSlice with the shared expert (host inputs, pipelined copies) returns the
    device call's output (routed slice + shared expert in one kernel) over more
    calls than it has staging slots, bit for bit."""
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import HostSlice
    dev = cuda_ready
    ar = Arena(dev, 1, 16, 0, 512)
    ar.load_layer(0, H.small_layer(41, 16, inter=512))
    sh = Arena(dev, 1, 1, 0, 512)
    sh.load_layer(0, H.small_layer(42, 1, inter=512))
    hs = HostSlice(ar, 6, shared=sh.view(0))
    cases, got = [], []
    for step in range(4):
        ids, tw = H.random_routing(6, 16, 60 + step)
        _, q, inv = H.activations(6, 60 + step)
        cases.append((q, inv, ids, tw))
        got.append(hs(0, q, inv, ids, tw, out=torch.empty(6, 5120, dtype=torch.bfloat16).pin_memory()))
    hs.synchronize()
    for step, (q, inv, ids, tw) in enumerate(cases):
        want = _fused(ar, sh, q.to(dev), inv.to(dev), ids.to(dev), tw.to(dev), 0, 512)
        assert torch.equal(got[step], want.cpu()), f"call {step}"
