"""Tensor-core slice internals on the GPU: the x-term operands the kernel
builds must equal the CPU model of the decomposition bit for bit
(tests/nvfp4_terms.py), so that a parity failure of the full slice can be told
apart from a failure of the operand encoding; and slices whose width is not a
multiple of the 64-column tile."""

import pytest
import torch

import helpers as H
import nvfp4_terms as NT
from oracle import nvfp4 as oq

pytestmark = pytest.mark.gpu

HID = 5120


def _al(v):
    return (v + 255) & ~255


def ws_offsets(rows, topk, width):
    """Byte offsets inside a qx_slice_decode_tc workspace (mirror of its layout)."""
    p = rows * topk
    ps = p + rows                                  # routed pairs, then the shared expert's rows
    maxsplit, maxsg, max_stiles = 512, (64 + 5) // 6, 64
    o, off = 0, {}
    for name, size in [("ctl", 256), ("cnt1", ps * 4), ("ready", ps * 4), ("fcnt", 40 * 4),
                       ("pcnt", (maxsplit + maxsg * max_stiles) * 4), ("emax", ps * 4),
                       ("eloc", ps * max_stiles * 4),
                       ("xexp", rows * 4), ("xt", rows * 10 * 4096)]:
        off[name] = o
        o = _al(o + size)
    return off


def _kb_unpack(blk, kb):
    """K block kb of one row's 16 x terms from that row's 4,096-byte stage block
    ([row group 2][K block 8][K half 2][term 8][16 bytes]) -> nibbles [16 terms, 64]."""
    b = blk.reshape(2, 8, 2, 8, 16)[:, kb % 8]                        # rg, half, term, byte
    nib = torch.stack([b & 15, b >> 4], dim=-1)                       # rg, half, term, byte, nibble
    return nib.permute(0, 2, 1, 3, 4).reshape(16, 64)


@pytest.mark.parametrize("rows,seed", [(1, 3), (6, 4)])
def test_x_terms_match_cpu_model(cuda_ready, rows, seed):
    """The prep kernel's x terms of every row, read back in the row-major operand
    layout, equal the CPU model of the decomposition bit for bit, and the row
    exponents match."""
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import alloc_workspace, expert_slice
    dev = cuda_ready
    layer = H.small_layer(31, 8, inter=256)
    ar = Arena(dev, 1, 8, 0, 256, layout="tc")
    ar.load_layer(0, layer)
    ids, tw = H.random_routing(rows, 8, seed)
    _, q, inv = H.activations(rows, seed)
    ws = alloc_workspace(rows, 6, 0, 256, dev, "tc")
    expert_slice(ar, 0, q.to(dev), ids.to(dev), tw.to(dev), x_scale=inv.to(dev), workspace=ws)
    torch.cuda.synchronize()
    off = ws_offsets(rows, 6, 256)
    w = ws.cpu()
    xexp = w[off["xexp"]:off["xexp"] + rows * 4].view(torch.int32)
    x = H.ingest(q, inv)
    codes, e = NT.decompose_x(x)
    assert torch.equal(xexp, e), (xexp, e)
    for r in range(rows):
        for kb in range(80):
            base = off["xt"] + (r * 10 + kb // 8) * 4096
            got = _kb_unpack(w[base:base + 4096], kb)
            want = codes[r, :, kb * 64:(kb + 1) * 64]
            assert torch.equal(got, want), f"row {r} K block {kb}"
    rec_x = NT.reconstruct_x(codes, e)
    amax = x.abs().amax(dim=1, keepdim=True).double()
    assert ((rec_x - x.double()).abs() <= amax * 2.0 ** -30).all()


def test_width_not_multiple_of_64(cuda_ready):
    """An arena of 288 columns (the 8-way shard width): the last 64-column tile is
    half padding, and the slice still matches the oracle."""
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import expert_slice
    dev = cuda_ready
    layer = H.small_layer(32, 8, inter=576)
    ar = Arena(dev, 1, 8, 288, 576, layout="tc")
    ar.load_layer(0, layer)
    rows = 6
    ids, tw = H.random_routing(rows, 8, 7)
    _, q, inv = H.activations(rows, 7)
    out = expert_slice(ar, 0, q.to(dev), ids.to(dev), tw.to(dev), x_scale=inv.to(dev))
    torch.cuda.synchronize()
    H.assert_parity(out, H.oracle_out(H.ingest(q, inv), ids, tw, layer, 288, 576), "288-column arena")
    # a 64-aligned sub-range ending inside a tile
    out2 = expert_slice(ar, 0, q.to(dev), ids.to(dev), tw.to(dev), c0=288, c1=416, x_scale=inv.to(dev))
    torch.cuda.synchronize()
    H.assert_parity(out2, H.oracle_out(H.ingest(q, inv), ids, tw, layer, 288, 416), "[288, 416)")
    _ = oq


def test_host_slice_matches_device_call(cuda_ready):
    """HostSlice (host inputs, one packed copy each way) returns the device call's
    output, over more calls than it has staging slots and with a short call."""
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import HostSlice, expert_slice
    dev = cuda_ready
    layer = H.small_layer(33, 8, inter=256)
    ar = Arena(dev, 1, 8, 0, 256, layout="tc")
    ar.load_layer(0, layer)
    hs = HostSlice(ar, 6)
    outs = []
    for step, rows in enumerate([6, 6, 3, 6]):
        ids, tw = H.random_routing(rows, 8, 50 + step)
        _, q, inv = H.activations(rows, 50 + step)
        got = hs(0, q, inv, ids, tw)
        want = expert_slice(ar, 0, q.to(dev), ids.to(dev), tw.to(dev), x_scale=inv.to(dev))
        outs.append((got, want))
        torch.cuda.synchronize()
        assert torch.equal(got, want.cpu()), f"call {step}"


def test_host_slice_pipelined_calls(cuda_ready):
    """Back-to-back HostSlice calls with no host synchronisation between them
    (input copies overlap the previous call's slice, output copies the next
    call's): after synchronize() the last two calls' outputs (one per staging
    slot) equal the device calls'."""
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import HostSlice, expert_slice
    dev = cuda_ready
    layer = H.small_layer(34, 8, inter=256)
    ar = Arena(dev, 1, 8, 0, 256, layout="tc")
    ar.load_layer(0, layer)
    hs = HostSlice(ar, 6)
    cases, got = [], []
    for step in range(5):
        ids, tw = H.random_routing(6, 8, 70 + step)
        _, q, inv = H.activations(6, 70 + step)
        cases.append((q, inv, ids, tw))
        got.append(hs(0, q, inv, ids, tw))
    hs.synchronize()
    for step in (3, 4):
        q, inv, ids, tw = cases[step]
        want = expert_slice(ar, 0, q.to(dev), ids.to(dev), tw.to(dev), x_scale=inv.to(dev))
        torch.cuda.synchronize()
        assert torch.equal(got[step], want.cpu()), f"call {step}"


def test_host_slice_out_keeps_every_call(cuda_ready):
    """With `out`, each of five pipelined calls' outputs lands in the caller's own
    pinned tensor and all five stay valid (without it only the last two would)."""
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import HostSlice, expert_slice
    dev = cuda_ready
    layer = H.small_layer(35, 8, inter=256)
    ar = Arena(dev, 1, 8, 0, 256, layout="tc")
    ar.load_layer(0, layer)
    hs = HostSlice(ar, 6)
    cases, outs = [], []
    for step in range(5):
        ids, tw = H.random_routing(6, 8, 90 + step)
        _, q, inv = H.activations(6, 90 + step)
        cases.append((q, inv, ids, tw))
        o = torch.empty(6, 5120, dtype=torch.bfloat16).pin_memory()
        assert hs(0, q, inv, ids, tw, out=o) is o
        outs.append(o)
    hs.synchronize()
    for step, (q, inv, ids, tw) in enumerate(cases):
        want = expert_slice(ar, 0, q.to(dev), ids.to(dev), tw.to(dev), x_scale=inv.to(dev))
        torch.cuda.synchronize()
        assert torch.equal(outs[step], want.cpu()), f"call {step}"
