"""Tensor-core slice internals on the GPU: the activation-term operands the
prologue builds must equal the CPU model of the decomposition bit for bit
(tests/nvfp4_terms.py), so that a parity failure of the full slice can be told
apart from a failure of the operand encoding."""

import pytest
import torch

import helpers as H
import nvfp4_terms as NT
from oracle import nvfp4 as oq

pytestmark = pytest.mark.gpu

HID = 5120
XT_ROW = 80 * 256 + 80 * 32


def _al(v):
    return (v + 255) & ~255


def ws_offsets(rows, topk, width):
    """Byte offsets inside a qx_slice_decode_tc workspace (mirror of its layout)."""
    p, nt = rows * topk, (width + 63) // 64
    o, off = 0, {}
    for name, size in [("ctl", 256), ("groups", p * 64), ("pexp", p * 4), ("pos_pair", p * 4), ("cnt1", p * 4),
                       ("ready", p * 4), ("xready", p * 4), ("emax", p * 4), ("eloc", p * nt * 4),
                       ("xexp", rows * 4), ("xt", rows * XT_ROW)]:
        off[name] = o
        o = _al(o + size)
    return off


def _xt_unpack(xt_row):
    """One staged row -> (codes [8, 5120] nibbles, scales [8, 320])."""
    codes = xt_row[:80 * 256].reshape(80, 2, 8, 16)                  # kb, half, term, byte
    nib = torch.stack([codes & 15, codes >> 4], dim=-1)              # kb, half, term, byte, nibble
    nib = nib.permute(2, 0, 1, 3, 4).reshape(8, HID)
    sc = xt_row[80 * 256:].reshape(80, 8, 4).permute(1, 0, 2).reshape(8, 320)
    return nib, sc


@pytest.mark.parametrize("rows,seed", [(1, 3), (6, 4)])
def test_row_terms_match_cpu_model(cuda_ready, rows, seed):
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
    codes, scales, e = NT.decompose(x)
    assert torch.equal(xexp, e), (xexp, e)
    for r in range(rows):
        nib, sc = _xt_unpack(w[off["xt"] + r * XT_ROW:off["xt"] + (r + 1) * XT_ROW])
        assert torch.equal(sc, scales[r]), f"row {r}: scale bytes differ at {(sc != scales[r]).nonzero()[:5].tolist()}"
        assert torch.equal(nib, codes[r]), f"row {r}: codes differ at {(nib != codes[r]).nonzero()[:5].tolist()}"
    # the terms reproduce the activation to ~2^-24 of each block's maximum
    rec = NT.reconstruct(codes, scales, e)
    blk = x.abs().view(rows, -1, 16).amax(dim=2).repeat_interleave(16, dim=1).double()
    assert ((rec - x.double()).abs() <= blk * 2.0 ** -22 + 1e-30).all()


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
