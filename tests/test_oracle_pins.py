"""Pin the CPU oracle to the reference: golden fixtures made by running the
reference's own code (tests/golden/make_golden.py) and known-answer tables."""

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import moe, nvfp4 as q4


def test_e4m3_decode_all_bytes_match_torch():
    b = torch.arange(256, dtype=torch.uint8)
    ours = q4.e4m3_decode(b)
    ref = b.view(torch.float8_e4m3fn).float()
    same = (ours == ref) | (torch.isnan(ours) & torch.isnan(ref))
    assert bool(same.all())
    assert torch.isnan(ours[0x7F]) and torch.isnan(ours[0xFF])
    assert ours[0x7E] == 448.0 and ours[0x01] == 2.0 ** -9


def test_e2m1_table_known_answers():
    # NVFP4 e2m1: sign bit 3, magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}
    want = [0, .5, 1, 1.5, 2, 3, 4, 6, -0.0, -.5, -1, -1.5, -2, -3, -4, -6]
    got = q4.e2m1_decode(torch.arange(16, dtype=torch.uint8)).tolist()
    assert got == want
    assert torch.signbit(q4.e2m1_decode(torch.tensor([8], dtype=torch.uint8)))[0]


def test_e2m1_encode_round_to_nearest_even():
    v = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 0.26, 7.0, -0.74, -100.0])
    codes = q4.e2m1_encode(v)
    assert q4.e2m1_decode(codes).tolist() == [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 0.5, 6.0, -0.5, -6.0]


def test_nibble_order_low_is_even():
    # byte 0x21: low nibble 1 (0.5) is element 0, high nibble 2 (1.0) is element 1
    vals = q4.e2m1_decode(q4.unpack_codes(torch.tensor([[0x21]], dtype=torch.uint8)))
    assert vals.tolist() == [[0.5, 1.0]]
    nib = torch.randint(0, 16, (4, 64), dtype=torch.uint8)
    assert torch.equal(q4.unpack_codes(q4.pack_codes(nib)), nib)


def test_hand_computed_block():
    # one 16-element block: codes 0..15 (nibbles), scale e4m3 0x38 (= 1.0), gscale 0.5
    nib = torch.arange(16, dtype=torch.uint8).reshape(1, 16)
    codes = q4.pack_codes(nib)
    w = q4.dequant(codes, torch.tensor([[0x38]], dtype=torch.uint8), 0.5)
    want = [0, .25, .5, .75, 1, 1.5, 2, 3, -0.0, -.25, -.5, -.75, -1, -1.5, -2, -3]
    assert w.tolist() == [want]


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_swizzle_map_matches_vllm(case):
    d = np.load(GOLDEN / "swizzle.npz")
    lin = torch.from_numpy(d[f"{case}_lin"])
    swz = torch.from_numpy(d[f"{case}_swz"])
    ours = q4.swizzle_scales(lin)
    assert ours.shape == swz.shape
    assert torch.equal(ours, swz)
    m, kb = lin.shape[-2:]
    assert torch.equal(q4.unswizzle_scales(swz, m, kb), lin)


def test_swiglu_matches_reference_form():
    d = np.load(GOLDEN / "swiglu.npz")
    h = torch.from_numpy(d["h"])
    cp = h.shape[1] // 2
    g, u = h[:, :cp], h[:, cp:]
    ours = g / (1.0 + torch.exp(-g)) * u
    torch.testing.assert_close(ours, torch.from_numpy(d["out"]), rtol=2e-6, atol=1e-6)


def test_ingest_matches_reference_kernel():
    """The FP32 product float(e4m3) * inv of gx_ingest._ingest, run by Triton's CPU
    interpreter, matches the oracle bit for bit.

    The interpreter narrows FP32 -> BF16 by truncation, while the compiled kernel
    uses Triton's default round-to-nearest-even (``fp_downcast_rounding`` unset),
    so the fixture is compared with the oracle's product truncated the same way;
    the oracle itself keeps the hardware's nearest-even rounding.
    """
    d = np.load(GOLDEN / "ingest.npz")
    n = int(d["n"])
    slab = torch.from_numpy(d["slab"])
    inv = torch.full((n,), float(d["inv"]), dtype=torch.float32)
    prod = q4.e4m3_decode(slab) * inv.unsqueeze(-1)
    trunc = (prod.view(torch.int32) & ~0xFFFF).view(torch.float32)
    assert torch.equal(trunc, torch.from_numpy(d["x"][:n]))
    x = q4.fp8_ingest(slab, inv)
    assert torch.equal(x, prod.to(torch.bfloat16).float())
    assert ((x - prod).abs() <= (trunc - prod).abs() + 0).all()  # nearest is never farther
    assert not d["x"][n:].any()  # padding rows are zero
    # sentinel policy of the same kernel: -1 -> padding, other out-of-range -> corrupt
    assert int(d["pad"][0]) == 1 and int(d["bad"][0]) == 2
    assert (d["tw_out"][0] == d["tw"][0]).all() and d["tw_out"][1, 0] == 0.0


def test_fp8_row_quant_round_trip():
    g = torch.Generator().manual_seed(3)
    x = q4.bf16_round(torch.randn(4, 5120, generator=g) * 2)
    q, inv = q4.fp8_quant_rows(x)
    # the per-row maximum maps onto 448 and back within e4m3 precision
    back = q4.fp8_ingest(q, inv)
    rel = ((back - x).norm() / x.norm()).item()
    assert rel < 0.04
    assert (q4.e4m3_decode(q).abs().amax(dim=1) == 448.0).all()


def test_quantizer_reconstructs_within_fp4_error():
    g = torch.Generator().manual_seed(5)
    w = torch.randn(64, 512, generator=g) * 0.02
    gs = q4.global_scale(w)
    codes, scales = q4.quantize_nvfp4(w, gs)
    back = q4.dequant(codes, scales, gs)
    rel = ((back - w).norm() / w.norm()).item()
    assert 0.03 < rel < 0.15


def test_routing_matches_reference():
    from qmesh_b200 import routing
    d = json.loads((GOLDEN / "routing.json").read_text())
    for n, v in d["bucket_of"].items():
        assert routing.bucket_of(int(n)) == v
    for n, v in d["graph_rows"].items():
        assert routing.graph_rows(int(n)) == v
    for ids, want in d["classify_ids"]:
        assert list(routing.classify_ids(np.array(ids))) == want
    assert routing.E == d["E"] and routing.TOPK == d["TOPK"] and routing.GRAPH_MAX == d["GRAPH_MAX"]


def test_routing_gate_refuses_corrupt_ids():
    from qmesh_b200 import routing
    assert routing.routing_gate(np.array([[-1, 0, 5, 383, -1, 1]])) == 2
    with pytest.raises(routing.RoutingError):
        routing.routing_gate(np.array([[0, 384, 1, 2, 3, 4]]))
    with pytest.raises(routing.RoutingError):
        routing.routing_gate(np.array([[-2, 0, 1, 2, 3, 4]]))


def test_arena_bytes_equal_reference_at_its_geometry():
    """The tile layout stores exactly the reference arena's bytes at CP = 896."""
    from qmesh_b200.arena import Arena
    d = json.loads((GOLDEN / "arena.json").read_text())
    assert Arena.layer_bytes(384, d["cp"]) == d["bytes_per_layer"]


def test_oracle_column_split_is_additive():
    """Partials over column shards sum (before rounding) to the full slice."""
    c = moe.config0(seed=7, n_experts=4, rows=2, inter=256)
    x = q4.fp8_ingest(c["q"], c["inv"])
    full = moe.slice_w4a16(x, c["ids"], c["tw"], c, 0, 256)
    parts = [moe.slice_w4a16(x, c["ids"], c["tw"], c, a, b) for a, b in moe.shard_ranges(256, 4)]
    comb = moe.combine_ordered(parts)
    rel = ((comb - full).norm() / full.norm()).item()
    assert rel < 5e-3


def test_ulp_floor_definition():
    import helpers as H
    ref = torch.tensor([[1.0, 0.5, 1e-6, -1e-6] + [1.0] * 60])
    u = H.element_ulp(ref)
    assert u[0, 0] == 2.0 ** -7 and u[0, 1] == 2.0 ** -8
    # tiny elements use the floor 2^-10 * rms (rms just under 1) -> ulp 2^-18
    assert u[0, 2] == u[0, 3] == 2.0 ** -18
