"""The W4A4 prefill oracle (oracle/prefill.py) pinned to vLLM's own NVFP4
activation quantiser and clamp SwiGLU (fixtures in tests/golden/prefill_quant.npz,
made by tests/golden/make_golden.py), plus a small end-to-end self-check of the
restated prefill body against a float64 evaluation of the same expression."""

from pathlib import Path

import numpy as np
import torch

from oracle import moe
from oracle import nvfp4 as q4
from oracle import prefill as pf

GOLD = Path(__file__).resolve().parent / "golden" / "prefill_quant.npz"


def test_act_quant_matches_vllm_reference():
    z = np.load(GOLD)
    x = torch.from_numpy(z["x"])
    for i in range(4):
        nib, sb = pf.act_quant(x, torch.tensor(float(z[f"gs{i}"])))
        assert torch.equal(q4.e2m1_decode(nib), torch.from_numpy(z[f"codes{i}"])), f"codes, global scale {i}"
        assert torch.equal(q4.e4m3_decode(sb), torch.from_numpy(z[f"scale{i}"])), f"scales, global scale {i}"


def test_silu_clamp_matches_vllm_native():
    z = np.load(GOLD)
    h = torch.from_numpy(z["swiglu_h"])
    want = q4.bf16_round(torch.from_numpy(z["swiglu_out"]))
    got = pf.silu_clamp(h[:, :64], h[:, 64:], 10.0)
    ulp = torch.pow(2.0, torch.floor(torch.log2(want.abs().clamp_min(1e-30))) - 7)
    assert ((got - want).abs() <= ulp).all()          # silu as x/(1+e^-x) vs x*sigmoid(x): <= 1 bf16 ulp
    assert (got == want).float().mean() > 0.99


def test_a1_scale_is_bf16():
    x = q4.bf16_round(torch.randn(4, 64) * 3)
    a = pf.a1_scale(x)
    assert float(a) == float(q4.bf16_round(torch.tensor(6.0) / x.abs().amax()))


def test_w4a4_body_small():
    g = torch.Generator().manual_seed(5)
    layer = moe.make_layer(4, g, hidden=5120, inter=64)
    t = 8
    x = q4.bf16_round(torch.randn(t, 5120, generator=g))
    logits = torch.randn(t, 4, generator=g)
    ids, tw = moe.routing(logits, 3)
    a2 = torch.full((4,), 6.0 / 2.0)
    out = pf.slice_w4a4(x, ids, tw, layer, 0, 64, a2, limit=10.0)
    # float64 restatement with the same quantisation decisions
    a1g = pf.a1_scale(x)
    xn, xs = pf.act_quant(x, a1g)
    xq = pf.act_dequant_unscaled(xn, xs).double()
    ref = torch.zeros(t, 5120, dtype=torch.float64)
    for r in range(t):
        for j in range(3):
            e = int(ids[r, j])
            w13 = q4.dequant(layer["c13"][e], layer["s13"][e], 1.0).double()
            c1 = q4.bf16_round(((layer["g13"][e] / a1g).double() * (xq[r] @ w13.T)).float())
            c2 = pf.silu_clamp(c1[:64], c1[64:], 10.0)
            an, as_ = pf.act_quant(c2.view(1, -1), a2[e])
            aq = pf.act_dequant_unscaled(an, as_).double()[0]
            w2 = q4.dequant(layer["c2"][e], layer["s2"][e], 1.0).double()
            c3 = q4.bf16_round(((layer["g2"][e] / a2[e]).double() * (aq @ w2.T)).float())
            ref[r] += q4.bf16_round(c3 * q4.bf16_round(tw[r, j].float())).double()
    assert torch.equal(out, q4.bf16_round(ref.float()))
