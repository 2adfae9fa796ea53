"""Shared test helpers: the parity tolerance and small synthetic layers."""

from __future__ import annotations

import functools
import json
import os

import torch

from oracle import moe, nvfp4 as q4

# BF16 partial and combined output within relative-L2 5e-3
# and max-abs 2 BF16 ulp per element.
#
# The ulp of an element is the BF16 spacing at max(|ref|, 2^-10 * rms(row)).
# Below that floor an element is a near-cancellation of terms ~2^10 times
# larger, and any two FP32 summation orders already disagree there by several
# of its own ulps: the FP32 oracle itself is up to 11 ulp from a float64
# evaluation of the same expression on such elements, while the floor still
# allows only ~2^-16 * rms, about 20x the FP32 noise observed.
REL_L2 = 5e-3
MAX_ULP = 2.0
ULP_FLOOR = 2.0 ** -10


def bf16_ulp(v: torch.Tensor) -> torch.Tensor:
    """Spacing of BF16 numbers at |v| (normal range; 2^-133 below it)."""
    a = v.abs().float().clamp_min(2.0 ** -126)
    return torch.pow(2.0, torch.floor(torch.log2(a)) - 7.0)


def element_ulp(ref: torch.Tensor, mag: torch.Tensor | None = None) -> torch.Tensor:
    """BF16 ulp per element at max(|ref|, mag, 2^-10 * rms(row)).

    `mag` is for outputs that are sums of BF16-rounded terms (the combine of
    per-rank partials): their ulp is taken at the largest term, because one
    ulp of a partial is the protocol's own resolution there.
    """
    r2 = ref.reshape(-1, ref.shape[-1]) if ref.dim() > 1 else ref.reshape(1, -1)
    rms = r2.pow(2).mean(dim=-1, keepdim=True).sqrt()
    floor = (ULP_FLOOR * rms).expand_as(r2)
    m = torch.maximum(r2.abs(), floor)
    if mag is not None:
        m = torch.maximum(m, mag.float().cpu().abs().reshape(m.shape))
    return bf16_ulp(m).reshape(ref.shape)


def parity(out: torch.Tensor, ref: torch.Tensor, mag: torch.Tensor | None = None) -> dict:
    """Errors of `out` against `ref`: relative L2; the ulp measure the tolerance
    uses (max_ulp, with the row floor and `mag`); and the literal per-element
    figure of the north star, the BF16 ulp at |ref| alone (max_ulp_floorless),
    with the count of elements beyond 2 such ulp."""
    out = out.float().cpu()
    ref = ref.float().cpu()
    err = (out - ref).abs()
    rel = (err.norm() / ref.norm().clamp_min(1e-30)).item()
    u = err / element_ulp(ref, mag)
    u0 = err / bf16_ulp(ref)
    i = int(u.argmax())
    idx = [int(v) for v in torch.unravel_index(torch.tensor(i), ref.shape)]
    return {"rel_l2": rel, "max_ulp": u.max().item(), "max_abs": err.max().item(),
            "max_ulp_floorless": u0.max().item(), "n_over_2ulp_floorless": int((u0 > MAX_ULP).sum()),
            "n_over_1ulp_floorless": int((u0 > 1.0).sum()), "elements": ref.numel(),
            "exact": float((err == 0).float().mean()), "worst": {"at": idx, "out": out.flatten()[i].item(),
                                                                "ref": ref.flatten()[i].item()}}


def assert_parity(out, ref, what="", mag=None):
    """The north-star tolerance (relative L2 and ulp with the floor). Every call
    prints its figures, floor-free ones included, and appends them as a JSON
    line to $QX_PARITY_LOG when that is set."""
    p = parity(out, ref, mag)
    print(f"parity {what}: relL2 {p['rel_l2']:.2e} max_ulp {p['max_ulp']:.2f} floor-free max_ulp "
          f"{p['max_ulp_floorless']:.2f} ({p['n_over_2ulp_floorless']} of {p['elements']} elements > 2 ulp)")
    log = os.environ.get("QX_PARITY_LOG")
    if log:
        with open(log, "a") as f:
            f.write(json.dumps({"what": what, "test": os.environ.get("PYTEST_CURRENT_TEST", ""),
                                **{k: v for k, v in p.items() if k != "worst"}}) + "\n")
    assert p["rel_l2"] <= REL_L2 and p["max_ulp"] <= MAX_ULP, f"{what} {p}"
    return p


def small_layer(seed: int, n_experts: int, inter: int = 2304):
    gen = torch.Generator().manual_seed(seed)
    return moe.make_layer(n_experts, gen, inter=inter)


@functools.lru_cache(maxsize=2)
def config0_cached(seed: int = 0):
    return moe.config0(seed)


def activations(rows: int, seed: int):
    gen = torch.Generator().manual_seed(seed)
    return moe.make_activation(rows, gen)


def random_routing(rows: int, n_experts: int, seed: int, topk: int = 6):
    gen = torch.Generator().manual_seed(seed)
    return moe.routing(torch.randn(rows, n_experts, generator=gen), topk)


def oracle_out(x_used, ids, tw, layer, c0, c1, limit=10.0, has_limit=True):
    return moe.slice_w4a16(x_used, ids, tw, layer, c0, c1, limit=limit, has_limit=has_limit)


def ingest(q, inv):
    return q4.fp8_ingest(q, inv)
