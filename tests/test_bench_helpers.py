"""Host-side helpers of bench.py on the CPU: the parity statistics that every
bench line reports (BF16 ulp at the largest of |ref|, a floor of 2^-10 rms of
the row and, at N > 1, the largest partial; and the literal, floor-free ulp)."""

import importlib.util
import sys

import torch

from conftest import ROOT


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    argv, sys.argv = sys.argv, ["bench.py"]
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    return mod


def _bf16_next(x: torch.Tensor, k: int = 1) -> torch.Tensor:
    """x (BF16 values) moved k BF16 steps away from zero."""
    b = x.to(torch.bfloat16).view(torch.int16)
    return (b + k).view(torch.bfloat16).float()


def test_ulp_stats_counts_bf16_steps():
    b = _bench()
    g = torch.Generator().manual_seed(5)
    # inside one binade ([4, 8), steps of 2^-5), so a few steps stay in it
    ref = (5.0 + torch.rand(3, 5120, generator=g)).to(torch.bfloat16).float()
    assert b.ulp_stats(ref, ref)["max_ulp"] == 0.0
    one = b.ulp_stats(_bf16_next(ref, 1), ref)
    assert one["max_ulp"] == 1.0 and one["n_over_2ulp"] == 0
    three = b.ulp_stats(_bf16_next(ref, 3), ref)
    assert three["max_ulp"] == 3.0 and three["n_over_2ulp"] == ref.numel()


def test_ulp_stats_floor_and_partial_magnitude():
    b = _bench()
    ref = torch.zeros(1, 5120)
    ref[0, 0] = 64.0                       # rms = 64 / sqrt(5120): the floor 2^-10 rms is tiny
    out = ref.clone()
    out[0, 1] = 2.0 ** -20                 # an error next to a zero reference element
    st = b.ulp_stats(out, ref)
    assert st["max_ulp_floorless"] > 1e6   # literal: the ulp of zero
    assert st["max_ulp"] < 2.0 ** -20 / 2.0 ** -30   # against the floor
    mag = torch.full((1, 5120), 1.0)       # partials of magnitude 1 on every element
    assert b.ulp_stats(out, ref, mag)["max_ulp"] < 1.0

