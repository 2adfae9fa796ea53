"""Routed-expert slice, combine and synthetic configs on the CPU -- test infrastructure.

The W4A16 decode body restated here is the arithmetic of the reference's v7
kernel (gx/kernels/fp4_decode_moe_swz.cu) written as a float32
dequantize-and-matmul, one expert at a time (the "reference torch path" the
benchmark times on host cores).
"""

from __future__ import annotations

import os
import time

import torch

from . import nvfp4 as q4

HIDDEN = 5120        # gx/gx_expert_worker.py:52 (K)
INTER = 2304         # pack/build_packs.py:50 (moe_intermediate_size)
TOPK = 6             # gx/gx_expert_worker.py:54
SWIGLU_LIMIT = 10.0  # gx/gx_expert_worker.py:1211 (deployed --swiglu-limit)


# ---------------------------------------------------------------- synthetic data

def routing(logits: torch.Tensor, topk: int = TOPK) -> tuple[torch.Tensor, torch.Tensor]:
    """FP32 logits -> softmax -> top-k distinct ids -> weights renormalised to 1."""
    p = torch.softmax(logits.to(torch.float32), dim=-1)
    w, ids = torch.topk(p, topk, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    return ids.to(torch.int32), w.to(torch.float32)


def zipf_bias(n_experts: int, s: float, gen: torch.Generator) -> torch.Tensor:
    """Per-expert logit bias -s*ln(rank), ranks a seeded permutation of 1..E."""
    rank = torch.randperm(n_experts, generator=gen).to(torch.float32) + 1.0
    return -s * torch.log(rank)


def make_activation(rows: int, gen: torch.Generator, hidden: int = HIDDEN):
    """RMSNorm-like N(0,1) rows as bf16, FP8-quantised with one scale per row.

    Returns (x_bf16 as float32, q uint8 [rows, hidden], inv float32 [rows]).
    """
    x = q4.bf16_round(torch.randn(rows, hidden, generator=gen, dtype=torch.float32))
    q, inv = q4.fp8_quant_rows(x)
    return x, q, inv


def make_expert(gen: torch.Generator, hidden: int = HIDDEN, inter: int = INTER, std: float = 0.02):
    """One expert drawn as FP32 N(0, std) and quantised to NVFP4.

    Returns the pack-format tensors (pack/build_packs.py:9-20): w13 codes
    [2*inter, hidden/2] (gate rows then up rows), w13 scales [2*inter, hidden/16],
    g13 (shared by w1 and w3), w2 codes [hidden, inter/2], w2 scales
    [hidden, inter/16], g2.
    """
    w1 = torch.randn(inter, hidden, generator=gen) * std
    w3 = torch.randn(inter, hidden, generator=gen) * std
    w2 = torch.randn(hidden, inter, generator=gen) * std
    w13 = torch.cat([w1, w3], dim=0)
    g13 = q4.global_scale(w13)
    c13, s13 = q4.quantize_nvfp4(w13, g13)
    g2 = q4.global_scale(w2)
    c2, s2 = q4.quantize_nvfp4(w2, g2)
    return dict(c13=c13, s13=s13, g13=g13, c2=c2, s2=s2, g2=g2)


def make_layer(n_experts: int, gen: torch.Generator, hidden: int = HIDDEN, inter: int = INTER):
    """Stacked pack tensors for one MoE layer: c13 [E, 2I, H/2] ... g2 [E]."""
    ex = [make_expert(gen, hidden, inter) for _ in range(n_experts)]
    out = {k: torch.stack([e[k] for e in ex]) for k in ex[0]}
    return out


def random_code_layer(n_experts: int, gen: torch.Generator, hidden: int = HIDDEN, inter: int = INTER):
    """Pack tensors filled with uniform random NVFP4 codes and moderate e4m3 scales.

    For timing only: the CPU path's cost depends on the shapes, not on the
    values, and drawing codes directly skips the quantiser (seconds per expert).
    """
    def codes(*shape):
        return torch.randint(0, 256, shape, generator=gen, dtype=torch.uint8)

    def scales(*shape):  # e4m3 bytes 0x30..0x47: 0.5 .. 3.75
        return torch.randint(0x30, 0x48, shape, generator=gen, dtype=torch.uint8)

    e = n_experts
    return dict(c13=codes(e, 2 * inter, hidden // 2), s13=scales(e, 2 * inter, hidden // 16),
                g13=torch.full((e,), 1e-3), c2=codes(e, hidden, inter // 2),
                s2=scales(e, hidden, inter // 16), g2=torch.full((e,), 1e-3))


def config0(seed: int = 0, n_experts: int = 8, rows: int = 1, hidden: int = HIDDEN,
            inter: int = INTER):
    """8 experts, hidden 5120, intermediate 2304, rows=1, top-6.

    Draw order (fixed): logits, activation, then experts 0..E-1 (w1, w3, w2).
    """
    gen = torch.Generator().manual_seed(seed)
    logits = torch.randn(rows, n_experts, generator=gen)
    ids, tw = routing(logits, min(TOPK, n_experts))
    x, q, inv = make_activation(rows, gen, hidden)
    layer = make_layer(n_experts, gen, hidden, inter)
    return dict(x=x, q=q, inv=inv, ids=ids, tw=tw, **layer)


# ---------------------------------------------------------------- the slice

def slice_w4a16(x: torch.Tensor, ids: torch.Tensor, tw: torch.Tensor, layer: dict,
                c0: int, c1: int, limit: float = SWIGLU_LIMIT, has_limit: bool = True,
                return_act: bool = False, dtype: torch.dtype = torch.float32, round_out: bool = True):
    """BF16 partial [R, H] of the routed experts over intermediate columns [c0, c1).

    x: bf16-valued float32 [R, H] (what the ingest hands the body);
    ids int32 [R, k] in [0, E); tw float32 [R, k];
    layer: pack tensors over the FULL intermediate (c13 [E, 2I, H/2] ...).

    Stage 1 (fp4_decode_moe_swz.cu:287-299): g = x.Wg, u = x.Wu with
    W = e2m1*e4m3*g13; if has_limit: g = min(g, L), u = clamp(u, -L, L);
    act = g / (1 + exp(-g)) * u in float32.
    Stage 2 (:356-385): y_j = (g2[e_j] * tw_j) * act_j.W2 (W2 = e2m1*e4m3 over
    columns [c0, c1)); out = bf16(sum_j y_j), j ascending, one rounding.
    dtype=float64 with round_out=False gives a high-precision value of the same
    expression (diagnostics only).
    """
    r, k = ids.shape
    inter = layer["c13"].shape[1] // 2
    acc = torch.zeros(r, k, x.shape[1], dtype=dtype)
    act_all = torch.zeros(r * k, c1 - c0, dtype=dtype)
    for e in torch.unique(ids).tolist():
        sel = (ids == e).nonzero().tolist()
        rows = [p[0] for p in sel]
        g13 = layer["g13"][e].to(dtype)
        wg = q4.dequant(layer["c13"][e, c0:c1], layer["s13"][e, c0:c1], 1.0).to(dtype) * g13
        wu = q4.dequant(layer["c13"][e, inter + c0:inter + c1],
                        layer["s13"][e, inter + c0:inter + c1], 1.0).to(dtype) * g13
        xr = x[rows].to(dtype)
        g = xr @ wg.T
        u = xr @ wu.T
        del wg, wu
        if has_limit:
            g = torch.clamp(g, max=limit)
            u = torch.clamp(u, min=-limit, max=limit)
        act = g / (1.0 + torch.exp(-g)) * u
        w2 = q4.dequant(layer["c2"][e][:, c0 // 2:c1 // 2], layer["s2"][e][:, c0 // 16:c1 // 16], 1.0).to(dtype)
        y = act @ w2.T
        del w2
        for i, (row, j) in enumerate(sel):
            gw = (layer["g2"][e].to(torch.float32) * tw[row, j].to(torch.float32)).to(dtype)
            acc[row, j] = y[i] * gw
            act_all[row * k + j] = act[i]
    out = acc[:, 0].clone()
    for j in range(1, k):
        out = out + acc[:, j]
    out = q4.bf16_round(out) if round_out else out
    return (out, act_all) if return_act else out


def combine_ordered(parts: list[torch.Tensor], shared: torch.Tensor | None = None,
                    out_f32: bool = False) -> torch.Tensor:
    """Fixed-order combine of BF16 partials: bf16(p0 + p1 + ... [+ shared]) in FP32.

    native/qmesh_afd_seam.cu:310-361: one FP32 accumulator, partials added in
    rank order, one BF16 rounding (or none with out_f32). README.md:88-90 puts
    the shared expert after the routed ranks.
    """
    acc = parts[0].to(torch.float32).clone()
    for p in parts[1:]:
        acc = acc + p.to(torch.float32)
    if shared is not None:
        acc = acc + shared.to(torch.float32)
    return acc if out_f32 else q4.bf16_round(acc)


def shard_ranges(inter: int, n: int) -> list[tuple[int, int]]:
    """N contiguous equal column shards of the intermediate dimension."""
    w = inter // n
    return [(i * w, (i + 1) * w) for i in range(n)]


def cpu_threads() -> int:
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def time_slice(x, ids, tw, layer, c0, c1, reps: int = 1) -> float:
    """Seconds per call of the CPU restatement (the timed CPU baseline)."""
    t0 = time.perf_counter()
    for _ in range(reps):
        slice_w4a16(x, ids, tw, layer, c0, c1)
    return (time.perf_counter() - t0) / reps
