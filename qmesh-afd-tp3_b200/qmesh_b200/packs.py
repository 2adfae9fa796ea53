"""Rank-pack importer: the reference's NVFP4 routed-expert packs into an Arena.

The reference slices the checkpoint's routed experts into one pack per rank
(pack/build_packs.py): a directory per rank holding `experts-L{l:02d}.safetensors`
per MoE layer, with intermediate columns [a, b) of every expert and the bytes
left exactly as the checkpoint stores them:

  stacked form (node-b, node-c; build_packs.py:138-148):
    L{l}.w13.weight          U8       [E, 2C, 2560]   gate rows, then up rows
    L{l}.w13.weight_scale    F8_E4M3  [E, 2C, 320]
    L{l}.w13.weight_scale_2  F32      [E, 2]          w1 and w3 share it
    L{l}.w13.input_scale     F32      [E, 2]
    L{l}.w2.weight           U8       [E, 5120, C/2]
    L{l}.w2.weight_scale     F8_E4M3  [E, 5120, C/16]
    L{l}.w2.weight_scale_2   F32      [E]
    L{l}.w2.input_scale      F32      [E]
  per-expert form (p7, the rank vLLM itself loads; build_packs.py:120-135):
    L{l}.e{e}.{w1,w3}.{weight [C, 2560], weight_scale [C, 320], weight_scale_2 [], input_scale []}
    L{l}.e{e}.w2.{weight [5120, C/2], weight_scale [5120, C/16], weight_scale_2 [], input_scale []}

`read_layer` returns the pack tensors the Arena loads (c13, s13, g13, c2, s2,
g2, plus the W4A4 input scales in13 / in2); `load_rank` fills an arena whose
columns lie inside the rank's slice. Scales are the checkpoint's linear e4m3
bytes; a reference arena already on a device (vLLM-swizzled scales) imports
through `qmesh_b200.nvfp4.unswizzle_scales`.
"""

from __future__ import annotations

import os
import re

import torch

HIDDEN = 5120
SPLIT = {"p7": (0, 576), "node-b": (576, 1440), "node-c": (1440, 2304)}   # build_packs.py:43


def layer_file(root: str, rank: str, layer: int) -> str:
    return os.path.join(root, rank, f"experts-L{layer:02d}.safetensors")


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.dtype != torch.uint8 else t


def _shared_scale(a: torch.Tensor, what: str) -> torch.Tensor:
    a = a.to(torch.float32)
    if a.dim() == 2:
        if not torch.equal(a[:, 0], a[:, 1]):
            raise ValueError(f"{what}: w1 and w3 scales differ")
        a = a[:, 0]
    return a.contiguous()


def read_layer(path: str, layer: int) -> dict:
    """One layer of a rank pack -> {c13, s13, g13, c2, s2, g2, in13, in2} (CPU tensors)."""
    from safetensors import safe_open
    with safe_open(path, framework="pt") as f:
        keys = set(f.keys())
        get = f.get_tensor
        if f"L{layer}.w13.weight" in keys:
            p = f"L{layer}."
            out = dict(c13=_u8(get(p + "w13.weight")), s13=_u8(get(p + "w13.weight_scale")),
                       c2=_u8(get(p + "w2.weight")), s2=_u8(get(p + "w2.weight_scale")),
                       g13=_shared_scale(get(p + "w13.weight_scale_2"), "weight_scale_2"),
                       g2=get(p + "w2.weight_scale_2").to(torch.float32).contiguous())
            out["in13"] = (_shared_scale(get(p + "w13.input_scale"), "input_scale")
                           if p + "w13.input_scale" in keys else None)
            out["in2"] = get(p + "w2.input_scale").to(torch.float32) if p + "w2.input_scale" in keys else None
        else:
            pat = re.compile(rf"^L{layer}\.e(\d+)\.w1\.weight$")
            experts = sorted(int(m.group(1)) for k in keys if (m := pat.match(k)))
            if experts != list(range(len(experts))) or not experts:
                raise ValueError(f"{path}: no complete expert list for layer {layer}")
            c13, s13, c2, s2, g13, g2, in13, in2 = [], [], [], [], [], [], [], []
            for e in experts:
                p = f"L{layer}.e{e}."
                c13.append(torch.cat([_u8(get(p + "w1.weight")), _u8(get(p + "w3.weight"))]))
                s13.append(torch.cat([_u8(get(p + "w1.weight_scale")), _u8(get(p + "w3.weight_scale"))]))
                c2.append(_u8(get(p + "w2.weight")))
                s2.append(_u8(get(p + "w2.weight_scale")))
                a, b = get(p + "w1.weight_scale_2").float(), get(p + "w3.weight_scale_2").float()
                if not torch.equal(a, b):
                    raise ValueError(f"{path}: expert {e} w1 and w3 weight_scale_2 differ")
                g13.append(a.reshape(()))
                g2.append(get(p + "w2.weight_scale_2").float().reshape(()))
                if p + "w1.input_scale" in keys:
                    in13.append(get(p + "w1.input_scale").float().reshape(()))
                    in2.append(get(p + "w2.input_scale").float().reshape(()))
            out = dict(c13=torch.stack(c13), s13=torch.stack(s13), c2=torch.stack(c2), s2=torch.stack(s2),
                       g13=torch.stack(g13), g2=torch.stack(g2),
                       in13=torch.stack(in13) if in13 else None, in2=torch.stack(in2) if in2 else None)
    e, two_c, kh = out["c13"].shape
    c = two_c // 2
    if (kh != HIDDEN // 2 or tuple(out["s13"].shape) != (e, two_c, HIDDEN // 16)
            or tuple(out["c2"].shape) != (e, HIDDEN, c // 2) or tuple(out["s2"].shape) != (e, HIDDEN, c // 16)
            or out["g13"].shape != (e,) or out["g2"].shape != (e,)):
        raise ValueError(f"{path}: layer {layer} tensors do not have the pack shapes "
                         f"(c13 {tuple(out['c13'].shape)}, c2 {tuple(out['c2'].shape)})")
    return out


def load_rank(arena, root: str, rank: str, layers=None, split: dict | None = None) -> None:
    """Fill `arena` (columns [a0, a1) inside the rank's slice) from a rank pack."""
    a, b = (split or SPLIT)[rank]
    if arena.a0 < a or arena.a1 > b:
        raise ValueError(f"arena columns [{arena.a0}, {arena.a1}) are not inside rank {rank}'s [{a}, {b})")
    for li in (range(arena.layers) if layers is None else layers):
        pack = read_layer(layer_file(root, rank, li), li)
        if pack["c13"].shape[1] // 2 != b - a:
            raise ValueError(f"rank {rank} layer {li} holds {pack['c13'].shape[1] // 2} columns, split says {b - a}")
        arena.load_layer(li, pack, src_a0=a)


def write_layer(path: str, layer: int, full: dict, a: int, b: int, per_expert: bool = False) -> None:
    """Columns [a, b) of full-width pack tensors written in the reference's pack
    format (the stacked or the per-expert form), e.g. to make test packs."""
    from safetensors.torch import save_file
    inter = full["c13"].shape[1] // 2
    e = full["c13"].shape[0]
    f8 = lambda t: t.contiguous().view(torch.float8_e4m3fn)
    g13 = full["g13"].to(torch.float32).reshape(e)
    g2 = full["g2"].to(torch.float32).reshape(e)
    in13 = full.get("in13", torch.ones(e)).to(torch.float32).reshape(e)
    in2 = full.get("in2", torch.ones(e)).to(torch.float32).reshape(e)
    t = {}
    if per_expert:
        for x in range(e):
            p = f"L{layer}.e{x}."
            t[p + "w1.weight"] = full["c13"][x, a:b].contiguous()
            t[p + "w3.weight"] = full["c13"][x, inter + a:inter + b].contiguous()
            t[p + "w1.weight_scale"] = f8(full["s13"][x, a:b])
            t[p + "w3.weight_scale"] = f8(full["s13"][x, inter + a:inter + b])
            t[p + "w2.weight"] = full["c2"][x, :, a // 2:b // 2].contiguous()
            t[p + "w2.weight_scale"] = f8(full["s2"][x, :, a // 16:b // 16])
            for w in ("w1", "w3"):
                t[p + w + ".weight_scale_2"] = g13[x].clone()
                t[p + w + ".input_scale"] = in13[x].clone()
            t[p + "w2.weight_scale_2"] = g2[x].clone()
            t[p + "w2.input_scale"] = in2[x].clone()
    else:
        p = f"L{layer}."
        t[p + "w13.weight"] = torch.cat([full["c13"][:, a:b], full["c13"][:, inter + a:inter + b]], dim=1).contiguous()
        t[p + "w13.weight_scale"] = f8(torch.cat([full["s13"][:, a:b], full["s13"][:, inter + a:inter + b]], dim=1))
        t[p + "w2.weight"] = full["c2"][:, :, a // 2:b // 2].contiguous()
        t[p + "w2.weight_scale"] = f8(full["s2"][:, :, a // 16:b // 16])
        t[p + "w13.weight_scale_2"] = torch.stack([g13, g13], dim=1).contiguous()
        t[p + "w13.input_scale"] = torch.stack([in13, in13], dim=1).contiguous()
        t[p + "w2.weight_scale_2"] = g2.contiguous()
        t[p + "w2.input_scale"] = in2.contiguous()
    os.makedirs(os.path.dirname(path), exist_ok=True)
    save_file(t, path)
