"""Device-resident NVFP4 expert arena (the build's counterpart of the reference's
gx/gx_expert_worker.py:143-314 ``Arena``).

One Arena holds intermediate columns [a0, a1) of every routed expert of some MoE
layers on one GPU, in the tile layout its slice kernel streams: "tc" for the
tensor-core kernel (qmesh_b200.tc_layout), "frag" for the register-dequant
kernel (qmesh_b200.nvfp4). Weights come either from pack-format tensors (a rank
pack or a checkpoint slice) or from a seeded synthetic draw made on the device.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from . import nvfp4 as q4
from . import tc_layout as tl

HIDDEN = q4.HIDDEN
INTER = 2304
TOPK = 6


LAYOUTS = ("tc", "frag")


class Arena:
    def __init__(self, device, layers: int, n_experts: int, a0: int = 0, a1: int = INTER, layout: str = "tc"):
        if (a1 - a0) <= 0 or a0 % q4.TC or a1 % q4.TC:
            raise ValueError(f"arena columns [{a0}, {a1}) must be 32-aligned and non-empty")
        if layout not in LAYOUTS:
            raise ValueError(f"layout must be one of {LAYOUTS}, got {layout!r}")
        self.layout = layout
        self.dev = torch.device(device)
        self.layers = layers
        self.n_experts = n_experts
        self.a0, self.a1 = a0, a1
        self.width = a1 - a0
        self.w13: list[torch.Tensor | None] = [None] * layers
        self.w2: list[torch.Tensor | None] = [None] * layers
        self.g13: list[torch.Tensor | None] = [None] * layers
        self.g2: list[torch.Tensor | None] = [None] * layers

    # -- size accounting (gx_expert_worker.py:156-165 counterpart) ---------------
    def bytes_per_layer(self) -> int:
        lib = _lib.load()
        if self.layout == "tc":
            return (lib.qx_arena_tc_w13_bytes(self.n_experts, self.width)
                    + lib.qx_arena_tc_w2_bytes(self.n_experts, self.width) + 8 * self.n_experts)
        return (lib.qx_arena_w13_bytes(self.n_experts, self.width)
                + lib.qx_arena_w2_bytes(self.n_experts, self.width) + 8 * self.n_experts)

    @staticmethod
    def layer_bytes(n_experts: int, width: int, layout: str = "tc") -> int:
        if layout == "tc":
            nta = tl.tiles_of(width)
            return n_experts * nta * (tl.KB1 + tl.HT) * tl.A_KB + 8 * n_experts
        n_cb = width // q4.TC
        return n_experts * n_cb * (q4.NKC * q4.P1_STAGE + q4.NKT * q4.P2_CB) + 8 * n_experts

    def _pack(self, c13, s13, c2, s2, src_a0: int):
        mod = tl if self.layout == "tc" else q4
        return mod.pack_w13(c13, s13, src_a0, self.a0, self.a1), mod.pack_w2(c2, s2, src_a0, self.a0, self.a1)

    def _per_expert(self) -> tuple[int, int]:
        if self.layout == "tc":
            nta = tl.tiles_of(self.width)
            return nta * tl.KB1 * tl.A_KB, tl.HT * nta * tl.A_KB
        n_cb = self.width // q4.TC
        return n_cb * q4.NKC * q4.P1_STAGE, q4.NKT * n_cb * q4.P2_CB

    def check_memory(self, layers: int | None = None) -> None:
        """Refuse to fill more than the device has free (gx_expert_worker.py:229-240)."""
        need = (layers or self.layers) * self.layer_bytes(self.n_experts, self.width, self.layout)
        free, _ = torch.cuda.mem_get_info(self.dev)
        if need > free:
            raise MemoryError(f"arena needs {need / 2**30:.1f} GiB, device has {free / 2**30:.1f} GiB free")

    # -- loading ----------------------------------------------------------------
    def load_layer(self, li: int, pack: dict, src_a0: int = 0) -> None:
        """Pack-format tensors (c13, s13, g13, c2, s2, g2; columns from src_a0) -> arena."""
        d = self.dev
        c13 = pack["c13"].to(d)
        s13 = pack["s13"].to(d)
        c2 = pack["c2"].to(d)
        s2 = pack["s2"].to(d)
        if c13.shape[0] != self.n_experts:
            raise ValueError(f"pack has {c13.shape[0]} experts, arena {self.n_experts}")
        self.w13[li], self.w2[li] = self._pack(c13, s13, c2, s2, src_a0)
        g13 = torch.as_tensor(pack["g13"], dtype=torch.float32).reshape(self.n_experts, -1)[:, 0]
        self.g13[li] = g13.contiguous().to(d)
        self.g2[li] = torch.as_tensor(pack["g2"], dtype=torch.float32).reshape(-1).contiguous().to(d)

    def fill_synthetic(self, li: int, seed: int, std: float = 0.02, chunk: int = 8) -> None:
        """Seeded FP32 N(0, std) experts (full 2304 columns) quantised to NVFP4 on the
        device, then sliced to the arena's columns. Deterministic per (seed, layer,
        expert chunk), so arenas of different column ranges hold slices of the same
        experts."""
        d = self.dev
        e_all = self.n_experts
        per13, per2 = self._per_expert()
        w13 = torch.empty(e_all * per13, dtype=torch.uint8, device=d)
        w2 = torch.empty(e_all * per2, dtype=torch.uint8, device=d)
        g13 = torch.empty(e_all, dtype=torch.float32, device=d)
        g2 = torch.empty(e_all, dtype=torch.float32, device=d)
        for e0 in range(0, e_all, chunk):
            e1 = min(e_all, e0 + chunk)
            n = e1 - e0
            gen = torch.Generator(device=d)
            gen.manual_seed((seed * 1000003 + li * 10007 + e0) & 0x7FFFFFFFFFFF)
            w13f = torch.randn(n, 2 * INTER, HIDDEN, generator=gen, device=d) * std
            w2f = torch.randn(n, HIDDEN, INTER, generator=gen, device=d) * std
            a13 = w13f.abs().amax(dim=(1, 2))
            a2 = w2f.abs().amax(dim=(1, 2))
            gg13 = torch.where(a13 > 0, a13 / (6.0 * 448.0), torch.ones_like(a13))
            gg2 = torch.where(a2 > 0, a2 / (6.0 * 448.0), torch.ones_like(a2))
            c13, s13 = q4.quantize_nvfp4(w13f, gg13.view(n, 1, 1))
            del w13f
            c2, s2 = q4.quantize_nvfp4(w2f, gg2.view(n, 1, 1))
            del w2f
            w13[e0 * per13:e1 * per13], w2[e0 * per2:e1 * per2] = self._pack(c13, s13, c2, s2, 0)
            g13[e0:e1] = gg13
            g2[e0:e1] = gg2
            del c13, s13, c2, s2
        self.w13[li], self.w2[li], self.g13[li], self.g2[li] = w13, w2, g13, g2

    def expert_pack(self, li: int, experts: list[int]) -> dict:
        """Pack-format CPU tensors of some experts over the arena's columns (for checks)."""
        per13, per2 = self._per_expert()
        mod = tl if self.layout == "tc" else q4
        out = {"c13": [], "s13": [], "c2": [], "s2": []}
        for e in experts:
            c13, s13 = mod.unpack_w13(self.w13[li][e * per13:(e + 1) * per13].cpu(), 1, self.width)
            c2, s2 = mod.unpack_w2(self.w2[li][e * per2:(e + 1) * per2].cpu(), 1, self.width)
            out["c13"].append(c13[0]); out["s13"].append(s13[0])
            out["c2"].append(c2[0]); out["s2"].append(s2[0])
        res = {k: torch.stack(v) for k, v in out.items()}
        res["g13"] = self.g13[li][experts].cpu()
        res["g2"] = self.g2[li][experts].cpu()
        return res

    # -- C view ------------------------------------------------------------------
    def loaded(self, li: int) -> bool:
        return 0 <= li < self.layers and self.w13[li] is not None and self.w2[li] is not None

    def view(self, li: int) -> _lib.QxArena:
        if not self.loaded(li):
            raise RuntimeError(f"layer {li} is not loaded in the arena")
        return _lib.QxArena(
            ctypes.c_void_p(self.w13[li].data_ptr()), ctypes.c_void_p(self.w2[li].data_ptr()),
            ctypes.c_void_p(self.g13[li].data_ptr()), ctypes.c_void_p(self.g2[li].data_ptr()),
            self.n_experts, self.a0, self.a1, _lib.QX_LAYOUT_TC if self.layout == "tc" else _lib.QX_LAYOUT_FRAG)
