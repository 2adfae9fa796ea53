"""NVFP4 weight quantisation and the build's arena tile layout (torch, any device).

Pack format (what a rank pack or a checkpoint slice holds; pack/build_packs.py:9-20
of the reference): per layer
    w13 codes  uint8 [E, 2C, H/2]   gate rows then up rows, two e2m1 per byte,
                                     low nibble = even element
    w13 scales uint8 [E, 2C, H/16]  e4m3 block scale per 16 elements, linear
    g13        f32   [E]             weight_scale_2 (w1 and w3 share it)
    w2 codes   uint8 [E, H, C/2]
    w2 scales  uint8 [E, H, C/16]
    g2         f32   [E]
C = the slice's width, H = 5120.

Arena layout (this build; what the kernels stream), for arena columns [a0, a1),
n_cb = (a1 - a0) / 32 column blocks:
    w13 tiles [E][n_cb][10 K-chunks][18432 B]; one chunk holds the codes and
        block scales of 64 rows (32 gate columns and their 32 up columns) x 512
        elements, ordered so that each thread's tensor-core A fragment is one
        4-byte word (see pack_w13). One (expert, column block) is one contiguous
        184,320-byte run, so any 32-aligned column range streams as whole bulk
        copies.
    w2 tiles  [E][20 row tiles][n_cb x 4096 B codes | n_cb x 512 B scales]; per
        256-row output tile and 32-column block, the same fragment order
        (see pack_w2). A column range is one contiguous run of codes and one of
        scales per (expert, row tile).
Both layouts hold exactly the pack's bytes, only permuted.
"""

from __future__ import annotations

import torch

HIDDEN = 5120
TC = 32
KC = 512
NKC = HIDDEN // KC
TK = 256
NKT = HIDDEN // TK
P1_STAGE = 2 * TC * KC // 2 + 2 * TC * KC // 16   # 18432
P2_CB = TK * 16 + TK * 2                          # 4608

_E2M1_MID = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)


def _e2m1_encode(v: torch.Tensor) -> torch.Tensor:
    mid = torch.tensor(_E2M1_MID, dtype=torch.float32, device=v.device)
    a = torch.clamp(v.abs(), max=6.0)
    i = torch.searchsorted(mid, a.contiguous(), right=False)
    tie = (i < 7) & (a == mid[torch.clamp(i, max=6)]) & ((i & 1) == 1)
    c = torch.where(tie, i + 1, i).to(torch.uint8)
    return torch.where(torch.signbit(v), c | 8, c)


def quantize_nvfp4(w: torch.Tensor, g: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """FP32 [..., K] -> (codes [..., K/2], e4m3 scales [..., K/16]).

    scale = e4m3_rne(amax16 / 6 / g), code = e2m1_rne(w / (scale * g)), saturating.
    """
    blk = w.float().reshape(*w.shape[:-1], w.shape[-1] // 16, 16)
    amax = blk.abs().amax(dim=-1)
    s = torch.clamp(amax / 6.0 / g, max=448.0).to(torch.float8_e4m3fn)
    denom = (s.float() * g).unsqueeze(-1)
    scaled = torch.where(denom > 0, blk / torch.where(denom > 0, denom, torch.ones_like(denom)),
                         torch.zeros_like(blk))
    nib = _e2m1_encode(scaled).reshape(*w.shape[:-1], w.shape[-1] // 2, 2)
    codes = (nib[..., 0] & 0x0F) | ((nib[..., 1] & 0x0F) << 4)
    return codes.to(torch.uint8), s.view(torch.uint8)


def global_scale(w: torch.Tensor) -> torch.Tensor:
    a = w.abs().amax().float()
    return torch.where(a > 0, a / (6.0 * 448.0), torch.ones_like(a))


def pack_w13(c13: torch.Tensor, s13: torch.Tensor, src_a0: int, a0: int, a1: int) -> torch.Tensor:
    """Pack-format w13 (codes [E, 2C, H/2], scales [E, 2C, H/16] of source columns
    [src_a0, src_a0 + C)) -> arena w13 tiles for columns [a0, a1), flat uint8.

    Per (expert, 32-column block, 512-element K chunk) one 18,432-byte stage:
      codes  [tile 4][step group 8][lane 32][step 4][4 B]  (16,384 B)
      scales [tile 4][step group 8][g 8][step 4][2 B]      (2,048 B)
    A tile is 8 gate rows then their 8 up rows (columns tile*8 + g). The 4 code
    bytes of (lane = 4g + t, k16 step) are the m16n8k16 A fragment:
    (gate g, k 2t..2t+1), (up g, k 2t..), (gate g, k 2t+8..), (up g, k 2t+8..);
    the 2 scale bytes are (gate g, up g) of that step's 16-element block.
    """
    e, two_c, _ = c13.shape
    c = two_c // 2
    lo, hi = a0 - src_a0, a1 - src_a0
    if lo < 0 or hi > c or (hi - lo) % TC:
        raise ValueError(f"columns [{a0}, {a1}) not inside the source slice or not 32-aligned")
    n_cb = (hi - lo) // TC
    # codes: [E, cb, tile, g, kc, sg, j, h, t] per gate/up, then bytes (h, hh)
    gc = c13[:, lo:hi].reshape(e, n_cb, 4, 8, NKC, 8, 4, 2, 4)
    uc = c13[:, c + lo:c + hi].reshape(e, n_cb, 4, 8, NKC, 8, 4, 2, 4)
    x = torch.stack([gc, uc], dim=-1)                       # [.., h, t, hh]
    codes = x.permute(0, 1, 4, 2, 5, 3, 8, 6, 7, 9).reshape(e, n_cb, NKC, 16384)
    gs = s13[:, lo:hi].reshape(e, n_cb, 4, 8, NKC, 8, 4)
    us = s13[:, c + lo:c + hi].reshape(e, n_cb, 4, 8, NKC, 8, 4)
    y = torch.stack([gs, us], dim=-1)                       # [E, cb, tile, g, kc, sg, j, hh]
    scales = y.permute(0, 1, 4, 2, 5, 3, 6, 7).reshape(e, n_cb, NKC, 2048)
    return torch.cat([codes, scales], dim=-1).contiguous().view(-1)


def pack_w2(c2: torch.Tensor, s2: torch.Tensor, src_a0: int, a0: int, a1: int) -> torch.Tensor:
    """Pack-format w2 (codes [E, H, C/2], scales [E, H, C/16]) -> arena w2 tiles.

    Per (expert, 256-row output tile kt): codes [cb][tile 16][lane 32][step 2][4 B]
    for every 32-column block, then scales [cb][tile 16][g 8][step 2][2 B]. Tile
    rows are kt*256 + tile*16 + (g | g+8); fragment bytes as in pack_w13 with
    rows g and g+8 in place of gate and up.
    """
    e, h, c_half = c2.shape
    lo, hi = a0 - src_a0, a1 - src_a0
    if lo < 0 or hi > 2 * c_half or (hi - lo) % TC:
        raise ValueError(f"columns [{a0}, {a1}) not inside the source slice or not 32-aligned")
    n_cb = (hi - lo) // TC
    cc = c2[:, :, lo // 2:hi // 2].reshape(e, NKT, 16, 2, 8, n_cb, 2, 2, 4)   # [E, kt, tile, hh, g, cb, s, h, t]
    cc = cc.permute(0, 1, 5, 2, 4, 8, 6, 7, 3).reshape(e, NKT, n_cb * 4096)
    ss = s2[:, :, lo // 16:hi // 16].reshape(e, NKT, 16, 2, 8, n_cb, 2)      # [E, kt, tile, hh, g, cb, s]
    ss = ss.permute(0, 1, 5, 2, 4, 6, 3).reshape(e, NKT, n_cb * 512)
    return torch.cat([cc, ss], dim=-1).contiguous().view(-1)


def unpack_w13(tiles: torch.Tensor, n_experts: int, width: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of pack_w13 (arena -> pack-format codes/scales of the arena's columns)."""
    e, n_cb = n_experts, width // TC
    t = tiles.view(e, n_cb, NKC, P1_STAGE)
    x = t[..., :16384].reshape(e, n_cb, NKC, 4, 8, 8, 4, 4, 2, 2)   # [E, cb, kc, tile, sg, g, t, j, h, hh]
    x = x.permute(0, 1, 3, 5, 2, 4, 7, 8, 6, 9)                      # [E, cb, tile, g, kc, sg, j, h, t, hh]
    gate = x[..., 0].reshape(e, width, HIDDEN // 2)
    up = x[..., 1].reshape(e, width, HIDDEN // 2)
    y = t[..., 16384:].reshape(e, n_cb, NKC, 4, 8, 8, 4, 2)          # [E, cb, kc, tile, sg, g, j, hh]
    y = y.permute(0, 1, 3, 5, 2, 4, 6, 7)                            # [E, cb, tile, g, kc, sg, j, hh]
    gs = y[..., 0].reshape(e, width, HIDDEN // 16)
    us = y[..., 1].reshape(e, width, HIDDEN // 16)
    return torch.cat([gate, up], 1).contiguous(), torch.cat([gs, us], 1).contiguous()


def unpack_w2(tiles: torch.Tensor, n_experts: int, width: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of pack_w2."""
    e, n_cb = n_experts, width // TC
    t = tiles.view(e, NKT, n_cb * P2_CB)
    cc = t[..., :n_cb * 4096].reshape(e, NKT, n_cb, 16, 8, 4, 2, 2, 2)  # [E, kt, cb, tile, g, t, s, h, hh]
    cc = cc.permute(0, 1, 3, 8, 4, 2, 6, 7, 5)                          # [E, kt, tile, hh, g, cb, s, h, t]
    ss = t[..., n_cb * 4096:].reshape(e, NKT, n_cb, 16, 8, 2, 2)        # [E, kt, cb, tile, g, s, hh]
    ss = ss.permute(0, 1, 3, 6, 4, 2, 5)                                # [E, kt, tile, hh, g, cb, s]
    return (cc.reshape(e, HIDDEN, width // 2).contiguous(), ss.reshape(e, HIDDEN, width // 16).contiguous())


def swizzle_offset(row: torch.Tensor, kb: torch.Tensor, kbp: int) -> torch.Tensor:
    """Byte offset of block scale (row, kb) in the vLLM/CUTLASS swizzled scale layout
    the reference arena stores (gx/kernels/fp4_decode_moe_swz.cu:19-21)."""
    return ((row // 128) * (kbp * 128) + (kb // 4) * 512 + (row % 32) * 16
            + ((row % 128) // 32) * 4 + kb % 4)


def unswizzle_scales(swz: torch.Tensor, m: int, kb: int) -> torch.Tensor:
    """Reference-arena scales [..., Mp, KBp] (swizzled) -> linear [..., m, kb]."""
    *lead, mp, kbp = swz.shape
    r = torch.arange(m, device=swz.device).unsqueeze(-1).expand(m, kb)
    c = torch.arange(kb, device=swz.device).unsqueeze(0).expand(m, kb)
    off = swizzle_offset(r, c, kbp).reshape(-1)
    return swz.reshape(*lead, mp * kbp)[..., off].reshape(*lead, m, kb)
