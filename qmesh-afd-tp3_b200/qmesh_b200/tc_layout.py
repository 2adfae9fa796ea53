"""Tensor-core operand layouts of the tcgen05 NVFP4 path (host side).

One MMA consumes a 64-wide K block. For R rows (R % 8 == 0) the block's e2m1
codes are stored K-major without swizzle as [R/8 row groups][2 K halves][8 rows]
[16 bytes] (element 2i in the low nibble of byte i), and its UE4M3 scales (one
per 16 elements) as a 512-byte atom: byte (r % 32) * 16 + (r // 32) * 4 + j is the
scale of elements [16j, 16j + 16) of row r (r < 128); rows 128..255 use a
second atom. This is the arrangement
`tcgen05.cp.32x128b.warpx4` copies into TMEM for the MMA's block scales, and the
same as the vLLM-swizzled scale layout the reference's packs use
(gx/gx_decode_swz.py:108-118) restricted to one 128-row x 4-block atom.
"""

from __future__ import annotations

import torch

KBLK = 64
ROWB = KBLK // 2
SF_ATOM = 512


def pack_operand(nib: torch.Tensor) -> torch.Tensor:
    """e2m1 nibbles uint8 [R, K] -> uint8 [K/64, R*32] tile bytes, one row per K block."""
    r, k = nib.shape
    if r % 8 or k % KBLK:
        raise ValueError(f"operand {r}x{k}: rows must be a multiple of 8 and K of 64")
    t = nib.to(torch.uint8).reshape(r // 8, 8, k // KBLK, 2, 16, 2)
    t = t.permute(2, 0, 3, 1, 4, 5)                   # kb, row group, half, row, byte, nibble
    b = t[..., 0] | (t[..., 1] << 4)
    return b.reshape(k // KBLK, r * ROWB).contiguous()


def unpack_operand(tiles: torch.Tensor, r: int) -> torch.Tensor:
    """Inverse of pack_operand: uint8 [K/64, R*32] -> nibbles [R, K]."""
    kb = tiles.shape[0]
    b = tiles.reshape(kb, r // 8, 2, 8, 16)
    nib = torch.stack([b & 15, b >> 4], dim=-1)      # kb, rg, half, row, byte, nibble
    return nib.permute(1, 3, 0, 2, 4, 5).reshape(r, kb * KBLK).contiguous()


def sf_atoms(r: int) -> int:
    """512-byte scale atoms per K block for r rows (one per 128 rows)."""
    return (r + 127) // 128


def pack_sf(scales: torch.Tensor) -> torch.Tensor:
    """UE4M3 scale bytes [R, K/16] -> uint8 [K/64, 512 * ceil(R/128)]: per K block one
    atom per 128 rows (rows past R zero); atom a holds rows [128a, 128a + 128)."""
    r, kb16 = scales.shape
    if kb16 % 4:
        raise ValueError(f"scales {r}x{kb16}: the block count must be a multiple of 4")
    na = sf_atoms(r)
    s = torch.zeros(na * 128, kb16, dtype=torch.uint8)
    s[:r] = scales.to(torch.uint8)
    s = s.reshape(na, 4, 32, kb16 // 4, 4)            # atom, row/32, row%32, kb, j
    return s.permute(3, 0, 2, 1, 4).reshape(kb16 // 4, na * SF_ATOM).contiguous()


def unpack_sf(atoms: torch.Tensor, r: int) -> torch.Tensor:
    """Inverse of pack_sf: uint8 [K/64, 512 * ceil(R/128)] -> [R, K/16]."""
    kb = atoms.shape[0]
    na = atoms.shape[1] // SF_ATOM
    s = atoms.reshape(kb, na, 32, 4, 4).permute(1, 3, 2, 0, 4).reshape(na * 128, kb * 4)
    return s[:r].contiguous()


def interleave(tiles: torch.Tensor, atoms: torch.Tensor) -> torch.Tensor:
    """[KB, R*32] tiles + [KB, 512] atoms -> flat bytes [KB * (R*32 + 512)], each K
    block's tile followed by its scale atom (the unit one bulk copy stages)."""
    return torch.cat([tiles, atoms], dim=1).reshape(-1).contiguous()


# ---------------------------------------------------------------- arena layout
# For arena columns [a0, a1) (width W, NTA = ceil(W / 64) column tiles; columns
# past a1 are zero rows):
#   w13  [E][NTA][80 K blocks][4608 B]: tile i is rows 0..63 = gate columns
#        a0 + 64i + r, rows 64..127 = their up columns, over K = 5120; each K block
#        is the 4096-byte operand tile then its 512-byte scale atom. A column
#        tile streams as one contiguous 368,640-byte run.
#   w2   [E][40 row tiles][NTA K blocks][4608 B]: row tile j is output rows
#        128j .. 128j + 127 over K = the arena's columns (zero past a1). Any
#        64-aligned column range of one row tile is one contiguous run.

HIDDEN = 5120
KB1 = HIDDEN // KBLK         # 80
HT = HIDDEN // 128           # 40
A_KB = 128 * ROWB + SF_ATOM  # 4608


def tiles_of(width: int) -> int:
    return (width + KBLK - 1) // KBLK


def _operand_from_bytes(rows_bytes: torch.Tensor) -> torch.Tensor:
    """[..., 128, KB*32] code bytes -> [..., KB, 4096] operand tiles."""
    *lead, r, nb = rows_bytes.shape
    kb = nb // ROWB
    t = rows_bytes.reshape(*lead, r // 8, 8, kb, 2, 16)
    n = len(lead)
    perm = list(range(n)) + [n + 2, n, n + 3, n + 1, n + 4]
    return t.permute(*perm).reshape(*lead, kb, r * ROWB)


def _bytes_from_operand(tiles: torch.Tensor, r: int = 128) -> torch.Tensor:
    """Inverse of _operand_from_bytes."""
    *lead, kb, _ = tiles.shape
    t = tiles.reshape(*lead, kb, r // 8, 2, 8, 16)
    n = len(lead)
    perm = list(range(n)) + [n + 1, n + 3, n, n + 2, n + 4]
    return t.permute(*perm).reshape(*lead, r, kb * ROWB)


def _atoms_from_scales(sc: torch.Tensor) -> torch.Tensor:
    """[..., 128, KB*4] scale bytes -> [..., KB, 512] atoms."""
    *lead, r, nb = sc.shape
    kb = nb // 4
    t = sc.reshape(*lead, 4, 32, kb, 4)
    n = len(lead)
    perm = list(range(n)) + [n + 2, n + 1, n, n + 3]
    return t.permute(*perm).reshape(*lead, kb, SF_ATOM)


def _scales_from_atoms(atoms: torch.Tensor) -> torch.Tensor:
    """Inverse of _atoms_from_scales."""
    *lead, kb, _ = atoms.shape
    t = atoms.reshape(*lead, kb, 32, 4, 4)
    n = len(lead)
    perm = list(range(n)) + [n + 2, n + 1, n, n + 3]
    return t.permute(*perm).reshape(*lead, 128, kb * 4)


def _pad_rows(t: torch.Tensor, dim: int, n: int) -> torch.Tensor:
    if t.shape[dim] == n:
        return t
    shape = list(t.shape)
    shape[dim] = n - t.shape[dim]
    return torch.cat([t, torch.zeros(shape, dtype=t.dtype, device=t.device)], dim=dim)


def pack_w13(c13: torch.Tensor, s13: torch.Tensor, src_a0: int, a0: int, a1: int) -> torch.Tensor:
    """Pack-format w13 (codes [E, 2C, H/2], scales [E, 2C, H/16], source columns
    from src_a0) -> tensor-core arena w13 for columns [a0, a1), flat uint8."""
    e, two_c, _ = c13.shape
    c = two_c // 2
    lo, hi = a0 - src_a0, a1 - src_a0
    if lo < 0 or hi > c or (hi - lo) % 32:
        raise ValueError(f"columns [{a0}, {a1}) not inside the source slice or not 32-aligned")
    nta = tiles_of(hi - lo)
    w = nta * KBLK
    gate = _pad_rows(c13[:, lo:hi], 1, w).reshape(e, nta, 64, HIDDEN // 2)
    up = _pad_rows(c13[:, c + lo:c + hi], 1, w).reshape(e, nta, 64, HIDDEN // 2)
    ops = _operand_from_bytes(torch.cat([gate, up], dim=2))                     # [E, NTA, 80, 4096]
    gs = _pad_rows(s13[:, lo:hi], 1, w).reshape(e, nta, 64, HIDDEN // 16)
    us = _pad_rows(s13[:, c + lo:c + hi], 1, w).reshape(e, nta, 64, HIDDEN // 16)
    atoms = _atoms_from_scales(torch.cat([gs, us], dim=2))                      # [E, NTA, 80, 512]
    return torch.cat([ops, atoms], dim=-1).contiguous().view(-1)


def pack_w2(c2: torch.Tensor, s2: torch.Tensor, src_a0: int, a0: int, a1: int) -> torch.Tensor:
    """Pack-format w2 (codes [E, H, C/2], scales [E, H, C/16]) -> tensor-core arena
    w2 for columns [a0, a1), flat uint8."""
    e, h, c_half = c2.shape
    lo, hi = a0 - src_a0, a1 - src_a0
    if lo < 0 or hi > 2 * c_half or (hi - lo) % 32:
        raise ValueError(f"columns [{a0}, {a1}) not inside the source slice or not 32-aligned")
    nta = tiles_of(hi - lo)
    codes = _pad_rows(c2[:, :, lo // 2:hi // 2], 2, nta * ROWB).reshape(e, HT, 128, nta * ROWB)
    scales = _pad_rows(s2[:, :, lo // 16:hi // 16], 2, nta * 4).reshape(e, HT, 128, nta * 4)
    return torch.cat([_operand_from_bytes(codes), _atoms_from_scales(scales)], dim=-1).contiguous().view(-1)


def unpack_w13(flat: torch.Tensor, n_experts: int, width: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of pack_w13 -> (codes [E, 2W, H/2], scales [E, 2W, H/16])."""
    e, nta = n_experts, tiles_of(width)
    t = flat.view(e, nta, KB1, A_KB)
    rows = _bytes_from_operand(t[..., :128 * ROWB])                            # [E, NTA, 128, 2560]
    sc = _scales_from_atoms(t[..., 128 * ROWB:])                               # [E, NTA, 128, 320]
    gate = rows[:, :, :64].reshape(e, nta * 64, -1)[:, :width]
    up = rows[:, :, 64:].reshape(e, nta * 64, -1)[:, :width]
    gs = sc[:, :, :64].reshape(e, nta * 64, -1)[:, :width]
    us = sc[:, :, 64:].reshape(e, nta * 64, -1)[:, :width]
    return torch.cat([gate, up], 1).contiguous(), torch.cat([gs, us], 1).contiguous()


def unpack_w2(flat: torch.Tensor, n_experts: int, width: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of pack_w2 -> (codes [E, H, W/2], scales [E, H, W/16])."""
    e, nta = n_experts, tiles_of(width)
    t = flat.view(e, HT, nta, A_KB)
    codes = _bytes_from_operand(t[..., :128 * ROWB]).reshape(e, HIDDEN, nta * ROWB)[:, :, :width // 2]
    scales = _scales_from_atoms(t[..., 128 * ROWB:]).reshape(e, HIDDEN, nta * 4)[:, :, :width // 16]
    return codes.contiguous(), scales.contiguous()
