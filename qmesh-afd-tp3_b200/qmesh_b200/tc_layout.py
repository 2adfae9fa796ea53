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
