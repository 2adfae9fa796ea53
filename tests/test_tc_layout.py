"""Tensor-core operand layout (qmesh_b200.tc_layout) on the CPU: round trips and
the byte addresses the kernels compute (qx_tc.cuh opnd_off / sf_off)."""

import torch

from qmesh_b200 import tc_layout as L


def opnd_off(row, k):
    return (row >> 3) * 256 + (k >> 5) * 128 + (row & 7) * 16 + ((k & 31) >> 1)


def sf_off(row, j):
    return (row & 31) * 16 + (row >> 5) * 4 + j


def test_operand_round_trip_and_addresses():
    g = torch.Generator().manual_seed(0)
    nib = torch.randint(0, 16, (48, 192), generator=g, dtype=torch.uint8)
    tiles = L.pack_operand(nib)
    assert tiles.shape == (3, 48 * 32)
    assert torch.equal(L.unpack_operand(tiles, 48), nib)
    for row, k in [(0, 0), (0, 1), (7, 31), (8, 32), (47, 191), (13, 100), (40, 64)]:
        kb, kk = divmod(k, 64)
        byte = int(tiles[kb, opnd_off(row, kk)])
        assert (byte >> (4 * (kk & 1))) & 15 == int(nib[row, k])


def test_scale_atoms_round_trip_and_addresses():
    g = torch.Generator().manual_seed(1)
    sc = torch.randint(0, 127, (100, 12), generator=g, dtype=torch.uint8)
    atoms = L.pack_sf(sc)
    assert atoms.shape == (3, 512)
    assert torch.equal(L.unpack_sf(atoms, 100), sc)
    for row, b in [(0, 0), (31, 3), (32, 4), (99, 11), (64, 7)]:
        kb, j = divmod(b, 4)
        assert int(atoms[kb, sf_off(row, j)]) == int(sc[row, b])
    # rows beyond R are zero in the atom
    assert int(atoms[0, sf_off(120, 0)]) == 0


def test_interleave_order():
    t = torch.arange(2 * 256, dtype=torch.int64).to(torch.uint8).reshape(2, 256)
    a = torch.full((2, 512), 7, dtype=torch.uint8)
    flat = L.interleave(t, a)
    assert flat.numel() == 2 * (256 + 512)
    assert torch.equal(flat[:256], t[0]) and torch.equal(flat[256:768], a[0]) and torch.equal(flat[768:1024], t[1])


def test_scale_atoms_beyond_128_rows():
    g = torch.Generator().manual_seed(2)
    sc = torch.randint(0, 127, (200, 8), generator=g, dtype=torch.uint8)
    atoms = L.pack_sf(sc)
    assert atoms.shape == (2, 1024)
    assert torch.equal(L.unpack_sf(atoms, 200), sc)
    for row, b in [(130, 1), (199, 7), (127, 4)]:
        kb, j = divmod(b, 4)
        assert int(atoms[kb, (row // 128) * 512 + sf_off(row % 128, j)]) == int(sc[row, b])
