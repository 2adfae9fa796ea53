"""Properties of the CPU model of the tensor-core path's activation terms
(tests/nvfp4_terms.py): the bounds the kernel's numerics rest on."""

import torch

import nvfp4_terms as NT


def _rows(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    v = torch.randn(n, k, generator=g) * torch.exp(torch.randn(n, 1, generator=g) * 4)
    v[0] = 0.0                                                     # an all-zero row
    v[1, :64] = 0.0                                                # a zero tile
    v[2] *= 2.0 ** -80                                             # tiny magnitudes
    v[3, 5] = 6.0                                                  # a value on the e2m1 grid top
    return v.to(torch.float32)


def test_x_terms_bound_and_exponent():
    v = _rows(8, 512, 1)
    codes, e = NT.decompose_x(v)
    amax = v.abs().amax(dim=1).double()
    assert (6.0 * torch.pow(2.0, e.double()) >= amax).all()
    nz = amax > 0
    assert (6.0 * torch.pow(2.0, e.double() - 1)[nz] < amax[nz]).all()   # smallest such E
    assert int(e[0]) == 0
    err = (NT.reconstruct_x(codes, e) - v.double()).abs()
    assert (err <= torch.pow(2.0, e.double() - 30).view(-1, 1)).all()


def test_act_terms_common_exponent_and_bound():
    v = _rows(8, 2304, 2)
    codes, e, eloc = NT.decompose_act(v)
    assert (eloc % 2 == 0).all() and (e % 2 == 0).all()
    assert torch.equal(e, eloc.max(dim=1).values)
    assert int(e[0]) == NT.AE_MIN and int(eloc[1, 0]) == NT.AE_MIN
    err = (NT.reconstruct_x(codes, e) - v.double()).abs()
    assert (err <= torch.pow(2.0, e.double() - 30).view(-1, 1)).all()
    assert (codes[0] == 0).all() and (codes[1, :, :64] == 0).all()


def test_act_shift_moves_whole_terms():
    """A tile below the pair's maximum keeps its own digits, moved down by
    d = (E - E_loc) / 2 terms, with the first d terms zero."""
    v = torch.zeros(1, 128)
    v[0, :64] = torch.linspace(-3.0, 5.0, 64)
    v[0, 64:] = torch.linspace(-1.0, 1.0, 64) * 2.0 ** -9
    codes, e, eloc = NT.decompose_act(v.to(torch.float32))
    d = int(e[0] - eloc[0, 1]) // 2
    assert d >= 4
    local = NT._digits(v[:, 64:].to(torch.float32), eloc[:, 1], 16)
    assert (codes[0, :d, 64:] == 0).all()
    assert torch.equal(codes[0, d:, 64:], local[0, :16 - d])
