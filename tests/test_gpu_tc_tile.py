"""The block-scaled NVFP4 tensor-core path (tcgen05.mma.kind::mxf4nvf4) against a
float64 CPU product, through qx_diag_nvf4_tile: operand tile layout, nibble
order, scale atoms in TMEM, instruction and shared-memory descriptors and the
accumulator read-back, for several N and K-block counts."""

import ctypes

import pytest
import torch

from oracle import nvfp4 as q4

pytestmark = pytest.mark.gpu


def _operands(n, nkb, seed, sparse=None):
    from qmesh_b200 import tc_layout as L
    g = torch.Generator().manual_seed(seed)
    k = nkb * 64
    an = torch.randint(0, 16, (128, k), generator=g, dtype=torch.uint8)
    bn = torch.randint(0, 16, (n, k), generator=g, dtype=torch.uint8)
    # e4m3 scale bytes 0x28..0x47 (0.25 .. 3.75)
    asf = torch.randint(0x28, 0x48, (128, k // 16), generator=g, dtype=torch.uint8)
    bsf = torch.randint(0x28, 0x48, (n, k // 16), generator=g, dtype=torch.uint8)
    if sparse is not None:
        an, bn, asf, bsf = sparse(an, bn, asf, bsf)
    a = L.interleave(L.pack_operand(an), L.pack_sf(asf))
    b = L.interleave(L.pack_operand(bn), L.pack_sf(bsf))
    ad = q4.e2m1_decode(an).double() * q4.e4m3_decode(asf).double().repeat_interleave(16, 1)
    bd = q4.e2m1_decode(bn).double() * q4.e4m3_decode(bsf).double().repeat_interleave(16, 1)
    return a, b, ad, bd


def _run(a, b, n, nkb, dev):
    from qmesh_b200 import _lib
    lib = _lib.load()
    a_d, b_d = a.to(dev), b.to(dev)
    d = torch.full((128, n), float("nan"), dtype=torch.float32, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = lib.qx_diag_nvf4_tile(a_d.data_ptr(), b_d.data_ptr(), n, nkb, d.data_ptr(), st.data_ptr(),
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.QX_OK
    torch.cuda.synchronize()
    assert int(st.item()) == 0, f"device status {int(st.item())}"
    return d.cpu().double()


@pytest.mark.parametrize("n,nkb", [(16, 1), (48, 3), (128, 2), (256, 8), (96, 5), (144, 2)])
def test_nvf4_tile_matches_cpu_product(cuda_ready, n, nkb):
    a, b, ad, bd = _operands(n, nkb, seed=n * 10 + nkb)
    d = _run(a, b, n, nkb, cuda_ready)
    ref = ad @ bd.T
    bound = (ad.abs() @ bd.abs().T) * 2.0 ** -20 + 1e-30
    err = (d - ref).abs()
    assert torch.isfinite(d).all()
    worst = (err / bound).max().item()
    assert worst <= 1.0, f"max err {err.max().item()} (x{worst:.2f} of the fp32 bound) at {divmod(int((err / bound).argmax()), n)}"


def test_nvf4_tile_single_elements(cuda_ready):
    """One non-zero element in A and B at a time: pins where each (row, k) and
    each scale lands (a layout mistake shows up as the wrong output cell)."""
    n, nkb = 32, 2
    cases = [(0, 0, 0), (5, 1, 3), (37, 33, 17), (100, 64, 31), (127, 127, 8), (70, 90, 20)]
    for (m, k, nn) in cases:
        def sparse(an, bn, asf, bsf, m=m, k=k, nn=nn):
            an = torch.zeros_like(an)
            bn = torch.zeros_like(bn)
            an[m, k] = 2          # 1.0
            bn[nn, k] = 5         # 3.0
            asf = torch.full_like(asf, 0x38)   # 1.0
            bsf = torch.full_like(bsf, 0x38)
            asf[m, k // 16] = 0x40             # 2.0
            bsf[nn, k // 16] = 0x30            # 0.5
            return an, bn, asf, bsf
        a, b, ad, bd = _operands(n, nkb, seed=0, sparse=sparse)
        d = _run(a, b, n, nkb, cuda_ready)
        nz = (d != 0).nonzero().tolist()
        assert nz == [[m, nn]] and d[m, nn].item() == 3.0, f"element (m={m}, k={k}, n={nn}): non-zeros {nz[:8]}"
