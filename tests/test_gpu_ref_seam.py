"""The producer quantiser and the ordered combine against the reference's own
seam kernels, run on the same GPU.

oracle/_ref/libref_seam.so is native/qmesh_afd_seam.cu compiled unmodified
(oracle/ref_seam/build.py): seam_amax_kernel with the folded seam_finish, then
seam_pack_kernel (the post quantiser, native/qmesh_afd_seam.cu:88-176), and
seam_combine_kernel / seam_combine_vec_kernel (:310-484). This build's
qx_quant_fp8 in per-post mode and qx_combine_ordered must give the same bytes;
the CPU restatement in oracle/nvfp4.py (fp8_quant_post) is checked against the
reference kernels as well, so the oracle the other tests use is pinned to what
the reference computes.
"""

import ctypes
from pathlib import Path

import pytest
import torch

from oracle import nvfp4 as oq

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libref_seam.so"


@pytest.fixture(scope="module")
def ref(cuda_ready):
    if not LIB.is_file():
        pytest.fail(f"{LIB} is not built (oracle/ref_seam/build.py)")
    lib = ctypes.CDLL(str(LIB))
    lib.ref_seam_status_bytes.restype = ctypes.c_size_t
    lib.ref_seam_quant_post.restype = ctypes.c_int
    lib.ref_seam_quant_post.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.ref_seam_combine.restype = ctypes.c_int
    lib.ref_seam_combine.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p),
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    return lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _rows(rows, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, 5120, generator=g) * torch.exp(torch.randn(rows, 1, generator=g) * 3)
    x[0, :7] = torch.tensor([448.0, -1e-30, 0.0, -0.0, 3.0e5, 1e-7, -2.5])
    if rows > 2:
        x[2] = 0.0
    return x.to(torch.bfloat16)


def _ref_quant(ref, x, fill=0):
    dev = x.device
    rows = x.shape[0]
    q = torch.full((rows, 5120), fill, dtype=torch.uint8, device=dev)
    scale = torch.zeros(2, dtype=torch.float32, device=dev)
    work = torch.zeros(2, dtype=torch.int32, device=dev)
    status = torch.zeros(int(ref.ref_seam_status_bytes()), dtype=torch.uint8, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert ref.ref_seam_quant_post(_p(x), x.stride(0), rows, _p(q), _p(scale), _p(work), _p(status), stream) == 0
    torch.cuda.synchronize()
    return q, scale, status


@pytest.mark.parametrize("rows,seed", [(1, 11), (6, 12), (48, 13), (128, 14)])
def test_post_quantiser_equals_reference_kernels(cuda_ready, ref, rows, seed):
    from qmesh_b200.front import quant_fp8
    x = _rows(rows, seed).to(cuda_ready)
    rq, rscale, _ = _ref_quant(ref, x)
    q, inv = quant_fp8(x, per_post=True)
    torch.cuda.synchronize()
    assert torch.equal(q, rq), f"e4m3 bytes differ in {(q != rq).sum().item()} places"
    assert torch.equal(inv.cpu().view(torch.int32), rscale[1:].cpu().view(torch.int32))
    # the CPU restatement the other tests use, pinned to the same kernels
    wq, winv = oq.fp8_quant_post(x.float().cpu())
    assert torch.equal(wq, rq.cpu()) and torch.equal(winv.view(torch.int32), rscale[1:].cpu().view(torch.int32))


def test_post_quantiser_nonfinite_equals_reference(cuda_ready, ref):
    """A non-finite maximum: the reference skips the payload and posts inv = 1;
    qx_quant_fp8 leaves the bytes and reports QX_DEV_NONFINITE."""
    from qmesh_b200.front import quant_fp8
    dev = cuda_ready
    x = _rows(6, 15)
    x[3, 77] = float("inf")
    x = x.to(dev)
    rq, rscale, rstatus = _ref_quant(ref, x, fill=0x5A)
    q = torch.full((6, 5120), 0x5A, dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    q, inv = quant_fp8(x, per_post=True, q=q, status=status)
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and (q == 0x5A).all()
    assert float(rscale[1]) == 1.0 and float(inv[0]) == 1.0
    assert int(status.item()) == 8
    assert int(rstatus[:8].view(torch.int64).item()) == 1    # SeamStatus.nonfinite


@pytest.mark.parametrize("np_,rows,vec", [(1, 1, 0), (3, 6, 1), (4, 6, 0), (4, 48, 1), (2, 300, 1)])
def test_ordered_combine_equals_reference_kernels(cuda_ready, ref, np_, rows, vec):
    """out = bf16(local + p0 + ... + p_{np-1}) in FP32, peers ascending: the
    reference's in-place seam combine against qx_combine_ordered([local, p0, ...])."""
    from qmesh_b200.combine import combine_ordered
    dev = cuda_ready
    g = torch.Generator().manual_seed(100 + np_ * 7 + rows)
    scales = torch.exp(torch.randn(np_ + 1, 1, 1, generator=g) * 2)
    parts = (torch.randn(np_ + 1, rows, 5120, generator=g) * scales).to(torch.bfloat16).to(dev)
    local = parts[0].clone()
    peers = [parts[i + 1].contiguous() for i in range(np_)]
    arr = (ctypes.c_void_p * 4)(*[p.data_ptr() for p in peers], *([0] * (4 - np_)))
    status = torch.zeros(int(ref.ref_seam_status_bytes()), dtype=torch.uint8, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert ref.ref_seam_combine(_p(local), local.stride(0), arr, np_, rows, vec, _p(status), stream) == 0
    ours = combine_ordered([parts[0]] + peers)
    torch.cuda.synchronize()
    assert torch.equal(ours, local), f"{(ours != local).sum().item()} elements differ"
