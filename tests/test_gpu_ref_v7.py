"""Pin the oracle to the reference's own v7 CUDA kernel, run on the GPU.

oracle/_ref/libref_v7.so is the reference kernel (gx/kernels/fp4_decode_moe_swz.cu)
compiled unmodified by oracle/ref_v7/build.py. Its inputs are laid out exactly as
the reference arena holds them (gx/gx_expert_worker.py:178-227): gate rows
[0, C), 32*k zero rows, up rows [CP, CP+C); w2 columns padded C -> CP; block
scales padded and then swizzled per expert (the vLLM layout pinned in
test_oracle_pins). Three checks per case: reference kernel vs oracle, this
build's kernel vs oracle, and this build's kernel vs the reference kernel.
"""

import ctypes

import pytest
import torch

import helpers as H
from conftest import ROOT
from oracle import nvfp4 as oq

pytestmark = pytest.mark.gpu

REF = ROOT / "oracle" / "_ref" / "libref_v7.so"
CPS = {864: 896, 576: 640, 288: 384}


@pytest.fixture(scope="module")
def ref_lib(cuda_ready):
    if not REF.is_file():
        pytest.fail(f"{REF} missing: run oracle/ref_v7/build.py where the reference tree exists")
    lib = ctypes.CDLL(str(REF))
    for c in CPS:
        fn = getattr(lib, f"ref_v7_decode_{c}")
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.c_void_p] * 11 + [ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    return lib


@pytest.fixture(scope="module")
def layer():
    return H.small_layer(31, 8, inter=1152)


def ref_arena(layer, c0, c, cp, dev):
    e = layer["c13"].shape[0]
    inter = layer["c13"].shape[1] // 2
    w13 = torch.zeros(e, 2 * cp, 2560, dtype=torch.uint8)
    s13 = torch.zeros(e, 2 * cp, 320, dtype=torch.uint8)
    w13[:, :c] = layer["c13"][:, c0:c0 + c]
    w13[:, cp:cp + c] = layer["c13"][:, inter + c0:inter + c0 + c]
    s13[:, :c] = layer["s13"][:, c0:c0 + c]
    s13[:, cp:cp + c] = layer["s13"][:, inter + c0:inter + c0 + c]
    w2 = torch.zeros(e, 5120, cp // 2, dtype=torch.uint8)
    s2 = torch.zeros(e, 5120, cp // 16, dtype=torch.uint8)
    w2[:, :, :c // 2] = layer["c2"][:, :, c0 // 2:(c0 + c) // 2]
    s2[:, :, :c // 16] = layer["s2"][:, :, c0 // 16:(c0 + c) // 16]
    return dict(w13=w13.to(dev), s13=oq.swizzle_scales(s13).to(dev), w2=w2.to(dev),
                s2=oq.swizzle_scales(s2).to(dev), g13=layer["g13"].float().to(dev), g2=layer["g2"].float().to(dev))


@pytest.mark.parametrize("c", [864, 576, 288])
@pytest.mark.parametrize("rows", [1, 6, 16])
def test_reference_kernel_pins_oracle(ref_lib, layer, cuda_ready, c, rows):
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import expert_slice
    dev = cuda_ready
    cp = CPS[c]
    c0 = 288 if c < 864 else 0
    ra = ref_arena(layer, c0, c, cp, dev)
    ids, tw = H.random_routing(rows, 8, 100 + rows + c)
    _, q, inv = H.activations(rows, 100 + rows)
    x = H.ingest(q, inv)
    xb = x.to(torch.bfloat16).to(dev)
    act = torch.zeros(rows * 6 * c, dtype=torch.float32, device=dev)
    out_ref = torch.zeros(rows, 5120, dtype=torch.bfloat16, device=dev)
    idd, twd = ids.to(dev), tw.to(dev)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = getattr(ref_lib, f"ref_v7_decode_{c}")(
        P(xb), P(idd), P(twd), P(ra["w13"]), P(ra["s13"]), P(ra["g13"]), P(ra["w2"]), P(ra["s2"]), P(ra["g2"]),
        P(act), P(out_ref), rows, 10.0, 1, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    oracle = H.oracle_out(x, ids, tw, layer, c0, c0 + c)
    p_ref = H.assert_parity(out_ref, oracle, "reference v7 vs oracle")
    ar = Arena(dev, 1, 8, c0, c0 + c)
    ar.load_layer(0, layer)
    ours = expert_slice(ar, 0, q.to(dev), idd, twd, x_scale=inv.to(dev))
    torch.cuda.synchronize()
    p_ours = H.assert_parity(ours, oracle, "qmesh_b200 vs oracle")
    p_x = H.assert_parity(ours, out_ref, "qmesh_b200 vs reference v7")
    print(f"C={c} rows={rows} ref-vs-oracle {p_ref} ours-vs-ref {p_x}")
