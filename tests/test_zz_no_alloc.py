"""qx_slice_decode_static: the decode slice for callers that cannot allocate.

A serving process whose device memory is already claimed by its expert arena
and pools, or a host runtime calling through an FFI with no CUDA allocator,
cannot hand the slice a workspace. This entry point uses a fixed scratch array
inside the library instead. The test calls it through the C ABI twice in a row
with different inputs and checks each result against the workspace-taking
entry point on the same inputs (same kernels, so the outputs are identical),
and that a call larger than the array's limits is refused. It also runs the
largest call the array admits (8 rows, 8 slots, 2304 columns) against the
workspace entry point, and reads a bad-id report back through
qx_slice_decode_static_status, the only way such a caller sees device-side
conditions (it never holds the scratch address).

Kept in a file of its own that pytest collects last; it passes alone in a
fresh process and after the other tests.
"""

import ctypes

import pytest
import torch

import helpers as H

pytestmark = pytest.mark.gpu


def _args(_lib, x, inv, ids, tw, out, c0, c1, ws=None):
    return _lib.QxSliceArgs(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(inv.data_ptr()), x.stride(0), _lib.QX_X_E4M3,
        ctypes.c_void_p(ids.data_ptr()), 0, ctypes.c_void_p(tw.data_ptr()),
        x.shape[0], ids.shape[1], c0, c1, 10.0, 1,
        ctypes.c_void_p(out.data_ptr()), out.stride(0),
        ctypes.c_void_p(ws.data_ptr() if ws is not None else 0), ws.numel() if ws is not None else 0)


def test_static_scratch_entry_matches_workspace_entry(cuda_ready):
    from qmesh_b200 import _lib
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import alloc_workspace
    lib = _lib.load()
    dev = cuda_ready
    layer = H.small_layer(41, 16, inter=512)
    ar = Arena(dev, 1, 16, 0, 512, layout="frag")
    ar.load_layer(0, layer)
    view = ar.view(0)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call, (rows, seed) in enumerate([(6, 51), (3, 52)]):
        ids, tw = H.random_routing(rows, 16, seed)
        _, q, inv = H.activations(rows, seed)
        q, inv, ids, tw = q.to(dev), inv.to(dev), ids.to(dev), tw.to(dev)
        out_static = torch.full((rows, 5120), float("nan"), dtype=torch.bfloat16, device=dev)
        out_ref = torch.empty(rows, 5120, dtype=torch.bfloat16, device=dev)
        a = _args(_lib, q, inv, ids, tw, out_static, 0, 512)
        assert lib.qx_slice_decode_static(ctypes.byref(view), ctypes.byref(a), stream) == _lib.QX_OK
        ws = alloc_workspace(rows, 6, 0, 512, dev, "frag")
        b = _args(_lib, q, inv, ids, tw, out_ref, 0, 512, ws)
        assert lib.qx_slice_decode(ctypes.byref(view), ctypes.byref(b), stream) == _lib.QX_OK
        torch.cuda.synchronize()
        assert torch.equal(out_static, out_ref), f"call {call}"
        H.assert_parity(out_static, H.oracle_out(H.ingest(q.cpu(), inv.cpu()), ids.cpu(), tw.cpu(), layer, 0, 512),
                         f"static call {call}")


def test_static_scratch_entry_at_its_largest_call(cuda_ready):
    """rows = QX_STATIC_MAX_ROWS, topk = QX_STATIC_MAX_TOPK, width = QX_STATIC_MAX_WIDTH:
    the regions at the end of the array are in use; the result equals the
    workspace entry point's, on two calls in a row."""
    from qmesh_b200 import _lib
    from qmesh_b200.arena import Arena
    from qmesh_b200.expert_slice import alloc_workspace
    lib = _lib.load()
    dev = cuda_ready
    rows, topk, width = _lib.STATIC_MAX_ROWS, _lib.STATIC_MAX_TOPK, _lib.STATIC_MAX_WIDTH
    ar = Arena(dev, 1, 24, 0, width, layout="frag")
    ar.fill_synthetic(0, seed=43)
    view = ar.view(0)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ws = alloc_workspace(rows, topk, 0, width, dev, "frag")
    for call, seed in enumerate((61, 62)):
        ids, tw = H.random_routing(rows, 24, seed, topk=topk)
        _, q, inv = H.activations(rows, seed)
        q, inv, ids, tw = q.to(dev), inv.to(dev), ids.to(dev), tw.to(dev)
        out_static = torch.full((rows, 5120), float("nan"), dtype=torch.bfloat16, device=dev)
        out_ref = torch.empty(rows, 5120, dtype=torch.bfloat16, device=dev)
        a = _args(_lib, q, inv, ids, tw, out_static, 0, width)
        assert lib.qx_slice_decode_static(ctypes.byref(view), ctypes.byref(a), stream) == _lib.QX_OK
        st = ctypes.c_uint32(99)
        assert lib.qx_slice_decode_static_status(ctypes.byref(st), stream) == _lib.QX_OK
        assert st.value == 0, f"call {call}: device status {st.value}"
        b = _args(_lib, q, inv, ids, tw, out_ref, 0, width, ws)
        assert lib.qx_slice_decode(ctypes.byref(view), ctypes.byref(b), stream) == _lib.QX_OK
        torch.cuda.synchronize()
        assert torch.equal(out_static, out_ref), f"call {call}"
        assert torch.isfinite(out_static.float()).all()


def test_static_scratch_entry_reports_bad_ids(cuda_ready):
    """An id outside [0, E) is skipped and reported as QX_DEV_BAD_ID in the
    array's status word; the next clean call clears it."""
    from qmesh_b200 import _lib
    from qmesh_b200.arena import Arena
    lib = _lib.load()
    dev = cuda_ready
    layer = H.small_layer(44, 8, inter=256)
    ar = Arena(dev, 1, 8, 0, 256, layout="frag")
    ar.load_layer(0, layer)
    view = ar.view(0)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rows = 2
    ids, tw = H.random_routing(rows, 8, 7)
    _, q, inv = H.activations(rows, 7)
    bad = ids.clone()
    bad[1, 2] = 8                        # one past the last expert
    q, inv, tw = q.to(dev), inv.to(dev), tw.to(dev)
    out = torch.empty(rows, 5120, dtype=torch.bfloat16, device=dev)
    for id_tensor, want in ((bad, _lib.QX_DEV_BAD_ID), (ids, 0)):
        d_ids = id_tensor.to(dev)
        a = _args(_lib, q, inv, d_ids, tw, out, 0, 256)
        assert lib.qx_slice_decode_static(ctypes.byref(view), ctypes.byref(a), stream) == _lib.QX_OK
        st = ctypes.c_uint32(0)
        assert lib.qx_slice_decode_static_status(ctypes.byref(st), stream) == _lib.QX_OK
        assert st.value == want


def test_static_scratch_entry_refuses_calls_beyond_its_limits(cuda_ready):
    from qmesh_b200 import _lib
    from qmesh_b200.arena import Arena
    lib = _lib.load()
    dev = cuda_ready
    layer = H.small_layer(42, 8, inter=256)
    ar = Arena(dev, 1, 8, 0, 256, layout="frag")
    ar.load_layer(0, layer)
    view = ar.view(0)
    rows = _lib.STATIC_MAX_ROWS + 1
    ids, tw = H.random_routing(rows, 8, 5)
    _, q, inv = H.activations(rows, 5)
    q, inv, ids, tw = q.to(dev), inv.to(dev), ids.to(dev), tw.to(dev)
    out = torch.empty(rows, 5120, dtype=torch.bfloat16, device=dev)
    a = _args(_lib, q, inv, ids, tw, out, 0, 256)
    rc = lib.qx_slice_decode_static(ctypes.byref(view), ctypes.byref(a), None)
    assert rc == _lib.QX_ERR_SHAPE
    # one slot too many, and one 32-column step too wide (on an arena that has the columns)
    rows = 2
    ids, tw = H.random_routing(rows, 8, 6)
    _, q, inv = H.activations(rows, 6)
    q, inv, ids, tw = q.to(dev), inv.to(dev), ids.to(dev), tw.to(dev)
    wide_ids = torch.zeros(rows, _lib.STATIC_MAX_TOPK + 1, dtype=torch.int32, device=dev)
    wide_tw = torch.zeros(rows, _lib.STATIC_MAX_TOPK + 1, dtype=torch.float32, device=dev)
    out = torch.empty(rows, 5120, dtype=torch.bfloat16, device=dev)
    a = _args(_lib, q, inv, wide_ids, wide_tw, out, 0, 256)
    assert lib.qx_slice_decode_static(ctypes.byref(view), ctypes.byref(a), None) == _lib.QX_ERR_SHAPE
    wide = _lib.QxArena(view.w13, view.w2, view.g13, view.g2, 8, 0, _lib.STATIC_MAX_WIDTH + 32, _lib.QX_LAYOUT_FRAG)
    a = _args(_lib, q, inv, ids, tw, out, 0, _lib.STATIC_MAX_WIDTH + 32)
    assert lib.qx_slice_decode_static(ctypes.byref(wide), ctypes.byref(a), None) == _lib.QX_ERR_SHAPE
