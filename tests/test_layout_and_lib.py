"""Host logic: arena tile packing, the product quantiser, and the C-ABI library
(loads, exports every declared symbol, validates arguments) -- no GPU needed."""

import ctypes
import re

import pytest
import torch

from conftest import ROOT
from oracle import moe, nvfp4 as oq


@pytest.fixture(scope="module")
def lib():
    from qmesh_b200 import _lib, build
    build.build()
    return _lib.load()


def test_product_quantizer_matches_oracle():
    from qmesh_b200 import nvfp4 as q4
    g = torch.Generator().manual_seed(2)
    w = torch.randn(3, 96, 1024, generator=g) * 0.02
    gs = oq.global_scale(w)
    c_o, s_o = oq.quantize_nvfp4(w, gs)
    c_p, s_p = q4.quantize_nvfp4(w, gs)
    assert torch.equal(c_o, c_p) and torch.equal(s_o, s_p)


@pytest.mark.parametrize("a0,a1", [(0, 2304), (576, 1440), (1152, 1440), (2016, 2304)])
def test_pack_unpack_round_trip(a0, a1):
    from qmesh_b200 import nvfp4 as q4
    e, inter = 2, 2304
    g = torch.Generator().manual_seed(a0 + 1)
    c13 = torch.randint(0, 256, (e, 2 * inter, 2560), generator=g, dtype=torch.uint8)
    s13 = torch.randint(0, 256, (e, 2 * inter, 320), generator=g, dtype=torch.uint8)
    c2 = torch.randint(0, 256, (e, 5120, inter // 2), generator=g, dtype=torch.uint8)
    s2 = torch.randint(0, 256, (e, 5120, inter // 16), generator=g, dtype=torch.uint8)
    w = a1 - a0
    t13 = q4.pack_w13(c13, s13, 0, a0, a1)
    t2 = q4.pack_w2(c2, s2, 0, a0, a1)
    assert t13.numel() == e * (w // 32) * 184320 and t2.numel() == e * 20 * (w // 32) * 4608
    u13, v13 = q4.unpack_w13(t13, e, w)
    u2, v2 = q4.unpack_w2(t2, e, w)
    assert torch.equal(u13[:, :w], c13[:, a0:a1]) and torch.equal(u13[:, w:], c13[:, inter + a0:inter + a1])
    assert torch.equal(v13[:, :w], s13[:, a0:a1]) and torch.equal(v13[:, w:], s13[:, inter + a0:inter + a1])
    assert torch.equal(u2, c2[:, :, a0 // 2:a1 // 2]) and torch.equal(v2, s2[:, :, a0 // 16:a1 // 16])
    # a rank pack (source slice [a0, a1)) packs to the same tiles
    src13 = torch.cat([c13[:, a0:a1], c13[:, inter + a0:inter + a1]], 1)
    srcs13 = torch.cat([s13[:, a0:a1], s13[:, inter + a0:inter + a1]], 1)
    assert torch.equal(q4.pack_w13(src13, srcs13, a0, a0, a1), t13)


def test_tile_bytes_match_kernel_fragment_addressing():
    """Spot-check the byte addresses the decode kernel reads (qx_decode.cu consumer):
    gate/up codes at ((tile*8 + sg)*32 + lane)*16 + j*4 + b, scales at
    16384 + ((tile*8 + sg)*8 + g)*8 + j*2 + hh; down codes at
    cb*4096 + (tile*32 + lane)*8 + s*4 + b, scales at n_cb*4096 + cb*512 + (tile*8 + g)*4 + s*2 + hh."""
    from qmesh_b200 import nvfp4 as q4
    g0 = torch.Generator().manual_seed(4)
    e, inter = 1, 64
    c13 = torch.randint(0, 256, (e, 2 * inter, 2560), generator=g0, dtype=torch.uint8)
    s13 = torch.randint(0, 256, (e, 2 * inter, 320), generator=g0, dtype=torch.uint8)
    t13 = q4.pack_w13(c13, s13, 0, 0, 64)
    for cb, kc, tile, sg, lane, j, b in [(0, 0, 0, 0, 0, 0, 0), (1, 3, 2, 5, 17, 3, 1), (1, 9, 3, 7, 31, 2, 3),
                                         (0, 5, 1, 4, 6, 1, 2)]:
        g, t = lane // 4, lane % 4
        h, hh = b // 2, b % 2
        row = cb * 32 + tile * 8 + g + (inter if hh else 0)
        step = kc * 32 + sg * 4 + j
        off = (cb * 10 + kc) * 18432 + ((tile * 8 + sg) * 32 + lane) * 16 + j * 4 + b
        assert t13[off] == c13[0, row, step * 8 + h * 4 + t]
        soff = (cb * 10 + kc) * 18432 + 16384 + ((tile * 8 + sg) * 8 + g) * 8 + j * 2 + hh
        assert t13[soff] == s13[0, row, step]
    w = 96
    n_cb = w // 32
    c2 = torch.randint(0, 256, (e, 5120, w // 2), generator=g0, dtype=torch.uint8)
    s2 = torch.randint(0, 256, (e, 5120, w // 16), generator=g0, dtype=torch.uint8)
    t2 = q4.pack_w2(c2, s2, 0, 0, w)
    for kt, cb, tile, lane, s_, b in [(0, 0, 0, 0, 0, 0), (7, 2, 15, 29, 1, 3), (19, 1, 4, 10, 0, 2)]:
        g, t = lane // 4, lane % 4
        h, hh = b // 2, b % 2
        row = kt * 256 + tile * 16 + hh * 8 + g
        base = kt * n_cb * 4608
        off = base + cb * 4096 + (tile * 32 + lane) * 8 + s_ * 4 + b
        assert t2[off] == c2[0, row, cb * 16 + s_ * 8 + h * 4 + t]
        soff = base + n_cb * 4096 + cb * 512 + (tile * 8 + g) * 4 + s_ * 2 + hh
        assert t2[soff] == s2[0, row, cb * 2 + s_]


def test_unswizzle_reference_arena_scales():
    from qmesh_b200 import nvfp4 as q4
    lin = torch.randint(0, 127, (2, 1792, 320), dtype=torch.uint8)
    swz = oq.swizzle_scales(lin)
    assert torch.equal(q4.unswizzle_scales(swz, 1792, 320), lin)


def declared_symbols():
    text = (ROOT / "include" / "qmesh_b200.h").read_text()
    return sorted(set(re.findall(r"^[A-Za-z_][\w\s\*]*?\b(qx_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol(lib):
    from qmesh_b200 import _lib
    names = declared_symbols()
    assert len(names) >= 7
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == {s[0] for s in _lib.SIGNATURES}
    assert lib.qx_version().startswith(b"qmesh_b200")


def test_size_queries(lib):
    assert lib.qx_arena_w13_bytes(384, 2304) == 384 * 72 * 184320
    assert lib.qx_arena_w2_bytes(384, 2304) == 384 * 20 * 72 * 4608
    assert lib.qx_arena_w13_bytes(384, 100) == 0  # not 32-aligned
    assert lib.qx_slice_workspace_bytes(6, 6, 0, 2304) > 6 * 6 * (2304 + 5120) * 4
    assert lib.qx_slice_workspace_bytes(65, 6, 0, 2304) == 0
    assert lib.qx_slice_workspace_bytes(1, 9, 0, 2304) == 0


def test_exchange_buffer_layout(lib):
    """Exchange buffer = header (chunk flags/acks/seqs for 8 ranks x 64 chunks,
    unit acks/seqs for 40 x 16 finalize units, 256-aligned) + the BF16 slots of
    the chunk protocol [2][8][rows_max][5120] + the 64-bit receive words of the
    fused protocol [2][8][rows_max][1280][2]."""
    from qmesh_b200 import _lib
    hdr = (8 * 64 + 64 + 64 + 640 + 640) * 4
    hdr = (hdr + 255) // 256 * 256
    for rows_max in (1, 6, 64):
        want = hdr + 2 * 8 * rows_max * 5120 * 2 + 2 * 8 * rows_max * 1280 * 2 * 8
        assert lib.qx_xchg_bytes(rows_max) == want
    assert lib.qx_xchg_bytes(0) == 0 and lib.qx_xchg_bytes(_lib.MAX_ROWS + 1) == 0


def test_decode_rejects_bad_arguments_before_touching_the_device(lib):
    from qmesh_b200 import _lib
    ar = _lib.QxArena(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16),
                      8, 0, 2304, _lib.QX_LAYOUT_FRAG)
    base = dict(x=16, x_scale=16, x_stride=5120, x_fmt=0, ids=16, ids_int64=0, tw=16, rows=1, topk=6,
                c0=0, c1=2304, swiglu_limit=10.0, has_limit=1, out=16, out_stride=5120, workspace=256,
                workspace_bytes=1 << 30)

    def call(**kw):
        a = dict(base, **kw)
        args = _lib.QxSliceArgs(*[a[f[0]] for f in _lib.QxSliceArgs._fields_])
        return lib.qx_slice_decode(ctypes.byref(ar), ctypes.byref(args), None)

    assert call(x=0) == _lib.QX_ERR_ARG
    assert call(x_scale=0) == _lib.QX_ERR_ARG
    assert call(rows=0) == _lib.QX_ERR_SHAPE
    assert call(rows=65) == _lib.QX_ERR_SHAPE
    assert call(topk=9) == _lib.QX_ERR_SHAPE
    assert call(c0=16) == _lib.QX_ERR_SHAPE
    assert call(c1=2336) == _lib.QX_ERR_SHAPE
    assert call(x_stride=100) == _lib.QX_ERR_SHAPE
    assert call(x=24) == _lib.QX_ERR_ALIGN
    assert call(workspace=128) == _lib.QX_ERR_ALIGN
    assert call(workspace_bytes=1024) == _lib.QX_ERR_WORKSPACE
    assert lib.qx_slice_decode(None, None, None) == _lib.QX_ERR_ARG


def test_entry_points_refuse_an_arena_of_the_other_layout(lib):
    """The tensor-core and fragment layouts have equal byte counts, so the arena's
    layout tag is what keeps a tc arena out of the fragment kernels (and the
    reverse): refused with QX_ERR_ARG before any device work."""
    from qmesh_b200 import _lib
    base = dict(x=16, x_scale=16, x_stride=5120, x_fmt=0, ids=16, ids_int64=0, tw=16, rows=1, topk=6,
                c0=0, c1=2304, swiglu_limit=10.0, has_limit=1, out=16, out_stride=5120, workspace=256,
                workspace_bytes=1 << 30)
    args = _lib.QxSliceArgs(*[base[f[0]] for f in _lib.QxSliceArgs._fields_])
    p = [ctypes.c_void_p(16)] * 4
    for layout, refused_by in ((_lib.QX_LAYOUT_TC, ("qx_slice_decode", "qx_slice_decode_static")),
                               (_lib.QX_LAYOUT_FRAG, ("qx_slice_decode_tc",)),
                               (0, ("qx_slice_decode", "qx_slice_decode_tc", "qx_slice_decode_static"))):
        ar = _lib.QxArena(*p, 8, 0, 2304, layout)
        for name in refused_by:
            assert getattr(lib, name)(ctypes.byref(ar), ctypes.byref(args), None) == _lib.QX_ERR_ARG, (name, layout)
        if layout != _lib.QX_LAYOUT_TC:
            assert lib.qx_slice_prefill_tc(ctypes.byref(ar), ctypes.byref(args), ctypes.c_void_p(16),
                                           None) == _lib.QX_ERR_ARG


def test_combine_rejects_bad_arguments(lib):
    from qmesh_b200 import _lib
    arr = (ctypes.c_void_p * 2)(16, 0)
    assert lib.qx_combine_ordered(arr, 2, 5120, ctypes.c_void_p(16), 5120, 0, 1, None) == _lib.QX_ERR_ALIGN
    assert lib.qx_combine_ordered(arr, 0, 5120, ctypes.c_void_p(16), 5120, 0, 1, None) == _lib.QX_ERR_ARG
    assert lib.qx_combine_ordered(arr, 17, 5120, ctypes.c_void_p(16), 5120, 0, 1, None) == _lib.QX_ERR_ARG


def test_product_path_has_no_oracle_or_cpu_fallback():
    """The package never imports the oracle and fails loudly without its library."""
    pkg = ROOT / "qmesh-afd-tp3_b200" / "qmesh_b200"
    for f in pkg.glob("*.py"):
        src = f.read_text()
        assert "import oracle" not in src and "from oracle" not in src, f
