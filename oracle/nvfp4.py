"""NVFP4 / FP8 codec restated on the CPU (torch, float32) -- test infrastructure.

Every function states the reference line it follows. Paths are relative to the
QMesh AFD-TP3 tree.
"""

from __future__ import annotations

import torch

K_BLOCK = 16            # elements per e4m3 block scale (fp4_decode_moe_swz.cu:19-24)
E2M1_MAX = 6.0
E4M3_MAX = 448.0        # qmesh_afd_seam.cu:9-16, afd_session.py:47-50

# e2m1 magnitudes indexed by the low three bits of a nibble; bit 3 is the sign
# (fp4_decode_moe_swz.cu:82-89 decodes with cvt.rn.f16x2.e2m1x2, which implements
# this table).
E2M1_MAG = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
_E2M1_TABLE = torch.tensor(list(E2M1_MAG) + [-v for v in E2M1_MAG], dtype=torch.float32)
# midpoints between consecutive magnitudes, for round-to-nearest-even encoding
_E2M1_MID = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=torch.float32)


def e2m1_decode(nib: torch.Tensor) -> torch.Tensor:
    """Nibble (0..15, uint8) -> float32. Code 8 is -0.0."""
    return _E2M1_TABLE[nib.to(torch.int64) & 15]


def e4m3_decode(b: torch.Tensor) -> torch.Tensor:
    """e4m3fn byte -> float32 from the bit fields (bias 7, subnormals, 0x7f/0xff NaN).

    Restates the scale decode of fp4_decode_moe_swz.cu:91-96 (hardware
    cvt.rn.f16x2.e4m3x2) without going through torch's own float8 cast, so the
    two can be checked against each other.
    """
    b = b.to(torch.int64) & 0xFF
    sign = torch.where((b >> 7) == 1, -1.0, 1.0)
    ex = (b >> 3) & 0xF
    man = (b & 7).to(torch.float32)
    sub = man / 8.0 * 2.0 ** -6
    nrm = (1.0 + man / 8.0) * torch.pow(2.0, (ex - 7).to(torch.float32))
    val = torch.where(ex == 0, sub, nrm) * sign
    nan = (ex == 15) & ((b & 7) == 7)
    return torch.where(nan, torch.full_like(val, float("nan")), val).to(torch.float32)


def e4m3_encode(v: torch.Tensor) -> torch.Tensor:
    """float32 -> e4m3fn byte, round to nearest even, saturating at +-448.

    The clamp before the cast is the seam's satfinite convention
    (qmesh_afd_seam.cu:157-160): torch's own cast turns 500 into NaN.
    """
    v = torch.clamp(v.to(torch.float32), -E4M3_MAX, E4M3_MAX)
    return v.to(torch.float8_e4m3fn).view(torch.uint8)


def e2m1_encode(v: torch.Tensor) -> torch.Tensor:
    """float32 -> e2m1 nibble, round to nearest even, saturating at +-6."""
    v = v.to(torch.float32)
    a = torch.clamp(v.abs(), max=E2M1_MAX)
    i = torch.searchsorted(_E2M1_MID, a.contiguous(), right=False)
    mid = _E2M1_MID[torch.clamp(i, max=6)]
    tie = (i < 7) & (a == mid) & ((i & 1) == 1)
    c = torch.where(tie, i + 1, i).to(torch.uint8)
    neg = torch.signbit(v)
    return torch.where(neg, c | 8, c).to(torch.uint8)


def unpack_codes(codes: torch.Tensor) -> torch.Tensor:
    """[..., K/2] bytes -> [..., K] nibbles; low nibble is the even element
    (fp4_decode_moe_swz.cu:58, :82-89)."""
    lo = codes & 0x0F
    hi = (codes >> 4) & 0x0F
    return torch.stack([lo, hi], dim=-1).reshape(*codes.shape[:-1], codes.shape[-1] * 2)


def pack_codes(nib: torch.Tensor) -> torch.Tensor:
    """[..., K] nibbles -> [..., K/2] bytes (inverse of unpack_codes)."""
    n = nib.reshape(*nib.shape[:-1], nib.shape[-1] // 2, 2).to(torch.uint8)
    return (n[..., 0] & 0x0F) | ((n[..., 1] & 0x0F) << 4)


def dequant(codes: torch.Tensor, scales: torch.Tensor, gscale) -> torch.Tensor:
    """NVFP4 -> float32: e2m1(code) * e4m3(block scale) * weight_scale_2.

    Convention of gx/gx_expert_worker.py:19-26 (dequant = code * block_scale *
    weight_global_scale). e2m1 * e4m3 is exact in float32; the global-scale
    multiply is the one rounding.
    """
    vals = e2m1_decode(unpack_codes(codes))
    s = e4m3_decode(scales)
    s = s.repeat_interleave(K_BLOCK, dim=-1)
    w = vals * s
    if not (isinstance(gscale, (int, float)) and gscale == 1.0):
        w = w * torch.as_tensor(gscale, dtype=torch.float32)
    return w


def global_scale(w: torch.Tensor) -> torch.Tensor:
    """Per-tensor FP32 global scale: amax / (6 * 448)."""
    a = w.abs().amax().to(torch.float32)
    return torch.where(a > 0, a / (E2M1_MAX * E4M3_MAX), torch.ones_like(a))


def quantize_nvfp4(w: torch.Tensor, g: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """float32 [..., K] -> (codes [..., K/2] uint8, scales [..., K/16] uint8).

    Block scale = e4m3(amax16 / 6 / g) (RNE), element code = e2m1(w / (scale * g))
    with RNE and saturation; the standard NVFP4 recipe the checkpoint packs use
    (e2m1 codes, e4m3 scale per 16 elements along K, FP32 per-tensor scale).
    """
    w = w.to(torch.float32)
    g = torch.as_tensor(g, dtype=torch.float32)
    blk = w.reshape(*w.shape[:-1], w.shape[-1] // K_BLOCK, K_BLOCK)
    amax = blk.abs().amax(dim=-1)
    s = e4m3_encode(amax / E2M1_MAX / g)
    sdec = e4m3_decode(s)
    denom = (sdec * g).unsqueeze(-1)
    scaled = torch.where(denom > 0, blk / torch.where(denom > 0, denom, 1.0), 0.0)
    codes = pack_codes(e2m1_encode(scaled).reshape(w.shape))
    return codes, s


def bf16_round(x: torch.Tensor) -> torch.Tensor:
    """float32 -> nearest-even bfloat16, returned as float32."""
    return x.to(torch.float32).to(torch.bfloat16).to(torch.float32)


BF16_FLOOR = float(torch.tensor(1e-6, dtype=torch.bfloat16).float())


def fp8_quant_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Producer-side FP8 activation transport, one scale per row.

    Arithmetic of native/qmesh_afd_seam.cu:9-16 (and afd_session.py:106-110),
    applied per row instead of per post:
        mc  = max(amax|x|, bf16(1e-6))
        s   = float(448 / double(mc)),  inv = float(1 / double(448 / mc))
        q   = e4m3_rne(clamp(bf16_rn(float(x) * s), +-448))
    `x` holds bfloat16 values (float32 tensor). Returns (q uint8 [R,K], inv [R]).
    """
    x = x.to(torch.float32)
    m = x.abs().amax(dim=-1).to(torch.float64)
    mc = torch.clamp(m, min=BF16_FLOOR)
    sd = 448.0 / mc
    s = sd.to(torch.float32)
    inv = (1.0 / sd).to(torch.float32)
    y = bf16_round(x * s.unsqueeze(-1))
    q = e4m3_encode(y)
    return q, inv


def fp8_quant_post(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The same transport with ONE scale for all rows of a post, the reference's
    form (p7/afd_overlay/afd_session.py:106-107: scale = 448 / amax over the
    post's rows; native/qmesh_afd_seam.cu:88-176 on the device). Returns
    (q uint8 [R,K], inv float32 [1])."""
    x = x.to(torch.float32)
    m = x.abs().amax().to(torch.float64)
    mc = torch.clamp(m, min=BF16_FLOOR)
    sd = 448.0 / mc
    s = sd.to(torch.float32)
    inv = (1.0 / sd).to(torch.float32)
    q = e4m3_encode(bf16_round(x * s))
    return q, inv.reshape(1)


def fp8_ingest(q: torch.Tensor, inv: torch.Tensor) -> torch.Tensor:
    """Consumer side, gx/gx_ingest.py:151-154: x = bf16(float(e4m3) * inv)."""
    v = e4m3_decode(q)
    return bf16_round(v * inv.to(torch.float32).unsqueeze(-1))


def swizzle_offset(row: torch.Tensor, kb: torch.Tensor, kbp: int) -> torch.Tensor:
    """Byte offset of block scale (row, kb) in the vLLM/CUTLASS swizzled layout.

    fp4_decode_moe_swz.cu:19-21:
        (row/128)*(kbp*128) + (kb/4)*512 + (row%32)*16 + ((row%128)/32)*4 + kb%4
    kbp is the padded number of 16-element blocks per row (multiple of 4).
    """
    row = row.to(torch.int64)
    kb = kb.to(torch.int64)
    return ((row // 128) * (kbp * 128) + (kb // 4) * 512 + (row % 32) * 16
            + ((row % 128) // 32) * 4 + kb % 4)


def swizzle_scales(lin: torch.Tensor) -> torch.Tensor:
    """[..., M, KB] linear scales -> [..., Mp, KBp] swizzled bytes (padding zero)."""
    *lead, m, kb = lin.shape
    mp = (m + 127) // 128 * 128
    kbp = (kb + 3) // 4 * 4
    out = torch.zeros(*lead, mp * kbp, dtype=torch.uint8)
    r = torch.arange(m).unsqueeze(-1).expand(m, kb)
    c = torch.arange(kb).unsqueeze(0).expand(m, kb)
    off = swizzle_offset(r, c, kbp).reshape(-1)
    out[..., off] = lin.reshape(*lead, m * kb).to(torch.uint8)
    return out.reshape(*lead, mp, kbp)


def unswizzle_scales(swz: torch.Tensor, m: int, kb: int) -> torch.Tensor:
    """Inverse of swizzle_scales: [..., Mp, KBp] -> [..., m, kb]."""
    *lead, mp, kbp = swz.shape
    flat = swz.reshape(*lead, mp * kbp)
    r = torch.arange(m).unsqueeze(-1).expand(m, kb)
    c = torch.arange(kb).unsqueeze(0).expand(m, kb)
    off = swizzle_offset(r, c, kbp).reshape(-1)
    return flat[..., off].reshape(*lead, m, kb)
