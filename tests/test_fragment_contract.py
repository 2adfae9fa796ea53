"""CPU emulation of the decode kernel's tensor-core fragment contract.

Reads the packed arena tiles and the activation buffers exactly at the byte
addresses the consumer warps of qx_decode.cu read, assembles the m16n8k16
A (16x16, row) and B (16x8, col) fragments per the PTX fragment map
(groupID g = lane/4, t = lane%4: A regs {(g,2t..), (g+8,2t..), (g,2t+8..),
(g+8,2t+8..)}, B regs {(2t.., g), (2t+8.., g)}), and checks the products
against a direct evaluation. No GPU needed.
"""

import numpy as np
import torch

from oracle import nvfp4 as oq

KC = 512


def frag_word_off(k: int) -> int:
    """Mirror of qx_decode.cu frag_word_off (x16 B-fragment order)."""
    i, e = k >> 4, k & 15
    t, word = (e & 7) >> 1, e >> 3
    return (i >> 1) * 64 + t * 16 + ((i & 1) * 2 + word) * 4


def act_off(w: int, q: int, c: int) -> int:
    """Mirror of qx_decode.cu act_off (down-projection B-fragment order)."""
    cb, s, kk = c >> 5, (c >> 4) & 1, c & 15
    t, word, half = (kk & 7) >> 1, kk >> 3, kk & 1
    return q * w * 4 + cb * 128 + s * 64 + t * 16 + word * 4 + half * 2


def e2m1_pair(byte: int):
    v = oq.e2m1_decode(torch.tensor([byte & 15, byte >> 4], dtype=torch.uint8))
    return float(v[0]), float(v[1])


def e4m3(b: int) -> float:
    return float(oq.e4m3_decode(torch.tensor([b], dtype=torch.uint8))[0])


def a_fragment(word_bytes, sc_lo, sc_hi, g, t, a):
    """Place one lane's 4 code bytes into the 16x16 A tile (scales folded)."""
    A, B, C, D = word_bytes
    a[g, 2 * t:2 * t + 2] = np.array(e2m1_pair(A)) * sc_lo
    a[g + 8, 2 * t:2 * t + 2] = np.array(e2m1_pair(B)) * sc_hi
    a[g, 2 * t + 8:2 * t + 10] = np.array(e2m1_pair(C)) * sc_lo
    a[g + 8, 2 * t + 8:2 * t + 10] = np.array(e2m1_pair(D)) * sc_hi


def test_gate_up_fragments_reproduce_the_dot_products():
    from qmesh_b200 import nvfp4 as q4
    gen = torch.Generator().manual_seed(8)
    inter, hid = 32, 5120
    c13 = torch.randint(0, 256, (1, 2 * inter, hid // 2), generator=gen, dtype=torch.uint8)
    s13 = torch.randint(0x20, 0x48, (1, 2 * inter, hid // 16), generator=gen, dtype=torch.uint8)
    tiles = q4.pack_w13(c13, s13, 0, 0, 32).numpy()
    # one activation row in the x16 fragment order
    x = (torch.randn(hid, generator=gen) * 4).to(torch.float16).float().numpy()
    x16 = np.zeros(hid, dtype=np.float16)
    xb = x16.view(np.uint8)
    for k in range(0, hid, 2):
        off = (k // KC) * KC * 2 + frag_word_off(k % KC)
        xb[off:off + 4] = np.array([x[k], x[k + 1]], dtype=np.float16).view(np.uint8)
    wg = oq.dequant(c13[0], s13[0], 1.0).double().numpy()
    tile, kc = 2, 7
    got = np.zeros((16, 8))
    stage = tiles[kc * 18432:(kc + 1) * 18432]
    chunk = xb[kc * KC * 2:(kc + 1) * KC * 2]
    for sg in range(8):
        for j in range(4):
            a = np.zeros((16, 16))
            b = np.zeros((16, 8))
            for lane in range(32):
                g, t = lane // 4, lane % 4
                base = ((tile * 8 + sg) * 32 + lane) * 16 + j * 4
                sbase = 16384 + ((tile * 8 + sg) * 8 + g) * 8 + j * 2
                a_fragment(stage[base:base + 4], e4m3(stage[sbase]), e4m3(stage[sbase + 1]), g, t, a)
                if g == 0:  # pair 0 is the only routed row here
                    sp, si = (sg * 4 + j) // 2, (sg * 4 + j) % 2
                    u = chunk[sp * 64 + t * 16 + si * 8:sp * 64 + t * 16 + si * 8 + 8].view(np.float16)
                    b[2 * t:2 * t + 2, 0] = u[0:2]
                    b[2 * t + 8:2 * t + 10, 0] = u[2:4]
            got += a @ b
    k0 = kc * KC
    rows_g = [tile * 8 + g for g in range(8)]
    want_gate = wg[rows_g, k0:k0 + KC] @ x[k0:k0 + KC]
    want_up = wg[[inter + r for r in rows_g], k0:k0 + KC] @ x[k0:k0 + KC]
    np.testing.assert_allclose(got[:8, 0], want_gate, rtol=1e-9, atol=1e-9)
    np.testing.assert_allclose(got[8:, 0], want_up, rtol=1e-9, atol=1e-9)


def test_down_fragments_reproduce_the_dot_products():
    from qmesh_b200 import nvfp4 as q4
    gen = torch.Generator().manual_seed(9)
    w, hid = 96, 5120
    c2 = torch.randint(0, 256, (1, hid, w // 2), generator=gen, dtype=torch.uint8)
    s2 = torch.randint(0x20, 0x48, (1, hid, w // 16), generator=gen, dtype=torch.uint8)
    tiles = q4.pack_w2(c2, s2, 0, 0, w).numpy()
    n_cb = w // 32
    w2 = oq.dequant(c2[0], s2[0], 1.0).double().numpy()
    # two pairs of activations stored as (hi, lo) f16 in the act fragment order
    P = 2
    act = (torch.randn(P, w, generator=gen) * 3).numpy()
    buf = np.zeros(P * w * 4, dtype=np.uint8)
    for q in range(P):
        for c in range(w):
            hi = np.float16(act[q, c])
            lo = np.float16(act[q, c] - np.float32(hi))
            o = act_off(w, q, c)
            buf[o:o + 2] = np.array([hi], dtype=np.float16).view(np.uint8)
            buf[o + 8:o + 10] = np.array([lo], dtype=np.float16).view(np.uint8)
    eff = np.zeros((P, w))
    for q in range(P):
        for c in range(w):
            o = act_off(w, q, c)
            eff[q, c] = float(buf[o:o + 2].view(np.float16)[0]) + float(buf[o + 8:o + 10].view(np.float16)[0])
    kt, tile = 11, 9
    got = np.zeros((16, 8))
    base_kt = kt * n_cb * 4608
    for cb in range(n_cb):
        for s in range(2):
            a = np.zeros((16, 16))
            b = np.zeros((16, 8))
            for lane in range(32):
                g, t = lane // 4, lane % 4
                off = base_kt + cb * 4096 + (tile * 32 + lane) * 8 + s * 4
                soff = base_kt + n_cb * 4096 + cb * 512 + (tile * 8 + g) * 4 + s * 2
                a_fragment(tiles[off:off + 4], e4m3(tiles[soff]), e4m3(tiles[soff + 1]), g, t, a)
                if g < P:
                    ab = buf[g * w * 4 + cb * 128 + s * 64 + t * 16:][:16]
                    hi = ab[0:8].view(np.float16).astype(np.float64)
                    lo = ab[8:16].view(np.float16).astype(np.float64)
                    b[2 * t:2 * t + 2, g] = hi[0:2] + lo[0:2]
                    b[2 * t + 8:2 * t + 10, g] = hi[2:4] + lo[2:4]
            got += a @ b
    rows = [kt * 256 + tile * 16 + r for r in range(16)]
    want = w2[rows] @ eff.T
    np.testing.assert_allclose(got[:, :P], want, rtol=1e-9, atol=1e-9)
    # the (hi, lo) pair carries the FP32 activation to ~22 bits
    assert np.abs(eff - act).max() <= np.abs(act).max() * 2.0 ** -21
