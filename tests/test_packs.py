"""Rank-pack importer (qmesh_b200.packs) on CPU: packs written in the reference's
two forms (pack/build_packs.py: per-expert keys for NODE-A, stacked keys for the
other ranks) read back byte for byte, the ranks' slices concatenate to the full
tensors (the builder's own verification), and pack -> arena -> pack is the
identity for both arena layouts."""

import pytest
import torch

from oracle import moe

INTER = 256
SPLIT = {"p7": (0, 64), "node-b": (64, 160), "node-c": (160, 256)}


@pytest.fixture(scope="module")
def full():
    gen = torch.Generator().manual_seed(21)
    layer = moe.random_code_layer(3, gen, inter=INTER)
    layer["g13"] = torch.rand(3, generator=gen) * 1e-3 + 1e-4
    layer["g2"] = torch.rand(3, generator=gen) * 1e-3 + 1e-4
    return layer


@pytest.fixture(scope="module")
def packdir(full, tmp_path_factory):
    from qmesh_b200 import packs
    root = tmp_path_factory.mktemp("packs")
    for li in range(2):
        for r, (a, b) in SPLIT.items():
            packs.write_layer(packs.layer_file(str(root), r, li), li, full, a, b, per_expert=(r == "p7"))
    return str(root)


def test_read_both_forms_byte_exact(full, packdir):
    from qmesh_b200 import packs
    got = {r: packs.read_layer(packs.layer_file(packdir, r, 1), 1) for r in SPLIT}
    for r, (a, b) in SPLIT.items():
        p = got[r]
        assert torch.equal(p["c13"], torch.cat([full["c13"][:, a:b], full["c13"][:, INTER + a:INTER + b]], dim=1))
        assert torch.equal(p["s13"], torch.cat([full["s13"][:, a:b], full["s13"][:, INTER + a:INTER + b]], dim=1))
        assert torch.equal(p["c2"], full["c2"][:, :, a // 2:b // 2])
        assert torch.equal(p["s2"], full["s2"][:, :, a // 16:b // 16])
        assert torch.equal(p["g13"], full["g13"].float()) and torch.equal(p["g2"], full["g2"].float())
    # the slices of the three ranks concatenate to the full tensors
    c = [got[r]["c13"].shape[1] // 2 for r in SPLIT]
    gate = torch.cat([got[r]["c13"][:, :n] for r, n in zip(SPLIT, c)], dim=1)
    assert torch.equal(gate, full["c13"][:, :INTER])
    assert torch.equal(torch.cat([got[r]["s2"] for r in SPLIT], dim=2), full["s2"])


@pytest.mark.parametrize("layout", ["tc", "frag"])
@pytest.mark.parametrize("rank", ["p7", "node-b"])
def test_pack_arena_roundtrip(full, packdir, layout, rank):
    from qmesh_b200 import packs
    from qmesh_b200.arena import Arena
    a, b = SPLIT[rank]
    ar = Arena("cpu", 2, 3, a, b, layout=layout)
    packs.load_rank(ar, packdir, rank, split=SPLIT)
    back = ar.expert_pack(1, [0, 1, 2])
    want = packs.read_layer(packs.layer_file(packdir, rank, 1), 1)
    for k in ("c13", "s13", "c2", "s2"):
        assert torch.equal(back[k], want[k]), k
    assert torch.equal(back["g13"], want["g13"]) and torch.equal(back["g2"], want["g2"])


def test_rejects_mismatched_arena_and_shapes(full, packdir, tmp_path):
    from qmesh_b200 import packs
    from qmesh_b200.arena import Arena
    with pytest.raises(ValueError):
        packs.load_rank(Arena("cpu", 1, 3, 32, 128), packdir, "node-b", split=SPLIT)   # not inside [64, 160)
    path = str(tmp_path / "x" / "experts-L00.safetensors")
    packs.write_layer(path, 0, full, 0, 64)
    from safetensors.torch import load_file, save_file
    t = load_file(path)
    t["L0.w13.weight_scale_2"][:, 1] += 1.0       # w1 and w3 global scales must agree
    save_file(t, path)
    with pytest.raises(ValueError):
        packs.read_layer(path, 0)
