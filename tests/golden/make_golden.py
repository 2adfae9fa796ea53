"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run once in a container that has the reference tree (read-only) and vLLM:

    python tests/golden/make_golden.py /path/to/QMesh-AFD-TP3

Every fixture comes from running the reference's own Python code (or the
third-party function it calls) on the CPU; nothing is restated here:

* swizzle.npz   vLLM ``swizzle_blockscale`` (vllm 0.22.0 as installed; the reference
                pins 0.24.0, GX_FP4_DECODE_CEILING.md:3-4) on random e4m3 scale
                tensors. Its trailing ``.cuda()`` is replaced by the identity so
                it runs without a GPU; the permutation itself is untouched.
* routing.json  gx/gx_ingest.py ``bucket_of``, ``graph_rows``, ``classify_ids``.
* swiglu.npz    gx/gx_expert_worker.py ``swiglu`` (unclamped gate-first form).
* ingest.npz    gx/gx_ingest.py ``_ingest`` Triton kernel run by Triton's CPU
                interpreter: e4m3 slab * header inv -> bf16 x, id sanitising.
* arena.json    gx/gx_expert_worker.py ``Arena.bytes_per_layer`` for CP=896.
* prefill_quant.npz
                vLLM ``ref_nvfp4_quant`` (nvfp4_emulation_utils.py): the NVFP4
                activation quantiser of the reference's W4A4 prefill body
                (scaled_fp4_experts_quant, gx/gx_ingest.py:225-237), on rows with
                zero blocks, ties and a range of magnitudes and global scales; and
                ``SiluAndMulWithClamp.forward_native`` (the clamp SwiGLU of
                gx/gx_ingest.py:235) on bf16 gate/up values.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path
from unittest import mock

import numpy as np

HERE = Path(__file__).resolve().parent


def main(ref: str) -> None:
    sys.path.insert(0, os.path.join(ref, "gx"))
    import torch

    # ---- vLLM swizzle ----------------------------------------------------------
    from vllm.model_executor.layers.quantization.utils.nvfp4_utils import swizzle_blockscale
    g = torch.Generator().manual_seed(11)
    cases = {}
    for name, (b, m, k) in {"a": (2, 200, 10), "b": (1, 256, 320), "c": (3, 96, 56)}.items():
        raw = torch.randint(0, 127, (b, m, k), generator=g, dtype=torch.uint8)
        lin = raw.view(torch.float8_e4m3fn)
        with mock.patch.object(torch.Tensor, "cuda", lambda self, *a, **kw: self):
            swz = swizzle_blockscale(lin)
        cases[f"{name}_lin"] = raw.numpy()
        cases[f"{name}_swz"] = swz.view(torch.uint8).numpy()
    np.savez_compressed(HERE / "swizzle.npz", **cases)

    # ---- routing policy / buckets ----------------------------------------------
    import gx_ingest as gxi
    ids = [
        [[0, 1, 2, 3, 4, 5]],
        [[-1, -1, -1, -1, -1, -1]],
        [[0, 383, 384, -2, 7, -1]],
        [[5, 5, 5, 5, 5, 5], [-7, 1000, 3, 2, 1, 0]],
    ]
    routing = {
        "bucket_of": {str(n): gxi.bucket_of(n) for n in range(1, 70)},
        "graph_rows": {str(n): gxi.graph_rows(n) for n in range(1, 70)},
        "classify_ids": [[i, list(gxi.classify_ids(np.array(i)))] for i in ids],
        "E": gxi.E,
        "TOPK": gxi.TOPK,
        "GRAPH_MAX": gxi.GRAPH_MAX,
    }
    (HERE / "routing.json").write_text(json.dumps(routing, indent=1))

    # ---- reference SwiGLU ---------------------------------------------------------
    import gx_expert_worker as gxw
    h = torch.randn(5, 2 * 64, generator=g) * 4
    sw = gxw.swiglu(h.to(torch.bfloat16), 64)
    np.savez_compressed(HERE / "swiglu.npz", h=h.to(torch.bfloat16).float().numpy(), out=sw.numpy())

    make_prefill_fixture(torch.Generator().manual_seed(17))

    # ---- arena size accounting -------------------------------------------------------
    a = gxw.Arena.__new__(gxw.Arena)
    a.cp = gxw.CP
    (HERE / "arena.json").write_text(json.dumps({"cp": gxw.CP, "bytes_per_layer": a.bytes_per_layer()}))

    # ---- the ingest kernel under Triton's interpreter (fresh process: the
    # interpreter must be chosen before triton is first imported) -----------------
    import subprocess
    env = dict(os.environ, TRITON_INTERPRET="1")
    subprocess.run([sys.executable, __file__, ref, "--ingest"], env=env, check=True)


def make_prefill_fixture(g) -> None:
    import types

    import torch
    from vllm.model_executor.layers.activation import SiluAndMulWithClamp
    from vllm.model_executor.layers.quantization.utils.nvfp4_emulation_utils import ref_nvfp4_quant
    x = torch.randn(6, 256, generator=g)
    x[0] *= 1e-3
    x[1] *= 40.0
    x[2, :16] = 0.0                                            # an all-zero block
    x[3, :16] = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 2)   # grid midpoints
    x[4] = torch.randn(256, generator=g).to(torch.bfloat16).float()
    x[5] = torch.exp(torch.randn(256, generator=g) * 3) * torch.sign(torch.randn(256, generator=g))
    out = {"x": x.numpy()}
    for i, gs in enumerate([3.0, 6.0 / float(x.abs().max()), 0.02, 1e4]):
        codes, scale = ref_nvfp4_quant(x, torch.tensor(gs, dtype=torch.float32), 16)
        out[f"gs{i}"] = np.float32(gs)
        out[f"codes{i}"] = codes.numpy()                        # e2m1 values (float32)
        out[f"scale{i}"] = scale.numpy()                        # e4m3 values (float32)
    h = (torch.randn(7, 2 * 64, generator=g) * 6).to(torch.bfloat16)
    sw = SiluAndMulWithClamp.forward_native(types.SimpleNamespace(swiglu_limit=10.0), h.float())
    out["swiglu_h"] = h.float().numpy()
    out["swiglu_out"] = sw.numpy()
    np.savez_compressed(HERE / "prefill_quant.npz", **out)


def make_ingest_fixture(ref: str) -> None:
    sys.path.insert(0, os.path.join(ref, "gx"))
    import torch
    import gx_ingest as gxi
    g = torch.Generator().manual_seed(13)
    n, b = 3, 4
    k = gxi.K
    x = torch.randn(n, k, generator=g) * 3
    amax = float(x.abs().max())
    s = 448.0 / amax
    slab = (x * s).clamp(-448, 448).to(torch.float8_e4m3fn)
    inv = 1.0 / s
    ids = torch.tensor([[0, 5, 9, 383, 17, 2], [-1, 1, 2, 3, 4, 5], [7, 384, -3, 1, 2, 3]], dtype=torch.int32)
    tw = torch.rand(n, 6, generator=g)
    rout = torch.zeros(4 + 2 * n * 6, dtype=torch.int32)
    rout[0] = 1
    rout[1] = n
    rout[2] = torch.tensor([inv], dtype=torch.float32).view(torch.int32)[0]
    rout[3] = 1
    rout[4:4 + n * 6] = ids.reshape(-1)
    rout[4 + n * 6:] = tw.reshape(-1).view(torch.int32)
    xo = torch.zeros(b, k, dtype=torch.bfloat16)
    io = torch.zeros(b, 6, dtype=torch.int32)
    to = torch.zeros(b, 6, dtype=torch.float32)
    isum = torch.zeros(1, dtype=torch.int32)
    pad = torch.zeros(1, dtype=torch.int32)
    bad = torch.zeros(1, dtype=torch.int32)
    gxi._ingest[(b,)](slab.view(torch.uint8).view(torch.float8_e4m3fn), rout, xo, io, to, isum, pad, bad, 0,
                      K_=k, BLK_=gxi.BLK, TOPK_=6, TOPKP=8, E_=gxi.E)
    np.savez_compressed(HERE / "ingest.npz", slab=slab.view(torch.uint8).numpy(), inv=np.float32(inv),
                        ids=ids.numpy(), tw=tw.numpy(), x=xo.float().numpy(), ids_out=io.numpy(),
                        tw_out=to.numpy(), pad=pad.numpy(), bad=bad.numpy(), n=n)


if __name__ == "__main__":
    # the reference tree: the first argument that is not an option, else QX_REFERENCE_ROOT
    _pos = [a for a in sys.argv[1:] if not a.startswith("--")]
    _ref = _pos[0] if _pos else os.environ.get("QX_REFERENCE_ROOT", "")
    if not _ref and "--prefill" not in sys.argv:
        sys.exit("usage: make_golden.py REFERENCE_TREE [--ingest | --prefill] (or set QX_REFERENCE_ROOT)")
    if "--ingest" in sys.argv:
        make_ingest_fixture(_ref)
    elif "--prefill" in sys.argv:
        import torch
        make_prefill_fixture(torch.Generator().manual_seed(17))
    else:
        main(_ref)
