"""Generate the golden fixtures in this folder by running the reference itself.

Run from the repository root, in a container where the reference tree is
mounted, naming its root with ``--reference`` or the ``FQKV_REFERENCE``
environment variable (one of them is required)::

    python tests/golden/make_golden.py --reference <path-to-reference-root>

The reference's Python functions live inside notebook cells and a test
function, so this script extracts their definitions from the reference files
(``notebooks/integration_and_benchmarks.ipynb`` cells defining ``sdpa_ref``,
``qpt``, ``quant_int4_per_token``, ``dequant_int4``; ``tests/test_kernels.py``
``_sdpa`` and the ``qpt`` nested in ``test_int8``), executes those definitions
unmodified, and calls them on seeded CPU inputs.  Only inputs and outputs are
written (``*.npz``); no reference source is copied.  The GPU box never runs
this script -- the committed ``.npz`` files travel instead.
"""
from __future__ import annotations

import ast
import json
import math
import os
import pathlib
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = pathlib.Path(__file__).resolve().parent
REF = pathlib.Path(".")  # set by main() from --reference / FQKV_REFERENCE


def _notebook_defs() -> dict:
    nb = json.loads((REF / "notebooks" / "integration_and_benchmarks.ipynb").read_text())
    wanted = {"sdpa_ref", "qpt", "quant_int4_per_token", "dequant_int4"}
    ns: dict = {"torch": torch, "F": F, "math": math}
    for cell in nb["cells"]:
        if cell["cell_type"] != "code":
            continue
        src = "".join(cell["source"])
        try:
            tree = ast.parse(src)
        except SyntaxError:          # cells with shell magics
            continue
        defs = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in wanted]
        if defs:
            exec(compile(ast.Module(body=defs, type_ignores=[]), "<reference-notebook>", "exec"), ns)
    missing = wanted - ns.keys()
    if missing:
        raise RuntimeError(f"reference notebook lacks {missing}")
    return ns


def _testfile_defs() -> dict:
    tree = ast.parse((REF / "tests" / "test_kernels.py").read_text())
    ns: dict = {"torch": torch, "F": F, "math": math}
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == "_sdpa":
            keep.append(node)
        if isinstance(node, ast.FunctionDef) and node.name == "test_int8":
            for inner in node.body:
                if isinstance(inner, ast.FunctionDef) and inner.name == "qpt":
                    keep.append(inner)
    exec(compile(ast.Module(body=keep, type_ignores=[]), "<reference-tests>", "exec"), ns)
    return {"_sdpa": ns["_sdpa"], "qpt_test": ns["qpt"]}


def _edge_tokens(D: int) -> torch.Tensor:
    """Hand-made tokens that exercise every branch of the quantizer rules."""
    rows = []
    z = torch.zeros(D, dtype=torch.float16)
    rows.append(z.clone())                                         # all zero -> s=0, codes 0
    t = z.clone(); t[3] = 1e-7; t[5] = -3e-7; rows.append(t)       # scale underflows to 0 -> +-inf codes
    t = z.clone(); t[0] = 65504.0; t[1] = -65504.0; t[2] = 1.0; rows.append(t)   # fp16 max
    t = torch.full((D,), -2.5, dtype=torch.float16); rows.append(t)              # constant negative
    # ties: values that land exactly on k + 0.5 after the fp16 division
    t = torch.tensor([(i % 16) * 0.5 for i in range(D)], dtype=torch.float16)
    t[0] = 127.0; rows.append(t)
    t = torch.tensor([(i % 16) * 0.5 for i in range(D)], dtype=torch.float16)
    t[0] = 7.0; rows.append(t)
    t = torch.randn(D, dtype=torch.float16) * 1e-4; rows.append(t)             # subnormal scales
    t = torch.randn(D, dtype=torch.float16) * 3000; rows.append(t)             # large magnitude
    t = torch.randn(D, dtype=torch.float16); t[7] = float("nan"); rows.append(t)  # NaN token
    t = torch.randn(D, dtype=torch.float16); t[9] = float("inf"); rows.append(t)  # inf token
    return torch.stack(rows)


def make_quant(nb: dict, tf: dict) -> None:
    out = {}
    for D in (64, 128):
        torch.manual_seed(0)
        X = torch.randn(3, 37, D, dtype=torch.float16)
        E = _edge_tokens(D).view(1, -1, D)
        for tag, T in (("rand", X), ("edge", E)):
            c8, s8 = nb["qpt"](T)
            c8t, s8t = tf["qpt_test"](T)
            assert torch.equal(c8, c8t) and torch.equal(s8.view(torch.int16), s8t.view(torch.int16))
            p4, s4 = nb["quant_int4_per_token"](T)
            dq4 = nb["dequant_int4"](p4, s4)
            out[f"X_{tag}_D{D}"] = T.numpy()
            out[f"codes8_{tag}_D{D}"] = c8.numpy()
            out[f"scales8_{tag}_D{D}"] = s8.numpy()
            out[f"packed4_{tag}_D{D}"] = p4.numpy()
            out[f"scales4_{tag}_D{D}"] = s4.numpy()
            out[f"deq4_{tag}_D{D}"] = dq4.numpy()
    np.savez_compressed(HERE / "quant_golden.npz", **out)


def make_attention(nb: dict, tf: dict) -> None:
    out = {}
    # single-row ops (fp16 / int8 / int4) at the reference test shapes' D
    for D, R, N in ((64, 4, 3), (64, 2, 100), (128, 2, 131), (128, 2, 1)):
        torch.manual_seed(0)
        q = torch.randn(R, D, dtype=torch.float16)
        K = torch.randn(R, N, D, dtype=torch.float16)
        V = torch.randn(R, N, D, dtype=torch.float16)
        key = f"R{R}_N{N}_D{D}"
        out[f"q_{key}"] = q.numpy(); out[f"K_{key}"] = K.numpy(); out[f"V_{key}"] = V.numpy()
        out[f"sdpa_{key}"] = tf["_sdpa"](q, K, V).numpy()
        out[f"sdparef_{key}"] = nb["sdpa_ref"](q, K, V).numpy()
        # fp32 einsum oracle of the notebook's int4 accuracy cell (lines 483-484)
        p = torch.softmax(torch.einsum("bnd,bd->bn", K.float(), q.float()) / math.sqrt(D), 1)
        out[f"einsum_{key}"] = torch.einsum("bn,bnd->bd", p, V.float()).numpy()
        # int8: reference quantizer + its dequantised SDPA oracle (tests/test_kernels.py:35-38)
        Kq, Ks = nb["qpt"](K); Vq, Vs = nb["qpt"](V)
        Kd = (Kq.float() * Ks.float()[:, :, None]).half(); Vd = (Vq.float() * Vs.float()[:, :, None]).half()
        out[f"int8ref_{key}"] = F.scaled_dot_product_attention(
            q.view(R, 1, 1, D), Kd.view(R, 1, N, D), Vd.view(R, 1, N, D)).view(R, D).numpy()
        # int4: reference packer + dequant SDPA oracle (notebook lines 462-466)
        Kp, Ks4 = nb["quant_int4_per_token"](K); Vp, Vs4 = nb["quant_int4_per_token"](V)
        Kd4 = nb["dequant_int4"](Kp, Ks4).half(); Vd4 = nb["dequant_int4"](Vp, Vs4).half()
        out[f"int4ref_{key}"] = F.scaled_dot_product_attention(
            q.view(R, 1, 1, D), Kd4.view(R, 1, N, D), Vd4.view(R, 1, N, D)).view(R, D).numpy()
    # GQA (tests/test_kernels.py:41-51) and split-K (:57-70) oracles, small shapes
    for D, B, N in ((64, 2, 37), (128, 1, 29)):
        torch.manual_seed(0)
        Hq, Hkv = 32, 8
        q = torch.randn(B, Hq, D, dtype=torch.float16)
        K = torch.randn(B, Hkv, N, D, dtype=torch.float16)
        V = torch.randn(B, Hkv, N, D, dtype=torch.float16)
        Ke = K.repeat_interleave(Hq // Hkv, 1); Ve = V.repeat_interleave(Hq // Hkv, 1)
        ref = F.scaled_dot_product_attention(q.view(B, Hq, 1, D), Ke, Ve).view(B, Hq, D)
        key = f"gqa_B{B}_N{N}_D{D}"
        out[f"q_{key}"] = q.numpy(); out[f"K_{key}"] = K.numpy(); out[f"V_{key}"] = V.numpy()
        out[f"sdpa_{key}"] = ref.numpy()
    np.savez_compressed(HERE / "attention_golden.npz", **out)


def main() -> int:
    global REF
    import argparse
    ap = argparse.ArgumentParser(description="regenerate the golden fixtures from the reference's own code")
    ap.add_argument("--reference", default=os.environ.get("FQKV_REFERENCE"),
                    help="root of the reference tree (default: $FQKV_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference tree with --reference or FQKV_REFERENCE")
    REF = pathlib.Path(args.reference)
    if not REF.exists():
        print(f"reference tree not found at {REF}; fixtures unchanged", file=sys.stderr)
        return 1
    nb = _notebook_defs()
    tf = _testfile_defs()
    make_quant(nb, tf)
    make_attention(nb, tf)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size, "bytes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
