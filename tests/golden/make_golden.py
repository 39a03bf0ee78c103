"""Regenerate the golden fixtures from the REFERENCE implementation (run in the build
container, where the reference checkout exists; the outputs are committed).

For each small seeded model this script
  1. draws the expert weights with the same recipe as ``wisp_b200.converter``,
  2. quantises them with the reference's ``wisp.converter.quantizer.quantize_int4``
     and writes the blobs with ``wisp.converter.partitioner.write_expert_file``,
  3. records each blob's sha256, and
  4. runs the reference engine's own CPU ``run_moe`` (oracle/_ref harness) on a seeded
     input, recording outputs, routed indices and gate weights (block and stack).
It also records quantiser edge cases (constant group, odd sizes with padding), and one
model directory in the form the reference converter writes for a real checkpoint
(``REF_CONV``): fp16 real-valued shared experts under ``layers.i.shared.*`` with no
int4 copy, a router-less dense-MLP layer, and one routed expert file absent.

Usage: python tests/golden/make_golden.py [reference_root]
"""

from __future__ import annotations

import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import oracle as orc  # noqa: E402
from wisp_b200 import converter as cv  # noqa: E402

MODELS = {
    "mx_small": dict(shape=cv.MoEShape(hidden=128, inter=256, n_experts=8, top_k=2, n_layers=2),
                     seed=1234, bias="random", T=4),
    "ds_small": dict(shape=cv.MoEShape(hidden=256, inter=128, n_experts=32, top_k=8, n_layers=2,
                                       shared_inter=128),
                     seed=77, bias="zipf", T=6),
    "gs32": dict(shape=cv.MoEShape(hidden=192, inter=96, n_experts=4, top_k=2, group_size=32,
                                   n_layers=1),
                 seed=5, bias=None, T=3),
}


# The reference-converter-form model: layer 0 dense MLP (384 rows), layers 1-2 MoE
# with an fp16 shared expert; the expert file of layer 1 that token 0 routes first
# is removed before the outputs are recorded.
REF_CONV = dict(shape=cv.MoEShape(hidden=256, inter=128, n_experts=16, top_k=4, n_layers=3,
                                  shared_inter=128),
                seed=4242, bias="random", T=5, dense_layers=[0], dense_inter=384)


def write_ref_conv(ref_root: Path, d: Path, spec: dict, missing=()):
    """REF_CONV written with the reference converter's own writers: expert blobs by
    ``write_expert_file`` on ``quantize_int4`` codes, the dense file by safetensors'
    ``save_file`` (what ``Partitioner`` uses), fp16 tensors under canonical names.
    The weights are drawn with this build's seeded recipe.  Returns the sha256 of
    every blob and of every dense tensor's bytes."""
    sys.path.insert(0, str(ref_root))
    from safetensors.torch import save_file
    from wisp.converter.partitioner import write_expert_file
    from wisp.converter.quantizer import quantize_int4
    shape, seed = spec["shape"], spec["seed"]
    # manifest and the dense tensors this build's writer would produce, then the
    # dense file rewritten by safetensors and the blobs by the reference
    cv.write_model_dir(d, shape, seed, router_bias=True, shared_form="fp16",
                       dense_layers=tuple(spec["dense_layers"]), dense_inter=spec["dense_inter"],
                       missing=[(l, e) for l in range(shape.n_layers)
                                for e in range(shape.n_experts)])
    from safetensors.torch import load_file
    dense = {k: v.clone() for k, v in
             load_file(str(d / "dense" / "model_dense.safetensors")).items()}
    tensors = {k: hashlib.sha256(v.contiguous().numpy().tobytes()).hexdigest()
               for k, v in dense.items()}
    save_file({k: v.contiguous() for k, v in dense.items()},
              str(d / "dense" / "model_dense.safetensors"))
    dims = {"gate_proj": (shape.inter, shape.hidden), "up_proj": (shape.inter, shape.hidden),
            "down_proj": (shape.hidden, shape.inter)}
    hashes = {}
    for l in range(shape.n_layers):
        if l in spec["dense_layers"]:
            continue
        for e in range(shape.n_experts):
            if (l, e) in missing:
                continue
            mats = {}
            for m, name in enumerate(("gate_proj", "up_proj", "down_proj")):
                g = torch.Generator().manual_seed(cv.expert_seed(seed, l, e, m, shape.n_experts))
                w = torch.randn(dims[name], generator=g) * 0.02
                mats[name] = quantize_int4(w, shape.group_size)
            p = d / "experts" / cv.expert_filename(l, e)
            write_expert_file(p, l, e, mats)
            hashes[p.name] = hashlib.sha256(p.read_bytes()).hexdigest()
    return hashes, tensors


def ref_conv_golden(ref_root: Path, arrays: dict) -> dict:
    spec = REF_CONV
    shape, seed, T = spec["shape"], spec["seed"], spec["T"]
    x = cv.make_input(shape, T, seed).numpy()
    with tempfile.TemporaryDirectory() as td:
        d = Path(td) / "ref_conv"
        write_ref_conv(ref_root, d, spec)
        ref = orc.RefEngine(d, threads=4)
        _, idx1, _ = ref.moe(1, x)
        ref.close()
        drop = (1, int(idx1[0, 0]))
    with tempfile.TemporaryDirectory() as td:
        d = Path(td) / "ref_conv"
        hashes, tensors = write_ref_conv(ref_root, d, spec, missing=[drop])
        ref = orc.RefEngine(d, threads=4)
        for l in range(shape.n_layers):
            y, idx, w = ref.moe(l, x)
            arrays.update({f"ref_conv.L{l}.y": y, f"ref_conv.L{l}.idx": idx,
                           f"ref_conv.L{l}.w": w})
        xs, sidx, sw = ref.stack(x, shape.n_layers)
        ref.close()
    arrays.update({"ref_conv.x": x, "ref_conv.stack_x": xs, "ref_conv.stack_idx": sidx,
                   "ref_conv.stack_w": sw})
    return {"shape": {k: getattr(shape, k) for k in ("hidden", "inter", "n_experts", "top_k",
                                                    "group_size", "n_layers", "shared_inter",
                                                    "rms_eps")},
            "seed": seed, "T": T, "dense_layers": spec["dense_layers"],
            "dense_inter": spec["dense_inter"], "missing": [list(drop)],
            "blob_sha256": hashes, "dense_sha256": tensors}


def write_with_reference(ref_root: Path, d: Path, shape: cv.MoEShape, seed: int, bias):
    sys.path.insert(0, str(ref_root))
    from wisp.converter.partitioner import write_expert_file
    from wisp.converter.quantizer import dequantize_int4, quantize_int4
    cv.write_model_dir(d, shape, seed, router_bias=(bias == "random"),
                       zipf_s=1.1 if bias == "zipf" else None)
    dims = {"gate_proj": (shape.inter, shape.hidden), "up_proj": (shape.inter, shape.hidden),
            "down_proj": (shape.hidden, shape.inter)}
    hashes = {}
    for l in range(shape.n_layers):
        for e in range(shape.n_experts):
            mats = {}
            for m, name in enumerate(("gate_proj", "up_proj", "down_proj")):
                g = torch.Generator().manual_seed(cv.expert_seed(seed, l, e, m, shape.n_experts))
                w = torch.randn(dims[name], generator=g) * 0.02
                mats[name] = quantize_int4(w, shape.group_size)
            p = d / "experts" / cv.expert_filename(l, e)
            write_expert_file(p, l, e, mats)
            hashes[p.name] = hashlib.sha256(p.read_bytes()).hexdigest()
        if shape.shared_inter:
            # the reference keeps shared experts fp16-dense: check our dense copy is
            # exactly the reference dequantisation of the same codes
            from safetensors.numpy import load_file
            dense = load_file(str(d / "dense" / "model_dense.safetensors"))
            s = cv.MoEShape(shape.hidden, shape.shared_inter, shape.n_experts + 1, shape.top_k,
                            shape.group_size)
            sdims = {"gate_proj": (s.inter, s.hidden), "up_proj": (s.inter, s.hidden),
                     "down_proj": (s.hidden, s.inter)}
            for m, name in enumerate(("gate_proj", "up_proj", "down_proj")):
                g = torch.Generator().manual_seed(cv.expert_seed(seed, l, shape.n_experts, m,
                                                                 s.n_experts))
                w = torch.randn(sdims[name], generator=g) * 0.02
                ref = dequantize_int4(quantize_int4(w, shape.group_size)).numpy()
                ours = dense[f"layers.{l}.shared.{name.split('_')[0]}"]
                assert np.array_equal(ref.view(np.uint16), ours.view(np.uint16)), name
    return hashes


def quantizer_cases(ref_root: Path) -> dict:
    sys.path.insert(0, str(ref_root))
    from wisp.converter.quantizer import quantize_int4
    out = {}
    cases = {"const_2x64": (torch.full((2, 64), 1.0), 64),
             "odd_7x9_gs16": (torch.randn(7, 9, generator=torch.Generator().manual_seed(3)), 16),
             "neg_3x64_gs32": (-torch.rand(3, 64, generator=torch.Generator().manual_seed(4)), 32)}
    for k, (w, gs) in cases.items():
        q = quantize_int4(w, gs)
        out[k] = {"shape": list(w.shape), "gs": gs, "weight": w.flatten().tolist(),
                  "packed": q.packed.numpy().tobytes().hex(),
                  "scales": q.scales.numpy().tobytes().hex(),
                  "zeros": q.zeros.numpy().tobytes().hex()}
    return out


def main(ref_root: Path) -> None:
    meta = {"models": {}, "quantizer": quantizer_cases(ref_root)}
    arrays = {}
    for name, spec in MODELS.items():
        shape, seed, T = spec["shape"], spec["seed"], spec["T"]
        with tempfile.TemporaryDirectory() as td:
            d = Path(td) / name
            hashes = write_with_reference(ref_root, d, shape, seed, spec["bias"])
            ref = orc.RefEngine(d, threads=4)
            x = cv.make_input(shape, T, seed).numpy()
            y, idx, w = ref.moe(0, x)
            xs, sidx, sw = ref.stack(x, shape.n_layers)
            ref.close()
        meta["models"][name] = {
            "shape": {k: getattr(shape, k) for k in ("hidden", "inter", "n_experts", "top_k",
                                                     "group_size", "n_layers", "shared_inter",
                                                     "rms_eps")},
            "seed": seed, "bias": spec["bias"], "T": T, "blob_sha256": hashes}
        arrays.update({f"{name}.x": x, f"{name}.y": y, f"{name}.idx": idx, f"{name}.w": w,
                       f"{name}.stack_x": xs, f"{name}.stack_idx": sidx, f"{name}.stack_w": sw})
    meta["ref_conv"] = ref_conv_golden(ref_root, arrays)
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1))
    np.savez_compressed(HERE / "golden_outputs.npz", **arrays)
    print("wrote", HERE / "golden.json", HERE / "golden_outputs.npz")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout root>")
    main(Path(sys.argv[1]))
