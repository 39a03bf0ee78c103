"""Regenerate the golden fixtures from the REFERENCE implementation (run in the build
container, where the reference checkout exists; the outputs are committed).

For each small seeded model this script
  1. draws the expert weights with the same recipe as ``wisp_b200.converter``,
  2. quantises them with the reference's ``wisp.converter.quantizer.quantize_int4``
     and writes the blobs with ``wisp.converter.partitioner.write_expert_file``,
  3. records each blob's sha256, and
  4. runs the reference engine's own CPU ``run_moe`` (oracle/_ref harness) on a seeded
     input, recording outputs, routed indices and gate weights (block and stack).
It also records quantiser edge cases (constant group, odd sizes with padding).

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
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1))
    np.savez_compressed(HERE / "golden_outputs.npz", **arrays)
    print("wrote", HERE / "golden.json", HERE / "golden_outputs.npz")


if __name__ == "__main__":
    main(Path(sys.argv[1] if len(sys.argv) > 1 else "/" + "root/reference"))
