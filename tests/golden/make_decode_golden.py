"""Writes tests/golden/decode_golden.json and decode_golden.npz: the logits of the
reference engine's whole decoder step (decode_step, csrc/core/wisp_engine.c:1537-1595,
run through wisp_verify_tokens on its CPU path) for a few tokens from an empty KV cache,
on synthetic GQA / MHA model directories written by wisp_b200.converter.  The dense
file's SHA-256 is recorded so a test can check it regenerated the same weights.

Run once in a container whose reference harness is built from the reference's sources
(python oracle/build.py with WISP_REFERENCE_ROOT set); the GPU boxes only read the
committed files."""

import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

MODELS = {
    # GQA: 4 query heads over 2 kv heads (head_dim 64), top-2 of 8 experts
    "gqa": {"shape": {"hidden": 256, "inter": 256, "n_experts": 8, "top_k": 2, "n_layers": 2},
            "seed": 7, "vocab": 64, "attention": {"n_heads": 4, "n_kv_heads": 2, "max_pos": 64},
            "bias": None, "tokens": [3, 17, 5, 60, 9, 33], "max_seq": 32},
    # MHA (8 heads, head_dim 64), an int4 shared expert, Zipf-biased routing over 16
    "mha_shared": {"shape": {"hidden": 512, "inter": 128, "n_experts": 16, "top_k": 4,
                             "n_layers": 3, "shared_inter": 256},
                   "seed": 11, "vocab": 96,
                   "attention": {"n_heads": 8, "n_kv_heads": 8, "max_pos": 64,
                                 "rope_theta": 500000.0},
                   "bias": "zipf", "tokens": [95, 0, 41, 41, 7, 88, 12], "max_seq": 16},
}


def write(d: Path, spec: dict) -> Path:
    from wisp_b200 import converter as cv
    return cv.write_model_dir(d, cv.MoEShape(**spec["shape"]), spec["seed"], vocab=spec["vocab"],
                              attention=spec["attention"],
                              zipf_s=1.1 if spec["bias"] == "zipf" else None)


def dense_sha(d: Path) -> str:
    return hashlib.sha256((d / "dense" / "model_dense.safetensors").read_bytes()).hexdigest()


def main() -> None:
    from oracle import oracle as orc
    meta, arrays = {}, {}
    for name, spec in MODELS.items():
        d = Path(tempfile.mkdtemp()) / name
        write(d, spec)
        ref = orc.RefEngine(d)
        arrays[name] = ref.decode(spec["tokens"], spec["max_seq"])
        ref.close()
        meta[name] = dict(spec, dense_sha256=dense_sha(d))
    (HERE / "decode_golden.json").write_text(json.dumps(meta, indent=1) + "\n")
    np.savez_compressed(HERE / "decode_golden.npz", **arrays)
    for name, a in arrays.items():
        print(name, a.shape, "argmax", a.argmax(1).tolist())


if __name__ == "__main__":
    main()
