"""The decoder step around the MoE block, CPU side: the converted model directories
with attention weights, the golden logits of the reference's own decode_step and the
numpy restatements the GPU tests check the kernels against."""

import hashlib
import json
import math

import numpy as np
import pytest

from oracle import decoder_oracle as dor
from oracle import oracle as orc

GOLD = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def _golden():
    meta = json.loads((GOLD / "decode_golden.json").read_text())
    arrays = dict(np.load(GOLD / "decode_golden.npz"))
    return meta, arrays


def _write(tmp_path, name, spec):
    from wisp_b200 import converter as cv
    return cv.write_model_dir(tmp_path / name, cv.MoEShape(**spec["shape"]), spec["seed"],
                              vocab=spec["vocab"], attention=spec["attention"],
                              zipf_s=1.1 if spec["bias"] == "zipf" else None)


@pytest.mark.parametrize("name", ["gqa", "mha_shared"])
def test_converter_regenerates_the_golden_weights(tmp_path, name):
    meta, arrays = _golden()
    d = _write(tmp_path, name, meta[name])
    sha = hashlib.sha256((d / "dense" / "model_dense.safetensors").read_bytes()).hexdigest()
    assert sha == meta[name]["dense_sha256"]
    man = json.loads((d / "manifest.json").read_text())["architecture"]
    assert man["attention_type"] == "GQA"
    assert man["num_attention_heads"] == meta[name]["attention"]["n_heads"]
    assert arrays[name].shape == (len(meta[name]["tokens"]), meta[name]["vocab"])


@pytest.mark.parametrize("name", ["gqa", "mha_shared"])
def test_reference_decoder_reproduces_the_golden_logits(tmp_path, name):
    """The live reference harness (its decode_step on the CPU) gives the committed
    logits again: the fixture and the checker agree."""
    if orc.ref_lib() is None:
        pytest.skip("reference harness not built")
    meta, arrays = _golden()
    spec = meta[name]
    ref = orc.RefEngine(_write(tmp_path, name, spec), threads=4)
    got = ref.decode(spec["tokens"], spec["max_seq"])
    ref.close()
    np.testing.assert_allclose(got, arrays[name], rtol=0, atol=1e-6)


def test_reference_decoder_rejects_out_of_range_tokens(tmp_path):
    if orc.ref_lib() is None:
        pytest.skip("reference harness not built")
    meta, _ = _golden()
    spec = meta["gqa"]
    ref = orc.RefEngine(_write(tmp_path, "gqa", spec), threads=2)
    with pytest.raises(RuntimeError, match="decode failed"):
        ref.decode([spec["vocab"]], 4)
    ref.close()


def test_attention_restatement_matches_a_direct_softmax():
    """The numpy restatement against an independent formulation (GQA, 3 heads per
    kv head, a single position and a long cache)."""
    rng = np.random.default_rng(3)
    nh, nkv, d = 6, 2, 16
    for seq in (1, 37):
        q = rng.standard_normal(nh * d)
        K = rng.standard_normal((seq, nkv, d)).astype(np.float16)
        V = rng.standard_normal((seq, nkv, d)).astype(np.float16)
        out = dor.attention(q, K, V, seq, nh, nkv, d, d, 0.25).reshape(nh, d)
        for h in range(nh):
            s = K[:, h // 3, :].astype(np.float64) @ q.reshape(nh, d)[h] * 0.25
            p = np.exp(s) / np.exp(s).sum()
            np.testing.assert_allclose(out[h], p @ V[:, h // 3, :].astype(np.float64), rtol=1e-12)


def test_rope_restatement_rotates_pairs():
    v = np.arange(8, dtype=np.float64) + 1
    r = dor.rope(v, 1, 8, 0, 8, 3, 10000.0)
    # each pair (i, i+4) keeps its norm and turns by pos * theta^(-2i/8)
    for i in range(4):
        a = math.atan2(r[i + 4], r[i]) - math.atan2(v[i + 4], v[i])
        want = 3 * 10000.0 ** (-2 * i / 8)
        assert abs(math.remainder(a - want, 2 * math.pi)) < 1e-9
        assert abs(math.hypot(r[i], r[i + 4]) - math.hypot(v[i], v[i + 4])) < 1e-12
