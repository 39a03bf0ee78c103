"""The golden model written the way the reference converter writes a real
checkpoint (tests/golden/make_golden.py, REF_CONV): fp16 real-valued shared
experts under layers.i.shared.* with no int4 copy, a router-less dense-MLP
layer (layer 0), and one routed expert file absent (the reference's fetch fails
with WISP_ERR_IO and run_moe skips the expert, csrc/core/wisp_engine.c:1473-1477).

CPU checks: this package's writer reproduces those bytes, and the C restatement
reproduces the reference's recorded outputs (block per layer, 3-layer stack)."""

import hashlib

import numpy as np
from safetensors.numpy import load_file

from oracle import oracle as orc


def test_ref_conv_bytes_match_reference_writers(golden, ref_conv_dir):
    meta, _ = golden
    rc = meta["ref_conv"]
    for fname, digest in rc["blob_sha256"].items():
        data = (ref_conv_dir / "experts" / fname).read_bytes()
        assert hashlib.sha256(data).hexdigest() == digest, fname
    layer, expert = rc["missing"][0]
    assert not (ref_conv_dir / "experts" / f"L{layer:03d}_E{expert:05d}.bin").exists()
    assert not list((ref_conv_dir / "experts").glob("*_shared.bin"))
    dense = load_file(str(ref_conv_dir / "dense" / "model_dense.safetensors"))
    assert set(dense) == set(rc["dense_sha256"])
    for name, digest in rc["dense_sha256"].items():
        assert hashlib.sha256(np.ascontiguousarray(dense[name]).tobytes()).hexdigest() == \
            digest, name
    assert "layers.0.router" not in dense and "layers.0.shared.gate" in dense


def test_ref_conv_oracle_matches_reference_golden(golden, ref_conv_dir):
    meta, arr = golden
    rc = meta["ref_conv"]
    m = orc.Model(ref_conv_dir)
    x = arr["ref_conv.x"]
    for l in range(rc["shape"]["n_layers"]):
        y, idx, w = orc.port_moe_block(m, l, x)
        np.testing.assert_array_equal(idx, arr[f"ref_conv.L{l}.idx"])
        np.testing.assert_allclose(w, arr[f"ref_conv.L{l}.w"], rtol=0, atol=1e-7)
        np.testing.assert_allclose(y, arr[f"ref_conv.L{l}.y"], rtol=0, atol=1e-6)
    xs, sidx, sw = orc.port_stack(m, x)
    np.testing.assert_array_equal(sidx, arr["ref_conv.stack_idx"])
    np.testing.assert_allclose(xs, arr["ref_conv.stack_x"], rtol=0, atol=1e-5)
    # the skipped expert matters: token 0 routes it first in layer 1
    layer, expert = rc["missing"][0]
    assert arr[f"ref_conv.L{layer}.idx"][0, 0] == expert


def test_ref_conv_port_equals_reference_harness(golden, ref_conv_dir):
    """Bit for bit against the reference engine itself, where its harness is built."""
    import pytest
    if orc.ref_lib() is None:
        pytest.skip("reference harness not built here")
    meta, arr = golden
    m = orc.Model(ref_conv_dir)
    ref = orc.RefEngine(ref_conv_dir, threads=2)
    x = np.random.default_rng(3).standard_normal((3, m.H)).astype(np.float32)
    for l in range(m.n_layers):
        y0, i0, w0 = ref.moe(l, x)
        y1, i1, w1 = orc.port_moe_block(m, l, x)
        assert np.array_equal(i0, i1) and np.array_equal(w0, w1) and np.array_equal(y0, y1), l
    ref.close()
