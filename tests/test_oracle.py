"""The CPU checker itself, pinned: the C restatement (oracle/moe_oracle.c) must
reproduce the reference engine's run_moe outputs recorded in the golden fixtures
(block and 2-layer stack), and -- where the reference harness is built -- agree
with it bit for bit on fresh inputs."""

import numpy as np
import pytest

from oracle import oracle as orc
from wisp_b200 import converter as cv


@pytest.mark.parametrize("name", ["mx_small", "ds_small", "gs32"])
def test_port_matches_reference_golden(golden, golden_dirs, name):
    meta, arr = golden
    m = orc.Model(golden_dirs[name])
    x = arr[f"{name}.x"]
    y, idx, w = orc.port_moe_block(m, 0, x)
    np.testing.assert_array_equal(idx, arr[f"{name}.idx"])
    np.testing.assert_allclose(w, arr[f"{name}.w"], rtol=0, atol=1e-7)
    np.testing.assert_allclose(y, arr[f"{name}.y"], rtol=0, atol=1e-6)
    xs, sidx, sw = orc.port_stack(m, x)
    if meta["models"][name]["shape"]["shared_inter"] == 0:
        np.testing.assert_array_equal(sidx, arr[f"{name}.stack_idx"])
        np.testing.assert_allclose(xs, arr[f"{name}.stack_x"], rtol=0, atol=1e-5)


def test_port_bit_exact_with_reference_harness(golden_dirs):
    if orc.ref_lib() is None:
        pytest.skip("reference harness not built here")
    d = golden_dirs["mx_small"]
    m = orc.Model(d)
    ref = orc.RefEngine(d, threads=2)
    x = np.random.default_rng(9).standard_normal((5, m.H)).astype(np.float32) * 3
    y0, i0, w0 = ref.moe(1, x)
    y1, i1, w1 = orc.port_moe_block(m, 1, x)
    assert np.array_equal(i0, i1) and np.array_equal(w0, w1) and np.array_equal(y0, y1)
    ref.close()


def test_router_tie_break_lowest_index():
    # identical router rows -> identical probabilities -> lowest indices win
    E, H = 6, 32
    W = np.zeros((E, H), np.float16)
    W[:] = np.float16(0.01)
    W[4] = np.float16(0.02)
    idx, w, p = orc.port_router(W.view(np.uint16), None, np.ones(H, np.float32), 3)
    assert list(idx) == [4, 0, 1]
    assert abs(w.sum() - 1) < 1e-6


def test_dequant_matches_python(golden_dirs):
    m = orc.Model(golden_dirs["gs32"])
    blob = m.blobs[0][1]
    info = cv.parse_blob_header(blob.tobytes())
    got = orc.port_dequant(blob, 2, 500)
    mt = info["mats"][2]
    raw = blob.tobytes()
    q = cv.QMat(packed=__import__("torch").frombuffer(bytearray(raw[mt["packed_off"]:mt["scales_off"]]), dtype=__import__("torch").uint8),
                scales=__import__("torch").frombuffer(bytearray(raw[mt["scales_off"]:mt["zeros_off"]]), dtype=__import__("torch").float16),
                zeros=__import__("torch").frombuffer(bytearray(raw[mt["zeros_off"]:mt["zeros_off"] + mt["zeros_bytes"]]), dtype=__import__("torch").float16),
                rows=mt["rows"], cols=mt["cols"], group_size=info["group_size"])
    ref = cv.dequantize_int4(q).flatten()[:500].numpy()
    np.testing.assert_allclose(got, ref, rtol=0, atol=1e-7)
