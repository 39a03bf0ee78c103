"""Int4 format contract: the restated quantiser and blob writer reproduce the
reference's bytes (golden hashes made with wisp/converter/quantizer.py and
partitioner.py), plus the reference's own format tests
(tests/test_adapters.py:392-493) restated against this package."""

import hashlib
import struct

import numpy as np
import pytest
import torch

from wisp_b200 import converter as cv


def test_quantizer_matches_reference_edge_cases(golden):
    meta, _ = golden
    for name, case in meta["quantizer"].items():
        w = torch.tensor(case["weight"], dtype=torch.float32).view(*case["shape"])
        q = cv.quantize_int4(w, case["gs"])
        assert q.packed.numpy().tobytes().hex() == case["packed"], name
        assert q.scales.numpy().tobytes().hex() == case["scales"], name
        assert q.zeros.numpy().tobytes().hex() == case["zeros"], name


def test_blobs_hash_match_reference(golden, golden_dirs):
    meta, _ = golden
    for name, spec in meta["models"].items():
        for fname, digest in spec["blob_sha256"].items():
            data = (golden_dirs[name] / "experts" / fname).read_bytes()
            assert hashlib.sha256(data).hexdigest() == digest, f"{name}/{fname}"


def test_roundtrip_error_is_small():
    torch.manual_seed(0)
    w = torch.randn(64, 128) * 0.02
    q = cv.quantize_int4(w, 64)
    err = (w - cv.dequantize_int4(q)).abs().max().item()
    step = (w.view(-1, 64).amax(1) - w.view(-1, 64).amin(1)) / 15
    assert err <= step.max().item() * 0.51 + 1e-6


def test_packing_low_nibble_first():
    q = cv.quantize_int4(torch.full((2, 64), 1.0), 64)
    assert q.packed[0].item() == 0x88
    assert torch.allclose(cv.dequantize_int4(q), torch.ones(2, 64), atol=1e-3)


def test_rejects_bad_input():
    with pytest.raises(ValueError):
        cv.quantize_int4(torch.randn(4), 64)
    with pytest.raises(ValueError):
        cv.quantize_int4(torch.randn(4, 4), 0)


def test_expert_blob_layout():
    torch.manual_seed(1)
    H, I, gs = 32, 16, 16
    mats = {"gate": cv.quantize_int4(torch.randn(I, H), gs), "up": cv.quantize_int4(torch.randn(I, H), gs),
            "down": cv.quantize_int4(torch.randn(H, I), gs)}
    blob = cv.expert_blob(3, 42, mats)
    assert cv.HEADER_BYTES == 120
    assert struct.unpack_from("<6I", blob) == (cv.EXPERT_MAGIC, 1, 3, 42, gs, 3)
    info = cv.parse_blob_header(blob)
    assert info["total_bytes"] == len(blob)
    for m, name in zip(info["mats"], cv.MAT_ORDER):
        assert (m["rows"], m["cols"]) == (mats[name].rows, mats[name].cols)
        assert m["packed_bytes"] == mats[name].packed.numel()


def test_incomplete_expert_rejected():
    q = cv.quantize_int4(torch.randn(8, 8), 8)
    with pytest.raises(ValueError, match="missing"):
        cv.expert_blob(0, 0, {"gate": q})


def test_truncated_blob_rejected():
    q = cv.quantize_int4(torch.randn(8, 64), 64)
    blob = cv.expert_blob(0, 0, {"gate": q, "up": q, "down": q})
    with pytest.raises(ValueError, match="truncated"):
        cv.parse_blob_header(blob[:-1])
    with pytest.raises(ValueError, match="corrupt"):
        cv.parse_blob_header(b"\0" * 120)


def test_mixtral_blob_size_constant():
    # reference measurement: 99,090,552 bytes per Mixtral int4 expert
    s = cv.MIXTRAL
    per = (s.inter * s.hidden) // 2 + 2 * 2 * (s.inter * s.hidden) // s.group_size
    assert cv.HEADER_BYTES + 3 * per == 99_090_552


def test_quantizer_same_bits_on_any_device_layout():
    # a non-contiguous view quantises the same as its contiguous copy
    w = torch.randn(64, 256) * 0.02
    a = cv.quantize_int4(w.t().contiguous().t(), 64)
    b = cv.quantize_int4(w.clone(), 64)
    assert torch.equal(a.packed, b.packed) and torch.equal(a.scales, b.scales)


@pytest.mark.parametrize("H,I,gs", [(128, 256, 64), (192, 96, 32), (512, 256, 128), (4096, 64, 64)])
def test_tiled_layout_round_trip(H, I, gs):
    """The tiled device layout is a pure permutation of each matrix region: untile
    restores the .bin bytes exactly; block b of a matrix holds, for group g, the
    gs/2 code bytes of rows 8b..8b+7 in order, then their (scale, zero) pairs."""
    shape = cv.MoEShape(hidden=H, inter=I, n_experts=2, top_k=1, group_size=gs)
    b = cv.expert_blob(0, 1, cv.make_expert(shape, 0, 1, 9))
    raw = np.frombuffer(b, dtype=np.uint8)
    t = cv.tile_blob(b)
    assert len(t) == len(raw) and cv.parse_blob_header(t.tobytes())["tiled"]
    assert np.array_equal(cv.untile_blob(t), raw)
    h = cv.parse_blob_header(b)
    for m in h["mats"]:
        R, Cc, G = m["rows"], m["cols"], m["cols"] // gs
        bb = 4 * Cc + 32 * G
        for (blk, g, j) in [(0, 0, 0), (R // 8 - 1, G - 1, 7), (R // 16, G // 2, 3)]:
            row = 8 * blk + j
            src = raw[m["packed_off"] + row * Cc // 2 + g * gs // 2:][:gs // 2]
            dst = t[m["packed_off"] + blk * bb + (g * 8 + j) * gs // 2:][:gs // 2]
            assert np.array_equal(src, dst)
            sz = t[m["packed_off"] + blk * bb + 4 * Cc + (g * 8 + j) * 4:][:4]
            assert np.array_equal(sz[:2], raw[m["scales_off"] + 2 * (row * G + g):][:2])
            assert np.array_equal(sz[2:], raw[m["zeros_off"] + 2 * (row * G + g):][:2])
