"""The decoder step on the GPU (wisp_b200/csrc/decoder.cu and the engine's
wisp_decode_one): against the reference's own decode_step logits (golden fixture made
by the reference harness), against the numpy restatements of its pieces
(oracle/decoder_oracle.py) at long caches and odd head layouts, and the KV-cache
bookkeeping of prefill / rollback / clear.

Tolerances: logits within max-abs 2e-2 and rel-L2 1e-2 of the reference (the north
star's output bound), with a tighter regression bound rel-L2 <= 2e-3, and the same
argmax wherever the reference's top two logits differ by more than 1e-3.  Kernels
against float64 restatements: relative error <= 1e-4 of the largest magnitude.
"""

import ctypes as C
import json
import math

import numpy as np
import pytest
import torch

from oracle import decoder_oracle as dor
from wisp_b200 import core
from wisp_b200.lib import WispAttnLayer, WispErrCtx, lib

pytestmark = pytest.mark.gpu

GOLD = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def _golden():
    return (json.loads((GOLD / "decode_golden.json").read_text()),
            dict(np.load(GOLD / "decode_golden.npz")))


def _write(tmp_path, name, spec, attention=True):
    from wisp_b200 import converter as cv
    return cv.write_model_dir(tmp_path / name, cv.MoEShape(**spec["shape"]), spec["seed"],
                              vocab=spec["vocab"],
                              attention=spec["attention"] if attention else None,
                              zipf_s=1.1 if spec["bias"] == "zipf" else None)


def _check_logits(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert np.abs(got - want).max() <= 2e-2
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel <= 2e-3, rel
    for g, w in zip(got, want):
        top2 = np.sort(w)[-2:]
        if top2[1] - top2[0] > 1e-3:
            assert g.argmax() == w.argmax()


@pytest.mark.parametrize("name", ["gqa", "mha_shared"])
def test_decode_matches_the_reference_decoder(cuda, tmp_path, name):
    meta, arrays = _golden()
    spec = meta[name]
    h = core.engine_create(str(_write(tmp_path, name, spec)), 1 << 30, 1 << 30, [0], 1)
    try:
        kv = core.kv_cache_alloc(h, spec["max_seq"])
        rows = core.verify_tokens(h, spec["tokens"], kv)
        assert core.kv_cache_len(kv) == len(spec["tokens"])
        _check_logits(rows, arrays[name])
        core.kv_cache_free(h, kv)
    finally:
        core.engine_destroy(h)


def test_prefill_rollback_clear_and_limits(cuda, tmp_path):
    meta, arrays = _golden()
    spec = meta["gqa"]
    toks = spec["tokens"]
    h = core.engine_create(str(_write(tmp_path, "gqa", spec)), 1 << 30, 1 << 30, [0], 1)
    try:
        kv = core.kv_cache_alloc(h, 16)
        rows = np.array(core.verify_tokens(h, toks[:4], kv))
        core.kv_cache_clear(h, kv)
        assert core.kv_cache_len(kv) == 0
        last = np.array(core.prefill(h, toks[:4], kv))
        np.testing.assert_array_equal(last, rows[3])  # same work, deterministic kernels
        core.kv_cache_rollback(h, kv, 2)
        assert core.kv_cache_len(kv) == 2
        np.testing.assert_array_equal(np.array(core.decode_one(h, toks[2], kv)), rows[2])
        core.kv_cache_clear(h, kv)
        np.testing.assert_array_equal(np.array(core.decode_one(h, toks[0], kv)), rows[0])
        with pytest.raises(RuntimeError, match=r"\[4\].*out of range"):
            core.decode_one(h, spec["vocab"], kv)
        core.kv_cache_free(h, kv)
        small = core.kv_cache_alloc(h, 2)
        core.decode_one(h, toks[0], small)
        core.decode_one(h, toks[1], small)
        with pytest.raises(RuntimeError, match=r"\[4\].*KV cache full"):
            core.decode_one(h, toks[2], small)
        core.kv_cache_free(h, small)
    finally:
        core.engine_destroy(h)


def test_moe_only_model_refuses_the_decoder(cuda, tmp_path):
    meta, _ = _golden()
    spec = meta["gqa"]
    h = core.engine_create(str(_write(tmp_path, "plain", spec, attention=False)), 1 << 30,
                           1 << 30, [0], 1)
    try:
        with pytest.raises(RuntimeError, match=r"\[6\].*attn\.q_proj"):
            core.kv_cache_alloc(h, 8)
    finally:
        core.engine_destroy(h)


def _dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).cuda()


@pytest.mark.parametrize("seq,nh,nkv,d", [(1, 4, 4, 64), (7, 8, 2, 128), (300, 16, 1, 64),
                                          (1500, 8, 2, 128), (700, 12, 4, 96)])
def test_attention_launcher_matches_the_restatement(cuda, seq, nh, nkv, d):
    rng = np.random.default_rng(seq + nh)
    q = rng.standard_normal(nh * d).astype(np.float32)
    K = rng.standard_normal((seq, nkv, d)).astype(np.float16)
    V = rng.standard_normal((seq, nkv, d)).astype(np.float16)
    scale = 1.0 / math.sqrt(d)
    qd, Kd, Vd = _dev(q, torch.float32), _dev(K, torch.float16), _dev(V, torch.float16)
    out = torch.zeros(nh * d, dtype=torch.float32, device="cuda")
    scratch = torch.zeros(nh * seq, dtype=torch.float32, device="cuda")
    lib().wisp_gpu_attention(qd.data_ptr(), Kd.data_ptr(), Vd.data_ptr(), out.data_ptr(),
                             scratch.data_ptr(), seq, nh, nkv, d, d, C.c_float(scale),
                             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    want = dor.attention(q, K, V, seq, nh, nkv, d, d, scale)
    got = out.cpu().numpy().astype(np.float64)
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()


@pytest.mark.parametrize("seq", [600, 2100])
def test_attention_launcher_with_values_aliased_to_keys(cuda, seq):
    """MLA's compressed cache: one kv head, k_dim 576, the value = the first 512 dims
    of the key (V == K), 16 query heads; 2100 positions take three chunks."""
    nh, kd, vd = 16, 576, 512
    rng = np.random.default_rng(seq)
    q = (rng.standard_normal(nh * kd) * 0.05).astype(np.float32)
    K = rng.standard_normal((seq, 1, kd)).astype(np.float16)
    qd, Kd = _dev(q, torch.float32), _dev(K, torch.float16)
    out = torch.zeros(nh * vd, dtype=torch.float32, device="cuda")
    scratch = torch.zeros(nh * seq, dtype=torch.float32, device="cuda")
    lib().wisp_gpu_attention(qd.data_ptr(), Kd.data_ptr(), Kd.data_ptr(), out.data_ptr(),
                             scratch.data_ptr(), seq, nh, 1, kd, vd, C.c_float(0.1),
                             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    want = dor.attention(q, K, None, seq, nh, 1, kd, vd, 0.1)
    got = out.cpu().numpy().astype(np.float64)
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()


@pytest.mark.parametrize("H,nh,nkv,pos", [(512, 8, 2, 0), (512, 8, 2, 517), (1024, 8, 8, 300),
                                          (384, 6, 2, 45)])  # the last: the non-tensor-core path
def test_attn_decode_layer_matches_the_restatement(cuda, H, nh, nkv, pos):
    hd, max_seq, eps, theta = H // nh, 600, 1e-5, 10000.0
    rng = np.random.default_rng(H + pos)
    w = {"input_norm": (1 + 0.1 * rng.standard_normal(H)).astype(np.float16),
         "q_proj": (rng.standard_normal((nh * hd, H)) * 0.5 / H ** 0.5).astype(np.float16),
         "k_proj": (rng.standard_normal((nkv * hd, H)) * 0.5 / H ** 0.5).astype(np.float16),
         "v_proj": (rng.standard_normal((nkv * hd, H)) / H ** 0.5).astype(np.float16),
         "o_proj": (rng.standard_normal((H, nh * hd)) * 0.5 / (nh * hd) ** 0.5).astype(np.float16)}
    x = rng.standard_normal(H).astype(np.float32)
    Kc = (rng.standard_normal((max_seq, nkv, hd)) * 2).astype(np.float16)
    Vc = rng.standard_normal((max_seq, nkv, hd)).astype(np.float16)
    want_x, want_K, want_V = dor.attn_layer(x, w, Kc, Vc, pos, nh, nkv, eps, theta)
    dw = {k: _dev(v, torch.float16) for k, v in w.items()}
    xd, Kd, Vd = _dev(x, torch.float32), _dev(Kc, torch.float16), _dev(Vc, torch.float16)
    L = WispAttnLayer(dw["input_norm"].data_ptr(), dw["q_proj"].data_ptr(),
                      dw["k_proj"].data_ptr(), dw["v_proj"].data_ptr(), dw["o_proj"].data_ptr(),
                      H, nh, nkv, hd, theta, eps)
    n = int(lib().wisp_attn_workspace_bytes(C.byref(L), max_seq))
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")  # zero before first use
    err = WispErrCtx()
    rc = lib().wisp_attn_decode(C.byref(L), xd.data_ptr(), Kd.data_ptr(), Vd.data_ptr(), pos,
                                max_seq, ws.data_ptr(), n,
                                torch.cuda.current_stream().cuda_stream, C.byref(err))
    assert rc == 0, err.message
    torch.cuda.synchronize()
    got = xd.cpu().numpy().astype(np.float64)
    assert np.abs(got - want_x).max() <= 1e-4 * np.abs(want_x).max()
    # the new cache row: fp16 of the rotated k (and of v), within one fp16 rounding
    kg = Kd.cpu().numpy().astype(np.float64)[pos]
    vg = Vd.cpu().numpy().astype(np.float64)[pos]
    kw = want_K.astype(np.float64)[pos]
    vw = want_V.astype(np.float64)[pos]
    assert np.abs(kg - kw).max() <= 2e-3 * max(1.0, np.abs(kw).max())
    assert np.abs(vg - vw).max() <= 2e-3 * max(1.0, np.abs(vw).max())
    # the other rows are untouched
    keep = np.ones(max_seq, bool)
    keep[pos] = False
    np.testing.assert_array_equal(Kd.cpu().numpy()[keep], Kc[keep])


def test_rope_kv_append_and_embedding_launchers(cuda):
    rng = np.random.default_rng(5)
    s = torch.cuda.current_stream().cuda_stream
    x = rng.standard_normal(3 * 40).astype(np.float32)
    xd = _dev(x, torch.float32)
    lib().wisp_gpu_rope(xd.data_ptr(), 3, 40, 8, 32, 77, C.c_float(10000.0), s)
    k = rng.standard_normal(2 * 16).astype(np.float32)
    v = rng.standard_normal(2 * 16).astype(np.float32)
    K = torch.zeros((4, 2, 16), dtype=torch.float16, device="cuda")
    V = torch.zeros((4, 2, 16), dtype=torch.float16, device="cuda")
    kd, vd = _dev(k, torch.float32), _dev(v, torch.float32)  # held until the kernels ran
    lib().wisp_gpu_kv_append(K.data_ptr(), V.data_ptr(), kd.data_ptr(), vd.data_ptr(), 2, 2, 16,
                             16, s)
    table = rng.standard_normal((10, 24)).astype(np.float16)
    td = _dev(table, torch.float16)
    emb = torch.zeros(24, dtype=torch.float32, device="cuda")
    lib().wisp_gpu_embed_lookup(td.data_ptr(), 7, emb.data_ptr(), 24, s)
    torch.cuda.synchronize()
    np.testing.assert_allclose(xd.cpu().numpy(), dor.rope(x, 3, 40, 8, 32, 77, 10000.0),
                               rtol=0, atol=1e-5)
    np.testing.assert_array_equal(K.cpu().numpy()[2].reshape(-1), k.astype(np.float16))
    np.testing.assert_array_equal(V.cpu().numpy()[2].reshape(-1), v.astype(np.float16))
    assert not K.cpu().numpy()[[0, 1, 3]].any()
    np.testing.assert_array_equal(emb.cpu().numpy(), table[7].astype(np.float32))
