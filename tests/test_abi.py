"""C ABI of libwisp_b200.so on a machine without a GPU: the library loads, exports
every entry point include/wisp_b200.h declares, its host-only self-tests pass, the
byte-layout probe agrees with the Python packer (the reference's
test_c_engine_reads_python_packed_expert, tests/test_adapters.py:453-487), and
argument validation fails with the reference's error codes before any GPU work."""

import ctypes as C
import re
import subprocess

import pytest
import torch

from wisp_b200 import converter as cv
from wisp_b200 import core
from wisp_b200.lib import LIB_PATH, WispErrCtx, WispMoeLayer, exported_symbols, lib

HEADER = LIB_PATH.parents[2] / "include" / "wisp_b200.h"


def declared_functions() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    names = set()
    for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M):
        if not m.group(0).lstrip().startswith(("typedef", "#", "return")):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol(built_lib):
    declared = declared_functions()
    assert len(declared) >= 35
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = declared - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    assert declared <= set(exported_symbols()) | {"wisp_b200_version"}


def test_version_and_selftests(built_lib):
    from wisp_b200 import build
    v = lib().wisp_b200_version().decode()
    assert "sm_100a" in v and v.endswith("src:" + build.source_hash())
    assert core._selftest_lru() is True
    for _ in range(5):
        assert core._selftest_double_buffer() is True


@pytest.mark.parametrize("gs,H,I", [(16, 32, 16), (64, 128, 64), (32, 96, 64)])
def test_probe_reads_python_packed_expert(built_lib, tmp_path, gs, H, I):
    torch.manual_seed(7)
    mats = {"gate": cv.quantize_int4(torch.randn(I, H), gs), "up": cv.quantize_int4(torch.randn(I, H), gs),
            "down": cv.quantize_int4(torch.randn(H, I), gs)}
    p = tmp_path / cv.expert_filename(5, 123)
    p.write_bytes(cv.expert_blob(5, 123, mats))
    for i, name in enumerate(cv.MAT_ORDER):
        probe = core._debug_expert_probe(str(p), i, 64)
        q = mats[name]
        assert probe["rows"][i] == q.rows and probe["cols"][i] == q.cols
        assert probe["group_size"] == gs and probe["total_bytes"] == p.stat().st_size
        vals = torch.tensor(probe["values"])
        ref = cv.dequantize_int4(q).flatten()[:len(vals)]
        assert torch.allclose(vals, ref, atol=1e-6)


def test_probe_errors_use_reference_format(built_lib, tmp_path):
    with pytest.raises(RuntimeError, match=r"wisp engine error \[2\]"):
        core._debug_expert_probe(str(tmp_path / "missing.bin"), 0, 4)
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"\0" * 200)
    with pytest.raises(RuntimeError, match=r"wisp engine error \[6\].*corrupt"):
        core._debug_expert_probe(str(bad), 0, 4)
    with pytest.raises(RuntimeError, match=r"\[4\]"):
        core._debug_expert_probe(str(bad), 3, 4)


def test_engine_requires_gpu_index(built_lib, tmp_path):
    with pytest.raises(RuntimeError, match=r"wisp engine error \[4\]"):
        core.engine_create(str(tmp_path), 0, 0, [], 1)


def _layer(H=128, I=256, E=8, K=2, gs=64):
    from wisp_b200.moe import blob_header, parse_meta
    mats = {n: cv.quantize_int4(torch.zeros(r, c), gs)
            for n, (r, c) in {"gate": (I, H), "up": (I, H), "down": (H, I)}.items()}
    total = cv.HEADER_BYTES + sum(sum(q.section_bytes()) for q in mats.values())
    L = WispMoeLayer()
    L.meta = parse_meta(blob_header(0, 0, mats), total)
    L.expert_blobs = 16
    L.router_w = 16
    L.n_experts, L.top_k = E, K
    return L


def test_workspace_size_grows_with_tokens(built_lib):
    L = _layer()
    a = lib().wisp_moe_workspace_bytes(C.byref(L), 1, 1)
    b = lib().wisp_moe_workspace_bytes(C.byref(L), 1, 16)
    assert 0 < a < b


@pytest.mark.parametrize("kw,msg", [({"gs": 16, "H": 128, "I": 256}, "unsupported shape"),
                                    ({"K": 9}, "top_k"), ({"H": 100, "gs": 4}, "unsupported")])
def test_block_forward_rejects_bad_layers(built_lib, kw, msg):
    L = _layer(**kw)
    err = WispErrCtx()
    rc = lib().wisp_moe_block_forward(C.byref(L), 256, 512, 1, None, None, 1024, 1 << 30, None,
                                      C.byref(err))
    assert rc == 4 and msg in err.message.decode()


def test_core_mirror_surface():
    for name in ("engine_create", "engine_destroy", "cache_stats", "cache_clear", "ram_trim",
                 "drain_expert_log", "expert_prefetch_hint", "get_vram_used_bytes",
                 "get_ram_used_bytes", "get_tok_per_sec", "_selftest_lru",
                 "_selftest_double_buffer", "_debug_expert_probe", "prefill", "decode_one",
                 "verify_tokens", "kv_cache_alloc", "kv_cache_free", "kv_cache_clear",
                 "kv_cache_rollback", "moe_forward", "moe_stack"):
        assert callable(getattr(core, name)), name
    assert core.__version__ and core.cuda_enabled is True
    # unknown handles are refused before any engine call, as in the reference
    with pytest.raises(ValueError, match="invalid wisp engine handle"):
        core.decode_one(123456, 0, 0)
