"""Mirror of the reference's ``wisp._wisp_core`` module (csrc/bindings/wisp_bindings.cpp:66-404).

Same function names, argument order and meaning, integer engine handles, and
failures raised as ``RuntimeError("wisp engine error [code]: msg (file:line)")``.
The calls go through ``libwisp_b200.so``'s C ABI.

Coverage: the engine lifecycle, expert tiers, statistics, the expert access log,
prefetch hints, self-tests and the byte-layout probe behave as in the reference.
``prefill`` / ``decode_one`` / ``verify_tokens`` / ``kv_cache_*`` run the whole
decoder step on the GPU for GQA / MHA models (embedding, attention over an fp16 KV
cache, the MoE block, logits); a model without those weights, or with MLA
attention, raises ``wisp engine error [6]`` naming what is missing.
New entry points for the MoE path: ``moe_forward``, ``moe_stack``, ``pin_experts``,
``engine_stream``, ``engine_dims``.
"""

from __future__ import annotations

import ctypes as C
import threading

from .lib import WispErrCtx, WispExpertMeta, lib

__version__ = "1.0.0"
cuda_enabled = True

_registry: dict[int, int] = {}
_reg_lock = threading.Lock()
_next = [1]


def _raise(err: WispErrCtx, code: int | None = None):
    c = err.code if code is None else code
    msg = f"wisp engine error [{c}]: {err.message.decode(errors='replace')}"
    if err.file:
        msg += f" ({err.file.decode(errors='replace')}:{err.line})"
    raise RuntimeError(msg)


def _engine(handle: int) -> int:
    with _reg_lock:
        p = _registry.get(handle)
    if p is None:
        raise ValueError(f"invalid wisp engine handle {handle}")
    return p


def engine_create(model_path: str, vram_expert_budget_bytes: int, ram_expert_budget_bytes: int,
                  gpu_indices: list[int], omp_threads: int) -> int:
    err = WispErrCtx()
    idx = (C.c_int * max(1, len(gpu_indices)))(*gpu_indices)
    p = lib().wisp_engine_create(model_path.encode(), max(0, int(vram_expert_budget_bytes)),
                                 max(0, int(ram_expert_budget_bytes)), idx, len(gpu_indices),
                                 int(omp_threads), C.byref(err))
    if not p:
        _raise(err)
    with _reg_lock:
        h = _next[0]
        _next[0] += 1
        _registry[h] = p
    return h


def engine_destroy(handle: int) -> None:
    with _reg_lock:
        p = _registry.pop(handle, None)
    if p:
        lib().wisp_engine_destroy(p)


def cache_stats(handle: int) -> dict:
    v, r, s = C.c_uint64(), C.c_uint64(), C.c_uint64()
    rate = C.c_double()
    lib().wisp_cache_stats(_engine(handle), C.byref(v), C.byref(r), C.byref(s), C.byref(rate))
    return {"vram_hits": v.value, "ram_hits": r.value, "ssd_hits": s.value, "hit_rate": rate.value}


def cache_clear(handle: int) -> None:
    lib().wisp_cache_clear_all(_engine(handle))


def ram_trim(handle: int, count: int) -> int:
    return int(lib().wisp_ram_trim(_engine(handle), count))


def drain_expert_log(handle: int, max_entries: int = 0) -> dict:
    if max_entries <= 0:
        max_entries = 1 << 16
    buf = (C.c_uint32 * max_entries)()
    dropped = C.c_uint64()
    n = lib().wisp_drain_expert_log(_engine(handle), buf, max_entries, C.byref(dropped))
    return {"hits": [(int(buf[i] >> 16), int(buf[i] & 0xFFFF)) for i in range(n)],
            "dropped": dropped.value}


def expert_prefetch_hint(handle: int, layer_idx: int, expert_ids: list[int]) -> None:
    arr = (C.c_int * max(1, len(expert_ids)))(*expert_ids)
    lib().wisp_expert_prefetch_hint(_engine(handle), layer_idx, arr, len(expert_ids))


def get_vram_used_bytes(handle: int) -> int:
    return int(lib().wisp_vram_used(_engine(handle)))


def get_ram_used_bytes(handle: int) -> int:
    return int(lib().wisp_ram_used(_engine(handle)))


def get_tok_per_sec(handle: int) -> float:
    return float(lib().wisp_tok_per_sec(_engine(handle)))


def _selftest_lru() -> bool:
    return lib().wisp_selftest_lru() == 1


def _selftest_double_buffer() -> bool:
    return lib().wisp_selftest_double_buffer() == 1


def _debug_expert_probe(path: str, mat: int, n: int) -> dict:
    vals = (C.c_float * max(1, n))()
    meta = WispExpertMeta()
    err = WispErrCtx()
    rc = lib().wisp_debug_expert_probe(path.encode(), mat, n, vals, C.byref(meta), C.byref(err))
    if rc != 0:
        _raise(err, rc)
    total = meta.rows[mat] * meta.cols[mat]
    k = min(n, total)
    return {"rows": [int(meta.rows[i]) for i in range(3)],
            "cols": [int(meta.cols[i]) for i in range(3)],
            "group_size": int(meta.group_size), "total_bytes": int(meta.total_bytes),
            "values": [float(vals[i]) for i in range(k)]}


# ---------------------------------------------------------------- MoE path (new)
def moe_forward(handle: int, layer: int, x_ptr: int, y_ptr: int, n_tokens: int,
                stream: int = 0) -> None:
    """y[T,H] = MoE_layer(x[T,H]); device pointers, on `stream` (0 = engine stream)."""
    err = WispErrCtx()
    rc = lib().wisp_moe_forward(_engine(handle), layer, x_ptr, y_ptr, n_tokens, stream or None,
                                C.byref(err))
    if rc != 0:
        _raise(err, rc)


def moe_decode(handle: int, layer: int, x_ptr: int, y_ptr: int, stream: int = 0) -> None:
    """y[H] = MoE_layer(x[H]) for one token (``wisp_moe_decode``); device pointers."""
    err = WispErrCtx()
    rc = lib().wisp_moe_decode(_engine(handle), layer, x_ptr, y_ptr, stream or None,
                               C.byref(err))
    if rc != 0:
        _raise(err, rc)


def moe_stack(handle: int, layer0: int, n_layers: int, x_ptr: int, n_tokens: int,
              stream: int = 0) -> None:
    """x <- x + MoE_l(rmsnorm(x)) for layers [layer0, layer0 + n_layers), in place."""
    err = WispErrCtx()
    rc = lib().wisp_moe_stack(_engine(handle), layer0, n_layers, x_ptr, n_tokens, stream or None,
                              C.byref(err))
    if rc != 0:
        _raise(err, rc)


def pin_experts(handle: int, layer0: int, n_layers: int) -> int:
    err = WispErrCtx()
    return int(lib().wisp_engine_pin_experts(_engine(handle), layer0, n_layers, C.byref(err)))


def engine_stream(handle: int) -> int:
    return int(lib().wisp_engine_stream(_engine(handle)) or 0)


def engine_dims(handle: int) -> dict:
    h, e, k, l = C.c_int(), C.c_int(), C.c_int(), C.c_int()
    lib().wisp_engine_dims(_engine(handle), C.byref(h), C.byref(e), C.byref(k), C.byref(l))
    return {"hidden": h.value, "n_experts": e.value, "top_k": k.value, "n_layers": l.value}


# --- the decoder step (wisp_bindings.cpp:115-218): KV caches are integer
# handles in a registry, logits come back as Python lists of vocab floats.
_kv: dict[int, int] = {}
_next_kv = [1]


def _kv_of(kv_cache_ptr: int) -> int:
    with _reg_lock:
        p = _kv.get(kv_cache_ptr)
    if p is None:
        raise ValueError(f"invalid kv cache handle {kv_cache_ptr}")
    return p


def _vocab(handle: int) -> int:
    return int(lib().wisp_engine_vocab(_engine(handle)))


def kv_cache_alloc(handle: int, max_seq_len: int) -> int:
    err = WispErrCtx()
    p = lib().wisp_kv_cache_alloc(_engine(handle), int(max_seq_len), C.byref(err))
    if not p:
        _raise(err)
    with _reg_lock:
        h = _next_kv[0]
        _next_kv[0] += 1
        _kv[h] = p
    return h


def kv_cache_free(handle: int, kv_cache_ptr: int) -> None:
    with _reg_lock:
        p = _kv.pop(kv_cache_ptr, None)
    if p is not None:
        lib().wisp_kv_cache_free(_engine(handle), p)


def kv_cache_clear(handle: int, kv_cache_ptr: int) -> None:
    lib().wisp_kv_cache_clear(_engine(handle), _kv_of(kv_cache_ptr))


def kv_cache_rollback(handle: int, kv_cache_ptr: int, n_tokens: int) -> None:
    lib().wisp_kv_cache_rollback(_engine(handle), _kv_of(kv_cache_ptr), int(n_tokens))


def kv_cache_len(kv_cache_ptr: int) -> int:
    """New: positions held by the cache."""
    return int(lib().wisp_kv_cache_len(_kv_of(kv_cache_ptr)))


def prefill(handle: int, token_ids: list[int], kv_cache_ptr: int) -> list[float]:
    e, kv = _engine(handle), _kv_of(kv_cache_ptr)
    ids = (C.c_int * max(1, len(token_ids)))(*token_ids)
    out = (C.c_float * max(1, _vocab(handle)))()
    err = WispErrCtx()
    rc = lib().wisp_prefill(e, ids, len(token_ids), kv, out, C.byref(err))
    if rc:
        _raise(err, rc)
    return list(out)


def decode_one(handle: int, token_id: int, kv_cache_ptr: int) -> list[float]:
    e, kv = _engine(handle), _kv_of(kv_cache_ptr)
    out = (C.c_float * max(1, _vocab(handle)))()
    err = WispErrCtx()
    rc = lib().wisp_decode_one(e, int(token_id), kv, out, C.byref(err))
    if rc:
        _raise(err, rc)
    return list(out)


def verify_tokens(handle: int, token_ids: list[int], kv_cache_ptr: int) -> list[list[float]]:
    e, kv = _engine(handle), _kv_of(kv_cache_ptr)
    n, vocab = len(token_ids), _vocab(handle)
    ids = (C.c_int * max(1, n))(*token_ids)
    flat = (C.c_float * max(1, n * vocab))()
    err = WispErrCtx()
    rc = lib().wisp_verify_tokens(e, ids, n, kv, flat, C.byref(err))
    if rc:
        _raise(err, rc)
    return [list(flat[i * vocab:(i + 1) * vocab]) for i in range(n)]
