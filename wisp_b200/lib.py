"""ctypes binding of ``libwisp_b200.so`` (the C ABI declared in include/wisp_b200.h).

The library is built in-tree (``python -m wisp_b200.build``); importing this module
loads it and fails loudly if it is missing -- there is no Python or CPU stand-in
for any entry point.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("WISP_B200_LIB") or
               Path(__file__).resolve().parent / "_lib" / "libwisp_b200.so")

WISP_OK = 0
ERROR_NAMES = {0: "OK", 1: "OOM", 2: "IO", 3: "CUDA", 4: "INVALID_ARG", 5: "EXPERT_MISS",
               6: "MODEL", 7: "TIMEOUT"}


class WispErrCtx(C.Structure):
    _fields_ = [("code", C.c_int), ("message", C.c_char * 512), ("file", C.c_char_p),
                ("line", C.c_int)]


class WispExpertMeta(C.Structure):
    _fields_ = [("packed_off", C.c_size_t * 3), ("scales_off", C.c_size_t * 3),
                ("zeros_off", C.c_size_t * 3), ("rows", C.c_uint32 * 3),
                ("cols", C.c_uint32 * 3), ("group_size", C.c_uint32),
                ("total_bytes", C.c_size_t), ("valid", C.c_int), ("tiled", C.c_int)]


class WispAttnLayer(C.Structure):
    _fields_ = [("input_norm", C.c_void_p), ("q_proj", C.c_void_p), ("k_proj", C.c_void_p),
                ("v_proj", C.c_void_p), ("o_proj", C.c_void_p), ("hidden", C.c_int),
                ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float)]


class WispMoeLayer(C.Structure):
    _fields_ = [("meta", WispExpertMeta), ("expert_blobs", C.c_void_p), ("router_w", C.c_void_p),
                ("router_bias", C.c_void_p), ("norm_w", C.c_void_p), ("shared_blob", C.c_void_p),
                ("shared_meta", WispExpertMeta), ("n_experts", C.c_int), ("top_k", C.c_int),
                ("gating", C.c_int), ("shared_gate", C.c_void_p), ("shared_up", C.c_void_p),
                ("shared_down", C.c_void_p), ("shared_inter", C.c_int)]


class WispError(RuntimeError):
    """Raised with the reference's message format: ``wisp engine error [code]: msg (file:line)``."""

    def __init__(self, err: WispErrCtx, code: int | None = None):
        c = err.code if code is None else code
        msg = f"wisp engine error [{c}]: {err.message.decode(errors='replace')}"
        if err.file:
            msg += f" ({err.file.decode(errors='replace')}:{err.line})"
        super().__init__(msg)
        self.code = c


_lib: C.CDLL | None = None

_SIGS = {
    # fused block
    "wisp_moe_workspace_bytes": (C.c_size_t, [C.c_void_p, C.c_int, C.c_int]),
    "wisp_moe_block_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p,
                                         C.POINTER(WispErrCtx)]),
    "wisp_expert_tile": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.POINTER(WispErrCtx)]),
    "wisp_moe_experts_routed": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                          C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                          C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_moe_route": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                 C.c_void_p, C.c_size_t, C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_moe_ep_combine": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                      C.c_int, C.c_int, C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_moe_prefill_workspace_bytes": (C.c_size_t, [C.c_void_p, C.c_int]),
    "wisp_moe_prefill_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                           C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_moe_prefill_stack_workspace_bytes": (C.c_size_t, [C.c_void_p, C.c_int, C.c_int]),
    "wisp_moe_prefill_stack_forward": (C.c_int, [C.c_void_p, C.c_int, C.c_float, C.c_void_p,
                                                 C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                                 C.c_size_t, C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_stream_create": (C.c_void_p, [C.c_int, C.c_int, C.c_size_t, C.c_size_t,
                                        C.POINTER(WispErrCtx)]),
    "wisp_stream_destroy": (None, [C.c_void_p]),
    "wisp_stream_register": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                       C.POINTER(WispErrCtx)]),
    "wisp_stream_table": (C.c_void_p, [C.c_void_p, C.c_int]),
    "wisp_stream_ensure": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_stream_prefetch": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                       C.POINTER(WispErrCtx)]),
    "wisp_stream_layer_done": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p,
                                         C.POINTER(WispErrCtx)]),
    "wisp_stream_stats": (None, [C.c_void_p, C.c_void_p]),
    "wisp_stream_reset": (None, [C.c_void_p]),
    # the decoder step
    "wisp_kv_cache_alloc": (C.c_void_p, [C.c_void_p, C.c_int, C.POINTER(WispErrCtx)]),
    "wisp_kv_cache_free": (None, [C.c_void_p, C.c_void_p]),
    "wisp_kv_cache_clear": (None, [C.c_void_p, C.c_void_p]),
    "wisp_kv_cache_rollback": (None, [C.c_void_p, C.c_void_p, C.c_int]),
    "wisp_kv_cache_len": (C.c_int, [C.c_void_p]),
    "wisp_decode_one": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                  C.POINTER(WispErrCtx)]),
    "wisp_prefill": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                               C.POINTER(WispErrCtx)]),
    "wisp_verify_tokens": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                     C.POINTER(WispErrCtx)]),
    "wisp_engine_vocab": (C.c_int, [C.c_void_p]),
    "wisp_attn_workspace_bytes": (C.c_size_t, [C.c_void_p, C.c_int]),
    "wisp_attn_decode": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                   C.c_int, C.c_void_p, C.c_size_t, C.c_void_p,
                                   C.POINTER(WispErrCtx)]),
    "wisp_lm_head_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                       C.c_int, C.c_float, C.c_void_p, C.c_size_t, C.c_void_p,
                                       C.POINTER(WispErrCtx)]),
    "wisp_gpu_embed_lookup": (None, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p]),
    "wisp_gpu_rope": (None, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                             C.c_void_p]),
    "wisp_gpu_kv_append": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                  C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "wisp_gpu_attention": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                  C.c_void_p]),
    "wisp_moe_prefill_routed_workspace_bytes": (C.c_size_t, [C.c_void_p, C.c_int, C.c_int]),
    "wisp_moe_prefill_routed": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                          C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                          C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_moe_block_forward_static": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                                C.c_void_p, C.c_void_p, C.c_void_p,
                                                C.POINTER(WispErrCtx)]),
    "wisp_moe_block_static_status": (C.c_int, [C.c_void_p]),
    "wisp_moe_stack_forward": (C.c_int, [C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_int,
                                         C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                         C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_moe_block_route": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_size_t, C.c_void_p,
                                       C.POINTER(WispErrCtx)]),
    "wisp_moe_block_experts": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p,
                                         C.POINTER(WispErrCtx)]),
    "wisp_moe_status": (C.c_int, [C.c_void_p, C.c_void_p]),
    "wisp_moe_profile_events": (None, [C.c_void_p, C.c_int]),
    "wisp_moe_profile_count": (C.c_int, []),
    # reference launchers
    "wisp_gpu_gemv_f16": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "wisp_gpu_gemv_t_f16": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                   C.c_void_p]),
    "wisp_gpu_rmsnorm": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_float,
                                C.c_void_p]),
    "wisp_gpu_residual_add": (None, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "wisp_gpu_swiglu": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "wisp_gpu_swiglu_ffn": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                   C.c_int, C.c_void_p]),
    "wisp_gpu_scale_accum": (None, [C.c_void_p, C.c_void_p, C.c_float, C.c_int, C.c_void_p]),
    "wisp_gpu_router_topk": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                    C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "launch_dequant_expert": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                        C.c_int, C.c_void_p]),
    "async_load_expert": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "wisp_dense_ffn_workspace_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "wisp_dense_ffn_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                         C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_size_t,
                                         C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_quantize_int4": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_nccl_available": (C.c_int, []),
    "wisp_pipeline_init": (C.c_int, [C.c_void_p, C.c_int]),
    "wisp_pipeline_shutdown": (None, []),
    "wisp_pipeline_send_activation": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "wisp_pipeline_recv_activation": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "wisp_peer_enable": (C.c_int, [C.c_int, C.c_int]),
    "wisp_peer_copy_async": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_size_t,
                                       C.c_void_p]),
    # engine
    "wisp_expert_parse_header": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(WispExpertMeta),
                                           C.POINTER(WispErrCtx)]),
    "wisp_engine_create": (C.c_void_p, [C.c_char_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_int,
                                        C.c_int, C.POINTER(WispErrCtx)]),
    "wisp_engine_destroy": (None, [C.c_void_p]),
    "wisp_expert_fetch": (C.c_void_p, [C.c_void_p, C.c_uint32, C.c_uint32, C.POINTER(WispErrCtx)]),
    "wisp_read_expert_file": (C.c_size_t, [C.c_char_p, C.c_void_p, C.c_size_t,
                                           C.POINTER(C.c_int), C.POINTER(WispErrCtx)]),
    "wisp_expert_prefetch_hint": (None, [C.c_void_p, C.c_int, C.c_void_p, C.c_int]),
    "wisp_moe_forward": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                   C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_moe_decode": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                   C.c_void_p, C.POINTER(WispErrCtx)]),
    "wisp_moe_stack": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                 C.POINTER(WispErrCtx)]),
    "wisp_engine_pin_experts": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(WispErrCtx)]),
    "wisp_engine_stream": (C.c_void_p, [C.c_void_p]),
    "wisp_engine_dims": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "wisp_cache_stats": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "wisp_cache_clear_all": (None, [C.c_void_p]),
    "wisp_ram_trim": (C.c_int, [C.c_void_p, C.c_int]),
    "wisp_drain_expert_log": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "wisp_vram_used": (C.c_size_t, [C.c_void_p]),
    "wisp_ram_used": (C.c_size_t, [C.c_void_p]),
    "wisp_tok_per_sec": (C.c_double, [C.c_void_p]),
    "wisp_selftest_lru": (C.c_int, []),
    "wisp_selftest_double_buffer": (C.c_int, []),
    "wisp_debug_expert_probe": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.c_void_p,
                                          C.POINTER(WispExpertMeta), C.POINTER(WispErrCtx)]),
    "wisp_b200_version": (C.c_char_p, []),
}


def lib() -> C.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: run `python -m wisp_b200.build` "
                              "(there is no CPU fallback)")
        _lib = C.CDLL(str(LIB_PATH), mode=os.RTLD_LOCAL)
        for name, (res, args) in _SIGS.items():
            f = getattr(_lib, name)
            f.restype = res
            f.argtypes = args
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(rc: int, err: WispErrCtx) -> None:
    if rc != WISP_OK:
        raise WispError(err, rc)
