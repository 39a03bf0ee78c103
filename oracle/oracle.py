"""ctypes front-end of the CPU checkers (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs
use this module.  Two checkers:

* ``Port*`` -- ``moe_oracle.c``, the C restatement (works on in-memory blobs);
* ``RefEngine`` -- the reference engine's own CPU ``run_moe`` built from its
  sources (``oracle/_ref/libwisp_ref.so``); it reads a converted model directory.
"""

from __future__ import annotations

import ctypes as C
import json
import os
from pathlib import Path

import numpy as np

from . import build as _build

_port = None
_ref = None


def port_lib() -> C.CDLL:
    global _port
    if _port is None:
        _port = C.CDLL(str(_build.build_port()))
        f = _port.oracle_moe_block
        f.restype = C.c_int
        f.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                      C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                      C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        f = _port.oracle_stack
        f.restype = C.c_int
        f.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_int, C.c_int,
                      C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                      C.c_void_p, C.c_int]
        _port.oracle_router_topk.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                             C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        _port.oracle_rmsnorm.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_float]
        f = _port.oracle_experts_routed
        f.restype = C.c_int
        f.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                      C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                      C.c_void_p, C.c_int]
        f = _port.oracle_dense_ffn
        f.restype = C.c_int
        f.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                      C.c_int, C.c_void_p, C.c_int]
        f = _port.oracle_stack_layers
        f.restype = C.c_int
        f.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_int, C.c_int,
                      C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                      C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int]
        _port.oracle_dequant.argtypes = [C.c_void_p, C.c_int, C.c_long, C.c_void_p]
    return _port


def ref_lib() -> C.CDLL | None:
    global _ref
    if _ref is None:
        so = _build.build_ref()
        if so is None or not Path(so).exists():
            return None
        _ref = C.CDLL(str(so))
        _ref.ref_open.restype = C.c_void_p
        _ref.ref_open.argtypes = [C.c_char_p, C.c_ulonglong, C.c_int, C.c_char_p, C.c_int]
        _ref.ref_close.argtypes = [C.c_void_p]
        _ref.ref_moe.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                 C.c_void_p, C.c_void_p]
        _ref.ref_stack.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                   C.c_void_p, C.c_void_p]
        _ref.ref_probe.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_void_p]
        _ref.ref_cache_stats.argtypes = [C.c_void_p, C.c_void_p]
        _ref.ref_vocab.argtypes = [C.c_void_p]
        _ref.ref_decode.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
    return _ref


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def _ptr_array(arrs) -> np.ndarray:
    return np.array([0 if a is None else a.ctypes.data for a in arrs], dtype=np.uint64)


def host_threads() -> int:
    return len(os.sched_getaffinity(0))


class Model:
    """A converted model directory held in host memory.  An expert whose file is
    absent is held as None (the reference's fetch fails with WISP_ERR_IO and
    run_moe skips it); a layer without a router is a dense-MLP layer."""

    def __init__(self, path: str | Path):
        from safetensors.numpy import load_file
        self.path = Path(path)
        man = json.loads((self.path / "manifest.json").read_text())
        a = man["architecture"]
        self.n_layers = int(a["num_layers"])
        self.E = int(a["num_experts_per_layer"])
        self.k = int(a["top_k_routing"])
        self.H = int(a["hidden_size"])
        self.eps = float(a.get("rms_norm_eps", 1e-6))
        self.dense = {k: v.view(np.uint16) for k, v in
                      load_file(str(self.path / "dense" / "model_dense.safetensors")).items()}
        def blob(l, e):
            p = self.path / "experts" / f"L{l:03d}_E{e:05d}.bin"
            return np.fromfile(p, dtype=np.uint8) if p.exists() else None
        self.blobs = [[blob(l, e) for e in range(self.E)] for l in range(self.n_layers)]

    def is_dense(self, layer: int) -> bool:
        return self.d(f"layers.{layer}.router") is None

    def shared(self, layer: int):
        """(gate, up, down) fp16 bits of the layer's shared.* tensors, or None."""
        t = tuple(self.d(f"layers.{layer}.shared.{n}") for n in ("gate", "up", "down"))
        return None if any(a is None for a in t) else t

    def d(self, name: str):
        return self.dense.get(name)


def port_moe_block(m: Model, layer: int, x: np.ndarray, threads: int | None = None,
                   with_shared: bool = True):
    """The restated block on x [T,H] fp32 -> (y [T,H], idx [T,k], w [T,k]); a dense-MLP
    layer gives its FFN with idx -1 and w 0."""
    lib = port_lib()
    x = np.ascontiguousarray(x, dtype=np.float32)
    T = x.shape[0]
    y = np.zeros((T, m.H), np.float32)
    idx = np.zeros((T, m.k), np.int32)
    w = np.zeros((T, m.k), np.float32)
    if m.is_dense(layer):
        sg, su, sd = m.shared(layer)
        rc = lib.oracle_dense_ffn(_ptr(sg), _ptr(su), _ptr(sd), sg.shape[0], m.H, _ptr(x), T,
                                  _ptr(y), threads or host_threads())
        if rc:
            raise RuntimeError(f"oracle_dense_ffn failed: {rc}")
        idx[:] = -1
        return y, idx, w
    blobs = _ptr_array(m.blobs[layer])
    sg, su, sd = (m.d(f"layers.{layer}.shared.{n}") for n in ("gate", "up", "down"))
    si = sg.shape[0] if (sg is not None and with_shared) else 0
    rc = lib.oracle_moe_block(_ptr(m.d(f"layers.{layer}.router")),
                              _ptr(m.d(f"layers.{layer}.router_bias")), m.E, m.H, m.k,
                              _ptr(blobs), _ptr(sg) if si else None, _ptr(su) if si else None,
                              _ptr(sd) if si else None, si, _ptr(x), T, _ptr(y), _ptr(idx),
                              _ptr(w), threads or host_threads())
    if rc:
        raise RuntimeError(f"oracle_moe_block failed: {rc}")
    return y, idx, w


def port_moe_block_arrays(router_w: np.ndarray, router_bias: np.ndarray | None, blobs: list,
                          k: int, x: np.ndarray, threads: int | None = None, shared=None):
    """Same as ``port_moe_block`` on explicit arrays (fp16 bits as uint16, blob bytes);
    `shared` = (gate [I,H], up [I,H], down [H,I]) fp16 bits of a dense shared expert."""
    lib = port_lib()
    E, H = router_w.shape
    x = np.ascontiguousarray(x, dtype=np.float32)
    T = x.shape[0]
    y = np.zeros((T, H), np.float32)
    idx = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float32)
    bp = _ptr_array(blobs)
    sg = su = sd = None
    si = 0
    if shared is not None:
        sg, su, sd = (np.ascontiguousarray(a) for a in shared)
        si = sg.shape[0]
    rc = lib.oracle_moe_block(_ptr(router_w), _ptr(router_bias), E, H, k, _ptr(bp), _ptr(sg),
                              _ptr(su), _ptr(sd), si, _ptr(x), T, _ptr(y), _ptr(idx), _ptr(w),
                              threads or host_threads())
    if rc:
        raise RuntimeError(f"oracle_moe_block failed: {rc}")
    return y, idx, w


def port_experts_routed(blobs: list, H: int, idx: np.ndarray, w: np.ndarray, x: np.ndarray,
                        shared=None, threads: int | None = None) -> np.ndarray:
    """The expert half of the restated block on a given routing (idx/w [T,k]):
    y = [shared(x)] + sum_j w_j * E_idx_j(x), skipping idx < 0 and absent blobs."""
    lib = port_lib()
    x = np.ascontiguousarray(x, dtype=np.float32)
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    T, k = idx.shape
    y = np.zeros((T, H), np.float32)
    sg = su = sd = None
    si = 0
    if shared is not None:
        sg, su, sd = (np.ascontiguousarray(a) for a in shared)
        si = sg.shape[0]
    bp = _ptr_array(blobs)
    rc = lib.oracle_experts_routed(len(blobs), H, k, _ptr(bp), _ptr(sg), _ptr(su), _ptr(sd), si,
                                   _ptr(x), T, _ptr(idx), _ptr(w), _ptr(y),
                                   threads or host_threads())
    if rc:
        raise RuntimeError(f"oracle_experts_routed failed: {rc}")
    return y


def port_stack(m: Model, x: np.ndarray, layers: int | None = None, threads: int | None = None):
    """x <- x + moe_l(rmsnorm(x)) for l < layers -> (x_out, idx [T,L,k], w [T,L,k])."""
    lib = port_lib()
    L = layers or m.n_layers
    x = np.ascontiguousarray(x, dtype=np.float32)
    T = x.shape[0]
    out = np.empty_like(x)
    idx = np.zeros((T, L, m.k), np.int32)
    w = np.zeros((T, L, m.k), np.float32)
    rw = _ptr_array([m.d(f"layers.{l}.router") for l in range(L)])
    rb = [m.d(f"layers.{l}.router_bias") for l in range(L)]
    rbp = _ptr_array(rb) if any(b is not None for b in rb) else None
    nw = _ptr_array([m.d(f"layers.{l}.post_norm") for l in range(L)])
    bl = _ptr_array([b for l in range(L) for b in m.blobs[l]])
    sh = [m.shared(l) for l in range(L)]
    sg, su, sd = (_ptr_array([s[i] if s is not None else None for s in sh]) for i in range(3))
    si = np.array([s[0].shape[0] if s is not None else 0 for s in sh], dtype=np.int32)
    rc = lib.oracle_stack_layers(L, _ptr(rw), _ptr(rbp), _ptr(nw), m.eps, m.E, m.H, m.k,
                                 _ptr(bl), _ptr(sg), _ptr(su), _ptr(sd), _ptr(si), _ptr(x),
                                 _ptr(out), T, _ptr(idx), _ptr(w), threads or host_threads())
    if rc:
        raise RuntimeError(f"oracle_stack failed: {rc}")
    return out, idx, w


def port_router(router_w: np.ndarray, bias: np.ndarray | None, x: np.ndarray, k: int):
    """Router on one token -> (idx [k], w [k], probs [E])."""
    lib = port_lib()
    E, H = router_w.shape
    idx = np.zeros(k, np.int32)
    w = np.zeros(k, np.float32)
    p = np.zeros(E, np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    lib.oracle_router_topk(_ptr(router_w), _ptr(bias), _ptr(x), E, H, k, _ptr(idx), _ptr(w), _ptr(p))
    return idx, w, p


def port_dequant(blob: np.ndarray, mat: int, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    rc = port_lib().oracle_dequant(_ptr(blob), mat, n, _ptr(out))
    if rc:
        raise RuntimeError("oracle_dequant: bad blob")
    return out


class RefEngine:
    """The reference engine's CPU MoE path on a model directory."""

    def __init__(self, path: str | Path, threads: int | None = None, ram_budget: int | None = None):
        lib = ref_lib()
        if lib is None:
            raise RuntimeError("reference harness not built (oracle/_ref/libwisp_ref.so missing)")
        self.lib = lib
        man = json.loads((Path(path) / "manifest.json").read_text())
        a = man["architecture"]
        self.H = int(a["hidden_size"])
        self.k = int(a["top_k_routing"])
        if ram_budget is None:
            n = int(a["num_layers"]) * int(a["num_experts_per_layer"])
            ram_budget = (n + 1) * int(man["performance"]["expert_size_bytes"]) * 2
        err = C.create_string_buffer(600)
        self.h = lib.ref_open(str(path).encode(), ram_budget, threads or host_threads(), err, 600)
        if not self.h:
            raise RuntimeError(f"reference engine_create failed: {err.value.decode()}")

    def moe(self, layer: int, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        y = np.zeros((T, self.H), np.float32)
        idx = np.zeros((T, self.k), np.int32)
        w = np.zeros((T, self.k), np.float32)
        rc = self.lib.ref_moe(self.h, layer, _ptr(x), T, _ptr(y), _ptr(idx), _ptr(w))
        if rc:
            raise RuntimeError(f"reference run_moe failed: {rc}")
        return y, idx, w

    def stack(self, x: np.ndarray, n_layers: int, layer0: int = 0):
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        T = x.shape[0]
        idx = np.zeros((T, n_layers, self.k), np.int32)
        w = np.zeros((T, n_layers, self.k), np.float32)
        rc = self.lib.ref_stack(self.h, layer0, n_layers, _ptr(x), T, _ptr(idx), _ptr(w))
        if rc:
            raise RuntimeError(f"reference stack failed: {rc}")
        return x, idx, w

    def decode(self, tokens, max_seq: int) -> np.ndarray:
        """The reference decoder step for each token in turn from an empty KV cache:
        logits [n, vocab] (wisp_verify_tokens)."""
        ids = np.ascontiguousarray(tokens, dtype=np.int32)
        vocab = int(self.lib.ref_vocab(self.h))
        out = np.zeros((len(ids), vocab), np.float32)
        rc = self.lib.ref_decode(self.h, _ptr(ids), len(ids), max_seq, _ptr(out))
        if rc:
            raise RuntimeError(f"reference decode failed: {rc}")
        return out

    def cache_stats(self):
        out = np.zeros(3, np.uint64)
        self.lib.ref_cache_stats(self.h, _ptr(out))
        return tuple(int(v) for v in out)

    def close(self):
        if self.h:
            self.lib.ref_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ref_probe(path: str | Path, mat: int, n: int) -> np.ndarray:
    lib = ref_lib()
    out = np.zeros(n, np.float32)
    rc = lib.ref_probe(str(path).encode(), mat, n, _ptr(out))
    if rc:
        raise RuntimeError(f"reference probe failed: {rc}")
    return out
