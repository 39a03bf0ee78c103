"""Oversubscribed decode: the routed experts of a stack live in pinned host memory and
stream into a device cache (``wisp_stream_*`` in ``csrc/stream_cache.cpp``) -- the
configuration where the expert pool is larger than HBM.

Per layer and step (the FFN half of the reference's decode_step with attention as
identity, csrc/core/wisp_engine.c:1563-1570; tier policy after wisp_expert_fetch,
:891-1078):

1. ``x += y`` (previous layer), ``xn = rmsnorm(x)`` (reference launchers);
2. route (``wisp_moe_block_route``) and read the routed ids back (the reference also
   reads its top-k back to the host, :1424);
3. ``wisp_stream_ensure``: hits are touched, misses are copied from the pinned pool by
   ``cudaMemcpyAsync`` on the transfer streams; the compute stream waits on the copies;
4. lookahead: the *next* layer's router runs on this layer's ``xn`` (the residual stream
   changes little from one layer to the next) and its predicted experts are prefetched
   on the transfer streams while this layer's experts compute;
5. ``wisp_moe_block_experts`` (plan from the routing, gate/up, down, combine), then
   ``wisp_stream_layer_done`` so the slots it reads are not overwritten early.

With a ``tier_cache.ExpertPredictor`` passed to ``step``, each layer's routing is
recorded and the next layer's most frequent experts are prefetched beside the
router lookahead's; ``prewarm`` fills a cold cache from a ``LearningCache``'s hottest
experts (the reference's warm start).

The shared expert, routers and norms stay resident.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import converter as cv
from .lib import WispErrCtx, WispMoeLayer, check, lib
from .moe import MoEStack


class StreamingStack:
    """A seeded synthetic stack (the ``MoEStack`` recipe, layer for layer identical)
    whose routed experts are served from a pinned host pool through a device cache of
    `cache_slots` expert slots."""

    def __init__(self, shape: cv.MoEShape, seed: int, n_layers: int, cache_slots: int,
                 device="cuda", zipf_s: float | None = None, random_bias: bool = False):
        self.shape = shape
        self.device = torch.device(device)
        self.L = n_layers
        L = lib()
        err = WispErrCtx()
        self._keep = []
        self.host = []
        self._c = (WispMoeLayer * n_layers)()
        self.cache = None
        for l in range(n_layers):
            st = MoEStack(shape, seed, self.device, zipf_s=zipf_s, random_bias=random_bias,
                          n_layers=1, layer0=l)
            if self.cache is None:
                self.blob_bytes = st.blob_bytes
                self.cache = L.wisp_stream_create(n_layers, shape.n_experts, st.blob_bytes,
                                                  cache_slots, C.byref(err))
                if not self.cache:
                    check(err.code or 1, err)
            lw = st.layers[0]
            a = st.arena
            h = torch.empty(a.buf.numel(), dtype=torch.uint8, pin_memory=True)
            h.copy_(a.buf)
            self.host.append(h)
            for e, slot in enumerate(lw.slots):
                check(L.wisp_stream_register(self.cache, l, e,
                                             h.data_ptr() + slot * a.slot_bytes + 8,
                                             C.byref(err)), err)
            shared = None
            if lw.shared_slot is not None:
                o = lw.shared_slot * a.slot_bytes
                shared = a.buf[o:o + a.slot_bytes].clone()
            c = WispMoeLayer.from_buffer_copy(st.layer_c(0))
            c.expert_blobs = L.wisp_stream_table(self.cache, l)
            c.shared_blob = shared.data_ptr() + 8 if shared is not None else None
            self._c[l] = c
            self._keep.append((lw.router, lw.router_bias, lw.norm, shared))
            del st, a, lw
            torch.cuda.empty_cache()
        self.pool_bytes = n_layers * shape.n_experts * self.blob_bytes
        self._ws = self._pws = None
        self._T = 0

    def close(self):
        if self.cache:
            lib().wisp_stream_destroy(self.cache)
            self.cache = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _buffers(self, T: int):
        if self._T == T:
            return
        L = lib()
        K, H = self.shape.top_k, self.shape.hidden
        n = int(L.wisp_moe_workspace_bytes(C.byref(self._c), self.L, T))
        self._ws = torch.empty(n, dtype=torch.uint8, device=self.device)
        self._pws = torch.empty(n, dtype=torch.uint8, device=self.device)
        self._idx = torch.empty((T, K), dtype=torch.int32, device=self.device)
        self._w = torch.empty((T, K), dtype=torch.float32, device=self.device)
        self._pidx = torch.empty((T, K), dtype=torch.int32, device=self.device)
        self._pw = torch.empty((T, K), dtype=torch.float32, device=self.device)
        self._hidx = torch.empty((T, K), dtype=torch.int32, pin_memory=True)
        self._hpidx = torch.empty((T, K), dtype=torch.int32, pin_memory=True)
        self._xn = torch.empty((T, H), dtype=torch.float32, device=self.device)
        self._y = torch.empty((T, H), dtype=torch.float32, device=self.device)
        self._ev = torch.cuda.Event()
        self._pev = torch.cuda.Event()
        self._T = T

    def reset(self) -> None:
        """A cold cache: no expert resident, statistics zeroed."""
        torch.cuda.synchronize(self.device)
        lib().wisp_stream_reset(self.cache)

    def prewarm(self, pairs) -> int:
        """Copy the given (layer, expert) pairs into the cache, hottest first, at
        most one cache's worth; returns the experts copied."""
        L = lib()
        err = WispErrCtx()
        slots = self.stats()["slots"]
        by_layer: dict[int, list[int]] = {}
        for layer, e in list(pairs)[:slots]:
            if 0 <= layer < self.L and 0 <= e < self.shape.n_experts:
                by_layer.setdefault(layer, []).append(e)
        n = 0
        k = C.c_int(0)
        for layer, ids in by_layer.items():
            a = (C.c_int * len(ids))(*ids)
            check(L.wisp_stream_prefetch(self.cache, layer, a, len(ids), C.byref(k), C.byref(err)),
                  err)
            n += k.value
        torch.cuda.synchronize(self.device)
        return n

    def step(self, x: torch.Tensor, predict: bool = True, predictor=None) -> dict:
        """x <- x + MoE_l(rmsnorm(x)) for every layer, in place (current stream).
        Returns this step's demand hits / misses and prefetches issued."""
        L = lib()
        T, H = x.shape
        K = self.shape.top_k
        self._buffers(T)
        s = torch.cuda.current_stream(self.device)
        sp = s.cuda_stream
        err = WispErrCtx()
        hits = misses = issued = 0
        h, m, k = C.c_int(0), C.c_int(0), C.c_int(0)
        ws, pws = self._ws, self._pws
        for l in range(self.L):
            c = self._c[l]
            if l > 0:
                L.wisp_gpu_residual_add(x.data_ptr(), self._y.data_ptr(), T * H, sp)
            for t in range(T):
                L.wisp_gpu_rmsnorm(x[t].data_ptr(), c.norm_w, self._xn[t].data_ptr(), H,
                                   C.c_float(self.shape.rms_eps), sp)
            check(L.wisp_moe_block_route(C.byref(c), self._xn.data_ptr(), T,
                                         self._idx.data_ptr(), self._w.data_ptr(),
                                         ws.data_ptr(), ws.numel(), sp, C.byref(err)), err)
            self._hidx.copy_(self._idx, non_blocking=True)
            self._ev.record(s)
            self._ev.synchronize()
            check(L.wisp_stream_ensure(self.cache, l, self._hidx.data_ptr(), T * K, sp,
                                       C.byref(h), C.byref(m), C.byref(err)), err)
            hits += h.value
            misses += m.value
            if predictor is not None:
                predictor.observe(l, self._hidx.view(-1).tolist())
            ahead = predict and l + 1 < self.L
            if ahead:
                check(L.wisp_moe_route(C.byref(self._c[l + 1]), self._xn.data_ptr(), T,
                                       self._pidx.data_ptr(), self._pw.data_ptr(),
                                       pws.data_ptr(), pws.numel(), sp, C.byref(err)), err)
                self._hpidx.copy_(self._pidx, non_blocking=True)
                self._pev.record(s)
            check(L.wisp_moe_block_experts(C.byref(c), self._xn.data_ptr(), self._y.data_ptr(),
                                           T, self._idx.data_ptr(), self._w.data_ptr(),
                                           ws.data_ptr(), ws.numel(), sp, C.byref(err)), err)
            check(L.wisp_stream_layer_done(self.cache, l, sp, C.byref(err)), err)
            if ahead:
                self._pev.synchronize()
                check(L.wisp_stream_prefetch(self.cache, l + 1, self._hpidx.data_ptr(), T * K,
                                             C.byref(k), C.byref(err)), err)
                issued += k.value
                if predictor is not None:
                    freq = predictor.predict(l + 1)
                    if freq:
                        a = (C.c_int * len(freq))(*freq)
                        check(L.wisp_stream_prefetch(self.cache, l + 1, a, len(freq), C.byref(k),
                                                     C.byref(err)), err)
                        issued += k.value
        L.wisp_gpu_residual_add(x.data_ptr(), self._y.data_ptr(), T * H, sp)
        return {"hits": hits, "misses": misses, "prefetched": issued}

    def status(self) -> int:
        return int(lib().wisp_moe_status(self._ws.data_ptr(),
                                         torch.cuda.current_stream(self.device).cuda_stream))

    def stats(self) -> dict:
        out = (C.c_uint64 * 6)()
        lib().wisp_stream_stats(self.cache, out)
        return {"hits": out[0], "misses": out[1], "prefetched": out[2], "prefetch_used": out[3],
                "bytes": out[4], "slots": out[5]}
