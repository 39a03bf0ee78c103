"""Device-resident MoE layers and stacks over the fused C ABI.

``ExpertArena`` holds int4 expert blobs in the WISP ``.bin`` layout on the GPU, each
at ``slot * slot_bytes + 8`` so its packed/scales/zeros sections start 16-byte
aligned.  ``MoEStack`` owns per-layer routers, norm weights and the device table of
blob pointers, and calls ``wisp_moe_block_forward`` / ``wisp_moe_stack_forward``
on the caller's current CUDA stream.  torch is used for device memory and streams
only; every kernel is in ``libwisp_b200.so``.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import converter as cv
from .lib import WispErrCtx, WispExpertMeta, WispMoeLayer, check, lib


def _round_up(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def blob_header(layer: int, expert: int, mats: dict[str, cv.QMat]) -> bytes:
    ordered = [mats[m] for m in cv.MAT_ORDER]
    h = cv.HEADER.pack(cv.EXPERT_MAGIC, cv.EXPERT_VERSION, layer, expert,
                       ordered[0].group_size, 3)
    return h + b"".join(cv.MAT_RECORD.pack(q.rows, q.cols, *q.section_bytes()) for q in ordered)


def parse_meta(blob_head: bytes, total: int | None = None) -> WispExpertMeta:
    """WispExpertMeta from a blob's first 120 bytes (via the library's parser)."""
    m = WispExpertMeta()
    err = WispErrCtx()
    buf = C.create_string_buffer(bytes(blob_head), len(blob_head))
    size = total if total is not None else len(blob_head)
    if total is not None and total > len(blob_head):
        # the parser checks the sections fit; give it the claimed size
        big = C.create_string_buffer(total)
        C.memmove(big, buf, len(blob_head))
        buf = big
    check(lib().wisp_expert_parse_header(buf, size, C.byref(m), C.byref(err)), err)
    return m


def blob_bytes_of(mats: dict[str, cv.QMat]) -> int:
    return cv.HEADER_BYTES + sum(sum(q.section_bytes()) for q in mats.values())


class ExpertArena:
    """One device allocation of fixed-size expert slots (blob at slot + 8), holding
    blobs in the tiled device layout (``wisp_expert_tile``)."""

    def __init__(self, n_slots: int, blob_bytes: int, device):
        self.slot_bytes = _round_up(blob_bytes + 8, 256)
        self.blob_bytes = blob_bytes
        self.n = n_slots
        self.buf = torch.empty(n_slots * self.slot_bytes, dtype=torch.uint8, device=device)
        self._tmp = torch.empty(self.slot_bytes, dtype=torch.uint8, device=device)

    def blob(self, i: int) -> torch.Tensor:
        o = i * self.slot_bytes + 8
        return self.buf[o:o + self.blob_bytes]

    def ptr(self, i: int) -> int:
        return self.buf.data_ptr() + i * self.slot_bytes + 8

    def write(self, i: int, layer: int, expert: int, mats: dict[str, cv.QMat]) -> None:
        """Assemble the .bin blob in a staging slot, then tile it into slot i."""
        dst = self._tmp[8:8 + self.blob_bytes]
        head = blob_header(layer, expert, mats)
        dst[:cv.HEADER_BYTES].copy_(torch.frombuffer(bytearray(head), dtype=torch.uint8))
        off = cv.HEADER_BYTES
        for name in cv.MAT_ORDER:
            q = mats[name]
            for t in (q.packed, q.scales.view(torch.uint8), q.zeros.view(torch.uint8)):
                n = t.numel()
                dst[off:off + n].copy_(t.reshape(-1), non_blocking=True)
                off += n
        meta = parse_meta(head, self.blob_bytes)
        err = WispErrCtx()
        check(lib().wisp_expert_tile(C.byref(meta), dst.data_ptr(), self.ptr(i),
                                     torch.cuda.current_stream(self.buf.device).cuda_stream,
                                     C.byref(err)), err)


@dataclass
class LayerWeights:
    router: torch.Tensor          # fp16 [E, H]
    router_bias: torch.Tensor | None
    norm: torch.Tensor            # fp16 [H]
    table: torch.Tensor           # int64 [E] device blob pointers
    slots: list[int]
    shared_slot: int | None = None
    shared_dense: tuple | None = None  # fp16 (gate, up, down) device tensors


class MoEStack:
    """A seeded synthetic MoE stack resident on one GPU (see ``converter`` for the recipe)."""

    def __init__(self, shape: cv.MoEShape, seed: int, device="cuda", zipf_s: float | None = None,
                 random_bias: bool = False, n_layers: int | None = None, layer0: int = 0,
                 expert_ids=None, with_shared: bool = True, gating: int = 0,
                 shared_form: str = "int4"):
        """`expert_ids`: the experts this stack holds (default all; the expert-parallel
        path holds a slice, table entry i = expert expert_ids[i]); `with_shared`: build
        the shape's shared expert (if any) -- `shared_form` "int4" (an int4 blob like the
        routed experts) or "fp16" (real-valued fp16-dense weights, the form the reference
        converter writes, ``converter.make_dense_ffn``); `gating`: 0 the reference's
        softmax(+bias), 1 sigmoid scores (``WISP_GATING_SIGMOID``)."""
        self.shape = shape
        self.device = torch.device(device)
        self.L = n_layers or shape.n_layers
        self.layer0 = layer0
        self.expert_ids = list(range(shape.n_experts)) if expert_ids is None else list(expert_ids)
        has_shared = bool(shape.shared_inter) and with_shared
        E = len(self.expert_ids)
        probe = cv.make_expert(cv.MoEShape(shape.hidden, shape.inter, E, shape.top_k,
                                           shape.group_size), 0, 0, seed, device=self.device)
        self.blob_bytes = blob_bytes_of(probe)
        dense_shared = has_shared and shared_form == "fp16"
        n_slots = self.L * E + (self.L if has_shared and not dense_shared else 0)
        self.arena = ExpertArena(n_slots, self.blob_bytes, self.device)
        self.layers: list[LayerWeights] = []
        slot = 0
        for li in range(self.L):
            l = layer0 + li
            slots = []
            for e in self.expert_ids:
                mats = cv.make_expert(shape, l, e, seed, device=self.device)
                self.arena.write(slot, l, e, mats)
                slots.append(slot)
                slot += 1
            sh = None
            sd = None
            if dense_shared:
                sd = tuple(t.to(self.device) for t in
                           cv.make_dense_ffn(shape.hidden, shape.shared_inter, l, seed, 1).values())
            elif has_shared:
                self.arena.write(slot, l, 0xFFFF, cv.make_shared_expert(shape, l, seed, self.device))
                sh = slot
                slot += 1
            router = cv.make_router(shape, l, seed, device=self.device)
            bias = None
            if zipf_s is not None:
                bias = cv.zipf_router_bias(shape, zipf_s).to(self.device)
            elif random_bias:
                g = torch.Generator().manual_seed(seed + 3 + l)
                bias = (torch.randn(E, generator=g) * 0.5).half().to(self.device)
            table = torch.tensor([self.arena.ptr(s) for s in slots], dtype=torch.int64,
                                 device=self.device) if slots else None
            self.layers.append(LayerWeights(router, bias, torch.ones(shape.hidden,
                                                                     dtype=torch.float16,
                                                                     device=self.device),
                                            table, slots, sh, sd))
        torch.cuda.synchronize(self.device)
        head = self.arena.blob(0)[:cv.HEADER_BYTES].cpu().numpy().tobytes()
        self.meta = parse_meta(head, self.blob_bytes)
        self._c_layers = (WispMoeLayer * self.L)()
        for l, lw in enumerate(self.layers):
            c = self._c_layers[l]
            c.meta = self.meta
            c.expert_blobs = lw.table.data_ptr() if lw.table is not None else None
            c.router_w = lw.router.data_ptr()
            c.router_bias = lw.router_bias.data_ptr() if lw.router_bias is not None else None
            c.norm_w = lw.norm.data_ptr()
            if lw.shared_slot is not None:
                c.shared_blob = self.arena.ptr(lw.shared_slot)
                c.shared_meta = self.meta
            if lw.shared_dense is not None:
                c.shared_gate, c.shared_up, c.shared_down = (t.data_ptr() for t in lw.shared_dense)
                c.shared_inter = shape.shared_inter
            c.n_experts = E
            c.top_k = shape.top_k
            c.gating = gating
        self._ws: torch.Tensor | None = None

    # ------------------------------------------------------------------
    def layer_c(self, l: int) -> WispMoeLayer:
        return self._c_layers[l]

    def workspace_bytes(self, T: int, layers: int | None = None) -> int:
        n = layers or self.L
        return int(lib().wisp_moe_workspace_bytes(C.byref(self._c_layers), n, T))

    def workspace(self, T: int) -> torch.Tensor:
        need = self.workspace_bytes(T)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def block(self, l: int, x: torch.Tensor, y: torch.Tensor | None = None, routing: bool = False):
        """y = MoE_l(x) on the current stream; x [T,H] fp32 on the device."""
        T = x.shape[0]
        if y is None:
            y = torch.empty_like(x)
        idx = torch.empty((T, self.shape.top_k), dtype=torch.int32, device=self.device)
        w = torch.empty((T, self.shape.top_k), dtype=torch.float32, device=self.device)
        ws = self.workspace(T)
        err = WispErrCtx()
        rc = lib().wisp_moe_block_forward(
            C.byref(self._c_layers[l]), x.data_ptr(), y.data_ptr(), T, idx.data_ptr(),
            w.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream,
            C.byref(err))
        check(rc, err)
        return (y, idx, w) if routing else y

    def prefill_workspace(self, T: int) -> torch.Tensor:
        need = int(lib().wisp_moe_prefill_stack_workspace_bytes(C.byref(self._c_layers), self.L,
                                                                 T)) + 1024
        if getattr(self, "_pws", None) is None or self._pws.numel() < need:
            self._pws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._pws

    def prefill(self, l: int, x: torch.Tensor, y: torch.Tensor | None = None,
                routing: bool = False):
        """y = MoE_l(x) for a batch of tokens on the tensor-core path
        (``wisp_moe_prefill_forward``); x [T,H] fp32 on the device."""
        T = x.shape[0]
        if y is None:
            y = torch.empty_like(x)
        idx = torch.empty((T, self.shape.top_k), dtype=torch.int32, device=self.device)
        w = torch.empty((T, self.shape.top_k), dtype=torch.float32, device=self.device)
        ws = self.prefill_workspace(T)
        off = (-ws.data_ptr()) % 1024
        err = WispErrCtx()
        rc = lib().wisp_moe_prefill_forward(
            C.byref(self._c_layers[l]), x.data_ptr(), y.data_ptr(), T, idx.data_ptr(),
            w.data_ptr(), ws.data_ptr() + off, ws.numel() - off,
            torch.cuda.current_stream().cuda_stream, C.byref(err))
        check(rc, err)
        return (y, idx, w) if routing else y

    def prefill_stack(self, x: torch.Tensor, routing: bool = False, layers: int | None = None):
        """x <- x + MoE_l(rmsnorm(x)) for every layer on the tensor-core path
        (``wisp_moe_prefill_stack_forward``), in place, on the current stream."""
        T = x.shape[0]
        n = layers or self.L
        idx = w = None
        if routing:
            idx = torch.empty((n, T, self.shape.top_k), dtype=torch.int32, device=self.device)
            w = torch.empty((n, T, self.shape.top_k), dtype=torch.float32, device=self.device)
        ws = self.prefill_workspace(T)
        off = (-ws.data_ptr()) % 1024
        err = WispErrCtx()
        rc = lib().wisp_moe_prefill_stack_forward(
            C.byref(self._c_layers), n, self.shape.rms_eps, x.data_ptr(), T,
            idx.data_ptr() if routing else None, w.data_ptr() if routing else None,
            ws.data_ptr() + off, ws.numel() - off, torch.cuda.current_stream().cuda_stream,
            C.byref(err))
        check(rc, err)
        return (x, idx, w) if routing else x

    def prefill_status(self) -> int:
        ws = getattr(self, "_pws", None)
        if ws is None:
            return 0
        off = (-ws.data_ptr()) % 1024
        return int(lib().wisp_moe_status(ws.data_ptr() + off,
                                         torch.cuda.current_stream().cuda_stream))

    def stack(self, x: torch.Tensor, routing: bool = False, layers: int | None = None,
              layer0: int = 0):
        """x <- x + MoE_l(rmsnorm(x)) for `layers` layers from `layer0` (default: every
        layer), in place, on the current stream."""
        T = x.shape[0]
        n = layers or self.L - layer0
        if layer0 < 0 or layer0 + n > self.L:
            raise ValueError(f"layers [{layer0}, {layer0 + n}) outside the stack of {self.L}")
        idx = w = None
        if routing:
            idx = torch.empty((n, T, self.shape.top_k), dtype=torch.int32, device=self.device)
            w = torch.empty((n, T, self.shape.top_k), dtype=torch.float32, device=self.device)
        ws = self.workspace(T)
        err = WispErrCtx()
        rc = lib().wisp_moe_stack_forward(
            C.byref(self._c_layers, layer0 * C.sizeof(WispMoeLayer)), n, self.shape.rms_eps,
            x.data_ptr(), T,
            idx.data_ptr() if routing else None, w.data_ptr() if routing else None,
            ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream, C.byref(err))
        check(rc, err)
        return (x, idx, w) if routing else x

    def status(self) -> int:
        if self._ws is None:
            return 0
        return int(lib().wisp_moe_status(self._ws.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream))

    # ------------------------------------------------------------------ oracle views
    def host_blobs(self, l: int) -> list[np.ndarray]:
        """The layer's expert blobs as .bin bytes (read back from the device and
        untiled), for the CPU oracle."""
        return [cv.untile_blob(self.arena.blob(s).cpu().numpy()) for s in self.layers[l].slots]

    def host_shared(self, l: int):
        """The shared expert of layer l as fp16 dense gate/up/down (raw bits, the
        form the reference computes it in), or None."""
        lw = self.layers[l]
        if lw.shared_dense is not None:
            return tuple(t.cpu().numpy().view(np.uint16) for t in lw.shared_dense)
        if lw.shared_slot is None:
            return None
        q = cv.qmats_from_blob(cv.untile_blob(self.arena.blob(lw.shared_slot).cpu().numpy()))
        return tuple(cv.dequantize_int4(q[n]).half().numpy().view(np.uint16)
                     for n in cv.MAT_ORDER)

    def host_router(self, l: int) -> tuple[np.ndarray, np.ndarray | None]:
        lw = self.layers[l]
        b = lw.router_bias.cpu().numpy().view(np.uint16) if lw.router_bias is not None else None
        return lw.router.cpu().numpy().view(np.uint16), b

    def active_bytes(self, idx: np.ndarray) -> int:
        """Algorithmic bytes of one step given its routing [L?, T, k]: distinct experts'
        int4 sections + router + activations, summed over layers."""
        idx = np.asarray(idx).reshape(-1, *np.asarray(idx).shape[-2:]) if np.ndim(idx) == 3 \
            else np.asarray(idx)[None]
        per_expert = self.blob_bytes - cv.HEADER_BYTES
        H, E = self.shape.hidden, self.shape.n_experts
        total = 0
        for li in idx:
            T = li.shape[0]
            distinct = len(np.unique(li[li >= 0]))
            total += distinct * per_expert + E * H * 2 + T * H * (2 + 4)
            if self.shape.shared_inter:
                total += per_expert
        return total
