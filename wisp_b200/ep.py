"""Expert parallelism for a DeepSeek-shaped MoE layer: the routed
experts are sharded over the ranks of a process group (rank r holds experts
[r*E/N, (r+1)*E/N)), every rank holds the router and the shared expert, and each rank
routes its own tokens.

One step on a rank (tokens x [B, H] fp32 on its GPU):

1. route (``wisp_moe_route``, the full router): top-k expert ids and weights per token;
2. dispatch: the (token, slot) assignments are ordered by owner rank, counts are
   exchanged, and the token rows travel to the owners with one NCCL all-to-all
   (``torch.distributed.all_to_all_single``) together with their local expert ids;
3. each owner runs its experts on the rows it received (``wisp_moe_experts_routed``,
   one expert per row, weight 1);
4. the result rows travel back with the reverse all-to-all;
5. the home rank adds the shared expert (computed on its own tokens meanwhile) and the
   gate-weighted rows in top-k order (``wisp_moe_ep_combine``) -- the reference's
   combine order (shared first, then the routed experts in top-k order,
   csrc/core/wisp_engine.c:1443-1522).

The reference declares no expert-parallel path; this one is new.  The bookkeeping of
step 2 (``dispatch_plan``) is plain numpy so it is tested on CPU with gloo ranks.
"""

from __future__ import annotations

import ctypes as C

import numpy as np


def dispatch_plan(idx: np.ndarray, per: int, world: int):
    """For routing idx [B, K] (expert ids, -1 = none) and `per` experts per rank:
    the assignments in send order (sorted by owner rank, then token, then slot), the
    send count per rank, each sent row's token and local expert id, and row_idx [B, K]:
    the position of assignment (t, j) in the send order (-1 if unrouted)."""
    B, K = idx.shape
    flat = idx.reshape(-1)
    live = np.nonzero(flat >= 0)[0]
    owner = flat[live] // per
    order = live[np.argsort(owner, kind="stable")]  # stable: token, then slot order
    counts = np.bincount(flat[order] // per, minlength=world).astype(np.int64)
    tokens = (order // K).astype(np.int64)
    local_eid = (flat[order] % per).astype(np.int32)
    row_idx = np.full(B * K, -1, dtype=np.int32)
    row_idx[order] = np.arange(order.size, dtype=np.int32)
    return order, counts, tokens, local_eid, row_idx.reshape(B, K)


def exchange(send, send_counts, row_elems: int, group=None):
    """all_to_all of `send` rows ([n, row_elems], grouped by destination rank with
    send_counts[d] rows each); returns (received rows, recv_counts)."""
    import torch
    import torch.distributed as dist
    sc = torch.as_tensor(send_counts, dtype=torch.int64, device=send.device)
    rc = torch.empty_like(sc)
    dist.all_to_all_single(rc, sc, group=group)
    rcl = rc.cpu().tolist()
    recv = torch.empty((int(sum(rcl)), row_elems), dtype=send.dtype, device=send.device)
    dist.all_to_all_single(recv, send, output_split_sizes=rcl,
                           input_split_sizes=[int(c) for c in send_counts], group=group)
    return recv, rcl


def exchange_back(rows, send_counts, recv_counts, group=None):
    """The reverse all_to_all: rows received per source go back to it."""
    import torch
    import torch.distributed as dist
    out = torch.empty((int(sum(send_counts)), rows.shape[1]), dtype=rows.dtype,
                      device=rows.device)
    dist.all_to_all_single(out, rows, output_split_sizes=[int(c) for c in send_counts],
                           input_split_sizes=list(recv_counts), group=group)
    return out


class EPLayer:
    """One expert-sharded MoE layer on this rank's GPU (see the module doc)."""

    def __init__(self, shape, seed: int, rank: int, world: int, device, zipf_s=None,
                 random_bias: bool = False, group=None, gating: int = 0):
        import torch
        from .lib import WispMoeLayer
        from .moe import MoEStack
        if shape.n_experts % world:
            raise ValueError(f"{shape.n_experts} experts do not split over {world} ranks")
        self.shape, self.rank, self.world, self.group = shape, rank, world, group
        self.device = torch.device(device)
        self.per = shape.n_experts // world
        ids = range(rank * self.per, (rank + 1) * self.per)
        self.local = MoEStack(shape, seed, device, zipf_s=zipf_s, random_bias=random_bias,
                              n_layers=1, expert_ids=ids, with_shared=True, gating=gating)
        lw = self.local.layers[0]
        H = shape.hidden
        # routing: the full router, no expert table
        self.route_layer = WispMoeLayer()
        C.memmove(C.byref(self.route_layer), C.byref(self.local.layer_c(0)),
                  C.sizeof(WispMoeLayer))
        self.route_layer.expert_blobs = None
        self.route_layer.n_experts = shape.n_experts
        self.route_layer.shared_blob = None
        # this rank's experts on dispatched rows: one expert per row, weight 1
        self.expert_layer = WispMoeLayer()
        C.memmove(C.byref(self.expert_layer), C.byref(self.local.layer_c(0)),
                  C.sizeof(WispMoeLayer))
        self.expert_layer.router_w = None
        self.expert_layer.router_bias = None
        self.expert_layer.shared_blob = None
        self.expert_layer.n_experts = self.per
        self.expert_layer.top_k = 1
        # the shared expert as a one-expert layer on the home tokens
        self.shared_layer = None
        if lw.shared_slot is not None:
            self._shared_table = torch.tensor([self.local.arena.ptr(lw.shared_slot)],
                                              dtype=torch.int64, device=self.device)
            self.shared_layer = WispMoeLayer()
            C.memmove(C.byref(self.shared_layer), C.byref(self.expert_layer),
                      C.sizeof(WispMoeLayer))
            self.shared_layer.expert_blobs = self._shared_table.data_ptr()
            self.shared_layer.n_experts = 1
        self._ws = None
        self._ws_bytes = 0
        self._one = torch.ones((1, 1), dtype=torch.float32, device=self.device)
        self.last_counts = None
        del H

    def _workspace(self, layer, T):
        import torch
        from .lib import lib
        need = int(lib().wisp_moe_workspace_bytes(C.byref(layer), 1, max(T, 1)))
        if need > self._ws_bytes:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            self._ws_bytes = need
        return self._ws

    def route(self, x):
        import torch
        from .lib import WispErrCtx, check, lib
        B = x.shape[0]
        K = self.shape.top_k
        idx = torch.empty((B, K), dtype=torch.int32, device=self.device)
        w = torch.empty((B, K), dtype=torch.float32, device=self.device)
        ws = self._workspace(self.route_layer, B)
        err = WispErrCtx()
        check(lib().wisp_moe_route(C.byref(self.route_layer), x.data_ptr(), B, idx.data_ptr(),
                                   w.data_ptr(), ws.data_ptr(), ws.numel(),
                                   torch.cuda.current_stream().cuda_stream, C.byref(err)), err)
        return idx, w

    # this rank's experts run on the tensor-core path (each routed expert streamed
    # once per 128 rows) instead of the decode kernels (once per 4-row tile) from
    # TENSOR_MIN_ROWS rows and TENSOR_MIN_PER_EXPERT rows per local expert: the ranks
    # holding the hot experts of a Zipf-skewed routing get hundreds of rows each
    TENSOR_MIN_ROWS = 256
    TENSOR_MIN_PER_EXPERT = 8

    def experts(self, layer, x, eid, wt):
        """y[r] = sum_j wt[r,j] * E_eid[r,j](x[r]) for this rank's experts."""
        import torch
        from .lib import WispErrCtx, check, lib
        y = torch.empty_like(x)
        if x.shape[0] == 0:
            return y
        R, K = x.shape[0], eid.shape[1]
        if (R >= self.TENSOR_MIN_ROWS and layer.n_experts > 1
                and R >= self.TENSOR_MIN_PER_EXPERT * layer.n_experts):
            need = int(lib().wisp_moe_prefill_routed_workspace_bytes(C.byref(layer), R, K)) + 1024
            if getattr(self, "_pws", None) is None or self._pws.numel() < need:
                self._pws = torch.empty(need, dtype=torch.uint8, device=self.device)
            off = (-self._pws.data_ptr()) % 1024
            err = WispErrCtx()
            check(lib().wisp_moe_prefill_routed(C.byref(layer), x.data_ptr(), y.data_ptr(), R, K,
                                                eid.data_ptr(), wt.data_ptr(),
                                                self._pws.data_ptr() + off,
                                                self._pws.numel() - off,
                                                torch.cuda.current_stream().cuda_stream,
                                                C.byref(err)), err)
            return y
        ws = self._workspace(layer, x.shape[0])
        err = WispErrCtx()
        check(lib().wisp_moe_experts_routed(C.byref(layer), x.data_ptr(), y.data_ptr(),
                                            x.shape[0], eid.data_ptr(), wt.data_ptr(),
                                            ws.data_ptr(), ws.numel(),
                                            torch.cuda.current_stream().cuda_stream,
                                            C.byref(err)), err)
        return y

    def forward(self, x):
        """y [B, H] for this rank's tokens x [B, H] (fp32, on this rank's GPU)."""
        import torch
        from .lib import WispErrCtx, check, lib
        B, H = x.shape
        idx, w = self.route(x)
        order, counts, tokens, local_eid, row_idx = dispatch_plan(
            idx.cpu().numpy(), self.per, self.world)
        self.last_counts = counts
        tok = torch.as_tensor(tokens, device=self.device)
        send = x.index_select(0, tok) if tokens.size else x[:0]
        eid_send = torch.as_tensor(local_eid, device=self.device).view(-1, 1)
        if self.world > 1:
            recv, rcl = exchange(send, counts, H, self.group)
            eid_recv, _ = exchange(eid_send, counts, 1, self.group)
        else:
            recv, rcl, eid_recv = send, [int(counts[0])], eid_send
        wt = torch.ones((recv.shape[0], 1), dtype=torch.float32, device=self.device)
        rows = self.experts(self.expert_layer, recv.contiguous(), eid_recv.contiguous(), wt)
        back = exchange_back(rows, counts, rcl, self.group) if self.world > 1 else rows
        if self.shared_layer is not None:
            y = self.experts(self.shared_layer, x,
                             torch.zeros((B, 1), dtype=torch.int32, device=self.device),
                             torch.ones((B, 1), dtype=torch.float32, device=self.device))
        else:
            y = torch.zeros_like(x)
        ridx = torch.as_tensor(row_idx, device=self.device)
        err = WispErrCtx()
        check(lib().wisp_moe_ep_combine(y.data_ptr(), back.data_ptr() if back.numel() else None,
                                        ridx.data_ptr(), w.data_ptr(), B, idx.shape[1], H,
                                        torch.cuda.current_stream().cuda_stream,
                                        C.byref(err)), err)
        return y, idx, w
