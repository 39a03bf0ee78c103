"""Expert parallelism for a DeepSeek-shaped MoE layer: the routed
experts are sharded over the ranks of a process group (rank r holds experts
[r*E/N, (r+1)*E/N)), every rank holds the router and the shared expert, and each rank
routes its own tokens.

One step on a rank (tokens x [B, H] fp32 on its GPU):

1. route (``wisp_moe_route``, the full router): top-k expert ids and weights per token;
2. dispatch (``Dispatch``): the (token, slot) assignments are ordered by owner rank on
   the device; one fixed-size NCCL all-to-all carries, to each owner, the number of
   rows it will receive and their local expert ids; one small device-to-host read gives
   both count vectors; the token rows travel with a second all-to-all
   (``torch.distributed.all_to_all_single``);
3. each owner runs its experts on the rows it received (``wisp_moe_experts_routed``,
   one expert per row, weight 1);
4. the result rows travel back with the third, reverse all-to-all;
5. the home rank adds the shared expert (computed on its own tokens meanwhile) and the
   gate-weighted rows in top-k order (``wisp_moe_ep_combine``) -- the reference's
   combine order (shared first, then the routed experts in top-k order,
   csrc/core/wisp_engine.c:1443-1522).

The reference declares no expert-parallel path; this one is new.  Steps 2 and 4 are
torch operations on whatever device the tensors are on, so the same code is tested on
CPU with gloo ranks.
"""

from __future__ import annotations

import ctypes as C


def dispatch_plan(idx, per: int, world: int):
    """Device-side bookkeeping (torch ops on idx's device, no host round trip).  For
    routing idx [B, K] (expert ids, -1 = none) and `per` experts per rank: the send
    order of the assignments (sorted by owner rank, then token, then slot; unrouted
    slots last), the send count per rank, each sent row's token and local expert id,
    its owner, and row_idx [B, K]: the position of assignment (t, j) in the send order
    (-1 if unrouted)."""
    import torch
    B, K = idx.shape
    flat = idx.reshape(-1).long()
    live = flat >= 0
    owner = torch.where(live, flat.div(per, rounding_mode="floor"), torch.full_like(flat, world))
    order = torch.argsort(owner, stable=True)  # stable: token, then slot order
    counts = torch.bincount(owner, minlength=world + 1)[:world]
    sorted_owner = owner[order]
    tokens = order.div(K, rounding_mode="floor")
    local_eid = torch.where(live[order], flat[order] % per, torch.zeros_like(flat)).int()
    pos = torch.arange(B * K, device=idx.device)
    row_idx = torch.full((B * K,), -1, dtype=torch.int32, device=idx.device)
    row_idx[order] = torch.where(live[order], pos, torch.full_like(pos, -1)).int()
    return order, counts, tokens, local_eid, sorted_owner, row_idx.view(B, K)


def exchange_counts(counts, sorted_owner, local_eid, world: int, cap: int, group=None):
    """The first all-to-all, of fixed size: to each rank d, [the number of rows this
    rank will send it, then those rows' local expert ids] (padded to `cap`).  Returns
    the received [world, 1 + cap] table (row s: what rank s sends here)."""
    import torch
    import torch.distributed as dist
    dev = counts.device
    table = torch.zeros((world, 1 + cap), dtype=torch.int32, device=dev)
    table[:, 0] = counts.int()
    start = torch.cumsum(counts, 0) - counts
    n = sorted_owner.numel()
    live = sorted_owner < world
    d = torch.where(live, sorted_owner, torch.zeros_like(sorted_owner))
    j = torch.arange(n, device=dev) - start[d]
    dst = torch.where(live, d * (1 + cap) + 1 + j, torch.full_like(j, -1))
    flat = table.view(-1)
    keep = dst >= 0
    flat.index_put_((dst[keep],), local_eid[keep])
    if world == 1:
        return table
    recv = torch.empty_like(table)
    dist.all_to_all_single(recv, table, group=group)
    return recv


def exchange_rows(send, send_counts, recv_counts, group=None):
    """all_to_all of `send` rows (grouped by destination, send_counts[d] rows each);
    recv_counts[s] rows arrive from each rank s (host lists)."""
    import torch
    import torch.distributed as dist
    recv = torch.empty((int(sum(recv_counts)), send.shape[1]), dtype=send.dtype,
                       device=send.device)
    dist.all_to_all_single(recv, send, output_split_sizes=list(recv_counts),
                           input_split_sizes=list(send_counts), group=group)
    return recv


def exchange_back(rows, send_counts, recv_counts, group=None):
    """The reverse all_to_all: rows received per source go back to it."""
    return exchange_rows(rows, recv_counts, send_counts, group)


class Dispatch:
    """Steps 2-4 of the module doc for one layer call: three collectives (the fixed-size
    count/expert-id table, the rows out, the rows back) and one small device-to-host
    read (both count vectors, which the variable all-to-alls need on the host)."""

    def __init__(self, x, idx, per: int, world: int, group=None, max_tokens: int | None = None):
        """`max_tokens`: the most tokens any rank of the group dispatches in this call;
        every rank must pass the same value (the count table has a fixed size).  The
        default, this rank's own token count, is right when every rank has as many."""
        import torch
        B, K = idx.shape
        if max_tokens is None:
            max_tokens = B
        if B > max_tokens:
            raise ValueError(f"{B} tokens on this rank, above max_tokens={max_tokens}")
        cap = max_tokens * K
        self.world, self.group = world, group
        _, counts, tokens, local_eid, owner, self.row_idx = dispatch_plan(idx, per, world)
        table = exchange_counts(counts, owner, local_eid, world, cap, group)
        both = torch.stack([counts.int(), table[:, 0]]).cpu()  # the one host read
        self.send_counts = [int(c) for c in both[0]]
        self.recv_counts = [int(c) for c in both[1]]
        n_send = sum(self.send_counts)
        send = x.index_select(0, tokens[:n_send])
        self.rows = (exchange_rows(send, self.send_counts, self.recv_counts, group)
                     if world > 1 else send)
        # local expert ids of the received rows, in source order: received row j
        # came from the rank s whose count range holds j (no host round trip)
        n_recv = sum(self.recv_counts)
        rc = table[:, 0].long()
        end = torch.cumsum(rc, 0)
        j = torch.arange(n_recv, device=x.device)
        src = torch.searchsorted(end, j, right=True)
        sel = src * (1 + cap) + 1 + (j - (end - rc)[src])
        self.eids = table.view(-1)[sel].view(-1, 1)

    def back(self, out_rows):
        """The expert outputs of the received rows, returned to their home ranks."""
        if self.world == 1:
            return out_rows
        return exchange_back(out_rows, self.send_counts, self.recv_counts, self.group)


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

    def forward(self, x, max_tokens: int | None = None):
        """y [B, H] for this rank's tokens x [B, H] (fp32, on this rank's GPU).  When the
        ranks hold different numbers of tokens, every rank passes the largest of them as
        `max_tokens` (see Dispatch)."""
        import torch
        from .lib import WispErrCtx, check, lib
        B, H = x.shape
        idx, w = self.route(x)
        dsp = Dispatch(x, idx, self.per, self.world, self.group, max_tokens)
        self.last_counts = dsp.send_counts
        wt = torch.ones((dsp.rows.shape[0], 1), dtype=torch.float32, device=self.device)
        rows = self.experts(self.expert_layer, dsp.rows.contiguous(), dsp.eids.contiguous(), wt)
        back = dsp.back(rows)
        if self.shared_layer is not None:
            y = self.experts(self.shared_layer, x,
                             torch.zeros((B, 1), dtype=torch.int32, device=self.device),
                             torch.ones((B, 1), dtype=torch.float32, device=self.device))
        else:
            y = torch.zeros_like(x)
        err = WispErrCtx()
        check(lib().wisp_moe_ep_combine(y.data_ptr(), back.data_ptr() if back.numel() else None,
                                        dsp.row_idx.data_ptr(), w.data_ptr(), B, idx.shape[1], H,
                                        torch.cuda.current_stream().cuda_stream,
                                        C.byref(err)), err)
        return y, idx, w
