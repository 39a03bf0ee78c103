"""Expert parallelism (config 2).  On CPU: the dispatch bookkeeping and 2- and 4-rank gloo
round trips of dispatch -> per-owner expert compute -> return -> top-k-ordered combine,
with stand-in experts.  On one GPU: the expert-parallel layer (world size 1, every
expert local) against the fused block and against the oracle."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wisp_b200.ep import Dispatch, dispatch_plan


def test_dispatch_plan_orders_by_owner_then_token_then_slot():
    idx = torch.tensor([[5, 0, -1], [1, 7, 4], [6, 2, 3]], dtype=torch.int32)
    order, counts, tokens, eid, owner, row_idx = dispatch_plan(idx, per=4, world=2)
    assert counts.tolist() == [4, 4]
    # owner 0: (0,1)=0 (1,0)=1 (2,1)=2 (2,2)=3 ; owner 1: (0,0)=5 (1,1)=7 (1,2)=4 (2,0)=6
    assert order.tolist()[:8] == [1, 3, 7, 8, 0, 4, 5, 6]
    assert order.tolist()[8] == 2 and owner.tolist()[8] == 2  # the unrouted slot, last
    assert tokens.tolist()[:8] == [0, 1, 2, 2, 0, 1, 1, 2]
    assert eid.tolist()[:8] == [0, 1, 2, 3, 1, 3, 0, 2]
    assert row_idx.tolist() == [[4, 0, -1], [1, 5, 6], [7, 2, 3]]


def test_single_rank_dispatch_keeps_rows_and_ids():
    """World size 1: no collective; the rows and local expert ids come back in send
    order and `back` is the identity."""
    idx = torch.tensor([[2, 0], [-1, 3], [1, 2]], dtype=torch.int32)
    x = torch.arange(12, dtype=torch.float32).view(3, 4)
    d = Dispatch(x, idx, per=4, world=1)
    assert d.send_counts == [5] and d.recv_counts == [5]
    # send order: (0,0)=2 (0,1)=0 (1,1)=3 (2,0)=1 (2,1)=2
    assert d.eids.view(-1).tolist() == [2, 0, 3, 1, 2]
    assert torch.equal(d.rows, x[[0, 0, 1, 2, 2]])
    assert d.back(d.rows) is d.rows


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_rank(rank, world, port, out, idle_last=False, uneven=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    per, K, H = 3, 2, 4
    # uneven: rank r holds 5 + r tokens, and every rank passes the largest count
    B = 5 + rank if uneven else 5
    max_tokens = 5 + world - 1 if uneven else None
    # idle_last: no token routes to the last rank's experts, so it receives no rows
    E = per * (world - 1) if idle_last else per * world
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(B, H, generator=g)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(B)]).int()
    idx[1, 1] = -1  # an unrouted slot
    w = torch.rand(B, K, generator=g)
    d = Dispatch(x, idx, per, world, max_tokens=max_tokens)
    # stand-in expert e (global id rank*per + local): y = (e + 1) * x + e
    ge = d.eids.view(-1).float() + rank * per
    rows = d.rows * (ge + 1).view(-1, 1) + ge.view(-1, 1)
    back = d.back(rows)
    y = torch.zeros(B, H)
    for t in range(B):
        for j in range(K):
            r = int(d.row_idx[t, j])
            if r >= 0:
                y[t] += w[t, j] * back[r]
    # what the experts compute directly on this rank's tokens
    want = torch.zeros(B, H)
    for t in range(B):
        for j in range(K):
            e = int(idx[t, j])
            if e >= 0:
                want[t] += w[t, j] * ((e + 1) * x[t] + e)
    out.put((rank, float((y - want).abs().max()), sum(d.recv_counts)))
    dist.destroy_process_group()


# (2, False, False): config 2's exchange at two ranks; (4, True, True): four ranks
# holding 5..8 tokens, the last one owning experts no token chose (it sends its own
# tokens' rows and receives none)
@pytest.mark.parametrize("world,idle_last,uneven", [(2, False, False), (4, True, True)])
def test_dispatch_compute_return_combine(world, idle_last, uneven):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_rank, args=(r, world, port, out, idle_last, uneven))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [out.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(err < 1e-5 for _, err, _ in res), res
    if idle_last:
        assert [n for r, _, n in res if r == world - 1] == [0]


@pytest.mark.gpu
@pytest.mark.parametrize("B", [1, 12])
def test_ep_layer_matches_block_and_oracle(cuda, B):
    from oracle import oracle as orc
    from wisp_b200 import converter as cv
    from wisp_b200.ep import EPLayer
    from wisp_b200.moe import MoEStack
    from parity import check_block, check_outputs
    shape = cv.MoEShape(hidden=1024, inter=512, n_experts=32, top_k=8, shared_inter=512)
    ep = EPLayer(shape, 41, 0, 1, cuda, zipf_s=1.1)
    st = MoEStack(shape, 41, device=cuda, zipf_s=1.1)
    x = cv.make_input(shape, B, 9).to(cuda)
    y, idx, w = ep.forward(x)
    yb, ib, wb = st.block(0, x, routing=True)
    torch.cuda.synchronize()
    assert st.status() == 0
    assert np.array_equal(idx.cpu().numpy(), ib.cpu().numpy())
    np.testing.assert_allclose(y.cpu().numpy(), yb.cpu().numpy(), rtol=1e-5, atol=1e-6)
    Wb, bb = st.host_router(0)
    yr, ir, wr = orc.port_moe_block_arrays(Wb, bb, st.host_blobs(0), 8, x.cpu().numpy(),
                                           shared=st.host_shared(0))
    check_block(y.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), yr, ir, wr, Wb, bb,
                x.cpu().numpy(), st.host_blobs(0), shared=st.host_shared(0), tight=False)


@pytest.mark.gpu
def test_ep_layer_tensor_path_for_many_rows(cuda):
    """At 64 tokens x top-8 the rank receives 512 rows: its experts run on the
    tensor-core path (wisp_moe_prefill_routed); the result matches the fused block and
    the oracle."""
    from oracle import oracle as orc
    from wisp_b200 import converter as cv
    from wisp_b200.ep import EPLayer
    from wisp_b200.moe import MoEStack
    from parity import check_block, check_outputs
    shape = cv.MoEShape(hidden=1024, inter=512, n_experts=32, top_k=8, shared_inter=512)
    ep = EPLayer(shape, 43, 0, 1, cuda, zipf_s=1.1)
    assert 64 * 8 >= max(ep.TENSOR_MIN_ROWS, ep.TENSOR_MIN_PER_EXPERT * ep.per)
    st = MoEStack(shape, 43, device=cuda, zipf_s=1.1)
    x = cv.make_input(shape, 64, 10).to(cuda)
    y, idx, w = ep.forward(x)
    yb, ib, _ = st.block(0, x, routing=True)
    torch.cuda.synchronize()
    assert np.array_equal(idx.cpu().numpy(), ib.cpu().numpy())
    check_outputs(y.cpu().numpy(), yb.cpu().numpy())
    Wb, bb = st.host_router(0)
    yr, ir, wr = orc.port_moe_block_arrays(Wb, bb, st.host_blobs(0), 8, x.cpu().numpy(),
                                           shared=st.host_shared(0))
    check_block(y.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), yr, ir, wr, Wb, bb,
                x.cpu().numpy(), st.host_blobs(0), shared=st.host_shared(0))
