"""The layer pipeline's ring protocol on CPU: world_size-2 and -4 gloo ranks, a stand-in
for each rank's layers (an affine map per rank), and the same LayerPipeline the GPU
bench drives.  After K decode steps every micro-batch must equal the composition of
all ranks' maps applied K times, in rank order -- which checks the send/receive
pairing, the wrap-around from the last rank to rank 0, the first/last-step rules and
the two-group send/receive split."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, steps, M, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from wisp_b200.pipeline import LayerPipeline
    groups = [dist.new_group(list(range(world))), dist.new_group(list(range(world)))]
    bufs = [torch.full((3, 4), float(m + 1)) for m in range(M)]

    def run(m):  # this rank's "layers"
        bufs[m].mul_(2.0).add_(rank + 1)

    pipe = LayerPipeline(run, bufs, rank, world, groups)
    for s in range(steps):
        pipe.step(first=(s == 0), last=(s == steps - 1))
    pipe.close()
    if rank == world - 1:
        out.put([b[0, 0].item() for b in bufs])
    for g in groups:
        dist.destroy_process_group(g)
    dist.destroy_process_group()


# (4, 4, 2): config 1's four micro-batches at four stages; (4, 2, 3): fewer
# micro-batches than stages, as at eight GPUs
@pytest.mark.parametrize("world,M,steps", [(2, 2, 3), (2, 3, 2), (4, 4, 2), (4, 2, 3)])
def test_ring_applies_every_rank_in_order(world, M, steps):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, steps, M, out))
             for r in range(world)]
    for p in procs:
        p.start()
    got = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = []
    for m in range(M):
        v = float(m + 1)
        for _ in range(steps):
            for r in range(world):
                v = v * 2.0 + (r + 1)
        want.append(v)
    assert got == want


def test_layer_split_covers_the_stack_contiguously():
    from wisp_b200.pipeline import layer_split
    for L, world in ((58, 8), (58, 4), (58, 2), (32, 8), (7, 3), (4, 4)):
        parts = layer_split(L, world)
        assert len(parts) == world
        assert parts[0][0] == 0
        for (a, n), (b, _) in zip(parts, parts[1:]):
            assert a + n == b
        assert sum(n for _, n in parts) == L
        assert max(n for _, n in parts) - min(n for _, n in parts) <= 1


def _two_rings_main(rank, world, port, out):
    """Two rings on the same process groups, one after the other, each a complete
    ring_run (as the config-3 bench drives them)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from wisp_b200.pipeline import LayerPipeline, ring_run
    groups = [dist.new_group(list(range(world))), dist.new_group(list(range(world)))]
    res = []
    for M, steps in ((3, 2), (2, 3), (3, 1)):
        bufs = [torch.full((2, 2), float(m)) for m in range(M)]

        def run(m, bufs=bufs):
            bufs[m].add_(1.0)

        pipe = LayerPipeline(run, bufs, rank, world, groups)
        ring_run(pipe, steps)
        dist.barrier()  # nothing may be in flight here
        pipe.close()
        res.append([b[0, 0].item() for b in bufs])
    if rank == world - 1:
        out.put(res)
    dist.barrier()
    for g in groups:
        dist.destroy_process_group(g)
    dist.destroy_process_group()


def test_complete_rings_back_to_back():
    """Each ring_run leaves no send in flight: the next ring receives only its own
    micro-batches, and every micro-batch went through steps x world passes."""
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rings_main, args=(r, world, port, out))
             for r in range(world)]
    for p in procs:
        p.start()
    got = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == [[float(m) + steps * world for m in range(M)]
                   for M, steps in ((3, 2), (2, 3), (3, 1))]
