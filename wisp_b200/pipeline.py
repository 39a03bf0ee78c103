"""Layer pipeline over NCCL for MoE stacks (one process per GPU, torch.distributed).

The reference declares a single-process NCCL pipeline that sends one fp32 hidden
vector per token between stages (csrc/cuda/multi_gpu.cu:84-133) but never calls it.
Here each rank owns a contiguous layer range and runs it with the fused stack
kernels (one CUDA graph per micro-batch); micro-batches of hidden states
``[mb, H]`` fp32 move between neighbouring ranks with NCCL send/recv, and the last
rank hands every micro-batch back to rank 0, which is where the next decode step of
that micro-batch starts (the autoregressive dependency).  With M micro-batches and
S ranks the steady-state utilisation bound is min(1, M/S); the benchmark keeps
M = 4S.

Ordering: a micro-batch buffer is re-filled by a receive only after its previous
send completed (the send's work handle is waited on the compute stream first), and
compute waits on the receive; the sends/receives of different peers run on
torch's per-peer NCCL streams, overlapping the next micro-batch's compute.
"""

from __future__ import annotations

import datetime
import json
import os
import statistics
import time


class LayerPipeline:
    def __init__(self, stack, micro_inputs, rank: int, world: int):
        import torch
        self.stack, self.rank, self.world = stack, rank, world
        self.bufs = [x.clone() for x in micro_inputs]
        self.M = len(self.bufs)
        self.send_work = [None] * self.M
        self.graphs = []
        stack.workspace(self.bufs[0].shape[0])
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            tmp = self.bufs[0].clone()
            stack.stack(tmp)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        for b in self.bufs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                stack.stack(b)
            self.graphs.append(g)

    def step(self, first: bool, last: bool) -> None:
        import torch.distributed as dist
        r, w = self.rank, self.world
        src, dst = (r - 1) % w, (r + 1) % w
        for m in range(self.M):
            if r > 0 or not first:
                if self.send_work[m] is not None:
                    self.send_work[m].wait()
                    self.send_work[m] = None
                dist.irecv(self.bufs[m], src).wait()
            self.graphs[m].replay()
            if r < w - 1 or not last:
                self.send_work[m] = dist.isend(self.bufs[m], dst)

    def drain(self) -> None:
        for m in range(self.M):
            if self.send_work[m] is not None:
                self.send_work[m].wait()
                self.send_work[m] = None

    def close(self) -> None:
        self.drain()
        self.graphs.clear()


def bench_main(args) -> None:
    import torch
    import torch.distributed as dist

    from . import build
    from . import converter as cv
    from .moe import MoEStack

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if rank == 0:
        build.build()
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    dist.barrier()
    build.build()  # no-op when rank 0 already built it

    seed = 20251201
    L = args.layers
    if L % world:
        raise SystemExit(f"--layers {L} must be divisible by the world size {world}")
    per = L // world
    shape = cv.MoEShape(hidden=4096, inter=14336, n_experts=8, top_k=2, n_layers=L)
    stack = MoEStack(shape, seed, device=dev, n_layers=per, layer0=rank * per)
    mb = args.micro
    global_batch = args.batch * world
    M = global_batch // mb
    micro = [cv.make_input(shape, mb, seed + 1000 + m).to(dev) for m in range(M)]
    pipe = LayerPipeline(stack, micro, rank, world)

    total = args.warmup + args.steps
    for s in range(args.warmup):
        pipe.step(first=(s == 0), last=False)
    pipe.drain()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.time()
    e0.record()
    for s in range(args.warmup, total):
        pipe.step(first=False, last=(s == total - 1))
    pipe.drain()
    e1.record()
    torch.cuda.synchronize()
    t_wall = time.time() - t_wall
    ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    dist.barrier()
    ms_step = ms.item() / args.steps
    value = global_batch * 1000.0 / ms_step
    pipe.close()
    del pipe
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({
            "metric": "MoE-block decode tokens/s (Mixtral-8x7B-shaped 32-block stack)",
            "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4xf32", "data": "synthetic",
            "config": {"workload": f"config1: Mixtral-8x7B-shaped {L}-block stack decode, layer "
                                   f"pipeline over {world} GPUs, {M} micro-batches of {mb}",
                       "global_batch": global_batch, "parallelism": f"pp{world}",
                       "micro_batches": M, "layers_per_rank": per,
                       "l2": "weights per step exceed L2"},
            "gpu_launches": (4 * per + 1) * M * args.steps,
            "wall_s_timed": round(t_wall, 3)}), flush=True)
