"""Layer pipeline over NCCL for MoE stacks (one process per GPU, torch.distributed).

The reference declares a single-process NCCL pipeline that sends one fp32 hidden
vector per token between stages (csrc/cuda/multi_gpu.cu:84-133) but never calls it.
Here each rank owns a contiguous layer range and runs it with the fused stack
kernels (one CUDA graph per micro-batch); micro-batches of hidden states
``[mb, H]`` fp32 move between neighbouring ranks with NCCL send/recv, and the last
rank hands every micro-batch back to rank 0, which is where the next decode step of
that micro-batch starts (the autoregressive dependency).

Decode is bound by streaming the routed experts' weights, and every micro-batch
re-streams its layers' experts, so micro-batches are as large as the ring allows:
the default is one micro-batch per stage (M = S, the per-GPU batch each), which keeps
every stage busy in the steady state (utilisation bound min(1, M/S) = 1).

Ordering: a micro-batch buffer is re-filled by a receive only after its previous
send completed (the send's work handle is waited on the compute stream first), and
compute waits on the receive.  Sends and receives use two process groups (a rank
sends on group rank % 2 and receives on group (rank - 1) % 2), so a rank's send and
its next receive are not serialised behind each other.
"""

from __future__ import annotations

import datetime
import json
import os
import statistics
import time


class LayerPipeline:
    """The ring of one rank: `bufs` are its micro-batch buffers, `run(m)` applies this
    rank's layers to bufs[m] in place on the current stream."""

    def __init__(self, run, bufs, rank: int, world: int, groups=None):
        self.run, self.bufs, self.rank, self.world = run, bufs, rank, world
        self.M = len(bufs)
        self.send_work = [None] * self.M
        # (send group, receive group); None = the default group for both
        self.send_pg = groups[rank % 2] if groups else None
        self.recv_pg = groups[(rank - 1) % 2] if groups else None

    @classmethod
    def for_stack(cls, stack, micro_inputs, rank: int, world: int, groups=None):
        """One CUDA graph per micro-batch of `stack` (a MoEStack) over its layers."""
        import torch
        bufs = [x.clone() for x in micro_inputs]
        stack.workspace(bufs[0].shape[0])
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            tmp = bufs[0].clone()
            stack.stack(tmp)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graphs = []
        for b in bufs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                stack.stack(b)
            graphs.append(g)
        pipe = cls(lambda m: graphs[m].replay(), bufs, rank, world, groups)
        pipe.graphs = graphs
        return pipe

    def step(self, first: bool, last: bool, on_input=None, on_output=None) -> None:
        """One decode step of every micro-batch.  `first`: rank 0 has nothing to
        receive yet; `last`: the last rank keeps its outputs.  on_input(m) runs after
        micro-batch m's receive and before its compute, on_output(m) after it."""
        import torch.distributed as dist
        r, w = self.rank, self.world
        src, dst = (r - 1) % w, (r + 1) % w
        for m in range(self.M):
            if r > 0 or not first:
                if self.send_work[m] is not None:
                    self.send_work[m].wait()
                    self.send_work[m] = None
                dist.irecv(self.bufs[m], src, group=self.recv_pg).wait()
            if on_input is not None:
                on_input(m)
            self.run(m)
            if on_output is not None:
                on_output(m)
            if r < w - 1 or not last:
                self.send_work[m] = dist.isend(self.bufs[m], dst, group=self.send_pg)

    def drain(self) -> None:
        for m in range(self.M):
            if self.send_work[m] is not None:
                self.send_work[m].wait()
                self.send_work[m] = None

    def close(self) -> None:
        self.drain()
        getattr(self, "graphs", []).clear()


def launches_per_layer(shape, T: int) -> int:
    """Kernels the stack launches per layer: prep (+ the router kernel when the router
    does not run inside prep, i.e. T*E*H*2 bytes > 32 MB) + gate/up + down."""
    return 3 if T * shape.n_experts * shape.hidden * 2 <= (32 << 20) else 4


def _measure_ring(stack, shape, rank, world, dev, groups, global_batch, mb, args, seed,
                  with_e2e):
    """Decode steps of `global_batch` tokens as global_batch / mb micro-batches
    circulating through the layer pipeline: the steady-state time per step (every
    micro-batch one decode step through every stage), max over ranks, and optionally
    the same with the inputs from and outputs to pinned host memory."""
    import torch
    import torch.distributed as dist

    from . import converter as cv
    from .benchutil import ClockSampler, alg_bytes

    M = global_batch // mb
    micro = [cv.make_input(shape, mb, seed + 1000 + m).to(dev) for m in range(M)]
    pipe = LayerPipeline.for_stack(stack, micro, rank, world, groups)

    def run(steps, first, last, host_in=None, host_out=None):
        # the ring stays primed between runs (last=False) except for the final one
        on_in = on_out = None
        if host_in is not None and rank == 0:
            def on_in(m):  # fresh hidden states enter at rank 0 from pinned host memory
                pipe.bufs[m].copy_(host_in[m], non_blocking=True)
        if host_out is not None and rank == world - 1:
            def on_out(m):
                host_out[m].copy_(pipe.bufs[m], non_blocking=True)
        for s in range(steps):
            pipe.step(first=first and s == 0, last=last and s == steps - 1, on_input=on_in,
                      on_output=on_out)
        pipe.drain()

    def timed(steps, last, host_in=None, host_out=None):
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run(steps, False, last, host_in, host_out)
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return ms.item() / steps

    run(args.warmup, True, False)
    with ClockSampler(dev.index or 0) as clk:
        ms_step = timed(args.steps, not with_e2e)
    out = {"ms": ms_step, "value": global_batch * 1000.0 / ms_step, "M": M, "mb": mb,
           "clocks": clk.summary()}
    if with_e2e:
        host_in = [x.cpu().pin_memory() for x in micro]
        host_out = [torch.empty_like(h).pin_memory() for h in host_in]
        e2e_ms = timed(args.steps, True, host_in, host_out)
        out["e2e"] = {"value": round(global_batch * 1000.0 / e2e_ms, 2), "unit": "tokens/s",
                      "h2d_bytes_per_step": int(sum(h.numel() for h in host_in) * 4),
                      "d2h_bytes_per_step": int(sum(h.numel() for h in host_out) * 4),
                      "ms_per_step": round(e2e_ms, 4)}
    # algorithmic bytes of this rank's layers per step (routing of the last step's
    # activations), summed over ranks
    step_bytes = 0
    for m in range(M):
        xb = pipe.bufs[m].clone()
        _, idx, _ = stack.stack(xb, routing=True)
        torch.cuda.synchronize()
        step_bytes += alg_bytes(stack, idx.cpu().numpy(), mb)[0]
    tb = torch.tensor([float(step_bytes)], device=dev)
    dist.all_reduce(tb)
    out["step_bytes"] = tb.item()
    pipe.close()
    del pipe
    torch.cuda.synchronize()
    dist.barrier()
    return out


def bench_main(args) -> None:
    """Config 1 over N GPUs (layer pipeline), as the configuration states it: a global
    batch of `args.batch` tokens (16) decoded as 4 micro-batches circulating through the
    N-stage pipeline; total work is fixed, so the scaling is strong.  The weak-scaling
    ring (`args.batch` tokens per GPU, one micro-batch per stage) is reported beside it."""
    import torch
    import torch.distributed as dist

    from . import build
    from . import converter as cv
    from .benchutil import peaks
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
    groups = [dist.new_group(list(range(world))), dist.new_group(list(range(world)))]
    B = args.batch
    mb = args.micro or max(1, B // 4)  # the configuration's 4 micro-batches
    if B % mb:
        raise SystemExit(f"micro-batch {mb} does not divide the global batch {B}")
    head = _measure_ring(stack, shape, rank, world, dev, groups, B, mb, args, seed, True)
    weak = _measure_ring(stack, shape, rank, world, dev, groups, B * world, B, args, seed,
                         False)
    for g in groups:
        dist.destroy_process_group(g)
    dist.destroy_process_group()
    if rank == 0:
        pk = peaks()
        achieved = head["step_bytes"] / world / (head["ms"] * 1e-3) / 1e9  # per GPU
        weak_gbs = weak["step_bytes"] / world / (weak["ms"] * 1e-3) / 1e9
        print(json.dumps({
            "metric": "MoE-block decode tokens/s (Mixtral-8x7B-shaped 32-block stack)",
            "value": round(head["value"], 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(head["ms"], 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4xf32",
            "data": "synthetic (seeded N(0,0.02) weights quantised int4 gs64; fp16 N(0,1) "
                    "inputs)",
            "config": {"workload": f"config1: Mixtral-8x7B-shaped {L}-block stack decode, global "
                                   f"batch {B} as {head['M']} micro-batches of {mb} through a "
                                   f"{world}-stage layer pipeline (NCCL send/recv)",
                       "global_batch": B, "parallelism": f"pp{world}",
                       "micro_batches": head["M"], "layers_per_rank": per,
                       "l2": "weights per step exceed L2"},
            "roofline": {"bound": "hbm", "kernel": "whole step per GPU (all kernels)",
                         "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": None,
                         "peak_source": pk["source"]},
            "clocks": head["clocks"],
            "e2e": head["e2e"],
            "gpu_launches": (launches_per_layer(shape, mb) * per + 2) * head["M"] * args.steps
                            * world,
            "weak_scaling": {"tokens_per_s": round(weak["value"], 2),
                             "ms_per_step": round(weak["ms"], 4), "global_batch": B * world,
                             "micro_batches": weak["M"], "micro_batch": B,
                             "hbm_gbs_per_gpu": round(weak_gbs, 1)},
        }), flush=True)


def ring_run(pipe, steps: int) -> None:
    """A complete ring of `steps` steps: empty before (rank 0 receives nothing on the
    first step) and empty after (the last step sends nothing back), so no send is in
    flight when it returns.  A device-wide synchronisation with a send in flight would
    wait for a receive the peer has not posted yet (NCCL completes a send larger than
    its staging buffer only when the receiver arrives): synchronise between rings."""
    for s in range(steps):
        pipe.step(first=s == 0, last=s == steps - 1)
    pipe.drain()


def layer_split(L: int, world: int) -> list[tuple[int, int]]:
    """Contiguous (first layer, count) per rank; the first L % world ranks get one more."""
    base, extra = divmod(L, world)
    out, l0 = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((l0, n))
        l0 += n
    return out


def graphs_for(run_one, bufs):
    """One CUDA graph per buffer of `run_one(buf)` (warmed once outside capture)."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        tmp = bufs[0].clone()
        run_one(tmp)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graphs = []
    for b in bufs:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run_one(b)
        graphs.append(g)
    return graphs


def bench_prefill_main(args) -> None:
    """Config 3 over N GPUs: the 58-layer DeepSeek-V3-shaped stack split into contiguous
    layer ranges, one config-3 request (a 4096-token prefill, then 128 decode steps at
    batch 32) through the layer pipeline: the prefill as max(8, N) micro-batches on the
    tensor-core path, the decode batch as 8 micro-batches of 4 on the stream kernels
    (total work fixed: strong scaling).  The prefill is timed as one pass through the
    ring (fill and drain included); the 128 decode steps from two ring lengths (their
    difference is the steady-state step, their offset the fill and drain).  The
    weak-scaling ring (N requests in flight, N micro-batches of a full 4096-token
    prefill / batch-32 decode step) is reported beside it."""
    import torch
    import torch.distributed as dist

    from . import build
    from . import converter as cv
    from .benchutil import ClockSampler, peaks
    from .moe import MoEStack

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if rank == 0:
        build.build()
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    dist.barrier()
    build.build()

    seed = 20251201 + 3
    L = args.c3_total_layers
    l0, nl = layer_split(L, world)[rank]
    shape = cv.MoEShape(hidden=7168, inter=2048, n_experts=256, top_k=8, shared_inter=2048,
                        n_layers=L)
    t0 = time.time()
    stack = MoEStack(shape, seed, device=dev, zipf_s=1.1, n_layers=nl, layer0=l0)
    setup_s = time.time() - t0
    groups = [dist.new_group(list(range(world))), dist.new_group(list(range(world)))]
    Tp, Bd, dsteps = 4096, 32, 128

    def timed_ring(pipe, steps):
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ring_run(pipe, steps)
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return ms.item()

    def prefill_pipe(mb, M):
        bufs = [cv.make_input(shape, mb, seed + 100 + m).to(dev) for m in range(M)]
        stack.prefill_workspace(mb)
        graphs = graphs_for(stack.prefill_stack, bufs)
        pipe = LayerPipeline(lambda m: graphs[m].replay(), bufs, rank, world, groups)
        pipe.graphs = graphs
        return pipe

    def decode_pipe(mb, M):
        din = [cv.make_input(shape, mb, seed + 200 + m).to(dev) for m in range(M)]
        return LayerPipeline.for_stack(stack, din, rank, world, groups)

    with ClockSampler(local) as clk:
        # one request
        Mp = max(8, world)
        ppipe = prefill_pipe(Tp // Mp, Mp)
        ring_run(ppipe, 1)  # warm
        p1_ms = timed_ring(ppipe, 1)
        ppipe.close()
        Md, mbd = 8, Bd // 8
        dpipe = decode_pipe(mbd, Md)
        ring_run(dpipe, max(3, args.warmup))
        s1, s2 = 2, 2 + max(2, args.c3_decode_steps // 8)
        t1, t2 = timed_ring(dpipe, s1), timed_ring(dpipe, s2)
        d_step = (t2 - t1) / (s2 - s1)
        d_total = t1 + (dsteps - s1) * d_step
        dpipe.close()
        del ppipe, dpipe
        # weak scaling: N requests in flight
        wp = prefill_pipe(args.prefill_micro, max(world, Tp // args.prefill_micro))
        ring_run(wp, 2)
        w1, w2 = timed_ring(wp, 2), timed_ring(wp, 2 + args.c3_prefill_steps)
        wp_ms = (w2 - w1) / args.c3_prefill_steps
        wMp = wp.M
        wp.close()
        wd = decode_pipe(Bd, world)
        ring_run(wd, max(3, args.warmup))
        v1, v2 = timed_ring(wd, 4), timed_ring(wd, 4 + args.c3_decode_steps)
        wd_ms = (v2 - v1) / args.c3_decode_steps
        wd.close()
        del wp, wd
    status = stack.prefill_status() | stack.status()
    st_t = torch.tensor([status], device=dev)
    dist.all_reduce(st_t, op=dist.ReduceOp.MAX)
    torch.cuda.synchronize()
    dist.barrier()
    for g in groups:
        dist.destroy_process_group(g)
    dist.destroy_process_group()
    if rank == 0:
        H, I, E, K = 7168, 2048, 256, 8
        flops = L * (2 * 3 * H * I * (Tp * K + Tp) + 2 * H * E * Tp)
        total_ms = p1_ms + d_total
        tokens = Tp + dsteps * Bd
        w_ptps = wMp * args.prefill_micro * 1000.0 / wp_ms
        w_dtps = world * Bd * 1000.0 / wd_ms
        w_total = world * Tp / w_ptps * 1e3 + world * dsteps * Bd / w_dtps * 1e3
        tflops_gpu = flops / (p1_ms * 1e-3) / 1e12 / world
        pk = peaks()
        print(json.dumps({
            "metric": "DeepSeek-V3-shaped 58-block stack: prefill 4096 + 128 decode steps at "
                      "batch 32, tokens/s", "value": round(tokens / total_ms * 1e3, 1),
            "unit": "tokens/s", "n_gpus": world, "steps": 1, "warmup": 1,
            "ms_per_step": round(total_ms, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int4xf16",
            "data": "synthetic (seeded N(0,0.02) weights quantised int4 gs64; fp16 N(0,1) "
                    "inputs)",
            "config": {"workload": f"config3: DeepSeek-V3-shaped {L}-layer stack, one request "
                                   f"through a {world}-stage layer pipeline: prefill of {Tp} "
                                   f"tokens as {Mp} micro-batches of {Tp // Mp}, {dsteps} decode "
                                   f"steps of batch {Bd} as {Md} micro-batches of {mbd}",
                       "parallelism": f"pp{world}", "layers_per_rank":
                       [n for _, n in layer_split(L, world)]},
            "prefill_ms": round(p1_ms, 2), "prefill_tflops_per_gpu": round(tflops_gpu, 1),
            "decode_ms_per_step": round(d_step, 3), "decode_ms_total": round(d_total, 1),
            "roofline": {"bound": "tensor", "achieved": round(tflops_gpu, 1),
                         "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(tflops_gpu / pk["bf16_tflops"], 4), "traffic": None,
                         "peak_source": pk["source"]},
            "weak_scaling": {"tokens_per_s": round(world * (Tp + dsteps * Bd) / w_total * 1e3, 1),
                             "requests_in_flight": world, "prefill_tokens_per_s": round(w_ptps, 1),
                             "decode_tokens_per_s": round(w_dtps, 1),
                             "prefill_micro_batches": wMp},
            "status": int(st_t.item()), "setup_s": round(setup_s, 1),
            "clocks": clk.summary()}), flush=True)
