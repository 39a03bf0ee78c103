"""Benchmark: Mixtral-8x7B-shaped MoE stack decode on B200.

One step = one decode step of a batch of tokens through 32 Mixtral-shaped MoE blocks
(router + top-2 softmax gating + int4 SwiGLU experts + gate-weighted combine, with
RMSNorm and the residual between blocks; attention = identity).  Seeded synthetic
weights (N(0, 0.02), quantised by the reference quantiser's rule) and inputs (fp16
N(0,1) upcast to fp32), generated on the GPU.

N = 1: the whole stack on one GPU, one CUDA graph per step, the global batch of 16
tokens in one pass (the configuration's 4-micro-batch schedule on one GPU, which only
serialises, is reported beside it as `pipeline_4mb`).
N > 1 (torchrun): layer pipeline -- rank r owns layers [32r/N, 32(r+1)/N); the global
batch of 16 tokens is split into the configuration's 4 micro-batches of 4 that flow
rank to rank with NCCL send/recv (torch.distributed), and the last rank hands each
micro-batch back to rank 0 for the next decode step.  Total work is fixed, so the
scaling is strong; the weak-scaling ring (16 tokens per GPU, N micro-batches of 16) is
reported beside it as `weak_scaling`.

Prints one JSON line (rank 0).  ``--impl reference`` times the reference engine's own
CPU run_moe (oracle/_ref, built from the reference sources) on a bounded sample of the
same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from wisp_b200.benchutil import ClockSampler, alg_bytes, peaks  # noqa: E402

METRIC = "MoE-block decode tokens/s (Mixtral-8x7B-shaped 32-block stack)"
UNIT = "tokens/s"
SEED = 20251201


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--batch", type=int, default=16, help="global batch of a decode step")
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--micro", type=int, default=0,
                   help="tokens per pipeline micro-batch (default: a quarter of the batch)")
    p.add_argument("--skip-cpu", action="store_true")
    p.add_argument("--skip-extra", action="store_true", help="no per-batch / e2e / profile legs")
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--decoder-pos", type=int, default=1023,
                   help="KV position of the decoder-step leg (0: skip the leg)")
    p.add_argument("--config3-layers", type=int, default=4,
                   help="resident DeepSeek-shaped layers of the config-3 leg (0 = skip)")
    p.add_argument("--c3-experts", type=int, default=256,
                   help="routed experts per config-3 layer (fewer: a small case for ncu)")
    p.add_argument("--c3-total-layers", type=int, default=58,
                   help="layers of the config-3 stack split over the ranks")
    p.add_argument("--prefill-micro", type=int, default=4096,
                   help="config-3 prefill micro-batch (tokens) of the multi-GPU ring")
    p.add_argument("--c3-prefill-steps", type=int, default=3)
    p.add_argument("--c3-prefill-tokens", type=int, default=4096,
                   help="prefill tokens of the one-GPU config-3 leg (config 3 is 4096; fewer: "
                        "a profiling case for the smaller-batch kernel variants)")
    p.add_argument("--c3-decode-steps", type=int, default=32)
    p.add_argument("--stream-layers", type=int, default=16,
                   help="layers of the config-4 host pool (6.3 GB each)")
    p.add_argument("--stream-steps", type=int, default=512)
    p.add_argument("--config4-layers", type=int, default=4,
                   help="layers of the config-4 leg of the default run (0 = skip)")
    p.add_argument("--config4-steps", type=int, default=128)
    p.add_argument("--workload", default="stack", choices=["stack", "ep", "prefill", "stream"],
                   help="stack: config 1 (default); ep: config 2, one DeepSeek-V3-shaped layer "
                        "expert-sharded over the GPUs, 64 tokens per GPU")
    return p.parse_args()


# --------------------------------------------------------------------------- CPU side
def write_ref_model(stack, layer: int, d: Path) -> None:
    """A one-layer converted-model directory holding `layer` of the GPU stack (so the
    reference CPU engine computes on exactly the bytes the GPU path reads)."""
    import numpy as np
    import torch
    from wisp_b200 import converter as cv
    (d / "experts").mkdir(parents=True, exist_ok=True)
    (d / "dense").mkdir(parents=True, exist_ok=True)
    H = stack.shape.hidden
    li = layer - stack.layer0
    for e, b in enumerate(stack.host_blobs(li)):
        raw = bytearray(b.tobytes())
        raw[8:12] = (0).to_bytes(4, "little")  # layer id 0 in this one-layer directory
        (d / "experts" / cv.expert_filename(0, e)).write_bytes(bytes(raw))
    lw = stack.layers[li]
    dense = {"embed_tokens": torch.zeros(2, H, dtype=torch.float16),
             "final_norm": torch.ones(H, dtype=torch.float16),
             "lm_head": torch.zeros(2, H, dtype=torch.float16),
             "layers.0.input_norm": torch.ones(H, dtype=torch.float16),
             "layers.0.post_norm": lw.norm.cpu(),
             "layers.0.attn.o_proj": torch.zeros(1, 1, dtype=torch.float16),
             "layers.0.router": lw.router.cpu()}
    if lw.router_bias is not None:
        dense["layers.0.router_bias"] = lw.router_bias.cpu()
    (d / "dense" / "model_dense.safetensors").write_bytes(cv._safetensors_bytes(dense))
    man = {"architecture": {"attention_type": "GQA", "num_layers": 1,
                            "num_experts_per_layer": stack.shape.n_experts,
                            "num_shared_experts": 0, "top_k_routing": stack.shape.top_k,
                            "hidden_size": H, "vocab_size": 2,
                            "moe_intermediate_size": stack.shape.inter,
                            "intermediate_size": stack.shape.inter, "num_attention_heads": 1,
                            "num_kv_heads": 1, "rms_norm_eps": stack.shape.rms_eps,
                            "max_position_embeddings": 16},
           "quantization": {"group_size": stack.shape.group_size},
           "performance": {"expert_size_bytes": stack.blob_bytes}}
    (d / "manifest.json").write_text(json.dumps(man))
    del np


def time_reference_cpu(model_dir: Path, x, seconds: float, threads: int):
    """Median seconds per token-block of the reference's own CPU run_moe."""
    from oracle import oracle as orc
    ref = orc.RefEngine(model_dir, threads=threads)
    y, idx, w = ref.moe(0, x[:1])  # warm: every routed expert now RAM-tier resident
    times = []
    t_end = time.time() + seconds
    while time.time() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        ref.moe(0, x[:1])
        times.append(time.perf_counter() - t0)
    ref.close()
    return statistics.median(times), len(times), y, idx, w


# --------------------------------------------------------------------------- GPU side
def run_single(args, dev) -> dict:
    import numpy as np
    import torch
    from wisp_b200 import converter as cv
    from wisp_b200.lib import lib
    from wisp_b200.moe import MoEStack

    shape = cv.MoEShape(hidden=4096, inter=14336, n_experts=8, top_k=2, n_layers=args.layers)
    t0 = time.time()
    stack = MoEStack(shape, SEED, device=dev)
    setup_s = time.time() - t0
    B = args.batch
    x0 = cv.make_input(shape, B, SEED).to(dev)
    x = x0.clone()
    stack.workspace(B)

    # capture one step into a graph (launch-bound inner loop -> one graph launch)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            x.copy_(x0)
            stack.stack(x)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    assert stack.status() == 0, "kernel status flag set"
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        stack.stack(x)

    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index or 0) as clk:
        ev0.record()
        for _ in range(args.steps):
            g.replay()
        ev1.record()
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    clocks = clk.summary()
    value = B * 1000.0 / ms

    # routing of one step -> algorithmic bytes
    x.copy_(x0)
    _, idx, _ = stack.stack(x, routing=True)
    torch.cuda.synchronize()
    idx_np = idx.cpu().numpy()
    step_bytes, gu_bytes = alg_bytes(stack, idx_np, B)

    out = {"ms": ms, "value": value, "clocks": clocks, "setup_s": setup_s,
           "step_bytes": step_bytes, "step_gbs": step_bytes / ms / 1e6}

    # per-kernel durations (profiling pass, events between launches).  The
    # library launches prep[+router]+gateup+down per layer and a final prep;
    # whether the router runs inside prep is read off the recorded count.
    n_prof = 3
    n_ev = (4 * args.layers + 2) * n_prof + 4
    events = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    handles = (C_void_p_array(events))
    lib().wisp_moe_profile_events(handles, n_ev)
    for _ in range(n_prof):
        x.copy_(x0)
        stack.stack(x)
    recorded = lib().wisp_moe_profile_count()
    lib().wisp_moe_profile_events(None, 0)
    torch.cuda.synchronize()
    per = recorded // n_prof - 1
    seq = ["prep", "gateup", "down"] if per == 3 * args.layers + 1 else \
        ["prep", "router", "gateup", "down"]
    assert per == len(seq) * args.layers + 1, (recorded, per)
    names = seq * args.layers + ["final"]
    dur = {k: [] for k in seq + ["final"]}
    gu_durs = []
    for r in range(n_prof):
        base = r * (per + 1)
        for j in range(per):
            dt = events[base + j].elapsed_time(events[base + j + 1])
            dur[names[j]].append(dt)
            if names[j] == "gateup":
                gu_durs.append(dt)
    gu_ms = statistics.mean(gu_durs)
    gu_alg = statistics.mean(gu_bytes)
    pk = peaks()
    achieved = gu_alg / (gu_ms * 1e-3) / 1e9
    # DRAM bytes per gate/up launch from the committed ncu capture of the same
    # workload (Mixtral-shaped layer, decode batch 16), when the batch matches
    traffic = None
    tf = ROOT / "profiles" / "roofline_traffic.json"
    if tf.exists() and B == 16:
        traffic = json.loads(tf.read_text())["gateup_kernel"]["dram_bytes_per_launch"]
    out["roofline"] = {"bound": "hbm", "kernel": "gateup_kernel (int4 gate/up + SwiGLU stream)",
                       "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                       "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": traffic,
                       "alg_bytes_per_launch": int(gu_alg), "avg_launch_ms": round(gu_ms, 5),
                       "peak_source": pk["source"] + " (MEASURED_PEAKS.json hbm_gbs)"}
    out["kernel_ms_mean"] = {k: round(statistics.mean(v), 5) for k, v in dur.items() if v}
    dn_alg = statistics.mean(gu_bytes) / 2  # down = one matrix per expert vs two
    out["down_gbs"] = round(dn_alg / (statistics.mean(dur["down"]) * 1e-3) / 1e9, 1)

    if not args.skip_extra:
        # e2e through the C ABI with host buffers: H2D of x, the stack, D2H of the result
        xh = x0.cpu().pin_memory()
        yh = torch.empty_like(xh).pin_memory()
        for _ in range(3):
            x.copy_(xh, non_blocking=True)
            g.replay()
            yh.copy_(x, non_blocking=True)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            x.copy_(xh, non_blocking=True)
            g.replay()
            yh.copy_(x, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        out["e2e"] = {"value": round(B * 1000.0 / e2e_ms, 2), "unit": UNIT,
                      "h2d_bytes_per_step": xh.numel() * 4, "d2h_bytes_per_step": yh.numel() * 4,
                      "ms_per_step": round(e2e_ms, 4)}
        # other batch sizes of config 1 (graph per batch)
        per_batch = {}
        for b in (1, 4):
            if b == B:
                continue
            xb0 = cv.make_input(shape, b, SEED + b).to(dev)
            xb = xb0.clone()
            stack.workspace(max(B, b))
            with torch.cuda.stream(s):
                stack.stack(xb)
            torch.cuda.synchronize()
            gb = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gb):
                stack.stack(xb)
            for _ in range(3):
                gb.replay()
            torch.cuda.synchronize()
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            nb = max(10, args.steps // 2)
            a0.record()
            for _ in range(nb):
                gb.replay()
            a1.record()
            torch.cuda.synchronize()
            bm = a0.elapsed_time(a1) / nb
            xb.copy_(xb0)
            _, ib, _ = stack.stack(xb, routing=True)
            torch.cuda.synchronize()
            sb, _ = alg_bytes(stack, ib.cpu().numpy(), b)
            per_batch[str(b)] = {"tokens_per_s": round(b * 1000.0 / bm, 1), "ms_per_step": round(bm, 4),
                                 "hbm_gbs": round(sb / bm / 1e6, 1)}
            del gb
        out["per_batch"] = per_batch
        # config 0: one Mixtral block (no norm/residual), 1 token, graph of the block
        x1 = cv.make_input(shape, 1, SEED + 7).to(dev)
        y1 = torch.empty_like(x1)
        stack.workspace(max(B, 1))
        with torch.cuda.stream(s):
            stack.block(0, x1, y1)
        torch.cuda.synchronize()
        g0 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g0):
            stack.block(0, x1, y1)
        for _ in range(5):
            g0.replay()
        torch.cuda.synchronize()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        nb = 200
        b0.record()
        for _ in range(nb):
            g0.replay()
        b1.record()
        torch.cuda.synchronize()
        blk_ms = b0.elapsed_time(b1) / nb
        _, i0, _ = stack.block(0, x1, y1, routing=True)
        torch.cuda.synchronize()
        blk_bytes, _ = alg_bytes(stack, i0.cpu().numpy()[None], 1)
        gbs = blk_bytes / blk_ms / 1e6
        out["config0"] = {"workload": "one Mixtral-shaped MoE block, decode batch 1 (graph of "
                                      "back-to-back blocks)",
                          "us_per_block": round(blk_ms * 1e3, 2),
                          "blocks_per_s": round(1000.0 / blk_ms, 1),
                          "alg_bytes_per_block": int(blk_bytes), "hbm_gbs": round(gbs, 1),
                          "frac_of_measured_hbm": round(gbs / peaks()["hbm_gbs"], 4)}
        del g0

    if not args.skip_extra and args.decoder_pos > 0:
        # an extra leg: its failure is recorded, not fatal to the headline line
        try:
            out["decoder_step"] = run_decoder(args, dev, stack, shape, s)
        except Exception as e:  # noqa: BLE001
            out["decoder_step"] = {"error": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.empty_cache()

    if not args.skip_extra and args.config3_layers > 0:
        # an extra leg: its failure is recorded, not fatal to the headline line
        try:
            out["config3"] = run_config3(args, dev, args.config3_layers)
        except Exception as e:  # noqa: BLE001
            out["config3"] = {"error": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.empty_cache()

    if not args.skip_extra and args.config4_layers > 0:
        # an extra leg: its failure is recorded, not fatal to the headline line
        try:
            out["config4"] = run_config4(args, dev, args.config4_layers, args.config4_steps)
        except Exception as e:  # noqa: BLE001
            out["config4"] = {"error": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.empty_cache()

    # CPU baseline + parity on the same bytes: layer 0, token 0
    if not args.skip_cpu:
        threads = len(os.sched_getaffinity(0))
        with tempfile.TemporaryDirectory() as td:
            d = Path(td) / "mx1"
            write_ref_model(stack, 0, d)
            xin = x0[:1].cpu().numpy()
            t_blk, n, yref, iref, _ = time_reference_cpu(d, xin, args.cpu_seconds, threads)
        yg, ig, _ = stack.block(0, x0[:1], routing=True)
        torch.cuda.synchronize()
        yg = yg.cpu().numpy()
        out["cpu_baseline"] = {"value": round(1.0 / (t_blk * args.layers), 4), "unit": UNIT,
                               "cores": threads, "kind": "reference",
                               "sample": f"reference run_moe (oracle/_ref), layer 0 of this stack, "
                                         f"1 token, warm RAM tier, median of {n} runs = "
                                         f"{t_blk * 1e3:.1f} ms/token-block, x{args.layers} blocks"}
        out["parity"] = {"idx_equal": bool(np.array_equal(ig.cpu().numpy(), iref)),
                         "max_abs": float(np.abs(yg - yref).max()),
                         "rel_l2": float(np.linalg.norm(yg - yref) / np.linalg.norm(yref))}
    # per layer, the final combine, and the zeroing of the workspace state
    out["gpu_launches_per_step"] = len(seq) * args.layers + 2
    del g
    return out


def run_decoder(args, dev, stack, shape, s) -> dict:
    """The whole decoder step at batch 1 on the config-1 stack: per layer the fused GQA
    attention block (Mixtral-8x7B shapes: 32 heads over 8 kv heads of 128, rotary,
    fp16 KV cache holding `decoder_pos` earlier positions) + RMSNorm + the MoE block +
    the residual, then the logits over a 32000-token vocabulary; one CUDA graph per
    token, every weight resident (random fp16 attention / embedding / lm_head weights:
    no checkpoint is available)."""
    import ctypes as C
    import torch
    from wisp_b200.lib import WispAttnLayer, WispErrCtx, check, lib
    H, L, nh, nkv, hd, vocab = shape.hidden, args.layers, 32, 8, 128, 32000
    pos, max_seq = args.decoder_pos, args.decoder_pos + 1
    g = torch.Generator(device=dev)
    g.manual_seed(SEED + 11)

    def w(*sz, std):
        return (torch.randn(*sz, generator=g, device=dev) * std).half()

    attn = []
    for _ in range(L):
        attn.append({"input_norm": torch.ones(H, dtype=torch.float16, device=dev),
                     "q": w(nh * hd, H, std=0.5 / H ** 0.5), "k": w(nkv * hd, H, std=0.5 / H ** 0.5),
                     "v": w(nkv * hd, H, std=1.0 / H ** 0.5),
                     "o": w(H, nh * hd, std=0.5 / (nh * hd) ** 0.5)})
    embed, lm_head = w(vocab, H, std=0.02), w(vocab, H, std=0.02)
    final_norm = torch.ones(H, dtype=torch.float16, device=dev)
    Kc = w(L, max_seq, nkv, hd, std=1.0)
    Vc = w(L, max_seq, nkv, hd, std=1.0)
    layers = [WispAttnLayer(a["input_norm"].data_ptr(), a["q"].data_ptr(), a["k"].data_ptr(),
                            a["v"].data_ptr(), a["o"].data_ptr(), H, nh, nkv, hd, 500000.0,
                            shape.rms_eps) for a in attn]
    n_ws = int(lib().wisp_attn_workspace_bytes(C.byref(layers[0]), max_seq))
    ws = torch.zeros(n_ws, dtype=torch.uint8, device=dev)  # zero before first use
    x = torch.empty((1, H), dtype=torch.float32, device=dev)
    logits = torch.empty(vocab, dtype=torch.float32, device=dev)
    lws = torch.empty(H, dtype=torch.float32, device=dev)
    stack.workspace(max(args.batch, 1))
    err = WispErrCtx()

    def step(with_moe=True):
        cs = torch.cuda.current_stream().cuda_stream
        lib().wisp_gpu_embed_lookup(embed.data_ptr(), 7, x.data_ptr(), H, cs)
        for l in range(L):
            check(lib().wisp_attn_decode(C.byref(layers[l]), x.data_ptr(), Kc[l].data_ptr(),
                                         Vc[l].data_ptr(), pos, max_seq, ws.data_ptr(), n_ws, cs,
                                         C.byref(err)), err)
            if with_moe:  # x += MoE_l(rmsnorm(x)): the fused one-layer stack
                stack.stack(x, layers=1, layer0=l)
        check(lib().wisp_lm_head_forward(final_norm.data_ptr(), lm_head.data_ptr(), x.data_ptr(),
                                         logits.data_ptr(), vocab, H, C.c_float(shape.rms_eps),
                                         lws.data_ptr(), lws.numel() * 4, cs, C.byref(err)), err)

    def timed(with_moe):
        with torch.cuda.stream(s):
            step(with_moe)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            step(with_moe)
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(10, args.steps // 2)
        e0.record()
        for _ in range(n):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        del gr
        return e0.elapsed_time(e1) / n

    ms = timed(True)
    ms_attn = timed(False)  # embedding + attention blocks + logits only
    assert stack.status() == 0, "kernel status flag set"
    assert bool(torch.isfinite(logits).all()), "non-finite logits"
    # bytes the attention half must read: its weights, the KV cache up to pos, the
    # embedding row and lm_head
    attn_bytes = L * ((2 * nh * hd * H + 2 * nkv * hd * H) * 2 + 2 * max_seq * nkv * hd * 2) \
        + vocab * H * 2 + H * 2
    return {"workload": f"Mixtral-8x7B-shaped decoder step at batch 1: {L} x (GQA attention "
                        f"32/8 heads x 128, KV position {pos} + MoE block) + logits over {vocab}",
            "ms_per_token": round(ms, 4), "tokens_per_s": round(1000.0 / ms, 1),
            "attention_and_logits_ms": round(ms_attn, 4),
            "attention_hbm_gbs": round(attn_bytes / ms_attn / 1e6, 1),
            "attention_frac_of_measured_hbm": round(attn_bytes / ms_attn / 1e6 / peaks()["hbm_gbs"], 4),
            "attention_alg_bytes": int(attn_bytes)}


def run_config3(args, dev, k: int) -> dict:
    """Config 3 on one GPU: a resident k-layer slice of the DeepSeek-V3-shaped stack
    (7168 / 2048, 256 experts, top-8, shared expert, Zipf(1.1) routing), prefill of
    4096 tokens on the tensor-core path, then 128 decode steps at batch 32 on the decode
    path (one CUDA graph per step).  The 58-layer pool (368 GB) does not fit one GPU:
    times are normalised per layer (x 58 / k)."""
    import numpy as np
    import torch
    from wisp_b200 import converter as cv
    from wisp_b200.moe import MoEStack
    E = args.c3_experts
    shape = cv.MoEShape(hidden=7168, inter=2048, n_experts=E, top_k=8, shared_inter=2048,
                        n_layers=k)
    t0 = time.time()
    st = MoEStack(shape, SEED + 3, device=dev, zipf_s=1.1)
    setup_s = time.time() - t0
    Tp, Bd, steps = args.c3_prefill_tokens, 32, 128
    xp0 = cv.make_input(shape, Tp, SEED + 3).to(dev)
    xp = xp0.clone()
    for _ in range(2):
        xp.copy_(xp0)
        st.prefill_stack(xp)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    ms = []
    with ClockSampler(dev.index or 0) as clk:
        for _ in range(reps):
            xp.copy_(xp0)  # a flush of L2 too: 117 MB
            e0.record()
            st.prefill_stack(xp)
            e1.record()
            torch.cuda.synchronize()
            ms.append(e0.elapsed_time(e1))
    pre_ms = statistics.median(ms)
    status = st.prefill_status()
    _, idx, _ = st.prefill_stack(xp0.clone(), routing=True)
    torch.cuda.synchronize()
    H, I, K = 7168, 2048, 8
    flops_layer = 2 * 3 * H * I * (Tp * K + Tp) + 2 * H * E * Tp
    tflops = k * flops_layer / pre_ms / 1e9
    # decode: batch 32, one graph per step
    xd0 = cv.make_input(shape, Bd, SEED + 5).to(dev)
    xd = xd0.clone()
    st.workspace(Bd)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        st.stack(xd)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st.stack(xd)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    xd.copy_(xd0)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    dec_ms = e0.elapsed_time(e1) / steps
    dstatus = st.status()
    del g
    scale = 58.0 / k
    total_ms = (pre_ms + steps * dec_ms) * scale
    cnt = np.bincount(idx[0].cpu().numpy().reshape(-1), minlength=E)
    return {
        "workload": f"config3: DeepSeek-V3-shaped stack ({E} routed experts), resident "
                    f"{k}-layer slice, prefill "
                    f"{Tp} tokens (tensor-core grouped GEMM) then {steps} decode steps at batch "
                    f"{Bd}; times x58/{k} for the 58-layer stack (368 GB does not fit one GPU)",
        "layers_resident": k, "setup_s": round(setup_s, 1),
        "prefill_ms_per_layer": round(pre_ms / k, 3),
        "prefill_tokens_per_s": round(Tp / (pre_ms * scale) * 1e3, 1),
        "prefill_tflops": round(tflops, 1),
        "prefill_frac_of_measured_bf16": round(tflops / peaks()["bf16_tflops"], 4),
        "decode_ms_per_layer_step": round(dec_ms / k, 4),
        "decode_tokens_per_s": round(Bd / (dec_ms * scale) * 1e3, 1),
        "config3_total_ms": round(total_ms, 1),
        "config3_tokens_per_s": round((Tp + steps * Bd) / total_ms * 1e3, 1),
        "max_tokens_per_expert_layer0": int(cnt.max()),
        "status": int(status | dstatus), "clocks": clk.summary(),
    }


def C_void_p_array(events):
    """Raw cudaEvent_t handles (torch creates events lazily: record each once first)."""
    import ctypes as C
    import torch
    for e in events:
        e.record()
    torch.cuda.synchronize()
    arr = (C.c_void_p * len(events))()
    for i, e in enumerate(events):
        arr[i] = e.cuda_event
    return arr


def main_ours(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        from wisp_b200 import pipeline
        return pipeline.bench_main(args)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from wisp_b200 import build
    build.build()
    r = run_single(args, dev)
    line = {
        "metric": METRIC, "value": round(r["value"], 2), "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms"], 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int4xf32",
        "precision": "int4 weights with fp16 scale/zero per 64; activations entered as two "
                     "int8 digits per quant group (|error| <= 1.6e-5 * max|x| of the group), "
                     "exact int32 MMA sums, fp32 epilogue, combine and norm",
        "data": "synthetic (seeded N(0,0.02) weights quantised int4 gs64; fp16 N(0,1) inputs)",
        "config": {"workload": f"config1: Mixtral-8x7B-shaped stack, {args.layers} MoE blocks, "
                               f"decode global batch {args.batch} in one pass on one GPU, "
                               f"attention=identity, RMSNorm eps 1e-5",
                   "global_batch": args.batch, "layers": args.layers, "hidden": 4096,
                   "inter": 14336, "experts": 8, "top_k": 2, "group_size": 64,
                   "parallelism": "single GPU", "l2": "weights per step (>=6 GB) exceed L2",
                   "graph": "one CUDA graph per step, PDL between kernels"},
        "roofline": r["roofline"], "clocks": r["clocks"],
        "gpu_launches": r["gpu_launches_per_step"] * args.steps,
        "step_hbm_gbs": round(r["step_gbs"], 1), "kernel_ms_mean": r["kernel_ms_mean"],
    }
    for k in ("e2e", "per_batch", "config0", "decoder_step", "config3", "config4", "cpu_baseline",
              "parity"):
        if k in r:
            line[k] = r[k]
    q = r.get("per_batch", {}).get(str(max(1, args.batch // 4)))
    if q and args.batch % 4 == 0:
        # the configuration's 4 micro-batches on one GPU run one after another
        line["pipeline_4mb"] = {"tokens_per_s": round(args.batch * 1000.0 / (4 * q["ms_per_step"]), 1),
                                "ms_per_step": round(4 * q["ms_per_step"], 4),
                                "micro_batches": 4, "micro_batch": args.batch // 4}
    print(json.dumps(line), flush=True)


def main_ep(args):
    """Config 2: one DeepSeek-V3-shaped MoE layer (256 routed experts, top-8, shared
    expert, Zipf(1.1) router bias) expert-sharded over N GPUs (256/N experts each),
    decode batch 64 in total (64/N tokens routed on each GPU), three NCCL all-to-alls
    per step (wisp_b200.ep.Dispatch); the total work is fixed, so the scaling is strong.
    The weak-scaling figure (64 tokens per GPU) is reported beside it."""
    import datetime
    import numpy as np
    import torch
    import torch.distributed as dist
    from wisp_b200 import build
    from wisp_b200 import converter as cv
    from wisp_b200.ep import EPLayer
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if rank == 0:
        build.build()
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
        dist.barrier()
    B_total = 64
    if B_total % world:
        raise SystemExit(f"64 tokens do not split over {world} GPUs")
    shape = cv.MoEShape(hidden=7168, inter=2048, n_experts=256, top_k=8, shared_inter=2048)
    ep = EPLayer(shape, SEED, rank, world, dev, zipf_s=1.1)

    def timed(x, steps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            ep.forward(x)
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return ms.item()

    def measure(B):
        x = cv.make_input(shape, B, SEED + 100 * rank).to(dev)
        for _ in range(max(3, args.warmup)):
            ep.forward(x)
        with ClockSampler(local) as clk:
            ms = timed(x, args.steps)
        # algorithmic bytes on this GPU per step: distinct local experts routed to it by
        # any rank + the shared expert + the router
        _, idx, _ = ep.forward(x)
        ids = idx.reshape(-1).to(dev)
        if world > 1:
            allidx = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(allidx, ids)
            ids = torch.cat(allidx)
        ids = ids.cpu().numpy()
        mine = np.unique(ids[(ids >= rank * ep.per) & (ids < (rank + 1) * ep.per)])
        blob = ep.local.blob_bytes - cv.HEADER_BYTES
        step_bytes = (len(mine) + 1) * blob + shape.n_experts * shape.hidden * 2
        tb = torch.tensor([float(step_bytes)], device=dev)
        if world > 1:
            dist.all_reduce(tb, op=dist.ReduceOp.MAX)
        return ms, tb.item(), clk.summary()

    ms, tb, clocks = measure(B_total // world)
    ms_w, tb_w, _ = measure(B_total)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        pk = peaks()
        gbs = tb / (ms * 1e-3) / 1e9
        print(json.dumps({
            "metric": "MoE-block decode tokens/s (DeepSeek-V3-shaped layer, expert parallel)",
            "value": round(B_total * 1000.0 / ms, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4xf32", "data": "synthetic (seeded; Zipf(1.1) router bias)",
            "config": {"workload": f"config2: DeepSeek-V3-shaped MoE layer (H 7168, 256 experts "
                                   f"top-8 + shared, inter 2048), decode batch {B_total} in "
                                   f"total ({B_total // world} per GPU), experts sharded over "
                                   f"{world} GPU(s), 3 NCCL all-to-alls per step",
                       "global_batch": B_total, "parallelism": f"ep{world}"},
            "roofline": {"bound": "hbm", "kernel": "whole step, most loaded GPU",
                         "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / pk["hbm_gbs"], 4), "traffic": None},
            "clocks": clocks,
            "weak_scaling": {"tokens_per_s": round(B_total * world * 1000.0 / ms_w, 2),
                             "ms_per_step": round(ms_w, 4), "tokens_per_gpu": B_total,
                             "hbm_gbs_most_loaded": round(tb_w / (ms_w * 1e-3) / 1e9, 1)}}),
              flush=True)


def main_prefill(args):
    """Config 3 as the headline line: one GPU (run_config3, per-layer normalised) or the
    layer pipeline over N GPUs (wisp_b200.pipeline.bench_prefill_main)."""
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        from wisp_b200 import pipeline
        return pipeline.bench_prefill_main(args)
    import torch
    from wisp_b200 import build
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    build.build()
    k = args.config3_layers or 4
    r = run_config3(args, dev, k)
    print(json.dumps({
        "metric": "DeepSeek-V3-shaped 58-block stack: prefill 4096 + 128 decode steps at batch "
                  "32, tokens/s", "value": r["config3_tokens_per_s"], "unit": "tokens/s",
        "n_gpus": 1, "steps": 1, "warmup": 2, "ms_per_step": r["config3_total_ms"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int4xf16",
        "data": "synthetic (seeded N(0,0.02) weights quantised int4 gs64; fp16 N(0,1) inputs)",
        "config": {"workload": r["workload"], "parallelism": "single GPU (per-layer normalised)"},
        "roofline": {"bound": "tensor", "achieved": r["prefill_tflops"],
                     "peak": peaks()["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": r["prefill_frac_of_measured_bf16"], "traffic": None,
                     "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops), of measured"},
        "clocks": r["clocks"], "config3": r}), flush=True)


def run_config4(args, dev, L: int, steps: int) -> dict:
    """Config 4 on `L` DeepSeek-V3-shaped layers in pinned host RAM behind an HBM cache
    of the reference configuration's cache/pool ratio (80 GB / 340 GB), decode batch 1,
    Zipf(1.1) routing.  Three sessions of `steps` tokens on the same inputs, each from a
    cold cache: the next layer's router lookahead alone; with the frequency predictor
    (wisp_b200.tier_cache); and with the predictor after a pre-warm from the learning
    cache (wisp_b200.learning_cache) of an earlier session on other inputs."""
    import tempfile
    import torch
    from wisp_b200 import converter as cv
    from wisp_b200.learning_cache import LearningCache
    from wisp_b200.stream import StreamingStack
    from wisp_b200.tier_cache import ExpertPredictor
    shape = cv.MoEShape(hidden=7168, inter=2048, n_experts=256, top_k=8, shared_inter=2048,
                        n_layers=L)
    slots = int(round(80.0 / 340.0 * L * shape.n_experts))
    t0 = time.time()
    ss = StreamingStack(shape, SEED + 11, L, slots, dev, zipf_s=1.1)
    setup_s = time.time() - t0
    # host-to-device copy peak of this box: one 2 GiB pinned copy
    hb = torch.empty(2 << 30, dtype=torch.uint8, pin_memory=True)
    db = torch.empty(2 << 30, dtype=torch.uint8, device=dev)
    db.copy_(hb, non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    db.copy_(hb, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    h2d_peak = (2 << 30) / e0.elapsed_time(e1) / 1e6
    del hb, db
    x = torch.empty((1, shape.hidden), dtype=torch.float32, device=dev)

    def session(xs, predictor=None, record=None):
        s0 = ss.stats()
        e0.record()
        for i in range(xs.shape[0]):
            x.copy_(xs[i:i + 1])
            ss.step(x, predictor=predictor)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        s1 = ss.stats()
        d = {k: s1[k] - s0[k] for k in ("hits", "misses", "prefetched", "prefetch_used", "bytes")}
        gbs = d["bytes"] / ms / 1e6
        return {"tokens_per_s": round(xs.shape[0] / ms * 1e3, 2),
                "ms_per_step": round(ms / xs.shape[0], 3),
                "hit_rate": round(d["hits"] / max(1, d["hits"] + d["misses"]), 4),
                "misses_per_token": round(d["misses"] / xs.shape[0], 2),
                "prefetched_per_token": round(d["prefetched"] / xs.shape[0], 2),
                "prefetch_used_frac": round(d["prefetch_used"] / max(1, d["prefetched"]), 4),
                "h2d_gbs": round(gbs, 2), "h2d_frac_of_peak": round(gbs / h2d_peak, 4)}

    xs = cv.make_input(shape, steps, SEED + 12).to(dev)
    hist = cv.make_input(shape, steps, SEED + 13).to(dev)
    # one unmeasured session first: the first copies and launches of a process carry
    # one-time costs that would otherwise land on the first measured session
    ss.reset()
    session(hist[: max(4, steps // 8)], ExpertPredictor(L, shape.top_k))
    with ClockSampler(dev.index or 0) as clk:
        ss.reset()
        plain = session(xs)
        ss.reset()
        pred = session(xs, ExpertPredictor(L, shape.top_k))
        with tempfile.TemporaryDirectory() as td:
            # an earlier session on other inputs writes the usage record ...
            lc = LearningCache(td)
            ss.reset()
            session(hist, ExpertPredictor(L, shape.top_k, lc))
            lc.save()
            # ... which the next start loads and pre-warms the cold cache from
            lc2 = LearningCache(td)
            lc2.load()
            ss.reset()
            warmed = ss.prewarm(lc2.get_hot_experts(slots))
            warm = session(xs, ExpertPredictor(L, shape.top_k))
    status = ss.status()
    out = {"workload": f"config4: {L}-layer DeepSeek-V3-shaped pool ({ss.pool_bytes / 1e9:.1f} GB "
                       f"pinned host) through a {slots}-slot HBM cache "
                       f"({slots * ss.blob_bytes / 1e9:.1f} GB, the 80/340 ratio), decode batch 1, "
                       f"Zipf(1.1), {steps} tokens per session from a cold cache",
           "layers": L, "cache_slots": slots, "h2d_peak_gbs": round(h2d_peak, 2),
           "router_lookahead": plain, "with_frequency_predictor": pred,
           "with_predictor_and_prewarm": dict(warm, prewarmed_experts=warmed),
           "setup_s": round(setup_s, 1), "status": status, "clocks": clk.summary()}
    ss.close()
    return out


def main_stream(args):
    """Config 4 as the headline line (run_config4): the router-lookahead session is the
    value; the predictor and pre-warm sessions ride beside it.  The 58-layer 368 GB pool
    does not fit this box's host RAM (196 GB): the pool is --stream-layers layers and
    the cache keeps the reference configuration's cache/pool ratio (80 GB / 340 GB)."""
    import torch
    from wisp_b200 import build
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    build.build()
    r = run_config4(args, dev, args.stream_layers, args.stream_steps)
    p = r["router_lookahead"]
    print(json.dumps({
        "metric": "oversubscribed decode tokens/s (DeepSeek-V3-shaped pool in pinned host "
                  "RAM, HBM expert cache under LRU)", "value": p["tokens_per_s"],
        "unit": "tokens/s", "n_gpus": 1, "steps": args.stream_steps, "warmup": 0,
        "ms_per_step": p["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int4xf32",
        "data": "synthetic (seeded N(0,0.02) weights quantised int4 gs64; fp16 N(0,1) inputs)",
        "config": {"workload": r["workload"], "layers": r["layers"],
                   "cache_slots": r["cache_slots"],
                   "prefetch": "next layer's router on this layer's input"},
        "hit_rate": p["hit_rate"], "h2d_gbs": p["h2d_gbs"],
        "roofline": {"bound": "host link", "achieved": p["h2d_gbs"], "peak": r["h2d_peak_gbs"],
                     "unit": "GB/s", "frac": p["h2d_frac_of_peak"], "traffic": None,
                     "peak_source": "measured in this run (2 GiB pinned host-to-device copy)"},
        "config4": r, "clocks": r["clocks"]}), flush=True)


def main_reference(args):
    """The reference's own CPU implementation (run_moe, built from its sources), all host
    threads, bounded sample: each step = 1 token through one Mixtral-shaped block, the
    metric extrapolated to the 32-block stack."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    from oracle import oracle as orc
    if orc.ref_lib() is None:
        print(json.dumps({"impl": "reference", "unavailable": "reference harness "
                          "oracle/_ref/libwisp_ref.so was not built"}))
        return
    from wisp_b200 import converter as cv
    threads = len(os.sched_getaffinity(0))
    shape = cv.MoEShape(hidden=4096, inter=14336, n_experts=8, top_k=2, n_layers=1)
    with tempfile.TemporaryDirectory() as td:
        d = Path(td) / "mx1"
        # the model directory comes from the CPU converter (same seeded recipe, CPU
        # generator): this arm never loads libwisp_b200 or touches the GPU
        cv.write_model_dir(d, shape, SEED)
        x = cv.make_input(shape, 1, SEED).numpy()
        ref = orc.RefEngine(d, threads=threads)
        for _ in range(max(1, args.warmup)):
            ref.moe(0, x)
        steps = max(1, min(args.steps, 40))
        t0 = time.perf_counter()
        for _ in range(steps):
            ref.moe(0, x)
        dt = (time.perf_counter() - t0) / steps
        ref.close()
    maps = Path("/proc/self/maps")
    if maps.exists() and "libwisp_b200" in maps.read_text():
        raise RuntimeError("the reference arm must not load libwisp_b200")
    value = 1.0 / (dt * 32)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int4xf32", "data": "synthetic",
        "config": {"workload": "config1: Mixtral-8x7B-shaped 32-block stack decode, sampled "
                               "as 1 token x 1 block per step, x32 blocks"},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads,
                         "kind": "reference",
                         "sample": f"1 token through one Mixtral block per step ({steps} steps), "
                                   "warm RAM tier, extrapolated x32 blocks"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)
    del np


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        main_reference(a)
    elif a.workload == "ep":
        main_ep(a)
    elif a.workload == "prefill":
        main_prefill(a)
    elif a.workload == "stream":
        main_stream(a)
    else:
        main_ours(a)
