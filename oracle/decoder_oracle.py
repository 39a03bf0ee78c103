"""TEST INFRASTRUCTURE ONLY (the checker, never the product): numpy restatements of
the reference's CPU decoder-step operations, used by the tests to check the CUDA
kernels of wisp_b200/csrc/decoder.cu at sizes the reference harness does not reach
cheaply (long KV caches, many heads, MLA-style aliased values).  Computed in float64
unless stated; the fp16 rounding points (the KV cache, the weights) are the
reference's.

Pinned: the whole decoder step is pinned separately against the reference's own
decode_step (oracle/_ref, tests/golden/decode_golden.*); these functions restate the
pieces of it.
"""

from __future__ import annotations

import numpy as np


def rmsnorm(x: np.ndarray, w: np.ndarray | None, eps: float) -> np.ndarray:
    """cpu_rmsnorm (csrc/core/wisp_engine.c:415-422): double sum of squares."""
    x = np.asarray(x, np.float64)
    scale = 1.0 / np.sqrt((x * x).sum() / x.size + eps)
    return x * scale * (1.0 if w is None else np.asarray(w, np.float64))


def rope(v: np.ndarray, n_heads: int, head_stride: int, rope_off: int, rope_dim: int,
         pos: int, theta: float) -> np.ndarray:
    """cpu_rope (wisp_engine.c:446-460): neox pairs (i, i + rope_dim/2) per head."""
    out = np.array(v, np.float64, copy=True)
    half = rope_dim // 2
    i = np.arange(half, dtype=np.float64)
    freq = theta ** (-2.0 * i / rope_dim)
    ang = pos * freq
    c, s = np.cos(ang), np.sin(ang)
    for h in range(n_heads):
        base = h * head_stride + rope_off
        a = out[base:base + half].copy()
        b = out[base + half:base + rope_dim].copy()
        out[base:base + half] = a * c - b * s
        out[base + half:base + rope_dim] = b * c + a * s
    return out


def attention(q: np.ndarray, K: np.ndarray, V: np.ndarray | None, seq: int, n_heads: int,
              kv_heads: int, k_dim: int, v_dim: int, scale: float) -> np.ndarray:
    """cpu_attention (wisp_engine.c:465-505): per head, softmax over the first `seq`
    positions of q . K * scale, then the weighted sum of V.  K [seq][kv_heads][k_dim]
    and V [seq][kv_heads][v_dim] as stored (fp16 values); V None: the first v_dim
    dims of K (MLA)."""
    group = n_heads // kv_heads
    Kf = np.asarray(K, np.float64).reshape(-1, kv_heads, k_dim)[:seq]
    Vf = (Kf[:, :, :v_dim] if V is None
          else np.asarray(V, np.float64).reshape(-1, kv_heads, v_dim)[:seq])
    qf = np.asarray(q, np.float64).reshape(n_heads, k_dim)
    out = np.zeros((n_heads, v_dim))
    for h in range(n_heads):
        kvh = h // group
        sc = Kf[:, kvh, :] @ qf[h] * scale
        p = np.exp(sc - sc.max())
        out[h] = (p / p.sum()) @ Vf[:, kvh, :]
    return out.reshape(-1)


def attn_layer(x: np.ndarray, w: dict, Kc: np.ndarray, Vc: np.ndarray, pos: int, n_heads: int,
               n_kv: int, eps: float, theta: float):
    """One GQA attention block as decode_step runs it (wisp_engine.c:1557-1559 with
    run_attention's GQA branch :1328-1348): returns x + o_proj(attn) and the caches
    with position `pos` written (fp16, as cpu_kv_append stores it).  w: fp16 arrays
    input_norm [H], q_proj, k_proj, v_proj, o_proj."""
    H = x.size
    hd = H // n_heads
    xn = rmsnorm(x, w["input_norm"], eps)
    q = w["q_proj"].astype(np.float64) @ xn
    k = w["k_proj"].astype(np.float64) @ xn
    v = w["v_proj"].astype(np.float64) @ xn
    q = rope(q, n_heads, hd, 0, hd, pos, theta)
    k = rope(k, n_kv, hd, 0, hd, pos, theta)
    Kc = np.array(Kc, copy=True)
    Vc = np.array(Vc, copy=True)
    Kc.reshape(-1, n_kv * hd)[pos] = k.astype(np.float16)
    Vc.reshape(-1, n_kv * hd)[pos] = v.astype(np.float16)
    a = attention(q, Kc, Vc, pos + 1, n_heads, n_kv, hd, hd, 1.0 / np.sqrt(hd))
    return np.asarray(x, np.float64) + w["o_proj"].astype(np.float64) @ a, Kc, Vc


def logits(x: np.ndarray, final_norm: np.ndarray, lm_head: np.ndarray, eps: float) -> np.ndarray:
    """decode_step's tail (wisp_engine.c:1575-1579): lm_head . rmsnorm(x)."""
    return lm_head.astype(np.float64) @ rmsnorm(x, final_norm, eps)
