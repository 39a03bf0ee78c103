"""Parity checks shared by the GPU tests (tolerances of the build's north star)."""

import numpy as np

MAX_ABS, REL_L2, REL_L2_TIGHT, TIE = 2e-2, 1e-2, 2e-3, 1e-5


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def logits64(Wbits, bias_bits, x):
    W = Wbits.view(np.float16).astype(np.float64)
    lg = W @ x.astype(np.float64)
    if bias_bits is not None:
        lg = lg + bias_bits.view(np.float16).astype(np.float64)
    return lg


def check_routing(idx_gpu, idx_ref, Wbits, bias_bits, x):
    """Indices equal, or the differing choices are near-ties (|dlogit| < 1e-5)."""
    bad = []
    for t in range(idx_ref.shape[0]):
        if np.array_equal(idx_gpu[t], idx_ref[t]):
            continue
        lg = logits64(Wbits, bias_bits, x[t])
        a, b = set(idx_gpu[t].tolist()), set(idx_ref[t].tolist())
        diff = sorted(a ^ b)
        gap = max(lg[diff]) - min(lg[diff]) if diff else 0.0
        if set(idx_gpu[t]) == set(idx_ref[t]):
            # same set, different order: the swapped pair must be a near-tie
            order_gap = max(abs(lg[i] - lg[j]) for i, j in zip(idx_gpu[t], idx_ref[t]) if i != j)
            gap = order_gap
        if gap >= TIE:
            bad.append((t, idx_gpu[t].tolist(), idx_ref[t].tolist(), gap))
    assert not bad, f"routing differs beyond ties: {bad[:4]}"
    return sum(1 for t in range(idx_ref.shape[0]) if not np.array_equal(idx_gpu[t], idx_ref[t]))


def check_outputs(y_gpu, y_ref, tight=True):
    d = np.abs(y_gpu - y_ref).max()
    r = rel_l2(y_gpu, y_ref)
    assert d <= MAX_ABS, f"max-abs {d}"
    assert r <= REL_L2, f"rel-L2 {r}"
    if tight:
        assert r <= REL_L2_TIGHT, f"rel-L2 {r} above the regression bound"
    return d, r
