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


def check_block(y_gpu, idx_gpu, w_gpu, y_ref, idx_ref, w_ref, Wbits, bias_bits, x, blobs,
                shared=None, tight=True, weights=True):
    """Every token of one block checked, whatever the routing:

    * routing equal to the oracle's or differing only by near-ties (check_routing);
    * tokens routed like the oracle: gate weights and outputs against the oracle;
    * tokens whose routing flipped on a near-tie: outputs against the oracle's
      expert arithmetic on the GPU's own routing (oracle_experts_routed), so the
      expert kernels are still checked on them.

    Returns the number of flipped tokens (also printed, for the test log)."""
    from oracle import oracle as orc
    idx_gpu, w_gpu = np.asarray(idx_gpu), np.asarray(w_gpu)
    nd = check_routing(idx_gpu, idx_ref, Wbits, bias_bits, x)
    same = (idx_gpu == idx_ref).all(axis=1)
    if same.any():
        if weights:
            # router logits are fp32 sums over H in another order than the reference's
            # sequential sum (about 1e-5 apart at H = 7168), which moves the softmax
            # weights by about that much relative to each other
            np.testing.assert_allclose(w_gpu[same], w_ref[same], rtol=1e-4, atol=1e-6)
        check_outputs(y_gpu[same], y_ref[same], tight)
    if (~same).any():
        y_alt = orc.port_experts_routed(blobs, x.shape[1], idx_gpu[~same], w_gpu[~same],
                                        x[~same], shared=shared)
        check_outputs(y_gpu[~same], y_alt, tight)
    if nd:
        print(f"check_block: {nd} of {len(same)} tokens routed differently on near-ties")
    return nd
