"""The sigmoid-score gating rule (``WISP_GATING_SIGMOID``), GPU tests.

BASELINE's DeepSeek-V3-shaped configurations name "top-8 sigmoid-score gating
normalised over the selected 8".  The reference implements only softmax(+bias)
gating (csrc/cuda/router.cu:60-120), so this mode has no reference to be pinned to:
parity unpinned.  It is tested against its own restatement here -- routing from a
float64 torch restatement of the rule (s = sigmoid(logits); selection on s + bias,
strict argmax, lowest index on ties; w = s / sum of the selected s), experts from
the oracle's pinned dequantisation (``oracle_dequant``) in float64 numpy -- with
the build's tolerances (indices exact away from near-ties, max-abs 2e-2, rel-L2
1e-2, regression bound 2e-3).
"""

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from wisp_b200 import converter as cv
from wisp_b200.moe import MoEStack

pytestmark = pytest.mark.gpu

from parity import check_outputs  # noqa: E402

SIGMOID = 1


def sigmoid_route(Wb: np.ndarray, bb, x: np.ndarray, k: int):
    """The rule restated: indices [T,k], weights [T,k], selection scores [T,E]."""
    W = Wb.view(np.float16).astype(np.float64)
    lg = x.astype(np.float64) @ W.T
    s = 1.0 / (1.0 + np.exp(-lg))
    sel = s + (bb.view(np.float16).astype(np.float64)[None, :] if bb is not None else 0.0)
    T = x.shape[0]
    idx = np.zeros((T, k), np.int64)
    w = np.zeros((T, k))
    for t in range(T):
        taken = np.zeros(sel.shape[1], bool)
        for j in range(k):
            v = np.where(taken, -np.inf, sel[t])
            e = int(np.argmax(v))  # first maximum = lowest index
            taken[e] = True
            idx[t, j] = e
        w[t] = s[t, idx[t]] / s[t, idx[t]].sum()
    return idx, w, sel


def experts_ref(blobs, shared, idx, w, x, inter):
    """y = [shared(x)] + sum_j w_j * down_j(silu(gate_j x) * up_j x) in float64, on the
    oracle's dequantisation of the routed blobs and the fp16 dense shared expert."""
    T, H = x.shape
    I = inter
    cache = {}

    def weights(e):
        if e not in cache:
            if e == "shared":
                g, u, d = (m.view(np.float16).astype(np.float64) for m in shared)
            else:
                g = orc.port_dequant(blobs[e], 0, I * H).astype(np.float64)
                u = orc.port_dequant(blobs[e], 1, I * H).astype(np.float64)
                d = orc.port_dequant(blobs[e], 2, H * I).astype(np.float64)
            cache[e] = (g.reshape(I, H), u.reshape(I, H), d.reshape(H, I))
        return cache[e]

    def ffn(e, v):
        G, U, D = weights(e)
        a, b = G @ v, U @ v
        return D @ (a / (1.0 + np.exp(-a)) * b)

    y = np.zeros((T, H), np.float64)
    for t in range(T):
        v = x[t].astype(np.float64)
        if shared is not None:
            y[t] += ffn("shared", v)
        for j in range(idx.shape[1]):
            if idx[t, j] >= 0:
                y[t] += w[t, j] * ffn(int(idx[t, j]), v)
    return y


def _near_tie(sel_row, k):
    """Two of the k+1 best selection scores within 1e-5: the rule's order (and, at
    the k-th place, its choice) is decided by float rounding there."""
    top = np.sort(sel_row)[::-1][:k + 1]
    return bool(np.any(np.abs(np.diff(top)) < 1e-5))


@pytest.mark.parametrize("path,T", [("decode", 1), ("decode", 7), ("prefill", 150)])
def test_sigmoid_gating_matches_restatement(cuda, path, T):
    shape = cv.MoEShape(hidden=256, inter=256, n_experts=16, top_k=4, group_size=64,
                        shared_inter=256)
    st = MoEStack(shape, seed=5 + T, device=cuda, zipf_s=1.1, gating=SIGMOID)
    x = torch.randn(T, 256, generator=torch.Generator().manual_seed(T + 3)).half().float()
    run = st.prefill if path == "prefill" else st.block
    y, idx, w = run(0, x.to(cuda), routing=True)
    torch.cuda.synchronize()
    assert (st.prefill_status() if path == "prefill" else st.status()) == 0
    Wb, bb = st.host_router(0)
    ir, wr, sel = sigmoid_route(Wb, bb, x.numpy(), shape.top_k)
    gi, gw = idx.cpu().numpy(), w.cpu().numpy()
    ok = [t for t in range(T) if not _near_tie(sel[t], shape.top_k)]
    assert len(ok) >= T // 2
    for t in ok:
        np.testing.assert_array_equal(gi[t], ir[t])
        np.testing.assert_allclose(gw[t], wr[t], rtol=1e-5, atol=1e-6)
    # the outputs on the device's own routing
    yr = experts_ref(st.host_blobs(0), st.host_shared(0), gi, gw.astype(np.float64), x.numpy(),
                     shape.inter)
    check_outputs(y.cpu().numpy(), yr.astype(np.float32))


def test_sigmoid_differs_from_softmax(cuda):
    """Same weights, the two rules: the softmax path is unchanged by the new field and
    the sigmoid weights are normalised sigmoid scores, not softmax probabilities."""
    shape = cv.MoEShape(hidden=256, inter=256, n_experts=16, top_k=4, group_size=64)
    a = MoEStack(shape, seed=9, device=cuda, zipf_s=1.1)
    b = MoEStack(shape, seed=9, device=cuda, zipf_s=1.1, gating=SIGMOID)
    x = torch.randn(5, 256, generator=torch.Generator().manual_seed(1)).to(cuda)
    _, ia, wa = a.block(0, x, routing=True)
    _, ib, wb = b.block(0, x, routing=True)
    torch.cuda.synchronize()
    assert not torch.allclose(wa, wb)
    np.testing.assert_allclose(wb.sum(1).cpu().numpy(), 1.0, rtol=1e-5)
