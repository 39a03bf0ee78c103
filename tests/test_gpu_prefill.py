"""Parity of the tensor-core prefill path (``wisp_moe_prefill_forward``) with the CPU
oracle (GPU tests).

The prefill path rounds the dequantised weights to fp16 (as the reference's own GPU
dequant does, csrc/cuda/expert_loader.cu:23-43) and the activations x and h to fp16,
and accumulates in fp32; the tolerances are the build's north star (max-abs 2e-2,
rel-L2 1e-2) plus the regression bound rel-L2 <= 2e-3.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from wisp_b200 import converter as cv
from wisp_b200.moe import MoEStack

pytestmark = pytest.mark.gpu

from parity import check_block, check_outputs, check_routing  # noqa: E402

CONFIGS = [
    # H, I, E, k, shared, bias, T
    (256, 256, 8, 2, False, "random", 40),
    (256, 256, 8, 2, False, None, 1),
    (512, 384, 16, 4, False, "zipf", 300),
    (1024, 512, 32, 8, True, "zipf", 700),
    (384, 640, 12, 3, True, None, 257),
]


def _stack(cuda, H, I, E, k, shared, bias, seed):
    shape = cv.MoEShape(hidden=H, inter=I, n_experts=E, top_k=k, group_size=64,
                        shared_inter=I if shared else 0)
    return MoEStack(shape, seed=seed, device=cuda, zipf_s=1.1 if bias == "zipf" else None,
                    random_bias=bias == "random")


@pytest.mark.parametrize("H,I,E,k,shared,bias,T", CONFIGS)
def test_prefill_matches_oracle(cuda, H, I, E, k, shared, bias, T):
    st = _stack(cuda, H, I, E, k, shared, bias, seed=H + I + E + T)
    x = (torch.randn(T, H, generator=torch.Generator().manual_seed(T + 1))).half().float()
    y, idx, w = st.prefill(0, x.to(cuda), routing=True)
    torch.cuda.synchronize()
    assert st.prefill_status() == 0
    Wb, bb = st.host_router(0)
    yr, ir, wr = orc.port_moe_block_arrays(Wb, bb, st.host_blobs(0), k, x.numpy(),
                                           shared=st.host_shared(0) if shared else None)
    check_block(y.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), yr, ir, wr, Wb, bb,
                x.numpy(), st.host_blobs(0), shared=st.host_shared(0) if shared else None)


@pytest.mark.parametrize("T", [300, 700])
def test_prefill_down_stage_sizes_match_oracle(cuda, T):
    """The down GEMM's stage size follows the rows per expert: 4 quant groups
    per stage at 300 tokens (82 rows per expert), 2 at 700 (191 rows)."""
    test_prefill_matches_oracle(cuda, 1024, 512, 32, 8, True, "zipf", T)


def test_prefill_matches_decode_path(cuda):
    """The tensor-core path and the decode stream kernels agree on the same batch."""
    st = _stack(cuda, 512, 512, 16, 4, True, "zipf", seed=77)
    x = torch.randn(64, 512, generator=torch.Generator().manual_seed(5)).to(cuda)
    yp, ip, _ = st.prefill(0, x, routing=True)
    yd, idd, _ = st.block(0, x, routing=True)
    torch.cuda.synchronize()
    assert st.prefill_status() == 0 and st.status() == 0
    assert torch.equal(ip, idd)
    check_outputs(yp.cpu().numpy(), yd.cpu().numpy())


def test_prefill_rejects_unsupported_geometry(cuda):
    """group_size 32 or sizes off the 128-row tiles fail before any GPU work."""
    from wisp_b200.lib import WispError
    shape = cv.MoEShape(hidden=192, inter=96, n_experts=4, top_k=2, group_size=32)
    st = MoEStack(shape, seed=3, device=cuda)
    with pytest.raises(WispError, match="prefill"):
        st.prefill(0, torch.randn(8, 192, device=cuda))


@pytest.mark.slow
def test_deepseek_shaped_prefill_matches_oracle(cuda):
    """DeepSeek-V3-shaped layer (7168 / 2048, 256 experts, top-8, shared expert,
    Zipf(1.1) routing) at 512 tokens: hot experts span several 256-token tiles."""
    shape = cv.MoEShape(hidden=7168, inter=2048, n_experts=256, top_k=8, shared_inter=2048)
    st = MoEStack(shape, seed=31, device=cuda, zipf_s=1.1)
    x = cv.make_input(shape, 512, 31)
    y, idx, w = st.prefill(0, x.to(cuda), routing=True)
    torch.cuda.synchronize()
    assert st.prefill_status() == 0
    Wb, bb = st.host_router(0)
    yr, ir, wr = orc.port_moe_block_arrays(Wb, bb, st.host_blobs(0), 8, x.numpy(),
                                           shared=st.host_shared(0))
    check_block(y.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), yr, ir, wr, Wb, bb,
                x.numpy(), st.host_blobs(0), shared=st.host_shared(0))


@pytest.mark.parametrize("T", [96, 333])
def test_prefill_stack_matches_oracle(cuda, T):
    """x <- x + MoE_l(rmsnorm(x)) over 3 layers on the tensor-core path against the
    oracle's per-layer recipe (rmsnorm, block, residual)."""
    H = 512
    shape = cv.MoEShape(hidden=H, inter=384, n_experts=16, top_k=4, shared_inter=384, n_layers=3)
    st = MoEStack(shape, seed=19, device=cuda, zipf_s=1.1)
    x0 = torch.randn(T, H, generator=torch.Generator().manual_seed(4)).half().float()
    x = x0.clone().to(cuda)
    _, idx, _ = st.prefill_stack(x, routing=True)
    torch.cuda.synchronize()
    assert st.prefill_status() == 0
    xr = x0.numpy().copy()
    ones = np.ones(H, np.float16).view(np.uint16)
    for l in range(shape.n_layers):
        Wb, bb = st.host_router(l)
        xn = np.empty_like(xr)
        for t in range(T):
            orc.port_lib().oracle_rmsnorm(xr[t].ctypes.data, ones.ctypes.data, xn[t].ctypes.data,
                                          H, np.float32(shape.rms_eps))
        yl, il, _ = orc.port_moe_block_arrays(Wb, bb, st.host_blobs(l), 4, xn,
                                              shared=st.host_shared(l))
        check_routing(idx[l].cpu().numpy(), il, Wb, bb, xn)
        xr = xr + yl
    check_outputs(x.cpu().numpy(), xr)


def test_prefill_stack_matches_decode_stack(cuda):
    """The tensor-core stack and the decode stream stack agree on the same tokens."""
    shape = cv.MoEShape(hidden=256, inter=256, n_experts=8, top_k=2, n_layers=4)
    st = MoEStack(shape, seed=23, device=cuda, random_bias=True)
    x0 = torch.randn(16, 256, generator=torch.Generator().manual_seed(9)).to(cuda)
    a = st.prefill_stack(x0.clone())
    b = st.stack(x0.clone())
    torch.cuda.synchronize()
    assert st.prefill_status() == 0 and st.status() == 0
    check_outputs(a.cpu().numpy(), b.cpu().numpy())
