"""wisp_moe_block_forward_static: the MoE block without a caller workspace.

The entry point runs the same kernels as wisp_moe_block_forward in a fixed device
array inside the library.  The GPU test calls both through the C ABI on the same
inputs and compares them within the parity tolerances, twice in a row (the second
call reuses the array the first one left behind); after each static call it reads
the status word through wisp_moe_block_static_status (0 = no misaligned or missing
expert, no plan overflow, no timed-out wait) and compares the output with the CPU
oracle too.  The CPU test checks that a request larger than the array is refused
before any GPU work.  This file is collected last so it also runs after every other
test has used the device.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from wisp_b200 import converter as cv
from wisp_b200.lib import WispErrCtx, WispMoeLayer, lib
from wisp_b200.moe import MoEStack

from parity import MAX_ABS, REL_L2, check_block, rel_l2

LIMIT = 8 << 20


def call_static(st, x, y, idx, w):
    err = WispErrCtx()
    rc = lib().wisp_moe_block_forward_static(
        C.byref(st.layer_c(0)), x.data_ptr(), y.data_ptr(), x.shape[0], idx.data_ptr(),
        w.data_ptr(), torch.cuda.current_stream().cuda_stream, C.byref(err))
    return rc, err


@pytest.mark.gpu
@pytest.mark.parametrize("H,I,E,k,T", [(512, 1024, 8, 2, 3), (4096, 14336, 8, 2, 2)])
def test_static_matches_workspace_entry(cuda, H, I, E, k, T):
    shape = cv.MoEShape(hidden=H, inter=I, n_experts=E, top_k=k)
    st = MoEStack(shape, seed=31 + H, device=cuda, random_bias=True)
    assert st.workspace_bytes(T) <= LIMIT
    x = cv.make_input(shape, T, 5).to(cuda)
    y_ref, idx_ref, w_ref = st.block(0, x, routing=True)
    torch.cuda.synchronize()
    assert st.status() == 0
    y_ref, idx_ref, w_ref = y_ref.cpu().numpy(), idx_ref.cpu().numpy(), w_ref.cpu().numpy()
    from oracle import oracle as orc
    Wb, bb = st.host_router(0)
    blobs = st.host_blobs(0)
    yo, io, wo = orc.port_moe_block_arrays(Wb, bb, blobs, k, x.cpu().numpy())
    for _ in range(2):
        y = torch.full_like(x, float("nan"))
        idx = torch.full((T, k), -7, dtype=torch.int32, device=cuda)
        w = torch.zeros((T, k), dtype=torch.float32, device=cuda)
        rc, err = call_static(st, x, y, idx, w)
        assert rc == 0, err.message.decode()
        assert lib().wisp_moe_block_static_status(torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        yg = y.cpu().numpy()
        check_block(yg, idx.cpu().numpy(), w.cpu().numpy(), yo, io, wo, Wb, bb,
                    x.cpu().numpy(), blobs)
        assert np.array_equal(idx.cpu().numpy(), idx_ref)
        np.testing.assert_allclose(w.cpu().numpy(), w_ref, rtol=1e-6, atol=1e-7)
        assert np.isfinite(yg).all()
        assert float(np.abs(yg - y_ref).max()) <= MAX_ABS
        assert rel_l2(yg, y_ref) <= REL_L2


def test_static_rejects_requests_beyond_the_array(built_lib):
    """A Mixtral-shaped layer at T=64 needs far more than 8 MiB: refused on the
    host with the sizes in the message (the fake device pointers are never used)."""
    shape = cv.MoEShape(hidden=4096, inter=14336, n_experts=8, top_k=2)
    from wisp_b200.moe import parse_meta
    dims = [(14336, 4096), (14336, 4096), (4096, 14336)]
    head = cv.HEADER.pack(cv.EXPERT_MAGIC, cv.TILED_VERSION, 0, 0, 64, 3) + b"".join(
        cv.MAT_RECORD.pack(r, c, r * c // 2, r * c // 32, r * c // 32) for r, c in dims)
    total = cv.HEADER_BYTES + sum(r * c // 2 + r * c // 16 for r, c in dims)
    meta = parse_meta(head, total)
    layer = WispMoeLayer()
    layer.meta = meta
    layer.expert_blobs = 0x1000
    layer.router_w = 0x2000
    layer.n_experts = shape.n_experts
    layer.top_k = shape.top_k
    n = lib().wisp_moe_workspace_bytes(C.byref(layer), 1, 64)
    assert n > LIMIT
    assert lib().wisp_moe_workspace_bytes(C.byref(layer), 1, 4) <= LIMIT
    err = WispErrCtx()
    rc = lib().wisp_moe_block_forward_static(C.byref(layer), 0x3000, 0x4000, 64, None, None,
                                             None, C.byref(err))
    assert rc == 4  # WISP_ERR_INVALID_ARG
    msg = err.message.decode()
    assert "fixed scratch" in msg and str(n) in msg
