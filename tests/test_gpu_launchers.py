"""The reference kernel-launcher ABI (wisp_engine.h:549-612 signatures) against
plain PyTorch fp32 references of the same ops (GPU tests)."""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from wisp_b200 import converter as cv
from wisp_b200.lib import lib

pytestmark = pytest.mark.gpu


def stream():
    return torch.cuda.current_stream().cuda_stream


def test_gemv_and_transpose(cuda):
    for rows, cols in [(64, 4096), (33, 100), (7, 8)]:
        W = (torch.randn(rows, cols, device=cuda) * 0.05).half()
        x = torch.randn(cols, device=cuda)
        y = torch.empty(rows, device=cuda)
        lib().wisp_gpu_gemv_f16(W.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, stream())
        torch.testing.assert_close(y, W.float() @ x, rtol=1e-4, atol=1e-4)
        xt = torch.randn(rows, device=cuda)
        yt = torch.empty(cols, device=cuda)
        lib().wisp_gpu_gemv_t_f16(W.data_ptr(), xt.data_ptr(), yt.data_ptr(), rows, cols, stream())
        torch.testing.assert_close(yt, W.float().t() @ xt, rtol=1e-4, atol=1e-4)


def test_swiglu_ffn_rmsnorm_residual_scale(cuda):
    I, H = 300, 512
    Wg = (torch.randn(I, H, device=cuda) * 0.05).half()
    Wu = (torch.randn(I, H, device=cuda) * 0.05).half()
    x = torch.randn(H, device=cuda)
    h = torch.empty(I, device=cuda)
    lib().wisp_gpu_swiglu_ffn(Wg.data_ptr(), Wu.data_ptr(), x.data_ptr(), h.data_ptr(), I, H, stream())
    g, u = Wg.float() @ x, Wu.float() @ x
    torch.testing.assert_close(h, torch.nn.functional.silu(g) * u, rtol=1e-4, atol=1e-4)
    o = torch.empty(I, device=cuda)
    lib().wisp_gpu_swiglu(g.data_ptr(), u.data_ptr(), o.data_ptr(), I, stream())
    torch.testing.assert_close(o, torch.nn.functional.silu(g) * u, rtol=1e-5, atol=1e-6)
    w = torch.rand(H, device=cuda).half()
    y = torch.empty(H, device=cuda)
    lib().wisp_gpu_rmsnorm(x.data_ptr(), w.data_ptr(), y.data_ptr(), H, C.c_float(1e-5), stream())
    ref = x * torch.rsqrt((x * x).mean() + 1e-5) * w.float()
    torch.testing.assert_close(y, ref, rtol=1e-5, atol=1e-5)
    acc = torch.randn(H, device=cuda)
    acc0 = acc.clone()
    lib().wisp_gpu_scale_accum(acc.data_ptr(), x.data_ptr(), C.c_float(0.25), H, stream())
    torch.testing.assert_close(acc, acc0 + 0.25 * x)
    lib().wisp_gpu_residual_add(acc.data_ptr(), x.data_ptr(), H, stream())
    torch.testing.assert_close(acc, acc0 + 1.25 * x)


@pytest.mark.parametrize("E,H,k,bias", [(8, 4096, 2, False), (256, 7168, 8, True), (5, 64, 5, True)])
def test_router_topk_matches_oracle(cuda, E, H, k, bias):
    g = torch.Generator().manual_seed(E + H)
    W = (torch.randn(E, H, generator=g) * 0.02).half()
    b = (torch.randn(E, generator=g) * 0.5).half() if bias else None
    x = torch.randn(H, generator=g)
    logits = torch.empty(E, device=cuda)
    out_idx = (C.c_int * k)()
    out_w = (C.c_float * k)()
    Wd, xd = W.to(cuda), x.to(cuda)
    bd = b.to(cuda) if bias else None
    lib().wisp_gpu_router_topk(Wd.data_ptr(), bd.data_ptr() if bias else None, xd.data_ptr(),
                               logits.data_ptr(), E, H, k, out_idx, out_w, stream())
    torch.cuda.synchronize()
    idx, w, _ = orc.port_router(W.numpy().view(np.uint16),
                                b.numpy().view(np.uint16) if bias else None, x.numpy(), k)
    assert list(out_idx) == idx.tolist()
    np.testing.assert_allclose(np.array(out_w[:]), w, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("n,gs", [(64 * 1024, 64), (1000, 16), (4096 * 8, 128)])
def test_dequant_and_async_load(cuda, n, gs):
    rows = 8
    w = torch.randn(rows, n // rows) * 0.02
    q = cv.quantize_int4(w, gs)
    ref = cv.dequantize_int4(q).flatten().half()
    pk, sc, ze = q.packed.to(cuda), q.scales.to(cuda), q.zeros.to(cuda)
    out = torch.empty(n, dtype=torch.float16, device=cuda)
    rc = lib().launch_dequant_expert(pk.data_ptr(), sc.data_ptr(), ze.data_ptr(), out.data_ptr(),
                                     n, gs, stream())
    assert rc == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=0, atol=1e-3)
    hp, hs, hz = q.packed.pin_memory(), q.scales.pin_memory(), q.zeros.pin_memory()
    tp, ts, tz = torch.empty_like(pk), torch.empty_like(sc), torch.empty_like(ze)
    out2 = torch.empty_like(out)
    rc = lib().async_load_expert(hp.data_ptr(), hs.data_ptr(), hz.data_ptr(), tp.data_ptr(),
                                 ts.data_ptr(), tz.data_ptr(), out2.data_ptr(), n, gs, stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    assert lib().launch_dequant_expert(pk.data_ptr(), sc.data_ptr(), ze.data_ptr(),
                                       out.data_ptr(), 0, gs, stream()) != 0
