"""The oversubscribed path (expert pool in pinned host memory streamed through a small
device cache, wisp_stream_* + wisp_b200.stream) against the resident stack (GPU tests)."""

import pytest
import torch

from wisp_b200 import converter as cv
from wisp_b200.moe import MoEStack
from wisp_b200.stream import StreamingStack

pytestmark = pytest.mark.gpu

from parity import check_outputs  # noqa: E402


@pytest.mark.parametrize("predict", [True, False])
def test_streamed_stack_matches_resident(cuda, predict):
    """6 cache slots for 3 layers x 16 experts (top-4): nearly every step evicts, and the
    result equals the resident stack's on the same tokens."""
    shape = cv.MoEShape(hidden=256, inter=256, n_experts=16, top_k=4, shared_inter=256,
                        n_layers=3)
    ss = StreamingStack(shape, seed=7, n_layers=3, cache_slots=6, device=cuda, zipf_s=1.1)
    st = MoEStack(shape, seed=7, device=cuda, zipf_s=1.1)
    g = torch.Generator().manual_seed(1)
    for _ in range(8):
        x0 = torch.randn(1, 256, generator=g).to(cuda)
        a = x0.clone()
        ss.step(a, predict=predict)
        b = x0.clone()
        st.stack(b)
        torch.cuda.synchronize()
        assert ss.status() == 0
        check_outputs(a.cpu().numpy(), b.cpu().numpy())
    s = ss.stats()
    assert s["misses"] > 0 and s["slots"] == 6
    assert (s["prefetched"] > 0) == predict
    ss.close()


def test_stream_cache_rejects_unregistered_and_full(cuda):
    """An expert without a host blob, or a layer needing more experts than slots,
    fails with an error instead of touching the device."""
    import ctypes as C
    from wisp_b200.lib import WispErrCtx, lib
    shape = cv.MoEShape(hidden=256, inter=256, n_experts=8, top_k=4, n_layers=1)
    ss = StreamingStack(shape, seed=3, n_layers=1, cache_slots=2, device=cuda)
    err = WispErrCtx()
    ids = (C.c_int * 4)(0, 1, 2, 3)
    s = torch.cuda.current_stream().cuda_stream
    rc = lib().wisp_stream_ensure(ss.cache, 0, ids, 4, s, None, None, C.byref(err))
    assert rc != 0 and b"slot" in err.message
    bad = (C.c_int * 1)(9)
    rc = lib().wisp_stream_ensure(ss.cache, 0, bad, 1, s, None, None, C.byref(err))
    assert rc != 0
    ss.close()
