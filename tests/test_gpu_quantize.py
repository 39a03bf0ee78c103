"""The GPU int4 quantiser (wisp_quantize_int4) is byte-identical to the converter's
restatement of the reference quantiser (wisp_b200.converter.quantize_int4, itself
pinned to wisp/converter/quantizer.py by tests/test_converter.py) -- GPU tests."""

import ctypes as C

import pytest
import torch

from wisp_b200 import converter as cv
from wisp_b200.lib import WispErrCtx, check, lib

pytestmark = pytest.mark.gpu


def _gpu_quant(w: torch.Tensor, gs: int):
    rows, cols = w.shape
    n = rows * cols
    wd = w.to(torch.float32).contiguous().cuda()
    packed = torch.empty(n // 2, dtype=torch.uint8, device="cuda")
    scales = torch.empty(n // gs, dtype=torch.float16, device="cuda")
    zeros = torch.empty(n // gs, dtype=torch.float16, device="cuda")
    err = WispErrCtx()
    check(lib().wisp_quantize_int4(wd.data_ptr(), rows, cols, gs, packed.data_ptr(),
                                   scales.data_ptr(), zeros.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream, C.byref(err)), err)
    torch.cuda.synchronize()
    return packed.cpu(), scales.cpu(), zeros.cpu()


def _cases():
    g = torch.Generator().manual_seed(7)
    yield "normal", torch.randn(256, 512, generator=g) * 0.02, 64
    yield "wide", torch.randn(64, 4096, generator=g) * 3.0, 128
    yield "gs32", torch.randn(96, 96, generator=g), 32
    # constant groups (scale clamps to 1e-8), exact half-way ties, huge range
    t = torch.zeros(8, 64)
    t[1] = 5.0
    t[2] = torch.arange(64, dtype=torch.float32) % 16      # min 0, max 15: ties at .5
    t[3] = torch.linspace(-1e4, 1e4, 64)
    t[4, ::2] = 1e-30
    t[5] = torch.tensor([0.0, 1.0] * 32)                   # every x - zero = +-0.5 * scale
    t[6] = -torch.arange(64, dtype=torch.float32) / 7.0
    t[7] = torch.randn(64, generator=g) * 1e-6
    yield "edges", t, 64


@pytest.mark.parametrize("name,w,gs", list(_cases()), ids=[c[0] for c in _cases()])
def test_gpu_quantiser_is_byte_identical(cuda, name, w, gs):
    ref = cv.quantize_int4(w, gs)
    packed, scales, zeros = _gpu_quant(w, gs)
    assert torch.equal(packed, ref.packed)
    assert torch.equal(scales.view(torch.int16), ref.scales.view(torch.int16))
    assert torch.equal(zeros.view(torch.int16), ref.zeros.view(torch.int16))


def test_gpu_quantiser_rejects_ragged_groups(cuda):
    from wisp_b200.lib import WispError
    with pytest.raises(WispError, match="quantize_int4"):
        _gpu_quant(torch.randn(3, 50), 64)
