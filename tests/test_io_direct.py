"""The SSD tier's expert-file reader (``wisp_read_expert_file``), on the CPU: direct
preads into an aligned buffer, buffered preads otherwise, the reference's error
behaviour (missing file or too large for the staging buffer -> 0, WISP_ERR_IO)."""

import ctypes as C

import numpy as np
import pytest

from wisp_b200.lib import WispErrCtx, lib

WISP_ERR_IO = 2


def _aligned(nbytes: int, align: int = 4096, offset: int = 0):
    buf = np.zeros(nbytes + 2 * align, np.uint8)
    a = (-buf.ctypes.data) % align + offset
    return buf, buf[a:a + nbytes]


@pytest.mark.parametrize("size", [1, 4096, 1_000_003, 3 * 4096 + 17])
@pytest.mark.parametrize("offset", [0, 8])
def test_reads_whole_file(tmp_path, size, offset):
    data = np.random.default_rng(size).integers(0, 256, size, dtype=np.uint8)
    for d in (tmp_path, ):
        p = d / f"e{size}.bin"
        p.write_bytes(data.tobytes())
        keep, dst = _aligned(size + 8192, offset=offset)
        err = WispErrCtx()
        direct = C.c_int(-1)
        n = lib().wisp_read_expert_file(str(p).encode(), dst.ctypes.data, dst.size,
                                        C.byref(direct), C.byref(err))
        assert n == size, err.message
        assert np.array_equal(dst[:size], data)
        assert direct.value in (0, 1)
        if offset:  # an unaligned destination is never read with O_DIRECT
            assert direct.value == 0


def test_errors(tmp_path):
    err = WispErrCtx()
    keep, dst = _aligned(4096)
    assert lib().wisp_read_expert_file(str(tmp_path / "missing.bin").encode(), dst.ctypes.data,
                                       dst.size, None, C.byref(err)) == 0
    assert err.code == WISP_ERR_IO
    p = tmp_path / "big.bin"
    p.write_bytes(b"\\1" * 5000)
    err = WispErrCtx()
    assert lib().wisp_read_expert_file(str(p).encode(), dst.ctypes.data, 4096, None,
                                       C.byref(err)) == 0
    assert err.code == WISP_ERR_IO
