"""The reference's multi-GPU C ABI (wisp_pipeline_*, wisp_peer_*, wisp_nccl_available;
csrc/cuda/multi_gpu.cu:37-160): argument handling on CPU, transfers on GPUs."""

import ctypes as C
import threading

import pytest
import torch

from wisp_b200.lib import lib


def test_nccl_probe_and_argument_errors():
    L = lib()
    assert L.wisp_nccl_available() in (0, 1)
    assert L.wisp_pipeline_init(None, 2) == -1
    devs = (C.c_int * 1)(0)
    assert L.wisp_pipeline_init(devs, 0) == -1
    # no pipeline: send / receive fail instead of touching a device
    assert L.wisp_pipeline_send_activation(None, 4, 1, None) == -1
    assert L.wisp_pipeline_recv_activation(None, 4, 1, None) == -1
    assert L.wisp_peer_copy_async(None, 0, None, 0, 16, None) == -1
    L.wisp_pipeline_shutdown()  # no-op without a pipeline


@pytest.mark.gpu
def test_peer_copy_same_device(cuda):
    L = lib()
    a = torch.arange(1000, dtype=torch.float32, device=cuda)
    b = torch.zeros_like(a)
    s = torch.cuda.current_stream()
    assert L.wisp_peer_copy_async(b.data_ptr(), 0, a.data_ptr(), 0, a.numel() * 4,
                                  s.cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_pipeline_send_recv_two_gpus():
    """Stage 0 (GPU 0) sends n fp32 values to stage 1 (GPU 1) and back, one host
    thread per GPU (the reference's single-process NCCL pipeline)."""
    L = lib()
    if not L.wisp_nccl_available():
        pytest.skip("NCCL not loadable")
    dev0 = torch.cuda.current_device()
    assert L.wisp_peer_enable(0, 1) in (0, -1)
    devs = (C.c_int * 2)(0, 1)
    assert L.wisp_pipeline_init(devs, 2) == 0
    n = 4096 * 16
    x0 = torch.arange(n, dtype=torch.float32, device="cuda:0")
    x1 = torch.zeros(n, dtype=torch.float32, device="cuda:1")
    rc = [None, None]

    def stage(i):
        torch.cuda.set_device(i)
        s = torch.cuda.current_stream(i).cuda_stream
        if i == 0:
            rc[0] = L.wisp_pipeline_send_activation(x0.data_ptr(), n, 1, s)
        else:
            rc[1] = L.wisp_pipeline_recv_activation(x1.data_ptr(), n, 0, s)
        torch.cuda.synchronize(i)

    th = [threading.Thread(target=stage, args=(i,)) for i in range(2)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=60)
    L.wisp_pipeline_shutdown()
    # the library leaves the caller's current device as it found it
    assert torch.cuda.current_device() == dev0
    assert rc == [0, 0]
    assert torch.equal(x1.cpu(), x0.cpu())
