"""Failure detection and launch-mechanics checks on the GPU, without faulting,
trapping or hanging it: bounded waits that run out report a status and leave
the context usable; launches can be captured in a CUDA graph (programmatic
launch edges included) and replayed; invalid calls are refused before any
work is queued."""
import ctypes

import numpy as np
import pytest

from problems import compare, make_problem, oracle_c, within_tolerance

pytestmark = pytest.mark.gpu


def _dev(torch, arr, dev):
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).to(dev)


@pytest.mark.parametrize("which", [0, 1])
def test_bounded_wait_gives_up_and_context_survives(cuda_device, which):
    import torch

    import spmm24

    fn = spmm24._lib.spmm24_selftest_bounded_wait
    fn.argtypes = [ctypes.c_int, ctypes.c_uint, ctypes.POINTER(ctypes.c_uint32)]
    fn.restype = ctypes.c_int
    status = ctypes.c_uint32(0)
    assert fn(which, 200000, ctypes.byref(status)) == 0  # 0.2 s limit
    assert status.value != 0
    # the device still computes correctly afterwards
    p = make_problem(256, 16, 512, seed=1)
    A, E, B = _dev(torch, p.vals, cuda_device), _dev(torch, p.meta, cuda_device), _dev(torch, p.b_packed, cuda_device)
    C = torch.empty((256, 16), dtype=torch.float16, device=cuda_device)
    assert spmm24.launch(None, A, B, E, C, 256, 16, 512, None, 0) == 0
    torch.cuda.synchronize(cuda_device)
    got = C.view(torch.int16).cpu().numpy().view(np.uint16)
    assert within_tolerance(compare(got, oracle_c(p)))
    assert spmm24.device_status(0) == 0


@pytest.mark.parametrize("shape", [(2048, 16, 2048), (1024, 512, 1024)])
def test_cuda_graph_capture_and_replay(cuda_device, shape):
    """A chain of three dependent calls captured into a CUDA graph (with
    programmatic launch edges) and replayed twice equals the eager chain."""
    import torch

    import spmm24

    M, N, K = shape
    assert M == K  # the output of one call is the next call's activation
    p = make_problem(M, N, K, seed=2, a_scale=0.03, b_dist="normal")
    A, E = _dev(torch, p.vals, cuda_device), _dev(torch, p.meta, cuda_device)
    x0 = torch.from_numpy(p.b_rowmajor.view(np.float16).reshape(K, N).copy()).to(cuda_device)

    def chain(stream):
        x = x0
        outs = []
        for _ in range(3):
            bp = x.reshape(K, N // 8, 8).permute(1, 0, 2).contiguous()
            c = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
            rc = spmm24.launch_ex(stream, A, bp, E, c, M, N, K, 0, spmm24.STATIC_WEIGHTS)
            assert rc == 0
            outs.append((bp, c))
            x = c
        return outs

    eager = chain(torch.cuda.current_stream(cuda_device))
    torch.cuda.synchronize(cuda_device)
    ref = eager[-1][1].clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        captured = chain(torch.cuda.current_stream(cuda_device))
    for _ in range(2):
        captured[-1][1].zero_()
        g.replay()
        torch.cuda.synchronize(cuda_device)
        assert torch.equal(captured[-1][1].view(torch.int16), ref.view(torch.int16))


def test_invalid_calls_queue_nothing(cuda_device):
    import torch

    import spmm24

    C = torch.zeros((256, 16), dtype=torch.float16, device=cuda_device)
    ok = 1 << 20
    assert spmm24.launch(None, ok + 8, ok, ok, C, 256, 16, 256, None, 0) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert spmm24.launch(None, ok, ok, ok, C, 256, 16, 100, None, 0) == spmm24.CUDA_ERROR_INVALID_VALUE
    torch.cuda.synchronize(cuda_device)
    assert int(C.abs().sum()) == 0
