"""spmm24_launch_noalloc: the allocation-free launch, for callers whose
device memory belongs to their own allocator or who may not allocate in the
middle of a latency-critical loop.  It is called through the C ABI and its
output is compared with spmm24_launch's on two consecutive calls (the
library-held scratch array keeps the previous call's contents, so the second
call checks that the flags are cleared between calls).  Tolerance: the
parity tolerance of tests/problems.py.

This file is named so that pytest collects it last; it also passes when run
on its own in a fresh process (the first call then does the one-time lookup
of the scratch array's address)."""
import ctypes

import numpy as np
import pytest

from problems import compare, make_problem, oracle_c, within_tolerance

pytestmark = pytest.mark.gpu


def _noalloc():
    import spmm24

    fn = ctypes.CDLL(spmm24.library_path()).spmm24_launch_noalloc
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 3
    fn.restype = ctypes.c_int
    return fn


def _dev(torch, arr, dev):
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).to(dev)


@pytest.mark.parametrize("shape", [(4096, 16, 4096), (1152, 24, 704), (144, 1, 320)])
def test_noalloc_matches_launch_on_two_calls(cuda_device, shape):
    import torch

    import spmm24

    M, N, K = shape
    p = make_problem(M, N, K, seed=M + 7 * N + K, a_scale=0.02, b_dist="normal")
    A, E, B = _dev(torch, p.vals, cuda_device), _dev(torch, p.meta, cuda_device), _dev(torch, p.b_packed, cuda_device)
    s = torch.cuda.current_stream(cuda_device)
    ref = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
    assert spmm24.launch(s, A, B, E, ref, M, N, K, None, 0) == 0
    torch.cuda.synchronize(cuda_device)
    ref_f32 = ref.float().cpu().numpy()
    fn = _noalloc()
    for call in range(2):
        C = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
        rc = fn(s.cuda_stream, A.data_ptr(), B.data_ptr(), E.data_ptr(), C.data_ptr(), M, N, K)
        assert rc == 0, spmm24._lib.spmm24_last_error().decode()
        torch.cuda.synchronize(cuda_device)
        got = C.view(torch.int16).cpu().numpy().view(np.uint16)
        stats = compare(got, ref_f32)
        assert within_tolerance(stats), (call, stats)
    assert within_tolerance(compare(got, oracle_c(p)))
    assert spmm24.device_status(0) == 0


def test_noalloc_rejects_wide_n(cuda_device):
    import spmm24

    rc = _noalloc()(None, 0x10000, 0x20000, 0x30000, 0x40000, 256, 64, 256)
    assert rc == spmm24.CUDA_ERROR_INVALID_VALUE
    assert "N <= 32" in spmm24._lib.spmm24_last_error().decode()
