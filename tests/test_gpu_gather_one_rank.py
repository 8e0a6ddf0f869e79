"""The fused all-gather's store path on one GPU: spmm24_launch_gather with a
single rank writes the shard's rows into its own full C at the row offset,
through every kernel's gather epilogue (cluster split-K, 256 x 256 pair,
512 x 240 pair, ragged N with element stores), equal bit for bit to the plain
launch with the same kernel; rows outside the shard stay untouched.  The
cross-GPU forms run in tests/test_gpu_multi.py."""
import numpy as np
import pytest

from problems import make_problem

pytestmark = pytest.mark.gpu


def _dev(torch, arr, dev):
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).to(dev)


@pytest.mark.parametrize("shape,tune", [
    ((1024, 16, 1024), {}),                      # cluster kernel, split-K
    ((512, 40, 512), {}),                        # mid N, ragged N (element stores)
    ((1024, 512, 1024), dict(pair=1, pair2=0)),  # 256 x 256 pair kernel
    ((1024, 480, 512), dict(pair2=1)),           # 512 x 240 pair kernel
    ((592, 500, 384), dict(pair2=1)),            # ragged M and N on the 512 x 240 tile
], ids=lambda v: "x".join(map(str, v)) if isinstance(v, tuple) else str(v))
def test_gather_into_own_buffer(cuda_device, tuning, shape, tune):
    import torch

    import spmm24

    tuning(**tune)
    M, N, K = shape
    p = make_problem(M, N, K, seed=M + 3 * N, a_scale=0.05, b_dist="normal")
    A, E, B = _dev(torch, p.vals, cuda_device), _dev(torch, p.meta, cuda_device), _dev(torch, p.b_packed, cuda_device)
    s = torch.cuda.current_stream(cuda_device)
    ref = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
    assert spmm24.launch(s, A, B, E, ref, M, N, K, None, 0) == 0
    row0 = 128
    full = torch.full((M + 256, N), float("nan"), dtype=torch.float16, device=cuda_device)
    rc = spmm24.launch_gather(s, A, B, E, M, N, K, [full.data_ptr()], row0, M + 256, 0, 0)
    assert rc == 0, spmm24._lib.spmm24_last_error().decode()
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(full[row0:row0 + M], ref)
    assert torch.isnan(full[:row0]).all() and torch.isnan(full[row0 + M:]).all()
    assert spmm24.device_status(0) == 0
