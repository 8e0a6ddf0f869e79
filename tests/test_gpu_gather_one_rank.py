"""The fused all-gather's store path on one GPU: spmm24_launch_gather with a
single rank writes the shard's rows into its own full C at the row offset,
through every kernel's gather epilogue (cluster split-K, 256 x 256 and
256 x 128 pair, 512 x 240 pair, ragged N with element stores), equal bit for bit to the plain
launch with the same kernel; rows outside the shard stay untouched.  The
same for the grouped kernel's gather (spmm24_launch_grouped_gather, with
its fused barrier of one rank).  The cross-GPU forms run in
tests/test_gpu_multi.py."""
import numpy as np
import pytest

from problems import make_problem

pytestmark = pytest.mark.gpu


def _dev(torch, arr, dev):
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).to(dev)


@pytest.mark.parametrize("shape,tune", [
    ((1024, 16, 1024), {}),                      # cluster kernel, split-K
    ((512, 40, 512), {}),                        # mid N, ragged N (element stores)
    ((1024, 512, 1024), dict(pair=1, pair2=0, tile_n=256)),  # 256 x 256 pair kernel
    ((1024, 384, 1024), dict(pair=1, tile_n=128)),  # 256 x 128 pair kernel
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


@pytest.mark.parametrize("group_split", [1, 2, 4])
def test_grouped_gather_into_own_buffers(cuda_device, tuning, group_split):
    """spmm24_launch_grouped_gather with one rank: every problem's rows land
    in its full C at the row offset, equal bit for bit to a plain grouped
    launch with the same split (whole tiles, or K over clusters of 2 or 4);
    the fused barrier of one rank passes twice (epochs 1 and 2); rows
    outside the shards stay untouched."""
    import torch

    import spmm24

    tuning(group_split=group_split)
    dev = cuda_device
    shapes = [(1024, 16, 1024), (256, 8, 2048), (384, 32, 704), (128, 1, 512)]
    row0 = 256
    probs, plain, fulls, keep = [], [], [], []
    for i, (M, N, K) in enumerate(shapes):
        p = make_problem(M, N, K, seed=7 * i + M, a_scale=0.05, b_dist="normal")
        A, E, B = _dev(torch, p.vals, dev), _dev(torch, p.meta, dev), _dev(torch, p.b_packed, dev)
        ref = torch.full((M, N), float("nan"), dtype=torch.float16, device=dev)
        full = torch.full((M + 512, N), float("nan"), dtype=torch.float16, device=dev)
        g = spmm24.make_gather([full.data_ptr()], row0, M + 512)
        plain.append((A, B, E, ref, M, N, K))
        probs.append((A, B, E, 0, M, N, K, g))
        fulls.append(full)
        keep += [A, E, B, ref, full]
    s = torch.cuda.current_stream(dev)
    assert spmm24.launch_grouped(s, plain, 0) == 0, spmm24._lib.spmm24_last_error().decode()
    flags = torch.zeros(2, dtype=torch.int32, device=dev)  # [epoch of rank 0, CTA counter]
    bar = spmm24.group_barrier([flags.data_ptr()], 0, limit_us=2_000_000)
    arr = spmm24.problem_array(probs)
    for _ in range(2):
        rc = spmm24.launch_grouped_gather(s, arr, bar, 0)
        assert rc == 0, spmm24._lib.spmm24_last_error().decode()
    torch.cuda.synchronize(dev)
    for (A, B, E, ref, M, N, K), full in zip(plain, fulls):
        assert torch.equal(full[row0:row0 + M], ref), (M, N, K)
        assert torch.isnan(full[:row0]).all() and torch.isnan(full[row0 + M:]).all()
    assert flags.tolist() == [2, 0]  # two epochs published, the CTA counter wrapped to zero
    assert spmm24.device_status(0) == 0
