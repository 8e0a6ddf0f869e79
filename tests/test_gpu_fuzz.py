"""Seeded random sweep over shapes, K splits, element types, epilogues and
output layouts, each compared with the oracle (fp32 GEMM on the pruned A,
epilogue in float64, rounded to C's type).  Shapes stay small enough for the
oracle to finish in seconds; every kernel path the picker can choose is hit
(cluster kernel with narrow, mid and wide tiles, split-K 1..8, the CTA pair
with and without its K split)."""
import numpy as np
import pytest

from test_gpu_epilogue import _run

pytestmark = pytest.mark.gpu


def _cases(n, seed):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        M = int(rng.integers(1, 48)) * 16
        K = int(rng.choice([64, 128, 192, 256, 448, 1024, 2048, 6144]))
        N = int(rng.choice([1, 3, 8, 13, 16, 24, 32, 40, 64, 100, 128, 136, 256, 264, 512]))
        split = int(rng.choice([0, 0, 0, 1, 2, 3, 5, 8]))
        bf16 = bool(rng.integers(0, 2))
        act = int(rng.integers(0, 4))
        bias = bool(rng.integers(0, 2))
        residual = bool(rng.integers(0, 2))
        packed = bool(rng.integers(0, 2))
        alpha = float(rng.choice([1.0, 0.5, -2.0]))
        out.append((M, N, K, split, bf16, act, bias, residual, packed, alpha))
    return out


@pytest.mark.parametrize("case", _cases(48, 2024), ids=lambda c: "M{}N{}K{}s{}{}a{}b{}r{}p{}x{}".format(
    c[0], c[1], c[2], c[3], "bf" if c[4] else "h", c[5], int(c[6]), int(c[7]), int(c[8]), c[9]))
def test_random_case(cuda_device, case):
    M, N, K, split, bf16, act, bias, residual, packed, alpha = case
    _run(cuda_device, M, N, K, bf16=bf16, bias=bias, residual=residual, alpha=alpha, act=act, packed=packed,
         split=split, seed=M * 7 + N * 3 + K)


def test_fused_launches_in_a_cuda_graph(cuda_device):
    """spmm24_launch_fused calls captured in a CUDA graph and replayed give
    the eager results bit for bit."""
    import torch

    import spmm24
    from test_gpu_epilogue import _dev, _problem

    shapes = [(512, 16, 2048), (256, 64, 1024), (512, 512, 1024)]
    bufs = []
    for i, (M, N, K) in enumerate(shapes):
        vals, meta, bp, _ = _problem(M, N, K, False, seed=40 + i)
        bias = torch.randn(M, device=cuda_device).half()
        bufs.append((M, N, K, _dev(vals, cuda_device), _dev(meta, cuda_device), _dev(bp, cuda_device), bias,
                     torch.empty(M * N, dtype=torch.int16, device=cuda_device),
                     torch.empty(M * N, dtype=torch.int16, device=cuda_device)))

    def run(use_second):
        for (M, N, K, A, E, B, bias, c1, c2) in bufs:
            rc = spmm24.launch_fused(torch.cuda.current_stream(cuda_device), A, B, E, c2 if use_second else c1, M, N,
                                     K, 0, spmm24.STATIC_WEIGHTS, bias=bias, activation=spmm24.ACT_GELU)
            assert rc == 0

    run(False)
    torch.cuda.synchronize(cuda_device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run(True)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(cuda_device)
    for (*_, c1, c2) in bufs:
        assert torch.equal(c1, c2)
    assert spmm24.device_status(cuda_device.index or 0) == 0
