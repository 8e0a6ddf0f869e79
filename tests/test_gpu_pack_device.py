"""The on-device packer (spmm24_pack_a_device, spmm24_prune_2of4_device,
spmm24_pack_b_device) against the host packer, bit for bit.  The host packer
is itself pinned to the reference's (test_packer.py), so these outputs equal
what toolCompressMatrixA + toolReorderMetadata / toolPackMatrixB
(SpeakOutLoudly/CUDA-Repo test/utils.h:91-229) produce."""
import numpy as np
import pytest

import oracle as O
from problems import compare, within_tolerance

pytestmark = pytest.mark.gpu

# fp16 bit patterns the packer must treat exactly like the host: signed
# zeros, infinities, a NaN, subnormals and ties.
SPECIAL = np.array([0x0000, 0x8000, 0x7C00, 0xFC00, 0x7E00, 0x0001, 0x8001, 0x3C00, 0xBC00, 0x3C00, 0x0400, 0x8400],
                   dtype=np.uint16)


def _dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device)


def _host(t):
    return t.cpu().numpy().view(np.uint16).reshape(-1)


def _dense(M, K, seed, special_frac=0.0):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K)).astype(np.float16).view(np.uint16)
    if special_frac:
        mask = rng.random((M, K)) < special_frac
        a[mask] = rng.choice(SPECIAL, size=int(mask.sum()))
    return a


@pytest.mark.parametrize("M,K", [(16, 64), (48, 192), (256, 256), (272, 320), (4096, 4096)])
def test_prune_and_pack_a_equals_host(cuda_device, M, K):
    import spmm24

    a = _dense(M, K, seed=M + K)
    vals, meta, bad = spmm24.pack_a_device(_dev(a, cuda_device), M, K, prune=True)
    pruned = spmm24.prune_2of4(a, M, K)
    hv, hm = spmm24.compress_reordered(pruned, M, K)
    assert bad == 0
    assert np.array_equal(_host(vals), hv)
    assert np.array_equal(_host(meta), hm)


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_special_values_and_ties(cuda_device, seed):
    """Signed zeros, inf, NaN, subnormals and equal magnitudes: the device
    prune keeps the same two positions as the host (first on ties) and the
    compress drops the same zeros."""
    import spmm24

    M, K = 64, 256
    a = _dense(M, K, seed, special_frac=0.5)
    vals, meta, bad = spmm24.pack_a_device(_dev(a, cuda_device), M, K, prune=True)
    hv, hm = spmm24.compress_reordered(spmm24.prune_2of4(a, M, K), M, K)
    assert bad == 0
    assert np.array_equal(_host(vals), hv)
    assert np.array_equal(_host(meta), hm)


def test_pack_a_without_prune_on_sparse_input(cuda_device):
    """Already 2:4-sparse weights (including groups of four zeros and -0) are
    compressed as toolCompressMatrixA does."""
    import spmm24

    M, K = 128, 512
    a = spmm24.prune_2of4(_dense(M, K, seed=7, special_frac=0.2), M, K).reshape(M, K)
    rng = np.random.default_rng(8)
    a[rng.random((M, K)) < 0.1] = 0x8000  # extra -0 entries keep the input 2:4
    vals, meta, bad = spmm24.pack_a_device(_dev(a, cuda_device), M, K, prune=False)
    hv, hm = spmm24.compress_reordered(a, M, K)
    assert bad == 0
    assert np.array_equal(_host(vals), hv)
    assert np.array_equal(_host(meta), hm)


def test_pack_a_counts_rows_that_are_not_2_4(cuda_device):
    import spmm24

    M, K = 64, 128
    a = spmm24.prune_2of4(_dense(M, K, seed=11), M, K).reshape(M, K)
    # break a known set of (row, 16-K block) units: three non-zeros in one group
    broken = [(0, 0), (5, 3), (63, 7), (17, 2)]
    for r, q in broken:
        a[r, 16 * q: 16 * q + 4] = np.array([1.0, 2.0, 3.0, 0.0], dtype=np.float16).view(np.uint16)
    _, _, bad = spmm24.pack_a_device(_dev(a, cuda_device), M, K, prune=False)
    assert bad == len(broken)
    with pytest.raises(ValueError):
        spmm24.compress_reordered(a, M, K)


@pytest.mark.parametrize("M,K", [(16, 4), (33, 20), (128, 4096)])
def test_prune_device_equals_host(cuda_device, M, K):
    import spmm24

    a = _dense(M, K, seed=M * K, special_frac=0.3)
    t = _dev(a, cuda_device)
    spmm24.prune_2of4_device(t, M, K)
    assert np.array_equal(_host(t), spmm24.prune_2of4(a, M, K))


@pytest.mark.parametrize("K,N", [(64, 1), (64, 8), (192, 13), (256, 64), (512, 100), (4096, 512)])
def test_pack_b_device_equals_host(cuda_device, K, N):
    import spmm24

    rng = np.random.default_rng(K + N)
    b = rng.standard_normal((K, N)).astype(np.float16).view(np.uint16)
    out = spmm24.pack_b_device(_dev(b, cuda_device), K, N)
    assert np.array_equal(_host(out), spmm24.pack_b(b, K, N))


def test_pack_b_device_unaligned_source(cuda_device):
    """A source that is only 2-byte aligned takes the element-wise path."""
    import torch

    import spmm24

    K, N = 128, 24
    rng = np.random.default_rng(5)
    b = rng.standard_normal((K, N)).astype(np.float16).view(np.uint16)
    buf = torch.zeros(K * N + 1, dtype=torch.int16, device=cuda_device)
    buf[1:] = _dev(b.reshape(-1), cuda_device)
    out = spmm24.pack_b_device(buf[1:], K, N)
    assert np.array_equal(_host(out), spmm24.pack_b(b, K, N))


def test_device_packed_operands_drive_the_spmm(cuda_device):
    """Dense weights and row-major activations packed on the device feed
    spmm24_launch; C matches the oracle's fp32 GEMM on the pruned weights."""
    import torch

    import spmm24

    M, N, K = 512, 32, 1024
    a = _dense(M, K, seed=21)
    rng = np.random.default_rng(22)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float16).view(np.uint16)
    vals, meta, bad = spmm24.pack_a_device(_dev(a, cuda_device), M, K, prune=True)
    assert bad == 0
    bp = spmm24.pack_b_device(_dev(b, cuda_device), K, N)
    c = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
    assert spmm24.launch(None, vals, bp, meta, c, M, N, K, None, 0) == 0
    torch.cuda.synchronize(cuda_device)
    ref = O.dense_gemm_f32(spmm24.prune_2of4(a, M, K), b.reshape(-1), M, N, K)
    got = c.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
    assert within_tolerance(compare(got, ref))
