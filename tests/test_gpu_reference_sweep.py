"""GPU parity on the reference's own test sweep, through the reference's own
launcher symbol.

The reference's correctness script (test/build/kernelTest.sh:4-11) runs 31
LLaMA / Qwen linear-layer shapes (M, K), each with its own Split_K, at
N in {8, 16, 32}, and a debug case M = K = 4096, N = 128, Split_K = 4
(kernelTest.sh:16-19).  Every case here goes through the C++ drop-in
exported under the reference's mangled name
(_Z16SpMM_N2M4_LaunchP11CUstream_stPK6__halfS3_PKtPS1_iiiS6_i, the symbol
test/kernelTest.cu:193,197 binds), and is checked

  * against the oracle's fp32 dense GEMM on the pruned A, on a seeded sample
    of rows (the tolerance of tests/problems.py);
  * against the reference's own kernel built for sm_100a (oracle/_ref), on
    the same packed inputs with the same Split_K, where that kernel supports
    the shape.  The reference rounds each split-K partial sum to fp16 before
    its reduction pass (src/SpMM_Kernel.cuh:473-489, reduce_Kernel.cuh:
    27-53), which can put it outside the fp16 tolerance of the exact result
    (up to 0.19 relative on single elements at Split_K 3-7 in this sweep); so both
    kernels are held to a per-element bound derived from that algorithm: the
    oracle emulates it (fp32 partials over the reference's K ranges, each
    rounded to fp16, summed in fp32, rounded), the reference kernel must match
    the emulation, and this library must match the reference kernel, within
    sum_s ulp(partial_s) + 2 ulp(C) + 2^-15 sum_k |a_k b_k| per element;
  * bit for bit against spmm24_launch with the same split_k.

Weights are N(0, 0.02) generated on the device, magnitude-pruned 2:4 by
spmm24_prune_2of4_device and packed by spmm24_pack_a_device (both bit-exact
with the host packer, tests/test_gpu_pack_device.py); activations N(0, 1),
packed by spmm24_pack_b_device.  The oracle sees only the pruned dense rows
and the row-major B, so it does not depend on either packer.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
from problems import compare, within_tolerance

pytestmark = pytest.mark.gpu

# test/build/kernelTest.sh:4-8 (M, K and SPLIT_K, in the script's order)
REF_M = [8192, 4096, 32000, 32000, 28672, 5120, 5120, 3584, 4096, 13824, 8192, 18944, 14336, 4096, 8192, 11008,
         32000, 20480, 3584, 21504, 7168, 28672, 7168, 27648, 9216, 36864, 9216, 36864, 12288, 49152, 12288]
REF_K = [29568, 4096, 5120, 8192, 8192, 5120, 13824, 20480, 11008, 5120, 8192, 3584, 4096, 14336, 28672, 4096,
         4096, 3584, 18944, 7168, 7168, 7168, 28672, 9216, 9216, 9216, 36864, 12288, 12288, 12288, 49152]
REF_SPLIT_K = [7, 7, 3, 3, 4, 5, 5, 7, 7, 3, 7, 7, 7, 7, 7, 7, 3, 6, 7, 1, 3, 4, 3, 7, 5, 2, 5, 2, 6, 3, 6]
REF_N = [8, 16, 32]
SWEEP = list(zip(REF_M, REF_K, REF_SPLIT_K))
DEBUG_CASE = (4096, 4096, 128, 4)  # kernelTest.sh:16-19

MANGLED = "_Z16SpMM_N2M4_LaunchP11CUstream_stPK6__halfS3_PKtPS1_iiiS6_i"
SAMPLE_ROWS = 48


def _dropin():
    import spmm24

    fn = getattr(ctypes.CDLL(spmm24.library_path()), MANGLED)
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 3 + [ctypes.c_void_p, ctypes.c_int]
    fn.restype = ctypes.c_int
    return fn


def _layer(dev, M, K, seed):
    import torch

    import spmm24

    g = torch.Generator(device=dev).manual_seed(seed)
    a = (torch.randn(M, K, generator=g, device=dev) * 0.02).half()
    spmm24.prune_2of4_device(a, M, K)
    vals, meta, bad = spmm24.pack_a_device(a, M, K)
    assert bad == 0
    return a, vals, meta


def _activations(dev, K, N, seed):
    import torch

    import spmm24

    g = torch.Generator(device=dev).manual_seed(seed)
    b = torch.randn(K, N, generator=g, device=dev).half()
    return b, spmm24.pack_b_device(b, K, N)


def _rows(M, seed):
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([[0, M - 1], rng.choice(M, SAMPLE_ROWS - 2, replace=False)]))


def _ulp16(x):
    """fp16 unit in the last place at |x| (subnormal spacing below 2^-14)."""
    ax = np.maximum(np.abs(x.astype(np.float64)), 2.0 ** -14)
    return 2.0 ** (np.floor(np.log2(ax)) - 10)


def _reference_emulation(a_rows, b, n_rows, N, K, split_k):
    """The reference's split-K arithmetic on the given rows: partial sums over
    its K ranges (64-wide K blocks, ceil(blocks / Split_K) per split, the last
    split the remainder; src/SpMM_Kernel.cuh:324-334), each rounded to fp16,
    summed in fp32 in split order and rounded (reduce_Kernel.cuh:27-53).
    Returns (C as fp32 values of fp16, the per-element bound
    sum_s ulp(partial_s) + 2 ulp(C) + 2^-15 sum_k |a_k b_k|; the last term
    covers fp32 accumulation in another order -- the tensor cores' against
    the oracle's sequential sum -- where the result cancels)."""
    kt = K // 64
    avg = (kt - 1) // split_k + 1
    A = a_rows.reshape(n_rows, K)
    Bm = b.reshape(K, N)
    acc = np.zeros((n_rows, N), dtype=np.float32)
    bound = np.zeros((n_rows, N), dtype=np.float64)
    for s in range(split_k):
        k0, k1 = 64 * s * avg, 64 * min((s + 1) * avg, kt)
        if k1 <= k0:
            continue
        part = O.dense_gemm_f32(np.ascontiguousarray(A[:, k0:k1]).reshape(-1),
                                np.ascontiguousarray(Bm[k0:k1]).reshape(-1), n_rows, N, k1 - k0).reshape(n_rows, N)
        p16 = part.astype(np.float16).astype(np.float32)
        acc += p16
        bound += _ulp16(part)
    c = acc.astype(np.float16).astype(np.float32)
    mag = O.dense_gemm_f32(np.ascontiguousarray(a_rows & 0x7FFF), np.ascontiguousarray(b & 0x7FFF), n_rows, N,
                           K).reshape(n_rows, N)
    return c, bound + 2 * _ulp16(c) + 2.0 ** -15 * mag


def _bits(t):
    import torch

    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _run_case(dev, a, vals, meta, M, K, N, split_k, seed, check_reference=True):
    import torch

    import spmm24

    b, bp = _activations(dev, K, N, seed)
    rows = _rows(M, seed)
    ref_c = O.dense_gemm_f32(_bits(a[torch.from_numpy(rows).to(dev)]).reshape(-1), _bits(b).reshape(-1),
                             len(rows), N, K).reshape(len(rows), N)
    s = torch.cuda.current_stream(dev).cuda_stream
    # the drop-in, called as the reference's callers call it (a workspace is
    # passed, as test/kernelTest.cu:136 allocates one; the library ignores it)
    ws = torch.empty(split_k * M * N, dtype=torch.float16, device=dev)
    c = torch.full((M, N), float("nan"), dtype=torch.float16, device=dev)
    rc = _dropin()(s, vals.data_ptr(), bp.data_ptr(), meta.data_ptr(), c.data_ptr(), M, N, K, ws.data_ptr(), split_k)
    assert rc == 0, spmm24._lib.spmm24_last_error().decode()
    torch.cuda.synchronize(dev)
    got = _bits(c)
    stats = compare(got[rows], ref_c)
    assert within_tolerance(stats), (M, K, N, split_k, stats)
    # the extern "C" entry point gives the same bits
    c2 = torch.full((M, N), float("nan"), dtype=torch.float16, device=dev)
    assert spmm24.launch(s, vals, bp, meta, c2, M, N, K, None, split_k) == 0
    torch.cuda.synchronize(dev)
    assert np.array_equal(got, _bits(c2))
    if check_reference and O.ref_spmm_available():
        ref = O.ref_spmm()
        if ref.ref_spmm_supported(M, N, K, split_k):
            c3 = torch.zeros((M, N), dtype=torch.float16, device=dev)
            rc = ref.ref_spmm_launch(s, vals.data_ptr(), bp.data_ptr(), meta.data_ptr(), c3.data_ptr(), M, N, K,
                                     ws.data_ptr(), split_k)
            assert rc == 0
            torch.cuda.synchronize(dev)
            refk = _bits(c3)
            a_rows = _bits(a[torch.from_numpy(rows).to(dev)]).reshape(-1)
            emu, bound = _reference_emulation(a_rows, _bits(b).reshape(-1), len(rows), N, K, split_k)
            rk = refk[rows].view(np.float16).astype(np.float32)
            ours = got[rows].view(np.float16).astype(np.float32)
            assert np.all(np.abs(rk - emu) <= bound), ("reference kernel vs its emulation", M, K, N, split_k,
                                                       float(np.max(np.abs(rk - emu) - bound)))
            assert np.all(np.abs(ours - rk) <= bound), ("ours vs reference kernel", M, K, N, split_k,
                                                        float(np.max(np.abs(ours - rk) - bound)))
            if split_k == 1:  # no partial rounding: the plain fp16 tolerance holds for the reference too
                assert within_tolerance(compare(refk[rows], ref_c)), ("reference kernel vs oracle", M, K, N)
    return got


@pytest.mark.parametrize("case", range(len(SWEEP)), ids=[f"{m}x{k}_sk{s}" for (m, k, s) in SWEEP])
def test_reference_sweep(cuda_device, case):
    """One (M, K, Split_K) of kernelTest.sh at N = 8, 16 and 32, plus the
    library's own split choice at N = 8."""
    import torch

    M, K, split_k = SWEEP[case]
    a, vals, meta = _layer(cuda_device, M, K, seed=case)
    for N in REF_N:
        _run_case(cuda_device, a, vals, meta, M, K, N, split_k, seed=1000 * case + N)
    _run_case(cuda_device, a, vals, meta, M, K, 8, 0, seed=1000 * case + 1, check_reference=False)
    del a, vals, meta
    torch.cuda.empty_cache()


def test_reference_debug_case(cuda_device):
    """kernelTest.sh's debug case: M = K = 4096, N = 128, Split_K = 4."""
    M, K, N, split_k = DEBUG_CASE
    a, vals, meta = _layer(cuda_device, M, K, seed=99)
    _run_case(cuda_device, a, vals, meta, M, K, N, split_k, seed=4242)


def test_square_16384_row_sample(cuda_device):
    """BASELINE config 5's largest square, M = N = K = 16384 (8.8 TFLOP
    dense-equivalent): U(-1,1) weights with a uniformly random 2:4 mask,
    B U(-1,1), checked on a row sample against the oracle."""
    import torch

    import spmm24

    M = N = K = 16384
    g = torch.Generator(device=cuda_device).manual_seed(16384)
    a = (torch.rand(M, K, generator=g, device=cuda_device) * 2 - 1).half()
    # random 2-of-4 mask: keep the two positions with the smallest keys of four random keys
    keys = torch.rand(M * K // 4, 4, generator=g, device=cuda_device)
    keep = keys.argsort(dim=1)[:, :2]
    mask = torch.zeros(M * K // 4, 4, dtype=torch.bool, device=cuda_device).scatter_(1, keep, True)
    a = (a.view(-1, 4) * mask).view(M, K)
    del keys, keep, mask
    vals, meta, bad = spmm24.pack_a_device(a, M, K)
    assert bad == 0
    b = (torch.rand(K, N, generator=g, device=cuda_device) * 2 - 1).half()
    bp = spmm24.pack_b_device(b, K, N)
    c = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
    assert spmm24.launch(torch.cuda.current_stream(cuda_device), vals, bp, meta, c, M, N, K, None, 0) == 0
    torch.cuda.synchronize(cuda_device)
    rows = _rows(M, 5)[:16]
    ref_c = O.dense_gemm_f32(_bits(a[torch.from_numpy(rows).to(cuda_device)]).reshape(-1), _bits(b).reshape(-1),
                             len(rows), N, K).reshape(len(rows), N)
    got = _bits(c[torch.from_numpy(rows).to(cuda_device)])
    stats = compare(got, ref_c)
    assert within_tolerance(stats), stats
    assert spmm24.device_status(0) == 0
