"""GPU parity: the sm_100a kernel through the C ABI against the CPU oracle
(and against the reference's own kernel built for sm_100a, where it
supports the shape).  Tolerance: see tests/problems.py (max relative error
1e-2, mean absolute error 1e-3 against the oracle's fp32 result rounded to
fp16); integer-valued known-answer cases must match exactly."""
import numpy as np
import pytest

import oracle as O
from problems import compare, make_problem, oracle_c, pack_problem, within_tolerance

pytestmark = pytest.mark.gpu


def _to_dev(torch, arr, dev):
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).to(dev)


def run_gpu(p, split_k=0, dev=None, flags=None, stream=None):
    import torch

    import spmm24

    A = _to_dev(torch, p.vals, dev)
    E = _to_dev(torch, p.meta, dev)
    B = _to_dev(torch, p.b_packed, dev)
    C = torch.full((p.M, p.N), float("nan"), dtype=torch.float16, device=dev)
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    if flags is None:
        rc = spmm24.launch(s, A, B, E, C, p.M, p.N, p.K, None, split_k)
    else:
        rc = spmm24.launch_ex(s, A, B, E, C, p.M, p.N, p.K, split_k, flags)
    assert rc == 0, spmm24._lib.spmm24_last_error().decode()
    torch.cuda.synchronize(dev)
    return C.view(torch.int16).cpu().numpy().view(np.uint16)


def check(p, split_k, dev):
    got = run_gpu(p, split_k, dev)
    stats = compare(got, oracle_c(p))
    assert within_tolerance(stats), stats
    return got


def test_config1_correctness_run(cuda_device):
    """M=256, K=256, N=128, A N(0,1) seed 0 magnitude-pruned,
    B U(-1,1) seed 1, split_K=1."""
    p = make_problem(256, 128, 256, seed=0)
    check(p, 1, cuda_device)


def test_known_answer_reference_inputs(cuda_device):
    """The reference harness's own inputs (kept values 1.0 with its glibc
    rand() mask, B all ones): every output is exactly K/2."""
    M, N, K = 256, 128, 256
    a = O.ref_init_pruned(M, K)
    b = np.full(K * N, 0x3C00, dtype=np.uint16)
    got = run_gpu(pack_problem(M, N, K, a, b), 1, cuda_device)
    assert np.all(got.view(np.float16) == K / 2)


@pytest.mark.parametrize("shape", [
    (128, 16, 128),   # one stage
    (128, 16, 64),    # a single (odd) 64-K group
    (256, 8, 192),    # odd group count, N below the MMA tile
    (16, 1, 64),      # one band, one column
    (144, 12, 320),   # ragged M tile, ragged N strip, odd groups
    (384, 40, 512),
    (512, 200, 1024),
    (256, 256, 256),
    (128, 520, 256),  # several N tiles with a ragged last tile
])
@pytest.mark.parametrize("split_k", [1, 2, 3, 0])
def test_shapes_and_splits(cuda_device, shape, split_k):
    M, N, K = shape
    p = make_problem(M, N, K, seed=M + N + K)
    check(p, split_k, cuda_device)


@pytest.mark.parametrize("shape", [(128, 1, 320), (144, 12, 320), (256, 16, 1024), (1152, 8, 704), (4096, 32, 4096),
                                   (16, 1, 64)])
def test_stream_k_kernel_shapes(cuda_device, shape):
    """The stream-K kernel (the allocation-free entry point's): grids of 3,
    6, 16, 54 and 148 CTAs sharing tiles, single-unit tiles, ragged M and N,
    odd 64-K group counts; a second call (its flags cleared again) agrees bit
    for bit."""
    import torch

    import spmm24

    M, N, K = shape
    p = make_problem(M, N, K, seed=M + 7 * N)
    A = _to_dev(torch, p.vals, cuda_device)
    E = _to_dev(torch, p.meta, cuda_device)
    B = _to_dev(torch, p.b_packed, cuda_device)
    import ctypes

    fn = ctypes.CDLL(spmm24.library_path()).spmm24_launch_noalloc
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 3
    fn.restype = ctypes.c_int
    outs = []
    for _ in range(2):
        C = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
        rc = fn(torch.cuda.current_stream(cuda_device).cuda_stream, A.data_ptr(), B.data_ptr(), E.data_ptr(),
                C.data_ptr(), M, N, K)
        assert rc == 0, spmm24._lib.spmm24_last_error().decode()
        torch.cuda.synchronize(cuda_device)
        outs.append(C.view(torch.int16).cpu().numpy().view(np.uint16))
    assert within_tolerance(compare(outs[0], oracle_c(p)))
    assert np.array_equal(outs[0], outs[1])


@pytest.mark.parametrize("deep_ring", [0, 1])
def test_flags_and_streams(cuda_device, tuning, deep_ring):
    """Static-weight prefetch, launches without PDL, and a second stream all
    give the same bits, with the shallow (two CTAs per SM) and the deep ring."""
    import torch

    import spmm24

    tuning(deep_ring=deep_ring)
    p = make_problem(2048, 16, 2048, seed=12, a_scale=0.02, b_dist="normal")
    ref = check(p, 0, cuda_device)
    assert np.array_equal(ref, run_gpu(p, 0, cuda_device, flags=spmm24.STATIC_WEIGHTS))
    assert np.array_equal(ref, run_gpu(p, 0, cuda_device, flags=spmm24.NO_PDL))
    s2 = torch.cuda.Stream(cuda_device)
    assert np.array_equal(ref, run_gpu(p, 0, cuda_device, stream=s2))
    assert within_tolerance(compare(run_gpu(p, 4, cuda_device, flags=spmm24.STATIC_WEIGHTS), oracle_c(p)))
    rc = spmm24.launch_ex(None, 16, 16, 16, 16, 256, 16, 256, 0, 8)
    assert rc == spmm24.CUDA_ERROR_INVALID_VALUE


def test_back_to_back_calls_pdl(cuda_device):
    """A chain of dependent calls on one stream (each call's output is the
    next call's activation), launched with programmatic dependent launch."""
    import torch

    import spmm24

    M = K = 1024
    N = 16
    p = make_problem(M, N, K, seed=13, a_scale=0.03, b_dist="normal")
    A = _to_dev(torch, p.vals, cuda_device)
    E = _to_dev(torch, p.meta, cuda_device)
    x = torch.from_numpy(p.b_rowmajor.view(np.float16).reshape(K, N).copy()).to(cuda_device)
    xs_host = [p.b_rowmajor.copy()]
    s = torch.cuda.current_stream(cuda_device)
    bufs = []
    for step in range(4):
        Bp = x.reshape(K, N // 8, 8).permute(1, 0, 2).contiguous()  # pack on device (strips of 8 columns)
        C = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
        rc = spmm24.launch_ex(s, A, Bp, E, C, M, N, K, 0, spmm24.STATIC_WEIGHTS)
        assert rc == 0
        bufs.append((Bp, C))
        x = C
    torch.cuda.synchronize(cuda_device)
    # replay the chain on the CPU oracle
    b = p.b_rowmajor
    for step in range(4):
        ref = O.dense_gemm_f32(p.a_dense, b, M, N, K)
        got = bufs[step][1].view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
        assert within_tolerance(compare(got, ref)), step
        b = got  # feed the GPU's fp16 output forward, as the chain did
        xs_host.append(b)


@pytest.mark.parametrize("shape", [
    (256, 256, 128),     # one pair, one stage
    (512, 512, 512),
    (272, 264, 384),     # ragged M (one band past a pair tile) and ragged N
    (4096, 520, 1024),   # several pairs, ragged last N tile
    (768, 1000, 256),    # N not a multiple of 8: scalar stores
    (1024, 512, 4096),   # few tiles, long K: the automatic K split
    (768, 520, 3200),    # odd stage count split unevenly, ragged N
])
@pytest.mark.parametrize("split", [1, 2])
def test_cta_pair_kernel(cuda_device, tuning, shape, split):
    """The cta_group::2 pair kernel (256 x 256 tiles, K % 128 == 0), one pair
    per tile or two pairs along K reducing through distributed shared
    memory."""
    import spmm24

    # pair=1: also the few-tile shapes the picker gives to split-K clusters;
    # tile_n=256: also the sub-wave shapes it gives to 256 x 128 pair tiles
    tuning(pair=1, pair2=0, pair_split=split, tile_n=256)
    M, N, K = shape
    cfg = spmm24.select_config(M, N, K)
    assert cfg["cta_pair"] == 1 and cfg["tile_n"] == 256 and cfg["split_k"] == (split if K >= 256 else 1)
    p = make_problem(M, N, K, seed=3 * M + N)
    check(p, 0, cuda_device)


@pytest.mark.parametrize("shape", [
    (256, 128, 128),     # one pair, one stage
    (512, 384, 512),
    (272, 200, 384),     # ragged M (one band past a pair tile) and ragged N
    (768, 1000, 256),    # N not a multiple of 8: scalar stores
    (1024, 512, 4096),   # the sub-wave case the picker gives this tile
    (768, 520, 3200),    # odd stage count, ragged N
])
def test_cta_pair_narrow_tiles(cuda_device, tuning, shape):
    """The pair kernel with 256 x 128 tiles (64 columns of B per CTA, a
    6-stage ring)."""
    import spmm24

    tuning(pair=1, tile_n=128)
    M, N, K = shape
    cfg = spmm24.select_config(M, N, K)
    assert cfg["cta_pair"] == 1 and cfg["tile_m"] == 256 and cfg["tile_n"] == 128 and cfg["stages"] == 6
    check(make_problem(M, N, K, seed=7 * M + N), 0, cuda_device)


def test_cta_pair_narrow_epilogues(cuda_device, tuning):
    """The 256 x 128 pair tile through the general epilogue: bias + SiLU,
    a residual, bf16 and a packed-B output, each bit for bit the wide pair
    tile's result (the same MMAs in the same K order, the same epilogue)."""
    import torch

    import spmm24

    dev = cuda_device
    M, N, K = 512, 384, 1024
    p = make_problem(M, N, K, seed=77, a_scale=0.05, b_dist="normal")
    A = torch.from_numpy(p.vals.view(np.int16)).to(dev)
    E = torch.from_numpy(p.meta.view(np.int16)).to(dev)
    B = torch.from_numpy(p.b_packed.view(np.int16)).to(dev)
    bias = (torch.randn(M, device=dev) * 0.1).half()
    res = torch.randn(M, N, device=dev).half()
    cases = [dict(bias=bias, activation=spmm24.ACT_SILU), dict(residual=res, alpha=0.5),
             dict(out_layout=spmm24.OUT_PACKED_B, bias=bias)]
    for kw in cases:
        outs = []
        for tn in (128, 256):
            tuning(pair=1, pair2=0, tile_n=tn)
            C = torch.full((M * N,), -1, dtype=torch.int16, device=dev)
            assert spmm24.launch_fused(None, A, B, E, C, M, N, K, 1, 0, **kw) == 0, \
                spmm24._lib.spmm24_last_error().decode()
            torch.cuda.synchronize(dev)
            outs.append(C)
        assert torch.equal(outs[0], outs[1]), kw
    assert spmm24.device_status(0) == 0


@pytest.mark.parametrize("shape", [
    (512, 240, 128),     # one pair tile, one stage
    (1024, 480, 512),
    (592, 500, 384),     # ragged M (second half of a pair partly past M) and ragged N
    (4096, 1004, 1024),  # N not a multiple of 8: scalar stores
    (2048, 2048, 1024),
    (1536, 4096, 640),   # odd stage count
])
def test_cta_pair_two_m_halves(cuda_device, tuning, shape):
    """The pair kernel with two M halves per pair (512 x 240 tiles: two
    M=256 MMAs share each B tile, two TMEM accumulators)."""
    import spmm24

    tuning(pair2=1)
    M, N, K = shape
    cfg = spmm24.select_config(M, N, K)
    assert cfg["cta_pair"] == 1 and cfg["tile_m"] == 512 and cfg["tile_n"] == 240
    check(make_problem(M, N, K, seed=5 * M + N), 0, cuda_device)


@pytest.mark.parametrize("shape", [(1024, 256, 8192), (3584, 256, 2048), (256, 200, 1024), (512, 136, 4096)],
                         ids=lambda s: "x".join(map(str, s)))
def test_few_tile_wide_n_takes_split_k_clusters(cuda_device, shape):
    """N <= 256 with pairs for less than three quarters of the SMs: the
    picker takes 128-wide cluster tiles with a K split (at most 4)."""
    import spmm24

    M, N, K = shape
    cfg = spmm24.select_config(M, N, K)
    assert cfg["cta_pair"] == 0 and cfg["tile_n"] == 128 and 1 <= cfg["split_k"] <= 4
    check(make_problem(M, N, K, seed=M + 11 * N), 0, cuda_device)


def test_cta_pair_forced_small_n(cuda_device, tuning):
    """The pair kernel forced on N below its tile (most of B is zero-filled)."""
    import spmm24

    tuning(pair=1)
    assert spmm24.select_config(384, 40, 512)["cta_pair"] == 1
    check(make_problem(384, 40, 512, seed=9), 0, cuda_device)


@pytest.mark.parametrize("parts", [2, 4, 8])
def test_m_shards_reproduce_full_launch(cuda_device, parts):
    """Launching every M-shard (shard views of A / metadata, rows of C) gives
    the unsharded result bit for bit -- the multi-GPU partition, on one GPU."""
    import torch

    import spmm24

    M, N, K = 2048, 32, 1024
    p = make_problem(M, N, K, seed=parts)
    A, E, B = _to_dev(torch, p.vals, cuda_device), _to_dev(torch, p.meta, cuda_device), _to_dev(torch, p.b_packed, cuda_device)
    full = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
    assert spmm24.launch(None, A, B, E, full, M, N, K, None, 1) == 0
    sharded = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
    for i in range(parts):
        r0, r1 = spmm24.shard_rows(M, parts, i, 128)
        a, e = spmm24.shard_views(A, E, M, K, r0, r1)
        assert spmm24.launch(None, a, B, e, sharded[r0:r1], r1 - r0, N, K, None, 1) == 0
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(full.view(torch.int16), sharded.view(torch.int16))


@pytest.mark.parametrize("split_k", [1, 2, 3, 4, 5, 6, 7, 8])
def test_llama7b_decode_split_sweep(cuda_device, split_k):
    """BASELINE config 2 shape (M=K=4096, N=16), split_K swept over 1..8."""
    p = make_problem(4096, 16, 4096, seed=2, a_scale=0.02, b_dist="normal")
    check(p, split_k, cuda_device)


@pytest.mark.parametrize("M,K", [(11008, 4096), (4096, 11008)])
@pytest.mark.parametrize("N", [1, 8, 32])
def test_llama7b_decode_full_size_row_sample(cuda_device, M, K, N):
    """Full-size decode layers, checked on a seeded sample of rows."""
    p = make_problem(M, N, K, seed=3, a_scale=0.02, b_dist="normal")
    got = run_gpu(p, 0, cuda_device).reshape(M, N)
    rows = np.sort(np.random.default_rng(0).choice(M, 256, replace=False))
    stats = compare(got[rows].reshape(-1), oracle_c(p, rows))
    assert within_tolerance(stats), stats


def test_prefill_shape_row_sample(cuda_device):
    """BASELINE config 3 shape (4096 x 4096, N=512), sampled rows."""
    M, N, K = 4096, 512, 4096
    p = make_problem(M, N, K, seed=4, a_scale=0.02, b_dist="normal")
    got = run_gpu(p, 1, cuda_device).reshape(M, N)
    rows = np.sort(np.random.default_rng(1).choice(M, 128, replace=False))
    stats = compare(got[rows].reshape(-1), oracle_c(p, rows))
    assert within_tolerance(stats), stats


@pytest.mark.parametrize("M,N,K", [(28672, 16, 8192), (8192, 256, 28672), (28672, 4096, 8192)])
def test_llama70b_full_size_row_sample(cuda_device, M, N, K):
    """BASELINE config 4's largest layers at full size (the cluster kernel
    with split-K, the CTA pair with its K split, the two-M-half pair),
    checked on a seeded sample of rows."""
    p = make_problem(M, N, K, seed=8, a_scale=0.01, b_dist="normal")
    got = run_gpu(p, 0, cuda_device).reshape(M, N)
    rows = np.sort(np.random.default_rng(2).choice(M, 96, replace=False))
    stats = compare(got[rows].reshape(-1), oracle_c(p, rows))
    assert within_tolerance(stats), stats


def test_long_k_integer_exact(cuda_device):
    """K = 65536 (512 stages of 128 K, split across a cluster) with A = +-1
    on a random 2:4 mask and B in {-1, 0, 1}: every partial sum is an exact
    integer in fp32, so C must equal the rounded exact product bit for bit."""
    M, N, K = 256, 16, 65536
    rng = np.random.default_rng(9)
    a = np.where(rng.random(M * K) < 0.5, 0x3C00, 0xBC00).astype(np.uint16)  # +-1.0
    a = O.random_mask_2of4(a, M, K, 99)
    b = np.array([0xBC00, 0x0000, 0x3C00], dtype=np.uint16)[rng.integers(0, 3, K * N)]
    p = pack_problem(M, N, K, a, b)
    got = run_gpu(p, 0, cuda_device)
    ref = O.f32_to_f16_bits(oracle_c(p).reshape(-1))
    assert np.array_equal(got.reshape(-1), ref)


def test_many_row_tiles(cuda_device):
    """M = 65536 (512 row tiles on the grid's third dimension), short K."""
    p = make_problem(65536, 16, 256, seed=10)
    check(p, 0, cuda_device)


def test_random_mask_square(cuda_device):
    """BASELINE config 5 inputs (U(-1,1) with a uniformly random 2:4 mask)."""
    p = make_problem(1024, 1024, 1024, seed=5, a_dist="uniform", mask="random")
    got = run_gpu(p, 0, cuda_device).reshape(1024, 1024)
    rows = np.arange(0, 1024, 7)
    stats = compare(got[rows].reshape(-1), oracle_c(p, rows))
    assert within_tolerance(stats), stats


def test_deterministic_for_fixed_split(cuda_device):
    p = make_problem(1024, 32, 2048, seed=6)
    a = run_gpu(p, 4, cuda_device)
    b = run_gpu(p, 4, cuda_device)
    assert np.array_equal(a, b)


@pytest.mark.skipif(not O.ref_spmm_available(), reason="reference kernel not built (oracle/_ref)")
@pytest.mark.parametrize("N", [8, 16, 32, 64, 128])
def test_matches_reference_kernel(cuda_device, N):
    """Same packed inputs through the reference's own SpMM_N2M4_Launch
    (compiled for sm_100a from its sources) and through this library."""
    import torch

    M, K = 512, 1024
    p = make_problem(M, N, K, seed=7)
    ref = O.ref_spmm()
    assert ref.ref_spmm_supported(M, N, K, 1)
    A = _to_dev(torch, p.vals, cuda_device)
    E = _to_dev(torch, p.meta, cuda_device)
    B = _to_dev(torch, p.b_packed, cuda_device)
    C = torch.zeros((M, N), dtype=torch.float16, device=cuda_device)
    rc = ref.ref_spmm_launch(torch.cuda.current_stream().cuda_stream, A.data_ptr(), B.data_ptr(), E.data_ptr(),
                             C.data_ptr(), M, N, K, None, 1)
    assert rc == 0
    torch.cuda.synchronize()
    ref_bits = C.view(torch.int16).cpu().numpy().view(np.uint16)
    ours = run_gpu(p, 1, cuda_device)
    ref_f32 = ref_bits.view(np.float16).astype(np.float32)
    stats = compare(ours, ref_f32)
    assert within_tolerance(stats), stats
    # and the reference kernel itself agrees with the oracle
    assert within_tolerance(compare(ref_bits, oracle_c(p)))


def test_no_bounded_wait_gave_up(cuda_device):
    import spmm24

    p = make_problem(512, 64, 1024, seed=8)
    run_gpu(p, 2, cuda_device)
    assert spmm24.device_status(0) == 0
