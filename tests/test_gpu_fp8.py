"""spmm24_launch_fp8 (OCP E4M3 / E5M2 operands, kind::f8f6f4 sparse MMAs)
against the oracle: fp8 decode -> fp32 GEMM in increasing k, epilogue in
float64, rounded to C's type.

Tolerance: fp8 products are exact in fp32; the GPU and the oracle differ
only in the order (and the tensor core's internal precision) of the fp32
sums, so |got - ref| <= 2^-10 |ref| + 2^-12 S, S = sum_k |a_mk b_nk|,
plus the final rounding to C's type, is a bound a wrong metadata index or
operand layout cannot meet.  Integer-valued cases are exact."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

from test_gpu_epilogue import _act, _bits_to_f32, _round  # noqa: E402


def _u8dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint8)).to(device)


def _i16dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).to(device)


def _dense_f32(bits, fmt, shape):
    return O.fp8_to_f32(bits.reshape(-1), fmt).reshape(shape).astype(np.float64)


def _problem(M, N, K, fmt_a, fmt_b, seed, integer=False):
    import spmm24

    rng = np.random.default_rng(seed)
    if integer:
        a = rng.integers(-4, 5, (M, K)).astype(np.float32)
        b = rng.integers(-3, 4, (N, K)).astype(np.float32)
    else:
        a = rng.standard_normal((M, K)).astype(np.float32)
        b = rng.standard_normal((N, K)).astype(np.float32)
    a_bits = spmm24.prune_2of4_fp8(O.f32_to_fp8(a.reshape(-1), fmt_a), M, K, fmt_a)
    b_bits = O.f32_to_fp8(b.reshape(-1), fmt_b)
    vals, meta = spmm24.compress_a_fp8(a_bits, M, K)
    acc = O.spmm_fp8_f32(vals, meta, b_bits, M, N, K, fmt_a, fmt_b).reshape(M, N).astype(np.float64)
    A = _dense_f32(a_bits, fmt_a, (M, K))
    B = _dense_f32(b_bits, fmt_b, (N, K))
    S = np.abs(A) @ np.abs(B).T
    return vals, meta, b_bits, acc, S


def _run(dev, M, N, K, *, fmt_a=0, fmt_b=0, split=0, bf16=False, bias=False, residual=False, alpha=1.0, act=0,
         packed=False, seed=0, integer=False):
    import torch

    import spmm24

    vals, meta, b_bits, acc, S = _problem(M, N, K, fmt_a, fmt_b, seed, integer)
    rng = np.random.default_rng(seed + 7)
    bias_bits = _round(rng.standard_normal(M), bf16) if bias else None
    res_bits = _round(rng.standard_normal((M, N)), bf16).reshape(M, N) if residual else None
    strips = (N + 7) // 8
    # every element of C (the pad columns of a packed C too) must be written
    c = torch.full((strips * 8 * M if packed else M * N,), -1, dtype=torch.int16, device=dev)
    res_dev = None
    if residual:
        if packed:
            pad = np.zeros((M, strips * 8), dtype=np.uint16)
            pad[:, :N] = res_bits
            res_layout = pad.reshape(M, strips, 8).transpose(1, 0, 2).reshape(-1)
        else:
            res_layout = res_bits.reshape(-1)
        res_dev = _i16dev(res_layout, dev)
    flags = (spmm24.FP8_A_E5M2 if fmt_a else 0) | (spmm24.FP8_B_E5M2 if fmt_b else 0) | (spmm24.BF16 if bf16 else 0)
    rc = spmm24.launch_fp8(None, _u8dev(vals, dev), _u8dev(b_bits, dev), _u8dev(meta, dev), c, M, N, K, split, flags,
                           bias=_i16dev(bias_bits, dev) if bias else None, residual=res_dev, alpha=alpha,
                           activation=act, out_layout=spmm24.OUT_PACKED_B if packed else spmm24.OUT_ROW_MAJOR)
    assert rc == 0, spmm24._lib.spmm24_last_error().decode()
    torch.cuda.synchronize(dev)
    got_bits = c.cpu().numpy().view(np.uint16)
    if packed:
        full = got_bits.reshape(strips, M, 8).transpose(1, 0, 2).reshape(M, strips * 8)
        assert not full[:, N:].any(), "pad columns of a packed C must be zero"
        got_bits = full[:, :N]
    got_bits = got_bits.reshape(M, N)
    assert spmm24.device_status(dev.index or 0) == 0

    y = alpha * acc
    if bias:
        y = y + _bits_to_f32(bias_bits, bf16).astype(np.float64)[:, None]
    y = _act(y, act)
    if residual:
        y = y + _bits_to_f32(res_bits, bf16).astype(np.float64).reshape(M, N)
    ref_bits = _round(y.astype(np.float32), bf16).reshape(M, N)
    if integer and not (bias or residual or act or alpha != 1.0):
        assert np.array_equal(got_bits, ref_bits), int((got_bits != ref_bits).sum())
        return
    got = _bits_to_f32(got_bits, bf16).reshape(M, N).astype(np.float64)
    ref = _bits_to_f32(ref_bits, bf16).reshape(M, N).astype(np.float64)
    assert np.isfinite(got).all()
    ulp = 2.0 ** (-7 if bf16 else -10)
    # the epilogue's slope (<= 1.1 for the activations) scales the sum error
    tol = ulp * np.abs(ref) + 1.2 * abs(alpha) * 2.0 ** -12 * S + 1e-6
    bad = np.abs(got - ref) > tol
    assert not bad.any(), (int(bad.sum()), float(np.abs(got - ref).max()))


# (M, N, K, split): one half-filled stage (odd metadata groups: the tail
# patch), decode shapes with cluster K splits, every N tile (16, 32, 64,
# 128), ragged N, N = 1.
SHAPES = [
    (128, 16, 128, 0),
    (256, 16, 384, 0),
    (4096, 16, 4096, 0),
    (2048, 32, 2048, 3),
    (1024, 64, 1024, 0),
    (512, 128, 512, 0),
    (256, 200, 768, 0),
    (512, 8, 4096, 0),
    (1024, 1, 2048, 0),
    (384, 24, 1152, 8),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_fp8_e4m3_matches_oracle(cuda_device, shape):
    M, N, K, split = shape
    _run(cuda_device, M, N, K, split=split, seed=M + N + K)


@pytest.mark.parametrize("fmts", [(0, 0), (1, 0), (0, 1), (1, 1)], ids=["e4m3xe4m3", "e5m2xe4m3", "e4m3xe5m2",
                                                                      "e5m2xe5m2"])
def test_fp8_formats(cuda_device, fmts):
    _run(cuda_device, 512, 16, 1024, fmt_a=fmts[0], fmt_b=fmts[1], seed=11)
    _run(cuda_device, 256, 64, 640, fmt_a=fmts[0], fmt_b=fmts[1], seed=12)


@pytest.mark.parametrize("shape", [(256, 16, 512), (128, 32, 1024), (512, 48, 384)], ids=lambda s: "x".join(map(str, s)))
def test_fp8_integer_exact(cuda_device, shape):
    """Small integers are exact in fp8 and in every partial sum: C must equal
    the rounded exact product bit for bit (any metadata or layout slip shows)."""
    M, N, K = shape
    _run(cuda_device, M, N, K, integer=True, seed=5)
    _run(cuda_device, M, N, K, integer=True, fmt_a=1, fmt_b=1, seed=6)


@pytest.mark.parametrize("split", [1, 2, 4, 5, 8])
def test_fp8_split_k(cuda_device, split):
    _run(cuda_device, 1024, 16, 2560, split=split, seed=split)


def test_fp8_epilogue_bf16_out(cuda_device):
    _run(cuda_device, 512, 32, 1024, bf16=True, bias=True, residual=True, alpha=0.25, act=2, seed=21)
    _run(cuda_device, 768, 16, 2048, bias=True, act=3, alpha=0.5, seed=22)
    _run(cuda_device, 256, 40, 512, residual=True, packed=True, act=1, seed=23)


def test_fp8_wide_tile(cuda_device, tuning):
    """The cluster kernel's 256-column tile (a tuning override; wide N
    otherwise takes the CTA pair)."""
    tuning(pair=0, tile_n=256)
    _run(cuda_device, 256, 256, 1024, seed=31)


# CTA-pair kernel (N > 128, K % 256 == 0): 256 x 256 tiles, M and N ragged.
PAIR_SHAPES = [
    (512, 256, 1024),
    (768, 520, 2048),
    (256, 1024, 512),
    (1024, 384, 4096),
    (384, 136, 256),
]


@pytest.mark.parametrize("shape", PAIR_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_fp8_pair_matches_oracle(cuda_device, tuning, shape):
    import spmm24

    tuning(pair=1)  # also the few-tile shapes the picker gives to split-K clusters
    M, N, K = shape
    assert spmm24.select_config_fp8(M, N, K)["cta_pair"] == 1
    _run(cuda_device, M, N, K, seed=M + 3 * N + K)


def test_fp8_pair_integer_exact_and_formats(cuda_device, tuning):
    tuning(pair=1)
    _run(cuda_device, 512, 256, 1024, integer=True, seed=51)
    _run(cuda_device, 256, 512, 512, integer=True, fmt_a=1, fmt_b=0, seed=52)
    _run(cuda_device, 512, 264, 768, fmt_a=0, fmt_b=1, seed=53)
    _run(cuda_device, 256, 256, 1280, fmt_a=1, fmt_b=1, seed=54)


def test_fp8_pair_k_split(cuda_device, tuning):
    """Two pairs per tile, each half of K, partial exchanged on chip."""
    tuning(pair=1, pair_split=2)
    _run(cuda_device, 512, 512, 4096, seed=61)
    _run(cuda_device, 256, 256, 2816, seed=62)  # odd number of 256-K stages
    _run(cuda_device, 512, 256, 2048, bias=True, act=3, alpha=0.5, seed=63)


def test_fp8_pair_epilogue(cuda_device, tuning):
    tuning(pair=1)
    _run(cuda_device, 512, 256, 1024, bf16=True, bias=True, residual=True, alpha=0.25, act=2, seed=71)
    _run(cuda_device, 256, 264, 512, residual=True, packed=True, act=1, seed=72)


def test_fp8_cuda_graph(cuda_device):
    """fp8 launches captured in a CUDA graph give the eager results."""
    import torch

    import spmm24

    M, N, K = 1024, 16, 2048
    vals, meta, b_bits, _, _ = _problem(M, N, K, 0, 0, 41)
    A, E, B = _u8dev(vals, cuda_device), _u8dev(meta, cuda_device), _u8dev(b_bits, cuda_device)
    c1 = torch.empty(M * N, dtype=torch.int16, device=cuda_device)
    c2 = torch.empty_like(c1)
    assert spmm24.launch_fp8(torch.cuda.current_stream(cuda_device), A, B, E, c1, M, N, K, 0,
                             spmm24.STATIC_WEIGHTS) == 0
    torch.cuda.synchronize(cuda_device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        assert spmm24.launch_fp8(torch.cuda.current_stream(cuda_device), A, B, E, c2, M, N, K, 0,
                                 spmm24.STATIC_WEIGHTS) == 0
    g.replay()
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(c1, c2)


# ---------------------------------------------------------- device packer
def _fp8_specials(M, K, fmt, seed):
    rng = np.random.default_rng(seed)
    a = O.f32_to_fp8(rng.standard_normal(M * K).astype(np.float32), fmt)
    codes = np.array([0x00, 0x80, 0x01, 0x81, 0x7E, 0xFE, 0x7F, 0xFF, 0x7C, 0xFC, 0x7D], dtype=np.uint8)
    pick = rng.random(M * K) < 0.15
    a[pick] = rng.choice(codes, int(pick.sum()))
    # magnitude ties inside groups
    a[::53] = a[1::53][: a[::53].size]
    return a


@pytest.mark.parametrize("fmt", [0, 1], ids=["e4m3", "e5m2"])
@pytest.mark.parametrize("shape", [(96, 1280), (256, 4096), (16, 128)], ids=lambda s: "x".join(map(str, s)))
def test_fp8_device_packer_matches_host(cuda_device, fmt, shape):
    """spmm24_pack_a_fp8_device (prune + compress in one pass) equals the host
    prune + compress bit for bit, including signed zeros, NaN / inf codes and
    magnitude ties; without the prune it equals the host compress of a
    pruned matrix."""
    import torch

    import spmm24

    M, K = shape
    a = _fp8_specials(M, K, fmt, 7 + fmt)
    pruned = spmm24.prune_2of4_fp8(a, M, K, fmt)
    v_ref, m_ref = spmm24.compress_a_fp8(pruned, M, K)
    bad = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    v, m = spmm24.pack_a_fp8_device(_u8dev(a, cuda_device), M, K, prune=1 + fmt, bad_blocks=bad)
    torch.cuda.synchronize(cuda_device)
    assert int(bad.item()) == 0
    assert np.array_equal(v.cpu().numpy(), v_ref) and np.array_equal(m.cpu().numpy(), m_ref)
    v2, m2 = spmm24.pack_a_fp8_device(_u8dev(pruned, cuda_device), M, K, prune=0, bad_blocks=bad)
    torch.cuda.synchronize(cuda_device)
    assert int(bad.item()) == 0
    assert np.array_equal(v2.cpu().numpy(), v_ref) and np.array_equal(m2.cpu().numpy(), m_ref)


def test_fp8_device_packer_counts_dense_rows(cuda_device):
    import torch

    import spmm24

    M, K = 64, 512
    a = O.prune_magnitude_2of4_fp8(_fp8_specials(M, K, 0, 3), M, K, 0)
    a = a.reshape(M, K)
    a[5, 40:44] = 0x38        # row 5, block 1: a dense group
    a[33, 300:304] = 0x40     # row 33, block 9
    a[33, 301] = 0x00         # three non-zeros
    bad = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    spmm24.pack_a_fp8_device(_u8dev(a.reshape(-1), cuda_device), M, K, prune=0, bad_blocks=bad)
    torch.cuda.synchronize(cuda_device)
    assert int(bad.item()) == 2


def test_fp8_device_packed_operands_drive_the_spmm(cuda_device):
    """Weights packed on the device give the same C as host-packed ones."""
    import torch

    import spmm24

    M, N, K = 1024, 16, 2048
    rng = np.random.default_rng(17)
    a = O.f32_to_fp8(rng.standard_normal(M * K).astype(np.float32), 0)
    b = _u8dev(O.f32_to_fp8(rng.standard_normal(N * K).astype(np.float32), 0), cuda_device)
    v_h, m_h = spmm24.compress_a_fp8(spmm24.prune_2of4_fp8(a, M, K, 0), M, K)
    v_d, m_d = spmm24.pack_a_fp8_device(_u8dev(a, cuda_device), M, K, prune=1)
    c1 = torch.empty(M * N, dtype=torch.float16, device=cuda_device)
    c2 = torch.empty_like(c1)
    assert spmm24.launch_fp8(None, _u8dev(v_h, cuda_device), b, _u8dev(m_h, cuda_device), c1, M, N, K) == 0
    assert spmm24.launch_fp8(None, v_d, b, m_d, c2, M, N, K) == 0
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(c1, c2)


def _fp8_cases(n, seed):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        M = int(rng.integers(1, 40)) * 16
        K = int(rng.choice([128, 256, 384, 640, 1024, 2048, 4096]))
        N = int(rng.choice([1, 5, 8, 16, 24, 32, 48, 64, 100, 128, 136, 256, 300]))
        split = int(rng.choice([0, 0, 0, 1, 2, 3, 6]))
        flag = lambda: bool(rng.random() < 0.3)  # noqa: E731
        out.append((M, N, K, split, int(rng.integers(0, 2)), int(rng.integers(0, 2)), flag(),
                    int(rng.integers(1, 4)) if flag() else 0, flag(), flag(), flag(),
                    float(rng.choice([1.0, 0.02, -0.5]))))
    return out


@pytest.mark.parametrize("case", _fp8_cases(32, 77), ids=lambda c: "M{}N{}K{}s{}a{}b{}o{}x{}r{}p{}bias{}al{}".format(
    c[0], c[1], c[2], c[3], c[4], c[5], "bf" if c[6] else "h", c[7], int(c[8]), int(c[9]), int(c[10]), c[11]))
def test_fp8_random_case(cuda_device, case):
    """Seeded sweep: shapes (both kernels), K splits, operand formats, output
    type, activation, residual, packed output, bias, alpha (the alpha-only
    fp16 instantiation whenever nothing else is set)."""
    M, N, K, split, fa, fb, bf16, act, res, packed, bias, alpha = case
    _run(cuda_device, M, N, K, fmt_a=fa, fmt_b=fb, split=split, bf16=bf16, act=act, residual=res, packed=packed,
         bias=bias, alpha=alpha, seed=M * 5 + N * 3 + K)


@pytest.mark.parametrize("shape", [(512, 240, 256), (1024, 480, 1024), (592, 500, 768), (2048, 2048, 2048),
                                   (1024, 720, 2560)],
                         ids=lambda s: "x".join(map(str, s)))
def test_fp8_two_m_half_pair(cuda_device, tuning, shape):
    """The fp8 pair kernel with two M halves (512 x 240 tiles, a two-slot
    metadata ring in TMEM; K = 2560 runs ten stages through it): E4M3 and
    E5M2, exact integer inputs, the epilogue, a packed-B output, and calls
    with a residual (which keep the 256 x 256 pair kernel)."""
    tuning(pair2=1)
    M, N, K = shape
    _run(cuda_device, M, N, K, seed=M + N + K)
    _run(cuda_device, M, N, K, integer=True, fmt_a=1, fmt_b=0, seed=M + 2 * N)
    _run(cuda_device, M, N, K, bf16=True, bias=True, act=2, alpha=0.02, fmt_b=1, seed=M + 3 * N)
    _run(cuda_device, M, N, K, residual=True, act=1, seed=M + 4 * N)
    _run(cuda_device, M, N, K, packed=True, bias=True, act=3, fmt_a=1, seed=M + 5 * N)
