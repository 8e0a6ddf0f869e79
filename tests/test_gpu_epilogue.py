"""spmm24_launch_fused (bias, activation, residual, alpha, packed-B output)
and the bf16 variant, on every kernel path, against the oracle's fp32 GEMM
with the epilogue applied in float64 and rounded to C's type."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2       # one output ulp of rounding apart (bf16: 2^-7) stays below this
MEAN_ABS = 1e-3


def _bits_to_f32(bits, bf16):
    bits = np.ascontiguousarray(bits, dtype=np.uint16).reshape(-1)
    if bf16:
        return (bits.astype(np.uint32) << 16).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


def _round(x, bf16):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    return O.f32_to_bf16_bits(x) if bf16 else O.f32_to_f16_bits(x)


def _act(y, act):
    if act == 1:
        return np.maximum(y, 0.0)
    if act == 2:
        return y / (1.0 + np.exp(-y))
    if act == 3:
        return 0.5 * y * (1.0 + np.tanh(0.7978845608028654 * (y + 0.044715 * y ** 3)))
    return y


def _problem(M, N, K, bf16, seed):
    import spmm24

    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    a_bits, b_bits = _round(a, bf16), _round(b, bf16)
    a_bits = spmm24.prune_2of4_bf16(a_bits, M, K) if bf16 else spmm24.prune_2of4(a_bits, M, K)
    vals, meta = spmm24.compress_reordered(a_bits, M, K)
    bp = spmm24.pack_b(b_bits, K, N)
    gemm = O.dense_gemm_bf16_f32 if bf16 else O.dense_gemm_f32
    acc = gemm(a_bits, b_bits, M, N, K).reshape(M, N).astype(np.float64)
    return vals, meta, bp, acc


def _dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).to(device)


def _unpack_c(bits, M, N, packed):
    bits = bits.reshape(-1)
    if not packed:
        return bits.reshape(M, N)
    strips = (N + 7) // 8
    full = bits.reshape(strips, M, 8).transpose(1, 0, 2).reshape(M, strips * 8)
    assert not full[:, N:].any(), "pad columns of a packed C must be zero"
    return full[:, :N]


def _pack_rowmajor(x_bits, M, N):
    strips = (N + 7) // 8
    pad = np.zeros((M, strips * 8), dtype=np.uint16)
    pad[:, :N] = x_bits.reshape(M, N)
    return pad.reshape(M, strips, 8).transpose(1, 0, 2).reshape(-1).copy()


def _run(cuda_device, M, N, K, *, bf16=False, bias=False, residual=False, alpha=1.0, act=0, packed=False,
         split=0, seed=0, in_place=False):
    import torch

    import spmm24

    vals, meta, bp, acc = _problem(M, N, K, bf16, seed)
    rng = np.random.default_rng(seed + 1)
    bias_bits = _round(rng.standard_normal(M), bf16) if bias else None
    res_bits = _round(rng.standard_normal((M, N)), bf16).reshape(M, N) if residual else None
    strips = (N + 7) // 8
    c_elems = strips * 8 * M if packed else M * N
    # every element of C (the pad columns of a packed C too) must be written
    c = torch.full((c_elems,), -1, dtype=torch.int16, device=cuda_device)
    res_dev = None
    if residual:
        res_layout = _pack_rowmajor(res_bits, M, N) if packed else res_bits.reshape(-1)
        res_dev = _dev(res_layout, cuda_device)
        if in_place:
            c.copy_(res_dev)
            res_dev = c
    rc = spmm24.launch_fused(None, _dev(vals, cuda_device), _dev(bp, cuda_device), _dev(meta, cuda_device), c, M, N,
                             K, split, spmm24.BF16 if bf16 else 0,
                             bias=_dev(bias_bits, cuda_device) if bias else None, residual=res_dev, alpha=alpha,
                             activation=act, out_layout=spmm24.OUT_PACKED_B if packed else spmm24.OUT_ROW_MAJOR)
    assert rc == 0, spmm24._lib.spmm24_last_error().decode()
    torch.cuda.synchronize(cuda_device)
    got_bits = _unpack_c(c.cpu().numpy().view(np.uint16), M, N, packed)

    y = alpha * acc
    if bias:
        y = y + _bits_to_f32(bias_bits, bf16).astype(np.float64)[:, None]
    y = _act(y, act)
    if residual:
        y = y + _bits_to_f32(res_bits, bf16).astype(np.float64).reshape(M, N)
    ref = _bits_to_f32(_round(y.astype(np.float32), bf16), bf16).reshape(M, N)
    got = _bits_to_f32(got_bits, bf16).reshape(M, N)
    assert np.isfinite(got).all()
    diff = np.abs(got.astype(np.float64) - ref)
    scale = float(np.abs(ref).max())
    denom = np.maximum(np.abs(ref), 1e-3 * scale + 1e-30)
    assert float((diff / denom).max()) <= MAX_REL, float((diff / denom).max())
    assert float(diff.mean()) <= MEAN_ABS * max(1.0, float(np.abs(ref).mean()))
    return got_bits


# (M, N, K, split): narrow N with K splits of 1, 3 and 8 (cluster kernel with
# the push reduction), mid N (deep ring), wide N (CTA pair), ragged shapes
SHAPES = [(256, 16, 1024, 1), (384, 16, 2048, 3), (512, 32, 4096, 8), (272, 40, 512, 0), (256, 128, 1024, 0),
          (512, 512, 1024, 0), (272, 264, 384, 0), (1024, 512, 6144, 0)]   # the last: pair kernel with a K split


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("bf16", [False, True])
def test_full_epilogue(cuda_device, shape, bf16):
    M, N, K, split = shape
    _run(cuda_device, M, N, K, bf16=bf16, bias=True, residual=True, alpha=0.5, act=2, split=split, seed=M + N)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("bf16", [False, True])
def test_packed_output(cuda_device, shape, bf16):
    M, N, K, split = shape
    _run(cuda_device, M, N, K, bf16=bf16, bias=True, act=1, packed=True, split=split, seed=M * 3 + N)


@pytest.mark.parametrize("act", [0, 1, 2, 3])
@pytest.mark.parametrize("shape", [(256, 16, 1024, 4), (512, 512, 1024, 0)])
def test_each_activation(cuda_device, act, shape):
    M, N, K, split = shape
    _run(cuda_device, M, N, K, act=act, bias=True, split=split, seed=act)


@pytest.mark.parametrize("shape", [(256, 16, 1024, 2), (512, 512, 1024, 0)])
@pytest.mark.parametrize("packed", [False, True])
def test_residual_in_place(cuda_device, shape, packed):
    """residual == C: every element is read before it is overwritten."""
    M, N, K, split = shape
    _run(cuda_device, M, N, K, residual=True, packed=packed, split=split, seed=11, in_place=True)


@pytest.mark.parametrize("shape", [(256, 8, 512), (512, 32, 1024), (1024, 16, 4096), (512, 512, 1024)])
def test_bf16_plain_launch(cuda_device, shape):
    """SPMM24_BF16 through spmm24_launch_ex (no epilogue)."""
    import torch

    import spmm24

    M, N, K = shape
    vals, meta, bp, acc = _problem(M, N, K, True, seed=5)
    c = torch.empty(M * N, dtype=torch.int16, device=cuda_device)
    assert spmm24.launch_ex(None, _dev(vals, cuda_device), _dev(bp, cuda_device), _dev(meta, cuda_device), c, M, N,
                            K, 0, spmm24.BF16) == 0
    torch.cuda.synchronize(cuda_device)
    got = _bits_to_f32(c.cpu().numpy().view(np.uint16), True).reshape(M, N)
    ref = _bits_to_f32(_round(acc.astype(np.float32), True), True).reshape(M, N)
    denom = np.maximum(np.abs(ref), 1e-3 * float(np.abs(ref).max()))
    assert float((np.abs(got - ref) / denom).max()) <= MAX_REL


def test_plain_epilogue_is_the_plain_launch(cuda_device):
    """alpha 1, no bias, no residual, no activation, row-major: bit for bit
    the result of spmm24_launch."""
    import torch

    import spmm24

    M, N, K = 512, 32, 2048
    vals, meta, bp, _ = _problem(M, N, K, False, seed=3)
    A, E, B = _dev(vals, cuda_device), _dev(meta, cuda_device), _dev(bp, cuda_device)
    c1 = torch.empty(M * N, dtype=torch.int16, device=cuda_device)
    c2 = torch.empty(M * N, dtype=torch.int16, device=cuda_device)
    assert spmm24.launch(None, A, B, E, c1, M, N, K, None, 0) == 0
    assert spmm24.launch_fused(None, A, B, E, c2, M, N, K, 0, 0) == 0
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(c1, c2)


@pytest.mark.parametrize("bf16", [False, True])
def test_packed_output_chains_into_the_next_layer(cuda_device, bf16):
    """Layer 1 writes its output in the packed-B layout; layer 2 consumes it
    as B directly.  Layer 2's result equals the one computed from layer 1's
    row-major output packed on the host -- bit for bit."""
    import torch

    import spmm24

    M1, N, K1 = 512, 24, 1024      # layer 1: 512 x 1024, its output is layer 2's K x N input
    M2, K2 = 256, M1
    flags = spmm24.BF16 if bf16 else 0
    v1, e1, b1, _ = _problem(M1, N, K1, bf16, seed=21)
    v2, e2, _, _ = _problem(M2, N, K2, bf16, seed=22)
    dv = lambda a: _dev(a, cuda_device)  # noqa: E731
    strips = (N + 7) // 8
    h_packed = torch.empty(strips * 8 * M1, dtype=torch.int16, device=cuda_device)
    h_row = torch.empty(M1 * N, dtype=torch.int16, device=cuda_device)
    A1, E1, B1 = dv(v1), dv(e1), dv(b1)
    assert spmm24.launch_fused(None, A1, B1, E1, h_packed, M1, N, K1, 0, flags, activation=spmm24.ACT_RELU,
                               out_layout=spmm24.OUT_PACKED_B) == 0
    assert spmm24.launch_fused(None, A1, B1, E1, h_row, M1, N, K1, 0, flags, activation=spmm24.ACT_RELU) == 0
    torch.cuda.synchronize(cuda_device)
    host_packed = spmm24.pack_b(h_row.cpu().numpy().view(np.uint16), K2, N)
    assert np.array_equal(h_packed.cpu().numpy().view(np.uint16), host_packed)
    c_chain = torch.empty(M2 * N, dtype=torch.int16, device=cuda_device)
    c_host = torch.empty(M2 * N, dtype=torch.int16, device=cuda_device)
    A2, E2 = dv(v2), dv(e2)
    assert spmm24.launch_ex(None, A2, h_packed, E2, c_chain, M2, N, K2, 0, flags) == 0
    assert spmm24.launch_ex(None, A2, dv(host_packed), E2, c_host, M2, N, K2, 0, flags) == 0
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(c_chain, c_host)


def test_device_packer_bf16(cuda_device):
    """SPMM24_PRUNE_BF16 in the device packer equals the host bf16 prune +
    compress, and the oracle's restatement of the bf16 prune."""
    import torch

    import spmm24

    M, K = 256, 512
    rng = np.random.default_rng(9)
    a = _round(rng.standard_normal((M, K)), True)
    special = np.array([0x0000, 0x8000, 0x7F80, 0xFF80, 0x7FC0, 0x0001, 0x3F80, 0x3F80], dtype=np.uint16)
    mask = rng.random(a.size) < 0.3
    a[mask] = rng.choice(special, size=int(mask.sum()))
    host_pruned = spmm24.prune_2of4_bf16(a, M, K)
    assert np.array_equal(host_pruned, O.prune_magnitude_2of4_bf16(a, M, K))
    vals, meta, bad = spmm24.pack_a_device(_dev(a, cuda_device), M, K, prune=spmm24.PRUNE_BF16)
    hv, hm = spmm24.compress_reordered(host_pruned, M, K)
    assert bad == 0
    assert np.array_equal(vals.cpu().numpy().view(np.uint16), hv)
    assert np.array_equal(meta.cpu().numpy().view(np.uint16), hm)
    t = _dev(a, cuda_device)
    spmm24.prune_2of4_device(t, M, K, bf16=True)
    torch.cuda.synchronize(cuda_device)
    assert np.array_equal(t.cpu().numpy().view(np.uint16), host_pruned)


@pytest.mark.parametrize("shape", [(1024, 480, 512), (592, 500, 384), (2048, 1024, 1024)], ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("bf16", [False, True])
def test_two_m_half_pair_epilogue(cuda_device, tuning, shape, bf16):
    """The 512 x 240 pair kernel with alpha, bias and an activation, fp16 and
    bf16, row-major or packed-B output (N = 500: a partial last strip whose
    pad columns must be zero); calls with a residual take the 256 x 256 pair
    kernel instead (same results)."""
    import spmm24

    tuning(pair2=1)
    M, N, K = shape
    assert spmm24.select_config(M, N, K)["tile_m"] == 512
    _run(cuda_device, M, N, K, bf16=bf16, bias=True, alpha=0.5, act=2, seed=M + 7 * N)
    _run(cuda_device, M, N, K, bf16=bf16, act=3, seed=M + 5 * N)
    _run(cuda_device, M, N, K, bf16=bf16, residual=True, bias=True, act=1, seed=M + 3 * N)
    _run(cuda_device, M, N, K, bf16=bf16, packed=True, seed=M + N)
    _run(cuda_device, M, N, K, bf16=bf16, packed=True, bias=True, alpha=-0.5, act=1, seed=M + 9 * N)
