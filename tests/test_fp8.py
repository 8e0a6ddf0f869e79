"""The fp8 extension on the CPU: the oracle's OCP E4M3 / E5M2 decode and
quantiser pinned against PyTorch's float8 types on every code, the
product's host packer (prune + compress) bit-exact with the oracle, and the
argument checks of spmm24_launch_fp8 (no GPU work is reached)."""
import ctypes

import numpy as np
import pytest

import oracle as O


@pytest.mark.parametrize("fmt", [0, 1], ids=["e4m3", "e5m2"])
def test_fp8_decode_matches_torch_on_every_code(fmt):
    import torch

    codes = np.arange(256, dtype=np.uint8)
    mine = O.fp8_to_f32(codes, fmt)
    dt = torch.float8_e4m3fn if fmt == 0 else torch.float8_e5m2
    ref = torch.from_numpy(codes.copy()).view(dt).float().numpy()
    same = (mine == ref) | (np.isnan(mine) & np.isnan(ref))
    assert same.all(), np.where(~same)[0]
    assert (np.signbit(mine) == np.signbit(ref))[~np.isnan(ref)].all()


@pytest.mark.parametrize("fmt", [0, 1], ids=["e4m3", "e5m2"])
def test_fp8_quantiser_matches_torch(fmt):
    import torch

    rng = np.random.default_rng(fmt)
    top = 448.0 if fmt == 0 else 57344.0
    x = np.concatenate([rng.standard_normal(100000) * (2.0 if fmt == 0 else 50.0),
                        rng.uniform(-top, top, 20000),
                        [0.0, -0.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10, 2.0 ** -16, 2.0 ** -17, top, -top]])
    x = x.astype(np.float32)
    x = x[np.abs(x) <= top]
    dt = torch.float8_e4m3fn if fmt == 0 else torch.float8_e5m2
    ref = torch.from_numpy(x).to(dt).view(torch.uint8).numpy()
    assert np.array_equal(O.f32_to_fp8(x, fmt), ref)


def _fp8_matrix(M, K, fmt, seed):
    rng = np.random.default_rng(seed)
    a = O.f32_to_fp8(rng.standard_normal(M * K).astype(np.float32), fmt)
    # signed zeros, NaN codes and (E5M2) infinities inside groups
    a[::97] = 0x80
    a[3::101] = 0x7F
    a[5::103] = 0xFF
    if fmt == 1:
        a[7::89] = 0x7C
        a[9::83] = 0xFC
    return a


@pytest.mark.parametrize("fmt", [0, 1], ids=["e4m3", "e5m2"])
def test_host_prune_and_compress_match_oracle(fmt):
    import spmm24

    M, K = 96, 1024
    a = _fp8_matrix(M, K, fmt, 3)
    pruned = spmm24.prune_2of4_fp8(a, M, K, fmt)
    assert np.array_equal(pruned, O.prune_magnitude_2of4_fp8(a, M, K, fmt))
    vals, meta = spmm24.compress_a_fp8(pruned, M, K)
    n, v_ref, m_ref = O.compress_a_fp8(pruned, M, K)
    assert n == M * K // 2
    assert np.array_equal(vals, v_ref) and np.array_equal(meta, m_ref)


def test_compress_round_trip_and_layout():
    """Values and metadata decode back to the pruned matrix (a dense GEMM
    against the identity gives it back), and the first row's first group
    lands where the format says."""
    import spmm24

    M, K = 32, 256
    a = O.prune_magnitude_2of4_fp8(_fp8_matrix(M, K, 0, 9), M, K, 0)
    a[a == 0x7F] = 0x38  # no NaN for the identity product
    a[a == 0xFF] = 0xB8
    a = O.prune_magnitude_2of4_fp8(a, M, K, 0)
    vals, meta = spmm24.compress_a_fp8(a, M, K)
    eye = np.zeros((K, K), dtype=np.float32)
    eye[np.arange(K), np.arange(K)] = 1.0
    eye_bits = O.f32_to_fp8(eye.reshape(-1), 0)
    back = O.spmm_fp8_f32(vals, meta, eye_bits, M, K, K).reshape(M, K)
    dense = O.fp8_to_f32(a, 0).reshape(M, K)
    assert np.array_equal(back, dense)
    g0 = a[:4]
    kept = [i for i in range(4) if (g0[i] & 0x7F) != 0] if sum((g0 & 0x7F) != 0) == 2 else None
    if kept:
        assert list(vals[:2]) == [g0[kept[0]], g0[kept[1]]]
        assert meta[0] & 0xF == kept[0] | (kept[1] << 2)


def test_compress_rejects_dense_group():
    import spmm24

    a = np.full(16 * 128, 0x38, dtype=np.uint8)
    with pytest.raises(ValueError):
        spmm24.compress_a_fp8(a, 16, 128)
    assert O.compress_a_fp8(a, 16, 128)[0] == -2
    with pytest.raises(ValueError):
        spmm24.compress_a_fp8(np.zeros(16 * 64, np.uint8), 16, 64)  # K % 128


def _launch(**kw):
    import spmm24

    args = dict(values=0x1000, b=0x2000, meta=0x3000, c=0x4000, M=128, N=16, K=256, split=0, flags=0, epi=None)
    args.update(kw)
    return spmm24._lib.spmm24_launch_fp8(None, args["values"], args["b"], args["meta"], args["c"], args["M"], args["N"],
                                         args["K"], args["split"], args["flags"], args["epi"])


def test_launch_fp8_argument_checks():
    import spmm24

    INVALID = spmm24.CUDA_ERROR_INVALID_VALUE
    assert _launch(values=None) == INVALID
    assert _launch(K=192) == INVALID                     # K % 128
    assert _launch(M=120) == INVALID                     # M % 16
    assert _launch(N=0) == INVALID
    assert _launch(split=-1) == INVALID
    assert _launch(b=0x2008) == INVALID                  # 16-byte alignment
    assert _launch(c=0x4001) == INVALID
    assert _launch(flags=32) == INVALID                  # unknown flag
    assert b"flag" in spmm24._lib.spmm24_last_error()
    epi = spmm24.Epilogue(None, None, float("nan"), 0, 0)
    assert _launch(epi=ctypes.addressof(epi)) == INVALID
    epi = spmm24.Epilogue(None, None, 1.0, 9, 0)
    assert _launch(epi=ctypes.addressof(epi)) == INVALID


def test_fp8_device_packer_argument_checks():
    import spmm24

    INVALID = spmm24.CUDA_ERROR_INVALID_VALUE
    f = spmm24._lib.spmm24_pack_a_fp8_device
    assert f(None, None, 64, 256, 1, 0x2000, 0x3000, None) == INVALID
    assert f(None, 0x1000, 64, 192, 1, 0x2000, 0x3000, None) == INVALID   # K % 128
    assert f(None, 0x1000, 60, 256, 1, 0x2000, 0x3000, None) == INVALID   # M % 16
    assert f(None, 0x1008, 64, 256, 1, 0x2000, 0x3000, None) == INVALID   # alignment
    assert f(None, 0x1000, 64, 256, 1, 0x2000, 0x3004, None) == INVALID
    assert f(None, 0x1000, 64, 256, 3, 0x2000, 0x3000, None) == INVALID   # prune mode


def test_fp8_symbols_exported():
    import spmm24

    for name in ("spmm24_launch_fp8", "spmm24_compress_a_fp8", "spmm24_prune_2of4_fp8", "spmm24_pack_a_fp8_device"):
        assert hasattr(spmm24._lib, name)


def test_select_config_fp8():
    """The fp8 plan: 256-K stages, automatic splits capped at 5, the
    two-M-half pair tile (512 x 240) when its waves cost less."""
    import spmm24

    c = spmm24.select_config_fp8(4096, 16, 4096)
    assert (c["stage_k"], c["tile_n"], c["split_k"], c["grid_ctas"]) == (256, 16, 5, 160)
    assert spmm24.select_config_fp8(11008, 16, 4096)["split_k"] == 3
    c = spmm24.select_config_fp8(11008, 4096, 4096)
    assert (c["cta_pair"], c["tile_m"], c["tile_n"], c["grid_ctas"]) == (1, 512, 240, 2 * 22 * 18)
    c = spmm24.select_config_fp8(4096, 4096, 4096)
    assert (c["cta_pair"], c["tile_m"], c["tile_n"]) == (1, 512, 240)
    assert spmm24.select_config_fp8(4096, 512, 4096)["tile_m"] == 256
    assert spmm24.select_config_fp8(512, 16, 4096, 3)["split_k"] == 3
    with pytest.raises(ValueError):
        spmm24.select_config_fp8(512, 16, 192)
