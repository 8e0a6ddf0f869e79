"""The CPU oracle pinned against the reference: golden fixtures made by the
reference's own packer, the reference build itself (oracle/_ref, when
present), and known-answer GEMMs."""
import json
import os

import numpy as np
import pytest

import oracle as O
from problems import make_problem

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "packer_golden.json")) as f:
        meta = json.load(f)
    arrays = dict(np.load(os.path.join(GOLDEN, "packer_golden.npz")))
    return meta, arrays


def test_half_to_float_all_bit_patterns():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.empty(65536, dtype=np.float32)
    O.lib().orc_f16_to_f32(bits.ctypes.data_as(O._u16p), got.ctypes.data_as(O._f32p), 65536)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_float_to_half_round_to_nearest_even():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 5, 200000),
        np.array([65504, 65519.99, 65520, 1e-8, 5.96e-8, 2.98e-8, 2.99e-8, -0.0, 0.0, np.inf, -np.inf], np.float32),
        # exact ties between adjacent halves
        (np.arange(1024, 2048, dtype=np.float32) + 0.5) / 1024,
    ]).astype(np.float32)
    want = x.astype(np.float16).view(np.uint16)
    got = O.f32_to_f16_bits(x)
    assert np.array_equal(got, want)


def test_generators_are_deterministic_and_shaped():
    a = O.normal_f16(100000, 5, 0.0, 1.0)
    assert np.array_equal(a, O.normal_f16(100000, 5, 0.0, 1.0))
    f = a.view(np.float16).astype(np.float64)
    assert abs(f.mean()) < 0.02 and abs(f.std() - 1.0) < 0.02
    u = O.uniform_f16(100000, 6, -1.0, 1.0).view(np.float16).astype(np.float64)
    assert u.min() >= -1.0 and u.max() <= 1.0 and abs(u.mean()) < 0.02


def test_magnitude_prune_keeps_two_largest():
    M, K = 8, 64
    a = O.normal_f16(M * K, 11, 0.0, 1.0)
    p = O.prune_magnitude_2of4(a, M, K).reshape(-1, 4)
    orig = np.abs(a.view(np.float16).astype(np.float32)).reshape(-1, 4)
    for g in range(p.shape[0]):
        kept = np.nonzero(p[g])[0]
        assert len(kept) == 2
        order = sorted(range(4), key=lambda i: (-orig[g, i], i))
        assert set(kept) == set(order[:2])


def test_random_mask_is_2of4():
    a = O.uniform_f16(64 * 128, 3, 0.5, 1.0)  # strictly positive: no accidental zeros
    p = O.random_mask_2of4(a, 64, 128, 9).reshape(-1, 4)
    assert np.all((p != 0).sum(axis=1) == 2)
    patterns = {tuple(np.nonzero(r)[0]) for r in p}
    assert len(patterns) == 6


def test_reference_generator_restatement_matches_golden(golden):
    meta, _ = golden
    case = meta["cases"]["ref_known_answer_256"]
    a = O.ref_init_pruned(case["M"], case["K"])
    assert hex(O.fnv1a64(a)) == case["fnv_a"]
    n, vals, raw = O.compress_a(a, case["M"], case["K"])
    re = O.reorder_metadata(raw, case["M"], case["K"])
    assert n == case["count"]
    assert hex(O.fnv1a64(vals)) == case["fnv_vals"]
    assert hex(O.fnv1a64(raw)) == case["fnv_meta_raw"]
    assert hex(O.fnv1a64(re)) == case["fnv_meta_reordered"]
    assert [int(x) for x in raw[:8]] == case["meta_raw_first8"]
    assert [int(x) for x in re[:8]] == case["meta_reordered_first8"]
    # first raw and reordered words as measured on the reference packer
    assert raw[0] == 0x98ED and [int(x) for x in re[:4]] == [0x98ED, 0x99D4, 0xC489, 0x4CE4]


@pytest.mark.parametrize("case", ["small", "edge"])
def test_oracle_packer_matches_golden_arrays(golden, case):
    meta, arr = golden
    c = meta["cases"][case]
    a = arr[f"{case}_a"]
    n, vals, raw = O.compress_a(a, c["M"], c["K"])
    assert n == c["count"]
    assert np.array_equal(vals, arr[f"{case}_vals"])
    assert np.array_equal(raw, arr[f"{case}_meta_raw"])
    assert np.array_equal(O.reorder_metadata(raw, c["M"], c["K"]), arr[f"{case}_meta_reordered"])
    if case == "small":
        assert np.array_equal(O.pack_b(arr["small_b"], c["K"], c["N"]), arr["small_b_packed"])


@pytest.mark.parametrize("case", ["config1", "decode_slice"])
def test_oracle_packer_matches_golden_hashes(golden, case):
    meta, _ = golden
    c = meta["cases"][case]
    M, K, N = c["M"], c["K"], c["N"]
    a = O.prune_magnitude_2of4(O.normal_f16(M * K, c["seed"], 0.0, c["a_std"]), M, K)
    b = O.uniform_f16(K * N, c["seed"] + 1, -1.0, 1.0)
    assert hex(O.fnv1a64(a)) == c["fnv_a"] and hex(O.fnv1a64(b)) == c["fnv_b"]
    n, vals, raw = O.compress_a(a, M, K)
    assert n == c["count"]
    assert hex(O.fnv1a64(vals)) == c["fnv_vals"]
    assert hex(O.fnv1a64(raw)) == c["fnv_meta_raw"]
    assert hex(O.fnv1a64(O.reorder_metadata(raw, M, K))) == c["fnv_meta_reordered"]
    assert hex(O.fnv1a64(O.pack_b(b, K, N))) == c["fnv_b_packed"]


def test_compress_rejects_non_2of4_groups():
    a = np.full(16 * 16, 0x3C00, dtype=np.uint16)  # all ones: no zeros
    n, _, _ = O.compress_a(a, 16, 16)
    assert n == -2
    n, _, _ = O.compress_a(np.zeros(8 * 16, np.uint16), 8, 16)
    assert n == -1


@pytest.mark.parametrize("shape", [(32, 16, 128), (48, 24, 192), (256, 128, 256)])
def test_abi_decoder_agrees_bitwise_with_dense_gemm(shape):
    M, N, K = shape
    p = make_problem(M, N, K, seed=21)
    dense = O.dense_gemm_f32(p.a_dense, p.b_rowmajor, M, N, K)
    n8 = (N + 7) // 8 * 8
    from_abi = O.spmm_from_abi_f32(p.vals, p.meta, p.b_packed, M, n8, K).reshape(M, n8)[:, :N].reshape(-1)
    assert np.array_equal(dense.view(np.uint32), np.ascontiguousarray(from_abi).view(np.uint32))


def test_known_answer_reference_generator():
    """The reference harness's inputs (ones, random 2:4 mask) give C == K/2."""
    M, K, N = 256, 256, 128
    a = O.ref_init_pruned(M, K)
    b = np.full(K * N, 0x3C00, dtype=np.uint16)
    c = O.dense_gemm_f32(a, b, M, N, K)
    assert np.all(c == K / 2)


@pytest.mark.skipif(not O.ref_packer_available(), reason="reference packer not built (oracle/_ref)")
@pytest.mark.parametrize("shape", [(16, 64), (64, 256), (128, 1024), (48, 448)])
def test_oracle_packer_equals_reference_build(shape):
    M, K = shape
    a = O.prune_magnitude_2of4(O.normal_f16(M * K, M + K, 0.0, 1.0), M, K)
    n1, v1, r1 = O.compress_a(a, M, K)
    n2, v2, r2 = O.ref_compress_a(a, M, K)
    assert n1 == n2 and np.array_equal(v1, v2) and np.array_equal(r1, r2)
    assert np.array_equal(O.reorder_metadata(r1, M, K), O.ref_reorder_metadata(r2, M, K))
    N = 24
    b = O.uniform_f16(K * N, 4, -1.0, 1.0)
    assert np.array_equal(O.pack_b(b, K, N), O.ref_pack_b(b, K, N))


@pytest.mark.skipif(not O.ref_packer_available(), reason="reference packer not built (oracle/_ref)")
def test_reference_generator_restatement_equals_reference_build():
    assert np.array_equal(O.ref_init_pruned(128, 512), O.ref_init_pruned_ref(128, 512))
