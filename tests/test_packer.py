"""The product's host packer (libspmm24: spmm24_compress_a & co. and the
reference-named C++ drop-ins) against the oracle and the golden fixtures.
Host code only -- no GPU needed."""
import ctypes
import json
import os

import numpy as np
import pytest

import oracle as O
import spmm24

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "packer_golden.json")) as f:
        meta = json.load(f)
    return meta, dict(np.load(os.path.join(GOLDEN, "packer_golden.npz")))


@pytest.mark.parametrize("case", ["small", "edge"])
def test_packer_matches_golden(golden, case):
    meta, arr = golden
    c = meta["cases"][case]
    vals, raw = spmm24.compress_a(arr[f"{case}_a"], c["M"], c["K"])
    assert np.array_equal(vals, arr[f"{case}_vals"])
    assert np.array_equal(raw, arr[f"{case}_meta_raw"])
    re = spmm24.reorder_metadata(raw, c["M"], c["K"])
    assert np.array_equal(re, arr[f"{case}_meta_reordered"])
    v2, re2 = spmm24.compress_reordered(arr[f"{case}_a"], c["M"], c["K"])
    assert np.array_equal(v2, vals) and np.array_equal(re2, re)
    if case == "small":
        assert np.array_equal(spmm24.pack_b(arr["small_b"], c["K"], c["N"]), arr["small_b_packed"])


def test_packer_matches_golden_hashes(golden):
    meta, _ = golden
    for name in ("config1", "decode_slice"):
        c = meta["cases"][name]
        M, K, N = c["M"], c["K"], c["N"]
        a = O.prune_magnitude_2of4(O.normal_f16(M * K, c["seed"], 0.0, c["a_std"]), M, K)
        vals, re = spmm24.compress_reordered(a, M, K)
        assert hex(O.fnv1a64(vals)) == c["fnv_vals"]
        assert hex(O.fnv1a64(re)) == c["fnv_meta_reordered"]
        b = O.uniform_f16(K * N, c["seed"] + 1, -1.0, 1.0)
        assert hex(O.fnv1a64(spmm24.pack_b(b, K, N))) == c["fnv_b_packed"]


@pytest.mark.parametrize("shape", [(16, 64), (96, 320), (1024, 1024)])
def test_packer_matches_oracle(shape):
    M, K = shape
    a = O.prune_magnitude_2of4(O.normal_f16(M * K, 5 + M, 0.0, 1.0), M, K)
    vals, raw = spmm24.compress_a(a, M, K)
    n, ov, oraw = O.compress_a(a, M, K)
    assert np.array_equal(vals, ov) and np.array_equal(raw, oraw)
    assert np.array_equal(spmm24.reorder_metadata(raw, M, K), O.reorder_metadata(oraw, M, K))


def test_weights_sharing_b_stack_along_m():
    """Values and (reordered) metadata are band-major, so layers that share
    their input B (Q/K/V, gate/up) run as one call on M1 + M2 rows by
    concatenating their packed arrays: packing the stacked dense matrix gives
    the same bytes.  fp16 and fp8."""
    K, M1, M2 = 256, 48, 80
    a1 = O.prune_magnitude_2of4(O.normal_f16(M1 * K, 21, 0.0, 1.0), M1, K)
    a2 = O.prune_magnitude_2of4(O.normal_f16(M2 * K, 22, 0.0, 1.0), M2, K)
    v1, e1 = spmm24.compress_reordered(a1, M1, K)
    v2, e2 = spmm24.compress_reordered(a2, M2, K)
    v, e = spmm24.compress_reordered(np.concatenate([a1, a2]), M1 + M2, K)
    assert np.array_equal(v, np.concatenate([v1, v2])) and np.array_equal(e, np.concatenate([e1, e2]))
    rng = np.random.default_rng(23)
    f1 = spmm24.prune_2of4_fp8(O.f32_to_fp8(rng.standard_normal(M1 * K).astype(np.float32), 0), M1, K, 0)
    f2 = spmm24.prune_2of4_fp8(O.f32_to_fp8(rng.standard_normal(M2 * K).astype(np.float32), 0), M2, K, 0)
    (w1, m1), (w2, m2) = spmm24.compress_a_fp8(f1, M1, K), spmm24.compress_a_fp8(f2, M2, K)
    w, m = spmm24.compress_a_fp8(np.concatenate([f1, f2]), M1 + M2, K)
    assert np.array_equal(w, np.concatenate([w1, w2])) and np.array_equal(m, np.concatenate([m1, m2]))


def test_prune_matches_oracle():
    M, K = 64, 256
    a = O.normal_f16(M * K, 77, 0.0, 1.0)
    a[::7] = 0  # include ties among zeros
    assert np.array_equal(spmm24.prune_2of4(a, M, K), O.prune_magnitude_2of4(a, M, K))


def test_pack_b_pads_ragged_n():
    K, N = 128, 13
    b = O.uniform_f16(K * N, 3, -1.0, 1.0)
    p = spmm24.pack_b(b, K, N).reshape(2, K, 8)
    bm = b.reshape(K, N)
    assert np.array_equal(p[0], bm[:, :8])
    assert np.array_equal(p[1][:, :5], bm[:, 8:])
    assert np.all(p[1][:, 5:] == 0)


def test_packer_rejects_bad_input():
    with pytest.raises(ValueError):
        spmm24.compress_a(np.full(256, 0x3C00, np.uint16), 16, 16)  # no zeros
    with pytest.raises(ValueError):
        spmm24.reorder_metadata(np.zeros(32, np.uint16), 16, 32)  # K % 64
    with pytest.raises(ValueError):
        spmm24.pack_b(np.zeros(32 * 8, np.uint16), 32, 8)


def test_cpp_dropins_with_reference_names():
    """toolCompressMatrixA / toolReorderMetadata / toolPackMatrixB exported
    under the reference's mangled names, malloc'ed outputs."""
    L = ctypes.CDLL(spmm24.library_path())
    libc = ctypes.CDLL(None)
    libc.free.argtypes = [ctypes.c_void_p]
    comp = getattr(L, "_Z19toolCompressMatrixAP6__halfiiiiPS0_PPt")
    reord = getattr(L, "_Z19toolReorderMetadataPtiiiiPS_")
    packb = getattr(L, "_Z15toolPackMatrixBP6__halfiiiiPS0_")
    M, K, N = 32, 128, 16
    a = O.prune_magnitude_2of4(O.normal_f16(M * K, 1, 0.0, 1.0), M, K)
    pv, pm = ctypes.c_void_p(), ctypes.c_void_p()
    comp.restype = ctypes.c_int
    n = comp(a.ctypes.data_as(ctypes.c_void_p), M, K, 16, 16, ctypes.byref(pv), ctypes.byref(pm))
    assert n == M * K // 2
    vals = np.ctypeslib.as_array(ctypes.cast(pv, ctypes.POINTER(ctypes.c_uint16)), (M * K // 2,)).copy()
    raw = np.ctypeslib.as_array(ctypes.cast(pm, ctypes.POINTER(ctypes.c_uint16)), (M * K // 16,)).copy()
    on, ov, oraw = O.compress_a(a, M, K)
    assert np.array_equal(vals, ov) and np.array_equal(raw, oraw)
    pr = ctypes.c_void_p()
    reord(pm, M, K, 16, 16, ctypes.byref(pr))
    re = np.ctypeslib.as_array(ctypes.cast(pr, ctypes.POINTER(ctypes.c_uint16)), (M * K // 16,)).copy()
    assert np.array_equal(re, O.reorder_metadata(oraw, M, K))
    b = O.uniform_f16(K * N, 2, -1.0, 1.0)
    pb = ctypes.c_void_p()
    packb(b.ctypes.data_as(ctypes.c_void_p), K, N, 64, 8, ctypes.byref(pb))
    bp = np.ctypeslib.as_array(ctypes.cast(pb, ctypes.POINTER(ctypes.c_uint16)), (K * N,)).copy()
    assert np.array_equal(bp, O.pack_b(b, K, N))
    for p in (pv, pm, pr, pb):
        libc.free(p)
    # unsupported block sizes are refused instead of silently mis-packing
    assert comp(a.ctypes.data_as(ctypes.c_void_p), M, K, 16, 32, ctypes.byref(pv), ctypes.byref(pm)) == -1
