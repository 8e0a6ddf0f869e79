"""ctypes front end of the CPU oracle (oracle.c) and of the reference's own
packer / kernel built into oracle/_ref/.

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
and by bench.py's CPU-baseline / reference arm.  The product package never
imports this module.

Reference anchors (SpeakOutLoudly/CUDA-Repo):
  toolCompressMatrixA  test/utils.h:91-150   -> compress_a
  toolReorderMetadata  test/utils.h:155-185  -> reorder_metadata
  toolPackMatrixB      test/utils.h:188-229  -> pack_b
  init_host_matrices_pruned test/utils.h:38-66 -> ref_init_pruned
  SpMM_N2M4_Kernel + SplitK_Reduction math (src/SpMM_Kernel.cuh:301-492,
  src/reduce_Kernel.cuh:27-53) -> dense_gemm_f32 / spmm_from_abi_f32
  The fp8 extension (no reference counterpart): the same prune, compress rule
  (test/utils.h:124-146) and GEMM on OCP E4M3 / E5M2 bytes -> *_fp8
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_REF_PACKER = os.path.join(_HERE, "_ref", "libref_packer.so")
_REF_SPMM = os.path.join(_HERE, "_ref", "libref_spmm.so")

_u16p = ctypes.POINTER(ctypes.c_uint16)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)


def reference_dir() -> str:
    """The reference checkout: $SPMM24_REFERENCE_DIR, else a directory named
    `reference` beside this repository (it need not exist)."""
    return os.environ.get("SPMM24_REFERENCE_DIR") or os.path.join(os.path.dirname(os.path.dirname(_HERE)), "reference")


def build() -> None:
    """Compile liboracle.so (and oracle/_ref when the reference tree exists)."""
    subprocess.check_call(["make", "-s", "-C", _HERE])
    ref = reference_dir()
    if os.path.isdir(ref):
        subprocess.check_call(["make", "-s", "-C", _HERE, "ref", f"REFERENCE={ref}"])


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_fill_uniform_f16.argtypes = [_u16p, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_double, ctypes.c_double]
        L.orc_fill_normal_f16.argtypes = [_u16p, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_double, ctypes.c_double]
        L.orc_prune_magnitude_2of4.argtypes = [_u16p, ctypes.c_int, ctypes.c_int]
        L.orc_random_mask_2of4.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, ctypes.c_uint64]
        L.orc_ref_init_pruned.argtypes = [_u16p, ctypes.c_int, ctypes.c_int]
        L.orc_compress_a.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, _u16p, _u16p]
        L.orc_compress_a.restype = ctypes.c_int
        L.orc_reorder_metadata.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, _u16p]
        L.orc_reorder_metadata.restype = ctypes.c_int
        L.orc_pack_b.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, _u16p]
        L.orc_pack_b.restype = ctypes.c_int
        L.orc_dense_gemm_f32.argtypes = [_u16p, _u16p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_spmm_from_abi_f32.argtypes = [_u16p, _u16p, _u16p, _f32p] + [ctypes.c_int] * 4
        L.orc_spmm_from_abi_f32.restype = ctypes.c_int
        L.orc_f32_to_f16.argtypes = [_f32p, _u16p, ctypes.c_size_t]
        L.orc_f32_to_bf16.argtypes = [_f32p, _u16p, ctypes.c_size_t]
        L.orc_prune_magnitude_2of4_bf16.argtypes = [_u16p, ctypes.c_int, ctypes.c_int]
        L.orc_dense_gemm_bf16_f32.argtypes = [_u16p, _u16p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int]
        L.orc_fp8_to_f32_array.argtypes = [_u8p, _f32p, ctypes.c_size_t, ctypes.c_int]
        L.orc_f32_to_fp8_array.argtypes = [_f32p, _u8p, ctypes.c_size_t, ctypes.c_int]
        L.orc_prune_magnitude_2of4_fp8.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_compress_a_fp8.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, _u8p, _u8p]
        L.orc_compress_a_fp8.restype = ctypes.c_int
        L.orc_spmm_fp8_f32.argtypes = [_u8p, _u8p, _u8p, _f32p] + [ctypes.c_int] * 6
        L.orc_spmm_fp8_f32.restype = ctypes.c_int
        L.orc_fnv1a64.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        L.orc_fnv1a64.restype = ctypes.c_uint64
        L.orc_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p16(a: np.ndarray):
    assert a.dtype == np.uint16 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_u16p)


def _pf(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_f32p)


# ------------------------------------------------------------ generators
def uniform_f16(n: int, seed: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib().orc_fill_uniform_f16(_p16(out), n, seed, lo, hi)
    return out


def normal_f16(n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib().orc_fill_normal_f16(_p16(out), n, seed, mean, std)
    return out


def prune_magnitude_2of4(a: np.ndarray, M: int, K: int) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16).copy()
    lib().orc_prune_magnitude_2of4(_p16(a), M, K)
    return a


def random_mask_2of4(a: np.ndarray, M: int, K: int, seed: int) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16).copy()
    lib().orc_random_mask_2of4(_p16(a), M, K, seed)
    return a


def ref_init_pruned(M: int, K: int) -> np.ndarray:
    a = np.empty(M * K, dtype=np.uint16)
    lib().orc_ref_init_pruned(_p16(a), M, K)
    return a


# ---------------------------------------------------------------- packer
def compress_a(dense: np.ndarray, M: int, K: int):
    dense = np.ascontiguousarray(dense, dtype=np.uint16)
    vals = np.zeros(M * K // 2, dtype=np.uint16)
    meta = np.zeros(M * K // 16, dtype=np.uint16)
    n = lib().orc_compress_a(_p16(dense), M, K, _p16(vals), _p16(meta))
    return n, vals, meta


def reorder_metadata(meta: np.ndarray, M: int, K: int) -> np.ndarray:
    meta = np.ascontiguousarray(meta, dtype=np.uint16)
    out = np.zeros_like(meta)
    rc = lib().orc_reorder_metadata(_p16(meta), M, K, _p16(out))
    if rc != 0:
        raise ValueError("reorder_metadata: unsupported shape")
    return out


def pack_b(b_rowmajor: np.ndarray, K: int, N: int) -> np.ndarray:
    b = np.ascontiguousarray(b_rowmajor, dtype=np.uint16)
    out = np.zeros(K * N, dtype=np.uint16)
    rc = lib().orc_pack_b(_p16(b), K, N, _p16(out))
    if rc != 0:
        raise ValueError("pack_b: unsupported shape")
    return out


# ----------------------------------------------------------------- GEMMs
def dense_gemm_f32(a: np.ndarray, b_rowmajor: np.ndarray, M: int, N: int, K: int, threads: int = 0) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    b = np.ascontiguousarray(b_rowmajor, dtype=np.uint16)
    c = np.empty(M * N, dtype=np.float32)
    lib().orc_dense_gemm_f32(_p16(a), _p16(b), _pf(c), M, N, K, threads)
    return c


def spmm_from_abi_f32(vals, meta_reordered, b_packed, M: int, N: int, K: int, threads: int = 0) -> np.ndarray:
    c = np.empty(M * N, dtype=np.float32)
    rc = lib().orc_spmm_from_abi_f32(_p16(np.ascontiguousarray(vals)), _p16(np.ascontiguousarray(meta_reordered)),
                                     _p16(np.ascontiguousarray(b_packed)), _pf(c), M, N, K, threads)
    if rc != 0:
        raise ValueError(f"spmm_from_abi_f32 failed ({rc})")
    return c


def prune_magnitude_2of4_bf16(a: np.ndarray, M: int, K: int) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16).copy()
    lib().orc_prune_magnitude_2of4_bf16(_p16(a), M, K)
    return a


def dense_gemm_bf16_f32(a: np.ndarray, b_rowmajor: np.ndarray, M: int, N: int, K: int, threads: int = 0) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    b = np.ascontiguousarray(b_rowmajor, dtype=np.uint16)
    c = np.empty(M * N, dtype=np.float32)
    lib().orc_dense_gemm_bf16_f32(_p16(a), _p16(b), _pf(c), M, N, K, threads)
    return c


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size, dtype=np.uint16)
    lib().orc_f32_to_bf16(_pf(x), _p16(out), x.size)
    return out


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size, dtype=np.uint16)
    lib().orc_f32_to_f16(_pf(x), _p16(out), x.size)
    return out


# ------------------------------------------------------------------ fp8
# fmt 0 = OCP E4M3 (no infinities), 1 = OCP E5M2.
def _p8(a: np.ndarray):
    assert a.dtype == np.uint8 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_u8p)


def fp8_to_f32(x: np.ndarray, fmt: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint8)
    out = np.empty(x.size, dtype=np.float32)
    lib().orc_fp8_to_f32_array(_p8(x), _pf(out), x.size, fmt)
    return out


def f32_to_fp8(x: np.ndarray, fmt: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size, dtype=np.uint8)
    lib().orc_f32_to_fp8_array(_pf(x), _p8(out), x.size, fmt)
    return out


def prune_magnitude_2of4_fp8(a: np.ndarray, M: int, K: int, fmt: int) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint8).copy()
    lib().orc_prune_magnitude_2of4_fp8(_p8(a), M, K, fmt)
    return a


def compress_a_fp8(dense: np.ndarray, M: int, K: int):
    dense = np.ascontiguousarray(dense, dtype=np.uint8)
    vals = np.zeros(M * K // 2, dtype=np.uint8)
    meta = np.zeros(M * K // 8, dtype=np.uint8)
    n = lib().orc_compress_a_fp8(_p8(dense), M, K, _p8(vals), _p8(meta))
    return n, vals, meta


def spmm_fp8_f32(vals, meta, b_nk, M: int, N: int, K: int, fmt_a: int = 0, fmt_b: int = 0,
                 threads: int = 0) -> np.ndarray:
    c = np.empty(M * N, dtype=np.float32)
    rc = lib().orc_spmm_fp8_f32(_p8(np.ascontiguousarray(vals, dtype=np.uint8)),
                                _p8(np.ascontiguousarray(meta, dtype=np.uint8)),
                                _p8(np.ascontiguousarray(b_nk, dtype=np.uint8)), _pf(c), M, N, K, fmt_a, fmt_b, threads)
    if rc != 0:
        raise ValueError(f"spmm_fp8_f32 failed ({rc})")
    return c


def fnv1a64(buf: np.ndarray) -> int:
    buf = np.ascontiguousarray(buf)
    return int(lib().orc_fnv1a64(buf.ctypes.data, buf.nbytes))


def max_threads() -> int:
    return int(lib().orc_max_threads())


# ------------------------------------------------ the reference's own code
def ref_packer_available() -> bool:
    return os.path.exists(_REF_PACKER)


_ref_packer = None


def ref_packer() -> ctypes.CDLL:
    global _ref_packer
    if _ref_packer is None:
        L = ctypes.CDLL(_REF_PACKER)
        L.ref_compress_a.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, _u16p, _u16p]
        L.ref_compress_a.restype = ctypes.c_int
        L.ref_reorder_metadata.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, _u16p]
        L.ref_pack_b.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, _u16p]
        L.ref_init_pruned.argtypes = [_u16p, ctypes.c_int, ctypes.c_int]
        _ref_packer = L
    return _ref_packer


def ref_compress_a(dense: np.ndarray, M: int, K: int):
    dense = np.ascontiguousarray(dense, dtype=np.uint16)
    vals = np.zeros(M * K // 2, dtype=np.uint16)
    meta = np.zeros(M * K // 16, dtype=np.uint16)
    n = ref_packer().ref_compress_a(_p16(dense), M, K, _p16(vals), _p16(meta))
    return n, vals, meta


def ref_reorder_metadata(meta: np.ndarray, M: int, K: int) -> np.ndarray:
    meta = np.ascontiguousarray(meta, dtype=np.uint16)
    out = np.zeros_like(meta)
    ref_packer().ref_reorder_metadata(_p16(meta), M, K, _p16(out))
    return out


def ref_pack_b(b: np.ndarray, K: int, N: int) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    out = np.zeros(K * N, dtype=np.uint16)
    ref_packer().ref_pack_b(_p16(b), K, N, _p16(out))
    return out


def ref_init_pruned_ref(M: int, K: int) -> np.ndarray:
    a = np.empty(M * K, dtype=np.uint16)
    ref_packer().ref_init_pruned(_p16(a), M, K)
    return a


def ref_spmm_available() -> bool:
    return os.path.exists(_REF_SPMM)


_ref_spmm = None


def ref_spmm() -> ctypes.CDLL:
    global _ref_spmm
    if _ref_spmm is None:
        L = ctypes.CDLL(_REF_SPMM)
        L.ref_spmm_supported.argtypes = [ctypes.c_int] * 4
        L.ref_spmm_supported.restype = ctypes.c_int
        L.ref_spmm_launch.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 3 + [ctypes.c_void_p, ctypes.c_int]
        L.ref_spmm_launch.restype = ctypes.c_int
        _ref_spmm = L
    return _ref_spmm
