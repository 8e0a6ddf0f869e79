"""Python host binding of libspmm24 (the sm_100a 2:4 SpMM library).

Mirrors the reference's host interface (SpeakOutLoudly/CUDA-Repo):
  SpMM_N2M4_Launch      src/SpMM_API.cu:61-70      -> SpMM_N2M4_Launch / launch
  toolCompressMatrixA   test/utils.h:91-150        -> toolCompressMatrixA / compress_a
  toolReorderMetadata   test/utils.h:155-185       -> toolReorderMetadata / reorder_metadata
  toolPackMatrixB       test/utils.h:188-229       -> toolPackMatrixB / pack_b

Everything goes through the C ABI of ``lib/libspmm24.so``; there is no
Python or CPU fallback.  Importing this module on a machine where the
library was not built raises ImportError.  PyTorch is used only to hand
device pointers and streams to the library.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(os.path.dirname(_PKG_DIR), "lib", "libspmm24.so")

if not os.path.exists(_LIB_PATH):
    raise ImportError(f"libspmm24.so not built ({_LIB_PATH}); run `make -C cuda-repo_b200`")

_lib = ctypes.CDLL(_LIB_PATH)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_vp = ctypes.c_void_p


class SpmmConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in
                ("tile_m", "tile_n", "stage_k", "stages", "split_k", "grid_ctas", "smem_bytes", "stream_k", "cta_pair")]


_lib.spmm24_launch.argtypes = [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int]
_lib.spmm24_launch.restype = ctypes.c_int
_lib.spmm24_launch_ex.argtypes = [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_uint]
_lib.spmm24_launch_ex.restype = ctypes.c_int
_lib.spmm24_compress_a.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, _u16p, _u16p]
_lib.spmm24_compress_a.restype = ctypes.c_int
_lib.spmm24_compress_reordered.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, _u16p, _u16p]
_lib.spmm24_compress_reordered.restype = ctypes.c_int
_lib.spmm24_reorder_metadata.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, _u16p]
_lib.spmm24_reorder_metadata.restype = ctypes.c_int
_lib.spmm24_pack_b.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, _u16p]
_lib.spmm24_pack_b.restype = ctypes.c_int
_lib.spmm24_prune_2of4.argtypes = [_u16p, ctypes.c_int, ctypes.c_int]
_lib.spmm24_prune_2of4.restype = ctypes.c_int
class PackedHeader(ctypes.Structure):
    """spmm24_packed_header (include/spmm24/SpMM_API.h)."""
    _fields_ = [("version", ctypes.c_uint32), ("dtype", ctypes.c_uint32), ("M", ctypes.c_uint32),
                ("K", ctypes.c_uint32), ("values_bytes", ctypes.c_uint64), ("meta_bytes", ctypes.c_uint64),
                ("checksum", ctypes.c_uint64)]


_lib.spmm24_save_packed.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp]
_lib.spmm24_save_packed.restype = ctypes.c_int
_lib.spmm24_load_packed_header.argtypes = [ctypes.c_char_p, ctypes.POINTER(PackedHeader)]
_lib.spmm24_load_packed_header.restype = ctypes.c_int
_lib.spmm24_load_packed.argtypes = [ctypes.c_char_p, _vp, ctypes.c_size_t, _vp, ctypes.c_size_t]
_lib.spmm24_load_packed.restype = ctypes.c_int


class Gather(ctypes.Structure):
    """spmm24_gather (include/spmm24/SpMM_API.h)."""
    _fields_ = [("c_full", ctypes.c_void_p * 8), ("n_ranks", ctypes.c_int), ("row_offset", ctypes.c_int),
                ("m_full", ctypes.c_int), ("c_multicast", ctypes.c_void_p)]


class IpcHandle(ctypes.Structure):
    """spmm24_ipc_handle (include/spmm24/SpMM_API.h)."""
    _fields_ = [("handle", ctypes.c_ubyte * 64), ("offset", ctypes.c_uint64)]


_lib.spmm24_launch_gather.argtypes = [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_uint, ctypes.POINTER(Gather)]
_lib.spmm24_launch_gather.restype = ctypes.c_int
_lib.spmm24_gather_barrier.argtypes = [_vp, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int,
                                       ctypes.c_uint32, ctypes.c_uint]
_lib.spmm24_gather_barrier.restype = ctypes.c_int
_lib.spmm24_ipc_export.argtypes = [_vp, ctypes.POINTER(IpcHandle)]
_lib.spmm24_ipc_export.restype = ctypes.c_int
_lib.spmm24_ipc_import.argtypes = [ctypes.POINTER(IpcHandle), ctypes.POINTER(ctypes.c_void_p)]
_lib.spmm24_ipc_import.restype = ctypes.c_int
_lib.spmm24_ipc_close.argtypes = [_vp]
_lib.spmm24_ipc_close.restype = ctypes.c_int


class Epilogue(ctypes.Structure):
    """spmm24_epilogue (include/spmm24/SpMM_API.h)."""
    _fields_ = [("bias", ctypes.c_void_p), ("residual", ctypes.c_void_p), ("alpha", ctypes.c_float),
                ("activation", ctypes.c_int), ("out_layout", ctypes.c_int)]


_lib.spmm24_launch_fused.argtypes = [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_uint, ctypes.POINTER(Epilogue)]
_lib.spmm24_launch_fused.restype = ctypes.c_int
_lib.spmm24_prune_2of4_bf16.argtypes = [_u16p, ctypes.c_int, ctypes.c_int]
_lib.spmm24_prune_2of4_bf16.restype = ctypes.c_int
_lib.spmm24_prune_2of4_bf16_device.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int]
_lib.spmm24_prune_2of4_bf16_device.restype = ctypes.c_int
_lib.spmm24_pack_a_device.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp]
_lib.spmm24_pack_a_device.restype = ctypes.c_int
_lib.spmm24_prune_2of4_device.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int]
_lib.spmm24_prune_2of4_device.restype = ctypes.c_int
_lib.spmm24_pack_b_device.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
_lib.spmm24_pack_b_device.restype = ctypes.c_int
_u8p = ctypes.POINTER(ctypes.c_uint8)
_lib.spmm24_prune_2of4_fp8.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
_lib.spmm24_prune_2of4_fp8.restype = ctypes.c_int
_lib.spmm24_compress_a_fp8.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, _u8p, _u8p]
_lib.spmm24_compress_a_fp8.restype = ctypes.c_int
_lib.spmm24_launch_fp8.argtypes = [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_uint, ctypes.c_void_p]
_lib.spmm24_launch_fp8.restype = ctypes.c_int
_lib.spmm24_pack_a_fp8_device.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp]
_lib.spmm24_pack_a_fp8_device.restype = ctypes.c_int
_lib.spmm24_workspace_bytes.argtypes = [ctypes.c_int] * 4
_lib.spmm24_workspace_bytes.restype = ctypes.c_size_t
_lib.spmm24_select_config.argtypes = [ctypes.c_int] * 4 + [ctypes.POINTER(SpmmConfig)]
_lib.spmm24_select_config_fp8.argtypes = [ctypes.c_int] * 4 + [ctypes.POINTER(SpmmConfig)]
_lib.spmm24_select_config_fp8.restype = ctypes.c_int
_lib.spmm24_select_config.restype = ctypes.c_int
_lib.spmm24_device_status.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint32)]
_lib.spmm24_device_status.restype = ctypes.c_int
_lib.spmm24_shard_rows.argtypes = [ctypes.c_int] * 4 + [ctypes.POINTER(ctypes.c_int)] * 2
_lib.spmm24_shard_rows.restype = ctypes.c_int
_lib.spmm24_last_error.restype = ctypes.c_char_p
_lib.spmm24_version.restype = ctypes.c_char_p

CUDA_SUCCESS = 0
CUDA_ERROR_INVALID_VALUE = 1
STATIC_WEIGHTS = 1  # SPMM24_STATIC_WEIGHTS
NO_PDL = 2          # SPMM24_NO_PDL
BF16 = 4            # SPMM24_BF16
ACT_NONE, ACT_RELU, ACT_SILU, ACT_GELU = 0, 1, 2, 3   # SPMM24_ACT_*
OUT_ROW_MAJOR, OUT_PACKED_B = 0, 1                    # SPMM24_OUT_*
PRUNE_NONE, PRUNE_F16, PRUNE_BF16 = 0, 1, 2           # SPMM24_PRUNE_*
FP8_E4M3, FP8_E5M2 = 0, 1                             # SPMM24_FP8_E4M3 / E5M2
FP8_A_E5M2, FP8_B_E5M2 = 8, 16                        # spmm24_launch_fp8 flags


class SpmmError(RuntimeError):
    def __init__(self, code: int, where: str):
        msg = _lib.spmm24_last_error().decode() if code == CUDA_ERROR_INVALID_VALUE else ""
        super().__init__(f"{where}: cudaError {code}" + (f" ({msg})" if msg else ""))
        self.code = code


def library_path() -> str:
    return _LIB_PATH


def version() -> str:
    return _lib.spmm24_version().decode()


def _ptr(x) -> int | None:
    """Device pointer of a torch tensor, an int address, or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _stream_handle(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


# -------------------------------------------------------------- launch
def launch(stream, compressed_a, b_packed, metadata, c, M: int, N: int, K: int, split_reduction=None,
           split_k: int = 0) -> int:
    """spmm24_launch through the C ABI; returns the cudaError_t code."""
    return _lib.spmm24_launch(_stream_handle(stream), _ptr(compressed_a), _ptr(b_packed), _ptr(metadata), _ptr(c),
                              M, N, K, _ptr(split_reduction), split_k)


def launch_ex(stream, compressed_a, b_packed, metadata, c, M: int, N: int, K: int, split_k: int = 0,
              flags: int = 0) -> int:
    """spmm24_launch_ex through the C ABI; returns the cudaError_t code."""
    return _lib.spmm24_launch_ex(_stream_handle(stream), _ptr(compressed_a), _ptr(b_packed), _ptr(metadata), _ptr(c),
                                 M, N, K, split_k, flags)


def launch_fused(stream, compressed_a, b_packed, metadata, c, M: int, N: int, K: int, split_k: int = 0,
                 flags: int = 0, bias=None, residual=None, alpha: float = 1.0, activation: int = ACT_NONE,
                 out_layout: int = OUT_ROW_MAJOR) -> int:
    """spmm24_launch_fused: C = act(alpha * A_sparse B + bias) + residual, in
    C's layout (row-major or the next layer's packed B); returns the
    cudaError_t code."""
    epi = Epilogue(_ptr(bias), _ptr(residual), float(alpha), int(activation), int(out_layout))
    return _lib.spmm24_launch_fused(_stream_handle(stream), _ptr(compressed_a), _ptr(b_packed), _ptr(metadata),
                                    _ptr(c), M, N, K, split_k, flags, ctypes.byref(epi))


def launch_fp8(stream, values, b_nk, metadata, c, M: int, N: int, K: int, split_k: int = 0, flags: int = 0,
               bias=None, residual=None, alpha: float = 1.0, activation: int = ACT_NONE,
               out_layout: int = OUT_ROW_MAJOR) -> int:
    """spmm24_launch_fp8: C = act(alpha * A_sparse B + bias) + residual with fp8
    A (values + metadata in the fp8 formats) and B as N x K fp8 bytes; C fp16
    (bf16 with BF16 in flags).  Returns the cudaError_t code."""
    epi = Epilogue(_ptr(bias), _ptr(residual), float(alpha), int(activation), int(out_layout))
    return _lib.spmm24_launch_fp8(_stream_handle(stream), _ptr(values), _ptr(b_nk), _ptr(metadata), _ptr(c), M, N, K,
                                  split_k, flags, ctypes.addressof(epi))


class Problem(ctypes.Structure):
    """spmm24_problem (include/spmm24/SpMM_API.h)."""
    _fields_ = [("compressed_a", ctypes.c_void_p), ("b_packed", ctypes.c_void_p), ("metadata", ctypes.c_void_p),
                ("c", ctypes.c_void_p), ("M", ctypes.c_int), ("N", ctypes.c_int), ("K", ctypes.c_int),
                ("gather", ctypes.c_void_p), ("epilogue", ctypes.c_void_p)]


_lib.spmm24_launch_grouped.argtypes = [_vp, ctypes.POINTER(Problem), ctypes.c_int, ctypes.c_uint]
_lib.spmm24_launch_grouped.restype = ctypes.c_int
_lib.spmm24_launch_grouped_fp8.argtypes = [_vp, ctypes.POINTER(Problem), ctypes.c_int, ctypes.c_uint]
_lib.spmm24_launch_grouped_fp8.restype = ctypes.c_int


def problem_array(problems):
    """A ctypes array of spmm24_problem from (compressed_a, b_packed, metadata,
    c, M, N, K[, gather[, epilogue]]) tuples (tensors or int addresses;
    gather: a Gather structure, epilogue: an Epilogue structure, either may
    be None; both kept alive by the returned array)."""
    arr = (Problem * len(problems))()
    keep = []
    for i, t in enumerate(problems):
        a, b, e, c, M, N, K = t[:7]
        g = t[7] if len(t) > 7 else None
        ep = t[8] if len(t) > 8 else None
        keep += [x for x in (g, ep) if x is not None]
        arr[i] = Problem(_ptr(a), _ptr(b), _ptr(e), _ptr(c), M, N, K,
                         ctypes.addressof(g) if g is not None else None,
                         ctypes.addressof(ep) if ep is not None else None)
    arr._keep = keep
    return arr


def make_gather(c_full_ptrs, row_offset: int, m_full: int, c_multicast=None) -> "Gather":
    """A spmm24_gather descriptor: rank r's full C at c_full_ptrs[r]."""
    if len(c_full_ptrs) > 8:
        raise ValueError("at most 8 ranks (SPMM24_MAX_GATHER_RANKS)")
    g = Gather()
    for r, p in enumerate(c_full_ptrs):
        g.c_full[r] = _ptr(p)
    g.n_ranks = len(c_full_ptrs)
    g.row_offset = row_offset
    g.m_full = m_full
    g.c_multicast = _ptr(c_multicast)
    return g


class GroupBarrier(ctypes.Structure):
    """spmm24_group_barrier (include/spmm24/SpMM_API.h)."""
    _fields_ = [("flag_arrays", ctypes.c_void_p * 8), ("n_ranks", ctypes.c_int), ("rank", ctypes.c_int),
                ("limit_us", ctypes.c_uint)]


_lib.spmm24_launch_grouped_gather.argtypes = [_vp, ctypes.POINTER(Problem), ctypes.c_int, ctypes.c_uint,
                                              ctypes.POINTER(GroupBarrier)]
_lib.spmm24_launch_grouped_gather.restype = ctypes.c_int


def group_barrier(flag_ptrs, rank: int, limit_us: int = 2_000_000) -> GroupBarrier:
    """A spmm24_group_barrier over the ranks' flag arrays (n_ranks + 1 u32 each)."""
    if len(flag_ptrs) > 8:
        raise ValueError("at most 8 ranks (SPMM24_MAX_GATHER_RANKS)")
    b = GroupBarrier()
    for r, p in enumerate(flag_ptrs):
        b.flag_arrays[r] = _ptr(p)
    b.n_ranks = len(flag_ptrs)
    b.rank = rank
    b.limit_us = limit_us
    return b


def launch_grouped_gather(stream, problems, barrier: GroupBarrier, flags: int = 0) -> int:
    """spmm24_launch_grouped_gather: a grouped launch whose problems gather,
    with the cross-GPU barrier at the end of the same kernel."""
    arr = problems if isinstance(problems, ctypes.Array) else problem_array(problems)
    return _lib.spmm24_launch_grouped_gather(_stream_handle(stream), arr, len(arr), flags, ctypes.byref(barrier))


def launch_grouped(stream, problems, flags: int = 0, fp8: bool = False) -> int:
    """spmm24_launch_grouped (fp8: spmm24_launch_grouped_fp8): several
    independent N <= 32 SpMMs in one persistent launch.  `problems`: a list
    of problem_array() tuples, or such an array.  Returns the cudaError_t
    code."""
    arr = problems if isinstance(problems, ctypes.Array) else problem_array(problems)
    fn = _lib.spmm24_launch_grouped_fp8 if fp8 else _lib.spmm24_launch_grouped
    return fn(_stream_handle(stream), arr, len(arr), flags)


def SpMM_N2M4_Launch(stream, Compressed_A, B, metadata, C, M_Global: int, N_Global: int, K_Global: int,
                     Split_Reduction=None, Split_K: int = 1) -> int:
    """The reference's launcher signature (src/SpMM_API.cu:61-70)."""
    return launch(stream, Compressed_A, B, metadata, C, M_Global, N_Global, K_Global, Split_Reduction, Split_K)


def spmm(compressed_a, metadata, b_packed, M: int, N: int, K: int, split_k: int = 0, out=None, stream=None):
    """C = A_sparse * B for device tensors in the ABI formats; returns C (M x N fp16).

    Raises SpmmError when the library rejects the call."""
    import torch

    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=compressed_a.device)
    if stream is None:
        stream = torch.cuda.current_stream(compressed_a.device)
    rc = launch(stream, compressed_a, b_packed, metadata, out, M, N, K, None, split_k)
    if rc != CUDA_SUCCESS:
        raise SpmmError(rc, "spmm24_launch")
    return out


def select_config(M: int, N: int, K: int, split_k: int = 0) -> dict:
    cfg = SpmmConfig()
    if _lib.spmm24_select_config(M, N, K, split_k, ctypes.byref(cfg)) != 0:
        raise ValueError("unsupported shape")
    return {n: getattr(cfg, n) for n, _ in SpmmConfig._fields_}


class Tuning(ctypes.Structure):
    """spmm24_tuning (include/spmm24/SpMM_API.h)."""
    _fields_ = [(n, ctypes.c_int) for n in ("pair", "pair2", "pair_split", "tile_n", "deep_ring", "group_split")]


_lib.spmm24_set_tuning.argtypes = [ctypes.POINTER(Tuning)]
_lib.spmm24_set_tuning.restype = ctypes.c_int


def set_tuning(pair: int = -1, pair2: int = -1, pair_split: int = 0, tile_n: int = 0, deep_ring: int = 0,
               group_split: int = 0) -> None:
    """spmm24_set_tuning: process-wide picker override (tests and tuning
    sweeps); called with no arguments it restores the automatic choice."""
    t = Tuning(pair, pair2, pair_split, tile_n, deep_ring, group_split)
    rc = _lib.spmm24_set_tuning(ctypes.byref(t))
    if rc != 0:
        raise ValueError(f"spmm24_set_tuning: {_lib.spmm24_last_error().decode()}")


def reset_tuning() -> None:
    """Restores the automatic kernel choice."""
    _lib.spmm24_set_tuning(None)


_IntArr = ctypes.POINTER(ctypes.c_int)
_lib.spmm24_group_schedule.argtypes = [_IntArr, _IntArr, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       _IntArr, _IntArr, ctypes.POINTER(ctypes.c_longlong)]
_lib.spmm24_group_schedule.restype = ctypes.c_int


def group_schedule(Ms, Ks, fp8: bool = False, sms: int = 148, max_clusters4: int = 33) -> dict:
    """spmm24_group_schedule: the K split, unit count and makespan (in
    stages) a grouped launch of problems with these M and K would use, from
    the host alone (no GPU)."""
    n = len(Ms)
    if len(Ks) != n:
        raise ValueError("Ms and Ks must have the same length")
    m = (ctypes.c_int * n)(*Ms)
    k = (ctypes.c_int * n)(*Ks)
    split, units, mk = ctypes.c_int(), ctypes.c_int(), ctypes.c_longlong()
    if _lib.spmm24_group_schedule(m, k, n, int(fp8), sms, max_clusters4, ctypes.byref(split), ctypes.byref(units),
                                  ctypes.byref(mk)) != 0:
        raise ValueError("bad grouped problems")
    return {"split": split.value, "units": units.value, "makespan": mk.value}


def select_config_fp8(M: int, N: int, K: int, split_k: int = 0) -> dict:
    """spmm24_select_config_fp8: the configuration spmm24_launch_fp8 uses."""
    cfg = SpmmConfig()
    if _lib.spmm24_select_config_fp8(M, N, K, split_k, ctypes.byref(cfg)) != 0:
        raise ValueError("unsupported shape (K % 128)")
    return {n: getattr(cfg, n) for n, _ in SpmmConfig._fields_}


def workspace_bytes(M: int, N: int, K: int, split_k: int) -> int:
    return int(_lib.spmm24_workspace_bytes(M, N, K, split_k))


def device_status(device: int = 0) -> int:
    """Reads and clears the sticky status word (non-zero: a bounded wait gave up)."""
    v = ctypes.c_uint32(0)
    rc = _lib.spmm24_device_status(device, ctypes.byref(v))
    if rc != CUDA_SUCCESS:
        raise SpmmError(rc, "spmm24_device_status")
    return int(v.value)


# ------------------------------------------------------ device packer
def pack_a_device(dense, M: int, K: int, prune=False, values=None, meta=None, stream=None):
    """spmm24_pack_a_device on a device tensor holding the dense M x K fp16
    (or bf16) weights: optional magnitude 2:4 prune (True / PRUNE_F16, or
    PRUNE_BF16), compress and reordered metadata in one kernel.  Returns (values (M*K/2 fp16 as int16 bits), metadata (M*K/16
    u16 as int16), bad_rows (int)); synchronises the stream to read bad_rows."""
    import torch

    dev = dense.device
    if values is None:
        values = torch.empty(M * K // 2, dtype=torch.int16, device=dev)
    if meta is None:
        meta = torch.empty(M * K // 16, dtype=torch.int16, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    if stream is None:
        stream = torch.cuda.current_stream(dev)
    mode = int(prune) if not isinstance(prune, bool) else (PRUNE_F16 if prune else PRUNE_NONE)
    rc = _lib.spmm24_pack_a_device(_stream_handle(stream), _ptr(dense), M, K, mode, _ptr(values),
                                   _ptr(meta), _ptr(bad))
    if rc != CUDA_SUCCESS:
        raise SpmmError(rc, "spmm24_pack_a_device")
    return values, meta, int(bad.item())


def prune_2of4_device(dense, M: int, K: int, stream=None, bf16: bool = False) -> None:
    """spmm24_prune_2of4_device (bf16: spmm24_prune_2of4_bf16_device):
    in-place magnitude 2:4 prune of a device matrix."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(dense.device)
    fn = _lib.spmm24_prune_2of4_bf16_device if bf16 else _lib.spmm24_prune_2of4_device
    rc = fn(_stream_handle(stream), _ptr(dense), M, K)
    if rc != CUDA_SUCCESS:
        raise SpmmError(rc, "spmm24_prune_2of4_device")


def pack_b_device(b, K: int, N: int, out=None, stream=None):
    """spmm24_pack_b_device: row-major K x N device fp16 -> packed strips
    (ceil(N/8)*8*K halves, returned as int16 bits unless `out` is given)."""
    import torch

    if out is None:
        out = torch.empty(((N + 7) // 8) * 8 * K, dtype=torch.int16, device=b.device)
    if stream is None:
        stream = torch.cuda.current_stream(b.device)
    rc = _lib.spmm24_pack_b_device(_stream_handle(stream), _ptr(b), K, N, _ptr(out))
    if rc != CUDA_SUCCESS:
        raise SpmmError(rc, "spmm24_pack_b_device")
    return out


# ---------------------------------------------------------- sharding
# ---------------------------------------- fused all-gather across GPUs
def ipc_export(tensor) -> bytes:
    """spmm24_ipc_export: a 72-byte description of a device tensor's memory
    that another process of the node can map with ipc_import."""
    h = IpcHandle()
    rc = _lib.spmm24_ipc_export(_ptr(tensor), ctypes.byref(h))
    if rc != CUDA_SUCCESS:
        raise SpmmError(rc, "spmm24_ipc_export")
    return bytes(h)


def ipc_import(handle: bytes) -> int:
    """spmm24_ipc_import: maps a peer's exported memory; returns the device address."""
    h = IpcHandle.from_buffer_copy(handle)
    out = ctypes.c_void_p()
    rc = _lib.spmm24_ipc_import(ctypes.byref(h), ctypes.byref(out))
    if rc != CUDA_SUCCESS:
        raise SpmmError(rc, "spmm24_ipc_import")
    return int(out.value)


def ipc_close(ptr: int) -> None:
    rc = _lib.spmm24_ipc_close(ptr)
    if rc != CUDA_SUCCESS:
        raise SpmmError(rc, "spmm24_ipc_close")


def launch_gather(stream, compressed_a, b_packed, metadata, M: int, N: int, K: int, c_full_ptrs, row_offset: int,
                  m_full: int, split_k: int = 0, flags: int = 0, c_multicast=None) -> int:
    """spmm24_launch_gather: this rank's M-shard, written into every rank's
    full C (c_full_ptrs in rank order, own buffer included; or, with
    c_multicast, once through the full C's NVLink multicast address)."""
    if len(c_full_ptrs) > 8:
        raise ValueError("at most 8 ranks (SPMM24_MAX_GATHER_RANKS)")
    g = Gather()
    for i, p in enumerate(c_full_ptrs):
        g.c_full[i] = _ptr(p)
    g.n_ranks, g.row_offset, g.m_full = len(c_full_ptrs), row_offset, m_full
    g.c_multicast = _ptr(c_multicast)
    return _lib.spmm24_launch_gather(_stream_handle(stream), _ptr(compressed_a), _ptr(b_packed), _ptr(metadata), M, N,
                                     K, split_k, flags, ctypes.byref(g))


def gather_barrier(stream, flag_ptrs, rank: int, epoch: int, limit_us: int = 2_000_000) -> int:
    """spmm24_gather_barrier over the ranks' flag arrays (rank order)."""
    arr = (ctypes.c_void_p * len(flag_ptrs))(*[_ptr(p) for p in flag_ptrs])
    return _lib.spmm24_gather_barrier(_stream_handle(stream), arr, len(flag_ptrs), rank, epoch, limit_us)


def shard_rows(M: int, parts: int, index: int, align: int = 128) -> tuple[int, int]:
    """[row_begin, row_end) of shard `index` of `parts` (split along M)."""
    b, e = ctypes.c_int(), ctypes.c_int()
    if _lib.spmm24_shard_rows(M, parts, index, align, ctypes.byref(b), ctypes.byref(e)) != 0:
        raise ValueError("shard_rows: bad arguments")
    return b.value, e.value


def shard_views(compressed_a, metadata, M: int, K: int, row_begin: int, row_end: int):
    """The contiguous slices of compressed A and metadata holding rows
    [row_begin, row_end) -- works for numpy arrays and torch tensors."""
    if row_begin % 16 or row_end % 16 or not 0 <= row_begin <= row_end <= M:
        raise ValueError("shard rows must be multiples of 16 inside [0, M]")
    a = compressed_a.reshape(-1)[row_begin * K // 2: row_end * K // 2]
    e = metadata.reshape(-1)[row_begin * K // 16: row_end * K // 16]
    return a, e


# -------------------------------------------------------------- packer
def _u16(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    if a.dtype != np.uint16:
        raise TypeError("expected fp16 data (as float16 or raw uint16 bits)")
    return a


def _p(a: np.ndarray):
    return a.ctypes.data_as(_u16p)


def compress_a(dense_a: np.ndarray, M: int, K: int):
    """(values[M*K/2], raw metadata[M*K/16]) of a 2:4-sparse fp16 matrix."""
    d = _u16(dense_a).reshape(-1)
    vals = np.empty(M * K // 2, dtype=np.uint16)
    meta = np.empty(M * K // 16, dtype=np.uint16)
    n = _lib.spmm24_compress_a(_p(d), M, K, _p(vals), _p(meta))
    if n == -2:
        raise ValueError("matrix is not 2:4 sparse along K (a group of four has fewer than two zeros)")
    if n < 0:
        raise ValueError("compress_a: M and K must be multiples of 16")
    return vals, meta


def reorder_metadata(meta: np.ndarray, M: int, K: int) -> np.ndarray:
    m = _u16(meta).reshape(-1)
    out = np.empty_like(m)
    if _lib.spmm24_reorder_metadata(_p(m), M, K, _p(out)) != 0:
        raise ValueError("reorder_metadata: M % 16 and K % 64 must be 0")
    return out


def compress_reordered(dense_a: np.ndarray, M: int, K: int):
    """(values, on-device metadata) in one pass."""
    d = _u16(dense_a).reshape(-1)
    vals = np.empty(M * K // 2, dtype=np.uint16)
    meta = np.empty(M * K // 16, dtype=np.uint16)
    n = _lib.spmm24_compress_reordered(_p(d), M, K, _p(vals), _p(meta))
    if n == -2:
        raise ValueError("matrix is not 2:4 sparse along K (a group of four has fewer than two zeros)")
    if n < 0:
        raise ValueError("compress_reordered: M % 16 and K % 64 must be 0")
    return vals, meta


def pack_b(b_rowmajor: np.ndarray, K: int, N: int) -> np.ndarray:
    """Packed B (ceil(N/8) strips of K x 8); pad columns are zero."""
    b = _u16(b_rowmajor).reshape(-1)
    out = np.empty(((N + 7) // 8) * 8 * K, dtype=np.uint16)
    if _lib.spmm24_pack_b(_p(b), K, N, _p(out)) != 0:
        raise ValueError("pack_b: K % 64 must be 0")
    return out


def prune_2of4(dense_a: np.ndarray, M: int, K: int) -> np.ndarray:
    """Magnitude 2:4 pruning along K (returns a pruned copy)."""
    a = _u16(dense_a).reshape(-1).copy()
    if _lib.spmm24_prune_2of4(_p(a), M, K) != 0:
        raise ValueError("prune_2of4: K % 4 must be 0")
    return a


def prune_2of4_bf16(dense_a: np.ndarray, M: int, K: int) -> np.ndarray:
    """Magnitude 2:4 pruning along K of bf16 bit patterns (returns a pruned copy)."""
    a = _u16(dense_a).reshape(-1).copy()
    if _lib.spmm24_prune_2of4_bf16(_p(a), M, K) != 0:
        raise ValueError("prune_2of4_bf16: K % 4 must be 0")
    return a


def _u8(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype != np.uint8:
        raise TypeError("fp8 arrays are passed as uint8 bit patterns")
    return a


def prune_2of4_fp8(dense_a: np.ndarray, M: int, K: int, fmt: int = FP8_E4M3) -> np.ndarray:
    """Magnitude 2:4 pruning along K of fp8 bytes (returns a pruned copy)."""
    a = _u8(dense_a).reshape(-1).copy()
    if _lib.spmm24_prune_2of4_fp8(a.ctypes.data_as(_u8p), M, K, fmt) != 0:
        raise ValueError("prune_2of4_fp8: K % 4 must be 0 and fmt 0 or 1")
    return a


def compress_a_fp8(dense_a: np.ndarray, M: int, K: int):
    """(values, metadata) of a 2:4-sparse fp8 matrix in the fp8 SpMM's formats."""
    d = _u8(dense_a).reshape(-1)
    vals = np.empty(M * K // 2, dtype=np.uint8)
    meta = np.empty(M * K // 8, dtype=np.uint8)
    n = _lib.spmm24_compress_a_fp8(d.ctypes.data_as(_u8p), M, K, vals.ctypes.data_as(_u8p), meta.ctypes.data_as(_u8p))
    if n == -2:
        raise ValueError("matrix is not 2:4 sparse along K (a group of four has fewer than two zeros)")
    if n < 0:
        raise ValueError("compress_a_fp8: M % 16 and K % 128 must be 0")
    return vals, meta


def pack_a_fp8_device(dense, M: int, K: int, prune: int = 0, values=None, meta=None, bad_blocks=None, stream=None):
    """spmm24_pack_a_fp8_device on uint8 device tensors; returns (values, meta).
    prune: 0 none, 1 E4M3, 2 E5M2."""
    import torch

    if values is None:
        values = torch.empty(M * K // 2, dtype=torch.uint8, device=dense.device)
    if meta is None:
        meta = torch.empty(M * K // 8, dtype=torch.uint8, device=dense.device)
    if stream is None:
        stream = torch.cuda.current_stream(dense.device)
    rc = _lib.spmm24_pack_a_fp8_device(_stream_handle(stream), _ptr(dense), M, K, int(prune), _ptr(values), _ptr(meta),
                                       _ptr(bad_blocks))
    if rc != CUDA_SUCCESS:
        raise SpmmError(rc, "spmm24_pack_a_fp8_device")
    return values, meta


# ------------------------------------------------- packed-weight files
PACKED_ERRORS = {-1: "bad argument or shape", -2: "I/O error or short file",
                 -3: "not a packed-weight file (magic, version or size)", -4: "checksum mismatch",
                 -5: "the file's payload is larger than the buffers given (file changed after its header was read)"}


def save_packed(path: str, values: np.ndarray, meta: np.ndarray, M: int, K: int, bf16: bool = False) -> None:
    """spmm24_save_packed: write compressed values + reordered metadata (host arrays)."""
    v = _u16(values).reshape(-1)
    m = _u16(meta).reshape(-1)
    if v.size != M * K // 2 or m.size != M * K // 16:
        raise ValueError("values / metadata sizes do not match M x K")
    rc = _lib.spmm24_save_packed(os.fsencode(path), 1 if bf16 else 0, M, K, v.ctypes.data, m.ctypes.data)
    if rc != 0:
        raise OSError(f"spmm24_save_packed: {PACKED_ERRORS.get(rc, rc)}")


def load_packed(path: str):
    """spmm24_load_packed: returns (values, metadata, M, K, bf16) as host arrays."""
    h = PackedHeader()
    rc = _lib.spmm24_load_packed_header(os.fsencode(path), ctypes.byref(h))
    if rc != 0:
        raise OSError(f"spmm24_load_packed_header: {PACKED_ERRORS.get(rc, rc)}")
    if h.dtype not in (0, 1):
        raise ValueError("an fp8 packed-weight file: use load_packed_fp8")
    v = np.empty(h.values_bytes // 2, dtype=np.uint16)
    m = np.empty(h.meta_bytes // 2, dtype=np.uint16)
    rc = _lib.spmm24_load_packed(os.fsencode(path), v.ctypes.data, v.nbytes, m.ctypes.data, m.nbytes)
    if rc != 0:
        raise OSError(f"spmm24_load_packed: {PACKED_ERRORS.get(rc, rc)}")
    return v, m, int(h.M), int(h.K), bool(h.dtype == 1)


def save_packed_fp8(path: str, values: np.ndarray, meta: np.ndarray, M: int, K: int, fmt: int = FP8_E4M3) -> None:
    """spmm24_save_packed with dtype 2 (E4M3) or 3 (E5M2): the fp8 SpMM's values and metadata."""
    v = _u8(values).reshape(-1)
    m = _u8(meta).reshape(-1)
    if v.size != M * K // 2 or m.size != M * K // 8:
        raise ValueError("values / metadata sizes do not match M x K")
    rc = _lib.spmm24_save_packed(os.fsencode(path), 2 + int(fmt), M, K, v.ctypes.data, m.ctypes.data)
    if rc != 0:
        raise OSError(f"spmm24_save_packed: {PACKED_ERRORS.get(rc, rc)}")


def load_packed_fp8(path: str):
    """Returns (values, metadata, M, K, fmt) of an fp8 packed-weight file (uint8 host arrays)."""
    h = PackedHeader()
    rc = _lib.spmm24_load_packed_header(os.fsencode(path), ctypes.byref(h))
    if rc != 0:
        raise OSError(f"spmm24_load_packed_header: {PACKED_ERRORS.get(rc, rc)}")
    if h.dtype not in (2, 3):
        raise ValueError("a 16-bit packed-weight file: use load_packed")
    v = np.empty(h.values_bytes, dtype=np.uint8)
    m = np.empty(h.meta_bytes, dtype=np.uint8)
    rc = _lib.spmm24_load_packed(os.fsencode(path), v.ctypes.data, v.nbytes, m.ctypes.data, m.nbytes)
    if rc != 0:
        raise OSError(f"spmm24_load_packed: {PACKED_ERRORS.get(rc, rc)}")
    return v, m, int(h.M), int(h.K), int(h.dtype) - 2


# Reference-named wrappers (Block sizes fixed as in the reference harness).
def toolCompressMatrixA(denseMatrixA: np.ndarray, Global_M: int, Global_K: int, Block_M: int = 16,
                        Block_K: int = 16):
    if (Block_M, Block_K) != (16, 16):
        raise ValueError("only 16x16 blocks are supported")
    vals, meta = compress_a(denseMatrixA, Global_M, Global_K)
    return vals.size, vals, meta


def toolReorderMetadata(matadata: np.ndarray, Global_M: int, Global_K: int, Block_M: int = 16, Block_K: int = 16):
    if (Block_M, Block_K) != (16, 16):
        raise ValueError("only 16x16 blocks are supported")
    return reorder_metadata(matadata, Global_M, Global_K)


def toolPackMatrixB(MatrixB: np.ndarray, Global_K: int, Global_N: int, Block_K: int = 64, Block_N: int = 8):
    if (Block_K, Block_N) != (64, 8):
        raise ValueError("only 64x8 blocks are supported")
    return pack_b(MatrixB, Global_K, Global_N)
