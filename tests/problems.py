"""Seeded 2:4 SpMM problems and the parity tolerance, shared by the tests.

Inputs come from the oracle's generator (splitmix64 + Box-Muller in
oracle/oracle.c), so every test sees bit-identical data on any machine.
The tolerance follows the north star: max relative error <= 1e-2 and mean
absolute error <= 1e-3 (scaled by the output magnitude when that exceeds 1)
against the oracle's fp32 result rounded to fp16.  The relative error's
denominator is max(|ref|, 1e-3 * max|ref|) so outputs near zero (where one
fp16 ulp is a large relative change) do not dominate.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

import oracle as O

MAX_REL = 1e-2
MEAN_ABS = 1e-3


@dataclass
class Problem:
    M: int
    N: int
    K: int
    a_dense: np.ndarray      # M*K fp16 bits, pruned 2:4
    b_rowmajor: np.ndarray   # K*N fp16 bits
    vals: np.ndarray         # M*K/2
    meta: np.ndarray         # M*K/16, reordered (on-device layout)
    b_packed: np.ndarray     # ceil(N/8)*8*K


def make_problem(M: int, N: int, K: int, seed: int = 0, a_dist: str = "normal", a_scale: float = 1.0,
                 b_dist: str = "uniform", b_scale: float = 1.0, mask: str = "magnitude") -> Problem:
    if a_dist == "normal":
        a = O.normal_f16(M * K, seed, 0.0, a_scale)
    else:
        a = O.uniform_f16(M * K, seed, -a_scale, a_scale)
    if mask == "magnitude":
        a = O.prune_magnitude_2of4(a, M, K)
    else:
        a = O.random_mask_2of4(a, M, K, seed + 1000)
    if b_dist == "normal":
        b = O.normal_f16(K * N, seed + 1, 0.0, b_scale)
    else:
        b = O.uniform_f16(K * N, seed + 1, -b_scale, b_scale)
    return pack_problem(M, N, K, a, b)


def pack_problem(M: int, N: int, K: int, a: np.ndarray, b: np.ndarray) -> Problem:
    n, vals, raw = O.compress_a(a, M, K)
    assert n == M * K // 2, n
    meta = O.reorder_metadata(raw, M, K)
    n8 = (N + 7) // 8 * 8
    if n8 != N:
        bp = np.zeros(K * n8, dtype=np.uint16)
        bp.reshape(K, n8)[:, :N] = b.reshape(K, N)
        b_packed = O.pack_b(bp, K, n8)
    else:
        b_packed = O.pack_b(b, K, N)
    return Problem(M, N, K, a, b, vals, meta, b_packed)


def oracle_c(p: Problem, rows: np.ndarray | None = None) -> np.ndarray:
    """fp32 oracle result (M x N), or only the given rows."""
    if rows is None:
        return O.dense_gemm_f32(p.a_dense, p.b_rowmajor, p.M, p.N, p.K).reshape(p.M, p.N)
    sub = p.a_dense.reshape(p.M, p.K)[rows].reshape(-1)
    return O.dense_gemm_f32(sub, p.b_rowmajor, len(rows), p.N, p.K).reshape(len(rows), p.N)


def f16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def compare(got_f16_bits: np.ndarray, ref_f32: np.ndarray) -> dict:
    ref16 = f16_bits_to_f32(O.f32_to_f16_bits(ref_f32.reshape(-1)))
    got = f16_bits_to_f32(got_f16_bits.reshape(-1))
    diff = np.abs(got - ref16)
    scale = float(np.max(np.abs(ref16))) if ref16.size else 0.0
    denom = np.maximum(np.abs(ref16), max(1e-3 * scale, 1e-30))
    return {
        "max_rel": float(np.max(diff / denom)) if diff.size else 0.0,
        "mean_abs": float(np.mean(diff)) if diff.size else 0.0,
        "mean_ref": float(np.mean(np.abs(ref16))) if diff.size else 0.0,
        "finite": bool(np.all(np.isfinite(got))),
        "mismatch": int(np.count_nonzero(diff)),
    }


def within_tolerance(stats: dict) -> bool:
    return (stats["finite"] and stats["max_rel"] <= MAX_REL
            and stats["mean_abs"] <= MEAN_ABS * max(1.0, stats["mean_ref"]))
