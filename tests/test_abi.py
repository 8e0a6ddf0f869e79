"""The C-ABI boundary: the library loads, exports every entry point that
include/spmm24/SpMM_API.h declares (plus the reference's mangled C++
names), and rejects bad calls before touching a GPU."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import oracle as O
import spmm24

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "spmm24", "SpMM_API.h")

# The reference's launcher as C++ code links to it (verified with nm on a
# build of src/SpMM_API.cu), plus the packer names from test/utils.h.
REFERENCE_MANGLED = [
    "_Z16SpMM_N2M4_LaunchP11CUstream_stPK6__halfS3_PKtPS1_iiiS6_i",
    "_Z19toolCompressMatrixAP6__halfiiiiPS0_PPt",
    "_Z19toolReorderMetadataPtiiiiPS_",
    "_Z15toolPackMatrixBP6__halfiiiiPS0_",
]


def declared_c_functions():
    text = open(HEADER).read()
    c_part = text.split("} /* extern \"C\" */")[0]
    return sorted(set(re.findall(r"\b(spmm24_[a-z_0-9]+)\s*\(", c_part)))


def exported_symbols(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_header_declares_entry_points():
    names = declared_c_functions()
    assert "spmm24_launch" in names and "spmm24_compress_a" in names and len(names) >= 10


def test_library_exports_all_declared_symbols():
    syms = exported_symbols(spmm24.library_path())
    missing = [n for n in declared_c_functions() if n not in syms]
    assert not missing, missing
    for m in REFERENCE_MANGLED:
        assert m in syms, m


@pytest.mark.skipif(not O.ref_spmm_available(), reason="reference kernel not built (oracle/_ref)")
def test_launcher_mangled_name_equals_reference_build():
    ref_syms = exported_symbols(os.path.join(REPO, "oracle", "_ref", "libref_spmm.so"))
    assert REFERENCE_MANGLED[0] in ref_syms


def test_version_and_workspace():
    assert "sm_100a" in spmm24.version()
    assert spmm24.workspace_bytes(4096, 16, 4096, 4) == 0




def _launch(a, b, e, c, M, N, K, split=1):
    return spmm24.launch(None, a, b, e, c, M, N, K, None, split)


def test_launch_rejects_bad_arguments_without_gpu():
    ok = (0x10000, 0x20000, 0x30000, 0x40000)
    assert _launch(0, *ok[1:], 256, 16, 256) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert "null" in spmm24._lib.spmm24_last_error().decode()
    assert _launch(*ok, 250, 16, 256) == spmm24.CUDA_ERROR_INVALID_VALUE   # M % 16
    assert _launch(*ok, 256, 16, 96) == spmm24.CUDA_ERROR_INVALID_VALUE    # K % 64
    assert _launch(*ok, 256, 0, 256) == spmm24.CUDA_ERROR_INVALID_VALUE    # N <= 0
    assert _launch(*ok, 256, 16, 256, split=-1) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert _launch(0x10008, *ok[1:], 256, 16, 256) == spmm24.CUDA_ERROR_INVALID_VALUE  # A misaligned
    assert _launch(ok[0], ok[1], ok[2], 0x40001, 256, 16, 256) == spmm24.CUDA_ERROR_INVALID_VALUE  # C odd
    assert "aligned" in spmm24._lib.spmm24_last_error().decode()


def test_fused_launch_rejects_bad_epilogues_without_gpu():
    ok = (0x10000, 0x20000, 0x30000, 0x40000)
    L = spmm24._lib

    def fused(c=ok[3], flags=0, **kw):
        e = spmm24.Epilogue(kw.get("bias"), kw.get("residual"), kw.get("alpha", 1.0), kw.get("act", 0),
                            kw.get("layout", 0))
        return L.spmm24_launch_fused(None, ok[0], ok[1], ok[2], c, 256, 16, 256, 0, flags, ctypes.byref(e))

    assert fused(act=7) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert "activation" in L.spmm24_last_error().decode()
    assert fused(layout=2) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert fused(alpha=float("nan")) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert fused(bias=0x50001) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert fused(c=0x40008, layout=1) == spmm24.CUDA_ERROR_INVALID_VALUE  # packed C must be 16-byte aligned
    assert fused(flags=8) == spmm24.CUDA_ERROR_INVALID_VALUE               # unknown flag
    assert L.spmm24_pack_a_device(None, ok[0], 256, 256, 3, ok[1], ok[2], None) == spmm24.CUDA_ERROR_INVALID_VALUE


def test_host_bf16_prune_matches_oracle():
    rng = np.random.default_rng(4)
    a = (rng.standard_normal(64 * 128).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    a[rng.random(a.size) < 0.2] = 0x8000
    a[rng.random(a.size) < 0.05] = 0x7FC0  # NaN
    assert np.array_equal(spmm24.prune_2of4_bf16(a, 64, 128), O.prune_magnitude_2of4_bf16(a, 64, 128))


def test_gather_rejects_bad_arguments_without_gpu():
    L = spmm24._lib
    A, B, E = 0x10000, 0x20000, 0x30000
    ok = [0x40000, 0x50000]

    def gather(ptrs, row_offset=0, m_full=512, M=256):
        return spmm24.launch_gather(None, A, B, E, M, 16, 256, ptrs, row_offset, m_full)

    assert gather([]) == spmm24.CUDA_ERROR_INVALID_VALUE
    g = spmm24.Gather()
    g.c_full[0], g.n_ranks, g.row_offset, g.m_full = ok[0], 9, 0, 512        # more than 8 ranks
    assert L.spmm24_launch_gather(None, A, B, E, 256, 16, 256, 0, 0, ctypes.byref(g)) == spmm24.CUDA_ERROR_INVALID_VALUE
    with pytest.raises(ValueError):
        gather(ok * 5)
    assert gather(ok, row_offset=300) == spmm24.CUDA_ERROR_INVALID_VALUE      # shard past the full C
    assert gather(ok, m_full=128) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert gather([0x40000, 0x50008]) == spmm24.CUDA_ERROR_INVALID_VALUE       # misaligned peer buffer
    assert "aligned" in L.spmm24_last_error().decode()
    assert spmm24.gather_barrier(None, [0x60000, 0x70000], 2, 1) == spmm24.CUDA_ERROR_INVALID_VALUE  # rank >= n
    assert spmm24.gather_barrier(None, [0x60000, 0x70002], 0, 1) == spmm24.CUDA_ERROR_INVALID_VALUE  # misaligned
    assert spmm24.gather_barrier(None, [0x60000], 0, 1, limit_us=0) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert L.spmm24_ipc_export(None, None) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert L.spmm24_ipc_close(0x1234) == spmm24.CUDA_ERROR_INVALID_VALUE      # never imported


def test_device_packer_rejects_bad_arguments_without_gpu():
    L = spmm24._lib
    ok = 0x10000
    assert L.spmm24_pack_a_device(None, 0, 256, 256, 1, ok, ok, None) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert "null" in L.spmm24_last_error().decode()
    assert L.spmm24_pack_a_device(None, ok, 250, 256, 1, ok, ok, None) == spmm24.CUDA_ERROR_INVALID_VALUE  # M % 16
    assert L.spmm24_pack_a_device(None, ok, 256, 96, 1, ok, ok, None) == spmm24.CUDA_ERROR_INVALID_VALUE   # K % 64
    assert L.spmm24_pack_a_device(None, ok + 8, 256, 256, 1, ok, ok, None) == spmm24.CUDA_ERROR_INVALID_VALUE
    assert "aligned" in L.spmm24_last_error().decode()
    assert L.spmm24_prune_2of4_device(None, ok, 16, 6) == spmm24.CUDA_ERROR_INVALID_VALUE  # K % 4
    assert L.spmm24_prune_2of4_device(None, ok + 4, 16, 8) == spmm24.CUDA_ERROR_INVALID_VALUE  # 8-byte alignment
    assert L.spmm24_pack_b_device(None, ok, 96, 16, ok) == spmm24.CUDA_ERROR_INVALID_VALUE  # K % 64
    assert L.spmm24_pack_b_device(None, ok, 64, 16, ok + 2) == spmm24.CUDA_ERROR_INVALID_VALUE  # output alignment
    assert L.spmm24_pack_b_device(None, ok + 1, 64, 16, ok) == spmm24.CUDA_ERROR_INVALID_VALUE  # odd source


def test_select_config_picks_tiles_and_splits():
    c = spmm24.select_config(4096, 16, 4096)
    assert c["tile_m"] == 128 and c["tile_n"] == 16 and c["stage_k"] == 128
    # narrow N with an automatic split: shallow ring (two CTAs per SM), a K
    # split towards two slots per SM, at least five stages per slice for long K
    assert c["stream_k"] == 0 and c["stages"] == 4 and c["split_k"] == 6 and c["grid_ctas"] == 192
    assert spmm24.select_config(11008, 16, 4096)["split_k"] == 3
    assert spmm24.select_config(4096, 16, 11008)["split_k"] == 8
    assert spmm24.select_config(4096, 16, 1024)["split_k"] == 4  # short K: two stages per slice
    assert spmm24.select_config(256, 16, 128)["split_k"] == 1  # at least two stages per slice
    # an explicit split is honoured
    c = spmm24.select_config(4096, 16, 4096, 4)
    assert c["stream_k"] == 0 and c["split_k"] == 4 and c["grid_ctas"] == 128
    # mid N: one CTA per 128 x 128 tile with the deep ring
    c = spmm24.select_config(4096, 128, 4096)
    assert c["tile_n"] == 128 and c["stages"] == 4 and c["cta_pair"] == 0
    # wide N with K % 128 == 0: 256 x 256 tiles on CTA pairs
    c = spmm24.select_config(2048, 2048, 2048)
    assert c["cta_pair"] == 1 and c["tile_m"] == 256 and c["tile_n"] == 256 and c["split_k"] == 1
    assert c["grid_ctas"] == 128
    # less than half a wave of those (32 tiles) and no K split: 256 x 128 tiles
    c = spmm24.select_config(4096, 512, 4096)
    assert c["cta_pair"] == 1 and c["tile_m"] == 256 and c["tile_n"] == 128 and c["split_k"] == 1
    assert c["grid_ctas"] == 128 and c["stages"] == 6
    assert spmm24.select_config(4096, 1024, 4096)["tile_n"] == 256  # 64 narrow tiles would not fit one wave
    assert spmm24.select_config(4096, 256, 4096)["cta_pair"] == 0  # N <= 256: split-K cluster tiles
    # 32 pair tiles (0.4 waves) and 86 stages: two pairs per tile, each with half of K
    c = spmm24.select_config(4096, 512, 11008)
    assert c["cta_pair"] == 1 and c["split_k"] == 2 and c["grid_ctas"] == 128
    assert spmm24.select_config(8192, 256, 28672)["split_k"] == 2
    assert spmm24.select_config(11008, 512, 4096)["split_k"] == 1   # 86 tiles: more than half a wave
    # two M halves per pair (512 x 240) when its waves of pairs cost less
    c = spmm24.select_config(4096, 4096, 4096)
    assert (c["tile_m"], c["tile_n"], c["stages"], c["grid_ctas"]) == (512, 240, 3, 2 * 8 * 18)
    assert spmm24.select_config(11008, 512, 4096)["tile_m"] == 512    # 1 wave against 2
    assert spmm24.select_config(4096, 512, 4096)["tile_m"] == 256     # 1 wave either way
    assert spmm24.select_config(2048, 2048, 2048)["tile_m"] == 256
    # one pair tile across N and pairs for < 3/4 of the SMs: split-K clusters (split <= 4)
    c = spmm24.select_config(1024, 256, 8192)
    assert (c["cta_pair"], c["tile_n"], c["split_k"]) == (0, 128, 4)
    assert spmm24.select_config(3584, 256, 8192)["split_k"] == 2
    assert spmm24.select_config(8192, 256, 8192)["cta_pair"] == 1     # 128 pair CTAs: stays
    assert spmm24.select_config(4096, 512, 4160)["cta_pair"] == 0  # K % 128 != 0
    assert spmm24.select_config(4096, 512, 4096, 2)["cta_pair"] == 0  # explicit split-K
    # explicit split honoured, clamped to the number of 128-K stages
    assert spmm24.select_config(256, 128, 256, 8)["split_k"] == 2
    assert spmm24.select_config(256, 16, 4096)["stages"] == 4
    assert spmm24.select_config(256, 128, 4096, 5)["split_k"] == 5
    assert spmm24.select_config(256, 128, 4096, 12)["split_k"] == 8
    assert spmm24.select_config(4096, 1, 4096)["tile_n"] == 16
    for n, t in ((17, 32), (64, 64), (65, 128), (128, 128), (4096, 256)):
        assert spmm24.select_config(1024, n, 1024, 1)["tile_n"] == t
    with pytest.raises(ValueError):
        spmm24.select_config(100, 16, 256)


def test_tuning_overrides_and_no_environment(monkeypatch):
    """spmm24_set_tuning steers the picker; out-of-range fields are refused;
    reset restores the automatic choice; environment variables of the old
    tuning knobs have no effect."""
    try:
        spmm24.set_tuning(pair=1)
        assert spmm24.select_config(384, 40, 512)["cta_pair"] == 1
        spmm24.set_tuning(pair=0, tile_n=256)
        c = spmm24.select_config(256, 256, 1024)
        assert c["cta_pair"] == 0 and c["tile_n"] == 256
        spmm24.set_tuning(pair2=1)
        assert spmm24.select_config(1024, 480, 512)["tile_m"] == 512
        spmm24.set_tuning(pair=1, pair2=0, pair_split=2)
        assert spmm24.select_config(1024, 512, 4096)["split_k"] == 2
        spmm24.set_tuning(deep_ring=1)
        assert spmm24.select_config(4096, 16, 4096)["stages"] == 8
        for bad in ({"pair": 2}, {"pair2": -2}, {"pair_split": 3}, {"tile_n": 48}, {"deep_ring": 2},
                    {"group_split": 3}, {"group_split": 5}):
            with pytest.raises(ValueError, match="out of range"):
                spmm24.set_tuning(**bad)
    finally:
        spmm24.reset_tuning()
    auto = spmm24.select_config(384, 40, 512)
    assert auto["cta_pair"] == 0
    for name, val in (("SPMM24_PAIR", "1"), ("SPMM24_TILE_N", "256"), ("SPMM24_STAGES", "8"), ("SPMM24_PATH", "2")):
        monkeypatch.setenv(name, val)
    assert spmm24.select_config(384, 40, 512) == auto
    assert spmm24.select_config(4096, 16, 4096)["stages"] == 4


def test_grouped_argument_checks():
    """spmm24_launch_grouped rejects bad groups before touching the device."""
    ok = 1 << 20
    good = (ok, ok, ok, ok, 256, 16, 512)
    cases = [
        ([], "count must be 1..16"),
        ([good] * 17, "count must be 1..16"),
        ([(ok, ok, ok, ok, 256, 33, 512)], "N must be <= 32"),
        ([(ok, ok, ok, ok, 250, 16, 512)], "multiple of 16"),
        ([(ok, ok, ok, ok, 256, 16, 500)], "multiple of 64"),
        ([(ok + 8, ok, ok, ok, 256, 16, 512)], "16-byte aligned"),
        ([(ok, ok, ok, ok + 1, 256, 16, 512)], "2-byte aligned"),
        ([(0, ok, ok, ok, 256, 16, 512)], "null pointer"),
        ([(ok, ok, ok, ok, 0, 16, 512)], "positive"),
        ([(ok, ok, ok, ok, 131072, 8, 64)] * 3, "2048 128-row tiles"),
    ]
    for probs, msg in cases:
        arr = spmm24.problem_array(probs) if probs else (spmm24.Problem * 1)()
        rc = spmm24._lib.spmm24_launch_grouped(None, arr, len(probs), 0)
        assert rc == spmm24.CUDA_ERROR_INVALID_VALUE, msg
        assert msg in spmm24._lib.spmm24_last_error().decode(), (msg, spmm24._lib.spmm24_last_error())
    rc = spmm24._lib.spmm24_launch_grouped(None, spmm24.problem_array([good]), 1, 64)
    assert rc == spmm24.CUDA_ERROR_INVALID_VALUE and "flag" in spmm24._lib.spmm24_last_error().decode()
    assert spmm24._lib.spmm24_launch_grouped(None, None, 1, 0) == spmm24.CUDA_ERROR_INVALID_VALUE
