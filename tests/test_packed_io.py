"""Packed-weight files (spmm24_save_packed / spmm24_load_packed): round trip
of the exact bytes spmm24_launch consumes, and every corruption detected."""
import numpy as np
import pytest

import spmm24


def _packed(M, K, seed):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K)).astype(np.float16).view(np.uint16)
    return spmm24.compress_reordered(spmm24.prune_2of4(a, M, K), M, K)


@pytest.mark.parametrize("M,K,bf16", [(16, 64, False), (256, 512, True), (4096, 1024, False)])
def test_round_trip(tmp_path, M, K, bf16):
    v, m = _packed(M, K, M + K)
    p = tmp_path / "w.spmm24"
    spmm24.save_packed(str(p), v, m, M, K, bf16=bf16)
    assert p.stat().st_size == 64 + M * K + M * K // 8
    v2, m2, M2, K2, b2 = spmm24.load_packed(str(p))
    assert (M2, K2, b2) == (M, K, bf16)
    assert np.array_equal(v, v2) and np.array_equal(m, m2)


def test_corruption_is_detected(tmp_path):
    M, K = 64, 256
    v, m = _packed(M, K, 1)
    p = tmp_path / "w.spmm24"
    spmm24.save_packed(str(p), v, m, M, K)
    raw = bytearray(p.read_bytes())
    cases = {
        "payload": (lambda b: b.__setitem__(200, b[200] ^ 0x10), "checksum"),
        "magic": (lambda b: b.__setitem__(0, ord("X")), "not a packed-weight file"),
        "version": (lambda b: b.__setitem__(8, 2), "not a packed-weight file"),
        "size": (lambda b: b.__setitem__(16, 17), "not a packed-weight file"),   # M not a multiple of 16
    }
    for name, (mutate, msg) in cases.items():
        b = bytearray(raw)
        mutate(b)
        q = tmp_path / f"{name}.spmm24"
        q.write_bytes(bytes(b))
        with pytest.raises(OSError, match=msg):
            spmm24.load_packed(str(q))
    q = tmp_path / "short.spmm24"
    q.write_bytes(bytes(raw[:-1]))
    with pytest.raises(OSError, match="short file"):
        spmm24.load_packed(str(q))
    q = tmp_path / "long.spmm24"
    q.write_bytes(bytes(raw) + b"\0")
    with pytest.raises(OSError, match="not a packed-weight file"):
        spmm24.load_packed(str(q))
    with pytest.raises(OSError):
        spmm24.load_packed(str(tmp_path / "missing.spmm24"))


def test_bad_arguments():
    assert spmm24._lib.spmm24_save_packed(b"/dev/null", 0, 250, 64, 1, 1) == -1   # M % 16
    assert spmm24._lib.spmm24_save_packed(b"/dev/null", 4, 256, 128, 1, 1) == -1  # dtype
    assert spmm24._lib.spmm24_save_packed(b"/dev/null", 2, 256, 64, 1, 1) == -1   # fp8 needs K % 128
    assert spmm24._lib.spmm24_save_packed(b"/dev/null", 0, 256, 64, None, 1) == -1


@pytest.mark.parametrize("fmt", [0, 1], ids=["e4m3", "e5m2"])
def test_fp8_round_trip(tmp_path, fmt):
    """dtype 2 / 3: the fp8 SpMM's values (M*K/2 bytes) and metadata (M*K/8)."""
    M, K = 128, 512
    rng = np.random.default_rng(fmt)
    a = rng.integers(0, 256, M * K, dtype=np.uint8)
    a[(a & 0x7F) == 0x7F] = 0x38
    v, m = spmm24.compress_a_fp8(spmm24.prune_2of4_fp8(a, M, K, fmt), M, K)
    p = tmp_path / "w8.spmm24"
    spmm24.save_packed_fp8(str(p), v, m, M, K, fmt)
    assert p.stat().st_size == 64 + M * K // 2 + M * K // 8
    v2, m2, M2, K2, f2 = spmm24.load_packed_fp8(str(p))
    assert (M2, K2, f2) == (M, K, fmt)
    assert np.array_equal(v, v2) and np.array_equal(m, m2)
    with pytest.raises(ValueError):
        spmm24.load_packed(str(p))
    raw = bytearray(p.read_bytes())
    raw[100] ^= 1
    p.write_bytes(bytes(raw))
    with pytest.raises(OSError, match="checksum"):
        spmm24.load_packed_fp8(str(p))


def test_file_replaced_after_header_read(tmp_path):
    """The buffers are sized from the header; if the file is replaced by a
    larger one before the payload is read, spmm24_load_packed reads nothing
    and reports the capacity error instead of writing past the buffers."""
    import ctypes

    v, m = _packed(64, 256, 2)
    p = tmp_path / "w.spmm24"
    spmm24.save_packed(str(p), v, m, 64, 256)
    h = spmm24.PackedHeader()
    assert spmm24._lib.spmm24_load_packed_header(bytes(p), ctypes.byref(h)) == 0
    # guard bytes after each buffer: they must stay untouched
    guard = 4096
    vbuf = np.full(h.values_bytes + guard, 0xA5, dtype=np.uint8)
    mbuf = np.full(h.meta_bytes + guard, 0x5A, dtype=np.uint8)
    v2, m2 = _packed(128, 256, 3)                       # the replacement: twice the rows
    spmm24.save_packed(str(p), v2, m2, 128, 256)
    rc = spmm24._lib.spmm24_load_packed(bytes(p), vbuf.ctypes.data, h.values_bytes, mbuf.ctypes.data, h.meta_bytes)
    assert rc == -5
    assert np.all(vbuf == 0xA5) and np.all(mbuf == 0x5A)
    # with capacities that fit the new file the load succeeds
    vb = np.empty(128 * 256, dtype=np.uint8)
    mb = np.empty(128 * 256 // 8, dtype=np.uint8)
    assert spmm24._lib.spmm24_load_packed(bytes(p), vb.ctypes.data, vb.nbytes, mb.ctypes.data, mb.nbytes) == 0
    assert np.array_equal(vb.view(np.uint16), v2) and np.array_equal(mb.view(np.uint16), m2)
