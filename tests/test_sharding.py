"""M-sharding of a layer across devices: the row partition (spmm24_shard_rows),
the contiguous shard views of the packed formats, and the multi-rank path
(2 gloo ranks on the CPU: each computes its shard with the oracle from the
shard views alone, then the C shards are all-gathered and compared with the
unsharded result)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
import spmm24
from problems import make_problem


@pytest.mark.parametrize("M", [16, 128, 4096, 4112, 8192, 28672])
@pytest.mark.parametrize("parts", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("align", [16, 128, 256])
def test_shard_rows_partition(M, parts, align):
    ranges = [spmm24.shard_rows(M, parts, i, align) for i in range(parts)]
    assert ranges[0][0] == 0 and ranges[-1][1] == M
    for (b0, e0), (b1, e1) in zip(ranges, ranges[1:]):
        assert e0 == b1
    for b, e in ranges:
        assert b <= e and (b % align == 0 or b == M) and (e % align == 0 or e == M)
    sizes = [e - b for b, e in ranges]
    assert max(sizes) - min(sizes) <= align


def test_shard_rows_rejects_bad_arguments():
    for args in [(100, 2, 0, 128), (128, 0, 0, 128), (128, 2, 2, 128), (128, 2, 0, 24)]:
        with pytest.raises(ValueError):
            spmm24.shard_rows(*args)


def test_shard_views_are_the_rows_of_the_shard():
    M, N, K = 256, 16, 256
    p = make_problem(M, N, K, seed=5)
    r0, r1 = 128, 256
    a, e = spmm24.shard_views(p.vals, p.meta, M, K, r0, r1)
    sub = p.a_dense.reshape(M, K)[r0:r1].reshape(-1)
    n, v2, raw2 = O.compress_a(sub, r1 - r0, K)
    assert np.array_equal(a, v2)
    assert np.array_equal(e, O.reorder_metadata(raw2, r1 - r0, K))


def _rank_main(rank, world, port, M, N, K, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p = make_problem(M, N, K, seed=11)
        r0, r1 = spmm24.shard_rows(M, world, rank, 128)
        a, e = spmm24.shard_views(p.vals, p.meta, M, K, r0, r1)
        c = O.spmm_from_abi_f32(np.ascontiguousarray(a), np.ascontiguousarray(e), p.b_packed, r1 - r0, N, K)
        shard = torch.from_numpy(c.reshape(r1 - r0, N))
        full = torch.empty((M, N), dtype=torch.float32)
        dist.all_gather_into_tensor(full, shard)
        if rank == 0:
            ref = O.dense_gemm_f32(p.a_dense, p.b_rowmajor, M, N, K).reshape(M, N)
            out.put(bool(np.array_equal(full.numpy().view(np.uint32), ref.view(np.uint32))))
    finally:
        dist.destroy_process_group()


def test_two_rank_m_sharding_gloo():
    """Rows computed per rank from the shard views, gathered with an all-gather,
    equal the unsharded result bit for bit (same fp32 order per row)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    M, N, K = 512, 16, 256
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, M, N, K, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=120)
    assert all(pr.exitcode == 0 for pr in procs)
    assert q.get(timeout=5) is True
