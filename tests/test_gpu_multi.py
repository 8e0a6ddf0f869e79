"""The fused SpMM + all-gather across two GPUs (spmm24_launch_gather +
spmm24_gather_barrier over CUDA IPC peer buffers), run as two processes, one
per GPU.  Skipped where fewer than two GPUs are visible.  Each rank's full C
must equal, bit for bit, the shards every rank computes locally with the
plain launch."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shapes):
    import sys
    from datetime import timedelta

    sys.path.insert(0, os.path.join(REPO, "cuda-repo_b200"))
    import torch
    import torch.distributed as dist

    import spmm24

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    flags = torch.zeros(world, dtype=torch.int32, device=dev)
    epoch = 0
    for (M, N, K, split) in shapes:
        rng = np.random.default_rng(M + N + K)   # same weights and activations on every rank
        a = rng.standard_normal((M, K)).astype(np.float16).view(np.uint16)
        vals, meta = spmm24.compress_reordered(spmm24.prune_2of4(a, M, K), M, K)
        b = rng.uniform(-1, 1, (K, N)).astype(np.float16).view(np.uint16)
        bp = torch.from_numpy(spmm24.pack_b(b, K, N).view(np.int16)).to(dev)
        A = torch.from_numpy(vals.view(np.int16)).to(dev)
        E = torch.from_numpy(meta.view(np.int16)).to(dev)
        # expected: every shard with the plain launch, on this GPU
        expect = torch.empty((M, N), dtype=torch.float16, device=dev)
        rows = [spmm24.shard_rows(M, world, r, 128) for r in range(world)]
        for (r0, r1) in rows:
            Av, Ev = spmm24.shard_views(A, E, M, K, r0, r1)
            assert spmm24.launch(None, Av, bp, Ev, expect[r0:r1], r1 - r0, N, K, None, split) == 0
        # the gathered C: this rank's buffer + the peers' through IPC
        c_full = torch.full((M, N), float("nan"), dtype=torch.float16, device=dev)
        torch.cuda.synchronize(dev)
        handles = [None] * world
        dist.all_gather_object(handles, (spmm24.ipc_export(c_full), spmm24.ipc_export(flags)))
        peers_c, peers_f = [], []
        for r in range(world):
            if r == rank:
                peers_c.append(c_full.data_ptr())
                peers_f.append(flags.data_ptr())
            else:
                peers_c.append(spmm24.ipc_import(handles[r][0]))
                peers_f.append(spmm24.ipc_import(handles[r][1]))
        dist.barrier()
        r0, r1 = rows[rank]
        Av, Ev = spmm24.shard_views(A, E, M, K, r0, r1)
        epoch += 1
        s = torch.cuda.current_stream(dev)
        assert spmm24.launch_gather(s, Av, bp, Ev, r1 - r0, N, K, peers_c, r0, M, split, spmm24.STATIC_WEIGHTS) == 0, \
            spmm24._lib.spmm24_last_error().decode()
        assert spmm24.gather_barrier(s, peers_f, rank, epoch) == 0
        torch.cuda.synchronize(dev)
        assert spmm24.device_status(rank) == 0
        assert torch.equal(c_full, expect), (rank, M, N, K)
        dist.barrier()  # every rank is done with the peers' buffers before they go away
        for r in range(world):
            if r != rank:
                spmm24.ipc_close(peers_c[r])
                spmm24.ipc_close(peers_f[r])
        dist.barrier()
    dist.destroy_process_group()


def test_fused_allgather_two_gpus():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    if not torch.cuda.can_device_access_peer(0, 1):
        pytest.skip("no peer access between GPU 0 and GPU 1")
    # decode (cluster kernel, split-K 4 and auto), mid N, prefill (pair kernel, with and without
    # the K split), ragged N
    shapes = [(1024, 16, 1024, 4), (2048, 32, 2048, 0), (1024, 64, 512, 0), (1024, 512, 1024, 0), (512, 40, 512, 0),
              (1024, 512, 6144, 0)]   # the last: pair kernel with a K split
    mp.spawn(_worker, args=(2, _free_port(), shapes), nprocs=2, join=True)


def _worker_multicast(rank, world, port, shapes, result_dir):
    import sys
    from datetime import timedelta

    sys.path.insert(0, os.path.join(REPO, "cuda-repo_b200"))
    import torch
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem

    import spmm24

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    group = dist.group.WORLD
    flags = symm_mem.empty((world,), dtype=torch.int32, device=dev)
    flags.zero_()
    fh = symm_mem.rendezvous(flags, group)
    flag_ptrs = [fh.buffer_ptrs[r] + (flags.data_ptr() - fh.buffer_ptrs[rank]) for r in range(world)]
    epoch = 0
    supported = True
    for (M, N, K, split) in shapes:
        rng = np.random.default_rng(M + N + K)
        a = rng.standard_normal((M, K)).astype(np.float16).view(np.uint16)
        vals, meta = spmm24.compress_reordered(spmm24.prune_2of4(a, M, K), M, K)
        b = rng.uniform(-1, 1, (K, N)).astype(np.float16).view(np.uint16)
        bp = torch.from_numpy(spmm24.pack_b(b, K, N).view(np.int16)).to(dev)
        A = torch.from_numpy(vals.view(np.int16)).to(dev)
        E = torch.from_numpy(meta.view(np.int16)).to(dev)
        expect = torch.empty((M, N), dtype=torch.float16, device=dev)
        rows = [spmm24.shard_rows(M, world, r, 128) for r in range(world)]
        for (r0, r1) in rows:
            Av, Ev = spmm24.shard_views(A, E, M, K, r0, r1)
            assert spmm24.launch(None, Av, bp, Ev, expect[r0:r1], r1 - r0, N, K, None, split) == 0
        c_full = symm_mem.empty((M, N), dtype=torch.float16, device=dev)
        c_full.fill_(float("nan"))
        h = symm_mem.rendezvous(c_full, group)
        if not h.multicast_ptr:  # no multicast object behind this buffer
            supported = False
            break
        off = c_full.data_ptr() - h.buffer_ptrs[rank]
        ptrs = [h.buffer_ptrs[r] + off for r in range(world)]
        mc = h.multicast_ptr + off
        torch.cuda.synchronize(dev)
        dist.barrier()
        r0, r1 = rows[rank]
        Av, Ev = spmm24.shard_views(A, E, M, K, r0, r1)
        epoch += 1
        s = torch.cuda.current_stream(dev)
        assert spmm24.launch_gather(s, Av, bp, Ev, r1 - r0, N, K, ptrs, r0, M, split, spmm24.STATIC_WEIGHTS,
                                    c_multicast=mc) == 0, spmm24._lib.spmm24_last_error().decode()
        assert spmm24.gather_barrier(s, flag_ptrs, rank, epoch) == 0
        torch.cuda.synchronize(dev)
        assert spmm24.device_status(rank) == 0
        assert torch.equal(c_full, expect), (rank, M, N, K)
        dist.barrier()
    with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
        f.write("ok" if supported else "unsupported")
    dist.barrier()
    dist.destroy_process_group()


def test_fused_allgather_multicast_two_gpus(tmp_path):
    """The same gather with each output chunk stored once through the full
    C's NVLink multicast address (multimem.st; a symmetric-memory buffer
    bound to both GPUs)."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    shapes = [(1024, 16, 1024, 4), (2048, 32, 2048, 0), (1024, 512, 1024, 0), (1024, 512, 6144, 0)]
    mp.spawn(_worker_multicast, args=(2, _free_port(), shapes, str(tmp_path)), nprocs=2, join=True)
    results = {(tmp_path / f"rank{r}").read_text() for r in range(2)}
    if results == {"unsupported"}:
        pytest.skip("no NVLink multicast between GPU 0 and GPU 1")
    assert results == {"ok"}


def _worker_grouped(rank, world, port, shapes):
    """Several M-sharded layers in one spmm24_launch_grouped whose epilogue
    gathers every layer's rows into every rank's full C, then one barrier."""
    import sys
    from datetime import timedelta

    sys.path.insert(0, os.path.join(REPO, "cuda-repo_b200"))
    import torch
    import torch.distributed as dist

    import spmm24

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    layers, expects, fulls = [], [], []
    for (M, N, K) in shapes:
        rng = np.random.default_rng(M + N + K)   # same weights and activations on every rank
        a = (rng.standard_normal((M, K)) * 0.05).astype(np.float16).view(np.uint16)
        vals, meta = spmm24.compress_reordered(spmm24.prune_2of4(a, M, K), M, K)
        b = rng.standard_normal((K, N)).astype(np.float16).view(np.uint16)
        bp = torch.from_numpy(spmm24.pack_b(b, K, N).view(np.int16)).to(dev)
        A = torch.from_numpy(vals.view(np.int16)).to(dev)
        E = torch.from_numpy(meta.view(np.int16)).to(dev)
        layers.append((M, N, K, A, E, bp))
        expects.append(torch.empty((M, N), dtype=torch.float16, device=dev))
        fulls.append(torch.full((M, N), float("nan"), dtype=torch.float16, device=dev))
    # expected: every rank's shards of every layer, one grouped launch on this
    # GPU, with whole tiles (as the gathered launches below, whose fewer tiles
    # would otherwise get another K split from the picker and other sums)
    spmm24.set_tuning(group_split=1)
    local = []
    for (M, N, K, A, E, bp), ex in zip(layers, expects):
        for r in range(world):
            r0, r1 = spmm24.shard_rows(M, world, r, 128)
            Av, Ev = spmm24.shard_views(A, E, M, K, r0, r1)
            local.append((Av, bp, Ev, ex[r0:r1], r1 - r0, N, K))
    assert spmm24.launch_grouped(None, local) == 0, spmm24._lib.spmm24_last_error().decode()
    flags = torch.zeros(world + 1, dtype=torch.int32, device=dev)  # + the fused barrier's CTA counter
    torch.cuda.synchronize(dev)
    handles = [None] * world
    dist.all_gather_object(handles, [spmm24.ipc_export(f) for f in fulls] + [spmm24.ipc_export(flags)])
    ptrs = [[None] * world for _ in range(len(fulls) + 1)]
    opened = []
    for r in range(world):
        for i in range(len(fulls) + 1):
            if r == rank:
                ptrs[i][r] = (fulls[i] if i < len(fulls) else flags).data_ptr()
            else:
                ptrs[i][r] = spmm24.ipc_import(handles[r][i])
                opened.append(ptrs[i][r])
    dist.barrier()
    probs = []
    for i, (M, N, K, A, E, bp) in enumerate(layers):
        r0, r1 = spmm24.shard_rows(M, world, rank, 128)
        Av, Ev = spmm24.shard_views(A, E, M, K, r0, r1)
        probs.append((Av, bp, Ev, None, r1 - r0, N, K, spmm24.make_gather(ptrs[i], r0, M)))
    s = torch.cuda.current_stream(dev)
    arr = spmm24.problem_array(probs)
    # an explicit epoch, then the barrier's automatic one (0: the next after
    # the last), then the same step captured in a CUDA graph, replayed twice
    for epoch in (1, 0):
        for f in fulls:
            f.fill_(float("nan"))
        torch.cuda.synchronize(dev)
        dist.barrier()
        assert spmm24.launch_grouped(s, arr, spmm24.STATIC_WEIGHTS) == 0, spmm24._lib.spmm24_last_error().decode()
        assert spmm24.gather_barrier(s, ptrs[-1], rank, epoch) == 0
        torch.cuda.synchronize(dev)
        assert spmm24.device_status(rank) == 0
        for i, (f, ex) in enumerate(zip(fulls, expects)):
            assert torch.equal(f, ex), (rank, epoch, shapes[i])
        dist.barrier()
    gs = torch.cuda.Stream(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(gs):
        with torch.cuda.graph(graph, stream=gs):
            assert spmm24.launch_grouped(gs, arr, spmm24.STATIC_WEIGHTS) == 0
            assert spmm24.gather_barrier(gs, ptrs[-1], rank, 0) == 0
    for rep in range(2):
        for f in fulls:
            f.fill_(float("nan"))
        torch.cuda.synchronize(dev)
        dist.barrier()
        graph.replay()
        torch.cuda.synchronize(dev)
        assert spmm24.device_status(rank) == 0
        for i, (f, ex) in enumerate(zip(fulls, expects)):
            assert torch.equal(f, ex), (rank, "graph", rep, shapes[i])
        dist.barrier()
    del graph
    # the same with each tile's K split over a cluster of 2 or 4 CTAs (the
    # modes a rank with fewer tiles than SMs gets: 4 and 8 GPUs on the decode
    # step)
    for gsplit in (2, 4):
        spmm24.set_tuning(group_split=gsplit)
        try:
            arr2 = spmm24.problem_array(probs)
            for f in fulls:
                f.fill_(float("nan"))
            torch.cuda.synchronize(dev)
            dist.barrier()
            assert spmm24.launch_grouped(s, arr2, spmm24.STATIC_WEIGHTS) == 0, \
                spmm24._lib.spmm24_last_error().decode()
            assert spmm24.gather_barrier(s, ptrs[-1], rank, 0) == 0
            torch.cuda.synchronize(dev)
            assert spmm24.device_status(rank) == 0
            # expected with the split: every shard again, K in gsplit shares
            for (M, N, K, A, E, bp), ex, f in zip(layers, expects, fulls):
                ex2 = torch.empty_like(ex)
                for r in range(world):
                    r0, r1 = spmm24.shard_rows(M, world, r, 128)
                    Av, Ev = spmm24.shard_views(A, E, M, K, r0, r1)
                    assert spmm24.launch(None, Av, bp, Ev, ex2[r0:r1], r1 - r0, N, K, None, gsplit) == 0
                torch.cuda.synchronize(dev)
                assert torch.equal(f, ex2), (rank, "split", gsplit, M, N, K)
            dist.barrier()
        finally:
            spmm24.set_tuning(group_split=1)
    # the barrier folded into the grouped kernel (spmm24_launch_grouped_gather),
    # on the same flag arrays, eagerly twice and then replayed from a graph
    bar = spmm24.group_barrier(ptrs[-1], rank)
    for rep in range(2):
        for f in fulls:
            f.fill_(float("nan"))
        torch.cuda.synchronize(dev)
        dist.barrier()
        assert spmm24.launch_grouped_gather(s, arr, bar, spmm24.STATIC_WEIGHTS) == 0, \
            spmm24._lib.spmm24_last_error().decode()
        torch.cuda.synchronize(dev)
        assert spmm24.device_status(rank) == 0
        for i, (f, ex) in enumerate(zip(fulls, expects)):
            assert torch.equal(f, ex), (rank, "fused barrier", rep, shapes[i])
        dist.barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(gs):
        with torch.cuda.graph(graph, stream=gs):
            assert spmm24.launch_grouped_gather(gs, arr, bar, spmm24.STATIC_WEIGHTS) == 0
    for rep in range(2):
        for f in fulls:
            f.fill_(float("nan"))
        torch.cuda.synchronize(dev)
        dist.barrier()
        graph.replay()
        torch.cuda.synchronize(dev)
        assert spmm24.device_status(rank) == 0
        for i, (f, ex) in enumerate(zip(fulls, expects)):
            assert torch.equal(f, ex), (rank, "fused barrier graph", rep, shapes[i])
        dist.barrier()
    del graph
    spmm24.reset_tuning()
    for p in opened:
        spmm24.ipc_close(p)
    dist.barrier()
    dist.destroy_process_group()


def test_grouped_allgather_two_gpus():
    """spmm24_launch_grouped with a gather descriptor per layer: each rank's
    full C of every layer equals, bit for bit, all shards computed locally by
    one grouped launch (ragged shards, N = 1 .. 32)."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    if not torch.cuda.can_device_access_peer(0, 1):
        pytest.skip("no peer access between GPU 0 and GPU 1")
    shapes = [(1024, 16, 1024), (2048, 8, 512), (512, 1, 256), (768, 24, 704), (640, 32, 512), (4096, 32, 4096)]
    mp.spawn(_worker_grouped, args=(2, _free_port(), shapes), nprocs=2, join=True)
