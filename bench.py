#!/usr/bin/env python3
"""Benchmark of the sm_100a 2:4 SpMM library on its headline workload.

Workload (LLaMA-7B decode linear layers): one step runs
the 12 SpMMs (M,K) in {(4096,4096), (11008,4096), (4096,11008)} x N in
{1, 8, 16, 32}.  A is fp16 N(0, 0.02) magnitude-pruned 2:4 along K, B is
fp16 N(0, 1) (synthetic, seeded).  Every call in a step reads its own copy
of the weights (481 MB of A + metadata in total, about 4x the 126 MB L2),
so no call finds its operands in L2.

Metric: dense-equivalent TFLOPS (2*M*N*K per SpMM) of the whole job, plus
microseconds per SpMM and the fraction of the HBM roofline (algorithmic
bytes = M*K + M*K/8 + 2*K*N + 2*M*N per call, against the measured copy
bandwidth in MEASURED_PEAKS.json).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload decode|prefill|70b|square|pack|packb] [--launch grouped|chain]
                  [--no-comparators] [--no-secondary] [--no-config4] [--no-extras] [--gather-mc]

A step of the decode workload is one spmm24_launch_grouped (one persistent
kernel for all 12 SpMMs); the same steps as one spmm24_launch per SpMM are
timed beside it ("chain").  At N=1 the line also carries same-run
comparators (cuSPARSELt 0.7.1 with algorithm search, dense cuBLAS fp16, the
reference kernel built for sm_100a; isolated calls, L2 flushed) and a
secondary block with BASELINE configs 3 (prefill) and 5 (squares up to
16384^3) against the sparse tensor-core ceiling measured in the same run,
the M-sharded LLaMA-70B block (config 4), and an extras block (fp8 decode,
a fused epilogue, the device packers; each a child run of this script).

--impl reference times the reference path's CPU implementation (the
oracle's dense GEMM on the pruned A -- the reference has no CPU GEMM of its
own) on the host cores, on a bounded row sample of the same workload.
Under torchrun (N > 1) the decode layers are split along M across the ranks
(strong scaling): each step is one grouped launch per rank whose epilogue
stores every output row into every rank's full C over NVLink and whose last
CTA runs the cross-GPU barrier; time is the max over ranks; rank 0 prints
one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "cuda-repo_b200"))

WORKLOADS = {
    # BASELINE config 2 (the headline): LLaMA-7B decode; on N > 1 GPUs every
    # layer is split along M across the ranks and the outputs are all-gathered
    # inside the step (strong scaling)
    "decode": {"shapes": [(M, N, K) for (M, K) in ((4096, 4096), (11008, 4096), (4096, 11008)) for N in (1, 8, 16, 32)],
               "a_std": 0.02, "bound": "hbm", "shard": True},
    # LLaMA-7B prefill
    "prefill": {"shapes": [(M, N, K) for (M, K) in ((4096, 4096), (11008, 4096), (4096, 11008)) for N in (512, 2048, 4096)],
                "a_std": 0.02, "bound": "tensor"},
    # LLaMA-70B layers, each layer split along M across the
    # ranks (strong scaling; no reduction; optional all-gather of C)
    "70b": {"shapes": [(M, N, K) for (M, K) in ((8192, 8192), (28672, 8192), (8192, 28672)) for N in (16, 256, 4096)],
            "a_std": 0.01, "bound": "tensor", "shard": True},
    # square sweep (up to 8192)
    "square": {"shapes": [(s, s, s) for s in (1024, 2048, 4096, 8192)], "a_std": None, "bound": "tensor"},
}


# --workload pack: the on-device packer over the LLaMA-7B layer weights of
# config 2 (dense fp16 N(0, 0.02), magnitude-pruned and compressed in one
# kernel per layer).
PACK_LAYERS = [(4096, 4096), (11008, 4096), (4096, 11008)]
# Activations K x N of BASELINE config 3 (prefill): what spmm24_pack_b_device
# turns into the packed B of the next SpMM.
PACKB_ACTS = [(K, N) for K in (4096, 11008) for N in (512, 2048, 4096)]


def packb_bytes(K, N):
    """Algorithmic bytes of one B packing: read 2KN, write the packed strips."""
    return 2 * K * N + 2 * K * ((N + 7) // 8) * 8


def pack_bytes(M, K, fp8=False):
    """Algorithmic bytes of one spmm24_pack_a_device call: the dense fp16
    read, the compressed values and the metadata written (fp8: the dense
    bytes, M*K/2 values, M*K/8 metadata)."""
    if fp8:
        return M * K + M * K // 2 + M * K // 8
    return 2 * M * K + M * K + M * K // 8


def algo_bytes(M, N, K, fp8=False):
    if fp8:  # fp8 values M*K/2, metadata M*K/8, B N*K bytes, fp16 C
        return M * K // 2 + M * K // 8 + K * N + 2 * M * N
    return M * K + M * K // 8 + 2 * K * N + 2 * M * N


def flops(M, N, K):
    return 2.0 * M * N * K


def load_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


def load_traffic(workload):
    """Per-launch DRAM traffic from the committed ncu summary, if present."""
    path = os.path.join(REPO, "profiles", f"spmm24_{workload}_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.25)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path:
            return None
        rows = []
        try:
            for line in open(self.path):
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        finally:
            os.unlink(self.path)
        if not rows:
            return None
        sm = [int(r[1]) for r in rows]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        load = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": int(statistics.median(load)), "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "sm_min_mhz": int(min(load))}


# --------------------------------------------------------------------- data
def make_layer(torch, spmm24, M, K, a_std, seed, mask_random=False, bf16=False):
    """Pruned, compressed weights of one layer, packed by the product's own
    host packer (spmm24_prune_2of4[_bf16] / spmm24_compress_reordered)."""
    g = torch.Generator().manual_seed(seed)
    dt = torch.bfloat16 if bf16 else torch.float16
    if a_std is None:
        a = (torch.rand(M, K, generator=g) * 2 - 1).to(dt)
        if mask_random:
            keep = torch.rand(M * K // 4, 4, generator=g).argsort(dim=1)[:, :2]
            m = torch.zeros(M * K // 4, 4, dtype=torch.bool).scatter_(1, keep, True)
            a = (a.reshape(-1, 4) * m).reshape(M, K).to(dt)
    else:
        a = (torch.randn(M, K, generator=g) * a_std).to(dt)
    a_np = a.view(torch.int16).numpy().view("uint16")
    if a_std is not None or not mask_random:
        a_np = spmm24.prune_2of4_bf16(a_np, M, K) if bf16 else spmm24.prune_2of4(a_np, M, K)
    vals, meta = spmm24.compress_reordered(a_np, M, K)
    return a_np, vals, meta


def make_activations(torch, spmm24, K, N, seed, uniform=False, bf16=False):
    g = torch.Generator().manual_seed(seed)
    dt = torch.bfloat16 if bf16 else torch.float16
    b = ((torch.rand(K, N, generator=g) * 2 - 1) if uniform else torch.randn(K, N, generator=g)).to(dt)
    b_np = b.view(torch.int16).numpy().view("uint16")
    return b_np, spmm24.pack_b(b_np, K, N)


def make_layer_fp8(torch, spmm24, M, K, seed):
    """fp8 (E4M3) weights of one layer: N(0,1) quantised by torch's float8
    cast (the dequantisation scale goes into the epilogue's alpha), pruned
    and compressed by the product's host packer."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).to(torch.float8_e4m3fn).view(torch.uint8).numpy().reshape(-1)
    a = spmm24.prune_2of4_fp8(a, M, K, spmm24.FP8_E4M3)
    vals, meta = spmm24.compress_a_fp8(a, M, K)
    return a, vals, meta


def make_activations_fp8(torch, K, N, seed):
    """fp8 (E4M3) activations, N x K row-major (the fp8 path's B layout)."""
    g = torch.Generator().manual_seed(seed)
    b = torch.randn(N, K, generator=g).to(torch.float8_e4m3fn).view(torch.uint8).numpy().reshape(-1)
    return b, b


def workload_config(args, world):
    """The `config` object of the JSON line, identical in both arms."""
    wl = WORKLOADS[args.workload]
    shapes = wl["shapes"]
    shard = bool(wl.get("shard"))
    fp8 = args.dtype == "fp8"
    wbytes = sum((M * K // 2 if fp8 else M * K) + M * K // 8 for (M, N, K) in shapes)
    return {"workload": f"{args.workload}: " + ", ".join(f"{M}x{N}x{K}" for (M, N, K) in shapes),
            "baseline_config": {"decode": 2, "prefill": 3, "70b": 4, "square": 5}[args.workload],
            "spmm_per_step": len(shapes), "split_k": "auto (library picker)",
            "l2": f"inputs larger than L2: {wbytes / 1e6:.0f} MB of distinct weights per step (whole job)",
            "parallelism": (("M-sharded" if world > 1 else "unsharded") +
                            f" x{world} (rows split by spmm24_shard_rows, no reduction" +
                            ("; outputs all-gathered into every rank's full C inside the step: the grouped kernel's "
                             "epilogue stores over NVLink, its last CTA runs the cross-GPU barrier)"
                             if world > 1 and args.workload == "decode" else ")") if shard
                            else f"replicas x{world} (each rank its own layers)")}


def to_dev(torch, arr, dev):
    if arr.dtype.itemsize == 1:
        return torch.from_numpy(arr.view("uint8")).to(dev)
    return torch.from_numpy(arr.view("int16")).to(dev)


# ------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import ctypes

    import numpy as np
    import torch
    import torch.distributed as dist

    import spmm24

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    wl = WORKLOADS[args.workload]
    shapes = wl["shapes"]
    square = args.workload == "square"
    shard = bool(wl.get("shard"))
    bf16 = args.dtype == "bf16"
    fp8 = args.dtype == "fp8"
    # With sharding every rank holds rows [r0, r1) of each layer (generated
    # for that range directly); otherwise every rank runs whole layers.
    rows = {M: (spmm24.shard_rows(M, world, rank, 128) if shard else (0, M)) for (M, N, K) in shapes}
    layers = {}
    for i, (M, K) in enumerate(sorted({(M, K) for (M, N, K) in shapes})):
        r0, r1 = rows[M]
        if fp8:
            layers[(M, K)] = make_layer_fp8(torch, spmm24, r1 - r0, K, seed=1000 * rank + i)
            continue
        a_np, vals, meta = make_layer(torch, spmm24, r1 - r0, K, wl["a_std"], seed=1000 * rank + i, mask_random=square,
                                      bf16=bf16)
        layers[(M, K)] = (a_np, vals, meta)
    acts = {}
    for j, (K, N) in enumerate(sorted({(K, N) for (M, N, K) in shapes})):
        if fp8:
            acts[(K, N)] = make_activations_fp8(torch, K, N, seed=5000 + (0 if shard else 100 * rank) + j)
            continue
        # sharded layers: every rank holds the same activations
        acts[(K, N)] = make_activations(torch, spmm24, K, N, seed=5000 + (0 if shard else 100 * rank) + j,
                                        uniform=square)

    # Device copies: every call of a step gets its own weights so that the
    # working set of a step exceeds L2.  Activations and outputs of a step are
    # views of two contiguous buffers, so a step's inputs and results move
    # host<->device in one copy each.
    b_sizes = [acts[(K, N)][1].size for (M, N, K) in shapes]
    packed_out = args.epilogue == "packed_b"
    # packed_b: C is written as the next layer's packed B (ceil(N/8) strips of M x 8)
    c_sizes = [(rows[M][1] - rows[M][0]) * (((N + 7) // 8) * 8 if packed_out else N) for (M, N, K) in shapes]
    bdt, bview = (torch.uint8, "uint8") if fp8 else (torch.int16, "int16")
    B_all = torch.empty(sum(b_sizes), dtype=bdt, device=dev)
    C_all = torch.empty(sum(c_sizes), dtype=torch.float16, device=dev)
    host_in = torch.from_numpy(np.concatenate([acts[(K, N)][1].view(bview) for (M, N, K) in shapes])).pin_memory()
    B_all.copy_(host_in)
    calls = []
    boff = coff = 0
    for (M, N, K), bs, cs in zip(shapes, b_sizes, c_sizes):
        _, vals, meta = layers[(M, K)]
        A = to_dev(torch, vals, dev)
        E = to_dev(torch, meta, dev)
        r0, r1 = rows[M]
        B = B_all[boff:boff + bs]
        C = C_all[coff:coff + cs] if packed_out else C_all[coff:coff + cs].view(r1 - r0, N)
        boff += bs
        coff += cs
        calls.append({"M": r1 - r0, "N": N, "K": K, "A": A, "E": E, "B": B, "C": C, "M_full": M,
                      "boff": boff - bs, "coff": coff - cs,
                      "split": (spmm24.select_config_fp8 if fp8 else spmm24.select_config)(max(16, r1 - r0), N, K,
                                                                                          0)["split_k"]})
    weight_bytes = sum(c["A"].numel() * c["A"].element_size() + c["E"].numel() * c["E"].element_size() for c in calls)
    stream = torch.cuda.current_stream(dev)
    h_stream = int(stream.cuda_stream)

    flags = (spmm24.STATIC_WEIGHTS if args.static_weights else 0) | (spmm24.BF16 if bf16 else 0)
    # Optional fused epilogue (spmm24_launch_fused): per-row bias + SiLU, or
    # per-row bias + residual add (the residual is another M x N tensor).
    # fp8: always through spmm24_launch_fp8, alpha = the weights' dequantisation scale.
    fused = args.epilogue != "none" or bf16 or fp8
    if fused:
        import ctypes

        edt = torch.bfloat16 if bf16 else torch.float16
        alpha = float(wl["a_std"] or 1.0) if fp8 else 1.0
        for c in calls:
            c["bias"] = (torch.randn(c["M"], device=dev) * 0.1).to(edt)
            c["res"] = torch.randn(c["M"], c["N"], device=dev).to(edt) if args.epilogue == "bias_residual" else None
            with_bias = args.epilogue in ("bias_silu", "bias_residual")
            c["epi"] = spmm24.Epilogue(c["bias"].data_ptr() if with_bias else None,
                                       c["res"].data_ptr() if c["res"] is not None else None, alpha,
                                       spmm24.ACT_SILU if args.epilogue == "bias_silu" else spmm24.ACT_NONE,
                                       spmm24.OUT_PACKED_B if packed_out else spmm24.OUT_ROW_MAJOR)

    def launch(c, hs=None):
        if fp8:
            rc = spmm24._lib.spmm24_launch_fp8(h_stream if hs is None else hs, c["A"].data_ptr(), c["B"].data_ptr(),
                                               c["E"].data_ptr(), c["C"].data_ptr(), c["M"], c["N"], c["K"], 0,
                                               flags, ctypes.addressof(c["epi"]))
        elif fused:
            rc = spmm24._lib.spmm24_launch_fused(h_stream if hs is None else hs, c["A"].data_ptr(), c["B"].data_ptr(),
                                                 c["E"].data_ptr(), c["C"].data_ptr(), c["M"], c["N"], c["K"], 0,
                                                 flags, ctypes.byref(c["epi"]))
        else:
            rc = spmm24._lib.spmm24_launch_ex(h_stream if hs is None else hs, c["A"].data_ptr(), c["B"].data_ptr(),
                                              c["E"].data_ptr(), c["C"].data_ptr(), c["M"], c["N"], c["K"], 0, flags)
        if rc != 0:
            raise RuntimeError(f"spmm24_launch failed: {rc} {spmm24._lib.spmm24_last_error().decode()}")

    # A step: every SpMM of the workload.  "grouped" issues them as one
    # spmm24_launch_grouped (one persistent kernel for all the step's N <= 32
    # layers); "chain" issues one spmm24_launch per SpMM.
    grouped = args.launch == "grouped" and all(c["N"] <= 32 for c in calls)
    group_flags = flags & (spmm24.STATIC_WEIGHTS | spmm24.BF16)
    group_fn = spmm24._lib.spmm24_launch_grouped_fp8 if fp8 else spmm24._lib.spmm24_launch_grouped
    # M-sharded decode on N > 1 GPUs: every rank's output rows go straight into
    # every rank's full C (the grouped kernel's epilogue stores over NVLink to
    # the peers' buffers, opened with CUDA IPC), then one cross-GPU barrier;
    # both inside the timed step.  Two full-C sets, for the e2e loop's two
    # buffer sets.
    gather_mode = grouped and shard and world > 1 and not (fp8 or bf16) and args.epilogue == "none"
    full_sets, flag_ptrs, imported = [], None, []
    mc_bases, symm_keep = [None, None], []
    if gather_mode:
        full_elems = sum(c["M_full"] * c["N"] for c in calls)
        flag_buf = torch.zeros(world + 1, dtype=torch.int32, device=dev)  # + the fused barrier's CTA counter
        bases = [[None] * world for _ in range(3)]
        if args.gather_mc:
            # --gather-mc: the full-C sets in symmetric memory, so that rows
            # whose N is a multiple of 8 are stored once through the NVLink
            # multicast address (multimem.st, replicated by the switch)
            import torch.distributed._symmetric_memory as symm_mem

            for k in range(2):
                t = symm_mem.empty((full_elems,), dtype=torch.float16, device=dev)
                t.zero_()
                hd = symm_mem.rendezvous(t, dist.group.WORLD)
                moff = t.data_ptr() - hd.buffer_ptrs[rank]
                bases[k] = [hd.buffer_ptrs[r] + moff for r in range(world)]
                mc_bases[k] = hd.multicast_ptr + moff if hd.multicast_ptr else None
                full_sets.append(t)
                symm_keep.append(hd)
        else:
            full_sets = [torch.zeros(full_elems, dtype=torch.float16, device=dev) for _ in range(2)]
        torch.cuda.synchronize(dev)
        ipc_bufs = ([] if args.gather_mc else full_sets) + [flag_buf]
        mine = [spmm24.ipc_export(t) for t in ipc_bufs]
        handles = [None] * world
        dist.all_gather_object(handles, mine)
        slots = [2] if args.gather_mc else [0, 1, 2]
        for r in range(world):
            for j, i in enumerate(slots):
                if r == rank:
                    bases[i][r] = (full_sets[i] if i < 2 else flag_buf).data_ptr()
                else:
                    bases[i][r] = spmm24.ipc_import(handles[r][j])
                    imported.append(bases[i][r])
        flag_ptrs = bases[2]
        group_bar = spmm24.group_barrier(flag_ptrs, rank)
        dist.barrier()

    def gathers_for(k):
        """Gather descriptors of full-C set k, one per call."""
        out_g, off = [], 0
        for c in calls:
            out_g.append(spmm24.make_gather([b + 2 * off for b in bases[k]], rows[c["M_full"]][0], c["M_full"],
                                            c_multicast=(mc_bases[k] + 2 * off) if mc_bases[k] else None))
            off += c["M_full"] * c["N"]
        return out_g

    def group_array(cs, k):
        gs = gathers_for(k) if gather_mode else [None] * len(cs)
        return spmm24.problem_array([(c["A"], c["B"], c["E"], c["C"], c["M"], c["N"], c["K"], g, c.get("epi"))
                                     for c, g in zip(cs, gs)])

    group_arrays = {}

    def step_launch(cs, hs=None, use_group=grouped, k=0):
        hs = h_stream if hs is None else hs
        if use_group and gather_mode:  # one kernel: the SpMMs, the gathered stores, the cross-GPU barrier
            arr = group_arrays.setdefault((id(cs), k), group_array(cs, k))
            rc = spmm24._lib.spmm24_launch_grouped_gather(hs, arr, len(arr), group_flags, ctypes.byref(group_bar))
            if rc != 0:
                raise RuntimeError(f"spmm24_launch_grouped_gather: {rc} {spmm24._lib.spmm24_last_error().decode()}")
            return
        if use_group:
            arr = group_arrays.setdefault((id(cs), k), group_array(cs, k))
            rc = group_fn(hs, arr, len(arr), group_flags)
            if rc != 0:
                raise RuntimeError(f"spmm24_launch_grouped failed: {rc} {spmm24._lib.spmm24_last_error().decode()}")
        elif gather_mode:  # the chain: one spmm24_launch_gather per SpMM
            off = 0
            for c in cs:
                rc = spmm24.launch_gather(hs, c["A"], c["B"], c["E"], c["M"], c["N"], c["K"],
                                          [b + 2 * off for b in bases[k]], rows[c["M_full"]][0], c["M_full"], 0,
                                          flags)
                off += c["M_full"] * c["N"]
                if rc != 0:
                    raise RuntimeError(f"spmm24_launch_gather: {rc} {spmm24._lib.spmm24_last_error().decode()}")
        else:
            for c in cs:
                launch(c, hs)
        if gather_mode:  # epoch 0: the barrier counts on the device, so the step can live in a CUDA graph
            if spmm24.gather_barrier(hs, flag_ptrs, rank, 0) != 0:
                raise RuntimeError("spmm24_gather_barrier failed")

    def timed_steps(use_group):
        """Device time (ms) of args.steps steps back to back.  A sleep kernel
        queued first lets the host enqueue every timed launch before the GPU
        reaches them, so the interval measures the kernels back to back
        (programmatic dependent launch lets each kernel's set-up overlap the
        previous kernel's tail)."""
        for _ in range(args.warmup):
            step_launch(calls, use_group=use_group)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(int(2e7))
        if gather_mode:
            # one untimed step: its cross-GPU barrier lines the ranks up on the
            # device, so no rank's interval holds another's late start
            step_launch(calls, use_group=use_group)
        t0.record(stream)
        for _ in range(args.steps):
            step_launch(calls, use_group=use_group)
        t1.record(stream)
        torch.cuda.synchronize(dev)
        return t0.elapsed_time(t1)

    chain_ms = None
    if grouped:
        chain_ms = timed_steps(False)  # the same steps as one launch per SpMM, for comparison
    nl = (1 if grouped else len(calls) + (1 if gather_mode else 0)) * args.steps  # chain: + the barrier kernel
    with ClockSampler(local_rank) as clk:
        elapsed_ms = timed_steps(grouped)
    clocks = clk.summary()

    # Per-shape kernel times: an event pair around every launch (this breaks
    # the launch overlap, so these are single-kernel durations).
    reps = max(3, min(args.steps, 10))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps * len(calls))]
    torch.cuda.synchronize(dev)
    torch.cuda._sleep(int(2e7))
    i = 0
    for _ in range(reps):
        for c in calls:
            ev[i][0].record(stream)
            launch(c)
            ev[i][1].record(stream)
            i += 1
    torch.cuda.synchronize(dev)
    per_launch_us = [a.elapsed_time(b) * 1e3 for a, b in ev]
    per_call = [statistics.median(per_launch_us[ci::len(calls)]) for ci in range(len(calls))]
    # The same single shapes through the grouped kernel (a group of one).
    per_call_grouped = None
    if grouped and not gather_mode:
        singles = [spmm24.problem_array([(c["A"], c["B"], c["E"], c["C"], c["M"], c["N"], c["K"], None, c.get("epi"))])
                   for c in calls]
        evg = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(reps * len(calls))]
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(int(2e7))
        i = 0
        for _ in range(reps):
            for arr in singles:
                evg[i][0].record(stream)
                group_fn(h_stream, arr, 1, group_flags)
                evg[i][1].record(stream)
                i += 1
        torch.cuda.synchronize(dev)
        us_g = [a.elapsed_time(b) * 1e3 for a, b in evg]
        per_call_grouped = [statistics.median(us_g[ci::len(calls)]) for ci in range(len(calls))]

    # Host time per call: eager launches (no graph), each call's own host
    # work (argument checks, plan, cached TMA descriptors, cudaLaunchKernelEx)
    # less the same ctypes call rejected at its first check (unknown flag),
    # with a sleep kernel ahead so the GPU never drains the launch queue.
    def host_us(fn, bad_fn, n=200):
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(int(1e8))
        t = time.perf_counter()
        for _ in range(n):
            fn()
        full = time.perf_counter() - t
        t = time.perf_counter()
        for _ in range(n):
            bad_fn()
        base = time.perf_counter() - t
        torch.cuda.synchronize(dev)
        return round(max(0.0, full - base) / n * 1e6, 3), round(full / n * 1e6, 3)

    c0 = calls[0]
    host = {}
    if not fp8:
        lx = spmm24._lib.spmm24_launch_ex
        args0 = (c0["A"].data_ptr(), c0["B"].data_ptr(), c0["E"].data_ptr(), c0["C"].data_ptr(), c0["M"], c0["N"],
                 c0["K"], 0)
        net, tot = host_us(lambda: lx(h_stream, *args0, flags), lambda: lx(h_stream, *args0, 1 << 20))
        host["spmm24_launch_ex_us"] = net
        host["spmm24_launch_ex_us_with_ctypes"] = tot
        if grouped and not gather_mode:
            arr_all = group_array(calls, 0)
            lg = group_fn
            net, tot = host_us(lambda: lg(h_stream, arr_all, len(arr_all), group_flags),
                               lambda: lg(h_stream, arr_all, len(arr_all), 1 << 20))
            host["spmm24_launch_grouped_12_us"] = net
            host["spmm24_launch_grouped_12_us_with_ctypes"] = tot
        host["note"] = ("host time per eager call, minus the same ctypes call rejected at its first argument check; "
                        "the kernels' device time per call is in per_shape_us")

    # End to end through the public C ABI with host buffers, as a serving
    # loop runs it: every step uploads all of its packed activations from
    # pinned host memory, runs its launches (a CUDA graph of spmm24 calls)
    # and downloads all of its results into pinned host memory.  Two buffer
    # sets alternate between steps, so step i's upload (its own stream)
    # overlaps step i-1's kernels and step i-1's download (another stream)
    # overlaps step i's; events order every reuse of a buffer.
    # Gather mode: every rank holds the whole C of the step, and rank r
    # downloads the r-th 1/N of it (one copy; together the ranks bring the
    # whole C to the host once).
    out_sets = full_sets if gather_mode else None
    B_set = [B_all, torch.empty_like(B_all)]
    C_set = out_sets if gather_mode else [C_all, torch.empty_like(C_all)]
    if gather_mode:
        ochunk = -(-C_set[0].numel() // world)
        out_src = [C_set[k][rank * ochunk:(rank + 1) * ochunk] for k in range(2)]
    else:
        out_src = C_set
    host_out = [torch.empty(out_src[0].shape, dtype=torch.float16).pin_memory() for _ in range(2)]
    h2d = host_in.numel() * host_in.element_size()
    d2h = host_out[0].numel() * 2
    call_sets = [calls, []]
    for c in calls:
        bs_, cs_ = c["B"].numel(), c["C"].numel()
        c1 = C_set[1][c["coff"]:c["coff"] + cs_]
        call_sets[1].append(dict(c, B=B_set[1][c["boff"]:c["boff"] + bs_],
                                 C=c1 if packed_out else c1.view(c["M"], c["N"])))
    graphs = [None, None]
    try:
        for k in range(2):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                hs = int(torch.cuda.current_stream(dev).cuda_stream)
                step_launch(call_sets[k], hs, k=k)
            graphs[k] = g
    except Exception:  # noqa: BLE001 -- fall back to eager launches
        graphs = [None, None]
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]

    def e2e_step(i):
        k = i % 2
        with torch.cuda.stream(up):
            if used[k]:
                up.wait_event(comp_done[k])  # the kernels of step i-2 have read this input set
            B_set[k].copy_(host_in, non_blocking=True)
            h2d_done[k].record(up)
        stream.wait_event(h2d_done[k])
        if used[k]:
            stream.wait_event(d2h_done[k])  # step i-2's results have left this output set
        if graphs[k] is not None:
            graphs[k].replay()
        else:
            step_launch(call_sets[k], k=k)
        comp_done[k].record(stream)
        with torch.cuda.stream(down):
            down.wait_event(comp_done[k])
            host_out[k].copy_(out_src[k], non_blocking=True)
            d2h_done[k].record(down)
        used[k] = True

    for i in range(max(2, args.warmup)):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    if gather_mode:
        e2e_step(-1)  # untimed: its cross-GPU barrier lines the ranks up on the device
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up.wait_event(e0)
    for i in range(args.steps):
        e2e_step(i)
    for k in range(2):
        stream.wait_event(d2h_done[k])
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    graph = graphs[0]

    if world > 1:
        t = torch.tensor([elapsed_ms, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, e2e_ms = float(t[0]), float(t[1])

    step_flops = sum(flops(c["M"], c["N"], c["K"]) for c in calls)
    if shard:
        # strong scaling: the job is the unsharded layers, whatever the ranks
        total_flops = sum(flops(c["M_full"], c["N"], c["K"]) for c in calls) * args.steps
    else:
        total_flops = step_flops * args.steps * world
    value = total_flops / (elapsed_ms * 1e-3) / 1e12
    e2e_value = total_flops / (e2e_ms * 1e-3) / 1e12

    peaks = load_peaks()
    # Average launch duration over the timed region = elapsed / launches.
    kernel_us_total = elapsed_ms * 1e3
    bytes_total = sum(algo_bytes(c["M"], c["N"], c["K"], fp8) for c in calls) * args.steps
    flops_total_rank = step_flops * args.steps
    if wl["bound"] == "hbm":
        achieved = bytes_total / (kernel_us_total * 1e-6) / 1e9
        peak = peaks["hbm_gbs"]
        unit = "GB/s"
    else:
        # Dense-equivalent rate against the 2:4 sparse tensor-core ceiling:
        # the sparse MMA does the same dense-equivalent work at twice the
        # dense rate, so the ceiling is 2x the measured dense bf16 burst.
        achieved = flops_total_rank / (kernel_us_total * 1e-6) / 1e12
        # fp8: the dense fp8 rate is twice the dense bf16 rate (4.5 vs 2.25
        # PFLOP/s nominal), so its 2:4 ceiling is 4x the measured bf16 burst.
        peak = (4.0 if fp8 else 2.0) * peaks["bf16_tflops"]
        unit = "TFLOP/s"
    traffic = None
    tr = load_traffic(args.workload)
    if tr and grouped:
        traffic = tr.get("grouped_step")  # one grouped launch = the whole step
    elif tr:
        per = [tr.get(f"{c['M']}x{c['N']}x{c['K']}") for c in calls]
        if all(v is not None for v in per):
            traffic = float(sum(per) / len(per))

    out = {
        "metric": "dense-equiv TFLOPS per 2:4 SpMM at LLaMA shapes (us per SpMM and % of roofline alongside)",
        "value": round(value, 4),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(elapsed_ms / args.steps, 5),
        "us_per_spmm": round(elapsed_ms * 1e3 / args.steps / len(calls), 3),
        "higher_is_better": True,
        "scaling": "strong" if shard else "weak",
        "vs_baseline": None,
        "dtype": ("fp8 e4m3 in, f32 accumulate, f16 out" if fp8
                  else f"{args.dtype} in, f32 accumulate, {args.dtype} out"),
        "data": ("synthetic (seeded torch RNG; A N(0,1) in E4M3, magnitude-pruned 2:4, dequantised by alpha = "
                 f"{wl['a_std']}; B N(0,1) in E4M3, N x K)" if fp8 else
                 f"synthetic (seeded torch RNG; A N(0,{wl['a_std']}) magnitude-pruned 2:4, B N(0,1))" if wl["a_std"]
                 else "synthetic (U(-1,1), random 2:4 mask)"),
        "config": workload_config(args, world),
        "per_shape_us": {f"{c['M']}x{c['N']}x{c['K']}": round(u, 3) for c, u in zip(calls, per_call)},
        "per_shape_note": "median single-kernel duration of one spmm24_launch per shape, an event pair around "
                          "each launch (per_shape_grouped_us: the same shape as a grouped launch of one problem)",
        "per_shape_grouped_us": ({f"{c['M']}x{c['N']}x{c['K']}": round(u, 3) for c, u in zip(calls, per_call_grouped)}
                                 if per_call_grouped else None),
        "host_per_call": host,
        "launch_flags": " | ".join(f for f, on in (("SPMM24_STATIC_WEIGHTS", args.static_weights), ("SPMM24_BF16", bf16),
                                                   ("spmm24_launch_fp8", fp8)) if on) or "none",
        "epilogue": args.epilogue,
        "roofline": {"bound": wl["bound"], "achieved": round(achieved, 2), "peak": peak, "unit": unit,
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_src": f"{peaks['src']} (" + ("hbm_gbs copy" if unit == "GB/s" else
                                                           "4 x dense bf16 cuBLAS burst (fp8 = 2 x bf16, 2:4 sparse = 2 x dense)"
                                                           if fp8 else "2 x dense bf16 cuBLAS burst (2:4 sparse rate)") + ")",
                     "per_launch_us": round(kernel_us_total / nl, 3),
                     "note": "achieved = algorithmic bytes (flops) of the timed region / its CUDA-event duration"},
        "e2e": {"value": round(e2e_value, 4), "unit": "TFLOPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms / args.steps, 5),
                "path": ("per step: one H2D of all packed activations (pinned), the step's spmm24 calls" +
                         (" replayed as a CUDA graph" if graph is not None else "") +
                         (", one D2H of the rank's 1/N share of the gathered C (pinned; the ranks together bring "
                          "the whole C to the host once); h2d/d2h bytes are per rank" if gather_mode else
                          ", one D2H of all results (pinned)") +
                         "; two buffer sets alternate so uploads and downloads overlap the neighbouring steps' "
                         "kernels")},
        "gpu_launches": nl,
        "clocks": clocks,
        "launch": ("grouped: one spmm24_launch_grouped per step (one persistent kernel for all the step's SpMMs)"
                   if grouped else "chain: one spmm24_launch per SpMM"),
    }
    if chain_ms is not None:
        # The same steps issued as one spmm24_launch per SpMM (programmatic
        # dependent launch between them), timed in the same run.
        out["chain"] = {"value": round(total_flops / (chain_ms * 1e-3) / 1e12, 4), "unit": "TFLOPS",
                        "us_per_spmm": round(chain_ms * 1e3 / args.steps / len(calls), 3),
                        "roofline_frac": round(bytes_total / (chain_ms * 1e-3) / 1e9 / peak, 4)
                        if wl["bound"] == "hbm" else None,
                        "gpu_launches": len(calls) * args.steps}

    if shard and args.allgather and world > 1:
        # NCCL all-gather of the C shards (contiguous row ranges) into the full
        # C on every rank, timed on its own, max over ranks.
        fulls = [torch.empty((c["M_full"], c["N"]), dtype=torch.float16, device=dev) for c in calls]
        equal = all(c["M_full"] % world == 0 and c["M"] * world == c["M_full"] for c in calls)
        def gather():
            for c, f in zip(calls, fulls):
                if equal:
                    dist.all_gather_into_tensor(f, c["C"])
                else:
                    dist.all_gather(list(f.split([spmm24.shard_rows(c["M_full"], world, i, 128)[1] -
                                                  spmm24.shard_rows(c["M_full"], world, i, 128)[0]
                                                  for i in range(world)])), c["C"])
        for _ in range(args.warmup):
            gather()
        torch.cuda.synchronize(dev)
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(args.steps):
            gather()
        g1.record(stream)
        torch.cuda.synchronize(dev)
        gt = torch.tensor([g0.elapsed_time(g1)], device=dev, dtype=torch.float64)
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
        gbytes = sum(2 * c["M_full"] * c["N"] for c in calls)
        out["allgather"] = {"us_per_step": round(float(gt[0]) * 1e3 / args.steps, 2), "bytes_per_step": gbytes,
                            "busbw_GBps": round(gbytes * (world - 1) / world / (float(gt[0]) * 1e-3 / args.steps) / 1e9, 1),
                            "op": "NCCL all_gather_into_tensor of the C shards"}

    if shard and args.gather and world > 1:
        out["gather"] = time_gather(torch, dist, spmm24, calls, stream, dev, rank, world, args, flags)

    if args.comparators and rank == 0 and world == 1 and not bf16 and not fp8:
        out["comparators"] = run_comparators(torch, spmm24, calls, layers, acts, dev, args)
    if args.secondary and rank == 0 and world == 1 and args.workload == "decode" and not bf16 and not fp8:
        with ClockSampler(local_rank) as sclk:  # the prefill shapes run long enough to meet the power cap
            out["secondary"] = run_secondary(torch, spmm24, dev, args)
        out["secondary"]["clocks"] = sclk.summary()

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(layers, acts, shapes, budget_s=args.cpu_seconds, bf16=bf16, fp8=fp8)
    if rank == 0 and world == 1 and args.extras and args.workload == "decode" and not (fp8 or bf16) \
            and args.epilogue == "none":
        out["extras"] = run_extras(args)

    if args.config4 and args.workload == "decode" and not (fp8 or bf16) and args.epilogue == "none":
        out["config4"] = run_config4(torch, dist, spmm24, dev, rank, world, args)
    if gather_mode:
        out["gather"] = {"status": spmm24.device_status(dev.index), "ranks": world,
                         "gathered_bytes_per_step": 2 * sum(c["M_full"] * c["N"] for c in calls),
                         "multicast": bool(mc_bases[0]),
                         "op": "one spmm24_launch_grouped_gather per step: each rank's output rows stored by the "
                               "grouped kernel's epilogue into all ranks' full C (" +
                               ("through the NVLink multicast address where N % 8 == 0, else peer stores"
                                if mc_bases[0] else "CUDA IPC peer pointers, NVLink") +
                               "), the cross-GPU barrier run by the grid's last CTA"}
        torch.cuda.synchronize(dev)
        dist.barrier()
        for p_ in imported:
            spmm24.ipc_close(p_)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def run_extras(args):
    """The rest of the hot path's measured rows in the default line, each as
    its own bench.py run (a child process on the same GPU, short steps): the
    fp8 decode step, the decode step with a fused bias + SiLU epilogue, the
    device A packer (prune + compress + reorder) and the packed-B producer.
    Each entry keeps the child's value, unit, roofline fraction and e2e; a
    child that fails is reported, not fatal."""
    runs = {
        "decode_fp8": ["--dtype", "fp8"],
        "decode_bias_silu": ["--epilogue", "bias_silu"],
        "pack_a_device": ["--workload", "pack"],
        "pack_b_device": ["--workload", "packb"],
    }
    out = {}
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    for name, extra in runs.items():
        cmd = [sys.executable, os.path.abspath(__file__), "--steps", "10", "--warmup", "3", "--no-comparators",
               "--no-secondary", "--no-config4", "--no-cpu-baseline", "--no-extras"] + extra
        t0 = time.time()
        try:
            r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
            line = [x for x in r.stdout.splitlines() if x.startswith("{")]
            if r.returncode != 0 or not line:
                out[name] = {"error": f"exit {r.returncode}: {r.stderr.strip()[-200:]}"}
                continue
            d = json.loads(line[-1])
            rf = d.get("roofline") or {}
            out[name] = {"value": d.get("value"), "unit": d.get("unit"), "dtype": d.get("dtype"),
                         "roofline_frac": rf.get("frac"), "roofline_peak": rf.get("peak"),
                         "e2e": (d.get("e2e") or {}).get("value"), "workload": (d.get("config") or {}).get("workload"),
                         "gpu_launches": d.get("gpu_launches"), "clocks": d.get("clocks"),
                         "wall_s": round(time.time() - t0, 1)}
        except Exception as e:  # noqa: BLE001 -- report, keep the main line
            out[name] = {"error": str(e)[:200]}
    out["how"] = ("bench.py " + "--steps 10 --warmup 3 --no-comparators --no-secondary --no-config4 "
                  "--no-cpu-baseline plus: " + "; ".join(f"{k}: {' '.join(v)}" for k, v in runs.items()))
    return out


def run_config4(torch, dist, spmm24, dev, rank, world, args):
    """BASELINE config 4 beside the decode line: the LLaMA-70B layers (M, K)
    in {(8192, 8192), (28672, 8192), (8192, 28672)} x N in {16, 256, 4096},
    each split along M across the ranks (spmm24_shard_rows, 128-row units),
    A N(0, 0.01) pruned 2:4 and B N(0, 1) generated and packed on the device.
    Timed twice, max over ranks: the shards alone (spmm24_launch per layer),
    and with the full C of every layer gathered on every rank inside the
    step (spmm24_launch_gather per layer -- the epilogue's stores over NVLink
    -- and one spmm24_gather_barrier per step).  The gather's NVLink bound:
    each rank receives (world - 1) / world of the full C, at the measured
    770 GB/s per direction of a peer copy on this pool."""
    layers_mk = [(8192, 8192), (28672, 8192), (8192, 28672)]
    ns = (16, 256, 4096)
    g = torch.Generator(device=dev)
    stream = torch.cuda.current_stream(dev)
    calls = []
    for li, (M, K) in enumerate(layers_mk):
        r0, r1 = spmm24.shard_rows(M, world, rank, 128)
        g.manual_seed(7000 + 100 * rank + li)
        a = (torch.randn(r1 - r0, K, generator=g, device=dev) * 0.01).half()
        spmm24.prune_2of4_device(a, r1 - r0, K)
        A, E, _ = spmm24.pack_a_device(a, r1 - r0, K)
        del a
        for N in ns:
            g.manual_seed(9000 + N + K)  # the same activations on every rank
            Bp = spmm24.pack_b_device(torch.randn(K, N, generator=g, device=dev).half(), K, N)
            calls.append({"M": r1 - r0, "M_full": M, "r0": r0, "N": N, "K": K, "A": A, "E": E, "B": Bp,
                          "C": torch.empty((r1 - r0, N), dtype=torch.float16, device=dev)})
    full_elems = sum(c["M_full"] * c["N"] for c in calls)
    full = torch.zeros(full_elems, dtype=torch.float16, device=dev)
    flag_buf = torch.zeros(world + 1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize(dev)
    imported = []
    if world > 1:
        handles = [None] * world
        dist.all_gather_object(handles, (spmm24.ipc_export(full), spmm24.ipc_export(flag_buf)))
        bases, flags_r = [], []
        for r in range(world):
            if r == rank:
                bases.append(full.data_ptr())
                flags_r.append(flag_buf.data_ptr())
            else:
                bases.append(spmm24.ipc_import(handles[r][0]))
                flags_r.append(spmm24.ipc_import(handles[r][1]))
                imported += [bases[-1], flags_r[-1]]
        dist.barrier()
    else:
        bases, flags_r = [full.data_ptr()], [flag_buf.data_ptr()]
    h = int(stream.cuda_stream)
    fl = spmm24.STATIC_WEIGHTS

    def shards():
        for c in calls:
            rc = spmm24._lib.spmm24_launch_ex(h, c["A"].data_ptr(), c["B"].data_ptr(), c["E"].data_ptr(),
                                              c["C"].data_ptr(), c["M"], c["N"], c["K"], 0, fl)
            if rc != 0:
                raise RuntimeError(f"spmm24_launch_ex: {rc}")

    def gathered():
        off = 0
        for c in calls:
            rc = spmm24.launch_gather(h, c["A"], c["B"], c["E"], c["M"], c["N"], c["K"],
                                      [b + 2 * off for b in bases], c["r0"], c["M_full"], 0, fl)
            off += c["M_full"] * c["N"]
            if rc != 0:
                raise RuntimeError(f"spmm24_launch_gather: {rc} {spmm24._lib.spmm24_last_error().decode()}")
        if spmm24.gather_barrier(h, flags_r, rank, 0) != 0:
            raise RuntimeError("spmm24_gather_barrier failed")

    steps = max(3, min(args.steps, 10))

    def timed(fn, sync=False):
        """sync: fn ends in a cross-GPU barrier; one untimed call after the
        sleep lines the ranks up on the device before the interval opens."""
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(int(2e7))
        if sync and world > 1:
            fn()
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / steps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0])

    us_shards = timed(shards)
    us_gather = timed(gathered, sync=True)
    status = spmm24.device_status(dev.index)
    if world > 1:
        dist.barrier()
        for p in imported:
            spmm24.ipc_close(p)
        dist.barrier()
    # The same gather with every output chunk stored once through the full
    # C's NVLink multicast address (a symmetric-memory buffer bound to every
    # rank; multimem.st, replicated by the switch): a rank sends its shard
    # once instead of once per peer.
    us_mc = None
    if world > 1:
        try:
            import torch.distributed._symmetric_memory as symm_mem

            grp = dist.group.WORLD
            mfull = symm_mem.empty((full_elems,), dtype=torch.float16, device=dev)
            mh = symm_mem.rendezvous(mfull, grp)
            mflags = symm_mem.empty((world + 1,), dtype=torch.int32, device=dev)
            mflags.zero_()
            fh = symm_mem.rendezvous(mflags, grp)
            torch.cuda.synchronize(dev)
            dist.barrier()
            if mh.multicast_ptr:
                moff = mfull.data_ptr() - mh.buffer_ptrs[rank]
                mbases = [mh.buffer_ptrs[r] + moff for r in range(world)]
                mcast = mh.multicast_ptr + moff
                foff = mflags.data_ptr() - fh.buffer_ptrs[rank]
                mflag_ptrs = [fh.buffer_ptrs[r] + foff for r in range(world)]

                def gathered_mc():
                    off = 0
                    for c in calls:
                        rc = spmm24.launch_gather(h, c["A"], c["B"], c["E"], c["M"], c["N"], c["K"],
                                                  [b + 2 * off for b in mbases], c["r0"], c["M_full"], 0, fl,
                                                  c_multicast=mcast + 2 * off)
                        off += c["M_full"] * c["N"]
                        if rc != 0:
                            raise RuntimeError(f"spmm24_launch_gather: {rc} {spmm24._lib.spmm24_last_error().decode()}")
                    if spmm24.gather_barrier(h, mflag_ptrs, rank, 0) != 0:
                        raise RuntimeError("spmm24_gather_barrier failed")

                us_mc = timed(gathered_mc, sync=True)
                status |= spmm24.device_status(dev.index)
            dist.barrier()
        except Exception as e:  # noqa: BLE001 -- report, keep the other numbers
            us_mc = f"unavailable: {str(e)[:120]}"
    flop = sum(flops(M, N, K) for (M, K) in layers_mk for N in ns)
    recv = 2 * full_elems * (world - 1) / world
    bound_us = recv / 770e9 * 1e6
    # the fused step's roofline: the slower of this rank's share of the flops
    # at the 2:4 tensor ceiling (2 x the measured dense bf16 burst) and the
    # bytes it must receive over NVLink
    compute_us = flop / world / (2.0 * load_peaks()["bf16_tflops"] * 1e12) * 1e6
    step_bound_us = max(compute_us, bound_us if world > 1 else 0.0)
    return {"baseline_config": 4, "workload": ", ".join(f"{M}x{N}x{K}" for (M, K) in layers_mk for N in ns),
            "parallelism": f"M-sharded x{world}", "steps": steps,
            "us_per_step_shards": round(us_shards, 2), "tflops_shards": round(flop / (us_shards * 1e-6) / 1e12, 1),
            "us_per_step_gathered": round(us_gather, 2),
            "tflops_gathered": round(flop / (us_gather * 1e-6) / 1e12, 1),
            "gather_share": round(max(0.0, us_gather - us_shards) / us_gather, 4),
            "us_per_step_gathered_multicast": round(us_mc, 2) if isinstance(us_mc, float) else us_mc,
            "tflops_gathered_multicast": round(flop / (us_mc * 1e-6) / 1e12, 1) if isinstance(us_mc, float) else None,
            "gathered_bytes_per_step": 2 * full_elems,
            "nvlink_receive_bound_us": round(bound_us, 2) if world > 1 else None,
            "compute_bound_us": round(compute_us, 2),
            "frac_of_step_bound": round(step_bound_us / us_gather, 4),
            "status": status,
            "op": "shards: spmm24_launch_ex per layer; gathered: spmm24_launch_gather per layer (peer stores over "
                  "NVLink into every rank's full C) + one spmm24_gather_barrier per step; device time, max over ranks"}


def time_gather(torch, dist, spmm24, calls, stream, dev, rank, world, args, flags):
    """The sharded layers with their C shards gathered into a full C on every
    rank, two ways, each timed on the device (max over ranks):
      fused -- spmm24_launch_gather (the epilogue writes every row into all
               ranks' full C over NVLink) + spmm24_gather_barrier, per layer;
      nccl  -- spmm24_launch_ex into the local shard + NCCL
               all_gather_into_tensor, per layer."""
    fulls = [torch.empty((c["M_full"], c["N"]), dtype=torch.float16, device=dev) for c in calls]
    flag_buf = torch.zeros(world, dtype=torch.int32, device=dev)
    torch.cuda.synchronize(dev)
    mine = [spmm24.ipc_export(f) for f in fulls] + [spmm24.ipc_export(flag_buf)]
    handles = [None] * world
    dist.all_gather_object(handles, mine)
    ptrs = [[None] * world for _ in range(len(calls) + 1)]
    imported = []
    for r in range(world):
        for i in range(len(calls) + 1):
            if r == rank:
                ptrs[i][r] = (fulls[i] if i < len(calls) else flag_buf).data_ptr()
            else:
                ptrs[i][r] = spmm24.ipc_import(handles[r][i])
                imported.append(ptrs[i][r])
    dist.barrier()
    rows = [spmm24.shard_rows(c["M_full"], world, rank, 128) for c in calls]
    epoch = [0]

    def fused():
        for i, c in enumerate(calls):
            rc = spmm24.launch_gather(stream, c["A"], c["B"], c["E"], c["M"], c["N"], c["K"], ptrs[i], rows[i][0],
                                      c["M_full"], 0, flags)
            if rc != 0:
                raise RuntimeError(f"spmm24_launch_gather: {rc} {spmm24._lib.spmm24_last_error().decode()}")
            epoch[0] += 1
            if spmm24.gather_barrier(stream, ptrs[-1], rank, epoch[0]) != 0:
                raise RuntimeError("spmm24_gather_barrier failed")

    equal = all(c["M_full"] % world == 0 and c["M"] * world == c["M_full"] for c in calls)

    def nccl():
        for i, c in enumerate(calls):
            rc = spmm24._lib.spmm24_launch_ex(int(stream.cuda_stream), c["A"].data_ptr(), c["B"].data_ptr(),
                                              c["E"].data_ptr(), c["C"].data_ptr(), c["M"], c["N"], c["K"], 0, flags)
            if rc != 0:
                raise RuntimeError("spmm24_launch_ex failed")
            if equal:
                dist.all_gather_into_tensor(fulls[i], c["C"])
            else:
                dist.all_gather(list(fulls[i].split([spmm24.shard_rows(c["M_full"], world, r, 128)[1] -
                                                     spmm24.shard_rows(c["M_full"], world, r, 128)[0]
                                                     for r in range(world)])), c["C"])

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        dist.barrier()
        fn()  # untimed: both forms end in a cross-GPU exchange, which lines the ranks up on the device
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0]) * 1e3 / args.steps

    us_fused = timed(fused)
    status = spmm24.device_status(dev.index)
    us_nccl = timed(nccl)
    dist.barrier()
    for p in imported:
        spmm24.ipc_close(p)
    dist.barrier()

    # The same with every output chunk stored once through an NVLink
    # multicast address (symmetric-memory buffers bound to all ranks).
    us_mc = None
    try:
        import torch.distributed._symmetric_memory as symm_mem

        group = dist.group.WORLD
        mfulls = [symm_mem.empty((c["M_full"], c["N"]), dtype=torch.float16, device=dev) for c in calls]
        mhandles = [symm_mem.rendezvous(t, group) for t in mfulls]
        mflags = symm_mem.empty((world,), dtype=torch.int32, device=dev)
        mflags.zero_()
        fh = symm_mem.rendezvous(mflags, group)
        if all(h.multicast_ptr for h in mhandles) and all(c["N"] % 8 == 0 for c in calls):
            foff = mflags.data_ptr() - fh.buffer_ptrs[rank]
            fptrs = [fh.buffer_ptrs[r] + foff for r in range(world)]
            mc = []
            for t, h in zip(mfulls, mhandles):
                off = t.data_ptr() - h.buffer_ptrs[rank]
                mc.append(([h.buffer_ptrs[r] + off for r in range(world)], h.multicast_ptr + off))
            mepoch = [0]

            def fused_mc():
                for i, c in enumerate(calls):
                    rc = spmm24.launch_gather(stream, c["A"], c["B"], c["E"], c["M"], c["N"], c["K"], mc[i][0],
                                              rows[i][0], c["M_full"], 0, flags, c_multicast=mc[i][1])
                    if rc != 0:
                        raise RuntimeError(f"spmm24_launch_gather: {rc} {spmm24._lib.spmm24_last_error().decode()}")
                    mepoch[0] += 1
                    if spmm24.gather_barrier(stream, fptrs, rank, mepoch[0]) != 0:
                        raise RuntimeError("spmm24_gather_barrier failed")

            us_mc = timed(fused_mc)
            status |= spmm24.device_status(dev.index)
        dist.barrier()
    except Exception as e:  # noqa: BLE001 -- report, keep the other numbers
        us_mc = f"unavailable: {str(e)[:120]}"
    fl = sum(flops(c["M_full"], c["N"], c["K"]) for c in calls)
    out = {"fused_us_per_step": round(us_fused, 2), "nccl_us_per_step": round(us_nccl, 2),
           "fused_tflops": round(fl / (us_fused * 1e-6) / 1e12, 2),
           "nccl_tflops": round(fl / (us_nccl * 1e-6) / 1e12, 2),
           "gathered_bytes_per_step": sum(2 * c["M_full"] * c["N"] for c in calls), "status": status,
           "op": "fused: spmm24_launch_gather + spmm24_gather_barrier per layer (peer stores over NVLink); "
                 "fused_multicast: the same, each chunk stored once through an NVLink multicast address "
                 "(multimem.st); nccl: spmm24_launch_ex + all_gather_into_tensor per layer"}
    if isinstance(us_mc, float):
        out["fused_multicast_us_per_step"] = round(us_mc, 2)
        out["fused_multicast_tflops"] = round(fl / (us_mc * 1e-6) / 1e12, 2)
    elif us_mc is not None:
        out["fused_multicast"] = us_mc
    return out


# ---------------------------------------------------------- comparators
# Same-run comparators (the reference times cuSPARSELt and cuBLAS beside its
# kernel: bench/main.cu:104, :136): dense cuBLAS fp16 (torch.matmul, fp32
# accumulation), cuSPARSELt 0.7.1 through its own plan / search / matmul API
# (comparators/cmp.cu) and the reference's kernel built for sm_100a
# (oracle/_ref, N in {8..128} only).  Each call is timed alone with CUDA
# events after an L2 flush (a 256 MB write), median of `iters`.
def _cmp_lib():
    import ctypes

    path = os.path.join(REPO, "comparators", "_build", "libspmm24_cmp.so")
    if not os.path.exists(path):
        return None
    L = ctypes.CDLL(path)
    vp = ctypes.c_void_p
    L.cmp_cslt_create.argtypes = [ctypes.c_int] * 3 + [vp, vp, vp, vp, ctypes.c_int, ctypes.POINTER(vp)]
    L.cmp_cslt_create.restype = ctypes.c_int
    L.cmp_cslt_run.argtypes = [vp, vp]
    L.cmp_cslt_run.restype = ctypes.c_int
    L.cmp_cslt_alg_id.argtypes = [vp]
    L.cmp_cslt_alg_id.restype = ctypes.c_int
    L.cmp_cslt_destroy.argtypes = [vp]
    L.cmp_last_error.restype = ctypes.c_char_p
    L.cmp_sparse_mma_peak.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]
    L.cmp_sparse_mma_peak.restype = ctypes.c_double
    return L


class _Timer:
    def __init__(self, torch, dev):
        self.torch = torch
        self.flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def __call__(self, fn, iters=10, warmup=3):
        torch = self.torch
        for _ in range(warmup):
            fn()
        ts = []
        for _ in range(iters):
            self.flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) * 1e3)
        return statistics.median(ts)


def compare_case(torch, spmm24, timer, cmp, ref, dev, M, N, K, A, E, Bp, Ad, Bd, iters=10):
    """One shape through every implementation; device operands given: the
    packed A / metadata / B of this library, and the pruned dense A (M x K)
    and row-major B (K x N) for the others.  Returns microseconds per call."""
    import ctypes

    h = int(torch.cuda.current_stream().cuda_stream)
    C = torch.empty((M, N), dtype=torch.float16, device=dev)
    row = {"ours_us": timer(lambda: spmm24._lib.spmm24_launch(h, A.data_ptr(), Bp.data_ptr(), E.data_ptr(),
                                                               C.data_ptr(), M, N, K, None, 0), iters)}
    prev = torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    try:
        row["cublas_dense_fp16_us"] = timer(lambda: torch.matmul(Ad, Bd), iters)
    finally:
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = prev
    if cmp is not None:
        # cuSPARSELt wants 16-byte rows of B and C: N padded to a multiple of 8 (at least 16)
        Np = max(16, (N + 7) // 8 * 8)
        Bq = Bd if Np == N else torch.nn.functional.pad(Bd, (0, Np - N))
        Cq = torch.empty((M, Np), dtype=torch.float16, device=dev)
        plan = ctypes.c_void_p()
        rc = cmp.cmp_cslt_create(M, Np, K, Ad.data_ptr(), Bq.data_ptr(), Cq.data_ptr(), h, 1, ctypes.byref(plan))
        if rc == 0:
            row["cusparselt_us"] = timer(lambda: cmp.cmp_cslt_run(plan, h), iters)
            row["cusparselt_alg_id"] = cmp.cmp_cslt_alg_id(plan)
            if Np != N:
                row["cusparselt_n_padded"] = Np
            cmp.cmp_cslt_destroy(plan)
        else:
            row["cusparselt_error"] = cmp.cmp_last_error().decode()
    if ref is not None and ref.ref_spmm_supported(M, N, K, 1):
        row["reference_kernel_us"] = timer(lambda: ref.ref_spmm_launch(h, A.data_ptr(), Bp.data_ptr(), E.data_ptr(),
                                                                       C.data_ptr(), M, N, K, None, 1), iters)
    if row.get("cusparselt_us"):
        row["x_vs_cusparselt"] = round(row["cusparselt_us"] / row["ours_us"], 3)
    row["x_vs_cublas"] = round(row["cublas_dense_fp16_us"] / row["ours_us"], 3)
    return {k: (round(v, 3) if isinstance(v, float) else v) for k, v in row.items()}


def _reference_kernel():
    try:
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import oracle as O

        return O.ref_spmm() if O.ref_spmm_available() else None
    except Exception:  # noqa: BLE001
        return None


def target_summary(rows):
    """The north star's targets per shape: >= 1.0x cuSPARSELt, >= 1.5x dense cuBLAS."""
    out = {}
    for key, field, bar in (("cusparselt_1.0x", "x_vs_cusparselt", 1.0), ("cublas_1.5x", "x_vs_cublas", 1.5)):
        have = {k: r[field] for k, r in rows.items() if r.get(field) is not None}
        out[key] = {"met": sum(1 for v in have.values() if v >= bar), "of": len(have),
                    "missed": {k: v for k, v in have.items() if v < bar}}
    return out


def run_comparators(torch, spmm24, calls, layers, acts, dev, args):
    """The step's shapes, one isolated call each, against the comparators."""
    timer = _Timer(torch, dev)
    cmp = _cmp_lib()
    ref = _reference_kernel()
    rows = {}
    for c in calls:
        key = f"{c['M']}x{c['N']}x{c['K']}"
        a_np = layers[(c["M"], c["K"])][0]
        b_np = acts[(c["K"], c["N"])][0]
        Ad = torch.from_numpy(a_np.view("int16")).to(dev).view(torch.float16).reshape(c["M"], c["K"])
        Bd = torch.from_numpy(b_np.view("int16")).to(dev).view(torch.float16).reshape(c["K"], c["N"])
        rows[key] = compare_case(torch, spmm24, timer, cmp, ref, dev, c["M"], c["N"], c["K"], c["A"], c["E"],
                                 c["B"], Ad, Bd)
        del Ad, Bd
    return {"per_shape": rows, "targets": target_summary(rows),
            "method": "isolated calls, L2 flushed (256 MB write) before each, CUDA events, median of 10; cuSPARSELt "
                      "0.7.1 plan + cusparseLtMatmulSearch (comparators/cmp.cu); cuBLAS = torch.matmul fp16 with "
                      "fp32 reduction"}


def run_secondary(torch, spmm24, dev, args):
    """BASELINE configs 3 (LLaMA-7B prefill) and 5 (squares up to 16384^3):
    per-shape isolated calls against the comparators, and the sparse
    tensor-core ceiling measured in the same run.  Operands are generated and
    packed on the device (spmm24_prune_2of4_device, spmm24_pack_a_device,
    spmm24_pack_b_device)."""
    import ctypes

    timer = _Timer(torch, dev)
    cmp = _cmp_lib()
    ref = _reference_kernel()
    out = {}
    peak = None
    if cmp is not None:
        # Burst figures (about 1 ms per run, best of 3), like the dense bf16
        # burst of MEASURED_PEAKS: the CTA-pair mix of the prefill kernels is
        # the ceiling; the one-CTA mix of the cluster kernels is reported too.
        ceil = {}
        for key, pair in (("cta_pair_m256", 1), ("one_cta_m128", 0)):
            best, best_ms = -1.0, 0.0
            for _ in range(3):
                ms = ctypes.c_float()
                v = cmp.cmp_sparse_mma_peak(4000, pair, ctypes.byref(ms))
                if v > best:
                    best, best_ms = v, ms.value
            if best > 0:
                ceil[key] = {"tflops": round(best, 1), "ms": round(best_ms, 3)}
        if ceil:
            peak = ceil.get("cta_pair_m256", ceil.get("one_cta_m128"))["tflops"]
            out["sparse_ceiling"] = dict(ceil, tflops=peak, what=(
                "the kernels' stage mix on operands resident in shared memory, one CTA (or CTA pair) per SM, 4000 "
                "stages, best of 3: tcgen05.cp + 4 x tcgen05.mma.sp kind::f16 K=32 (M=256 N=256 cta_group::2; "
                "M=128 N=256 cta_group::1) -- comparators/cmp.cu; dense-equivalent; the pair figure is the "
                "ceiling"))
    dense_peak = 2.0 * load_peaks()["bf16_tflops"]
    g = torch.Generator(device=dev).manual_seed(2024)
    for name, shapes, square in (("prefill", WORKLOADS["prefill"]["shapes"], False),
                                 ("square", [(s, s, s) for s in (1024, 2048, 4096, 8192, 16384)], True)):
        rows = {}
        fl = us = 0.0
        for (M, N, K) in shapes:
            if square:
                a = (torch.rand(M, K, generator=g, device=dev) * 2 - 1).half()
                keep = torch.rand(M * K // 4, 4, generator=g, device=dev).argsort(dim=1)[:, :2]
                mask = torch.zeros(M * K // 4, 4, dtype=torch.bool, device=dev).scatter_(1, keep, True)
                a = (a.view(-1, 4) * mask).view(M, K)
                del keep, mask
                b = (torch.rand(K, N, generator=g, device=dev) * 2 - 1).half()
            else:
                a = (torch.randn(M, K, generator=g, device=dev) * 0.02).half()
                spmm24.prune_2of4_device(a, M, K)
                b = torch.randn(K, N, generator=g, device=dev).half()
            A, E, _ = spmm24.pack_a_device(a, M, K)
            Bp = spmm24.pack_b_device(b, K, N)
            iters = 5 if M * N * K >= 8192 ** 3 else 10
            r = compare_case(torch, spmm24, timer, cmp, ref, dev, M, N, K, A, E, Bp, a, b, iters)
            r["ours_tflops"] = round(flops(M, N, K) / (r["ours_us"] * 1e-6) / 1e12, 1)
            rows[f"{M}x{N}x{K}"] = r
            fl += flops(M, N, K)
            us += r["ours_us"]
            del a, b, A, E, Bp
            torch.cuda.empty_cache()
        tf = fl / (us * 1e-6) / 1e12
        out[name] = {"baseline_config": 3 if name == "prefill" else 5, "tflops": round(tf, 1),
                     "frac_of_2x_dense_bf16": round(tf / dense_peak, 4),
                     "frac_of_sparse_ceiling": round(tf / peak, 4) if peak else None,
                     "per_shape": rows, "targets": target_summary(rows)}
    out["method"] = ("isolated calls, L2 flushed before each, CUDA events, median of 10 (5 at >= 8192^3); tflops = "
                     "sum of 2MNK / sum of the medians")
    return out


def host_threads():
    """All host cores this process may run on (torchrun sets OMP_NUM_THREADS=1,
    which must not throttle the CPU baseline)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(layers, acts, shapes, budget_s=10.0, bf16=False, fp8=False):
    """The oracle's OpenMP dense GEMM (fp16 or bf16 -> fp32, fp32 accumulate)
    on the pruned A, on a row sample of every shape of the workload (fp8:
    the oracle's fp8 SpMM -- decode of the first bands' values and metadata,
    then the fp32 GEMM)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O

    threads = host_threads()

    def run(M, N, K, r):
        if fp8:
            _, vals, meta = layers[(M, K)]
            O.spmm_fp8_f32(vals[: r * K // 2], meta[: r * K // 8], acts[(K, N)][0], r, N, K, 0, 0, threads)
        else:
            gemm = O.dense_gemm_bf16_f32 if bf16 else O.dense_gemm_f32
            gemm(layers[(M, K)][0][: r * K], acts[(K, N)][0], r, N, K, threads)

    # estimate: 64 rows of every shape
    probe_rows = 64
    t = time.perf_counter()
    for (M, N, K) in shapes:
        run(M, N, K, probe_rows)
    dt = time.perf_counter() - t
    rows = int(max(16, min(4096, probe_rows * budget_s / max(dt, 1e-3) / 1.2))) // 16 * 16
    fl = 0.0
    t = time.perf_counter()
    for (M, N, K) in shapes:
        r = min(rows, M)
        run(M, N, K, r)
        fl += flops(r, N, K)
    dt = time.perf_counter() - t
    what = "fp8 decode + fp32 GEMM" if fp8 else "dense fp32 GEMM on the pruned A"
    return {"value": round(fl / dt / 1e12, 6), "unit": "TFLOPS", "cores": threads, "kind": "port",
            "sample": f"first {rows} rows of each of the {len(shapes)} shapes ({what}), {dt:.1f} s"}


# ------------------------------------------------- on-device packer
def host_pack_baseline(dense_np, budget_s=10.0, fp8=False):
    """The reference's own host packer (toolCompressMatrixA +
    toolReorderMetadata built from its sources into oracle/_ref), else the
    oracle's restatement of it, on a row sample of each layer; single
    threaded as the reference is (fp8, which the reference lacks: the
    oracle's fp8 prune + compress).  Returns (GB/s, kind, sample)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O

    use_ref = O.ref_packer_available() and not fp8

    def pack(a, M, K):
        if fp8:
            O.compress_a_fp8(O.prune_magnitude_2of4_fp8(a, M, K, 0), M, K)
            return
        # the reference has no pruning step (its inputs are generated 2:4):
        # the oracle's prune runs first, inside the timed work
        a = O.prune_magnitude_2of4(a, M, K)
        if use_ref:
            _, _, meta = O.ref_compress_a(a, M, K)
            O.ref_reorder_metadata(meta, M, K)
        else:
            _, meta = O.compress_a(a, M, K)
            O.reorder_metadata(meta, M, K)

    probe = 64
    t = time.perf_counter()
    for (M, K), a in zip(PACK_LAYERS, dense_np):
        pack(a[: probe * K], probe, K)
    dt = time.perf_counter() - t
    rows = int(max(16, min(4096, probe * budget_s / max(dt, 1e-3) / 1.2))) // 16 * 16
    nbytes = 0
    t = time.perf_counter()
    for (M, K), a in zip(PACK_LAYERS, dense_np):
        r = min(rows, M)
        pack(a[: r * K], r, K)
        nbytes += pack_bytes(r, K, fp8)
    dt = time.perf_counter() - t
    kind = "reference" if use_ref else "port"
    return nbytes / dt / 1e9, kind, (f"first {rows} rows of each of the {len(PACK_LAYERS)} layers through "
                                     f"{'oracle prune, then toolCompressMatrixA + toolReorderMetadata (oracle/_ref)' if use_ref else 'orc_prune_magnitude_2of4_fp8 + orc_compress_a_fp8' if fp8 else 'oracle prune + orc_compress_a + orc_reorder_metadata'}, "
                                     f"1 thread, {dt:.1f} s")


def run_pack(args, rank, world, local_rank):
    """Times spmm24_pack_a_device (magnitude prune + compress + reordered
    metadata in one kernel) over the three LLaMA-7B layer shapes, weights
    resident in HBM (214 MB of dense weights per step, more than L2)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import spmm24

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    # fp8: spmm24_pack_a_fp8_device on E4M3 weights (N(0,1) through torch's float8 cast)
    fp8 = args.dtype == "fp8"
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    if fp8:
        dense = [torch.randn(M, K, generator=g, device=dev).to(torch.float8_e4m3fn).view(torch.uint8)
                 for (M, K) in PACK_LAYERS]
        vals = [torch.empty(M * K // 2, dtype=torch.uint8, device=dev) for (M, K) in PACK_LAYERS]
        meta = [torch.empty(M * K // 8, dtype=torch.uint8, device=dev) for (M, K) in PACK_LAYERS]
    else:
        dense = [(torch.randn(M, K, generator=g, device=dev) * 0.02).half() for (M, K) in PACK_LAYERS]
        vals = [torch.empty(M * K // 2, dtype=torch.int16, device=dev) for (M, K) in PACK_LAYERS]
        meta = [torch.empty(M * K // 16, dtype=torch.int16, device=dev) for (M, K) in PACK_LAYERS]
    bad = torch.zeros(len(PACK_LAYERS), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    hs = int(stream.cuda_stream)
    L = spmm24._lib
    pack_fn = L.spmm24_pack_a_fp8_device if fp8 else L.spmm24_pack_a_device

    def step():
        for i, (M, K) in enumerate(PACK_LAYERS):
            rc = pack_fn(hs, dense[i].data_ptr(), M, K, 1, vals[i].data_ptr(), meta[i].data_ptr(),
                         bad.data_ptr() + 4 * i)
            if rc != 0:
                raise RuntimeError(f"device packer failed: {rc} {L.spmm24_last_error().decode()}")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda._sleep(int(2e7))
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    elapsed_ms = t0.elapsed_time(t1)
    clocks = clk.summary()
    # the timed work is checked: no bad rows, and the smallest layer equals the host packer bit for bit
    assert int(bad.sum()) == 0
    if fp8:
        d0 = dense[0].cpu().numpy().reshape(-1)
        hv, hm = spmm24.compress_a_fp8(spmm24.prune_2of4_fp8(d0, *PACK_LAYERS[0], spmm24.FP8_E4M3), *PACK_LAYERS[0])
        assert np.array_equal(vals[0].cpu().numpy(), hv) and np.array_equal(meta[0].cpu().numpy(), hm)
    else:
        d0 = dense[0].view(torch.int16).cpu().numpy().view(np.uint16)
        hv, hm = spmm24.compress_reordered(spmm24.prune_2of4(d0, *PACK_LAYERS[0]), *PACK_LAYERS[0])
        assert np.array_equal(vals[0].cpu().numpy().view(np.uint16), hv)
        assert np.array_equal(meta[0].cpu().numpy().view(np.uint16), hm)

    # per-layer kernel durations (event pair around each launch)
    per = {}
    for i, (M, K) in enumerate(PACK_LAYERS):
        ts = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            pack_fn(hs, dense[i].data_ptr(), M, K, 1, vals[i].data_ptr(), meta[i].data_ptr(), None)
            b.record(stream)
            torch.cuda.synchronize(dev)
            ts.append(a.elapsed_time(b) * 1e3)
        per[f"{M}x{K}"] = round(statistics.median(ts), 3)

    # end to end: dense weights from pinned host memory, pack, compressed
    # values + metadata back to pinned host memory, every step
    host_dense = [d.cpu().pin_memory() for d in dense]
    host_vals = [torch.empty(v.shape, dtype=v.dtype).pin_memory() for v in vals]
    host_meta = [torch.empty(m.shape, dtype=m.dtype).pin_memory() for m in meta]

    def e2e_step():
        for i in range(len(PACK_LAYERS)):
            dense[i].copy_(host_dense[i], non_blocking=True)
        step()
        for i in range(len(PACK_LAYERS)):
            host_vals[i].copy_(vals[i], non_blocking=True)
            host_meta[i].copy_(meta[i], non_blocking=True)

    e2e_step()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([elapsed_ms, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, e2e_ms = float(t[0]), float(t[1])

    step_bytes = sum(pack_bytes(M, K, fp8) for (M, K) in PACK_LAYERS)
    dense_bytes = sum(M * K * (1 if fp8 else 2) for (M, K) in PACK_LAYERS)
    value = step_bytes * args.steps * world / (elapsed_ms * 1e-3) / 1e9
    achieved = step_bytes * args.steps / (elapsed_ms * 1e-3) / 1e9
    peaks = load_peaks()
    out = {
        "metric": ("GB/s of the on-device fp8 2:4 packer (magnitude prune + compress + metadata) "
                   "on the LLaMA-7B layer weights" if fp8 else
                   "GB/s of the on-device 2:4 packer (magnitude prune + compress + reordered metadata) "
                   "on the LLaMA-7B layer weights"),
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(elapsed_ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8 (fp8 E4M3 bit patterns; integer/byte work)" if fp8 else "u16 (fp16 bit patterns; integer/byte work)",
        "data": ("synthetic (seeded torch RNG on the device; dense E4M3 from N(0,1))" if fp8
                 else "synthetic (seeded torch RNG on the device; dense fp16 N(0,0.02))"),
        "config": {"workload": "pack: " + ", ".join(f"{M}x{K}" for (M, K) in PACK_LAYERS),
                   "baseline_config": 2, "calls_per_step": len(PACK_LAYERS),
                   "l2": f"inputs larger than L2: {dense_bytes / 1e6:.0f} MB of dense weights per step",
                   "parallelism": f"replicas x{world}"},
        "per_layer_us": per,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "peak_src": f"{peaks['src']} (hbm_gbs copy)",
                     "note": ("bytes = dense read MK + values MK/2 + metadata MK/8 per layer" if fp8 else
                              "bytes = dense read 2MK + values MK + metadata MK/8 per layer")},
        "e2e": {"value": round(step_bytes * args.steps * world / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": dense_bytes,
                "d2h_bytes_per_step": sum(v.numel() * v.element_size() + m.numel() * m.element_size()
                                          for v, m in zip(vals, meta)),
                "ms_per_step": round(e2e_ms / args.steps, 4),
                "path": f"per step: H2D of the dense weights (pinned), "
                        f"{'spmm24_pack_a_fp8_device' if fp8 else 'spmm24_pack_a_device'} per layer, "
                        "D2H of values + metadata"},
        "gpu_launches": len(PACK_LAYERS) * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if fp8:
            dn = [d.cpu().numpy().reshape(-1) for d in dense]
        else:
            dn = [d.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1) for d in dense]
        gbs, kind, sample = host_pack_baseline(dn, args.cpu_seconds, fp8=fp8)
        out["cpu_baseline"] = {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": kind, "sample": sample}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def host_pack_b_baseline(acts_np, budget_s=10.0):
    """The reference's toolPackMatrixB (built from its sources into
    oracle/_ref), else the oracle's restatement, on K-row samples of each
    activation; single threaded as the reference is.  Returns (GB/s, kind,
    sample)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O

    use_ref = O.ref_packer_available()
    pack = O.ref_pack_b if use_ref else O.pack_b
    probe = 64
    t = time.perf_counter()
    for (K, N), b in zip(PACKB_ACTS, acts_np):
        pack(b[: probe * N], probe, N)
    dt = time.perf_counter() - t
    rows = int(max(64, min(4096, probe * budget_s / max(dt, 1e-3) / 1.2))) // 64 * 64
    nbytes = 0
    t = time.perf_counter()
    for (K, N), b in zip(PACKB_ACTS, acts_np):
        r = min(rows, K)
        pack(b[: r * N], r, N)
        nbytes += packb_bytes(r, N)
    dt = time.perf_counter() - t
    kind = "reference" if use_ref else "port"
    return nbytes / dt / 1e9, kind, (f"first {rows} K rows of each of the {len(PACKB_ACTS)} activations through "
                                     f"{'toolPackMatrixB (oracle/_ref)' if use_ref else 'orc_pack_b'}, "
                                     f"1 thread, {dt:.1f} s")


def run_pack_b(args, rank, world, local_rank):
    """Times spmm24_pack_b_device (row-major K x N fp16 activations ->
    the packed 8-column strips the SpMM reads) over the prefill activations,
    resident in HBM (201 MB read and 201 MB written per step, more than L2)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import spmm24

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    acts = [torch.randn(K, N, generator=g, device=dev).half() for (K, N) in PACKB_ACTS]
    outs = [torch.empty(((N + 7) // 8) * 8 * K, dtype=torch.int16, device=dev) for (K, N) in PACKB_ACTS]
    stream = torch.cuda.current_stream(dev)
    hs = int(stream.cuda_stream)
    L = spmm24._lib

    def step():
        for i, (K, N) in enumerate(PACKB_ACTS):
            rc = L.spmm24_pack_b_device(hs, acts[i].data_ptr(), K, N, outs[i].data_ptr())
            if rc != 0:
                raise RuntimeError(f"spmm24_pack_b_device failed: {rc} {L.spmm24_last_error().decode()}")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda._sleep(int(2e7))
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    elapsed_ms = t0.elapsed_time(t1)
    clocks = clk.summary()
    # the timed work is checked: the smallest activation equals the host packer bit for bit
    K0, N0 = PACKB_ACTS[0]
    host = spmm24.pack_b(acts[0].view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1), K0, N0)
    assert np.array_equal(outs[0].cpu().numpy().view(np.uint16), host)

    per = {}
    for i, (K, N) in enumerate(PACKB_ACTS):
        ts = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            L.spmm24_pack_b_device(hs, acts[i].data_ptr(), K, N, outs[i].data_ptr())
            b.record(stream)
            torch.cuda.synchronize(dev)
            ts.append(a.elapsed_time(b) * 1e3)
        per[f"{K}x{N}"] = round(statistics.median(ts), 3)

    # end to end: activations from pinned host memory, pack, packed B back
    host_acts = [a.cpu().pin_memory() for a in acts]
    host_outs = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]

    def e2e_step():
        for i in range(len(PACKB_ACTS)):
            acts[i].copy_(host_acts[i], non_blocking=True)
        step()
        for i in range(len(PACKB_ACTS)):
            host_outs[i].copy_(outs[i], non_blocking=True)

    e2e_step()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([elapsed_ms, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, e2e_ms = float(t[0]), float(t[1])

    step_bytes = sum(packb_bytes(K, N) for (K, N) in PACKB_ACTS)
    value = step_bytes * args.steps * world / (elapsed_ms * 1e-3) / 1e9
    achieved = step_bytes * args.steps / (elapsed_ms * 1e-3) / 1e9
    peaks = load_peaks()
    out = {
        "metric": "GB/s of the on-device B packer (row-major activations -> packed 8-column strips) "
                  "on the LLaMA-7B prefill activations",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(elapsed_ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u16 (fp16 bit patterns; a permutation copy)",
        "data": "synthetic (seeded torch RNG on the device; activations N(0,1) fp16)",
        "config": {"workload": "packb: " + ", ".join(f"{K}x{N}" for (K, N) in PACKB_ACTS),
                   "baseline_config": 3, "calls_per_step": len(PACKB_ACTS),
                   "l2": f"inputs larger than L2: {sum(2 * K * N for (K, N) in PACKB_ACTS) / 1e6:.0f} MB "
                         "of activations per step",
                   "parallelism": f"replicas x{world}"},
        "per_act_us": per,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "peak_src": f"{peaks['src']} (hbm_gbs copy)",
                     "note": "bytes = read 2KN + write 2K*ceil(N/8)*8 per activation"},
        "e2e": {"value": round(step_bytes * args.steps * world / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": sum(2 * K * N for (K, N) in PACKB_ACTS),
                "d2h_bytes_per_step": sum(o.numel() * 2 for o in outs),
                "ms_per_step": round(e2e_ms / args.steps, 4),
                "path": "per step: H2D of the activations (pinned), spmm24_pack_b_device per activation, "
                        "D2H of the packed B"},
        "gpu_launches": len(PACKB_ACTS) * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        an = [a.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1) for a in acts]
        gbs, kind, sample = host_pack_b_baseline(an, args.cpu_seconds)
        out["cpu_baseline"] = {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": kind, "sample": sample}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


# -------------------------------------------------------- reference arm
def run_reference_pack_b(args):
    """--impl reference --workload packb: the reference's host
    toolPackMatrixB on K-row samples of the same activations, one step = one
    sample of each."""
    import numpy as np
    import torch

    g = torch.Generator().manual_seed(11)
    acts = [torch.randn(K, N, generator=g).half().numpy().view(np.uint16).reshape(-1) for (K, N) in PACKB_ACTS]
    for _ in range(args.warmup):
        host_pack_b_baseline(acts, 0.2)
    vals = [host_pack_b_baseline(acts, 1.0) for _ in range(args.steps)]
    gbs = statistics.median(v[0] for v in vals)
    kind, sample = vals[-1][1], vals[-1][2]
    print(json.dumps({
        "impl": "reference",
        "metric": "GB/s of the on-device B packer (row-major activations -> packed 8-column strips) "
                  "on the LLaMA-7B prefill activations",
        "value": round(gbs, 4), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u16 (fp16 bit patterns; a permutation copy)", "data": "synthetic",
        "config": {"workload": "packb: " + ", ".join(f"{K}x{N}" for (K, N) in PACKB_ACTS), "baseline_config": 3},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": kind, "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference packs B on the host only (toolPackMatrixB)",
    }), flush=True)


def run_reference_pack(args):
    """--impl reference --workload pack: the reference's host packer on row
    samples of the same layers, one step = one sample of each layer."""
    import numpy as np
    import torch

    g = torch.Generator().manual_seed(7)
    dense = [(torch.randn(M, K, generator=g) * 0.02).half().numpy().view(np.uint16).reshape(-1)
             for (M, K) in PACK_LAYERS]
    vals = []
    for _ in range(args.warmup):
        host_pack_baseline(dense, 0.2)
    for _ in range(args.steps):
        vals.append(host_pack_baseline(dense, 1.0))
    gbs = statistics.median(v[0] for v in vals)
    kind, sample = vals[-1][1], vals[-1][2]
    print(json.dumps({
        "impl": "reference",
        "metric": "GB/s of the on-device 2:4 packer (magnitude prune + compress + reordered metadata) "
                  "on the LLaMA-7B layer weights",
        "value": round(gbs, 4), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u16 (fp16 bit patterns; integer/byte work)", "data": "synthetic",
        "config": {"workload": "pack: " + ", ".join(f"{M}x{K}" for (M, K) in PACK_LAYERS), "baseline_config": 2},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": kind, "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference packs on the host only; it has no prune, so the oracle's prune runs before its "
                "compress + reorder",
    }), flush=True)


def run_reference(args, rank, world):
    if rank != 0:
        return
    if args.workload == "pack":
        run_reference_pack(args)
        return
    if args.workload == "packb":
        run_reference_pack_b(args)
        return
    # Inputs come from the oracle's own seeded generators and prune (the
    # product library is not loaded in this arm); same distributions as the
    # repo arm's.
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O

    wl = WORKLOADS[args.workload]
    shapes = wl["shapes"]
    square = args.workload == "square"
    layers = {}
    for i, (M, K) in enumerate(sorted({(M, K) for (M, N, K) in shapes})):
        if wl["a_std"] is None:
            a = O.uniform_f16(M * K, seed=i)
            a = O.random_mask_2of4(a, M, K, seed=100 + i) if square else a
        else:
            a = O.prune_magnitude_2of4(O.normal_f16(M * K, seed=i, std=wl["a_std"]), M, K)
        layers[(M, K)] = (a,)
    acts = {}
    for j, (K, N) in enumerate(sorted({(K, N) for (M, N, K) in shapes})):
        acts[(K, N)] = ((O.uniform_f16 if square else O.normal_f16)(K * N, seed=5000 + j),)
    threads = host_threads()

    def step(rows):
        fl = 0.0
        for (M, N, K) in shapes:
            r = min(rows, M)
            O.dense_gemm_f32(layers[(M, K)][0][: r * K], acts[(K, N)][0], r, N, K, threads)
            fl += flops(r, N, K)
        return fl

    t = time.perf_counter()
    step(32)
    dt = time.perf_counter() - t
    # each step ~2 s of CPU work so that --steps 20 --warmup 5 ends in about a minute
    rows = int(max(16, min(4096, 32 * 2.0 / max(dt, 1e-4))))
    for _ in range(args.warmup):
        step(rows)
    fl = 0.0
    t = time.perf_counter()
    for _ in range(args.steps):
        fl += step(rows)
    dt = time.perf_counter() - t
    value = fl / dt / 1e12
    sample = f"first {rows} rows of each of the {len(shapes)} shapes per step (dense fp32 GEMM on the pruned A)"
    print(json.dumps({
        "impl": "reference",
        "metric": "dense-equiv TFLOPS per 2:4 SpMM at LLaMA shapes (us per SpMM and % of roofline alongside)",
        "value": round(value, 6), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 in, f32 accumulate, f16 out", "data": "synthetic",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOPS", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 6), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU GEMM of its own; this is the oracle's restatement of its math "
                "(oracle/oracle.c orc_dense_gemm_f32) on all host threads",
    }), flush=True)


def run_single(args):
    """One shape, `warmup` launches then 3 more: the case profiler captures
    use (ncu -k regex:spmm24 -s <warmup> -c 3)."""
    import torch

    import spmm24

    parts = [int(x) for x in args.single.split(",")]
    M, N, K = parts[:3]
    split = parts[3] if len(parts) > 3 else 0
    dev = torch.device("cuda", 0)
    fp8 = args.dtype == "fp8"
    if fp8:
        _, vals, meta = make_layer_fp8(torch, spmm24, M, K, seed=1)
        _, bp = make_activations_fp8(torch, K, N, seed=2)
    else:
        _, vals, meta = make_layer(torch, spmm24, M, K, 0.02, seed=1)
        _, bp = make_activations(torch, spmm24, K, N, seed=2)
    A, E, B = to_dev(torch, vals, dev), to_dev(torch, meta, dev), to_dev(torch, bp, dev)
    C = torch.empty((M, N), dtype=torch.float16, device=dev)
    s = torch.cuda.current_stream(dev)
    for _ in range(args.warmup + 3):
        if fp8:
            rc = spmm24.launch_fp8(s, A, B, E, C, M, N, K, split, 0, alpha=0.02)
        else:
            rc = spmm24.launch(s, A, B, E, C, M, N, K, None, split)
        if rc != 0:
            raise SystemExit(f"launch failed {rc}")
    torch.cuda.synchronize(dev)
    print(json.dumps({"single": [M, N, K], "dtype": args.dtype,
                      "config": spmm24.select_config_fp8(M, N, K, split) if fp8 else spmm24.select_config(M, N, K, split),
                      "status": spmm24.device_status(0)}))


def run_single_group(args):
    """The decode step's 12 layers with M / DIV rows each (a rank's share of
    the step split over DIV GPUs) as one grouped launch, `warmup` launches
    then 3 more, with group_split SPLIT (0: the picker's choice): the case
    profiler captures of the grouped kernel use (ncu -k regex:spmm24_grouped
    -s <warmup> -c 1)."""
    import torch

    import spmm24

    parts = [int(x) for x in args.single_group.split(",")]
    div = parts[0]
    split = parts[1] if len(parts) > 1 else 0
    dev = torch.device("cuda", 0)
    probs, keep = [], []
    for i, (M, K) in enumerate(((4096, 4096), (11008, 4096), (4096, 11008))):
        m = spmm24.shard_rows(M, div, 0, 128)[1]
        for j, N in enumerate((1, 8, 16, 32)):
            # every problem its own weights, as in the bench step (no problem finds another's in L2)
            _, vals, meta = make_layer(torch, spmm24, m, K, 0.02, seed=1 + 4 * i + j)
            A, E = to_dev(torch, vals, dev), to_dev(torch, meta, dev)
            _, bp = make_activations(torch, spmm24, K, N, seed=10 * i + j)
            B = to_dev(torch, bp, dev)
            C = torch.empty((m, N), dtype=torch.float16, device=dev)
            probs.append((A, B, E, C, m, N, K))
            keep += [A, E, B, C]
    arr = spmm24.problem_array(probs)
    spmm24.set_tuning(group_split=split)
    s = torch.cuda.current_stream(dev)
    for _ in range(args.warmup + 3):
        rc = spmm24.launch_grouped(s, arr, spmm24.STATIC_WEIGHTS)
        if rc != 0:
            raise SystemExit(f"spmm24_launch_grouped failed {rc}: {spmm24._lib.spmm24_last_error().decode()}")
    torch.cuda.synchronize(dev)
    spmm24.reset_tuning()
    print(json.dumps({"single_group": {"rows_divisor": div, "group_split": split, "problems": len(probs)},
                      "status": spmm24.device_status(0)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["pack", "packb"], default="decode")
    ap.add_argument("--no-comparators", dest="comparators", action="store_false",
                    help="skip the same-run comparators (cuSPARSELt, dense cuBLAS, the reference kernel)")
    ap.add_argument("--no-config4", dest="config4", action="store_false",
                    help="skip the M-sharded LLaMA-70B block (config 4) of the default decode line")
    ap.add_argument("--no-secondary", dest="secondary", action="store_false",
                    help="skip the prefill / square block (configs 3 and 5) of the default decode line")
    ap.add_argument("--launch", choices=["grouped", "chain"], default="grouped",
                    help="a step as one spmm24_launch_grouped (N <= 32 workloads without an epilogue or fp8) "
                         "or as one spmm24_launch per SpMM")
    ap.add_argument("--allgather", action="store_true", help="70b workload: also time the NCCL all-gather of C")
    ap.add_argument("--gather-mc", dest="gather_mc", action="store_true",
                    help="sharded decode on N > 1 GPUs: store the gathered rows through the full C's NVLink "
                         "multicast address (symmetric memory) instead of once per peer")
    ap.add_argument("--gather", action="store_true",
                    help="70b workload: time the fused SpMM + NVLink all-gather against SpMM + NCCL all-gather")
    ap.add_argument("--no-static-weights", dest="static_weights", action="store_false",
                    help="launch without SPMM24_STATIC_WEIGHTS (no kernel in the step writes the weights)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", dest="extras", action="store_false",
                    help="skip the extras block of the default decode line (fp8 decode, fused epilogue, device "
                         "packers, each as a child run)")
    ap.add_argument("--dtype", choices=["f16", "bf16", "fp8"], default="f16",
                    help="operand and output type (SPMM24_BF16; fp8: E4M3 operands through spmm24_launch_fp8, fp16 out)")
    ap.add_argument("--epilogue", choices=["none", "bias_silu", "bias_residual", "packed_b"], default="none",
                    help="fused epilogue through spmm24_launch_fused (packed_b: C written as the next layer's "
                         "packed B, SPMM24_OUT_PACKED_B)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--single", default=None,
                    help="M,N,K[,split]: run one shape (warm-up + 3 launches) for profiler captures")
    ap.add_argument("--single-group", dest="single_group", default=None,
                    help="DIV[,SPLIT]: the decode step's layers with M / DIV rows as one grouped launch (warm-up + "
                         "3 launches, group_split SPLIT) for profiler captures")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.single:
        run_single(args)
        return
    if args.single_group:
        run_single_group(args)
        return
    if args.workload == "pack":
        run_pack(args, rank, world, local_rank)
        return
    if args.workload == "packb":
        run_pack_b(args, rank, world, local_rank)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
