"""spmm24_launch_grouped: several independent narrow-N SpMMs in one
persistent launch, against the oracle and against one spmm24_launch per
problem (split_k = 1: the same MMAs in the same K order, so the same bits).
Tolerance: tests/problems.py."""
import numpy as np
import pytest

from problems import compare, make_problem, oracle_c, within_tolerance

pytestmark = pytest.mark.gpu


def _dev(torch, arr, dev):
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).to(dev)


def _upload(torch, p, dev, bf16=False):
    C = torch.full((p.M, p.N), float("nan"), dtype=torch.bfloat16 if bf16 else torch.float16, device=dev)
    return {"A": _dev(torch, p.vals, dev), "E": _dev(torch, p.meta, dev), "B": _dev(torch, p.b_packed, dev), "C": C}


def _bits(t):
    import torch

    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _grouped(dev, probs, flags=0, stream=None):
    import torch

    import spmm24

    bufs = [_upload(torch, p, dev) for p in probs]
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    rc = spmm24.launch_grouped(s, [(b["A"], b["B"], b["E"], b["C"], p.M, p.N, p.K) for b, p in zip(bufs, probs)],
                               flags)
    assert rc == 0, spmm24._lib.spmm24_last_error().decode()
    torch.cuda.synchronize(dev)
    return bufs, [_bits(b["C"]) for b in bufs]


def _single(dev, p, bufs, split_k=1):
    import torch

    import spmm24

    C = torch.full((p.M, p.N), float("nan"), dtype=torch.float16, device=dev)
    assert spmm24.launch(torch.cuda.current_stream(dev), bufs["A"], bufs["B"], bufs["E"], C, p.M, p.N, p.K, None,
                         split_k) == 0
    torch.cuda.synchronize(dev)
    return _bits(C)


SHAPES = [
    (4096, 1, 1024),   # N = 1
    (1024, 8, 4096),
    (144, 12, 320),    # ragged M tile, ragged N, odd 64-K group count
    (16, 16, 64),      # one band, one (odd) group
    (768, 24, 704),    # N not a multiple of 8 above 16
    (2048, 32, 2048),
    (384, 17, 192),
]


@pytest.mark.parametrize("group_split", [1, 2, 4])
def test_grouped_mixed_shapes(cuda_device, tuning, group_split):
    """Whole tiles (group_split 1) or each tile's K over a cluster of 2 or 4
    CTAs: against the oracle, and bit for bit against spmm24_launch with
    split_k = group_split (the same K shares added in the same order; tiles
    of fewer stages than CTAs leave the last CTAs without a share)."""
    tuning(group_split=group_split)
    probs = [make_problem(M, N, K, seed=3 * M + N + K, a_scale=0.05, b_dist="normal") for (M, N, K) in SHAPES]
    bufs, outs = _grouped(cuda_device, probs)
    for p, b, got in zip(probs, bufs, outs):
        stats = compare(got, oracle_c(p))
        assert within_tolerance(stats), ((p.M, p.N, p.K), stats)
        assert np.array_equal(got, _single(cuda_device, p, b, group_split)), (p.M, p.N, p.K)


@pytest.mark.parametrize("group_split", [0, 2, 4])
def test_grouped_many_tiles_per_cta(cuda_device, tuning, group_split):
    """More tiles than SMs (630 here): every CTA (or cluster) walks several
    tiles of several problems and both TMEM accumulators (and both receive
    slots of every pushing CTA) alternate; a second launch of the same
    problem array reuses the cached launch and gives the same bits."""
    import spmm24

    tuning(group_split=group_split)
    shapes = [(65536, 8, 256), (4096, 16, 1024), (11008, 32, 512)]
    probs = [make_problem(M, N, K, seed=M + N, a_scale=0.05, b_dist="normal") for (M, N, K) in shapes]
    bufs, outs = _grouped(cuda_device, probs, flags=spmm24.STATIC_WEIGHTS)
    for p, got in zip(probs, outs):
        rows = np.unique(np.linspace(0, p.M - 1, 300).astype(int))
        stats = compare(got.reshape(p.M, p.N)[rows], oracle_c(p, rows))
        assert within_tolerance(stats), ((p.M, p.N, p.K), stats)
    import torch

    s = torch.cuda.current_stream(cuda_device)
    arr = spmm24.problem_array([(b["A"], b["B"], b["E"], b["C"], p.M, p.N, p.K) for b, p in zip(bufs, probs)])
    for b in bufs:
        b["C"].fill_(float("nan"))
    assert spmm24.launch_grouped(s, arr, spmm24.NO_PDL) == 0
    assert spmm24.launch_grouped(s, arr, 0) == 0
    torch.cuda.synchronize(cuda_device)
    for b, got in zip(bufs, outs):
        assert np.array_equal(_bits(b["C"]), got)
    assert spmm24.device_status(0) == 0


def test_grouped_llama_decode_layers(cuda_device):
    """The BASELINE config-2 decode step (LLaMA-7B, N in {1, 8, 16, 32}) as one
    grouped launch, checked on a row sample of every layer."""
    probs = [make_problem(M, N, K, seed=M + 7 * N + K, a_scale=0.02, b_dist="normal")
             for (M, K) in ((4096, 4096), (11008, 4096), (4096, 11008)) for N in (1, 8, 16, 32)]
    _, outs = _grouped(cuda_device, probs)
    for p, got in zip(probs, outs):
        rows = np.unique(np.linspace(0, p.M - 1, 64).astype(int))
        stats = compare(got.reshape(p.M, p.N)[rows], oracle_c(p, rows))
        assert within_tolerance(stats), ((p.M, p.N, p.K), stats)


def test_grouped_bf16(cuda_device):
    import torch

    import oracle as O
    import spmm24

    probs = []
    for i, (M, N, K) in enumerate([(512, 16, 1024), (256, 32, 512), (128, 5, 256)]):
        a = O.prune_magnitude_2of4_bf16(O.f32_to_bf16_bits(np.random.default_rng(i).standard_normal(M * K)
                                                            .astype(np.float32) * 0.1), M, K)
        b = O.f32_to_bf16_bits(np.random.default_rng(100 + i).standard_normal(K * N).astype(np.float32))
        from problems import pack_problem

        probs.append(pack_problem(M, N, K, a, b))
    bufs = [_upload(torch, p, cuda_device, bf16=True) for p in probs]
    rc = spmm24.launch_grouped(torch.cuda.current_stream(cuda_device),
                               [(b["A"], b["B"], b["E"], b["C"], p.M, p.N, p.K) for b, p in zip(bufs, probs)],
                               spmm24.BF16)
    assert rc == 0, spmm24._lib.spmm24_last_error().decode()
    torch.cuda.synchronize(cuda_device)
    for p, b in zip(probs, bufs):
        ref = O.dense_gemm_bf16_f32(p.a_dense, p.b_rowmajor, p.M, p.N, p.K)
        ref_bits = O.f32_to_bf16_bits(ref)
        got = _bits(b["C"]).reshape(-1)
        g = (got.astype(np.uint32) << 16).view(np.float32)
        r = (ref_bits.astype(np.uint32) << 16).view(np.float32)
        scale = np.max(np.abs(r))
        assert np.all(np.isfinite(g))
        assert np.max(np.abs(g - r) / np.maximum(np.abs(r), 1e-3 * scale)) <= 1e-2


def test_grouped_dependent_chain_pdl(cuda_device):
    """Grouped launches where each launch's output is the next one's input
    (N = 8: an M x 8 row-major C is the packed B of the next layer, K' = M),
    with static weights and programmatic dependent launch."""
    import torch

    import spmm24

    K0, N = 1024, 8
    sizes = [(1024, K0), (2048, 1024), (1024, 2048)]
    probs = [make_problem(M, N, K, seed=50 + M, a_scale=0.03, b_dist="normal") for (M, K) in sizes]
    dev = cuda_device
    A = [_dev(torch, p.vals, dev) for p in probs]
    E = [_dev(torch, p.meta, dev) for p in probs]
    x = _dev(torch, probs[0].b_packed, dev)
    outs = [torch.empty((M, N), dtype=torch.float16, device=dev) for (M, K) in sizes]
    s = torch.cuda.current_stream(dev)
    for i, (M, K) in enumerate(sizes):
        src = x if i == 0 else outs[i - 1]
        rc = spmm24.launch_grouped(s, [(A[i], src, E[i], outs[i], M, N, K)], spmm24.STATIC_WEIGHTS)
        assert rc == 0
    torch.cuda.synchronize(dev)
    # host chain through the oracle on the GPU's own intermediate outputs
    import oracle as O

    prev = probs[0].b_rowmajor
    for i, (M, K) in enumerate(sizes):
        ref = O.dense_gemm_f32(probs[i].a_dense, prev, M, N, K)
        got = _bits(outs[i]).reshape(-1)
        assert within_tolerance(compare(got, ref)), i
        prev = got


def test_grouped_cuda_graph(cuda_device):
    import torch

    import spmm24

    probs = [make_problem(M, N, K, seed=M + K) for (M, N, K) in ((512, 16, 512), (256, 8, 1024))]
    bufs = [_upload(torch, p, cuda_device) for p in probs]
    arr = spmm24.problem_array([(b["A"], b["B"], b["E"], b["C"], p.M, p.N, p.K) for b, p in zip(bufs, probs)])
    s = torch.cuda.Stream(cuda_device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        assert spmm24.launch_grouped(s, arr, 0) == 0  # warm-up outside capture
        torch.cuda.synchronize(cuda_device)
        for b in bufs:
            b["C"].fill_(float("nan"))
        with torch.cuda.graph(g, stream=s):
            assert spmm24.launch_grouped(s, arr, 0) == 0
    g.replay()
    torch.cuda.synchronize(cuda_device)
    for p, b in zip(probs, bufs):
        assert within_tolerance(compare(_bits(b["C"]), oracle_c(p)))


@pytest.mark.parametrize("group_split", [1, 2, 4])
def test_grouped_epilogues_match_fused_launches(cuda_device, tuning, group_split):
    """Each problem of a group with its own epilogue (bias + SiLU, alpha +
    GELU, a residual, a packed-B output, none): bit for bit the results of
    spmm24_launch_fused with split_k = group_split (the same accumulator,
    the same epilogue code), in fp16 and bf16."""
    import torch

    import spmm24

    tuning(group_split=group_split)
    dev = cuda_device
    cases = [((512, 16, 1024), dict(bias=True, act=spmm24.ACT_SILU)),
             ((256, 32, 512), dict(alpha=0.5, act=spmm24.ACT_GELU)),
             ((384, 24, 704), dict(residual=True, bias=True, act=spmm24.ACT_RELU)),
             ((256, 12, 256), dict(packed=True, alpha=-0.25)),
             ((144, 8, 320), dict()),
             ((1024, 1, 512), dict(bias=True))]
    for bf16 in (False, True):
        dt = torch.bfloat16 if bf16 else torch.float16
        flags = spmm24.BF16 if bf16 else 0
        probs, refs, outs, keep = [], [], [], []
        for i, ((M, N, K), kw) in enumerate(cases):
            p = make_problem(M, N, K, seed=17 * i + M, a_scale=0.05, b_dist="normal")
            b = _upload(torch, p, dev)
            strips = (N + 7) // 8
            size = strips * 8 * M if kw.get("packed") else M * N
            bias = torch.randn(M, device=dev).to(dt) if kw.get("bias") else None
            res = torch.randn(size, device=dev).to(dt) if kw.get("residual") else None
            epi = spmm24.Epilogue(bias.data_ptr() if bias is not None else None,
                                  res.data_ptr() if res is not None else None, kw.get("alpha", 1.0),
                                  kw.get("act", spmm24.ACT_NONE),
                                  spmm24.OUT_PACKED_B if kw.get("packed") else spmm24.OUT_ROW_MAJOR)
            c_g = torch.full((size,), -1, dtype=torch.int16, device=dev)
            c_r = torch.full((size,), -1, dtype=torch.int16, device=dev)
            rc = spmm24.launch_fused(None, b["A"], b["B"], b["E"], c_r, M, N, K, group_split, flags, bias=bias,
                                     residual=res,
                                     alpha=kw.get("alpha", 1.0), activation=kw.get("act", spmm24.ACT_NONE),
                                     out_layout=spmm24.OUT_PACKED_B if kw.get("packed") else spmm24.OUT_ROW_MAJOR)
            assert rc == 0, spmm24._lib.spmm24_last_error().decode()
            probs.append((b["A"], b["B"], b["E"], c_g, M, N, K, None, epi))
            refs.append(c_r)
            outs.append(c_g)
            keep += [b, bias, res]
        assert spmm24.launch_grouped(None, probs, flags) == 0, spmm24._lib.spmm24_last_error().decode()
        torch.cuda.synchronize(dev)
        for (shape, kw), r, g in zip(cases, refs, outs):
            assert torch.equal(r, g), (bf16, shape, kw)
        assert spmm24.device_status(0) == 0


@pytest.mark.parametrize("group_split", [1, 2, 4])
def test_grouped_fp8_matches_fp8_launches(cuda_device, tuning, group_split):
    """spmm24_launch_grouped_fp8: E4M3 and E5M2 operands, alpha per problem,
    bias / activation / residual / packed output: bit for bit the results of
    spmm24_launch_fp8 with split_k = group_split; one problem also against
    the oracle (fp8 decode, fp32 GEMM; bound of tests/test_gpu_fp8.py)."""
    import torch

    import oracle as O
    import spmm24
    from test_gpu_fp8 import _problem

    tuning(group_split=group_split)
    dev = cuda_device
    cases = [((512, 16, 1024), dict(alpha=0.02)),
             ((256, 32, 512), dict(alpha=0.5, bias=True, act=spmm24.ACT_SILU)),
             ((384, 24, 1152), dict(residual=True, alpha=1.0)),
             ((256, 8, 256), dict(packed=True, alpha=2.0)),
             ((1024, 1, 2048), dict(alpha=0.125))]
    for fmt_a, fmt_b in ((0, 0), (1, 0), (0, 1)):
        flags = (spmm24.FP8_A_E5M2 if fmt_a else 0) | (spmm24.FP8_B_E5M2 if fmt_b else 0)
        probs, refs, outs, keep, accs = [], [], [], [], []
        for i, ((M, N, K), kw) in enumerate(cases):
            vals, meta, b_bits, acc, S = _problem(M, N, K, fmt_a, fmt_b, seed=31 * i + M + fmt_a + 2 * fmt_b)
            A = torch.from_numpy(np.ascontiguousarray(vals)).to(dev)
            E = torch.from_numpy(np.ascontiguousarray(meta)).to(dev)
            B = torch.from_numpy(np.ascontiguousarray(b_bits)).to(dev)
            strips = (N + 7) // 8
            size = strips * 8 * M if kw.get("packed") else M * N
            bias = torch.randn(M, device=dev).half() if kw.get("bias") else None
            res = torch.randn(size, device=dev).half() if kw.get("residual") else None
            act = kw.get("act", spmm24.ACT_NONE)
            layout = spmm24.OUT_PACKED_B if kw.get("packed") else spmm24.OUT_ROW_MAJOR
            epi = spmm24.Epilogue(bias.data_ptr() if bias is not None else None,
                                  res.data_ptr() if res is not None else None, kw["alpha"], act, layout)
            c_g = torch.full((size,), -1, dtype=torch.int16, device=dev)
            c_r = torch.full((size,), -1, dtype=torch.int16, device=dev)
            rc = spmm24.launch_fp8(None, A, B, E, c_r, M, N, K, group_split, flags, bias=bias, residual=res,
                                   alpha=kw["alpha"], activation=act, out_layout=layout)
            assert rc == 0, spmm24._lib.spmm24_last_error().decode()
            probs.append((A, B, E, c_g, M, N, K, None, epi))
            refs.append(c_r)
            outs.append(c_g)
            keep += [A, B, E, bias, res]
            accs.append((acc, S))
        assert spmm24.launch_grouped(None, probs, flags, fp8=True) == 0, spmm24._lib.spmm24_last_error().decode()
        torch.cuda.synchronize(dev)
        for (shape, kw), r, g in zip(cases, refs, outs):
            assert torch.equal(r, g), (fmt_a, fmt_b, shape, kw)
        # the first problem against the oracle: alpha * acc rounded to fp16
        (M, N, K), kw = cases[0]
        acc, S = accs[0]
        got = outs[0].cpu().numpy().view(np.uint16).view(np.float16).astype(np.float64).reshape(M, N)
        ref = (kw["alpha"] * acc).astype(np.float32).astype(np.float16).astype(np.float64)
        tol = 2.0 ** -10 * np.abs(ref) + 1.2 * kw["alpha"] * 2.0 ** -12 * S + 1e-6
        assert np.all(np.abs(got - ref) <= tol)
        assert spmm24.device_status(0) == 0
