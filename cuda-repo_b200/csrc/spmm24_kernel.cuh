// spmm24_kernel.cuh -- the sm_100a 2:4 sparse SpMM kernels, C = A_sparse * B.
//
// Replace SpMM_N2M4_Kernel (SpeakOutLoudly/CUDA-Repo src/SpMM_Kernel.cuh:301)
// and the separate split-K pass SplitK_Reduction (src/reduce_Kernel.cuh:27).
// Formats and the tcgen05 mapping are described in spmm24_common.cuh.
//
// Four kernels share the stage layout and the MMA issue:
//
//   spmm24_cluster_kernel  one 128 x N_TILE tile per CTA; a split-K request
//       of S becomes a thread-block cluster of S CTAs along K whose fp32
//       partial tiles are reduce-scattered through distributed shared memory
//       (no global workspace, no second launch, fixed summation order).
//
//   spmm24_pair_kernel  a CTA pair (cluster of 2) computing one 256 x 256
//       tile with tcgen05.mma.sp.cta_group::2: each CTA holds 128 rows of A
//       and half of the tile's columns of B, so each SM feeds the tensor
//       core only half of B -- the prefill (compute-bound) path.  With a K
//       split, a cluster of two pairs takes the two halves of K and pair 1
//       sends its partial accumulator to pair 0 through distributed shared
//       memory.
//
//   spmm24_pair2_kernel  a CTA pair computing a 512 x 240 tile: each CTA
//       holds two 128-row halves of A and 120 columns of B, and the leader
//       issues two M=256 MMAs per K step that share the B tile -- 1.87x the
//       FLOPs per stage for 1.33x the bytes of the 256 x 256 pair, chosen for
//       wide N when its waves of pairs cost less.
//
//   spmm24_streamk_kernel  a persistent grid (one CTA per SM) in which every
//       CTA takes an equal share of the (tile, 128-K stage) units, walked
//       tile-major.  A tile shared by several CTAs is finished by the CTA
//       that holds its first unit; every other contributor starts its range
//       inside that tile, so it processes its share first and publishes the
//       fp32 partial (global workspace slot + release flag) early.  The
//       finisher's epilogue warps collect the published partials while its
//       own last segment is still streaming, so the end of the kernel only
//       adds the accumulator and stores.  Summation order is fixed.
//
// The cluster and pair kernels come in two instantiations: the plain fp16
// row-major SpMM, and EPI (alpha, bias, activation, residual, bf16, packed
// output, fused all-gather), kept apart because the epilogue of every tile
// is on the critical path.  All but stream-K also come in an FP8 form (OCP
// E4M3 / E5M2 operands, tcgen05.mma.sp kind::f8f6f4, stages of 256 K).
//
// Roles (192 threads; the pair kernel 256):
//   warp 0     TMA producer (lane 0)
//   warp 1     TMEM allocator, tcgen05.cp + tcgen05.mma issuer (lane 0)
//   warps 2-5  epilogue: TMEM -> registers -> stores (in the pair kernel
//              every warp joins the epilogue once its role is done)
// Every wait is bounded; the producer starts before TMEM is allocated; the
// kernels take part in programmatic dependent launch (they wait for the
// previous grid before touching global memory it may write, and let the
// next grid start launching early).
#pragma once
#include "spmm24_common.cuh"

namespace spmm24 {

constexpr int kThreads = 192;     // 6 warps
constexpr int kEpiThreads = 128;  // warps 2..5
// The pair kernel runs 8 warps: after the main loop every warp joins the
// epilogue, two warps per TMEM lane quadrant (each takes half the columns),
// because the epilogue -- on the critical path of every tile -- is bound by
// instruction latency, not bandwidth.
constexpr int kPairThreads = 256;
constexpr uint32_t kBarEpi = 1;   // named barrier: epilogue warps
constexpr uint32_t kBarTmem = 2;  // named barrier: warps 1..5 after TMEM allocation

struct ClusterParams {
    uint16_t* C;  // fp16 or bf16 elements (epi.bf16), row-major or packed (epi.packed)
    int M, N, K;
    int groups;        // K / 64 (fp8: K / 128, the metadata groups)
    int stages_total;  // ceil(groups / 2)
    int split;         // CTAs per cluster along K
    int weights_static;
    uint32_t mma_fmt;  // fp8 kernel: operand-format bits of the instruction descriptor
    Epilogue epi;
    SPMM24_TRACE_FIELD
};

struct PairParams {
    uint16_t* C;  // fp16 or bf16 elements (epi.bf16), row-major or packed (epi.packed)
    int M, N, K;
    int stages_total;  // K / 128 (the pair kernel requires K % 128 == 0)
    int weights_static;
    int split;         // pairs per cluster along K (1 or 2)
    uint32_t mma_fmt;  // fp8 kernel: operand-format bits of the instruction descriptor
    Epilogue epi;
    SPMM24_TRACE_FIELD
};

struct StreamKParams {
    __half* C;
    float* ws;        // one partial tile (128 x N_TILE fp32) per CTA
    uint32_t* flags;  // one per CTA: 1 = its partial is published; zero between launches
    int M, N, K;
    int groups;           // K / 64
    int stages_per_tile;  // ceil(groups / 2)
    int m_tiles, n_tiles;
    long long units;      // tiles * stages_per_tile
    int grid;
    int weights_static;
    SPMM24_TRACE_FIELD
};

// -------------------------------------------------------------------------
template <int N_TILE, int STAGES, bool FP8 = false>
struct ClusterCfg : Cfg<N_TILE, STAGES, 1, FP8> {
    using B_ = Cfg<N_TILE, STAGES, 1, FP8>;
    static constexpr int RED_PITCH = N_TILE + 4;  // floats per row of the reduction buffer
    static constexpr int RED_ROWS = 136;          // >= S * ceil(128 / S) for every S <= 8
    // Narrow tiles get a dedicated receive buffer, so partial rows can be
    // pushed to their owner with st.async as soon as the sender is done; wide
    // tiles reuse the idle stage ring behind two cluster barriers.
    static constexpr bool RECV_BUF = N_TILE <= 32;
    static constexpr int RECV_OFFSET = B_::RING_BYTES;
    static constexpr int RECV_BYTES = RECV_BUF ? RED_ROWS * RED_PITCH * 4 : 0;
    static constexpr int BAR_OFFSET = RECV_OFFSET + RECV_BYTES;
    static constexpr int NUM_BARS = 2 * STAGES + 2;  // full, empty, acc_full, recv
    static constexpr int HOLDER_OFFSET = BAR_OFFSET + NUM_BARS * 8;
    static constexpr int BIAS_OFFSET = HOLDER_OFFSET + 16;  // the owner rows' bias, prefetched (EPI)
    // Narrow tiles: the owner rows' residual, prefetched (EPI, 16-byte layouts).
    static constexpr int RES_OFFSET = BIAS_OFFSET + kTileM * 4;
    static constexpr int RES_BYTES = N_TILE <= 32 ? kTileM * N_TILE * 2 : 0;
    static constexpr int SMEM_BYTES = RES_OFFSET + RES_BYTES;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to align the base to 1024 B
    // CTAs that fit on one SM (228 KB, 1 KB reserved per CTA), at most 4.
    static constexpr int CTAS_PER_SM = 233472 / (SMEM_ALLOC + 1024) < 4 ? 233472 / (SMEM_ALLOC + 1024) : 4;
    static_assert(SMEM_ALLOC <= 232448, "shared memory overflow");
    static_assert(RECV_BUF || RED_ROWS * RED_PITCH * 4 <= B_::RING_BYTES, "reduction buffer does not fit");
    static_assert(CTAS_PER_SM * B_::TMEM_COLS <= 512, "co-resident CTAs must fit in TMEM together");
};

// EPI: the general epilogue (bias, activation, residual, alpha, bf16, packed
// output).  The plain fp16 row-major SpMM is a separate instantiation
// without it: the epilogue runs on the critical path at the end of every
// tile, and its extra code measurably slows the plain kernel.
// FP8: the fp8 operand formats and kind::f8f6f4 MMAs; without EPI the
// output is alpha * acc rounded to fp16, row-major (the dequantisation
// scale alone).
template <int N_TILE, int STAGES, bool EPI, bool FP8 = false>
__global__ void __launch_bounds__(kThreads, ClusterCfg<N_TILE, STAGES, FP8>::CTAS_PER_SM)
spmm24_cluster_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmE, const ClusterParams p) {
    using C_ = ClusterCfg<N_TILE, STAGES, FP8>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C_::BAR_OFFSET);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* recv_bar = acc_full + 1;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C_::HOLDER_OFFSET);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int S = p.split;
    const int rank = (S > 1) ? (int)ptx::cluster_ctarank() : 0;
    const int rows_per = (kTileM + S - 1) / S;
    const int my_start = (kTileM * rank + S - 1) / S;
    const int my_end = (kTileM * (rank + 1) + S - 1) / S;
    const int n_tile = blockIdx.y;
    const int m_tile = blockIdx.z;
    const int band0 = m_tile * (kTileM / 16);
    const int strip0 = n_tile * (N_TILE / 8);

    // This CTA's share of the K stages (each stage = two 64-K groups).
    const int st_base = p.stages_total / S, st_rem = p.stages_total % S;
    const int st_begin = rank * st_base + min(rank, st_rem);
    const int st_count = st_base + (rank < st_rem ? 1 : 0);

    if (threadIdx.x == 0) {
        SPMM24_STAMP(0);
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        ptx::mbar_init(acc_full, 1);
        ptx::mbar_init(recv_bar, 1);
        if (C_::RECV_BUF && S > 1)  // the other S-1 CTAs' partial rows of this CTA's slice
            ptx::mbar_arrive_expect_tx(recv_bar, (uint32_t)((S - 1) * (my_end - my_start) * N_TILE * 4));
        ptx::fence_mbarrier_init();
        ptx::prefetch_tmap(&tmA);
        ptx::prefetch_tmap(&tmB);
        ptx::prefetch_tmap(&tmE);
    }
    __syncthreads();
    // With a receive buffer, partial rows may arrive from the other CTAs of
    // the cluster at any time from here on, so every CTA's barriers must be
    // initialised first (the CTAs of a cluster start together: this costs one
    // barrier round trip, spent while the previous grid is still finishing).
    if (C_::RECV_BUF && S > 1) ptx::cluster_sync();
    if (threadIdx.x == 0) ptx::grid_dep_launch();

    uint32_t tmem_base = 0;
    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            const uint64_t pol_stream = ptx::policy_evict_first();  // A, E: read once
            const uint64_t pol_keep = ptx::policy_evict_last();     // B: re-read by every M tile
            const int pre = p.weights_static ? min(STAGES, st_count) : 0;
            for (int it = 0; it < pre; ++it) {  // weights of the first stages before the previous grid ends
                uint8_t* st = smem + it * C_::STAGE_BYTES;
                ptx::mbar_arrive_expect_tx(&full[it], C_::STAGE_BYTES);
                load_stage_weights<C_>(st, &full[it], &tmA, &tmE, band0, 2 * (st_begin + it), pol_stream);
            }
            ptx::grid_dep_wait();
            SPMM24_STAMP(1);
            for (int it = 0; it < pre; ++it)
                load_stage_acts<C_>(smem + it * C_::STAGE_BYTES, &full[it], &tmB, strip0, 2 * (st_begin + it), pol_keep);
            for (int it = pre; it < st_count; ++it) {
                const int s = it % STAGES;
                const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                if (!ptx::mbar_wait_bounded(&empty[s], ph ^ 1u, kWaitLimitNs)) {
                    atomicOr(&g_spmm24_status, kStatusProducerTimeout);
                    break;
                }
                uint8_t* st = smem + s * C_::STAGE_BYTES;
                const int g0 = 2 * (st_begin + it);
                ptx::mbar_arrive_expect_tx(&full[s], C_::STAGE_BYTES);
                load_stage_weights<C_>(st, &full[s], &tmA, &tmE, band0, g0, pol_stream);
                load_stage_acts<C_>(st, &full[s], &tmB, strip0, g0, pol_keep);
            }
        }
        __syncwarp();
    } else {
        if (warp == 1) {
            ptx::tmem_alloc(tmem_holder, C_::TMEM_COLS);
            ptx::tmem_relinquish();
        }
        ptx::tc_fence_before();
        ptx::named_barrier(kBarTmem, kThreads - 32);
        ptx::tc_fence_after();
        tmem_base = *tmem_holder;
    }
    // The epilogue warps are idle until the accumulator is ready: with a bias
    // (or, for narrow tiles, a residual in a 16-byte layout), they wait for the
    // previous grid now and bring this CTA's owner rows of it into shared
    // memory, off the critical path at the end.
    float* bias_s = reinterpret_cast<float*>(smem + C_::BIAS_OFFSET);
    uint4* res_s = reinterpret_cast<uint4*>(smem + C_::RES_OFFSET);  // [owner row][16-byte chunk]
    const bool res_pre = EPI && C_::RES_BYTES > 0 && p.epi.residual && !p.epi.gather_n &&
                         (p.epi.packed || ((p.N % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0)));
    if constexpr (EPI) {
        if (warp >= 2 && (p.epi.bias || res_pre)) {
            ptx::grid_dep_wait();
            const int m_first = m_tile * kTileM + my_start;
            const int nrows = my_end - my_start;
            if (p.epi.bias)
                for (int t = threadIdx.x - 64; t < nrows; t += kEpiThreads)
                    bias_s[t] = m_first + t < p.M ? elem_to_f32(p.epi.bias[m_first + t], p.epi.bf16) : 0.f;
            if constexpr (C_::RES_BYTES > 0) {
                if (res_pre) {
                    constexpr int CH = N_TILE / 8;
                    for (int t = threadIdx.x - 64; t < nrows * CH; t += kEpiThreads) {
                        const int gm = m_first + t / CH, gn = n_tile * N_TILE + (t % CH) * 8;
                        if (gm < p.M && gn < p.N)
                            res_s[t] = *reinterpret_cast<const uint4*>(p.epi.residual + c_offset(p.epi, gm, gn, p.M, p.N));
                    }
                }
            }
        }
    }

    if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        const uint32_t smem_base = ptx::smem_u32(smem);
        uint32_t accumulate = 0;
        for (int it = 0; it < st_count; ++it) {
            const int s = it % STAGES;
            const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
            if (!ptx::mbar_wait_bounded(&full[s], ph, kWaitLimitNs)) {
                if (lane == 0) atomicOr(&g_spmm24_status, kStatusMmaTimeout);
                break;
            }
            if (lane == 0 && it == 0) SPMM24_STAMP(2);
            if (lane == 0 && it == st_count - 1) SPMM24_STAMP(3);
            ptx::tc_fence_after();
            if (2 * (st_begin + it) + 1 >= p.groups) patch_tail_metadata<C_>(smem + s * C_::STAGE_BYTES, lane);
            if (lane == 0) {
                if constexpr (FP8)
                    mma_stage_fp8<C_, N_TILE>(smem_base + s * C_::STAGE_BYTES,
                                              tmem_base + C_::META_COL + C_::META_STRIDE * s, tmem_base, accumulate,
                                              p.mma_fmt);
                else
                    mma_stage<C_, N_TILE>(smem_base + s * C_::STAGE_BYTES, tmem_base + C_::META_COL + 4 * s,
                                          tmem_base, accumulate, (EPI && p.epi.bf16) ? kIdescBf16 : 0u);
                ptx::tc_commit(&empty[s]);
            }
            __syncwarp();
        }
        if (lane == 0) ptx::tc_commit(acc_full);
        __syncwarp();
    }

    // ----------------------------------------------------------- epilogue
    // Reduction buffer red[src][row][RED_PITCH] (fp32): the dedicated receive
    // buffer for narrow tiles, else the stage ring once it is idle.
    float* red = reinterpret_cast<float*>(smem + (C_::RECV_BUF ? C_::RECV_OFFSET : 0));
    const bool epi = warp >= 2;
    const bool push = C_::RECV_BUF && S > 1;  // st.async to the owners, no cluster barriers
    if (epi) {
        if (!ptx::mbar_wait_bounded(acc_full, 0, kWaitLimitNs)) atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
        if (threadIdx.x == 64) SPMM24_STAMP(4);
        ptx::tc_fence_after();
    }
    __syncwarp();
    if (S > 1 && !push) ptx::cluster_sync();  // every CTA's accumulator is final and its ring is idle
    if (epi) {
        const int quad = warp & 3;  // TMEM lane quadrant this warp may access
        const int row = quad * 32 + lane;
        const int owner = (row * S) / kTileM;
        const int owner_start = (kTileM * owner + S - 1) / S;
        const int lr = row - owner_start;
        float* dst_row = red + ((size_t)rank * rows_per + lr) * C_::RED_PITCH;
        const uint32_t dst_local = ptx::smem_u32(dst_row);
        const bool remote = S > 1 && owner != rank;
        const uint32_t dst = remote ? ptx::mapa_shared(dst_local, (uint32_t)owner) : dst_local;
        const uint32_t dst_bar = remote ? ptx::mapa_shared(ptx::smem_u32(recv_bar), (uint32_t)owner) : 0u;
#pragma unroll 1
        for (int c = 0; c < N_TILE / 16; ++c) {
            uint32_t v[16];
            ptx::tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(c * 16), v);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float a = __uint_as_float(v[4 * q]), b = __uint_as_float(v[4 * q + 1]);
                const float cc = __uint_as_float(v[4 * q + 2]), d = __uint_as_float(v[4 * q + 3]);
                if (remote && push) {
                    ptx::st_async_v4(dst + (uint32_t)((c * 16 + q * 4) * 4), a, b, cc, d, dst_bar);
                } else if (remote) {
                    ptx::st_cluster_v4(dst + (uint32_t)((c * 16 + q * 4) * 4), a, b, cc, d);
                } else {
                    *reinterpret_cast<float4*>(dst_row + c * 16 + q * 4) = make_float4(a, b, cc, d);
                }
            }
        }
        ptx::tc_fence_before();
    }
    __syncwarp();
    if (S > 1 && !push) {
        ptx::cluster_sync();  // all partial rows delivered to their owners
    } else if (epi) {
        ptx::named_barrier(kBarEpi, kEpiThreads);  // this CTA's own rows are in the buffer
        if (push && !ptx::mbar_wait_bounded(recv_bar, 0, kWaitLimitNs))  // and every other CTA's
            atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
    }
    if (epi) {
        ptx::grid_dep_wait();  // C may be read or written by the previous grid
        // Owner side: sum the S partial copies of this CTA's rows in a fixed
        // order, apply the epilogue, round and store with 16-byte coalesced
        // writes (row-major C: consecutive threads take consecutive column
        // chunks of a row; packed C: consecutive rows of a strip).
        const int nrows = my_end - my_start;
        constexpr int CHUNKS = N_TILE / 8;
        const int m0 = m_tile * kTileM;
        const int n0 = n_tile * N_TILE;
        const bool vec_ok = (p.N % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0);
        const bool packed = EPI && p.epi.packed;
        for (int w = threadIdx.x - 64; w < nrows * CHUNKS; w += kEpiThreads) {
            const int lr = packed ? w % nrows : w / CHUNKS;
            const int ch = packed ? w / nrows : w % CHUNKS;
            float acc[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = 0.f;
            for (int src = 0; src < S; ++src) {
                const float* r = red + ((size_t)src * rows_per + lr) * C_::RED_PITCH + ch * 8;
                const float4 x0 = *reinterpret_cast<const float4*>(r);
                const float4 x1 = *reinterpret_cast<const float4*>(r + 4);
                acc[0] += x0.x; acc[1] += x0.y; acc[2] += x0.z; acc[3] += x0.w;
                acc[4] += x1.x; acc[5] += x1.y; acc[6] += x1.z; acc[7] += x1.w;
            }
            const int gm = m0 + my_start + lr;
            const int gn = n0 + ch * 8;
            if (gm >= p.M || gn >= p.N) continue;
            if constexpr (EPI) {
                epilogue_store8(p.C, acc, p.epi, gm, gn, p.M, p.N, vec_ok, epilogue_is_plain(p.epi),
                                p.epi.bias ? bias_s + lr : nullptr, res_pre ? res_s + lr * CHUNKS + ch : nullptr);
            } else {
                if constexpr (FP8) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[e] *= p.epi.alpha;
                }
                store_h8(reinterpret_cast<__half*>(p.C) + (size_t)gm * p.N + gn, acc, vec_ok, p.N - gn);
            }
        }
    }

    if (threadIdx.x == 64) SPMM24_STAMP(5);
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, C_::TMEM_COLS);
    }
    if (threadIdx.x == 0) SPMM24_STAMP(6);
}

// -------------------------------------------------------------------------
// A CTA pair computes a 256 x 256 tile (256 x 128 with HALF_N = 64); each
// CTA holds 128 rows of A and HALF_N columns of B.  With a K split, a
// cluster of two pairs computes the tile:
// pair 1 sends its fp32 partial accumulator to pair 0 through distributed
// shared memory, and pair 0 adds it before the epilogue.
// FP8: a stage covers 256 logical K of fp8 operands in the same A and B bytes
// (B: two 128-byte-swizzled halves of HALF_N rows x 128 K) and two 128-K
// metadata groups.
// HALF_N_: 128 (256 x 256 tiles), or 64 (256 x 128 tiles, for shapes with
// less than half a wave of the wide ones).
template <int STAGES, bool FP8 = false, int HALF_N_ = 128>
struct PairCfg {
    static_assert(HALF_N_ == 64 || HALF_N_ == 128, "pair tiles are 256 or 128 columns wide");
    static constexpr bool kFp8 = FP8;
    static constexpr int HALF_N = HALF_N_;               // columns of B / C per CTA
    static constexpr int TILE_N = 2 * HALF_N;            // columns per pair
    static constexpr int TILE_M = 2 * kTileM;            // rows per pair
    static constexpr int A_BYTES = 8 * 8 * 256;          // this CTA's 128 rows x 128 logical K
    static constexpr int B_BYTES = (HALF_N / 8) * 2048;  // this CTA's HALF_N columns x 128 K
    static constexpr int E_BYTES = (FP8 ? 2 : 1) * 16 * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + E_BYTES;
    static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
    static constexpr int BAR_OFFSET = RING_BYTES;
    static constexpr int NUM_BARS = 2 * STAGES + 3;  // full, empty, acc_full, recv (pair 0), free (pair 1)
    static constexpr int HOLDER_OFFSET = BAR_OFFSET + NUM_BARS * 8;
    static constexpr int SMEM_BYTES = HOLDER_OFFSET + 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
    static constexpr int META_COL = TILE_N;  // accumulator: TILE_N fp32 columns
    static constexpr int META_STRIDE = FP8 ? 8 : 4;
    static constexpr int TMEM_NEED = META_COL + META_STRIDE * STAGES;
    static constexpr int TMEM_COLS = TMEM_NEED <= 128 ? 128 : TMEM_NEED <= 256 ? 256 : 512;
    static constexpr int C_PITCH = TILE_N + 8;  // halves per staged output row (bank-shifted)
    static constexpr int F_PITCH = TILE_N + 4;  // floats per staged fp32 row (epilogue with a residual)
    static constexpr int RES_OFFSET = kTileM * F_PITCH * 4;  // residual tile after the fp32 staging
    // K split: the partner pair's partial accumulator, fp32 rows of F_PITCH,
    // after the 16-bit output staging.
    static constexpr int RECV_OFFSET = ((kTileM * C_PITCH * 2 + 1023) / 1024) * 1024;
    static constexpr uint32_t RECV_BYTES = (uint32_t)kTileM * TILE_N * 4;  // bytes the partner sends
    static_assert(TMEM_NEED <= 512, "TMEM overflow");
    static_assert(SMEM_ALLOC <= 232448, "shared memory overflow");
    static_assert(kTileM * C_PITCH * 2 <= RING_BYTES, "output staging does not fit");
    static_assert(RES_OFFSET + kTileM * TILE_N * 2 <= RING_BYTES, "fp32 staging + residual tile do not fit");
    static_assert(RECV_OFFSET + kTileM * F_PITCH * 4 <= RING_BYTES, "16-bit staging + partner partial do not fit");
    static_assert(!FP8 || (A_BYTES % 1024 == 0 && (B_BYTES / 2) % 1024 == 0 && STAGE_BYTES % 1024 == 0),
                  "fp8 B halves must start on 1024-byte boundaries (128-byte swizzle atoms)");
};

// One stage's loads for one CTA of a pair (both CTAs' loads complete on the
// leader's barrier `bar`).  g: the stage index (128 logical K; fp8: 256).
template <class C_>
__device__ __forceinline__ void pair_load_weights(uint8_t* st, const CUtensorMap* tmA, const CUtensorMap* tmE,
                                                  uint32_t bar, int band0, int g, uint64_t pol) {
    ptx::tma_load_3d_pair(st, tmA, bar, 0, band0, 8 * g, pol);
    if constexpr (C_::kFp8)
        ptx::tma_load_3d_pair(st + C_::A_BYTES + C_::B_BYTES, tmE, bar, 0, band0, 2 * g, pol);
    else
        ptx::tma_load_2d_pair(st + C_::A_BYTES + C_::B_BYTES, tmE, bar, 128 * g, band0, pol);
}
template <class C_>
__device__ __forceinline__ void pair_load_acts(uint8_t* st, const CUtensorMap* tmB, uint32_t bar, int strip0, int g,
                                               uint64_t pol) {
    if constexpr (C_::kFp8) {
        ptx::tma_load_2d_pair(st + C_::A_BYTES, tmB, bar, 256 * g, 8 * strip0, pol);
        ptx::tma_load_2d_pair(st + C_::A_BYTES + C_::B_BYTES / 2, tmB, bar, 256 * g + 128, 8 * strip0, pol);
    } else {
        ptx::tma_load_4d_pair(st + C_::A_BYTES, tmB, bar, 0, 2 * g, 0, strip0, pol);
    }
}

constexpr int kPairGroupM = 8;  // tile rows per rasterisation group

// Instruction descriptor of the pair MMA: sparse, D=f32, A=B=f16, A K-major,
// B MN-major, M=256, N=TILE_N.
template <int TILE_N>
__host__ __device__ constexpr uint32_t pair_idesc() {
    return (1u << 2) | (1u << 4) | (1u << 16) | ((uint32_t)(TILE_N >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}
// The fp8 pair MMA (kind::f8f6f4): sparse, D=f32, A and B K-major, M=256,
// N=TILE_N; operand-format bits from the caller.
template <int TILE_N>
__host__ __device__ constexpr uint32_t pair_idesc_fp8() {
    return (1u << 2) | (1u << 4) | ((uint32_t)(TILE_N >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

// EPI: the general epilogue, as for spmm24_cluster_kernel.  KSPLIT: a
// cluster of two pairs, each taking half of the 128-K stages (p.split == 2;
// not with a residual, whose staging the partner partial would overlap).
// FP8: fp8 operand formats and kind::f8f6f4 MMAs (always with EPI).
template <int STAGES, bool EPI, bool KSPLIT, bool FP8 = false, int HALF_N = 128>
__global__ void __launch_bounds__(kPairThreads, 1)
spmm24_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmE, const PairParams p) {
    static_assert(EPI || !FP8, "the fp8 kernel always runs the general epilogue");
    using C_ = PairCfg<STAGES, FP8, HALF_N>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C_::BAR_OFFSET);  // used in the leader only
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* recv_bar = acc_full + 1;  // pair 0 of a K split: the partner's partial has arrived
    uint64_t* free_bar = acc_full + 2;  // pair 1 of a K split: pair 0 is ready to receive
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C_::HOLDER_OFFSET);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t crank = ptx::cluster_ctarank();
    const uint32_t rank = crank & 1u;         // within the pair: 0 = leader (issues the MMAs), 1 = peer
    const uint32_t lead_rank = crank & ~1u;   // the pair's leader in the cluster
    const int kpart = KSPLIT ? (int)(crank >> 1) : 0;  // which half of K this pair computes
    const uint16_t pair_mask = (uint16_t)(0x3u << (2 * kpart));
    const bool leader = rank == 0;
    // Grouped rasterisation: consecutive pairs walk down a group of
    // kPairGroupM tile rows before moving to the next tile column, so the A
    // and B panels of one wave of pairs stay in L2.
    int m_tile, n_tile;
    {
        const int pid = blockIdx.y + gridDim.y * blockIdx.z;  // pairs in launch order
        const int n_tiles = gridDim.y, m_tiles = gridDim.z;
        const int per_group = kPairGroupM * n_tiles;
        const int first_m = (pid / per_group) * kPairGroupM;
        const int group_m = min(m_tiles - first_m, kPairGroupM);
        const int in_group = pid % per_group;
        m_tile = first_m + in_group % group_m;
        n_tile = in_group / group_m;
    }
    const int band0 = (m_tile * C_::TILE_M + (int)rank * kTileM) / 16;
    const int strip0 = (n_tile * C_::TILE_N + (int)rank * C_::HALF_N) / 8;
    // This pair's 128-K stages: all of them, or its half under a K split.
    const int nsplit = KSPLIT ? 2 : 1;
    const int st_base = p.stages_total / nsplit, st_rem = p.stages_total % nsplit;
    const int st_begin = kpart * st_base + min(kpart, st_rem);
    const int st_count = st_base + (kpart < st_rem ? 1 : 0);

    if (threadIdx.x == 0) {
        SPMM24_STAMP(0);
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        ptx::mbar_init(acc_full, 1);
        ptx::mbar_init(recv_bar, 1);
        ptx::mbar_init(free_bar, 1);
        ptx::fence_mbarrier_init();
        ptx::prefetch_tmap(&tmA);
        ptx::prefetch_tmap(&tmB);
        ptx::prefetch_tmap(&tmE);
    }
    if (warp == 1) {
        ptx::tmem_alloc_pair(tmem_holder, C_::TMEM_COLS);
        ptx::tmem_relinquish_pair();
    }
    ptx::tc_fence_before();
    ptx::cluster_sync();  // every CTA of the cluster: barriers initialised, TMEM allocated
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    if (threadIdx.x == 0) ptx::grid_dep_launch();

    // Both CTAs' loads complete on the pair leader's full barrier; the leader
    // arms it once per stage with both CTAs' bytes.
    const uint64_t pol = ptx::policy_evict_last();  // A is re-read by every N tile, B by every M tile
    const uint32_t full0 = ptx::mapa_shared(ptx::smem_u32(&full[0]), lead_rank);
    const int pre = p.weights_static ? min(STAGES, st_count) : 0;
    // Two producers, one thread each, issue a stage's loads side by side
    // (one issuing thread keeps only about 60-90 GB/s of boxes in flight per
    // SM, below the 180 GB/s a stage needs to keep pace with the MMAs): warp
    // 0 arms the leader's barrier and loads A and the metadata, warp 2 loads
    // B.  Both wait on the same empty barrier and complete on the same full
    // barrier.
    if (warp == 0 || warp == 2) {
        // ------------------------------------------------- TMA producers
        const bool acts = warp == 2;
        if (lane == 0) {
            auto issue = [&](int it, int s) {
                uint8_t* st = smem + s * C_::STAGE_BYTES;
                const uint32_t bar = full0 + 8u * s;
                if (acts)
                    pair_load_acts<C_>(st, &tmB, bar, strip0, st_begin + it, pol);
                else
                    pair_load_weights<C_>(st, &tmA, &tmE, bar, band0, st_begin + it, pol);
            };
            if (!acts)
                for (int it = 0; it < pre; ++it) {
                    if (leader) ptx::mbar_arrive_expect_tx(&full[it], 2 * C_::STAGE_BYTES);
                    issue(it, it);
                }
            ptx::grid_dep_wait();
            if (acts) {
                SPMM24_STAMP(1);
                for (int it = 0; it < pre; ++it) issue(it, it);
            }
            for (int it = pre; it < st_count; ++it) {
                const int s = it % STAGES;
                const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                if (!ptx::mbar_wait_bounded(&empty[s], ph ^ 1u, kWaitLimitNs)) {
                    atomicOr(&g_spmm24_status, kStatusProducerTimeout);
                    break;
                }
                if (!acts && leader) ptx::mbar_arrive_expect_tx(&full[s], 2 * C_::STAGE_BYTES);
                issue(it, s);
            }
        }
        __syncwarp();
    } else if (warp == 1 && leader) {
        // ---------------------------------- MMA issuer (leader CTA only)
        const uint32_t idesc = FP8 ? pair_idesc_fp8<C_::TILE_N>() | p.mma_fmt
                                   : pair_idesc<C_::TILE_N>() | ((EPI && p.epi.bf16) ? kIdescBf16 : 0u);
        const uint32_t smem_base = ptx::smem_u32(smem);
        uint32_t accumulate = 0;
        for (int it = 0; it < st_count; ++it) {
            const int s = it % STAGES;
            const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
            if (!ptx::mbar_wait_bounded(&full[s], ph, kWaitLimitNs)) {
                if (lane == 0) atomicOr(&g_spmm24_status, kStatusMmaTimeout);
                break;
            }
            if (lane == 0 && it == 0) SPMM24_STAMP(2);
            if (lane == 0 && it == st_count - 1) SPMM24_STAMP(3);
            ptx::tc_fence_after();
            if (lane == 0) {
                const uint32_t st = smem_base + s * C_::STAGE_BYTES;
                const uint32_t stB = st + C_::A_BYTES;
                const uint32_t meta_col = tmem_base + C_::META_COL + C_::META_STRIDE * s;
                if constexpr (FP8) {
                    // as mma_stage_fp8, on both CTAs of the pair
                    ptx::tmem_cp_128x128b_pair(meta_col, smem_desc(stB + C_::B_BYTES, 0, 128));
                    ptx::tmem_cp_128x128b_pair(meta_col + 4, smem_desc(stB + C_::B_BYTES + 2048, 0, 128));
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint64_t adesc = smem_desc(st + j * 4096, 2048, 128);
                        const uint64_t bdesc = smem_desc_sw128(stB + (j >> 1) * (C_::B_BYTES / 2) + (j & 1) * 64);
                        ptx::mma_sp_f8_pair(tmem_base, adesc, bdesc, meta_col + 2 * j, idesc, accumulate);
                        accumulate = 1;
                    }
                } else {
                    ptx::tmem_cp_128x128b_pair(meta_col, smem_desc(stB + C_::B_BYTES, 0, 128));
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint64_t adesc = smem_desc(st + j * 2048, 4 * 2048, 128);
                        const uint64_t bdesc = smem_desc(stB + j * 512, 128, 2048);
                        ptx::mma_sp_f16_pair(tmem_base, adesc, bdesc, meta_col + (j & 2), idesc | (uint32_t)(j & 1),
                                             accumulate);
                        accumulate = 1;
                    }
                }
                ptx::tc_commit_pair_mc(&empty[s], pair_mask);  // frees ring slot s in both CTAs of the pair
            }
            __syncwarp();
        }
        if (lane == 0) ptx::tc_commit_pair_mc(acc_full, pair_mask);
        __syncwarp();
    }
    {
        // ---------------------------------- epilogue (every warp, both CTAs)
        if (!ptx::mbar_wait_bounded(acc_full, 0, kWaitLimitNs)) atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
        if (threadIdx.x == 64) SPMM24_STAMP(4);
        ptx::tc_fence_after();
        __syncwarp();
        const int quad = warp & 3;  // TMEM lane quadrant this warp may access
        const int row = quad * 32 + lane;
        constexpr int NCH16 = C_::TILE_N / 16;           // 16-column chunks per row
        const int c_begin = (warp >> 2) * (NCH16 / 2);  // this warp's half of the columns
        const int c_end = c_begin + NCH16 / 2;
        const int etid = threadIdx.x;
        // K split: pair 1 sends its fp32 partial to the matching CTA of pair 0
        // (st.async into its idle ring, counted on its receive barrier) once
        // pair 0 is ready; pair 0 adds it to its own accumulator row by row.
        const float* part = reinterpret_cast<const float*>(smem + C_::RECV_OFFSET);
        bool produce = true;
        if constexpr (KSPLIT) {
            if (kpart == 0) {
                if (threadIdx.x == 0) {
                    ptx::mbar_arrive_expect_tx(recv_bar, C_::RECV_BYTES);
                    ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_u32(free_bar), crank + 2u));
                }
                if (!ptx::mbar_wait_bounded(recv_bar, 0, kWaitLimitNs))
                    atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
            } else {
                produce = false;
                if (!ptx::mbar_wait_bounded(free_bar, 0, kWaitLimitNs)) {
                    atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
                } else {
                    const uint32_t dst0 = ptx::mapa_shared(ptx::smem_u32(smem + C_::RECV_OFFSET), crank - 2u);
                    const uint32_t dbar = ptx::mapa_shared(ptx::smem_u32(recv_bar), crank - 2u);
#pragma unroll 1
                    for (int c = c_begin; c < c_end; ++c) {
                        uint32_t v[16];
                        ptx::tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(c * 16), v);
                        ptx::tmem_wait_ld();
                        const uint32_t dst = dst0 + (uint32_t)((row * C_::F_PITCH + c * 16) * 4);
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            ptx::st_async_v4(dst + 16u * q, __uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                             __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]), dbar);
                    }
                }
            }
        }
        // the partner partial of (this thread's row, 16-column chunk c), added to v
        auto add_partial = [&](uint32_t* v, int c) {
            if constexpr (KSPLIT) {
                const float4* pp = reinterpret_cast<const float4*>(part + (size_t)row * C_::F_PITCH + c * 16);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 x = pp[q];
                    v[4 * q] = __float_as_uint(__uint_as_float(v[4 * q]) + x.x);
                    v[4 * q + 1] = __float_as_uint(__uint_as_float(v[4 * q + 1]) + x.y);
                    v[4 * q + 2] = __float_as_uint(__uint_as_float(v[4 * q + 2]) + x.z);
                    v[4 * q + 3] = __float_as_uint(__uint_as_float(v[4 * q + 3]) + x.w);
                }
            }
        };
        if (!produce) {
            // pair 1 of a K split: its partial has been sent
        } else if constexpr (!EPI) {
            // Plain fp16 row-major: stage the rounded tile in the (now idle)
            // ring -- rows bank-shifted by 16 bytes so the per-row writes do
            // not collide -- then copy it out with coalesced 16-byte stores.
            __half* cst = reinterpret_cast<__half*>(smem);
#pragma unroll 1
            for (int c = c_begin; c < c_end; ++c) {
                uint32_t v[16];
                ptx::tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(c * 16), v);
                ptx::tmem_wait_ld();
                add_partial(v, c);
                __align__(16) __half h[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) h[e] = __float2half_rn(__uint_as_float(v[e]));
                uint4* dst = reinterpret_cast<uint4*>(cst + (size_t)row * C_::C_PITCH + c * 16);
                dst[0] = reinterpret_cast<const uint4*>(h)[0];
                dst[1] = reinterpret_cast<const uint4*>(h)[1];
            }
            ptx::tc_fence_before();
            ptx::named_barrier(kBarEpi, kPairThreads);
            ptx::grid_dep_wait();  // C may be in use by the previous grid
            constexpr int LPR = C_::TILE_N / 8;      // threads per row (16-byte chunks)
            constexpr int RPP = kPairThreads / LPR;  // rows per pass
            const int chunk = etid % LPR;
            const int gm0 = m_tile * C_::TILE_M + (int)rank * kTileM;
            const int gn = n_tile * C_::TILE_N + chunk * 8;
            const bool vec_ok = (p.N % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0);
            for (int r = etid / LPR; r < kTileM; r += RPP) {
                const int gm = gm0 + r;
                if (gm >= p.M || gn >= p.N) continue;
                const __half* src = cst + (size_t)r * C_::C_PITCH + chunk * 8;
                if constexpr (EPI) {
                    if (p.epi.gather_n) {  // every rank's full C (or its multicast address)
                        if (vec_ok) {
                            store_row16(p.C, p.epi, gm, gn, p.N, *reinterpret_cast<const uint4*>(src));
                        } else {
                            const int lim = min(8, p.N - gn);
                            uint32_t w[4];
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                w[q] = (uint32_t)__half_as_ushort(src[2 * q]) |
                                       ((uint32_t)__half_as_ushort(src[2 * q + 1]) << 16);
                            store_row_elems(p.C, p.epi, gm, gn, p.N, w, lim);
                        }
                        continue;
                    }
                }
                __half* out = reinterpret_cast<__half*>(p.C) + (size_t)gm * p.N + gn;
                if (vec_ok) {
                    *reinterpret_cast<uint4*>(out) = *reinterpret_cast<const uint4*>(src);
                } else {
                    const int lim = min(8, p.N - gn);
                    for (int e = 0; e < lim; ++e) out[e] = src[e];
                }
            }
        } else {
            // General epilogue.  alpha * acc + bias, activated, is computed
            // from TMEM per row.  Without a residual it is rounded and staged
            // as 16-bit values; with one it is staged as fp32 while the
            // residual tile streams into the rest of the idle ring (cp.async,
            // coalesced, all of it in flight at once), and the copy-out adds
            // the residual before rounding once.  Each case has its own short
            // loop: the epilogue is bound by instruction latency.  Stores are
            // coalesced, row-major or packed.
            const int gm0 = m_tile * C_::TILE_M + (int)rank * kTileM;
            const int gn0 = n_tile * C_::TILE_N;
            const bool vec_ok = (p.N % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0);
            const bool has_res = p.epi.residual != nullptr;
            const bool vec_res = p.epi.packed ||
                                 ((p.N % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.epi.residual) & 15u) == 0));
            const int strips = (p.N + 7) / 8;
            constexpr int CH = C_::TILE_N / 8;  // 8-column chunks per row
            constexpr int ITEMS = kTileM * CH;   // (row, chunk) items of this CTA
            if (p.epi.bias || has_res) ptx::grid_dep_wait();  // they may be written by the previous grid
            uint4* rst = reinterpret_cast<uint4*>(smem + C_::RES_OFFSET);  // residual tile [row][chunk]
            if (has_res && vec_res) {
                // packed C: consecutive threads take consecutive rows of a
                // strip; row-major C: consecutive chunks of a row
                for (int idx = etid; idx < ITEMS; idx += kPairThreads) {
                    const int r = p.epi.packed ? idx % kTileM : idx / CH;
                    const int c = p.epi.packed ? idx / kTileM : idx % CH;
                    const int gm = gm0 + r, gn = gn0 + c * 8;
                    if (gm < p.M && gn < p.N)
                        ptx::cp_async16(rst + r * CH + c, p.epi.residual + c_offset(p.epi, gm, gn, p.M, p.N));
                }
                ptx::cp_async_commit();
            }
            float* fst = reinterpret_cast<float*>(smem);
            uint16_t* hst = reinterpret_cast<uint16_t*>(smem);
            const int gm = gm0 + row;
            if (has_res) {
#pragma unroll 1
                for (int c = c_begin; c < c_end; ++c) {
                    uint32_t v[16];
                    ptx::tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(c * 16), v);
                    ptx::tmem_wait_ld();
                    add_partial(v, c);
                    float f[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) f[e] = __uint_as_float(v[e]);
                    if (gm < p.M) epilogue_pre<16>(f, p.epi, gm);
                    float4* dst = reinterpret_cast<float4*>(fst + (size_t)row * C_::F_PITCH + c * 16);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        dst[q] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
                }
            } else {
#pragma unroll 1
                for (int c = c_begin; c < c_end; ++c) {
                    uint32_t v[16];
                    ptx::tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(c * 16), v);
                    ptx::tmem_wait_ld();
                    add_partial(v, c);
                    float f[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) f[e] = __uint_as_float(v[e]);
                    if (gm < p.M) epilogue_pre<16>(f, p.epi, gm);
                    const int gn = gn0 + c * 16;
                    uint32_t h[8];
                    if (gn + 16 <= p.N) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) h[e] = pack2(f[2 * e], f[2 * e + 1], p.epi.bf16);
                    } else {  // the last strip: columns at or past N become zero
                        round8(f, max(0, min(8, p.N - gn)), p.epi.bf16, h);
                        round8(f + 8, max(0, min(8, p.N - gn - 8)), p.epi.bf16, h + 4);
                    }
                    uint4* dst = reinterpret_cast<uint4*>(hst + (size_t)row * C_::C_PITCH + c * 16);
                    dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
                    dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
                }
            }
            if (has_res && vec_res) ptx::cp_async_wait_all();
            ptx::tc_fence_before();
            ptx::named_barrier(kBarEpi, kPairThreads);
            ptx::grid_dep_wait();  // C may be in use by the previous grid
            // The output chunk (row r, 8-column chunk c) as four words.
            auto chunk_out = [&](int r, int c, int gmr, int gn, uint4& out) {
                if (has_res) {
                    const float* src = fst + (size_t)r * C_::F_PITCH + c * 8;
                    const float4 y0 = *reinterpret_cast<const float4*>(src);
                    const float4 y1 = *reinterpret_cast<const float4*>(src + 4);
                    float y[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
                    if (vec_res) {
                        const uint4 q = rst[r * CH + c];
                        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            y[e] += elem_to_f32((uint16_t)(w[e >> 1] >> (16 * (e & 1))), p.epi.bf16);
                    } else {
                        const size_t off = c_offset(p.epi, gmr, gn, p.M, p.N);
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            if (gn + e < p.N) y[e] += elem_to_f32(p.epi.residual[off + e], p.epi.bf16);
                    }
                    uint32_t h[4];
                    round8(y, min(8, p.N - gn), p.epi.bf16, h);
                    out = make_uint4(h[0], h[1], h[2], h[3]);
                } else {
                    out = *reinterpret_cast<const uint4*>(hst + (size_t)r * C_::C_PITCH + c * 8);
                }
            };
            if (p.epi.gather_n && !p.epi.gather_mc && !has_res && vec_ok) {
                // Gathered output: every staged row goes to every rank's full C
                // as one bulk copy, spread over the threads; a CTA waits only
                // until its shared memory has been read, so the NVLink writes
                // drain while the next tile computes.
                ptx::fence_proxy_async_smem();  // the staged rows, written by other threads, to the async proxy
                const int ncols = min(C_::TILE_N, p.N - gn0);
                for (int idx = etid; idx < kTileM * p.epi.gather_n; idx += kPairThreads) {
                    const int r = idx % kTileM, d = idx / kTileM;
                    const int gmr = gm0 + r;
                    if (gmr >= p.M) continue;
                    ptx::bulk_store(p.epi.gather_dst[d] + (size_t)(p.epi.gather_row0 + gmr) * p.N + gn0,
                                    hst + (size_t)r * C_::C_PITCH, (uint32_t)ncols * 2u);
                }
                ptx::bulk_commit();
                ptx::bulk_wait_read_all();
            } else if (p.epi.packed) {
                // consecutive threads take consecutive rows of a strip
                for (int idx = etid; idx < ITEMS; idx += kPairThreads) {
                    const int r = idx % kTileM, c = idx / kTileM;
                    const int gmr = gm0 + r, gn = gn0 + c * 8;
                    if (gmr >= p.M || (gn >> 3) >= strips) continue;
                    uint4 out;
                    chunk_out(r, c, gmr, gn, out);
                    *reinterpret_cast<uint4*>(p.C + (((size_t)(gn >> 3) * p.M + gmr) << 3)) = out;
                }
            } else {
                // consecutive threads take consecutive chunks of a row
                constexpr int RPP = kPairThreads / CH;  // rows per pass
                const int c = etid % CH;
                const int gn = gn0 + c * 8;
                for (int r = etid / CH; r < kTileM; r += RPP) {
                    const int gmr = gm0 + r;
                    if (gmr >= p.M || gn >= p.N) continue;
                    uint4 out;
                    chunk_out(r, c, gmr, gn, out);
                    if (vec_ok) {
                        store_row16(p.C, p.epi, gmr, gn, p.N, out);
                    } else {
                        const uint32_t w[4] = {out.x, out.y, out.z, out.w};
                        store_row_elems(p.C, p.epi, gmr, gn, p.N, w, min(8, p.N - gn));
                    }
                }
            }
        }
    }

    if (threadIdx.x == 64) SPMM24_STAMP(5);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::cluster_sync();  // neither CTA may leave while the pair still shares shared memory / TMEM
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc_pair(tmem_base, C_::TMEM_COLS);
    }
    if (threadIdx.x == 0) SPMM24_STAMP(6);
}

// -------------------------------------------------------------------------
// Two M halves per pair: a 512 x 240 tile.  Each CTA holds two 128-row
// halves of A (rows m0 + 256h + 128 rank, h = 0, 1) and 120 columns of B;
// per K step the leader issues two M=256 MMAs that share the B tile, into
// two TMEM accumulators (columns 0 and 256).  Every stage moves 66 KB per
// CTA for 15.7 MFLOP (dense-equivalent) instead of 50 KB for 8.4 MFLOP,
// so the same shared-memory bytes in flight feed the tensor core 1.4x
// longer.  Row-major output; EPI adds alpha, bias, activation, bf16 and
// the packed-B output layout, the fused all-gather's row stores (no
// residual); no K split.  FP8: two
// 128-byte-swizzled B halves of 120 rows per stage and two 128-K metadata
// groups per M half; the metadata ring in TMEM has two slots instead of
// one per stage (the copy into a slot is issued after the MMAs that read
// it two stages earlier, and tcgen05 operations of one thread execute in
// issue order), which leaves room for the two 240-column accumulators;
// always EPI.
template <int STAGES, bool FP8 = false>
struct Pair2Cfg {
    static constexpr bool kFp8 = FP8;
    static constexpr int HALF_N = 120;                   // columns of B / C per CTA
    static constexpr int TILE_N = 2 * HALF_N;            // columns per pair
    static constexpr int TILE_M = 4 * kTileM;            // rows per pair
    static constexpr int A_HALF = 8 * 8 * 256;           // 128 rows x 128 logical K (fp8: 256)
    static constexpr int A_BYTES = 2 * A_HALF;
    static constexpr int B_BYTES = (HALF_N / 8) * 2048;  // HALF_N columns x 128 K (fp8: 256 K)
    static constexpr int E_HALF = (FP8 ? 2 : 1) * 16 * 128;
    static constexpr int E_BYTES = 2 * E_HALF;
    static constexpr int META_STRIDE = FP8 ? 8 : 4;      // TMEM columns per metadata slot
    static constexpr int META_SLOTS = FP8 ? 2 : STAGES;  // metadata ring slots per M half
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + E_BYTES;
    static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
    static constexpr int BAR_OFFSET = RING_BYTES;
    static constexpr int NUM_BARS = 2 * STAGES + 1;  // full, empty, acc_full
    static constexpr int HOLDER_OFFSET = BAR_OFFSET + NUM_BARS * 8;
    static constexpr int SMEM_BYTES = HOLDER_OFFSET + 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
    static constexpr int ACC1_COL = 256;                  // second accumulator
    static constexpr int META0_COL = TILE_N;              // metadata rings after each accumulator
    static constexpr int META1_COL = ACC1_COL + TILE_N;
    static constexpr int TMEM_COLS = 512;
    static constexpr int C_PITCH = TILE_N + 8;  // halves per staged output row (bank-shifted)
    static_assert(META0_COL + META_STRIDE * META_SLOTS <= ACC1_COL && META1_COL + META_STRIDE * META_SLOTS <= TMEM_COLS,
                  "TMEM overflow");
    static_assert(2 * kTileM * C_PITCH * 2 <= RING_BYTES, "output staging does not fit");
    static_assert(SMEM_ALLOC <= 232448, "shared memory overflow");
    static_assert(!FP8 || ((B_BYTES / 2) % 1024 == 0 && STAGE_BYTES % 1024 == 0),
                  "fp8 B halves must start on 1024-byte boundaries (128-byte swizzle atoms)");
};

template <int STAGES, bool EPI, bool FP8 = false>
__global__ void __launch_bounds__(kPairThreads, 1)
spmm24_pair2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmE, const PairParams p) {
    static_assert(EPI || !FP8, "the fp8 form always runs the epilogue (alpha)");
    using C_ = Pair2Cfg<STAGES, FP8>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C_::BAR_OFFSET);  // used in the leader only
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C_::HOLDER_OFFSET);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = ptx::cluster_ctarank();  // 0 = leader (issues the MMAs), 1 = peer
    const bool leader = rank == 0;
    int m_tile, n_tile;
    {
        const int pid = blockIdx.y + gridDim.y * blockIdx.z;
        const int n_tiles = gridDim.y, m_tiles = gridDim.z;
        const int per_group = kPairGroupM * n_tiles;
        const int first_m = (pid / per_group) * kPairGroupM;
        const int group_m = min(m_tiles - first_m, kPairGroupM);
        const int in_group = pid % per_group;
        m_tile = first_m + in_group % group_m;
        n_tile = in_group / group_m;
    }
    // this CTA's 128-row halves: rows m0 + 256 h + 128 rank
    const int band_h0 = (m_tile * C_::TILE_M + (int)rank * kTileM) / 16;
    const int band_h1 = band_h0 + 2 * kTileM / 16;
    const int strip0 = (n_tile * C_::TILE_N + (int)rank * C_::HALF_N) / 8;
    const int st_count = p.stages_total;

    if (threadIdx.x == 0) {
        SPMM24_STAMP(0);
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        ptx::mbar_init(acc_full, 1);
        ptx::fence_mbarrier_init();
        ptx::prefetch_tmap(&tmA);
        ptx::prefetch_tmap(&tmB);
        ptx::prefetch_tmap(&tmE);
    }
    if (warp == 1) {
        ptx::tmem_alloc_pair(tmem_holder, C_::TMEM_COLS);
        ptx::tmem_relinquish_pair();
    }
    ptx::tc_fence_before();
    ptx::cluster_sync();  // both CTAs: barriers initialised, TMEM allocated
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    if (threadIdx.x == 0) ptx::grid_dep_launch();

    const uint64_t pol = ptx::policy_evict_last();
    const uint32_t full0 = ptx::mapa_shared(ptx::smem_u32(&full[0]), 0u);
    const int pre = p.weights_static ? min(STAGES, st_count) : 0;
    // One M half's A and metadata (h = 0, 1).
    auto load_weights = [&](uint8_t* st, uint32_t bar, int g, int h) {
        const int band = h ? band_h1 : band_h0;
        ptx::tma_load_3d_pair(st + h * C_::A_HALF, &tmA, bar, 0, band, 8 * g, pol);
        uint8_t* se = st + C_::A_BYTES + C_::B_BYTES + h * C_::E_HALF;
        if constexpr (FP8)  // box (256 B, 8 bands, 2 groups)
            ptx::tma_load_3d_pair(se, &tmE, bar, 0, band, 2 * g, pol);
        else
            ptx::tma_load_2d_pair(se, &tmE, bar, 128 * g, band, pol);
    };
    auto load_acts = [&](uint8_t* st, uint32_t bar, int g) {
        if constexpr (FP8) {
            ptx::tma_load_2d_pair(st + C_::A_BYTES, &tmB, bar, 256 * g, 8 * strip0, pol);
            ptx::tma_load_2d_pair(st + C_::A_BYTES + C_::B_BYTES / 2, &tmB, bar, 256 * g + 128, 8 * strip0, pol);
        } else {
            ptx::tma_load_4d_pair(st + C_::A_BYTES, &tmB, bar, 0, 2 * g, 0, strip0, pol);
        }
    };
    // Three producers, one thread each, issue a stage's loads side by side
    // (one issuing thread keeps only about 60-90 GB/s of boxes in flight per
    // SM, below the 127 GB/s a stage needs to keep pace with the MMAs):
    // warp 0 arms the leader's barrier and loads M half 0's A and metadata,
    // warp 2 M half 1's, warp 3 B.  All three wait on the same empty barrier
    // and complete on the same full barrier.
    const int role = warp == 0 ? 0 : warp == 2 ? 1 : warp == 3 ? 2 : -1;
    if (role >= 0) {
        // ------------------------------------------------- TMA producers
        if (lane == 0) {
            auto issue = [&](int it, int s) {
                uint8_t* st = smem + s * C_::STAGE_BYTES;
                const uint32_t bar = full0 + 8u * s;
                if (role == 2)
                    load_acts(st, bar, it);
                else
                    load_weights(st, bar, it, role);
            };
            if (role < 2)
                for (int it = 0; it < pre; ++it) {
                    if (role == 0 && leader) ptx::mbar_arrive_expect_tx(&full[it], 2 * C_::STAGE_BYTES);
                    issue(it, it);
                }
            ptx::grid_dep_wait();
            if (role == 2) {
                SPMM24_STAMP(1);
                for (int it = 0; it < pre; ++it) issue(it, it);
            }
            for (int it = pre; it < st_count; ++it) {
                const int s = it % STAGES;
                const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                if (!ptx::mbar_wait_bounded(&empty[s], ph ^ 1u, kWaitLimitNs)) {
                    atomicOr(&g_spmm24_status, kStatusProducerTimeout);
                    break;
                }
                if (role == 0 && leader) ptx::mbar_arrive_expect_tx(&full[s], 2 * C_::STAGE_BYTES);
                issue(it, s);
            }
        }
        __syncwarp();
    } else if (warp == 1 && leader) {
        // ---------------------------------- MMA issuer (leader CTA only)
        const uint32_t idesc = FP8 ? pair_idesc_fp8<C_::TILE_N>() | p.mma_fmt
                                   : pair_idesc<C_::TILE_N>() | ((EPI && p.epi.bf16) ? kIdescBf16 : 0u);
        const uint32_t smem_base = ptx::smem_u32(smem);
        uint32_t accumulate = 0;
        for (int it = 0; it < st_count; ++it) {
            const int s = it % STAGES;
            const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
            if (!ptx::mbar_wait_bounded(&full[s], ph, kWaitLimitNs)) {
                if (lane == 0) atomicOr(&g_spmm24_status, kStatusMmaTimeout);
                break;
            }
            if (lane == 0 && it == 0) SPMM24_STAMP(2);
            if (lane == 0 && it == st_count - 1) SPMM24_STAMP(3);
            ptx::tc_fence_after();
            if (lane == 0) {
                const uint32_t st = smem_base + s * C_::STAGE_BYTES;
                const uint32_t stB = st + C_::A_BYTES;
                const uint32_t stE = stB + C_::B_BYTES;
                const uint32_t slot = (uint32_t)(it % C_::META_SLOTS);
                const uint32_t meta0 = tmem_base + C_::META0_COL + C_::META_STRIDE * slot;
                const uint32_t meta1 = tmem_base + C_::META1_COL + C_::META_STRIDE * slot;
                if constexpr (FP8) {
                    ptx::tmem_cp_128x128b_pair(meta0, smem_desc(stE, 0, 128));
                    ptx::tmem_cp_128x128b_pair(meta0 + 4, smem_desc(stE + 2048, 0, 128));
                    ptx::tmem_cp_128x128b_pair(meta1, smem_desc(stE + C_::E_HALF, 0, 128));
                    ptx::tmem_cp_128x128b_pair(meta1 + 4, smem_desc(stE + C_::E_HALF + 2048, 0, 128));
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint64_t bdesc = smem_desc_sw128(stB + (j >> 1) * (C_::B_BYTES / 2) + (j & 1) * 64);
                        ptx::mma_sp_f8_pair(tmem_base, smem_desc(st + j * 4096, 2048, 128), bdesc, meta0 + 2 * j, idesc,
                                            accumulate);
                        ptx::mma_sp_f8_pair(tmem_base + C_::ACC1_COL, smem_desc(st + C_::A_HALF + j * 4096, 2048, 128),
                                            bdesc, meta1 + 2 * j, idesc, accumulate);
                        accumulate = 1;
                    }
                } else {
                    ptx::tmem_cp_128x128b_pair(meta0, smem_desc(stE, 0, 128));
                    ptx::tmem_cp_128x128b_pair(meta1, smem_desc(stE + C_::E_HALF, 0, 128));
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint64_t bdesc = smem_desc(stB + j * 512, 128, 2048);
                        const uint32_t id = idesc | (uint32_t)(j & 1);
                        ptx::mma_sp_f16_pair(tmem_base, smem_desc(st + j * 2048, 4 * 2048, 128), bdesc,
                                             meta0 + (j & 2), id, accumulate);
                        ptx::mma_sp_f16_pair(tmem_base + C_::ACC1_COL,
                                             smem_desc(st + C_::A_HALF + j * 2048, 4 * 2048, 128), bdesc,
                                             meta1 + (j & 2), id, accumulate);
                        accumulate = 1;
                    }
                }
                ptx::tc_commit_pair_mc(&empty[s], (uint16_t)0x3);  // frees ring slot s in both CTAs
            }
            __syncwarp();
        }
        if (lane == 0) ptx::tc_commit_pair_mc(acc_full, (uint16_t)0x3);
        __syncwarp();
    }
    {
        // ------------------------------- epilogue (every warp, both CTAs)
        // TMEM -> (EPI: alpha, bias, activation) -> 16-bit -> staged rows
        // (two halves of 128 rows, bank-shifted) -> coalesced 16-byte stores.
        if (!ptx::mbar_wait_bounded(acc_full, 0, kWaitLimitNs)) atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
        if (threadIdx.x == 64) SPMM24_STAMP(4);
        ptx::tc_fence_after();
        __syncwarp();
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        constexpr int NCH16 = C_::TILE_N / 16;          // chunks of 16 columns per row (15; fp8 14)
        const int c_begin = (warp >> 2) ? (NCH16 + 1) / 2 : 0;  // warps 0-3 take the first half
        const int c_end = (warp >> 2) ? NCH16 : (NCH16 + 1) / 2;
        __half* cst = reinterpret_cast<__half*>(smem);
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
#pragma unroll 1
            for (int c = c_begin; c < c_end; ++c) {
                uint32_t v[16];
                ptx::tmem_ld_32x32b_x16(tmem_base + (uint32_t)(h * C_::ACC1_COL) + ((uint32_t)(quad * 32) << 16) +
                                            (uint32_t)(c * 16),
                                        v);
                ptx::tmem_wait_ld();
                uint4* dst = reinterpret_cast<uint4*>(cst + (size_t)(h * kTileM + row) * C_::C_PITCH + c * 16);
                if constexpr (EPI) {
                    float y[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) y[e] = __uint_as_float(v[e]);
                    const int gm = m_tile * C_::TILE_M + h * 2 * kTileM + (int)rank * kTileM + row;
                    if (gm < p.M) epilogue_pre<16>(y, p.epi, gm);
                    uint32_t w[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) w[e] = pack2(y[2 * e], y[2 * e + 1], p.epi.bf16);
                    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                } else {
                    __align__(16) __half hv[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) hv[e] = __float2half_rn(__uint_as_float(v[e]));
                    dst[0] = reinterpret_cast<const uint4*>(hv)[0];
                    dst[1] = reinterpret_cast<const uint4*>(hv)[1];
                }
            }
        }
        ptx::tc_fence_before();
        ptx::named_barrier(kBarEpi, kPairThreads);
        ptx::grid_dep_wait();  // C may be in use by the previous grid
        constexpr int LPR = C_::TILE_N / 8;      // threads per row (30; fp8 28)
        constexpr int RPP = kPairThreads / LPR;  // rows per pass (8; fp8 9)
        const int etid = threadIdx.x;
        bool packed_out = false;
        if constexpr (EPI) packed_out = p.epi.packed != 0;
        if (packed_out) {
            // C in the packed-B layout (8-column strips of M rows x 16
            // bytes, C 16-byte aligned): consecutive threads take consecutive
            // rows of one strip within an M half, so each warp writes 512
            // contiguous bytes.  Columns at or past N are written as zero.
            constexpr int CH = C_::TILE_N / 8;
            for (int i = etid; i < 2 * kTileM * CH; i += kPairThreads) {
                const int r = i % kTileM, rest = i / kTileM;
                const int sc = rest % CH, h = rest / CH;
                const int gm = m_tile * C_::TILE_M + h * 2 * kTileM + (int)rank * kTileM + r;
                const int gn = n_tile * C_::TILE_N + sc * 8;
                if (gm >= p.M || gn >= p.N) continue;
                uint4 v = *reinterpret_cast<const uint4*>(cst + (size_t)(h * kTileM + r) * C_::C_PITCH + sc * 8);
                const int lim = p.N - gn;
                if (lim < 8) {
                    uint32_t x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if (2 * q >= lim) x[q] = 0u;
                        else if (2 * q + 1 >= lim) x[q] &= 0xffffu;
                    }
                    v = make_uint4(x[0], x[1], x[2], x[3]);
                }
                *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(p.C) + (((size_t)(gn >> 3) * p.M + gm) << 3)) = v;
            }
        } else if (etid < LPR * RPP) {
            const int chunk = etid % LPR;
            const int gn = n_tile * C_::TILE_N + chunk * 8;
            const bool vec_ok = (p.N % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0);
            for (int r = etid / LPR; r < 2 * kTileM; r += RPP) {
                const int gm = m_tile * C_::TILE_M + (r / kTileM) * 2 * kTileM + (int)rank * kTileM + r % kTileM;
                if (gm >= p.M || gn >= p.N) continue;
                const __half* src = cst + (size_t)r * C_::C_PITCH + chunk * 8;
                if constexpr (EPI) {
                    if (p.epi.gather_n) {  // every rank's full C (or its multicast address)
                        if (vec_ok) {
                            store_row16(p.C, p.epi, gm, gn, p.N, *reinterpret_cast<const uint4*>(src));
                        } else {
                            const int lim = min(8, p.N - gn);
                            uint32_t w[4];
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                w[q] = (uint32_t)__half_as_ushort(src[2 * q]) |
                                       ((uint32_t)__half_as_ushort(src[2 * q + 1]) << 16);
                            store_row_elems(p.C, p.epi, gm, gn, p.N, w, lim);
                        }
                        continue;
                    }
                }
                __half* out = reinterpret_cast<__half*>(p.C) + (size_t)gm * p.N + gn;
                if (vec_ok) {
                    *reinterpret_cast<uint4*>(out) = *reinterpret_cast<const uint4*>(src);
                } else {
                    const int lim = min(8, p.N - gn);
                    for (int e = 0; e < lim; ++e) out[e] = src[e];
                }
            }
        }
    }

    if (threadIdx.x == 64) SPMM24_STAMP(5);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::cluster_sync();  // neither CTA may leave while the pair still shares shared memory / TMEM
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc_pair(tmem_base, C_::TMEM_COLS);
    }
    if (threadIdx.x == 0) SPMM24_STAMP(6);
}

// -------------------------------------------------------------------------
template <int N_TILE, int STAGES>
struct StreamKCfg : Cfg<N_TILE, STAGES, 2> {
    using B_ = Cfg<N_TILE, STAGES, 2>;
    static constexpr int BAR_OFFSET = B_::RING_BYTES;
    static constexpr int NUM_BARS = 2 * STAGES + 4;  // full, empty, acc_full[2], acc_empty[2]
    static constexpr int HOLDER_OFFSET = BAR_OFFSET + NUM_BARS * 8;
    static constexpr int SMEM_BYTES = HOLDER_OFFSET + 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
    static_assert(N_TILE <= 64, "stream-K keeps one accumulator row in registers");
    static_assert(SMEM_ALLOC <= 232448, "shared memory overflow");
};

__host__ __device__ __forceinline__ long long sk_unit_begin(long long c, long long units, long long grid) {
    return c * units / grid;
}
// CTA whose unit range contains unit u.
__host__ __device__ __forceinline__ int sk_cta_of(long long u, long long units, long long grid) {
    return (int)(((u + 1) * grid - 1) / units);
}

template <int N_TILE, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
spmm24_streamk_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmE, const StreamKParams p) {
    using C_ = StreamKCfg<N_TILE, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C_::BAR_OFFSET);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;  // [2]
    uint64_t* acc_empty = acc_full + 2;   // [2]
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C_::HOLDER_OFFSET);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    const long long U = p.units;
    const int SPT = p.stages_per_tile;
    const long long u_begin = sk_unit_begin(cta, U, p.grid);
    const long long u_end = sk_unit_begin(cta + 1, U, p.grid);

    if (threadIdx.x == 0) {
        SPMM24_STAMP(0);
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            ptx::mbar_init(&acc_full[b], 1);
            ptx::mbar_init(&acc_empty[b], kEpiThreads / 32);
        }
        ptx::fence_mbarrier_init();
        ptx::prefetch_tmap(&tmA);
        ptx::prefetch_tmap(&tmB);
        ptx::prefetch_tmap(&tmE);
    }
    __syncthreads();
    if (threadIdx.x == 0) ptx::grid_dep_launch();

    uint32_t tmem_base = 0;
    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            const uint64_t pol_stream = ptx::policy_evict_first();
            const uint64_t pol_keep = ptx::policy_evict_last();
            const int count = (int)(u_end - u_begin);
            const int pre = p.weights_static ? min(STAGES, count) : 0;
            for (int it = 0; it < pre; ++it) {
                const long long u = u_begin + it;
                const int tile = (int)(u / SPT), g0 = 2 * (int)(u % SPT);
                ptx::mbar_arrive_expect_tx(&full[it], C_::STAGE_BYTES);
                load_stage_weights<C_>(smem + it * C_::STAGE_BYTES, &full[it], &tmA, &tmE, (tile / p.n_tiles) * 8, g0,
                                       pol_stream);
            }
            ptx::grid_dep_wait();
            SPMM24_STAMP(1);
            for (int it = 0; it < pre; ++it) {
                const long long u = u_begin + it;
                const int tile = (int)(u / SPT), g0 = 2 * (int)(u % SPT);
                load_stage_acts<C_>(smem + it * C_::STAGE_BYTES, &full[it], &tmB, (tile % p.n_tiles) * (N_TILE / 8), g0,
                                    pol_keep);
            }
            for (int it = pre; it < count; ++it) {
                const int s = it % STAGES;
                const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                if (!ptx::mbar_wait_bounded(&empty[s], ph ^ 1u, kWaitLimitNs)) {
                    atomicOr(&g_spmm24_status, kStatusProducerTimeout);
                    break;
                }
                const long long u = u_begin + it;
                const int tile = (int)(u / SPT), g0 = 2 * (int)(u % SPT);
                uint8_t* st = smem + s * C_::STAGE_BYTES;
                ptx::mbar_arrive_expect_tx(&full[s], C_::STAGE_BYTES);
                load_stage_weights<C_>(st, &full[s], &tmA, &tmE, (tile / p.n_tiles) * 8, g0, pol_stream);
                load_stage_acts<C_>(st, &full[s], &tmB, (tile % p.n_tiles) * (N_TILE / 8), g0, pol_keep);
            }
        }
        __syncwarp();
    } else {
        if (warp == 1) {
            ptx::tmem_alloc(tmem_holder, C_::TMEM_COLS);
            ptx::tmem_relinquish();
        }
        ptx::tc_fence_before();
        ptx::named_barrier(kBarTmem, kThreads - 32);
        ptx::tc_fence_after();
        tmem_base = *tmem_holder;
    }

    if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        const uint32_t smem_base = ptx::smem_u32(smem);
        int it = 0;
        int seg = 0;
        bool ok = true;
        for (long long u = u_begin; u < u_end && ok; ++seg) {
            const long long tile = u / SPT;
            const long long seg_end = min(u_end, (tile + 1) * SPT);
            const int b = seg & 1;
            if (!ptx::mbar_wait_bounded(&acc_empty[b], (uint32_t)((seg >> 1) & 1) ^ 1u, kWaitLimitNs)) {
                if (lane == 0) atomicOr(&g_spmm24_status, kStatusMmaTimeout);
                break;
            }
            ptx::tc_fence_after();
            uint32_t accumulate = 0;
            for (; u < seg_end; ++u, ++it) {
                const int s = it % STAGES;
                const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                if (!ptx::mbar_wait_bounded(&full[s], ph, kWaitLimitNs)) {
                    if (lane == 0) atomicOr(&g_spmm24_status, kStatusMmaTimeout);
                    ok = false;
                    break;
                }
                if (lane == 0 && u == u_begin) SPMM24_STAMP(2);
                if (lane == 0 && u == u_end - 1) SPMM24_STAMP(3);
                ptx::tc_fence_after();
                if (2 * (int)(u % SPT) + 1 >= p.groups) patch_tail_metadata<C_>(smem + s * C_::STAGE_BYTES, lane);
                if (lane == 0) {
                    mma_stage<C_, N_TILE>(smem_base + s * C_::STAGE_BYTES, tmem_base + C_::META_COL + 4 * s,
                                          tmem_base + (uint32_t)(b * N_TILE), accumulate, 0u);
                    ptx::tc_commit(&empty[s]);
                }
                __syncwarp();
            }
            if (lane == 0) ptx::tc_commit(&acc_full[b]);
            __syncwarp();
        }
    } else if (warp >= 2) {
        // ----------------------------------------------------------- epilogue
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const int etid = threadIdx.x - 64;
        const bool vec_ok = (p.N % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0);
        ptx::grid_dep_wait();  // C and the workspace may be in use by the previous grid
        int seg = 0;
        for (long long u = u_begin; u < u_end; ++seg) {
            const long long tile = u / SPT;
            const long long tile_begin = tile * SPT, tile_end = tile_begin + SPT;
            const long long seg_end = min(u_end, tile_end);
            const int b = seg & 1;
            const bool publish = u != tile_begin;  // range starts inside the tile: someone else finishes it
            float acc[N_TILE];
#pragma unroll
            for (int e = 0; e < N_TILE; ++e) acc[e] = 0.f;
            if (!publish && seg_end != tile_end) {
                // Finisher of a shared tile: the partners (the CTAs after this
                // one up to the tile's last unit) published their shares at
                // the start of their ranges.  Collect them now, while this
                // segment is still streaming.
                const int c_last = sk_cta_of(tile_end - 1, U, p.grid);
                if (etid == 0) {
                    for (int pc = cta + 1; pc <= c_last; ++pc)
                        if (!ptx::wait_flag_bounded(p.flags + pc, kWaitLimitNs))
                            atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
                }
                ptx::named_barrier(kBarEpi, kEpiThreads);
                for (int pc = cta + 1; pc <= c_last; ++pc) {
                    const float* src = p.ws + ((size_t)pc * kTileM + row) * N_TILE;
#pragma unroll
                    for (int e = 0; e < N_TILE; e += 4) {
                        const float4 x = __ldcg(reinterpret_cast<const float4*>(src + e));
                        acc[e] += x.x; acc[e + 1] += x.y; acc[e + 2] += x.z; acc[e + 3] += x.w;
                    }
                }
                ptx::named_barrier(kBarEpi, kEpiThreads);
                if (etid == 0)
                    for (int pc = cta + 1; pc <= c_last; ++pc) ptx::st_relaxed_gpu(p.flags + pc, 0u);  // ready for the next launch
            }
            if (!ptx::mbar_wait_bounded(&acc_full[b], (uint32_t)((seg >> 1) & 1), kWaitLimitNs))
                atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
            if (etid == 0) SPMM24_STAMP(4);
            ptx::tc_fence_after();
            __syncwarp();
            float v[N_TILE];
#pragma unroll
            for (int c = 0; c < N_TILE / 16; ++c) {
                uint32_t r[16];
                ptx::tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * N_TILE + c * 16), r);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e) v[c * 16 + e] = __uint_as_float(r[e]);
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&acc_empty[b]);  // accumulator buffer b may be reused

            if (publish) {
                float* slot = p.ws + ((size_t)cta * kTileM + row) * N_TILE;
#pragma unroll
                for (int e = 0; e < N_TILE; e += 4)
                    __stcg(reinterpret_cast<float4*>(slot + e), make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]));
                __threadfence();
                ptx::named_barrier(kBarEpi, kEpiThreads);
                if (etid == 0) ptx::st_release_gpu(p.flags + cta, 1u);
            } else {
                const int m_tile = (int)(tile / p.n_tiles), n_tile = (int)(tile % p.n_tiles);
                const int gm = m_tile * kTileM + row;
                const int n0 = n_tile * N_TILE;
                if (gm < p.M) {
#pragma unroll
                    for (int e = 0; e < N_TILE; ++e) v[e] += acc[e];
                    __half* out = p.C + (size_t)gm * p.N + n0;
#pragma unroll
                    for (int e = 0; e < N_TILE; e += 8)
                        if (n0 + e < p.N) store_h8(out + e, v + e, vec_ok, p.N - n0 - e);
                }
            }
            u = seg_end;
        }
    }

    if (threadIdx.x == 64) SPMM24_STAMP(5);
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, C_::TMEM_COLS);
    }
    if (threadIdx.x == 0) SPMM24_STAMP(6);
}

}  // namespace spmm24
