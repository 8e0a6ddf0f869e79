// spmm24_grouped.cuh -- one persistent launch for a group of independent
// narrow-N (decode) 2:4 SpMMs.
//
// A decode step runs many SpMMs whose weights are each read once (the
// LLaMA-7B projections at N <= 32 tokens).  Launched one by one, every call
// pays a dependency release, a pipeline fill and a split-K epilogue at its
// end, during which the weight stream stops.  Here one CTA per SM walks a
// list of whole 128-row tiles, possibly of several problems, and its TMA
// producer streams the next tile's weights into the same stage ring while
// the previous tile's accumulator drains, so the stream does not stop
// between tiles or problems.  There is no K split, hence no reduction: a
// tile's full K goes into one TMEM accumulator, and two accumulators
// alternate so the epilogue of tile j overlaps the main loop of tile j + 1.
//
// The host balances the tiles over the CTAs (longest processing time first,
// cost = the tile's 128-K stages) and passes each CTA's list in the kernel
// parameters, with one TMA descriptor triple per problem.
//
// Instantiations: the plain 16-bit SpMM (C = A * B rounded, fp16 or bf16,
// with an optional fused all-gather); EPI, each problem with its own
// epilogue (alpha, bias, activation, residual, packed-B output); FP8, the
// fp8 operand formats of spmm24_launch_fp8 (kind::f8f6f4, stages of 256 K)
// with the general epilogue (alpha carries the dequantisation scale).
//
// Roles (192 threads): warp 0 TMA producer (lane 0), warp 1 TMEM allocator
// and MMA issuer, warps 2-5 epilogue (TMEM -> registers -> C).  Every wait
// is bounded (kWaitLimitNs); a wait that gives up records a status bit and
// the role stops, the others give up in turn, TMEM is freed.
#pragma once
#include "spmm24_common.cuh"

namespace spmm24 {

constexpr int kGroupMaxProblems = 16;
constexpr int kGroupMaxTiles = 2048;  // schedule entries (128-row tiles) per launch
constexpr int kGroupMaxCtas = 160;
constexpr int kGroupTileN = 32;       // N <= 32: columns of B past N are zero-filled by TMA, never fetched
constexpr int kGroupStages = 8;
// K split (SPLIT = 2 or 4, for groups with fewer tiles than SMs): a cluster
// of SPLIT CTAs takes each tile, one share of its K stages each; CTAs 1 ..
// SPLIT-1 push their fp32 partials (128 x 32) into receive slots of CTA 0
// through distributed shared memory, which adds them, in rank order, before
// the epilogue.  Each pushing CTA has two slots that alternate, like the
// accumulators; the ring gives up stages for them (SPLIT = 2: one, fp8 two;
// SPLIT = 4: four, fp8 four).
constexpr int kGroupSplitStages = 7;
constexpr int kGroupSplitStagesFp8 = 6;
constexpr int kGroupSplit4Stages = 4;
constexpr int kGroupRecvPitch = kGroupTileN + 4;  // floats per received row (16-byte reads free of bank conflicts)

struct GroupProblem {
    uint16_t* C;       // M x N, fp16 or bf16, row-major (or packed-B with epi.packed)
    int M, N, K;
    int groups;        // K / 64 (fp8: K / 128, the metadata groups)
    int stages_total;  // ceil(groups / 2): stages per tile
    // The problem's epilogue (EPI and FP8 instantiations) and its fused
    // all-gather (every instantiation; epi.gather_n > 0): output row gm goes
    // to row gather_row0 + gm of every rank's full row-major C, or once
    // through the full C's multicast address.
    Epilogue epi;
};

struct GroupParams {
    CUtensorMap tmA[kGroupMaxProblems];
    CUtensorMap tmB[kGroupMaxProblems];
    CUtensorMap tmE[kGroupMaxProblems];
    GroupProblem prob[kGroupMaxProblems];
    int n_problems;
    int weights_static;
    int bf16;
    uint32_t mma_fmt;  // fp8: operand-format bits of the instruction descriptor
    // Cross-GPU barrier at the end of the launch (bar_n > 0): when every CTA
    // of this grid has stored its rows, the last one publishes this rank's
    // next epoch into slot bar_rank of every rank's flag array and waits,
    // bounded, until every slot of its own array has reached it.  Word bar_n
    // of the own array counts finished CTAs (wraps to zero every launch).
    uint32_t* bar_flags[kMaxGatherRanks];
    int bar_n, bar_rank;
    unsigned long long bar_limit_ns;
    // CTA c (SPLIT > 1: cluster c) processes sched[sched_off[c] ..
    // sched_off[c + 1]); an entry is (problem << 12) | m_tile.
    uint16_t sched_off[kGroupMaxCtas + 1];
    uint16_t sched[kGroupMaxTiles];
    SPMM24_TRACE_FIELD
};

template <int STAGES, bool FP8 = false, int SPLIT = 1>
struct GroupCfg : Cfg<kGroupTileN, STAGES, 2, FP8> {
    using B_ = Cfg<kGroupTileN, STAGES, 2, FP8>;
    static constexpr int RECV_OFFSET = B_::RING_BYTES;
    static constexpr int RECV_SLOT_BYTES = kTileM * kGroupRecvPitch * 4;
    static constexpr int RECV_BYTES = (SPLIT - 1) * 2 * RECV_SLOT_BYTES;  // two slots per pushing CTA
    static constexpr uint32_t PARTIAL_BYTES = (uint32_t)kTileM * kGroupTileN * 4;  // pushed per tile
    static constexpr int BAR_OFFSET = RECV_OFFSET + RECV_BYTES;
    // full, empty, acc_full[2], acc_empty[2], recv_full[2 (SPLIT - 1)], slot_free[2], slot_read[2]
    static constexpr int NUM_BARS = 2 * STAGES + 8 + 2 * (SPLIT > 1 ? SPLIT - 1 : 1);
    static constexpr int HOLDER_OFFSET = BAR_OFFSET + NUM_BARS * 8;
    static constexpr int SMEM_BYTES = HOLDER_OFFSET + 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to align the base to 1024 B
    static_assert(SMEM_ALLOC <= 232448, "shared memory overflow");
    static_assert(B_::STAGE_BYTES % 1024 == 0, "stages must stay 1024-byte aligned");
};

__device__ __forceinline__ void group_entry(const GroupParams& p, int t, int& pi, int& m_tile) {
    const uint32_t e = p.sched[t];
    pi = (int)(e >> 12);
    m_tile = (int)(e & 0xFFFu);
}

// Rounds the first N (<= 32) of 32 fp32 values of one output row to C's type
// and stores them at `out` (16-byte stores when N % 8 == 0 and the row is
// 16-byte aligned; through the multicast address `mc` instead when given).
// Fully unrolled with predicates, so v stays in registers.
__device__ __forceinline__ void group_store_row(uint16_t* out, uint16_t* mc, int N, const uint32_t (&v)[32], int bf16,
                                                bool vec) {
    if (vec) {
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
            if (c < N) {
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    w[i] = pack2(__uint_as_float(v[c + 2 * i]), __uint_as_float(v[c + 2 * i + 1]), bf16);
                const uint4 q = make_uint4(w[0], w[1], w[2], w[3]);
                if (mc) ptx::multimem_st_v4(mc + c, q);
                else *reinterpret_cast<uint4*>(out + c) = q;
            }
        }
    } else {
#pragma unroll
        for (int c = 0; c < 32; ++c)
            if (c < N) out[c] = f32_to_elem(__uint_as_float(v[c]), bf16);
    }
}

// This CTA's share [lo, hi) of a tile's `n` stages: all of them, or (K split)
// n / SPLIT each, the first n % SPLIT ranks one more (the partition of the
// cluster kernel's split-K, so both add the same partial sums).
template <int SPLIT>
__device__ __forceinline__ void group_share(int n, int rank, int& lo, int& hi) {
    const int base = n / SPLIT, rem = n % SPLIT;
    lo = rank * base + min(rank, rem);
    hi = lo + base + (rank < rem ? 1 : 0);
}

template <int STAGES, bool EPI = false, bool FP8 = false, int SPLIT = 1>
__global__ void __launch_bounds__(kThreads, 1) spmm24_grouped_kernel(const __grid_constant__ GroupParams p) {
    static_assert(EPI || !FP8, "the fp8 grouped kernel always runs the general epilogue");
    static_assert(SPLIT == 1 || SPLIT == 2 || SPLIT == 4, "K split in one, two or four");
    using C_ = GroupCfg<STAGES, FP8, SPLIT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C_::BAR_OFFSET);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;  // [2]
    uint64_t* acc_empty = acc_full + 2;   // [2]
    // rank 0 of a split: recv_full[2 q + b], the partial of rank q + 1 in its slot b has arrived
    uint64_t* recv_full = acc_empty + 2;
    uint64_t* slot_free = recv_full + 2 * (SPLIT > 1 ? SPLIT - 1 : 1);  // [2] ranks > 0: rank 0 has read slot b
    uint64_t* slot_read = slot_free + 2;  // [2] rank 0: each epilogue warp has read its rows of every slot b
    float* recv = reinterpret_cast<float*>(smem + C_::RECV_OFFSET);  // [SPLIT - 1][2][128][kGroupRecvPitch]
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C_::HOLDER_OFFSET);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rank = SPLIT > 1 ? (int)(ptx::cluster_ctarank() % (uint32_t)SPLIT) : 0;
    const int unit = (int)blockIdx.x / SPLIT;
    const int t_begin = p.sched_off[unit];
    const int t_end = p.sched_off[unit + 1];

    if (threadIdx.x == 0) {
        SPMM24_STAMP(0);
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            ptx::mbar_init(&acc_full[b], 1);
            ptx::mbar_init(&acc_empty[b], kEpiThreads / 32);  // one arrival per epilogue warp
            ptx::mbar_init(&slot_free[b], 1);
            ptx::mbar_init(&slot_read[b], kEpiThreads / 32);
        }
        for (int i = 0; i < 2 * (SPLIT > 1 ? SPLIT - 1 : 1); ++i) ptx::mbar_init(&recv_full[i], 1);
        // Rank 0 of a split arms the receive barriers of its first two tiles
        // now, before the partners can push (the cluster barrier below); the
        // next arm of slot b follows the read of slot b.
        if (SPLIT > 1 && rank == 0)
            for (int q = 0; q < SPLIT - 1; ++q)
                for (int b = 0; b < 2 && t_begin + b < t_end; ++b)
                    ptx::mbar_arrive_expect_tx(&recv_full[2 * q + b], C_::PARTIAL_BYTES);
        ptx::fence_mbarrier_init();
        for (int i = 0; i < p.n_problems; ++i) {
            ptx::prefetch_tmap(&p.tmA[i]);
            ptx::prefetch_tmap(&p.tmB[i]);
            ptx::prefetch_tmap(&p.tmE[i]);
        }
    }
    __syncthreads();
    if (SPLIT > 1) ptx::cluster_sync();  // every CTA's barriers are initialised (and armed)
    if (threadIdx.x == 0) ptx::grid_dep_launch();

    uint32_t tmem_base = 0;
    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        // One walk over (tile, stage) of this CTA's list; the ring index `it`
        // runs on across tiles, so the next tile's weights stream in while
        // the current tile is still being multiplied.
        if (lane == 0) {
            const uint64_t pol_stream = ptx::policy_evict_first();  // A, E: read once
            const uint64_t pol_keep = ptx::policy_evict_last();     // B: re-read by every tile of its problem
            // Walk position: tile t, stage s_in of this CTA's share [lo, hi).
            auto first_of = [&](int t, int& s_in, int& hi) {
                for (; t < t_end; ++t) {
                    int pi, m_tile, lo;
                    group_entry(p, t, pi, m_tile);
                    group_share<SPLIT>(p.prob[pi].stages_total, rank, lo, hi);
                    if (lo < hi) {
                        s_in = lo;
                        return t;
                    }
                }
                return t;
            };
            int pre = 0;
            if (p.weights_static) {  // the first stages' weights before the previous grid ends
                int hi = 0, s_in = 0;
                int t = first_of(t_begin, s_in, hi);
                while (pre < STAGES && t < t_end) {
                    int pi, m_tile;
                    group_entry(p, t, pi, m_tile);
                    ptx::mbar_arrive_expect_tx(&full[pre], C_::STAGE_BYTES);
                    load_stage_weights<C_>(smem + pre * C_::STAGE_BYTES, &full[pre], &p.tmA[pi], &p.tmE[pi],
                                           m_tile * (kTileM / 16), 2 * s_in, pol_stream);
                    ++pre;
                    if (++s_in == hi) t = first_of(t + 1, s_in, hi);
                }
            }
            ptx::grid_dep_wait();
            SPMM24_STAMP(1);
            int hi = 0, s_in = 0;
            int t = first_of(t_begin, s_in, hi);
            for (int it = 0; t < t_end; ++it) {
                int pi, m_tile;
                group_entry(p, t, pi, m_tile);
                const int s = it % STAGES;
                uint8_t* st = smem + s * C_::STAGE_BYTES;
                if (it >= pre) {
                    const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                    if (!ptx::mbar_wait_bounded(&empty[s], ph ^ 1u, kWaitLimitNs)) {
                        atomicOr(&g_spmm24_status, kStatusProducerTimeout);
                        break;
                    }
                    ptx::mbar_arrive_expect_tx(&full[s], C_::STAGE_BYTES);
                    load_stage_weights<C_>(st, &full[s], &p.tmA[pi], &p.tmE[pi], m_tile * (kTileM / 16), 2 * s_in,
                                           pol_stream);
                }
                load_stage_acts<C_>(st, &full[s], &p.tmB[pi], 0, 2 * s_in, pol_keep);
                if (++s_in == hi) t = first_of(t + 1, s_in, hi);
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
        const uint32_t fmt = FP8 ? p.mma_fmt : p.bf16 ? kIdescBf16 : 0u;
        int it = 0;
        bool ok = true;
        for (int j = 0; t_begin + j < t_end && ok; ++j) {
            int pi, m_tile;
            group_entry(p, t_begin + j, pi, m_tile);
            int lo, hi;
            group_share<SPLIT>(p.prob[pi].stages_total, rank, lo, hi);
            const int groups = p.prob[pi].groups;
            const int b = j & 1;
            if (j >= 2) {  // accumulator b still holds tile j - 2 until the epilogue has read it
                if (!ptx::mbar_wait_bounded(&acc_empty[b], (uint32_t)((j >> 1) - 1) & 1u, kWaitLimitNs)) {
                    if (lane == 0) atomicOr(&g_spmm24_status, kStatusMmaTimeout);
                    break;
                }
                ptx::tc_fence_after();
            }
            uint32_t accumulate = 0;
            for (int s_in = lo; s_in < hi; ++s_in, ++it) {
                const int s = it % STAGES;
                if (!ptx::mbar_wait_bounded(&full[s], (uint32_t)(it / STAGES) & 1u, kWaitLimitNs)) {
                    if (lane == 0) atomicOr(&g_spmm24_status, kStatusMmaTimeout);
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                if (2 * s_in + 1 >= groups) patch_tail_metadata<C_>(smem + s * C_::STAGE_BYTES, lane);
                if (lane == 0) {
                    const uint32_t meta_col = tmem_base + C_::META_COL + C_::META_STRIDE * s;
                    const uint32_t d_tmem = tmem_base + (uint32_t)(b * kGroupTileN);
                    if constexpr (FP8)
                        mma_stage_fp8<C_, kGroupTileN>(smem_base + s * C_::STAGE_BYTES, meta_col, d_tmem, accumulate,
                                                       fmt);
                    else
                        mma_stage<C_, kGroupTileN>(smem_base + s * C_::STAGE_BYTES, meta_col, d_tmem, accumulate,
                                                   fmt);
                    ptx::tc_commit(&empty[s]);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) ptx::tc_commit(&acc_full[b]);
            __syncwarp();
        }
    } else if (warp >= 2) {
        // ----------------------------------------------------------- epilogue
        // Thread = output row (TMEM lane); the accumulator is released as
        // soon as it is in registers, then the row is rounded and stored.
        const int quad = warp & 3;  // TMEM lane quadrant this warp may access
        const int row = quad * 32 + lane;
        bool waited = false;
        for (int j = 0; t_begin + j < t_end; ++j) {
            int pi, m_tile;
            group_entry(p, t_begin + j, pi, m_tile);
            const int b = j & 1;
            if (!ptx::mbar_wait_bounded(&acc_full[b], (uint32_t)(j >> 1) & 1u, kWaitLimitNs)) {
                atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
                break;
            }
            ptx::tc_fence_after();
            const int N = p.prob[pi].N;
            int lo, hi;
            group_share<SPLIT>(p.prob[pi].stages_total, rank, lo, hi);
            uint32_t v[32];
            if (lo < hi) {
                uint32_t v0[16], v1[16];
                const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * kGroupTileN);
                ptx::tmem_ld_32x32b_x16(taddr, v0);
                if (N > 16) ptx::tmem_ld_32x32b_x16(taddr + 16, v1);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    v[i] = v0[i];
                    v[16 + i] = N > 16 ? v1[i] : 0u;
                }
            } else {  // a tile of fewer stages than SPLIT leaves the last ranks without a share
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = 0u;
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&acc_empty[b]);
            if constexpr (SPLIT > 1) {
                if (rank > 0) {
                    // push this row's partial into rank 0's slot (rank - 1, b),
                    // once rank 0 has read what the slot held two tiles ago
                    if (j >= 2 && !ptx::mbar_wait_bounded(&slot_free[b], (uint32_t)((j >> 1) - 1) & 1u, kWaitLimitNs)) {
                        atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
                        break;
                    }
                    const int q = 2 * (rank - 1) + b;
                    float* slot = recv + (size_t)q * kTileM * kGroupRecvPitch;
                    const uint32_t dst = ptx::mapa_shared(ptx::smem_u32(slot + row * kGroupRecvPitch), 0u);
                    const uint32_t bar = ptx::mapa_shared(ptx::smem_u32(&recv_full[q]), 0u);
#pragma unroll
                    for (int c = 0; c < kGroupTileN / 4; ++c)
                        ptx::st_async_v4(dst + 16u * c, __uint_as_float(v[4 * c]), __uint_as_float(v[4 * c + 1]),
                                         __uint_as_float(v[4 * c + 2]), __uint_as_float(v[4 * c + 3]), bar);
                    continue;  // rank 0 finishes the tile
                }
                // rank 0: add the partners' partials (fixed order: own share of K
                // first, then ranks 1, 2, ...)
                bool got = true;
                for (int r = 1; r < SPLIT && got; ++r) {
                    const int q = 2 * (r - 1) + b;
                    if (!ptx::mbar_wait_bounded(&recv_full[q], (uint32_t)(j >> 1) & 1u, kWaitLimitNs)) {
                        atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
                        got = false;
                        break;
                    }
                    const float* rr = recv + ((size_t)q * kTileM + row) * kGroupRecvPitch;
#pragma unroll
                    for (int c = 0; c < kGroupTileN / 4; ++c) {
                        const float4 x = *reinterpret_cast<const float4*>(rr + 4 * c);
                        v[4 * c] = __float_as_uint(__uint_as_float(v[4 * c]) + x.x);
                        v[4 * c + 1] = __float_as_uint(__uint_as_float(v[4 * c + 1]) + x.y);
                        v[4 * c + 2] = __float_as_uint(__uint_as_float(v[4 * c + 2]) + x.z);
                        v[4 * c + 3] = __float_as_uint(__uint_as_float(v[4 * c + 3]) + x.w);
                    }
                }
                if (!got) break;
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&slot_read[b]);  // this warp's rows of every slot b are read
                if (threadIdx.x == 64 && t_begin + j + 2 < t_end) {
                    // once every warp has read slot b: arm it for its next tile
                    // and tell the partners they may push into it
                    if (ptx::mbar_wait_bounded(&slot_read[b], (uint32_t)(j >> 1) & 1u, kWaitLimitNs)) {
                        for (int r = 1; r < SPLIT; ++r) {
                            ptx::mbar_arrive_expect_tx(&recv_full[2 * (r - 1) + b], C_::PARTIAL_BYTES);
                            ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_u32(&slot_free[b]), (uint32_t)r));
                        }
                    } else {
                        atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
                    }
                }
            }
            if (!waited) {  // C may be read or written by the previous grid
                ptx::grid_dep_wait();
                waited = true;
            }
            const int gm = m_tile * kTileM + row;
            const GroupProblem& q = p.prob[pi];
            if (gm < q.M) {
                if constexpr (EPI) {
                    // alpha, bias, activation, residual, rounding and the store
                    // (row-major, packed-B or gathered), 8 columns at a time
                    const bool vec = (N % 8 == 0) && ((reinterpret_cast<uintptr_t>(q.C) & 15u) == 0) &&
                                     ((reinterpret_cast<uintptr_t>(q.epi.residual) & 15u) == 0);
                    const bool plain = epilogue_is_plain(q.epi);
#pragma unroll
                    for (int c = 0; c < 32; c += 8) {
                        if (c < N) {
                            float y[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) y[e] = __uint_as_float(v[c + e]);
                            epilogue_store8(q.C, y, q.epi, gm, c, q.M, N, vec, plain);
                        }
                    }
                } else if (q.epi.gather_n) {  // destinations are 16-byte aligned (checked by the host)
                    const size_t off = (size_t)(q.epi.gather_row0 + gm) * N;
                    if (q.epi.gather_mc && N % 8 == 0) {
                        group_store_row(nullptr, q.epi.gather_mc + off, N, v, p.bf16, true);
                    } else {
                        for (int d = 0; d < q.epi.gather_n; ++d)
                            group_store_row(q.epi.gather_dst[d] + off, nullptr, N, v, p.bf16, N % 8 == 0);
                    }
                } else {
                    group_store_row(q.C + (size_t)gm * N, nullptr, N, v, p.bf16,
                                    (N % 8 == 0) && ((reinterpret_cast<uintptr_t>(q.C) & 15u) == 0));
                }
            }
        }
    }

    if (threadIdx.x == 64) SPMM24_STAMP(5);
    ptx::tc_fence_before();
    if (p.bar_n) __threadfence_system();  // this thread's stores (peer rows included) before the CTA's count
    __syncthreads();
    if (p.bar_n) {
        // The last CTA of the grid to get here runs the cross-GPU barrier:
        // thread 0 finds out and reads the epoch; then thread r publishes it
        // into rank r's flag array and waits, bounded, for rank r's epoch in
        // this rank's array -- one thread per rank, so the remote stores and
        // the waits overlap instead of running one rank after another.
        __shared__ uint32_t bar_epoch, bar_last;
        uint32_t* own = p.bar_flags[p.bar_rank];
        if (threadIdx.x == 0) {
            const uint32_t done = atomicInc(own + p.bar_n, gridDim.x - 1u);
            bar_last = done == gridDim.x - 1u ? 1u : 0u;
            if (bar_last) {
                __threadfence_system();
                bar_epoch = ptx::ld_acquire_sys(own + p.bar_rank) + 1u;
            }
        }
        __syncthreads();
        if (bar_last && threadIdx.x < p.bar_n) {
            const int r = threadIdx.x;
            const uint32_t epoch = bar_epoch;
            ptx::st_release_sys(p.bar_flags[r] + p.bar_rank, epoch);
            const uint64_t t0 = ptx::globaltimer();
            while ((int)(ptx::ld_acquire_sys(own + r) - epoch) < 0) {
                ptx::nanosleep_ns(100);
                if (ptx::globaltimer() - t0 > p.bar_limit_ns) {
                    atomicOr(&g_spmm24_status, kStatusBarrierTimeout);
                    break;
                }
            }
        }
    }
    if (SPLIT > 1) ptx::cluster_sync();  // no CTA leaves while a partner may still reach its shared memory
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, C_::TMEM_COLS);
    }
}

}  // namespace spmm24
