// spmm24_kernel.cuh -- the sm_100a 2:4 sparse SpMM kernel, C = A_sparse * B.
//
// Replaces SpMM_N2M4_Kernel (SpeakOutLoudly/CUDA-Repo src/SpMM_Kernel.cuh:301)
// and the separate split-K pass SplitK_Reduction (src/reduce_Kernel.cuh:27).
//
// Input formats are the reference ABI's, unchanged:
//   A  compressed fp16 values, 16x8 blocks band-major (test/utils.h:114-147):
//      band b (16 rows), 16-K block q, row r -> 8 halves at ((b*K/16+q)*16+r)*8
//   E  reordered 2-bit metadata (test/utils.h:155-185): per band and 64-K
//      group g, 8 rows of 16 bytes; row i holds four u32 words
//      (row i, block t) | (row i+8, block t) << 16 for t = 0..3
//   B  packed: N/8 strips of K x 8 row-major halves (test/utils.h:188-229)
//   C  row-major M x N fp16
//
// Mapping onto tcgen05.mma.sp (kind::f16, M=128, K=32 logical per MMA):
//   One pipeline stage covers two 64-K groups g0, g0+1 (128 logical K).
//   A single tcgen05.cp.128x128b moves the stage's metadata straight from
//   the reference layout into TMEM: smem row l = 16*band + 8*h + i (h picks
//   the group) lands in TMEM lane l, its four words in four columns.  The
//   sparse MMA reads lane m0 + 8*k1 + 16*band for rows (m0, m0+8) of a band
//   and the k1-th 16-K half of its 32-K step, so MMA j of the stage consumes
//   the K-slices {group g0 block j, group g0+1 block j}.  A and B are laid
//   out in shared memory with the same permutation of 16-K blocks, which is
//   free (the TMA boxes do it) and leaves the sum over K unchanged.
//
// Roles (192 threads):
//   warp 0     TMA producer (one elected lane)
//   warp 1     TMEM allocator, tcgen05.cp + tcgen05.mma issuer (one lane)
//   warps 2-5  epilogue: TMEM -> registers -> shared -> coalesced fp16 stores
// Split-K runs as a thread-block cluster of S CTAs along K; the partial
// fp32 tiles are reduce-scattered through distributed shared memory (no
// global workspace, no second launch, fixed summation order).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "ptx_sm100.cuh"

namespace spmm24 {

constexpr int kTileM = 128;          // rows of C per CTA (one M=128 MMA)
constexpr int kThreads = 192;        // 6 warps
constexpr int kEpiThreads = 128;     // warps 2..5
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s bound on any wait

// Status bits written to the device status word when a bounded wait gives up.
constexpr uint32_t kStatusProducerTimeout = 1u;
constexpr uint32_t kStatusMmaTimeout = 2u;
constexpr uint32_t kStatusEpilogueTimeout = 4u;

// Sticky device status word (per device, per process).  Bounded waits that
// give up OR their bit in; the host reads and clears it through
// spmm24_device_status().
static __device__ uint32_t g_spmm24_status;

struct KernelParams {
    __half* C;
    int M, N, K;
    int groups;        // K / 64
    int stages_total;  // ceil(groups / 2)
    int split;         // CTAs per cluster along K
};

template <int N_TILE, int STAGES>
struct Cfg {
    static_assert(N_TILE % 16 == 0 && N_TILE >= 16 && N_TILE <= 256, "M=128 sparse MMA needs N % 16 == 0");
    static constexpr int A_BYTES = 8 * 8 * 256;          // 8 16-K blocks x 8 bands x (16 rows x 16 B)
    static constexpr int B_BYTES = (N_TILE / 8) * 2048;  // strips x (4 blocks x 2 groups x 256 B)
    static constexpr int E_BYTES = 16 * 128;             // 16 core matrices of 8 x 16 B
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + E_BYTES;
    static constexpr int BAR_OFFSET = STAGES * STAGE_BYTES;
    static constexpr int NUM_BARS = 2 * STAGES + 1;
    static constexpr int HOLDER_OFFSET = BAR_OFFSET + NUM_BARS * 8;
    static constexpr int SMEM_BYTES = HOLDER_OFFSET + 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to align the base to 1024 B
    static constexpr int META_COL = N_TILE;               // TMEM column of the metadata ring
    static constexpr int TMEM_NEED = N_TILE + 4 * STAGES;
    static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128
                                                          : TMEM_NEED <= 256 ? 256 : 512;
    static constexpr int RED_PITCH = N_TILE + 4;  // floats per row of the reduction buffer
    static_assert(TMEM_NEED <= 512, "TMEM overflow");
    static_assert(SMEM_ALLOC <= 232448, "shared memory overflow");
    // The reduction buffer reuses the stage ring: S sources x ceil(128/S) rows.
    static_assert((kTileM + 7) * RED_PITCH * 4 <= STAGES * STAGE_BYTES, "reduction buffer does not fit");
};

// Shared-memory matrix descriptor, canonical no-swizzle layout (version 1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor: sparse, D=f32, A=B=f16, A K-major, B MN-major.
template <int N_TILE>
__host__ __device__ constexpr uint32_t make_idesc() {
    return (1u << 2) | (1u << 4) | (0u << 7) | (0u << 10) | (0u << 15) | (1u << 16) |
           ((uint32_t)(N_TILE >> 3) << 17) | ((uint32_t)(kTileM >> 4) << 24);
}

template <int N_TILE, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
spmm24_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmE, const KernelParams p) {
    using C_ = Cfg<N_TILE, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C_::BAR_OFFSET);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C_::HOLDER_OFFSET);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int S = p.split;
    const int rank = (S > 1) ? (int)ptx::cluster_ctarank() : 0;
    const int n_tile = blockIdx.y;
    const int m_tile = blockIdx.z;
    const int band0 = m_tile * (kTileM / 16);
    const int strip0 = n_tile * (N_TILE / 8);

    // This CTA's share of the K stages (each stage = two 64-K groups).
    const int st_base = p.stages_total / S, st_rem = p.stages_total % S;
    const int st_begin = rank * st_base + min(rank, st_rem);
    const int st_count = st_base + (rank < st_rem ? 1 : 0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        ptx::mbar_init(acc_full, 1);
        ptx::fence_mbarrier_init();
        ptx::fence_proxy_async_smem();
        ptx::prefetch_tmap(&tmA);
        ptx::prefetch_tmap(&tmB);
        ptx::prefetch_tmap(&tmE);
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_holder, C_::TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    const uint32_t smem_base = ptx::smem_u32(smem);

    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            const uint64_t pol_stream = ptx::policy_evict_first();  // A, E: read once
            const uint64_t pol_keep = ptx::policy_evict_last();     // B: re-read by every M tile
            for (int it = 0; it < st_count; ++it) {
                const int s = it % STAGES;
                const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                if (!ptx::mbar_wait_bounded(&empty[s], ph ^ 1u, kWaitLimitNs)) {
                    atomicOr(&g_spmm24_status, kStatusProducerTimeout);
                    break;
                }
                uint8_t* st = smem + s * C_::STAGE_BYTES;
                ptx::mbar_arrive_expect_tx(&full[s], C_::STAGE_BYTES);
                const int g0 = 2 * (st_begin + it);
                // A: box (128 halves, 8 bands, 8 blocks) -> smem [block][band][256 B]
                ptx::tma_load_3d(st, &tmA, &full[s], 0, band0, 4 * g0, pol_stream);
                // B: box (128 halves, 2 groups, 4 blocks, strips) -> smem [strip][block][group][256 B]
                ptx::tma_load_4d(st + C_::A_BYTES, &tmB, &full[s], 0, g0, 0, strip0, pol_keep);
                // E: box (128 words, 8 bands) -> smem [band][group][128 B]
                ptx::tma_load_2d(st + C_::A_BYTES + C_::B_BYTES, &tmE, &full[s], 64 * g0, band0, pol_stream);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        constexpr uint32_t idesc = make_idesc<N_TILE>();
        uint32_t accumulate = 0;
        for (int it = 0; it < st_count; ++it) {
            const int s = it % STAGES;
            const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
            if (!ptx::mbar_wait_bounded(&full[s], ph, kWaitLimitNs)) {
                if (lane == 0) atomicOr(&g_spmm24_status, kStatusMmaTimeout);
                break;
            }
            ptx::tc_fence_after();
            const uint32_t st = smem_base + s * C_::STAGE_BYTES;
            const uint32_t stB = st + C_::A_BYTES;
            const uint32_t stE = stB + C_::B_BYTES;
            if (2 * (st_begin + it) + 1 >= p.groups) {
                // Final stage of an odd number of 64-K groups: the second
                // group is past K, so TMA filled its A, B and metadata with
                // zeros.  Give those metadata rows a valid ordered index
                // pattern (kept positions 0,1 in every group of four); the
                // zero A values keep their contribution at zero.
                uint8_t* e = smem + s * C_::STAGE_BYTES + C_::A_BYTES + C_::B_BYTES;
                const uint4 pat = make_uint4(0x44444444u, 0x44444444u, 0x44444444u, 0x44444444u);
                for (int c = lane; c < 64; c += 32) {
                    const int cm = c >> 3;  // which of the 8 second-group core matrices
                    *reinterpret_cast<uint4*>(e + (2 * cm + 1) * 128 + (c & 7) * 16) = pat;
                }
                ptx::fence_proxy_async_smem();
                __syncwarp();
            }
            if (lane == 0) {
                const uint32_t meta_col = tmem_base + C_::META_COL + 4 * s;
                ptx::tmem_cp_128x128b(meta_col, smem_desc(stE, 0, 128));
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint64_t adesc = smem_desc(st + j * 2048, 4 * 2048, 128);
                    const uint64_t bdesc = smem_desc(stB + j * 512, 128, 2048);
                    ptx::mma_sp_f16(tmem_base, adesc, bdesc, meta_col + (j & 2), idesc | (uint32_t)(j & 1),
                                    accumulate);
                    accumulate = 1;
                }
                ptx::tc_commit(&empty[s]);
            }
            __syncwarp();
        }
        if (lane == 0) ptx::tc_commit(acc_full);
        __syncwarp();
    }

    // ----------------------------------------------------------- epilogue
    // Reduction buffer red[src][row][RED_PITCH] (fp32) reuses the stage ring.
    const int rows_per = (kTileM + S - 1) / S;
    float* red = reinterpret_cast<float*>(smem);
    const bool epi = warp >= 2;
    if (epi) {
        if (!ptx::mbar_wait_bounded(acc_full, 0, kWaitLimitNs)) atomicOr(&g_spmm24_status, kStatusEpilogueTimeout);
        ptx::tc_fence_after();
    }
    __syncwarp();
    if (S > 1) ptx::cluster_sync();  // every CTA's accumulator is final and its ring is idle
    if (epi) {
        const int quad = warp & 3;  // TMEM lane quadrant this warp may access
        const int row = quad * 32 + lane;
        const int owner = (row * S) / kTileM;
        const int owner_start = (kTileM * owner + S - 1) / S;
        const int lr = row - owner_start;
        float* dst_row = red + ((size_t)rank * rows_per + lr) * C_::RED_PITCH;
        const uint32_t dst_local = ptx::smem_u32(dst_row);
        const uint32_t dst = (S > 1) ? ptx::mapa_shared(dst_local, (uint32_t)owner) : dst_local;
#pragma unroll 1
        for (int c = 0; c < N_TILE / 16; ++c) {
            uint32_t v[16];
            ptx::tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(c * 16), v);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t a = dst + (uint32_t)((c * 16 + q * 4) * 4);
                if (S > 1) {
                    ptx::st_cluster_v4(a, __uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                       __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
                } else {
                    *reinterpret_cast<float4*>(dst_row + c * 16 + q * 4) =
                        make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                    __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
                }
            }
        }
        ptx::tc_fence_before();
    }
    __syncwarp();
    if (S > 1) {
        ptx::cluster_sync();  // all partial rows delivered to their owners
    } else if (epi) {
        asm volatile("barrier.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
    }
    if (epi) {
        // Owner side: sum the S partial copies of this CTA's rows in a fixed
        // order, round to fp16 and store with 16-byte coalesced writes.
        const int my_start = (kTileM * rank + S - 1) / S;
        const int my_end = (kTileM * (rank + 1) + S - 1) / S;
        const int nrows = my_end - my_start;
        constexpr int CHUNKS = N_TILE / 8;
        const int m0 = m_tile * kTileM;
        const int n0 = n_tile * N_TILE;
        const bool vec_ok = (p.N % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0);
        for (int w = threadIdx.x - 64; w < nrows * CHUNKS; w += kEpiThreads) {
            const int lr = w / CHUNKS;
            const int ch = w % CHUNKS;
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
            __half* out = p.C + (size_t)gm * p.N + gn;
            if (vec_ok) {
                __align__(16) __half h[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) h[e] = __float2half_rn(acc[e]);
                *reinterpret_cast<uint4*>(out) = *reinterpret_cast<const uint4*>(h);
            } else {
                const int lim = min(8, p.N - gn);
                for (int e = 0; e < lim; ++e) out[e] = __float2half_rn(acc[e]);
            }
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, C_::TMEM_COLS);
    }
}

}  // namespace spmm24
