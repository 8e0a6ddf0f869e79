// spmm24_common.cuh -- pieces shared by the sm_100a 2:4 SpMM kernels: the
// shared-memory stage layout, the TMA loads of one 128-K stage, the sparse
// MMAs of one stage, and the metadata fix-up for an odd final 64-K group.
//
// Input formats are the reference ABI's, unchanged (SpeakOutLoudly/CUDA-Repo
// test/utils.h:91-229):
//   A  compressed fp16 values, 16x8 blocks band-major: band b (16 rows),
//      16-K block q, row r -> 8 halves at ((b*K/16+q)*16+r)*8
//   E  reordered 2-bit metadata: per band and 64-K group g, 8 rows of 16
//      bytes; row i holds four u32 words (row i, block t) | (row i+8, block t)<<16
//   B  packed: ceil(N/8) strips of K x 8 row-major halves
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
//   out in shared memory with the same permutation of 16-K blocks -- the TMA
//   boxes do it -- which leaves the sum over K unchanged.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "ptx_sm100.cuh"

namespace spmm24 {

constexpr int kTileM = 128;                        // rows of C per tile (one M=128 MMA)
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s bound on any wait

// Status bits written to the device status word when a bounded wait gives up.
constexpr uint32_t kStatusProducerTimeout = 1u;
constexpr uint32_t kStatusMmaTimeout = 2u;
constexpr uint32_t kStatusEpilogueTimeout = 4u;
constexpr uint32_t kStatusBarrierTimeout = 8u;  // cross-GPU barrier of the fused all-gather

// Sticky device status word (per device, per process).  Bounded waits that
// give up OR their bit in; the host reads and clears it through
// spmm24_device_status().
static __device__ uint32_t g_spmm24_status;

// Optional per-CTA timeline for performance work: builds that define
// SPMM24_TRACE record %globaltimer and clock64 stamps into g_spmm24_trace
// (16 words per CTA; each launch writes its own records starting at the
// trace_base its parameters carry).  The product build compiles the stamps
// away.
#ifdef SPMM24_TRACE
__device__ unsigned long long* g_spmm24_trace;
__device__ __forceinline__ void trace_stamp(long long base, int slot) {
    if (g_spmm24_trace) {
        const size_t cta = (size_t)base + blockIdx.x + (size_t)gridDim.x * (blockIdx.y + (size_t)gridDim.y * blockIdx.z);
        unsigned long long t, c;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        c = clock64();
        g_spmm24_trace[cta * 16 + 2 * slot] = t;
        g_spmm24_trace[cta * 16 + 2 * slot + 1] = c;
    }
}
#define SPMM24_STAMP(slot) ::spmm24::trace_stamp(p.trace_base, slot)
#define SPMM24_TRACE_FIELD long long trace_base;
#else
#define SPMM24_STAMP(slot) \
    do {                   \
    } while (0)
#define SPMM24_TRACE_FIELD
#endif

// FP8: a stage covers 256 logical K of fp8 operands in the same A and B
// bytes (A: 8 blocks of 32 K; B: two 128-byte-swizzled halves of N_TILE
// rows x 128 K, each a multiple of 1024 bytes) and twice the metadata (two
// 128-K groups, 8 TMEM columns).
template <int N_TILE, int STAGES, int ACC_BUFS, bool FP8 = false>
struct Cfg {
    static_assert(N_TILE % 16 == 0 && N_TILE >= 16 && N_TILE <= 256, "M=128 sparse MMA needs N % 16 == 0");
    static constexpr bool kFp8 = FP8;
    static constexpr int A_BYTES = 8 * 8 * 256;          // 8 16-K blocks x 8 bands x (16 rows x 16 B)
    static constexpr int B_BYTES = (N_TILE / 8) * 2048;  // strips x (4 blocks x 2 groups x 256 B)
    static constexpr int E_BYTES = (FP8 ? 2 : 1) * 16 * 128;  // 16 core matrices of 8 x 16 B per copy
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + E_BYTES;
    static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
    static constexpr int META_COL = ACC_BUFS * N_TILE;  // TMEM column of the metadata ring
    static constexpr int META_STRIDE = FP8 ? 8 : 4;     // metadata columns per stage
    static constexpr int TMEM_NEED = META_COL + META_STRIDE * STAGES;
    static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128
                                                          : TMEM_NEED <= 256 ? 256 : 512;
    static_assert(TMEM_NEED <= 512, "TMEM overflow");
    static_assert(!FP8 || (A_BYTES % 1024 == 0 && (B_BYTES / 2) % 1024 == 0 && STAGE_BYTES % 1024 == 0),
                  "fp8 B halves must start on 1024-byte boundaries (128-byte swizzle atoms)");
};

// Shared-memory matrix descriptor, canonical no-swizzle layout (version 1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// K-major operand in the 128-byte swizzled layout: rows of 128 bytes, 8-row
// atoms of 1024 bytes (1024-byte aligned), 16-byte chunk c of row r stored
// at chunk c ^ (r % 8) -- what TMA writes with SWIZZLE_128B.  addr may
// point inside the first row (a K offset within the 128 bytes); the leading
// offset is unused for this layout.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

// Instruction descriptor: sparse, D=f32, A=B=f16, A K-major, B MN-major.
template <int N_TILE>
__host__ __device__ constexpr uint32_t make_idesc() {
    return (1u << 2) | (1u << 4) | (0u << 7) | (0u << 10) | (0u << 15) | (1u << 16) |
           ((uint32_t)(N_TILE >> 3) << 17) | ((uint32_t)(kTileM >> 4) << 24);
}
// Operand-format bits that turn an f16 descriptor into a bf16 one (A and B).
constexpr uint32_t kIdescBf16 = (1u << 7) | (1u << 10);

// The weight (A + metadata) half of one stage's loads.  g0: the stage's
// first 64-K group (fp8: its first 128-K metadata group).
template <class C_>
__device__ __forceinline__ void load_stage_weights(uint8_t* st, uint64_t* bar, const CUtensorMap* tmA,
                                                   const CUtensorMap* tmE, int band0, int g0, uint64_t pol) {
    // A: box (128 halves, 8 bands, 8 blocks) -> smem [block][band][256 B]
    // (fp8: the same bytes, blocks of 32 K)
    ptx::tma_load_3d(st, tmA, bar, 0, band0, 4 * g0, pol);
    if constexpr (C_::kFp8) {
        // E: box (256 B of one band and group, 8 bands, 2 groups) -> smem [group][band][256 B]
        ptx::tma_load_3d(st + C_::A_BYTES + C_::B_BYTES, tmE, bar, 0, band0, g0, pol);
    } else {
        // E: box (128 words, 8 bands) -> smem [band][group][128 B]
        ptx::tma_load_2d(st + C_::A_BYTES + C_::B_BYTES, tmE, bar, 64 * g0, band0, pol);
    }
}

// The activation (B) half of one stage's loads.
template <class C_>
__device__ __forceinline__ void load_stage_acts(uint8_t* st, uint64_t* bar, const CUtensorMap* tmB, int strip0, int g0,
                                                uint64_t pol) {
    if constexpr (C_::kFp8) {
        // B (N x K bytes): two boxes of (128 bytes of K, N_TILE rows), 128-byte
        // swizzle -> smem [half][row][128 B]
        ptx::tma_load_2d(st + C_::A_BYTES, tmB, bar, 128 * g0, 8 * strip0, pol);
        ptx::tma_load_2d(st + C_::A_BYTES + C_::B_BYTES / 2, tmB, bar, 128 * g0 + 128, 8 * strip0, pol);
    } else {
        // B: box (128 halves, 2 groups, 4 blocks, strips) -> smem [strip][block][group][256 B]
        ptx::tma_load_4d(st + C_::A_BYTES, tmB, bar, 0, g0, 0, strip0, pol);
    }
}

// Final stage of an odd number of 64-K groups: the second group lies past K,
// so TMA filled its A, B and metadata with zeros.  Give those metadata rows
// a valid ordered index pattern (kept positions 0 and 1 of every group of
// four); the zero A values keep the contribution at zero.  Whole warp.
template <class C_>
__device__ __forceinline__ void patch_tail_metadata(uint8_t* st, int lane) {
    uint8_t* e = st + C_::A_BYTES + C_::B_BYTES;
    const uint4 pat = make_uint4(0x44444444u, 0x44444444u, 0x44444444u, 0x44444444u);
    if constexpr (C_::kFp8) {
        for (int c = lane; c < 128; c += 32)  // the second group: smem [1][band][256 B]
            *reinterpret_cast<uint4*>(e + 2048 + c * 16) = pat;
    } else {
        for (int c = lane; c < 64; c += 32) {
            const int cm = c >> 3;  // which of the 8 second-group core matrices
            *reinterpret_cast<uint4*>(e + (2 * cm + 1) * 128 + (c & 7) * 16) = pat;
        }
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
}

// Metadata copy + the four sparse MMAs of one stage (single thread).
// `fmt` is 0 (f16 operands) or kIdescBf16.
template <class C_, int N_TILE>
__device__ __forceinline__ void mma_stage(uint32_t st_addr, uint32_t meta_col, uint32_t d_tmem, uint32_t& accumulate,
                                          uint32_t fmt) {
    const uint32_t idesc = make_idesc<N_TILE>() | fmt;
    const uint32_t stB = st_addr + C_::A_BYTES;
    const uint32_t stE = stB + C_::B_BYTES;
    ptx::tmem_cp_128x128b(meta_col, smem_desc(stE, 0, 128));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint64_t adesc = smem_desc(st_addr + j * 2048, 4 * 2048, 128);
        const uint64_t bdesc = smem_desc(stB + j * 512, 128, 2048);
        ptx::mma_sp_f16(d_tmem, adesc, bdesc, meta_col + (j & 2), idesc | (uint32_t)(j & 1), accumulate);
        accumulate = 1;
    }
}

// fp8 (kind::f8f6f4, sparse K = 64 logical per MMA).  Instruction
// descriptor: sparse, D=f32, A and B K-major, format bits from the caller
// (A: bit 7 = E5M2, B: bit 10 = E5M2; zero = E4M3).
template <int N_TILE>
__host__ __device__ constexpr uint32_t make_idesc_fp8() {
    return (1u << 2) | (1u << 4) | ((uint32_t)(N_TILE >> 3) << 17) | ((uint32_t)(kTileM >> 4) << 24);
}
constexpr uint32_t kIdescFp8AE5M2 = 1u << 7;
constexpr uint32_t kIdescFp8BE5M2 = 1u << 10;

// Metadata copies + the four fp8 sparse MMAs of one stage (single thread).
// Metadata: each 128-K group is 128 rows x 16 bytes, one tcgen05.cp into
// four TMEM columns (lane = row); MMA j reads columns 2j, 2j+1.  A: MMA j
// takes 32-K blocks 2j, 2j+1 (K-major core matrices, 2048 B apart along K,
// 128 B apart along M).  B: MMA j takes bytes 64 (j % 2) .. + 63 of every
// row of the 128-byte swizzled half j / 2 (N_TILE rows of 128 B).
template <class C_, int N_TILE>
__device__ __forceinline__ void mma_stage_fp8(uint32_t st_addr, uint32_t meta_col, uint32_t d_tmem,
                                              uint32_t& accumulate, uint32_t fmt) {
    const uint32_t idesc = make_idesc_fp8<N_TILE>() | fmt;
    const uint32_t stB = st_addr + C_::A_BYTES;
    const uint32_t stE = stB + C_::B_BYTES;
    ptx::tmem_cp_128x128b(meta_col, smem_desc(stE, 0, 128));
    ptx::tmem_cp_128x128b(meta_col + 4, smem_desc(stE + 2048, 0, 128));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint64_t adesc = smem_desc(st_addr + j * 4096, 2048, 128);
        const uint64_t bdesc = smem_desc_sw128(stB + (j >> 1) * (C_::B_BYTES / 2) + (j & 1) * 64);
        ptx::mma_sp_f8(d_tmem, adesc, bdesc, meta_col + 2 * j, idesc, accumulate);
        accumulate = 1;
    }
}

// ------------------------------------------------------------ epilogue
// Applied after the split-K reduction, before the output is rounded:
//   y = act(alpha * acc + bias[m]) + residual[m, n]
// stored in C's element type and layout.  Row-major C is M x N; the packed
// layout is the next layer's packed B: ceil(N/8) strips of M x 8 (element
// (m, n) at ((n / 8) * M + m) * 8 + n % 8, pad columns zero).
constexpr int kActNone = 0, kActRelu = 1, kActSilu = 2, kActGelu = 3;

constexpr int kMaxGatherRanks = 8;

struct Epilogue {
    const uint16_t* bias;      // M values in C's type, or null
    const uint16_t* residual;  // same type and layout as C, or null
    float alpha;               // accumulator scale
    int act;                   // kAct*
    int packed;                // 1: C (and residual) in packed-B strips
    int bf16;                  // 1: A, B, C, bias and residual are bf16; 0: fp16
    // Fused all-gather of an M-shard: each output row gm is written to row
    // gather_row0 + gm of every rank's full row-major C (peer pointers
    // reached over NVLink), instead of to C.  gather_n == 0: off.
    int gather_n;
    int gather_row0;
    uint16_t* gather_dst[kMaxGatherRanks];
    // Multicast address of the full C (NVSwitch replicates each store into
    // every rank's buffer), or null: one unicast store per rank instead.
    uint16_t* gather_mc;
};

// Stores 16 bytes of row-major output (row gm of the shard, columns gn..) to
// C, or to every rank's full C when the epilogue gathers.
__device__ __forceinline__ void store_row16(uint16_t* C, const Epilogue& e, int gm, int gn, int N, uint4 v) {
    if (e.gather_n) {
        const size_t off = (size_t)(e.gather_row0 + gm) * N + gn;
        if (e.gather_mc) {
            ptx::multimem_st_v4(e.gather_mc + off, v);
        } else {
            for (int d = 0; d < e.gather_n; ++d) *reinterpret_cast<uint4*>(e.gather_dst[d] + off) = v;
        }
    } else {
        *reinterpret_cast<uint4*>(C + (size_t)gm * N + gn) = v;
    }
}
// The element-wise form (N % 8 != 0 or a misaligned C).
__device__ __forceinline__ void store_row_elems(uint16_t* C, const Epilogue& e, int gm, int gn, int N, const uint32_t* w,
                                                int lim) {
    if (e.gather_n) {
        const size_t off = (size_t)(e.gather_row0 + gm) * N + gn;
        for (int d = 0; d < e.gather_n; ++d)
            for (int i = 0; i < lim; ++i) e.gather_dst[d][off + i] = (uint16_t)(w[i >> 1] >> (16 * (i & 1)));
    } else {
        for (int i = 0; i < lim; ++i) C[(size_t)gm * N + gn + i] = (uint16_t)(w[i >> 1] >> (16 * (i & 1)));
    }
}

__device__ __forceinline__ float elem_to_f32(uint16_t h, int bf16) {
    if (bf16) return __uint_as_float((uint32_t)h << 16);
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

__device__ __forceinline__ uint16_t f32_to_elem(float v, int bf16) {
    if (bf16) {
        const __nv_bfloat16 b = __float2bfloat16_rn(v);
        return static_cast<__nv_bfloat16_raw>(b).x;
    }
    const __half h = __float2half_rn(v);
    return static_cast<__half_raw>(h).x;
}

// Hardware tanh approximation (tanh.approx.f32: relative error about 2^-11,
// far below an fp16 / bf16 output ulp).
__device__ __forceinline__ float tanh_fast(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ReLU; SiLU y * sigmoid(y), with sigmoid(y) = 0.5 + 0.5 tanh(y / 2); GELU
// in its tanh form (Hendrycks & Gimpel, 2016): 0.5 y (1 + tanh(sqrt(2 / pi)
// (y + 0.044715 y^3))).  One hardware tanh per element.
__device__ __forceinline__ float activate(float y, int act) {
    if (act == kActRelu) return fmaxf(y, 0.f);
    if (act == kActSilu) return y * fmaf(0.5f, tanh_fast(0.5f * y), 0.5f);
    if (act == kActGelu) return 0.5f * y * (1.f + tanh_fast(0.7978845608028654f * (y + 0.044715f * y * y * y)));
    return y;
}

// Two values rounded to C's type, packed low-first in one word.
__device__ __forceinline__ uint32_t pack2(float a, float b, int bf16) {
    if (bf16) {
        const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<const uint32_t*>(&v);
    }
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// Element offset of (m, n) in C's layout.
__device__ __forceinline__ size_t c_offset(const Epilogue& e, int m, int n, int M, int N) {
    return e.packed ? ((((size_t)(n >> 3) * M + m) << 3) + (n & 7)) : ((size_t)m * N + n);
}

// True when the epilogue only rounds (the plain SpMM): the kernels then take
// a short path with no per-element epilogue work.
__device__ __forceinline__ bool epilogue_is_plain(const Epilogue& e) {
    return e.bias == nullptr && e.residual == nullptr && e.act == kActNone && e.alpha == 1.f;
}

// alpha, bias and activation on n values of row gm (no residual).
// bias_pre: the row's bias already loaded (e.g. prefetched into shared
// memory while the main loop ran), or null to read e.bias[gm].
template <int n>
__device__ __forceinline__ void epilogue_pre(float* y, const Epilogue& e, int gm, const float* bias_pre = nullptr) {
    if (e.alpha != 1.f) {
#pragma unroll
        for (int i = 0; i < n; ++i) y[i] *= e.alpha;
    }
    if (e.bias) {
        const float b = bias_pre ? *bias_pre : elem_to_f32(e.bias[gm], e.bf16);
#pragma unroll
        for (int i = 0; i < n; ++i) y[i] += b;
    }
    if (e.act == kActRelu) {
#pragma unroll
        for (int i = 0; i < n; ++i) y[i] = fmaxf(y[i], 0.f);
    } else if (e.act == kActSilu) {
#pragma unroll
        for (int i = 0; i < n; ++i) y[i] = activate(y[i], kActSilu);
    } else if (e.act == kActGelu) {
#pragma unroll
        for (int i = 0; i < n; ++i) y[i] = activate(y[i], kActGelu);
    }
}

// Rounds 8 values to C's type; columns at or past N (lim) become zero.
__device__ __forceinline__ void round8(const float* y, int lim, int bf16, uint32_t* w) {
#pragma unroll
    for (int i = 0; i < 8; i += 2) w[i >> 1] = pack2(i < lim ? y[i] : 0.f, i + 1 < lim ? y[i + 1] : 0.f, bf16);
}

// Epilogue of 8 consecutive columns gn..gn+7 (gn % 8 == 0) of row gm < M:
// returns the 8 output elements packed in four words (columns at or past N
// are zero).  `vec_rowmajor`: 16-byte accesses allowed for a row-major
// residual (N % 8 == 0 and 16-byte aligned); a packed residual is always
// read as whole 16-byte strip rows.  Each optional stage sits behind one
// uniform branch, so an unused stage costs nothing.
// res_pre: the 8 residual values already loaded (16-byte layouts only), or
// null to read them from e.residual.
__device__ __forceinline__ void epilogue8(const float* v, const Epilogue& e, int gm, int gn, int M, int N,
                                          bool vec_rowmajor, uint32_t* w, const float* bias_pre = nullptr,
                                          const uint4* res_pre = nullptr) {
    const int lim = min(8, N - gn);
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = v[i];
    epilogue_pre<8>(y, e, gm, bias_pre);
    if (e.residual) {
        const size_t base = c_offset(e, gm, gn, M, N);
        if (e.packed || vec_rowmajor) {
            const uint4 q = res_pre ? *res_pre : *reinterpret_cast<const uint4*>(e.residual + base);
            const uint32_t x[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] += elem_to_f32((uint16_t)(x[i >> 1] >> (16 * (i & 1))), e.bf16);
        } else {
            for (int i = 0; i < lim; ++i) y[i] += elem_to_f32(e.residual[base + i], e.bf16);
        }
    }
    round8(y, lim, e.bf16, w);
}

// Epilogue + the store into C of 8 columns of row gm < M (gn < N).  A packed
// C is always written as whole 16-byte strip rows.  `plain`: the caller's
// epilogue_is_plain(e), evaluated once per kernel.
__device__ __forceinline__ void epilogue_store8(uint16_t* C, const float* v, const Epilogue& e, int gm, int gn, int M,
                                                int N, bool vec_rowmajor, bool plain, const float* bias_pre = nullptr,
                                                const uint4* res_pre = nullptr) {
    const int lim = min(8, N - gn);
    uint32_t w[4];
    if (plain) round8(v, lim, e.bf16, w);
    else epilogue8(v, e, gm, gn, M, N, vec_rowmajor, w, bias_pre, res_pre);
    if (e.packed) {
        *reinterpret_cast<uint4*>(C + c_offset(e, gm, gn, M, N)) = make_uint4(w[0], w[1], w[2], w[3]);
    } else if (vec_rowmajor) {
        store_row16(C, e, gm, gn, N, make_uint4(w[0], w[1], w[2], w[3]));
    } else {
        store_row_elems(C, e, gm, gn, N, w, lim);
    }
}

// Round 8 fp32 values to fp16 and store them at `out` (16-byte store when
// allowed, else element by element up to `lim`).
__device__ __forceinline__ void store_h8(__half* out, const float* v, bool vec, int lim) {
    if (vec) {
        __align__(16) __half h[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) h[e] = __float2half_rn(v[e]);
        *reinterpret_cast<uint4*>(out) = *reinterpret_cast<const uint4*>(h);
    } else {
        for (int e = 0; e < lim && e < 8; ++e) out[e] = __float2half_rn(v[e]);
    }
}

}  // namespace spmm24
