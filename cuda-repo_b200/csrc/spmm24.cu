// spmm24.cu -- host launch API of the sm_100a 2:4 SpMM library.
//
// Replaces SpMM_N2M4_Launch / SpMM_N2M4_Kernel_API (SpeakOutLoudly/CUDA-Repo
// src/SpMM_API.cu:15-171): validates the call, picks a tile / stage / split
// configuration from the shape (the compile-time N switch of
// src/SpMM_API.cu:128-154 becomes a runtime picker), encodes the three TMA
// tensor maps and launches one kernel (a thread-block cluster along K when
// split-K is used; the reduction runs on chip, so the reference's second
// SplitK_Reduction launch is gone).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "spmm24/SpMM_API.h"
#include "spmm24_kernel.cuh"

namespace spmm24 {
namespace {

thread_local char g_last_error[256] = "";

cudaError_t invalid(const char* why) {
    std::snprintf(g_last_error, sizeof(g_last_error), "%s", why);
    return cudaErrorInvalidValue;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// All three operands are moved as raw 16-bit words (no conversion in TMA).
bool encode(CUtensorMap* m, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
            const cuuint32_t* box) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, (cuuint32_t)rank, const_cast<void*>(base), dims, strides_bytes,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

struct Plan {
    int tile_n;
    int stages;
    int split;
    int smem;
    int m_tiles, n_tiles;
    int stages_total;
};

template <int NT, int ST>
struct Variant {
    using C_ = Cfg<NT, ST>;
    static constexpr int kTileN = NT;
    static constexpr int kStages = ST;
};

// One configuration per N tile: the deepest ring that fits in 227 KB.
using V16 = Variant<16, 8>;
using V32 = Variant<32, 8>;
using V64 = Variant<64, 6>;
using V128 = Variant<128, 4>;
using V256 = Variant<256, 2>;

int stages_for(int tile_n) {
    switch (tile_n) {
        case 16: return V16::kStages;
        case 32: return V32::kStages;
        case 64: return V64::kStages;
        case 128: return V128::kStages;
        default: return V256::kStages;
    }
}
int smem_for(int tile_n) {
    switch (tile_n) {
        case 16: return V16::C_::SMEM_ALLOC;
        case 32: return V32::C_::SMEM_ALLOC;
        case 64: return V64::C_::SMEM_ALLOC;
        case 128: return V128::C_::SMEM_ALLOC;
        default: return V256::C_::SMEM_ALLOC;
    }
}

int env_int(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return (v && *v) ? std::atoi(v) : dflt;
}

constexpr int kNumSMs = 148;
constexpr int kMaxSplit = 8;

Plan make_plan(int M, int N, int K, int split_k) {
    Plan p{};
    int tn = N <= 16 ? 16 : N <= 32 ? 32 : N <= 64 ? 64 : 128;
    int forced = env_int("SPMM24_TILE_N", 0);  // tuning override (16/32/64/128/256)
    if (forced == 16 || forced == 32 || forced == 64 || forced == 128 || forced == 256) tn = forced;
    p.tile_n = tn;
    p.stages = stages_for(tn);
    p.smem = smem_for(tn);
    p.m_tiles = (M + kTileM - 1) / kTileM;
    p.n_tiles = (N + tn - 1) / tn;
    p.stages_total = (K / 64 + 1) / 2;
    int s;
    if (split_k > 0) {
        s = split_k;
    } else {
        long tiles = (long)p.m_tiles * p.n_tiles;
        s = (int)(kNumSMs / tiles);
        s = std::max(1, std::min(s, p.stages_total / 2));
    }
    s = std::max(1, std::min(std::min(s, kMaxSplit), p.stages_total));
    p.split = s;
    return p;
}

std::atomic<uint64_t> g_attr_done[5];  // per variant: bit per device (devices < 64)

template <class V>
cudaError_t launch_variant(const Plan& pl, cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tb,
                           const CUtensorMap& te, const KernelParams& kp, int variant_idx) {
    auto kern = spmm24_sm100_kernel<V::kTileN, V::kStages>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(g_attr_done[variant_idx].load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, V::C_::SMEM_ALLOC);
        if (e != cudaSuccess) return e;
        g_attr_done[variant_idx].fetch_or(bit, std::memory_order_acq_rel);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)pl.split, (unsigned)pl.n_tiles, (unsigned)pl.m_tiles);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = V::C_::SMEM_ALLOC;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)pl.split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pl.split > 1 ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, ta, tb, te, kp);
}

cudaError_t launch_impl(cudaStream_t stream, const void* A, const void* B, const uint16_t* E, void* C, int M, int N,
                        int K, int split_k) {
    g_last_error[0] = '\0';
    if (!A || !B || !E || !C) return invalid("null pointer");
    if (M <= 0 || N <= 0 || K <= 0) return invalid("M, N and K must be positive");
    if (M % 16) return invalid("M must be a multiple of 16");
    if (K % 64) return invalid("K must be a multiple of 64");
    if (split_k < 0) return invalid("split_k must be >= 0");
    if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)E) & 15u) return invalid("A, B and metadata must be 16-byte aligned");
    if ((uintptr_t)C & 1u) return invalid("C must be 2-byte aligned");
    if ((long)M / kTileM >= 65535) return invalid("M too large");

    const Plan pl = make_plan(M, N, K, split_k);

    // A: (128 halves of one 16x8 block, bands, 16-K blocks); box 8 bands x 8 blocks.
    CUtensorMap ta, tb, te;
    {
        cuuint64_t dims[3] = {128, (cuuint64_t)(M / 16), (cuuint64_t)(K / 16)};
        cuuint64_t str[2] = {(cuuint64_t)16 * K, 256};
        cuuint32_t box[3] = {128, 8, 8};
        if (!encode(&ta, 3, A, dims, str, box)) return invalid("TMA descriptor for A could not be encoded");
    }
    // B: (128 halves = 16 k-rows x 8 columns, 64-K groups, 16-K blocks of a group, strips);
    // box 2 groups x 4 blocks x tile_n/8 strips -> smem [strip][block][group].
    {
        cuuint64_t dims[4] = {128, (cuuint64_t)(K / 64), 4, (cuuint64_t)((N + 7) / 8)};
        cuuint64_t str[3] = {1024, 256, (cuuint64_t)16 * K};
        cuuint32_t box[4] = {128, 2, 4, (cuuint32_t)(pl.tile_n / 8)};
        if (!encode(&tb, 4, B, dims, str, box)) return invalid("TMA descriptor for B could not be encoded");
    }
    // E: (K words per band, bands); box two 64-K groups x 8 bands.
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)(M / 16)};
        cuuint64_t str[1] = {(cuuint64_t)2 * K};
        cuuint32_t box[2] = {128, 8};
        if (!encode(&te, 2, E, dims, str, box)) return invalid("TMA descriptor for metadata could not be encoded");
    }

    KernelParams kp;
    kp.C = static_cast<__half*>(C);
    kp.M = M;
    kp.N = N;
    kp.K = K;
    kp.groups = K / 64;
    kp.stages_total = pl.stages_total;
    kp.split = pl.split;

    switch (pl.tile_n) {
        case 16: return launch_variant<V16>(pl, stream, ta, tb, te, kp, 0);
        case 32: return launch_variant<V32>(pl, stream, ta, tb, te, kp, 1);
        case 64: return launch_variant<V64>(pl, stream, ta, tb, te, kp, 2);
        case 128: return launch_variant<V128>(pl, stream, ta, tb, te, kp, 3);
        default: return launch_variant<V256>(pl, stream, ta, tb, te, kp, 4);
    }
}

}  // namespace
}  // namespace spmm24

// ---------------------------------------------------------------- C ABI
extern "C" cudaError_t spmm24_launch(cudaStream_t stream, const void* compressed_a, const void* b_packed,
                                     const uint16_t* metadata, void* c, int M, int N, int K, void* split_reduction,
                                     int split_k) {
    (void)split_reduction;
    return spmm24::launch_impl(stream, compressed_a, b_packed, metadata, c, M, N, K, split_k);
}

extern "C" size_t spmm24_workspace_bytes(int, int, int, int) { return 0; }

extern "C" int spmm24_select_config(int M, int N, int K, int split_k, spmm24_config* out) {
    if (!out || M <= 0 || N <= 0 || K <= 0 || M % 16 || K % 64 || split_k < 0) return -1;
    const spmm24::Plan pl = spmm24::make_plan(M, N, K, split_k);
    out->tile_m = spmm24::kTileM;
    out->tile_n = pl.tile_n;
    out->stage_k = 128;
    out->stages = pl.stages;
    out->split_k = pl.split;
    out->grid_ctas = pl.split * pl.n_tiles * pl.m_tiles;
    out->smem_bytes = pl.smem;
    return 0;
}

extern "C" cudaError_t spmm24_device_status(int device, uint32_t* status_out) {
    if (!status_out) return cudaErrorInvalidValue;
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return e;
    if ((e = cudaSetDevice(device)) != cudaSuccess) return e;
    uint32_t v = 0, zero = 0;
    e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, spmm24::g_spmm24_status, sizeof(v));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(spmm24::g_spmm24_status, &zero, sizeof(zero));
    cudaSetDevice(prev);
    *status_out = v;
    return e;
}

extern "C" const char* spmm24_last_error(void) { return spmm24::g_last_error; }

extern "C" const char* spmm24_version(void) { return "spmm24 0.1.0 (sm_100a tcgen05.mma.sp)"; }

// ------------------------------------------------------- C++ drop-in
cudaError_t SpMM_N2M4_Launch(cudaStream_t stream, const half* Compressed_A, const half* B, const uint16_t* metadata,
                             half* C, const int M_Global, const int N_Global, const int K_Global,
                             half* Split_Reduction, const int Split_K) {
    return spmm24::launch_impl(stream, Compressed_A, B, metadata, C, M_Global, N_Global, K_Global, Split_K);
}
