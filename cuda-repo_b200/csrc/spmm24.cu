// spmm24.cu -- host launch API of the sm_100a 2:4 SpMM library.
//
// Replaces SpMM_N2M4_Launch / SpMM_N2M4_Kernel_API (SpeakOutLoudly/CUDA-Repo
// src/SpMM_API.cu:15-171): validates the call, picks a kernel and a tile /
// stage / split configuration from the shape (the compile-time N switch of
// src/SpMM_API.cu:128-154 becomes a runtime picker), encodes the three TMA
// tensor maps and launches one kernel.  The reference's second launch
// (SplitK_Reduction) is gone: split-K partials are reduced on chip, inside a
// thread-block cluster (the allocation-free entry point's stream-K kernel
// reduces through its fixed scratch array instead).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "spmm24/SpMM_API.h"
#include "spmm24_host.h"
#include "spmm24_kernel.cuh"
#include "spmm24_grouped.cuh"

namespace spmm24 {

thread_local char g_last_error[256] = "";

cudaError_t record_invalid(const char* why) {
    std::snprintf(g_last_error, sizeof(g_last_error), "%s", why);
    return cudaErrorInvalidValue;
}
void clear_last_error() { g_last_error[0] = '\0'; }

namespace {

cudaError_t invalid(const char* why) { return record_invalid(why); }

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

// A tensor map is a pure function of its inputs (address, sizes, strides,
// box, type, swizzle), so encoded maps are kept in a small per-thread cache:
// a serving loop that calls the same layers again skips the driver's
// encoder.  Direct-mapped, 64 entries, no locking (each host thread has its
// own); a freed and re-allocated buffer at the same address with the same
// shape encodes to the same map, so an entry never goes stale.
struct MapKey {
    const void* base;
    cuuint64_t dims[5];
    cuuint64_t strides[4];
    cuuint32_t box[5];
    int rank, type, swizzle;
};
struct MapEntry {
    MapKey key;
    CUtensorMap map;
    bool valid;
};
constexpr int kMapCacheSlots = 64;
thread_local MapEntry t_map_cache[kMapCacheSlots];

// Operands are moved as raw 16-bit words (the fp8 B as bytes): no conversion
// in TMA.
bool encode(CUtensorMap* m, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
            const cuuint32_t* box, CUtensorMapDataType type = CU_TENSOR_MAP_DATA_TYPE_UINT16,
            CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
    if (rank < 1 || rank > 5) return false;
    MapKey k;
    std::memset(&k, 0, sizeof(k));  // padding included: keys compare bytewise
    k.base = base;
    for (int i = 0; i < rank; ++i) {
        k.dims[i] = dims[i];
        k.box[i] = box[i];
        if (i + 1 < rank) k.strides[i] = strides_bytes[i];
    }
    k.rank = rank;
    k.type = (int)type;
    k.swizzle = (int)swizzle;
    uint64_t h = 1469598103934665603ull;  // FNV-1a over the key bytes
    const unsigned char* kb = reinterpret_cast<const unsigned char*>(&k);
    for (size_t i = 0; i < sizeof(k); ++i) h = (h ^ kb[i]) * 1099511628211ull;
    MapEntry& slot = t_map_cache[(h ^ (h >> 29)) % kMapCacheSlots];
    if (slot.valid && std::memcmp(&slot.key, &k, sizeof(k)) == 0) {
        *m = slot.map;
        return true;
    }
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(m, type, (cuuint32_t)rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    slot.key = k;
    slot.map = *m;
    slot.valid = true;
    return true;
}

// Picker overrides set by spmm24_set_tuning (tests and tuning sweeps); the
// library reads no environment variables.
struct Tuning {
    std::atomic<int> pair{-1}, pair2{-1}, pair_split{0}, tile_n{0}, deep_ring{0}, group_split{0};
};
Tuning g_tune;

constexpr int kMaxDevices = 64;
constexpr int kMaxSplit = 8;

int sm_count(int dev) {
    static std::atomic<int> cache[kMaxDevices];
    if (dev < 0 || dev >= kMaxDevices) return 148;
    int v = cache[dev].load(std::memory_order_relaxed);
    if (v > 0) return v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev].store(v, std::memory_order_relaxed);
    return v;
}

// ----------------------------------------------------------- configurations
enum class Path { kCluster, kStreamK, kPair };

template <int NT, int ST>
struct ClusterVariant {
    using C_ = ClusterCfg<NT, ST>;
    static constexpr int kTileN = NT;
    static constexpr int kStages = ST;
};
template <int NT, int ST>
struct StreamKVariant {
    using C_ = StreamKCfg<NT, ST>;
    static constexpr int kTileN = NT;
    static constexpr int kStages = ST;
};

// One configuration per N tile: the deepest ring that fits in 227 KB.
using CV16 = ClusterVariant<16, 8>;
using CV32 = ClusterVariant<32, 7>;
using CV64 = ClusterVariant<64, 6>;
using CV128 = ClusterVariant<128, 4>;
using CV256 = ClusterVariant<256, 2>;
// Pair tiles: 256 x 256 with a 4-stage ring (one CTA per SM).
constexpr int kPairStages = 4;
using PairC = PairCfg<kPairStages>;
// Narrow pair tiles: 256 x 128 with a 6-stage ring of 34 KB stages, for
// shapes with less than half a wave of 256 x 256 tiles (fp16 / bf16 only).
constexpr int kPairNarrowStages = 6;
using PairNC = PairCfg<kPairNarrowStages, false, 64>;
// Two M halves per pair (512 x 240 tiles, 3-stage ring of 66 KB stages).
constexpr int kPair2Stages = 3;
using Pair2C = Pair2Cfg<kPair2Stages>;
using Pair2C8 = Pair2Cfg<kPair2Stages, true>;
using PairC8 = PairCfg<kPairStages, true>;
// Stream-K variants: the scratch-array kernel of spmm24_launch_noalloc.
using SV16 = StreamKVariant<16, 8>;
using SV32 = StreamKVariant<32, 8>;
// Shallow rings (about 92 KB of shared memory): two CTAs fit on one SM, so
// consecutive launches overlap on the same SM under programmatic launch.
using CV16s = ClusterVariant<16, 4>;
using CV32s = ClusterVariant<32, 3>;

struct Plan {
    Path path;
    bool pair2;        // pair path with two M halves per pair (512 x 240 tiles)
    bool narrow;       // pair path with 256 x 128 tiles
    bool shallow;      // 4-stage ring, two CTAs per SM (narrow N only)
    int tile_n;
    int stages;
    int split;  // cluster path: CTAs per cluster
    int grid;   // stream-K path: persistent CTAs
    int smem;
    int m_tiles, n_tiles;
    int stages_total;  // 128-K stages per tile
};

int cluster_stages(int tn) {
    switch (tn) {
        case 16: return CV16::kStages;
        case 32: return CV32::kStages;
        case 64: return CV64::kStages;
        case 128: return CV128::kStages;
        default: return CV256::kStages;
    }
}
int cluster_smem(int tn) {
    switch (tn) {
        case 16: return CV16::C_::SMEM_ALLOC;
        case 32: return CV32::C_::SMEM_ALLOC;
        case 64: return CV64::C_::SMEM_ALLOC;
        case 128: return CV128::C_::SMEM_ALLOC;
        default: return CV256::C_::SMEM_ALLOC;
    }
}

// Two M halves per pair share each B tile: 512 x tile_n tiles, 1.6x the
// time of a 256 x 256 tile for 1.875x its area (measured, 4096^3, tile_n
// 240).  Switches a pair plan with one pair per tile to that kernel when
// its waves of pairs cost less: e.g. 4096 x 4096 x 4096 (2 waves against
// 4: -19%), 11008 x 512 x 4096 (1 against 2), not 4096 x 512 x 4096 (1
// wave either way).
void maybe_pair2(Plan& p, int M, int N, int sms, int tile_n, int stages, int smem) {
    const int env = g_tune.pair2.load(std::memory_order_relaxed);  // override: 0 = never, 1 = whenever legal
    if (env == 0) return;
    const long long slots = std::max(1, sms / 2);
    const long long m2 = (M + 4 * kTileM - 1) / (4 * kTileM), n2 = (N + tile_n - 1) / tile_n;
    const long long base_waves = ((long long)p.m_tiles * p.n_tiles + slots - 1) / slots;
    const long long p2_waves = (m2 * n2 + slots - 1) / slots;
    if (env != 1 && 16 * p2_waves >= 10 * base_waves) return;
    p.pair2 = true;
    p.tile_n = tile_n;
    p.stages = stages;
    p.smem = smem;
    p.m_tiles = (int)m2;
    p.n_tiles = (int)n2;
    p.grid = 2 * p.m_tiles * p.n_tiles;
}

// allow_pair: the CTA-pair path may be chosen.  max_split: the largest
// automatic K split.  pair2_ok: the two-M-half pair kernel may be chosen
// (no residual).
Plan make_plan(int M, int N, int K, int split_k, int sms, bool allow_pair = true, int max_split = kMaxSplit,
               bool pair2_ok = true, bool narrow_ok = true) {
    Plan p{};
    int tn = N <= 16 ? 16 : N <= 32 ? 32 : N <= 64 ? 64 : 128;
    const int forced = g_tune.tile_n.load(std::memory_order_relaxed);  // override (16/32/64/128/256)
    if (forced == 16 || forced == 32 || forced == 64 || forced == 128 || forced == 256) tn = forced;
    p.tile_n = tn;
    p.m_tiles = (M + kTileM - 1) / kTileM;
    p.n_tiles = (N + tn - 1) / tn;
    p.stages_total = (K / 64 + 1) / 2;
    const long long tiles = (long long)p.m_tiles * p.n_tiles;

    // Narrow N (decode) streams weights: a 4-stage ring (about 92 KB) puts two
    // CTAs on each SM, so consecutive launches overlap on the same SM under
    // programmatic launch, and the K split fills both slots of every SM.
    const bool deep = g_tune.deep_ring.load(std::memory_order_relaxed) == 1;  // override: the deepest ring
    p.shallow = tn <= 32 && !deep;

    // Wide N with K % 128 == 0: a CTA pair per 256 x 256 tile (cta_group::2),
    // so each SM feeds the tensor core half of B.
    const int pair_env = g_tune.pair.load(std::memory_order_relaxed);  // override: 0 = never, 1 = whenever legal
    const bool pair_ok = allow_pair && (K % 128 == 0) && (split_k <= 1);
    if (pair_ok && (pair_env == 1 || (pair_env != 0 && N > 128))) {
        p.path = Path::kPair;
        p.shallow = false;
        p.tile_n = PairC::TILE_N;
        p.stages = kPairStages;
        p.smem = PairC::SMEM_ALLOC;
        p.m_tiles = (M + 2 * kTileM - 1) / (2 * kTileM);
        p.n_tiles = (N + p.tile_n - 1) / p.tile_n;
        // Few tiles and long K (at most half a wave of pairs, at least 48
        // stages): two pairs per tile, each taking half of K (a cluster of 4
        // with an on-chip reduction).  Measured: 4096 x 512 x 11008 -10%
        // time; shorter K or more tiles lose (clusters of 4 leave SMs of
        // every GPC idle, and the 128 KB exchange costs a few us per tile).
        const long long ptiles = (long long)p.m_tiles * p.n_tiles;
        const int pair_split_env = g_tune.pair_split.load(std::memory_order_relaxed);  // override: 1 or 2
        int ps = 1;
        if (pair_split_env == 1 || pair_split_env == 2)
            ps = pair_split_env;
        else if (split_k == 0 && 2 * ptiles <= (long long)(sms / 2) && p.stages_total >= 48)
            ps = 2;
        if (p.stages_total < 2) ps = 1;
        p.split = ps;
        p.grid = 2 * ps * (int)ptiles;
        // Less than half a wave of 256 x 256 tiles and no K split (N > 256;
        // narrower N takes the cluster tiles below): 256 x 128 tiles on
        // twice as many pairs, when they still fit in one wave.  Measured
        // back to back: 4096 x 512 x 4096 17.35 -> 16.74 us, 2048 x 512 x
        // 2048 10.81 -> 9.98, 1024^3 7.81 -> 7.03 (isolated with L2 flushed:
        // equal or faster).  Tuning: tile_n 128 forces it, 256 keeps the wide
        // tile, a forced pair2 takes precedence.
        const bool pair2_forced = g_tune.pair2.load(std::memory_order_relaxed) == 1;
        if (narrow_ok && ps == 1 && forced != 256 && !pair2_forced &&
            (forced == 128 || (N > 256 && 2 * ptiles <= sms / 2))) {
            const long long ntiles = (long long)p.m_tiles * ((N + 127) / 128);
            if (forced == 128 || 2 * ntiles <= sms) {
                p.narrow = true;
                p.tile_n = PairNC::TILE_N;
                p.stages = kPairNarrowStages;
                p.smem = PairNC::SMEM_ALLOC;
                p.n_tiles = (N + p.tile_n - 1) / p.tile_n;
                p.grid = 2 * p.m_tiles * p.n_tiles;
                return p;
            }
        }
        // One pair tile across N (N <= 256) and pairs for less than three
        // quarters of the SMs: 128-wide cluster tiles with a K split fill more
        // of the GPU.  Measured (chains of one shape): 1024 x 256 x 8192
        // 23.5 -> 12.9 us, 3584 x 256 x 8192 24.9 -> 19.6 us, 1024 x 256 x
        // 28672 51.9 -> 27.9 us (the per-GPU shards of M-sharded 70B layers);
        // 8192 x 256 x 8192 stays on the pair (29.8 against 32.2 us).
        const bool few = N <= 256 && split_k == 0 && (long long)p.grid < (3LL * sms) / 4;
        if (!(few && pair_env != 1 && g_tune.pair2.load(std::memory_order_relaxed) != 1)) {
            if (pair2_ok && ps == 1 && split_k <= 1)
                maybe_pair2(p, M, N, sms, Pair2C::TILE_N, kPair2Stages, Pair2C::SMEM_ALLOC);
            return p;
        }
        p = Plan{};
        p.tile_n = tn;
        p.m_tiles = (M + kTileM - 1) / kTileM;
        p.n_tiles = (N + tn - 1) / tn;
        p.stages_total = (K / 64 + 1) / 2;
        p.shallow = tn <= 32 && !deep;
        max_split = std::min(max_split, 4);  // measured: 4 beats 8 for 128 x 128 tiles (cl4 12.9 us, cl8 19.5 us)
    }
    p.path = Path::kCluster;
    if (p.shallow) {
        p.stages = tn == 16 ? CV16s::kStages : CV32s::kStages;
        p.smem = tn == 16 ? CV16s::C_::SMEM_ALLOC : CV32s::C_::SMEM_ALLOC;
    } else {
        p.stages = cluster_stages(tn);
        p.smem = cluster_smem(tn);
    }
    int s;
    if (split_k > 0) {
        s = split_k;
    } else {
        // As many K slices as fill the resident CTA slots (two per SM with the
        // shallow ring), keeping at least two stages per slice -- five for
        // long K: measured on the 4096 x 4096 decode shapes, six slices of 5-6
        // stages beat eight of 4 (fewer CTAs leave SM slots to the next
        // launch's early CTAs).
        const long long slots = (long long)sms * (p.shallow ? 2 : 1);
        const int min_stages = p.stages_total >= 24 ? 5 : 2;
        s = (int)std::max<long long>(1, slots / tiles);
        s = std::max(1, std::min(std::min(s, max_split), p.stages_total / min_stages));
    }
    p.split = std::max(1, std::min(std::min(s, kMaxSplit), p.stages_total));
    p.grid = p.split * p.n_tiles * p.m_tiles;
    return p;
}

std::atomic<uint64_t> g_attr_done[96];  // per kernel variant: one bit per device

// The plain SpMM: fp16, row-major C, no epilogue work.
bool epilogue_plain_fp16(const Epilogue& e) {
    return e.bias == nullptr && e.residual == nullptr && e.act == kActNone && e.alpha == 1.f && !e.packed && !e.bf16 &&
           e.gather_n == 0;
}
#ifdef SPMM24_TRACE
std::atomic<long long> g_trace_next{0};  // next free CTA record in the trace buffer
#endif

template <class Kern>
cudaError_t prepare(Kern kern, int smem, int dev, int idx) {
    const uint64_t bit = 1ull << (dev & 63);
    if (g_attr_done[idx].load(std::memory_order_acquire) & bit) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    g_attr_done[idx].fetch_or(bit, std::memory_order_acq_rel);
    return cudaSuccess;
}

template <class Kern, class Params>
cudaError_t launch_kernel(Kern kern, dim3 grid, int smem, cudaStream_t stream, unsigned cluster_x, bool pdl,
                          const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& te, const Params& kp,
                          int threads = kThreads) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (cluster_x > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster_x;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
#ifdef SPMM24_TRACE
    Params kt = kp;
    kt.trace_base = g_trace_next.fetch_add((long long)grid.x * grid.y * grid.z);
    return cudaLaunchKernelEx(&cfg, kern, ta, tb, te, kt);
#else
    return cudaLaunchKernelEx(&cfg, kern, ta, tb, te, kp);
#endif
}

// Attribute-cache slots: variant index, plus kEpiSlot for the general-epilogue
// instantiation of the same variant.
constexpr int kEpiSlot = 32;

template <class V>
cudaError_t launch_cluster(const Plan& pl, cudaStream_t stream, int dev, bool pdl, const CUtensorMap& ta,
                           const CUtensorMap& tb, const CUtensorMap& te, const ClusterParams& kp, int idx) {
    const bool general = !epilogue_plain_fp16(kp.epi);
    auto kern = general ? spmm24_cluster_kernel<V::kTileN, V::kStages, true>
                        : spmm24_cluster_kernel<V::kTileN, V::kStages, false>;
    cudaError_t e = prepare(kern, V::C_::SMEM_ALLOC, dev, idx + (general ? kEpiSlot : 0));
    if (e != cudaSuccess) return e;
    return launch_kernel(kern, dim3((unsigned)pl.split, (unsigned)pl.n_tiles, (unsigned)pl.m_tiles),
                         V::C_::SMEM_ALLOC, stream, (unsigned)pl.split, pdl, ta, tb, te, kp);
}

// The fp8 instantiations: the general epilogue (attribute slots kFp8Slot +
// idx), and alpha-only fp16 row-major output (kFp8PlainSlot + idx).
constexpr int kFp8Slot = 48;
constexpr int kFp8PlainSlot = 64;

template <class V>
cudaError_t launch_cluster_fp8(const Plan& pl, cudaStream_t stream, int dev, bool pdl, const CUtensorMap& ta,
                               const CUtensorMap& tb, const CUtensorMap& te, const ClusterParams& kp, int idx) {
    using C8 = ClusterCfg<V::kTileN, V::kStages, true>;
    const Epilogue& ep = kp.epi;
    const bool general = ep.bias || ep.residual || ep.act != kActNone || ep.packed || ep.bf16 || ep.gather_n;
    auto kern = general ? spmm24_cluster_kernel<V::kTileN, V::kStages, true, true>
                        : spmm24_cluster_kernel<V::kTileN, V::kStages, false, true>;
    cudaError_t e = prepare(kern, C8::SMEM_ALLOC, dev, (general ? kFp8Slot : kFp8PlainSlot) + idx);
    if (e != cudaSuccess) return e;
    return launch_kernel(kern, dim3((unsigned)pl.split, (unsigned)pl.n_tiles, (unsigned)pl.m_tiles), C8::SMEM_ALLOC,
                         stream, (unsigned)pl.split, pdl, ta, tb, te, kp);
}

template <class V>
cudaError_t launch_streamk(const Plan& pl, cudaStream_t stream, int dev, bool pdl, const CUtensorMap& ta,
                           const CUtensorMap& tb, const CUtensorMap& te, const StreamKParams& kp, int idx) {
    auto kern = spmm24_streamk_kernel<V::kTileN, V::kStages>;
    cudaError_t e = prepare(kern, V::C_::SMEM_ALLOC, dev, idx);
    if (e != cudaSuccess) return e;
    return launch_kernel(kern, dim3((unsigned)pl.grid, 1, 1), V::C_::SMEM_ALLOC, stream, 1u, pdl, ta, tb, te, kp);
}

template <bool KSPLIT>
cudaError_t launch_pair_v(const Plan& pl, cudaStream_t stream, int dev, bool pdl, const CUtensorMap& ta,
                          const CUtensorMap& tb, const CUtensorMap& te, const PairParams& kp, int idx) {
    const bool general = !epilogue_plain_fp16(kp.epi);
    auto kern = general ? spmm24_pair_kernel<kPairStages, true, KSPLIT> : spmm24_pair_kernel<kPairStages, false, KSPLIT>;
    cudaError_t e = prepare(kern, PairC::SMEM_ALLOC, dev, idx + (general ? kEpiSlot : 0));
    if (e != cudaSuccess) return e;
    const unsigned cl = KSPLIT ? 4u : 2u;
    return launch_kernel(kern, dim3(cl, (unsigned)pl.n_tiles, (unsigned)pl.m_tiles), PairC::SMEM_ALLOC, stream, cl,
                         pdl, ta, tb, te, kp, kPairThreads);
}

template <bool KSPLIT>
cudaError_t launch_pair_fp8(const Plan& pl, cudaStream_t stream, int dev, bool pdl, const CUtensorMap& ta,
                            const CUtensorMap& tb, const CUtensorMap& te, const PairParams& kp) {
    auto kern = spmm24_pair_kernel<kPairStages, true, KSPLIT, true>;
    cudaError_t e = prepare(kern, PairC8::SMEM_ALLOC, dev, kFp8Slot + (KSPLIT ? 12 : 11));
    if (e != cudaSuccess) return e;
    const unsigned cl = KSPLIT ? 4u : 2u;
    return launch_kernel(kern, dim3(cl, (unsigned)pl.n_tiles, (unsigned)pl.m_tiles), PairC8::SMEM_ALLOC, stream, cl,
                         pdl, ta, tb, te, kp, kPairThreads);
}

cudaError_t launch_pair2(const Plan& pl, cudaStream_t stream, int dev, bool pdl, const CUtensorMap& ta,
                         const CUtensorMap& tb, const CUtensorMap& te, const PairParams& kp) {
    const bool general = !epilogue_plain_fp16(kp.epi);
    auto kern = general ? spmm24_pair2_kernel<kPair2Stages, true> : spmm24_pair2_kernel<kPair2Stages, false>;
    cudaError_t e = prepare(kern, Pair2C::SMEM_ALLOC, dev, general ? 14 : 13);
    if (e != cudaSuccess) return e;
    return launch_kernel(kern, dim3(2u, (unsigned)pl.n_tiles, (unsigned)pl.m_tiles), Pair2C::SMEM_ALLOC, stream, 2u,
                         pdl, ta, tb, te, kp, kPairThreads);
}

cudaError_t launch_pair_narrow(const Plan& pl, cudaStream_t stream, int dev, bool pdl, const CUtensorMap& ta,
                               const CUtensorMap& tb, const CUtensorMap& te, const PairParams& kp) {
    const bool general = !epilogue_plain_fp16(kp.epi);
    auto kern = general ? spmm24_pair_kernel<kPairNarrowStages, true, false, false, 64>
                        : spmm24_pair_kernel<kPairNarrowStages, false, false, false, 64>;
    cudaError_t e = prepare(kern, PairNC::SMEM_ALLOC, dev, 15 + (general ? kEpiSlot : 0));
    if (e != cudaSuccess) return e;
    return launch_kernel(kern, dim3(2u, (unsigned)pl.n_tiles, (unsigned)pl.m_tiles), PairNC::SMEM_ALLOC, stream, 2u,
                         pdl, ta, tb, te, kp, kPairThreads);
}

cudaError_t launch_pair(const Plan& pl, cudaStream_t stream, int dev, bool pdl, const CUtensorMap& ta,
                        const CUtensorMap& tb, const CUtensorMap& te, const PairParams& kp) {
    if (pl.narrow) return launch_pair_narrow(pl, stream, dev, pdl, ta, tb, te, kp);
    return pl.split == 2 ? launch_pair_v<true>(pl, stream, dev, pdl, ta, tb, te, kp, 12)
                         : launch_pair_v<false>(pl, stream, dev, pdl, ta, tb, te, kp, 11);
}

// True when an epilogue only rounds (the plain instantiations serve it).
bool epilogue_is_plain_host(const Epilogue& e) {
    return e.bias == nullptr && e.residual == nullptr && e.act == kActNone && e.alpha == 1.f && !e.packed;
}

// Validates a caller's epilogue and turns it into the kernels' form
// (SPMM24_BF16 in flags: 16-bit outputs are bf16).
cudaError_t make_epilogue(const spmm24_epilogue* user_epi, unsigned flags, const void* C, Epilogue* out) {
    Epilogue epi{nullptr, nullptr, 1.f, kActNone, 0, (flags & SPMM24_BF16) ? 1 : 0};
    if (user_epi) {
        if (user_epi->activation < SPMM24_ACT_NONE || user_epi->activation > SPMM24_ACT_GELU)
            return invalid("unknown epilogue activation");
        if (user_epi->out_layout != SPMM24_OUT_ROW_MAJOR && user_epi->out_layout != SPMM24_OUT_PACKED_B)
            return invalid("unknown output layout");
        if (!std::isfinite(user_epi->alpha)) return invalid("epilogue alpha must be finite");
        epi.bias = static_cast<const uint16_t*>(user_epi->bias);
        epi.residual = static_cast<const uint16_t*>(user_epi->residual);
        epi.alpha = user_epi->alpha;
        epi.act = user_epi->activation;
        epi.packed = user_epi->out_layout == SPMM24_OUT_PACKED_B ? 1 : 0;
        if ((uintptr_t)epi.bias & 1u) return invalid("bias must be 2-byte aligned");
        if ((uintptr_t)epi.residual & 1u) return invalid("residual must be 2-byte aligned");
        if (epi.packed && (((uintptr_t)C | (uintptr_t)epi.residual) & 15u))
            return invalid("a packed C (and its residual) must be 16-byte aligned");
    }
    *out = epi;
    return cudaSuccess;
}

cudaError_t launch_impl(cudaStream_t stream, const void* A, const void* B, const uint16_t* E, void* C, int M, int N,
                        int K, int split_k, unsigned flags, const spmm24_epilogue* user_epi = nullptr,
                        const spmm24_gather* gather = nullptr) {
    g_last_error[0] = '\0';
    if (!A || !B || !E || !C) return invalid("null pointer");
    if (M <= 0 || N <= 0 || K <= 0) return invalid("M, N and K must be positive");
    if (M % 16) return invalid("M must be a multiple of 16");
    if (K % 64) return invalid("K must be a multiple of 64");
    if (split_k < 0) return invalid("split_k must be >= 0");
    if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)E) & 15u) return invalid("A, B and metadata must be 16-byte aligned");
    if ((uintptr_t)C & 1u) return invalid("C must be 2-byte aligned");
    if ((long)M / kTileM >= 65535) return invalid("M too large");
    if (flags & ~(unsigned)(SPMM24_STATIC_WEIGHTS | SPMM24_NO_PDL | SPMM24_BF16)) return invalid("unknown flag");
    Epilogue epi;
    cudaError_t e = make_epilogue(user_epi, flags, C, &epi);
    if (e != cudaSuccess) return e;
    if (gather) {
        if (gather->n_ranks < 1 || gather->n_ranks > SPMM24_MAX_GATHER_RANKS)
            return invalid("gather: n_ranks must be 1..8");
        if (gather->row_offset < 0 || gather->m_full < M || gather->row_offset > gather->m_full - M)
            return invalid("gather: the shard's rows must lie inside the full C");
        if (epi.packed) return invalid("gather: the full C is row-major");
        for (int r = 0; r < gather->n_ranks; ++r) {
            if (!gather->c_full[r]) return invalid("gather: null full-C pointer");
            if ((uintptr_t)gather->c_full[r] & 15u) return invalid("gather: full-C buffers must be 16-byte aligned");
            epi.gather_dst[r] = static_cast<uint16_t*>(gather->c_full[r]);
        }
        epi.gather_n = gather->n_ranks;
        epi.gather_row0 = gather->row_offset;
        if (gather->c_multicast) {
            if (N % 8) return invalid("gather: a multicast C needs N % 8 == 0");
            if ((uintptr_t)gather->c_multicast & 15u) return invalid("gather: the multicast C must be 16-byte aligned");
            epi.gather_mc = static_cast<uint16_t*>(gather->c_multicast);
        }
    }
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const bool pair2_ok = !epi.residual;
    Plan pl = make_plan(M, N, K, split_k, sm_count(dev), true, kMaxSplit, pair2_ok);

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
        const int cta_n = pl.path != Path::kPair ? pl.tile_n
                          : pl.pair2             ? Pair2C::HALF_N
                          : pl.narrow            ? PairNC::HALF_N
                                                 : PairC::HALF_N;  // columns one CTA loads
        cuuint32_t box[4] = {128, 2, 4, (cuuint32_t)(cta_n / 8)};
        if (!encode(&tb, 4, B, dims, str, box)) return invalid("TMA descriptor for B could not be encoded");
    }
    // E: (K words per band, bands); box two 64-K groups x 8 bands.
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)(M / 16)};
        cuuint64_t str[1] = {(cuuint64_t)2 * K};
        cuuint32_t box[2] = {128, 8};
        if (!encode(&te, 2, E, dims, str, box)) return invalid("TMA descriptor for metadata could not be encoded");
    }

    const bool pdl = !(flags & SPMM24_NO_PDL);
    const int wstatic = (flags & SPMM24_STATIC_WEIGHTS) ? 1 : 0;
    if (pl.path == Path::kPair) {
        if (epi.residual && pl.split != 1) {  // the partner partial would overlap the residual's staging
            pl.split = 1;
            pl.grid = 2 * pl.m_tiles * pl.n_tiles;
        }
        PairParams kp;
        kp.C = static_cast<uint16_t*>(C);
        kp.epi = epi;
        kp.M = M;
        kp.N = N;
        kp.K = K;
        kp.stages_total = K / 128;
        kp.weights_static = wstatic;
        kp.split = pl.split;
        kp.mma_fmt = 0;
        if (pl.pair2) return launch_pair2(pl, stream, dev, pdl, ta, tb, te, kp);
        return launch_pair(pl, stream, dev, pdl, ta, tb, te, kp);
    }
    ClusterParams kp;
    kp.C = static_cast<uint16_t*>(C);
    kp.epi = epi;
    kp.M = M;
    kp.N = N;
    kp.K = K;
    kp.groups = K / 64;
    kp.stages_total = pl.stages_total;
    kp.split = pl.split;
    kp.weights_static = wstatic;
    kp.mma_fmt = 0;
    if (pl.shallow) {
        if (pl.tile_n == 16) return launch_cluster<CV16s>(pl, stream, dev, pdl, ta, tb, te, kp, 9);
        return launch_cluster<CV32s>(pl, stream, dev, pdl, ta, tb, te, kp, 10);
    }
    switch (pl.tile_n) {
        case 16: return launch_cluster<CV16>(pl, stream, dev, pdl, ta, tb, te, kp, 0);
        case 32: return launch_cluster<CV32>(pl, stream, dev, pdl, ta, tb, te, kp, 1);
        case 64: return launch_cluster<CV64>(pl, stream, dev, pdl, ta, tb, te, kp, 2);
        case 128: return launch_cluster<CV128>(pl, stream, dev, pdl, ta, tb, te, kp, 3);
        default: return launch_cluster<CV256>(pl, stream, dev, pdl, ta, tb, te, kp, 4);
    }
}

// ------------------------------------------------------------------- fp8
// The fp8 SpMM runs the cluster kernel with a stage of 256 logical K; its A
// values occupy the bytes of a 16-bit A with K/2, so the plan and the A
// descriptor are those of K/2.
//
// Automatic splits stop at 5: measured on the decode chain (M = 4096, K =
// 4096 and 11008, N <= 32), five K slices beat eight by 4-8% per call (a
// cheaper cluster reduction and more SM slots left to the next launch's
// early CTAs), and 11008-row layers pick 3 either way.  Wide N takes the CTA
// pair as for 16-bit operands (its stage is 256 K: K % 256), and the
// two-M-half pair (512 x 240) when its waves cost less and the epilogue has
// no residual (pair2_ok).
template <class V>
int fp8_smem() {
    return ClusterCfg<V::kTileN, V::kStages, true>::SMEM_ALLOC;
}

Plan plan_fp8(int M, int N, int K, int split_k, int sms, bool pair2_ok) {
    const int Kh = K / 2;
    Plan pl = make_plan(M, N, Kh, split_k, sms, Kh % 128 == 0, 5, false, false);
    if (pl.path == Path::kPair) {
        pl.smem = PairC8::SMEM_ALLOC;
        if (pl.split == 1 && split_k <= 1 && pair2_ok)
            maybe_pair2(pl, M, N, sms, Pair2C8::TILE_N, kPair2Stages, Pair2C8::SMEM_ALLOC);
    } else if (pl.shallow) {
        pl.smem = pl.tile_n == 16 ? fp8_smem<CV16s>() : fp8_smem<CV32s>();
    } else {
        switch (pl.tile_n) {
            case 16: pl.smem = fp8_smem<CV16>(); break;
            case 32: pl.smem = fp8_smem<CV32>(); break;
            case 64: pl.smem = fp8_smem<CV64>(); break;
            case 128: pl.smem = fp8_smem<CV128>(); break;
            default: pl.smem = fp8_smem<CV256>(); break;
        }
    }
    return pl;
}
cudaError_t launch_fp8_impl(cudaStream_t stream, const void* A, const void* B, const void* E, void* C, int M, int N,
                            int K, int split_k, unsigned flags, const spmm24_epilogue* user_epi) {
    g_last_error[0] = '\0';
    if (!A || !B || !E || !C) return invalid("null pointer");
    if (M <= 0 || N <= 0 || K <= 0) return invalid("M, N and K must be positive");
    if (M % 16) return invalid("M must be a multiple of 16");
    if (K % 128) return invalid("fp8: K must be a multiple of 128");
    if (split_k < 0) return invalid("split_k must be >= 0");
    if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)E) & 15u) return invalid("A, B and metadata must be 16-byte aligned");
    if ((uintptr_t)C & 1u) return invalid("C must be 2-byte aligned");
    if ((long)M / kTileM >= 65535) return invalid("M too large");
    if (flags & ~(unsigned)(SPMM24_STATIC_WEIGHTS | SPMM24_NO_PDL | SPMM24_BF16 | SPMM24_FP8_A_E5M2 |
                            SPMM24_FP8_B_E5M2))
        return invalid("unknown flag");
    Epilogue epi;
    cudaError_t e = make_epilogue(user_epi, flags, C, &epi);
    if (e != cudaSuccess) return e;
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int Kh = K / 2;  // the 16-bit-equivalent K of the A bytes
    Plan pl = plan_fp8(M, N, K, split_k, sm_count(dev), !epi.residual);
    const bool pair = pl.path == Path::kPair;

    CUtensorMap ta, tb, te;
    {
        cuuint64_t dims[3] = {128, (cuuint64_t)(M / 16), (cuuint64_t)(Kh / 16)};
        cuuint64_t str[2] = {(cuuint64_t)16 * Kh, 256};
        cuuint32_t box[3] = {128, 8, 8};
        if (!encode(&ta, 3, A, dims, str, box)) return invalid("TMA descriptor for A could not be encoded");
    }
    // B (N x K bytes): box 128 bytes of K x tile_n rows with the 128-byte
    // swizzle (two boxes per 256-K stage).
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
        cuuint64_t str[1] = {(cuuint64_t)K};
        cuuint32_t box[2] = {128, (cuuint32_t)(!pair ? pl.tile_n : pl.pair2 ? Pair2C8::HALF_N : PairC8::HALF_N)};
        if (!encode(&tb, 2, B, dims, str, box, CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B))
            return invalid("TMA descriptor for B could not be encoded");
    }
    // E: (256 bytes of one band and 128-K group, bands, groups); box 8 bands
    // x 2 groups -> smem [group][band][256 B].
    {
        cuuint64_t dims[3] = {128, (cuuint64_t)(M / 16), (cuuint64_t)(K / 128)};
        cuuint64_t str[2] = {(cuuint64_t)(K / 128) * 256, 256};
        cuuint32_t box[3] = {128, 8, 2};
        if (!encode(&te, 3, E, dims, str, box)) return invalid("TMA descriptor for metadata could not be encoded");
    }
    const uint32_t mma_fmt =
        ((flags & SPMM24_FP8_A_E5M2) ? kIdescFp8AE5M2 : 0u) | ((flags & SPMM24_FP8_B_E5M2) ? kIdescFp8BE5M2 : 0u);
    const bool pdl = !(flags & SPMM24_NO_PDL);
    if (pair) {
        if (epi.residual && pl.split != 1) {  // the partner partial would overlap the residual's staging
            pl.split = 1;
            pl.grid = 2 * pl.m_tiles * pl.n_tiles;
        }
        PairParams kp;
        kp.C = static_cast<uint16_t*>(C);
        kp.epi = epi;
        kp.M = M;
        kp.N = N;
        kp.K = K;
        kp.stages_total = K / 256;
        kp.weights_static = (flags & SPMM24_STATIC_WEIGHTS) ? 1 : 0;
        kp.split = pl.split;
        kp.mma_fmt = mma_fmt;
        if (pl.pair2) {
            auto kern = spmm24_pair2_kernel<kPair2Stages, true, true>;
            e = prepare(kern, Pair2C8::SMEM_ALLOC, dev, kFp8Slot + 13);
            if (e != cudaSuccess) return e;
            return launch_kernel(kern, dim3(2u, (unsigned)pl.n_tiles, (unsigned)pl.m_tiles), Pair2C8::SMEM_ALLOC,
                                 stream, 2u, pdl, ta, tb, te, kp, kPairThreads);
        }
        return pl.split == 2 ? launch_pair_fp8<true>(pl, stream, dev, pdl, ta, tb, te, kp)
                             : launch_pair_fp8<false>(pl, stream, dev, pdl, ta, tb, te, kp);
    }
    ClusterParams kp;
    kp.C = static_cast<uint16_t*>(C);
    kp.epi = epi;
    kp.M = M;
    kp.N = N;
    kp.K = K;
    kp.groups = K / 128;
    kp.stages_total = pl.stages_total;
    kp.split = pl.split;
    kp.weights_static = (flags & SPMM24_STATIC_WEIGHTS) ? 1 : 0;
    kp.mma_fmt = mma_fmt;
    if (pl.shallow) {
        if (pl.tile_n == 16) return launch_cluster_fp8<CV16s>(pl, stream, dev, pdl, ta, tb, te, kp, 9);
        return launch_cluster_fp8<CV32s>(pl, stream, dev, pdl, ta, tb, te, kp, 10);
    }
    switch (pl.tile_n) {
        case 16: return launch_cluster_fp8<CV16>(pl, stream, dev, pdl, ta, tb, te, kp, 0);
        case 32: return launch_cluster_fp8<CV32>(pl, stream, dev, pdl, ta, tb, te, kp, 1);
        case 64: return launch_cluster_fp8<CV64>(pl, stream, dev, pdl, ta, tb, te, kp, 2);
        case 128: return launch_cluster_fp8<CV128>(pl, stream, dev, pdl, ta, tb, te, kp, 3);
        default: return launch_cluster_fp8<CV256>(pl, stream, dev, pdl, ta, tb, te, kp, 4);
    }
}

// ------------------------------------------------------ grouped launch
// Independent narrow-N problems in one persistent launch (spmm24_grouped.cuh).
// The tiles (problem, 128-row block) are balanced over one CTA per SM with
// the longest-processing-time rule: tiles sorted by cost (K stages, plus one
// for the tile's epilogue) in decreasing order, each given to the CTA with
// the least work so far.  The encoded launch (descriptors, epilogues,
// schedule) is kept per host thread and reused while the same problems are
// launched again.
struct GroupCache {
    std::vector<unsigned char> key;  // the problems, their gathers and epilogues, byte for byte
    unsigned flags = 0;
    int sms = 0;
    int n_ctas = 0;
    bool epi = false;    // some problem has a non-plain epilogue
    int split = 1;       // CTAs per tile along K: 1, 2 or 4 (n_ctas then counts clusters)
    int tuned = 0;       // the group_split tuning the schedule was built under
    GroupParams params;
};
thread_local GroupCache* t_group_cache = nullptr;

// Tensor maps of one problem: the 16-bit formats of spmm24_launch, or (fp8)
// those of spmm24_launch_fp8; B boxes are kGroupTileN columns / rows wide.
cudaError_t encode_group_maps(const spmm24_problem& q, bool fp8, GroupParams& gp, int i) {
    const int Ka = fp8 ? q.K / 2 : q.K;  // the A bytes of an fp8 K are those of a 16-bit K / 2
    cuuint64_t adims[3] = {128, (cuuint64_t)(q.M / 16), (cuuint64_t)(Ka / 16)};
    cuuint64_t astr[2] = {(cuuint64_t)16 * Ka, 256};
    cuuint32_t abox[3] = {128, 8, 8};
    if (!encode(&gp.tmA[i], 3, q.compressed_a, adims, astr, abox))
        return invalid("grouped: TMA descriptor for A could not be encoded");
    if (fp8) {
        cuuint64_t bdims[2] = {(cuuint64_t)q.K, (cuuint64_t)q.N};
        cuuint64_t bstr[1] = {(cuuint64_t)q.K};
        cuuint32_t bbox[2] = {128, (cuuint32_t)kGroupTileN};
        if (!encode(&gp.tmB[i], 2, q.b_packed, bdims, bstr, bbox, CU_TENSOR_MAP_DATA_TYPE_UINT8,
                    CU_TENSOR_MAP_SWIZZLE_128B))
            return invalid("grouped: TMA descriptor for B could not be encoded");
        cuuint64_t edims[3] = {128, (cuuint64_t)(q.M / 16), (cuuint64_t)(q.K / 128)};
        cuuint64_t estr[2] = {(cuuint64_t)(q.K / 128) * 256, 256};
        cuuint32_t ebox[3] = {128, 8, 2};
        if (!encode(&gp.tmE[i], 3, q.metadata, edims, estr, ebox))
            return invalid("grouped: TMA descriptor for metadata could not be encoded");
    } else {
        cuuint64_t bdims[4] = {128, (cuuint64_t)(q.K / 64), 4, (cuuint64_t)((q.N + 7) / 8)};
        cuuint64_t bstr[3] = {1024, 256, (cuuint64_t)16 * q.K};
        cuuint32_t bbox[4] = {128, 2, 4, (cuuint32_t)(kGroupTileN / 8)};
        if (!encode(&gp.tmB[i], 4, q.b_packed, bdims, bstr, bbox))
            return invalid("grouped: TMA descriptor for B could not be encoded");
        cuuint64_t edims[2] = {(cuuint64_t)q.K, (cuuint64_t)(q.M / 16)};
        cuuint64_t estr[1] = {(cuuint64_t)2 * q.K};
        cuuint32_t ebox[2] = {128, 8};
        if (!encode(&gp.tmE[i], 2, q.metadata, edims, estr, ebox))
            return invalid("grouped: TMA descriptor for metadata could not be encoded");
    }
    return cudaSuccess;
}

// One 128-row tile of a grouped launch: its cost (K stages + 1 for the
// epilogue), problem and row tile.
struct GroupTile {
    int cost, prob, m_tile;
};
struct GroupSchedule {
    int split = 1;  // CTAs per tile along K: 1, 2 or 4
    int units = 0;  // CTAs, or clusters with a split
    long long makespan = 0;
    std::vector<std::vector<uint16_t>> lists;  // per unit: (problem << 12) | m_tile
};

// Three schedules by the longest-processing-time rule: whole tiles on one
// CTA per SM, or (K split) tiles on clusters of 2 or 4 CTAs with a half or a
// quarter of the stages each; a split is taken when it shortens the busiest
// unit's work by more than a tenth against the best schedule with less split
// (its ring is shallower and each tile pays a partial-sum exchange), or when
// `forced` (the group_split tuning: 1, 2 or 4) asks for it.  Few tiles of
// unequal K (a sharded decode step) balance over the SMs only in quarters.
// Host-only (no CUDA call): spmm24_group_schedule exposes it to tests.
GroupSchedule schedule_group(const std::vector<GroupTile>& tiles, int sms, int max_clusters4, int forced) {
    auto lpt = [&](int max_units, int parts) {
        GroupSchedule sc;
        sc.split = parts;
        std::vector<GroupTile> ts = tiles;
        // cost = stages + 1 (the epilogue); split in `parts`: ceil(stages / parts)
        // + 1, + 1 more for the four-way exchange
        for (GroupTile& t : ts)
            if (parts > 1) t.cost = (t.cost - 1 + parts - 1) / parts + (parts > 2 ? 2 : 1);
        std::stable_sort(ts.begin(), ts.end(), [](const GroupTile& a, const GroupTile& b) { return a.cost > b.cost; });
        sc.units = (int)std::min<size_t>((size_t)std::max(1, max_units), ts.size());
        std::vector<long long> load(sc.units, 0);
        sc.lists.assign(sc.units, {});
        for (const GroupTile& t : ts) {
            int best = 0;  // least loaded unit, lowest index on ties (a linear scan: <= 160 units)
            for (int c = 1; c < sc.units; ++c)
                if (load[c] < load[best]) best = c;
            load[best] += t.cost;
            sc.lists[best].push_back((uint16_t)((t.prob << 12) | t.m_tile));
        }
        for (long long l : load) sc.makespan = std::max(sc.makespan, l);
        return sc;
    };
    const int cap = std::min(sms, kGroupMaxCtas);
    const int c4 = std::min(cap / 4, max_clusters4);
    if (forced == 1) return lpt(cap, 1);
    if (forced == 2) return lpt(cap / 2, 2);
    if (forced == 4) return lpt(c4, 4);
    GroupSchedule best = lpt(cap, 1);
    if (cap >= 2) {
        GroupSchedule halves = lpt(cap / 2, 2);
        if (10 * halves.makespan < 9 * best.makespan) best = std::move(halves);
    }
    if (c4 >= 1) {
        GroupSchedule quarters = lpt(c4, 4);
        if (10 * quarters.makespan < 9 * best.makespan) best = std::move(quarters);
    }
    return best;
}

cudaError_t build_group(const spmm24_problem* probs, int count, unsigned flags, bool fp8, int sms, int max_clusters4,
                        GroupParams& gp, int& n_ctas, bool& any_epi, int& split) {
    std::memset(&gp, 0, sizeof(gp));
    std::vector<GroupTile> tiles;
    any_epi = false;
    for (int i = 0; i < count; ++i) {
        const spmm24_problem& q = probs[i];
        const int groups = fp8 ? q.K / 128 : q.K / 64, st = (groups + 1) / 2;
        GroupProblem& g = gp.prob[i];
        g.C = static_cast<uint16_t*>(q.c);
        g.M = q.M;
        g.N = q.N;
        g.K = q.K;
        g.groups = groups;
        g.stages_total = st;
        cudaError_t e = make_epilogue(q.epilogue, flags, q.c, &g.epi);
        if (e != cudaSuccess) return e;
        if (!epilogue_is_plain_host(g.epi)) any_epi = true;
        if (q.gather) {
            if (g.epi.packed) return invalid("gather: the full C is row-major");
            g.epi.gather_n = q.gather->n_ranks;
            g.epi.gather_row0 = q.gather->row_offset;
            for (int r = 0; r < q.gather->n_ranks; ++r)
                g.epi.gather_dst[r] = static_cast<uint16_t*>(q.gather->c_full[r]);
            g.epi.gather_mc = static_cast<uint16_t*>(q.gather->c_multicast);
        }
        const int mt = (q.M + kTileM - 1) / kTileM;
        for (int m = 0; m < mt; ++m) tiles.push_back({st + 1, i, m});
        if ((e = encode_group_maps(q, fp8, gp, i)) != cudaSuccess) return e;
    }
    GroupSchedule sc = schedule_group(tiles, sms, max_clusters4, g_tune.group_split.load(std::memory_order_relaxed));
    split = sc.split;
    n_ctas = sc.units;  // CTAs, or clusters with a split
    int off = 0;
    for (int c = 0; c < n_ctas; ++c) {
        gp.sched_off[c] = (uint16_t)off;
        for (uint16_t e : sc.lists[c]) gp.sched[off++] = e;
    }
    gp.sched_off[n_ctas] = (uint16_t)off;
    gp.n_problems = count;
    gp.weights_static = (flags & SPMM24_STATIC_WEIGHTS) ? 1 : 0;
    gp.bf16 = (flags & SPMM24_BF16) ? 1 : 0;
    gp.mma_fmt = ((flags & SPMM24_FP8_A_E5M2) ? kIdescFp8AE5M2 : 0u) | ((flags & SPMM24_FP8_B_E5M2) ? kIdescFp8BE5M2 : 0u);
    return cudaSuccess;
}

template <bool FP8, int SPLIT>
constexpr int group_stages() {
    return SPLIT == 4 ? kGroupSplit4Stages : SPLIT == 2 ? (FP8 ? kGroupSplitStagesFp8 : kGroupSplitStages) : kGroupStages;
}

template <bool EPI, bool FP8, int SPLIT>
cudaError_t prepare_group_kernel(int dev) {
    constexpr int ST = group_stages<FP8, SPLIT>();
    return prepare(spmm24_grouped_kernel<ST, EPI, FP8, SPLIT>, GroupCfg<ST, FP8, SPLIT>::SMEM_ALLOC, dev,
                   80 + (EPI ? 1 : 0) + (FP8 ? 2 : 0) + (SPLIT == 2 ? 4 : SPLIT == 4 ? 8 : 0));
}

// Clusters of four grouped CTAs that fit on the device at once (a GPC whose
// SM count is not a multiple of four leaves SMs idle), cached per device;
// 0 if the query fails (no four-way split then).
int group_max_clusters4(int dev, bool fp8) {
    static std::atomic<int> cache[2][64];
    std::atomic<int>& slot = cache[fp8 ? 1 : 0][dev & 63];
    int v = slot.load(std::memory_order_relaxed);
    if (v) return v - 1;
    constexpr int ST16 = group_stages<false, 4>(), ST8 = group_stages<true, 4>();
    cudaError_t e = fp8 ? prepare_group_kernel<true, true, 4>(dev) : prepare_group_kernel<false, false, 4>(dev);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(4 * 64, 1, 1);
    cfg.blockDim = dim3((unsigned)kThreads, 1, 1);
    cfg.dynamicSmemBytes = fp8 ? GroupCfg<ST8, true, 4>::SMEM_ALLOC : GroupCfg<ST16, false, 4>::SMEM_ALLOC;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 4;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (e == cudaSuccess)
        e = fp8 ? cudaOccupancyMaxActiveClusters(&n, spmm24_grouped_kernel<ST8, true, true, 4>, &cfg)
                : cudaOccupancyMaxActiveClusters(&n, spmm24_grouped_kernel<ST16, false, false, 4>, &cfg);
    if (e != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    slot.store(n + 1, std::memory_order_relaxed);
    return n;
}

template <bool EPI, bool FP8, int SPLIT>
cudaError_t launch_group_kernel(cudaStream_t stream, int dev, const GroupCache& gc, unsigned flags) {
    constexpr int ST = group_stages<FP8, SPLIT>();
    using GC = GroupCfg<ST, FP8, SPLIT>;
    auto kern = spmm24_grouped_kernel<ST, EPI, FP8, SPLIT>;
    cudaError_t e = prepare_group_kernel<EPI, FP8, SPLIT>(dev);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(gc.n_ctas * SPLIT), 1, 1);
    cfg.blockDim = dim3((unsigned)kThreads, 1, 1);
    cfg.dynamicSmemBytes = GC::SMEM_ALLOC;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = (flags & SPMM24_NO_PDL) ? 0 : 1;
    int n = 1;
    if (SPLIT > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = SPLIT;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        n = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kern, gc.params);
}

cudaError_t launch_grouped_impl(cudaStream_t stream, const spmm24_problem* probs, int count, unsigned flags,
                                bool fp8, const spmm24_group_barrier* bar = nullptr) {
    g_last_error[0] = '\0';
    if (!probs) return invalid("grouped: null problem array");
    if (bar) {
        if (bar->n_ranks < 1 || bar->n_ranks > SPMM24_MAX_GATHER_RANKS || bar->rank < 0 || bar->rank >= bar->n_ranks)
            return invalid("barrier: bad rank or rank count");
        if (bar->limit_us == 0 || bar->limit_us > 60000000u) return invalid("barrier: limit_us must be 1..60e6");
        for (int r = 0; r < bar->n_ranks; ++r)
            if (!bar->flag_arrays[r] || ((uintptr_t)bar->flag_arrays[r] & 3u))
                return invalid("barrier: bad flag array");
    }
    if (count < 1 || count > kGroupMaxProblems) return invalid("grouped: count must be 1..16");
    const unsigned allowed = SPMM24_STATIC_WEIGHTS | SPMM24_NO_PDL | SPMM24_BF16 |
                             (fp8 ? (unsigned)(SPMM24_FP8_A_E5M2 | SPMM24_FP8_B_E5M2) : 0u);
    if (flags & ~allowed) return invalid("unknown flag");
    long long tiles = 0;
    for (int i = 0; i < count; ++i) {
        const spmm24_problem& q = probs[i];
        if (!q.compressed_a || !q.b_packed || !q.metadata || (!q.c && !q.gather)) return invalid("grouped: null pointer");
        if (q.M <= 0 || q.N <= 0 || q.K <= 0) return invalid("grouped: M, N and K must be positive");
        if (q.M % 16) return invalid("grouped: M must be a multiple of 16");
        if (fp8 ? (q.K % 128) : (q.K % 64)) return invalid(fp8 ? "grouped fp8: K must be a multiple of 128"
                                                               : "grouped: K must be a multiple of 64");
        if (q.N > kGroupTileN) return invalid("grouped: N must be <= 32 (wider N: spmm24_launch)");
        if (((uintptr_t)q.compressed_a | (uintptr_t)q.b_packed | (uintptr_t)q.metadata) & 15u)
            return invalid("grouped: A, B and metadata must be 16-byte aligned");
        if ((uintptr_t)q.c & 1u) return invalid("grouped: C must be 2-byte aligned");
        if ((q.M + kTileM - 1) / kTileM > 4096) return invalid("grouped: M must be <= 524288");
        tiles += (q.M + kTileM - 1) / kTileM;
        if (const spmm24_gather* g = q.gather) {
            if (g->n_ranks < 1 || g->n_ranks > SPMM24_MAX_GATHER_RANKS) return invalid("gather: n_ranks must be 1..8");
            if (g->row_offset < 0 || g->m_full < q.M || g->row_offset > g->m_full - q.M)
                return invalid("gather: the shard's rows must lie inside the full C");
            for (int r = 0; r < g->n_ranks; ++r) {
                if (!g->c_full[r]) return invalid("gather: null full-C pointer");
                if ((uintptr_t)g->c_full[r] & 15u) return invalid("gather: full-C buffers must be 16-byte aligned");
            }
            if (g->c_multicast && ((uintptr_t)g->c_multicast & 15u))
                return invalid("gather: the multicast C must be 16-byte aligned");
        }
    }
    if (tiles > kGroupMaxTiles) return invalid("grouped: more than 2048 128-row tiles in one launch");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int sms = sm_count(dev);
    if (!t_group_cache) t_group_cache = new GroupCache();
    GroupCache& gc = *t_group_cache;
    // Cache key: every problem and the contents of its gather and epilogue.
    thread_local std::vector<unsigned char> key;
    key.clear();
    auto put = [](std::vector<unsigned char>& k, const void* p, size_t n) {
        const unsigned char* b = static_cast<const unsigned char*>(p);
        k.insert(k.end(), b, b + n);
    };
    key.push_back(fp8 ? 1 : 0);
    spmm24_group_barrier bk{};
    if (bar) bk = *bar;
    put(key, &bk, sizeof(bk));
    for (int i = 0; i < count; ++i) {
        put(key, &probs[i], sizeof(spmm24_problem));
        spmm24_gather g{};
        if (probs[i].gather) g = *probs[i].gather;
        put(key, &g, sizeof(g));
        spmm24_epilogue ep{};
        if (probs[i].epilogue) ep = *probs[i].epilogue;
        put(key, &ep, sizeof(ep));
    }
    const int tuned = g_tune.group_split.load(std::memory_order_relaxed);
    const bool hit = gc.n_ctas > 0 && gc.flags == flags && gc.sms == sms && gc.tuned == tuned && gc.key == key;
    if (!hit) {
        gc.n_ctas = 0;
        int n = 0, split = 1;
        bool any_epi = false;
        if ((e = build_group(probs, count, flags, fp8, sms, group_max_clusters4(dev, fp8), gc.params, n, any_epi,
                             split)) != cudaSuccess)
            return e;
        gc.key = key;
        gc.flags = flags;
        gc.sms = sms;
        gc.n_ctas = n;
        gc.epi = any_epi;
        gc.split = split;
        gc.tuned = tuned;
        if (bar) {
            for (int r = 0; r < bar->n_ranks; ++r) gc.params.bar_flags[r] = bar->flag_arrays[r];
            gc.params.bar_n = bar->n_ranks;
            gc.params.bar_rank = bar->rank;
            gc.params.bar_limit_ns = (unsigned long long)bar->limit_us * 1000ull;
        }
    }
#ifdef SPMM24_TRACE
    gc.params.trace_base = g_trace_next.fetch_add((long long)gc.n_ctas);
#endif
    if (gc.split == 4) {
        if (fp8) return launch_group_kernel<true, true, 4>(stream, dev, gc, flags);
        if (gc.epi) return launch_group_kernel<true, false, 4>(stream, dev, gc, flags);
        return launch_group_kernel<false, false, 4>(stream, dev, gc, flags);
    }
    if (gc.split == 2) {
        if (fp8) return launch_group_kernel<true, true, 2>(stream, dev, gc, flags);
        if (gc.epi) return launch_group_kernel<true, false, 2>(stream, dev, gc, flags);
        return launch_group_kernel<false, false, 2>(stream, dev, gc, flags);
    }
    if (fp8) return launch_group_kernel<true, true, 1>(stream, dev, gc, flags);
    if (gc.epi) return launch_group_kernel<true, false, 1>(stream, dev, gc, flags);
    return launch_group_kernel<false, false, 1>(stream, dev, gc, flags);
}

// ------------------------------------------------ allocation-free variant
// Scratch for spmm24_launch_noalloc, owned by the library as a file-scope
// device array instead of a cudaMalloc'ed buffer: 256 flag words followed by
// room for 256 partial tiles of 128 x 32 fp32 (4 MB + 1 KB in total, held by
// every GPU that loads the library until the process exits).
constexpr int kNoAllocMaxCtas = 256;
constexpr int kNoAllocMaxTileN = 32;
constexpr size_t kNoAllocFlagBytes = (size_t)kNoAllocMaxCtas * sizeof(uint32_t);  // 1 KB, keeps the partials 256-B aligned
constexpr size_t kNoAllocPartialBytes = (size_t)kNoAllocMaxCtas * kTileM * kNoAllocMaxTileN * sizeof(float);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocFlagBytes + kNoAllocPartialBytes];

// Device address of g_noalloc_scratch per device.  In host code the array's
// name is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress, once per device, with that device current.
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

cudaError_t noalloc_scratch(int dev, void** out) {
    if (dev < 0 || dev >= kMaxDevices) return invalid("device index out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        if (!p) return cudaErrorInvalidSymbol;
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return cudaSuccess;
}

cudaError_t launch_noalloc_impl(cudaStream_t stream, const void* A, const void* B, const uint16_t* E, void* C, int M,
                                int N, int K) {
    g_last_error[0] = '\0';
    if (!A || !B || !E || !C) return invalid("null pointer");
    if (M <= 0 || N <= 0 || K <= 0) return invalid("M, N and K must be positive");
    if (M % 16) return invalid("M must be a multiple of 16");
    if (K % 64) return invalid("K must be a multiple of 64");
    if (N > kNoAllocMaxTileN)
        return invalid("spmm24_launch_noalloc supports N <= 32: its fixed scratch holds 256 partial tiles of "
                       "128 x 32 fp32 (4 MB); use spmm24_launch for wider N");
    if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)E) & 15u) return invalid("A, B and metadata must be 16-byte aligned");
    if ((uintptr_t)C & 1u) return invalid("C must be 2-byte aligned");
    if ((long)M / kTileM >= 65535) return invalid("M too large");

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    void* scratch = nullptr;
    if ((e = noalloc_scratch(dev, &scratch)) != cudaSuccess) return e;

    Plan pl{};
    pl.path = Path::kStreamK;
    pl.shallow = false;
    pl.tile_n = N <= 16 ? 16 : 32;
    pl.stages = pl.tile_n == 16 ? SV16::kStages : SV32::kStages;
    pl.smem = pl.tile_n == 16 ? SV16::C_::SMEM_ALLOC : SV32::C_::SMEM_ALLOC;
    pl.m_tiles = (M + kTileM - 1) / kTileM;
    pl.n_tiles = 1;
    pl.stages_total = (K / 64 + 1) / 2;
    pl.split = 1;
    const long long units = (long long)pl.m_tiles * pl.stages_total;
    pl.grid = (int)std::max<long long>(1, std::min<long long>(std::min(sm_count(dev), kNoAllocMaxCtas), units));
    if ((size_t)pl.grid * kTileM * pl.tile_n * sizeof(float) > kNoAllocPartialBytes ||
        (size_t)pl.grid * sizeof(uint32_t) > kNoAllocFlagBytes)
        return invalid("problem needs more scratch than spmm24_launch_noalloc holds");

    uint32_t* flags = static_cast<uint32_t*>(scratch);
    float* partials = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + kNoAllocFlagBytes);
    // The scratch keeps whatever the previous call left; the flags must start
    // at zero, so clear the ones this call uses (a memset node, no allocation).
    if ((e = cudaMemsetAsync(flags, 0, (size_t)pl.grid * sizeof(uint32_t), stream)) != cudaSuccess) return e;

    CUtensorMap ta, tb, te;
    {
        cuuint64_t dims[3] = {128, (cuuint64_t)(M / 16), (cuuint64_t)(K / 16)};
        cuuint64_t str[2] = {(cuuint64_t)16 * K, 256};
        cuuint32_t box[3] = {128, 8, 8};
        if (!encode(&ta, 3, A, dims, str, box)) return invalid("TMA descriptor for A could not be encoded");
    }
    {
        cuuint64_t dims[4] = {128, (cuuint64_t)(K / 64), 4, (cuuint64_t)((N + 7) / 8)};
        cuuint64_t str[3] = {1024, 256, (cuuint64_t)16 * K};
        cuuint32_t box[4] = {128, 2, 4, (cuuint32_t)(pl.tile_n / 8)};
        if (!encode(&tb, 4, B, dims, str, box)) return invalid("TMA descriptor for B could not be encoded");
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)(M / 16)};
        cuuint64_t str[1] = {(cuuint64_t)2 * K};
        cuuint32_t box[2] = {128, 8};
        if (!encode(&te, 2, E, dims, str, box)) return invalid("TMA descriptor for metadata could not be encoded");
    }
    StreamKParams kp;
    kp.C = static_cast<__half*>(C);
    kp.ws = partials;
    kp.flags = flags;
    kp.M = M;
    kp.N = N;
    kp.K = K;
    kp.groups = K / 64;
    kp.stages_per_tile = pl.stages_total;
    kp.m_tiles = pl.m_tiles;
    kp.n_tiles = pl.n_tiles;
    kp.units = units;
    kp.grid = pl.grid;
    kp.weights_static = 0;
    if (pl.tile_n == 16) return launch_streamk<SV16>(pl, stream, dev, true, ta, tb, te, kp, 5);
    return launch_streamk<SV32>(pl, stream, dev, true, ta, tb, te, kp, 6);
}

// ------------------------------------------------------ bounded-wait self test
// A flag and an mbarrier that nothing ever completes: the self test waits on
// one of them with a short limit and must come back with a timeout status,
// leaving the context usable.  Failure detection is thereby tested without
// faulting, trapping or hanging the GPU.
static __device__ uint32_t g_selftest_flag;  // stays 0
static __device__ uint32_t g_selftest_result;

__global__ void spmm24_selftest_kernel(int which, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    uint32_t status = 0;
    if (threadIdx.x == 0) {
        if (which == 0) {
            ptx::mbar_init(&bar, 1);  // expects one arrival that never comes
            ptx::fence_mbarrier_init();
            if (!ptx::mbar_wait_bounded(&bar, 0, limit_ns)) status = kStatusMmaTimeout;
        } else {
            if (!ptx::wait_flag_bounded(&g_selftest_flag, limit_ns)) status = kStatusEpilogueTimeout;
        }
        g_selftest_result = status;
    }
}

// Cross-GPU barrier after a fused all-gather launch: rank `rank` publishes
// `epoch` in its slot of every rank's flag array (system-scope release,
// after a system fence: the previous kernel's peer stores are complete at
// the kernel boundary and ordered before the flag), then waits -- bounded --
// until every rank's slot in its own array has reached `epoch`.
struct BarrierArgs {
    uint32_t* flags[SPMM24_MAX_GATHER_RANKS];  // rank r's flag array (own one included)
    int n, rank;
    uint32_t epoch;
    unsigned long long limit_ns;
};

__global__ void spmm24_gather_barrier_kernel(BarrierArgs a) {
    __shared__ uint32_t epoch_s;
    const int t = threadIdx.x;
    ptx::grid_dep_wait();
    // The next kernel in the stream may be scheduled now (its weight
    // prefetch then overlaps this wait); it still waits for this grid to
    // finish before reading anything the gather wrote.
    if (t == 0) ptx::grid_dep_launch();
    // Epoch 0: one past this rank's last published epoch (slot `rank` of its
    // own array, written only by its own earlier barriers), read before any
    // thread publishes the new one.
    if (t == 0) epoch_s = a.epoch ? a.epoch : ptx::ld_acquire_sys(a.flags[a.rank] + a.rank) + 1u;
    __syncthreads();
    const uint32_t epoch = epoch_s;
    __threadfence_system();
    if (t < a.n) ptx::st_release_sys(a.flags[t] + a.rank, epoch);
    if (t < a.n) {
        const uint32_t* f = a.flags[a.rank] + t;
        const uint64_t t0 = ptx::globaltimer();
        while ((int)(ptx::ld_acquire_sys(f) - epoch) < 0) {
            ptx::nanosleep_ns(100);
            if (ptx::globaltimer() - t0 > a.limit_ns) {
                atomicOr(&g_spmm24_status, kStatusBarrierTimeout);
                break;
            }
        }
    }
}

using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn address_range_fn() {
    static GetAddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetAddressRangeFn>(p);
    });
    return fn;
}

// Pointers returned by spmm24_ipc_import -> the base address of the mapping.
std::mutex g_ipc_mu;
std::map<uintptr_t, void*>* g_ipc_bases = new std::map<uintptr_t, void*>();

}  // namespace
}  // namespace spmm24

// ---------------------------------------------------------------- C ABI
extern "C" cudaError_t spmm24_launch(cudaStream_t stream, const void* compressed_a, const void* b_packed,
                                     const uint16_t* metadata, void* c, int M, int N, int K, void* split_reduction,
                                     int split_k) {
    (void)split_reduction;
    return spmm24::launch_impl(stream, compressed_a, b_packed, metadata, c, M, N, K, split_k, 0u);
}

extern "C" cudaError_t spmm24_launch_ex(cudaStream_t stream, const void* compressed_a, const void* b_packed,
                                        const uint16_t* metadata, void* c, int M, int N, int K, int split_k,
                                        unsigned flags) {
    return spmm24::launch_impl(stream, compressed_a, b_packed, metadata, c, M, N, K, split_k, flags);
}

extern "C" cudaError_t spmm24_launch_noalloc(cudaStream_t stream, const void* compressed_a, const void* b_packed,
                                             const uint16_t* metadata, void* c, int M, int N, int K) {
    return spmm24::launch_noalloc_impl(stream, compressed_a, b_packed, metadata, c, M, N, K);
}

extern "C" cudaError_t spmm24_launch_grouped(cudaStream_t stream, const spmm24_problem* problems, int count,
                                            unsigned flags) {
    return spmm24::launch_grouped_impl(stream, problems, count, flags, false);
}

extern "C" cudaError_t spmm24_launch_grouped_fp8(cudaStream_t stream, const spmm24_problem* problems, int count,
                                                unsigned flags) {
    return spmm24::launch_grouped_impl(stream, problems, count, flags, true);
}

extern "C" cudaError_t spmm24_launch_grouped_gather(cudaStream_t stream, const spmm24_problem* problems, int count,
                                                   unsigned flags, const spmm24_group_barrier* barrier) {
    if (!barrier) return spmm24::record_invalid("barrier: null descriptor");
    return spmm24::launch_grouped_impl(stream, problems, count, flags, false, barrier);
}

extern "C" cudaError_t spmm24_launch_fused(cudaStream_t stream, const void* compressed_a, const void* b_packed,
                                           const uint16_t* metadata, void* c, int M, int N, int K, int split_k,
                                           unsigned flags, const spmm24_epilogue* epilogue) {
    return spmm24::launch_impl(stream, compressed_a, b_packed, metadata, c, M, N, K, split_k, flags, epilogue);
}

extern "C" cudaError_t spmm24_launch_fp8(cudaStream_t stream, const void* values, const void* b_nk, const void* metadata,
                                         void* c, int M, int N, int K, int split_k, unsigned flags,
                                         const spmm24_epilogue* epilogue) {
    return spmm24::launch_fp8_impl(stream, values, b_nk, metadata, c, M, N, K, split_k, flags, epilogue);
}

extern "C" cudaError_t spmm24_launch_gather(cudaStream_t stream, const void* compressed_a, const void* b_packed,
                                            const uint16_t* metadata, int M, int N, int K, int split_k, unsigned flags,
                                            const spmm24_gather* gather) {
    if (!gather) return spmm24::record_invalid("gather: null descriptor");
    if (gather->n_ranks < 1 || gather->n_ranks > SPMM24_MAX_GATHER_RANKS || !gather->c_full[0])
        return spmm24::record_invalid("gather: n_ranks must be 1..8 with non-null buffers");
    // C is only used for the alignment test of the 16-byte stores: the
    // shard's rows in the first rank's buffer.
    void* c = static_cast<uint16_t*>(gather->c_full[0]) + (size_t)(gather->row_offset > 0 ? gather->row_offset : 0) * N;
    return spmm24::launch_impl(stream, compressed_a, b_packed, metadata, c, M, N, K, split_k, flags, nullptr, gather);
}

extern "C" cudaError_t spmm24_gather_barrier(cudaStream_t stream, uint32_t* const* flag_arrays, int n_ranks, int rank,
                                             uint32_t epoch, unsigned limit_us) {
    spmm24::clear_last_error();
    if (!flag_arrays || n_ranks < 1 || n_ranks > SPMM24_MAX_GATHER_RANKS || rank < 0 || rank >= n_ranks)
        return spmm24::record_invalid("barrier: bad rank or rank count");
    if (limit_us == 0 || limit_us > 60000000u) return spmm24::record_invalid("barrier: limit_us must be 1..60e6");
    spmm24::BarrierArgs a{};
    for (int r = 0; r < n_ranks; ++r) {
        if (!flag_arrays[r] || ((uintptr_t)flag_arrays[r] & 3u)) return spmm24::record_invalid("barrier: bad flag array");
        a.flags[r] = flag_arrays[r];
    }
    a.n = n_ranks;
    a.rank = rank;
    a.epoch = epoch;
    a.limit_ns = (unsigned long long)limit_us * 1000ull;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 0;  // plain stream order: the gather kernel has completed
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, spmm24::spmm24_gather_barrier_kernel, a);
}

extern "C" cudaError_t spmm24_ipc_export(const void* dev_ptr, spmm24_ipc_handle* out) {
    spmm24::clear_last_error();
    if (!dev_ptr || !out) return spmm24::record_invalid("ipc: null pointer");
    auto fn = spmm24::address_range_fn();
    if (!fn) return spmm24::record_invalid("ipc: cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
        return spmm24::record_invalid("ipc: not a device allocation");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return e;
    static_assert(sizeof(h) <= sizeof(out->handle), "IPC handle size");
    std::memset(out, 0, sizeof(*out));
    std::memcpy(out->handle, &h, sizeof(h));
    out->offset = (uint64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
    return cudaSuccess;
}

extern "C" cudaError_t spmm24_ipc_import(const spmm24_ipc_handle* handle, void** dev_ptr) {
    spmm24::clear_last_error();
    if (!handle || !dev_ptr) return spmm24::record_invalid("ipc: null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle->handle, sizeof(h));
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return e;
    void* p = static_cast<uint8_t*>(base) + handle->offset;
    {
        std::lock_guard<std::mutex> lk(spmm24::g_ipc_mu);
        (*spmm24::g_ipc_bases)[reinterpret_cast<uintptr_t>(p)] = base;
    }
    *dev_ptr = p;
    return cudaSuccess;
}

extern "C" cudaError_t spmm24_ipc_close(void* dev_ptr) {
    spmm24::clear_last_error();
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(spmm24::g_ipc_mu);
        auto it = spmm24::g_ipc_bases->find(reinterpret_cast<uintptr_t>(dev_ptr));
        if (it == spmm24::g_ipc_bases->end()) return spmm24::record_invalid("ipc: not an imported pointer");
        base = it->second;
        spmm24::g_ipc_bases->erase(it);
    }
    return cudaIpcCloseMemHandle(base);
}

extern "C" size_t spmm24_workspace_bytes(int, int, int, int) { return 0; }

namespace spmm24 {
namespace {
int current_sms() {
    int dev = 0;
    int sms = (cudaGetDevice(&dev) == cudaSuccess) ? sm_count(dev) : 148;
    if (sms <= 0) sms = 148;
    cudaGetLastError();
    return sms;
}
void fill_config(const Plan& pl, int stage_k, spmm24_config* out);
}  // namespace
}  // namespace spmm24

extern "C" int spmm24_group_schedule(const int* M, const int* K, int count, int fp8, int sms, int max_clusters4,
                                     int* split, int* units, long long* makespan) {
    if (!M || !K || count < 1 || count > spmm24::kGroupMaxProblems || sms < 1 || max_clusters4 < 0) return -1;
    std::vector<spmm24::GroupTile> tiles;
    for (int i = 0; i < count; ++i) {
        if (M[i] <= 0 || M[i] % 16 || K[i] <= 0 || (fp8 ? K[i] % 128 : K[i] % 64)) return -1;
        const int groups = fp8 ? K[i] / 128 : K[i] / 64, st = (groups + 1) / 2;
        const int mt = (M[i] + spmm24::kTileM - 1) / spmm24::kTileM;
        if ((long long)tiles.size() + mt > spmm24::kGroupMaxTiles) return -1;
        for (int m = 0; m < mt; ++m) tiles.push_back({st + 1, i, m});
    }
    const spmm24::GroupSchedule sc =
        spmm24::schedule_group(tiles, sms, max_clusters4, spmm24::g_tune.group_split.load(std::memory_order_relaxed));
    if (split) *split = sc.split;
    if (units) *units = sc.units;
    if (makespan) *makespan = sc.makespan;
    return 0;
}

extern "C" cudaError_t spmm24_set_tuning(const spmm24_tuning* t) {
    spmm24::clear_last_error();
    spmm24_tuning v{-1, -1, 0, 0, 0, 0};
    if (t) {
        v = *t;
        const bool tn_ok = v.tile_n == 0 || v.tile_n == 16 || v.tile_n == 32 || v.tile_n == 64 || v.tile_n == 128 ||
                           v.tile_n == 256;
        if (v.pair < -1 || v.pair > 1 || v.pair2 < -1 || v.pair2 > 1 || v.pair_split < 0 || v.pair_split > 2 || !tn_ok ||
            v.deep_ring < 0 || v.deep_ring > 1 || v.group_split < 0 || v.group_split > 4 || v.group_split == 3)
            return spmm24::record_invalid("tuning: a field is out of range");
    }
    spmm24::g_tune.pair.store(v.pair);
    spmm24::g_tune.pair2.store(v.pair2);
    spmm24::g_tune.pair_split.store(v.pair_split);
    spmm24::g_tune.tile_n.store(v.tile_n);
    spmm24::g_tune.deep_ring.store(v.deep_ring);
    spmm24::g_tune.group_split.store(v.group_split);
    return cudaSuccess;
}

extern "C" int spmm24_select_config(int M, int N, int K, int split_k, spmm24_config* out) {
    if (!out || M <= 0 || N <= 0 || K <= 0 || M % 16 || K % 64 || split_k < 0) return -1;
    spmm24::fill_config(spmm24::make_plan(M, N, K, split_k, spmm24::current_sms()), 128, out);
    return 0;
}

extern "C" int spmm24_select_config_fp8(int M, int N, int K, int split_k, spmm24_config* out) {
    if (!out || M <= 0 || N <= 0 || K <= 0 || M % 16 || K % 128 || split_k < 0) return -1;
    spmm24::fill_config(spmm24::plan_fp8(M, N, K, split_k, spmm24::current_sms(), true), 256, out);
    return 0;
}

namespace spmm24 {
namespace {
void fill_config(const Plan& pl, int stage_k, spmm24_config* out) {
    out->tile_m = pl.path == spmm24::Path::kPair ? (pl.pair2 ? 4 : 2) * spmm24::kTileM : spmm24::kTileM;
    out->tile_n = pl.tile_n;
    out->stage_k = stage_k;
    out->stages = pl.stages;
    out->split_k = pl.path == spmm24::Path::kStreamK ? 0 : pl.split;
    out->grid_ctas = pl.grid;
    out->smem_bytes = pl.smem;
    out->stream_k = pl.path == spmm24::Path::kStreamK ? 1 : 0;
    out->cta_pair = pl.path == spmm24::Path::kPair ? 1 : 0;
}
}  // namespace
}  // namespace spmm24

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

extern "C" cudaError_t spmm24_selftest_bounded_wait(int which, unsigned limit_us, uint32_t* status_out) {
    if (!status_out || (which != 0 && which != 1) || limit_us == 0 || limit_us > 10000000u)
        return cudaErrorInvalidValue;
    spmm24::spmm24_selftest_kernel<<<1, 32>>>(which, (unsigned long long)limit_us * 1000ull);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    uint32_t v = 0;
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, spmm24::g_selftest_result, sizeof(v));
    *status_out = v;
    return e;
}

extern "C" const char* spmm24_last_error(void) { return spmm24::g_last_error; }

#ifdef SPMM24_TRACE
// Trace builds only: where the kernels write their per-CTA timeline.
extern "C" cudaError_t spmm24_set_trace(void* buf) {
    spmm24::g_trace_next = 0;
    return cudaMemcpyToSymbol(spmm24::g_spmm24_trace, &buf, sizeof(buf));
}
#endif

extern "C" const char* spmm24_version(void) { return "spmm24 0.2.0 (sm_100a tcgen05.mma.sp)"; }

// ------------------------------------------------------- C++ drop-in
cudaError_t SpMM_N2M4_Launch(cudaStream_t stream, const half* Compressed_A, const half* B, const uint16_t* metadata,
                             half* C, const int M_Global, const int N_Global, const int K_Global,
                             half* Split_Reduction, const int Split_K) {
    (void)Split_Reduction;
    return spmm24::launch_impl(stream, Compressed_A, B, metadata, C, M_Global, N_Global, K_Global, Split_K, 0u);
}
