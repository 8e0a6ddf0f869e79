// pack_device.cu -- the host packer (packer.cpp) as sm_100a kernels, so
// weights and activations can be brought into the SpMM's formats without a
// round trip through host memory:
//
//   spmm24_pack_a_device     optional magnitude 2:4 prune, then compress to
//                            16x8 value blocks and write the reordered
//                            metadata, in one pass over the dense weights
//                            (toolCompressMatrixA + toolReorderMetadata,
//                            SpeakOutLoudly/CUDA-Repo test/utils.h:91-185)
//   spmm24_prune_2of4_device the prune alone, in place
//   spmm24_pack_b_device     row-major K x N -> 8-column strips
//                            (toolPackMatrixB, test/utils.h:188-229)
//
// All three are bit-exact with packer.cpp on every input the host functions
// accept.  They are HBM-bound copies: each CTA stages a tile in shared
// memory so that both the reads and the writes are coalesced.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx_sm100.cuh"
#include "spmm24/SpMM_API.h"
#include "spmm24_host.h"

namespace spmm24 {
namespace {

constexpr int kPackThreads = 256;
constexpr int kTileBlocks = 16;                      // 16-K blocks per A tile (256 columns)
constexpr int kTileCols = kTileBlocks * 16;          // halves per A tile row
constexpr int kTilePitch = kTileCols + 8;            // padded row pitch (halves): 16-byte bank shift per row
constexpr int kBTileRows = 64, kBTileCols = 64;      // B tile: 64 K rows x 8 strips
constexpr int kBTilePitch = kBTileCols + 8;

// The kernels work on a group of four halves held in two 32-bit words
// (x = h0 | h1 << 16, y = h2 | h3 << 16) with integer operations only.
//
// Magnitudes: for fp16 and bf16 bit patterns alike, |x| orders like the
// 15-bit integer h & 0x7fff, except that a NaN (above the infinity pattern:
// 0x7c00 for fp16, 0x7f80 for bf16) compares false with everything -- the
// host's float comparisons, reproduced exactly.

// True when none of the four magnitudes (ax, ay: two 15-bit halves each)
// is above `inf`: adding 0x7fff - inf to each half carries into its bit 15
// exactly when it is above (no half overflows its 16 bits).
__device__ __forceinline__ bool no_nan(uint32_t ax, uint32_t ay, uint32_t inf) {
    const uint32_t add = (0x7fffu - inf) * 0x10001u;
    return (((ax + add) | (ay + add)) & 0x80008000u) == 0u;
}

// Magnitude 2:4 prune of one group (packer.cpp spmm24_prune_2of4): keep the
// largest |x| (first on ties), then the largest of the other three (first on
// ties), replace the other two by +0.
//
// Sequential form, exact for NaN (a NaN never wins or loses a comparison).
__device__ __forceinline__ uint32_t prune_keep_sequential(uint32_t ax, uint32_t ay, uint32_t inf) {
    const uint32_t m0 = ax & 0xffffu, m1 = ax >> 16, m2 = ay & 0xffffu, m3 = ay >> 16;
    const bool v0 = m0 <= inf, v1 = m1 <= inf, v2 = m2 <= inf, v3 = m3 <= inf;
    uint32_t k0 = 0, mk = m0;
    bool c = v0 && v1 && m1 > mk;
    k0 = c ? 1u : k0;
    mk = c ? m1 : mk;
    c = v0 && v2 && m2 > mk;
    k0 = c ? 2u : k0;
    mk = c ? m2 : mk;
    c = v0 && v3 && m3 > mk;
    k0 = c ? 3u : k0;
    uint32_t k1 = k0 == 0 ? 1u : 0u;
    uint32_t mk1 = k0 == 0 ? m1 : m0;
    const bool vk1 = k0 == 0 ? v1 : v0;
    c = k0 >= 2 && vk1 && v1 && m1 > mk1;
    k1 = c ? 1u : k1;
    mk1 = c ? m1 : mk1;
    c = k0 != 2 && vk1 && v2 && m2 > mk1;
    k1 = c ? 2u : k1;
    mk1 = c ? m2 : mk1;
    c = k0 != 3 && vk1 && v3 && m3 > mk1;
    k1 = c ? 3u : k1;
    return (1u << k0) | (1u << k1);
}

// `inf`: the infinity bit pattern of the element type (0x7c00 fp16, 0x7f80 bf16).
__device__ __forceinline__ void prune_group(uint32_t& x, uint32_t& y, uint32_t inf) {
    const uint32_t ax = x & 0x7fff7fffu, ay = y & 0x7fff7fffu;
    uint32_t keep;
    if (no_nan(ax, ay, inf)) {
        // No NaN: the sequential scan keeps the two largest of the unique keys
        // |x| << 2 | (3 - position) (equal magnitudes: the lower position wins).
        const uint32_t a0 = ((ax << 2) & 0x3fffcu) | 3u, a1 = ((ax >> 14) & 0x3fffcu) | 2u;
        const uint32_t a2 = ((ay << 2) & 0x3fffcu) | 1u, a3 = (ay >> 14) & 0x3fffcu;
        const uint32_t hi01 = max(a0, a1), lo01 = min(a0, a1), hi23 = max(a2, a3), lo23 = min(a2, a3);
        const uint32_t top = max(hi01, hi23), second = max(min(hi01, hi23), max(lo01, lo23));
        keep = (8u >> (top & 3u)) | (8u >> (second & 3u));
    } else {
        keep = prune_keep_sequential(ax, ay, inf);
    }
    x &= (keep & 1u) * 0xffffu + (keep & 2u) * 0x7fff8000u;
    y &= ((keep >> 2) & 1u) * 0xffffu + ((keep >> 2) & 2u) * 0x7fff8000u;
}

// Compress one group (test/utils.h:124-146): the first two zeros (+0 or -0)
// are dropped and the rest is kept.  With z the 4-bit mask of zero
// positions, a 16-entry nibble table gives the two kept positions (ia | ib
// << 2, the lower first); fewer than two zeros (z in {0, 1, 2, 4, 8}) keep
// more than two values and make the group invalid.  Returns the kept halves
// (the lower position in the low 16 bits) and the positions in *idx.
__device__ __forceinline__ bool compress_group(uint32_t x, uint32_t y, uint32_t* halves, uint32_t* idx) {
    const uint32_t ax = x & 0x7fff7fffu, ay = y & 0x7fff7fffu;
    const uint32_t z = ((ax & 0xffffu) == 0 ? 1u : 0u) | (ax < 0x10000u ? 2u : 0u) |
                       ((ay & 0xffffu) == 0 ? 4u : 0u) | (ay < 0x10000u ? 8u : 0u);
    const uint32_t id = (uint32_t)(0xECD4E894ECD4E444ull >> (4 * z)) & 0xfu;
    const uint32_t ia = id & 3u, ib = id >> 2;
    *halves = __byte_perm(x, y, ia * 0x22u + ib * 0x2200u + 0x1010u);
    *idx = id;
    return ((0x0117u >> z) & 1u) == 0;
}

// Prune + compress of one group in one step.  Common case (no NaN, both
// kept magnitudes non-zero): the kept positions are the top-2 of the unique
// keys, the two pruned positions are exactly the zeros the compress drops,
// so positions and values come straight from the selection.  Otherwise the
// two steps run as written above.  Same results bit for bit.
__device__ __forceinline__ bool prune_compress_group(uint32_t x, uint32_t y, uint32_t inf, uint32_t* halves,
                                                     uint32_t* idx) {
    const uint32_t ax = x & 0x7fff7fffu, ay = y & 0x7fff7fffu;
    if (no_nan(ax, ay, inf)) {
        const uint32_t a0 = ((ax << 2) & 0x3fffcu) | 3u, a1 = ((ax >> 14) & 0x3fffcu) | 2u;
        const uint32_t a2 = ((ay << 2) & 0x3fffcu) | 1u, a3 = (ay >> 14) & 0x3fffcu;
        const uint32_t hi01 = max(a0, a1), lo01 = min(a0, a1), hi23 = max(a2, a3), lo23 = min(a2, a3);
        const uint32_t top = max(hi01, hi23), second = max(min(hi01, hi23), max(lo01, lo23));
        if (second >= 4u) {  // both kept magnitudes non-zero
            const uint32_t k0 = 3u - (top & 3u), k1 = 3u - (second & 3u);
            const uint32_t ia = min(k0, k1), ib = max(k0, k1);
            *halves = __byte_perm(x, y, ia * 0x22u + ib * 0x2200u + 0x1010u);
            *idx = ia | (ib << 2);
            return true;
        }
    }
    prune_group(x, y, inf);
    return compress_group(x, y, halves, idx);
}

// One CTA: kPackBands 16-row bands x 16 blocks of 16 K.  All of the tile's
// loads are issued before any is used (8 x 16 bytes per thread), so each SM
// keeps about 200 KB of reads in flight.  Thread t then handles row t % 16
// of block t / 16 in every band; per band the value writes (block-major,
// then row) are one contiguous 4 KB run.
constexpr int kPackBands = 4;
constexpr int kLoadsPerThread = kPackBands * 16 * (kTileCols / 8) / kPackThreads;

// One row of a 16 x 16 block (row r of block qg of band `band`), staged in
// shared memory: optional prune, compress, the values and the reordered
// metadata word.  Returns false when a group keeps more than two values.
__device__ __forceinline__ bool pack_row16(const uint16_t* row, int prune, uint16_t* __restrict__ vals,
                                           uint16_t* __restrict__ meta, int band, int qg, int r, int nbc, int K) {
    const uint4 lo = *reinterpret_cast<const uint4*>(row);
    const uint4 hi = *reinterpret_cast<const uint4*>(row + 8);
    uint32_t wx[4] = {lo.x, lo.z, hi.x, hi.z}, wy[4] = {lo.y, lo.w, hi.y, hi.w};
    uint32_t w[4], md = 0;
    bool ok = true;
    if (prune) {
        const uint32_t inf = prune == 2 ? 0x7f80u : 0x7c00u;
        // Row fast path: no NaN in the row's 16 values and both kept
        // magnitudes of every group non-zero -- one test per row instead
        // of two branches per group; otherwise the per-group path.
        const uint32_t add = (0x7fffu - inf) * 0x10001u;
        uint32_t nan_bits = 0, top2[4], sec2[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t ax = wx[k] & 0x7fff7fffu, ay = wy[k] & 0x7fff7fffu;
            nan_bits |= (ax + add) | (ay + add);
            const uint32_t a0 = ((ax << 2) & 0x3fffcu) | 3u, a1 = ((ax >> 14) & 0x3fffcu) | 2u;
            const uint32_t a2 = ((ay << 2) & 0x3fffcu) | 1u, a3 = (ay >> 14) & 0x3fffcu;
            const uint32_t hi01 = max(a0, a1), lo01 = min(a0, a1), hi23 = max(a2, a3), lo23 = min(a2, a3);
            top2[k] = max(hi01, hi23);
            sec2[k] = max(min(hi01, hi23), max(lo01, lo23));
        }
        const uint32_t min_sec = min(min(sec2[0], sec2[1]), min(sec2[2], sec2[3]));
        if ((nan_bits & 0x80008000u) == 0u && min_sec >= 4u) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t k0 = ~top2[k] & 3u, k1 = ~sec2[k] & 3u;  // 3 - (key & 3)
                const uint32_t ia = min(k0, k1), ib = max(k0, k1);
                w[k] = __byte_perm(wx[k], wy[k], ia * 0x22u + ib * 0x2200u + 0x1010u);
                md |= (ia | (ib << 2)) << (4 * k);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                uint32_t idx;
                ok &= prune_compress_group(wx[k], wy[k], inf, &w[k], &idx);
                md |= idx << (4 * k);
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t idx;
            ok &= compress_group(wx[k], wy[k], &w[k], &idx);
            md |= idx << (4 * k);
        }
    }
    *reinterpret_cast<uint4*>(vals + (((size_t)band * nbc + qg) * 16 + r) * 8) = make_uint4(w[0], w[1], w[2], w[3]);
    // Reordered metadata (test/utils.h:179-180): per band and 64-K group,
    // word i*8 + j holds (row (j%2)*8 + i, block j/2 of the group).
    const size_t grp = (size_t)band * (K / 64) + qg / 4;
    meta[grp * 64 + (r % 8) * 8 + 2 * (qg % 4) + r / 8] = (uint16_t)md;
    return ok;
}

__global__ void __launch_bounds__(kPackThreads, 6) pack_a_kernel(const uint16_t* __restrict__ dense, int M, int K,
                                                              int prune, uint16_t* __restrict__ vals,
                                                              uint16_t* __restrict__ meta, int* bad_blocks) {
    __shared__ __align__(16) uint16_t tile[kPackBands * 16 * kTilePitch];
    const int band0 = blockIdx.y * kPackBands;
    const int nb = min(kPackBands, M / 16 - band0);
    const int nbc = K / 16;
    const int q0 = blockIdx.x * kTileBlocks;
    const int nq = min(kTileBlocks, nbc - q0);  // a multiple of 4 (K % 64 == 0)
    const uint16_t* base = dense + (size_t)band0 * 16 * K + (size_t)q0 * 16;
    ptx::grid_dep_wait();  // launched with programmatic serialization: the previous grid may write the input
    if (threadIdx.x == 0) ptx::grid_dep_launch();
    if (nq == kTileBlocks && nb == kPackBands) {  // full tile: 32 chunks of 16 bytes per row
        uint4 v[kLoadsPerThread];
#pragma unroll
        for (int i = 0; i < kLoadsPerThread; ++i) {
            const int c = threadIdx.x + i * kPackThreads;
            v[i] = *reinterpret_cast<const uint4*>(base + (size_t)(c >> 5) * K + (c & 31) * 8);
        }
#pragma unroll
        for (int i = 0; i < kLoadsPerThread; ++i) {
            const int c = threadIdx.x + i * kPackThreads;
            *reinterpret_cast<uint4*>(tile + (c >> 5) * kTilePitch + (c & 31) * 8) = v[i];
        }
    } else {  // ragged tile (last K tile or last bands)
        const int chunks_per_row = nq * 2;
        const int total = nb * 16 * chunks_per_row;
        for (int c = threadIdx.x; c < total; c += kPackThreads) {
            const int r = c / chunks_per_row, x = c % chunks_per_row;
            *reinterpret_cast<uint4*>(tile + r * kTilePitch + x * 8) =
                *reinterpret_cast<const uint4*>(base + (size_t)r * K + x * 8);
        }
    }
    __syncthreads();
    const int q = threadIdx.x / 16, r = threadIdx.x % 16;
    if (q >= nq) return;
    const int qg = q0 + q;
    int bad = 0;
    for (int b = 0; b < nb; ++b)
        bad += pack_row16(tile + (b * 16 + r) * kTilePitch + q * 16, prune, vals, meta, band0 + b, qg, r, nbc, K) ? 0 : 1;
    if (bad && bad_blocks) atomicAdd(bad_blocks, bad);
}

// ------------------------------------------------------------------- fp8
// The same steps on a group of four fp8 bytes held in one 32-bit word (byte
// i = position i).  Magnitudes are b & 0x7f; NaN is every magnitude above
// `top` (0x7e for E4M3, 0x7c for E5M2) and compares false with everything.

// True when none of the four magnitudes is above `top`: adding 0x7f - top
// to each byte carries into its bit 7 exactly when it is above.
__device__ __forceinline__ bool no_nan8(uint32_t a, uint32_t top) {
    return ((a + (0x7fu - top) * 0x01010101u) & 0x80808080u) == 0u;
}

// Kept positions (bit mask) of the sequential prune with NaN rules.
__device__ __forceinline__ uint32_t prune_keep_sequential8(uint32_t a, uint32_t top) {
    uint32_t m[4];
    bool v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = (a >> (8 * i)) & 0xffu;
        v[i] = m[i] <= top;
    }
    uint32_t k0 = 0, mk = m[0];
#pragma unroll
    for (int i = 1; i < 4; ++i) {
        const bool c = v[0] && v[i] && m[i] > mk;  // a NaN at position 0 keeps position 0
        k0 = c ? (uint32_t)i : k0;
        mk = c ? m[i] : mk;
    }
    // k0 is 0 whenever position 0 is NaN; otherwise the comparisons above
    // chained through the current best, which is never NaN.
    uint32_t k1 = k0 == 0 ? 1u : 0u;
    uint32_t mk1 = k0 == 0 ? m[1] : m[0];
    const bool vk1 = k0 == 0 ? v[1] : v[0];
#pragma unroll
    for (int i = 1; i < 4; ++i) {
        const bool c = (uint32_t)i != k0 && (uint32_t)i > k1 && vk1 && v[i] && m[i] > mk1;
        k1 = c ? (uint32_t)i : k1;
        mk1 = c ? m[i] : mk1;
    }
    return (1u << k0) | (1u << k1);
}

// 16-bit-lane max / min (native instructions on sm_90 and later).
__device__ __forceinline__ uint32_t vmax_u16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t vmin_u16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// Top-2 of two groups at once (w0 in the low 16-bit lanes, w1 in the high
// ones): key = magnitude << 8 | (3 - position), the scalar keys' order (ties
// to the lower position) in 16 bits.  Returns the top and second keys; ORs
// each byte + (0x7f - prune_top) into *nan_bits (bit 7 set: a NaN).
__device__ __forceinline__ void top2_pair8(uint32_t w0, uint32_t w1, uint32_t add, uint32_t* nan_bits, uint32_t* top,
                                           uint32_t* sec) {
    const uint32_t a0 = w0 & 0x7f7f7f7fu, a1 = w1 & 0x7f7f7f7fu;
    *nan_bits |= (a0 + add) | (a1 + add);
    const uint32_t even = __byte_perm(a0, a1, 0x6420u), odd = __byte_perm(a0, a1, 0x7531u);
    constexpr uint32_t kTags = 0x00010203u;  // byte j: 3 - j
    const uint32_t k0 = __byte_perm(even, kTags, 0x2404u), k1 = __byte_perm(odd, kTags, 0x2505u);
    const uint32_t k2 = __byte_perm(even, kTags, 0x3616u), k3 = __byte_perm(odd, kTags, 0x3717u);
    const uint32_t hi01 = vmax_u16x2(k0, k1), lo01 = vmin_u16x2(k0, k1);
    const uint32_t hi23 = vmax_u16x2(k2, k3), lo23 = vmin_u16x2(k2, k3);
    *top = vmax_u16x2(hi01, hi23);
    *sec = vmax_u16x2(vmin_u16x2(hi01, hi23), vmax_u16x2(lo01, lo23));
}

// From two groups' top and second keys: the four kept bytes (each group's
// lower position first; w0's in the low half) and the two metadata nibbles
// i0 | i1 << 2 (w0's at bit 0, w1's at bit 16).
__device__ __forceinline__ uint32_t emit_pair8(uint32_t w0, uint32_t w1, uint32_t top, uint32_t sec, uint32_t* nibs) {
    const uint32_t t = top & 0x00030003u, s = sec & 0x00030003u;
    const uint32_t hi = vmax_u16x2(t, s), lo = vmin_u16x2(t, s);  // tags of the lower and the higher position
    // per lane (i0 | i1 << 4), +4 on the high lane's positions (bytes of w1)
    const uint32_t sel = __byte_perm(0x00770033u - (hi | (lo << 4)), 0, 0x4420u);
    *nibs = 0x000f000fu - (hi | (lo << 2));
    return __byte_perm(w0, w1, sel);
}

// Prune + compress of one group: the two kept bytes (lower position first)
// in the low 16 bits of *pair, positions i0 | i1 << 2 in *idx; false when
// the group keeps more than two values.  prune_top: 0 = no prune.
__device__ __forceinline__ bool pack_group8(uint32_t w, uint32_t prune_top, uint32_t* pair, uint32_t* idx) {
    const uint32_t a = w & 0x7f7f7f7fu;
    if (prune_top) {
        uint32_t keep;
        if (no_nan8(a, prune_top)) {
            const uint32_t a0 = ((a << 2) & 0x1fcu) | 3u, a1 = ((a >> 6) & 0x1fcu) | 2u;
            const uint32_t a2 = ((a >> 14) & 0x1fcu) | 1u, a3 = (a >> 22) & 0x1fcu;
            const uint32_t hi01 = max(a0, a1), lo01 = min(a0, a1), hi23 = max(a2, a3), lo23 = min(a2, a3);
            const uint32_t top = max(hi01, hi23), second = max(min(hi01, hi23), max(lo01, lo23));
            if (second >= 4u) {  // both kept magnitudes non-zero: they are the compress's output
                const uint32_t k0 = 3u - (top & 3u), k1 = 3u - (second & 3u);
                const uint32_t ia = min(k0, k1), ib = max(k0, k1);
                *pair = __byte_perm(w, 0, ia | (ib << 4) | 0x4400u);  // bytes 2, 3 from the zero operand
                *idx = ia | (ib << 2);
                return true;
            }
            keep = (8u >> (top & 3u)) | (8u >> (second & 3u));
        } else {
            keep = prune_keep_sequential8(a, prune_top);
        }
        const uint32_t bytes = (keep & 1u) * 0xffu | (keep & 2u) * 0x7f80u | (keep & 4u) * 0x3fc000u |
                               (keep & 8u) * 0x1fe00000u;
        w &= bytes;
    }
    const uint32_t z = ((w & 0x7fu) == 0 ? 1u : 0u) | ((w & 0x7f00u) == 0 ? 2u : 0u) |
                       ((w & 0x7f0000u) == 0 ? 4u : 0u) | ((w & 0x7f000000u) == 0 ? 8u : 0u);
    const uint32_t id = (uint32_t)(0xECD4E894ECD4E444ull >> (4 * z)) & 0xfu;
    *pair = __byte_perm(w, 0, (id & 3u) | ((id >> 2) << 4) | 0x4400u);
    *idx = id;
    return ((0x0117u >> z) & 1u) == 0;
}

// One CTA: kPackBands 16-row bands x 512 bytes of K (16 blocks of 32 K), the
// 16-bit kernel's tile geometry in bytes.  Thread t handles row t % 16 of
// block t / 16 in every band: 32 bytes in, 16 value bytes and 4 metadata
// bytes out.
__global__ void __launch_bounds__(kPackThreads) pack_a_fp8_kernel(const uint8_t* __restrict__ dense, int M, int K,
                                                                  uint32_t prune_top, uint8_t* __restrict__ vals,
                                                                  uint8_t* __restrict__ meta, int* bad_blocks) {
    __shared__ __align__(16) uint8_t tile[kPackBands * 16 * kTilePitch * 2];
    constexpr int kPitch = kTilePitch * 2;  // bytes per staged row (512 + 16)
    const int band0 = blockIdx.y * kPackBands;
    const int nb = min(kPackBands, M / 16 - band0);
    const int nbc = K / 32;                     // 32-K blocks per row
    const int q0 = blockIdx.x * kTileBlocks;
    const int nq = min(kTileBlocks, nbc - q0);  // a multiple of 4 (K % 128 == 0)
    const uint8_t* base = dense + (size_t)band0 * 16 * K + (size_t)q0 * 32;
    ptx::grid_dep_wait();  // launched with programmatic serialization: the previous grid may write the input
    if (threadIdx.x == 0) ptx::grid_dep_launch();
    uint4 v[kLoadsPerThread];
    if (nq == kTileBlocks && nb == kPackBands) {  // full tile: 32 chunks of 16 bytes per row
#pragma unroll
        for (int i = 0; i < kLoadsPerThread; ++i) {
            const int c = threadIdx.x + i * kPackThreads;
            v[i] = *reinterpret_cast<const uint4*>(base + (size_t)(c >> 5) * K + (c & 31) * 16);
        }
#pragma unroll
        for (int i = 0; i < kLoadsPerThread; ++i) {
            const int c = threadIdx.x + i * kPackThreads;
            *reinterpret_cast<uint4*>(tile + (c >> 5) * kPitch + (c & 31) * 16) = v[i];
        }
    } else {
        const int chunks_per_row = nq * 2;
        const int total = nb * 16 * chunks_per_row;
        for (int c = threadIdx.x; c < total; c += kPackThreads) {
            const int r = c / chunks_per_row, x = c % chunks_per_row;
            *reinterpret_cast<uint4*>(tile + r * kPitch + x * 16) =
                *reinterpret_cast<const uint4*>(base + (size_t)r * K + x * 16);
        }
    }
    __syncthreads();
    const int q = threadIdx.x / 16, r = threadIdx.x % 16;
    if (q >= nq) return;
    const int qg = q0 + q;
    int bad = 0;
    for (int b = 0; b < nb; ++b) {
        const uint8_t* row = tile + (b * 16 + r) * kPitch + q * 32;
        const uint4 lo = *reinterpret_cast<const uint4*>(row);
        const uint4 hi = *reinterpret_cast<const uint4*>(row + 16);
        const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        uint32_t pr[8], md = 0;
        bool ok = true;
        // Row fast path (prune on, no NaN in the row's 32 bytes, both kept
        // magnitudes of every group non-zero); otherwise per group.
        bool fast = prune_top != 0;
        uint32_t top4[4], sec4[4];
        if (fast) {
            const uint32_t add = (0x7fu - prune_top) * 0x01010101u;
            uint32_t nan_bits = 0, min_sec = 0xffffffffu;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                top2_pair8(w[2 * k], w[2 * k + 1], add, &nan_bits, &top4[k], &sec4[k]);
                min_sec = vmin_u16x2(min_sec, sec4[k]);
            }
            // no NaN, and every group's second kept magnitude non-zero
            fast = (nan_bits & 0x80808080u) == 0u && (min_sec & 0xff00u) != 0u && (min_sec & 0xff000000u) != 0u;
        }
        uint4 out;
        if (fast) {
            uint32_t nib[4], vw[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) vw[k] = emit_pair8(w[2 * k], w[2 * k + 1], top4[k], sec4[k], &nib[k]);
            const uint32_t n03 = __byte_perm(nib[0], nib[1], 0x6420u), n47 = __byte_perm(nib[2], nib[3], 0x6420u);
            md = __byte_perm(n03, n47, 0x6420u) | (__byte_perm(n03, n47, 0x7531u) << 4);
            out = make_uint4(vw[0], vw[1], vw[2], vw[3]);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                uint32_t idx;
                ok &= pack_group8(w[k], prune_top, &pr[k], &idx);
                md |= idx << (4 * k);
            }
            out = make_uint4(pr[0] | (pr[1] << 16), pr[2] | (pr[3] << 16), pr[4] | (pr[5] << 16), pr[6] | (pr[7] << 16));
        }
        bad += ok ? 0 : 1;
        const int band = band0 + b;
        *reinterpret_cast<uint4*>(vals + (((size_t)band * nbc + qg) * 16 + r) * 16) = out;
        // metadata row (band, 128-K group qg / 4, row r): this block's 32 bits
        *reinterpret_cast<uint32_t*>(meta + (((size_t)band * (K / 128) + qg / 4) * 16 + r) * 16 + (qg % 4) * 4) = md;
    }
    if (bad && bad_blocks) atomicAdd(bad_blocks, bad);
}

// In-place magnitude prune, one group of four per thread.
__global__ void __launch_bounds__(kPackThreads) prune_kernel(uint16_t* __restrict__ a, long long groups, uint32_t inf) {
    for (long long g = blockIdx.x * (long long)kPackThreads + threadIdx.x; g < groups;
         g += (long long)gridDim.x * kPackThreads) {
        uint2 w = *reinterpret_cast<uint2*>(a + 4 * g);
        prune_group(w.x, w.y, inf);
        *reinterpret_cast<uint2*>(a + 4 * g) = w;
    }
}

// One CTA: 64 K rows x 64 columns (8 strips).  Reads row segments of 128
// bytes, writes each strip's 64 rows as one contiguous 1 KB run.
__global__ void __launch_bounds__(kPackThreads) pack_b_kernel(const uint16_t* __restrict__ b, int K, int N,
                                                              uint16_t* __restrict__ out) {
    __shared__ __align__(16) uint16_t tile[kBTileRows * kBTilePitch];
    const int k0 = blockIdx.y * kBTileRows;
    const int n0 = blockIdx.x * kBTileCols;
    const bool vec = (N % 8 == 0) && ((reinterpret_cast<uintptr_t>(b) & 15u) == 0);
    ptx::grid_dep_wait();  // launched with programmatic serialization: the previous grid may write B or read out
    if (threadIdx.x == 0) ptx::grid_dep_launch();
    for (int c = threadIdx.x; c < kBTileRows * (kBTileCols / 8); c += kPackThreads) {
        const int r = c / (kBTileCols / 8), x = c % (kBTileCols / 8);
        const int n = n0 + x * 8;
        const uint16_t* src = b + (size_t)(k0 + r) * N + n;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (vec) {
            if (n < N) v = *reinterpret_cast<const uint4*>(src);
        } else {
            __align__(16) uint16_t h[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) h[e] = (n + e < N) ? src[e] : (uint16_t)0;
            v = *reinterpret_cast<const uint4*>(h);
        }
        *reinterpret_cast<uint4*>(tile + r * kBTilePitch + x * 8) = v;
    }
    __syncthreads();
    const int strips = (N + 7) / 8;
    for (int c = threadIdx.x; c < kBTileRows * (kBTileCols / 8); c += kPackThreads) {
        const int s = c / kBTileRows, r = c % kBTileRows;
        const int strip = n0 / 8 + s;
        if (strip >= strips) continue;
        *reinterpret_cast<uint4*>(out + ((size_t)strip * K + k0 + r) * 8) =
            *reinterpret_cast<const uint4*>(tile + r * kBTilePitch + s * 8);
    }
}

bool misaligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

// Launches a packer kernel with programmatic stream serialization: its CTAs
// may be scheduled while the previous kernel in the stream finishes (each
// waits for that grid before reading), which hides the launch gap between
// back-to-back packer calls.
template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kPackThreads, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace
}  // namespace spmm24

extern "C" cudaError_t spmm24_pack_a_device(cudaStream_t stream, const void* dense_a, int M, int K, int prune,
                                            void* values_out, uint16_t* meta_out, int* bad_blocks) {
    using namespace spmm24;
    clear_last_error();
    if (!dense_a || !values_out || !meta_out) return record_invalid("null pointer");
    if (M <= 0 || K <= 0 || M % 16 || K % 64) return record_invalid("M must be a multiple of 16 and K of 64");
    if (misaligned16(dense_a) || misaligned16(values_out)) return record_invalid("dense A and values must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(meta_out) & 1u) || (reinterpret_cast<uintptr_t>(bad_blocks) & 3u))
        return record_invalid("metadata must be 2-byte and bad_blocks 4-byte aligned");
    const int nbc = K / 16;
    dim3 grid((unsigned)((nbc + kTileBlocks - 1) / kTileBlocks), (unsigned)((M / 16 + kPackBands - 1) / kPackBands));
    if (grid.y > 65535) return record_invalid("M too large");
    if (prune < SPMM24_PRUNE_NONE || prune > SPMM24_PRUNE_BF16) return record_invalid("unknown prune mode");
    return launch_pdl(pack_a_kernel, grid, stream, static_cast<const uint16_t*>(dense_a), M, K, prune,
                      static_cast<uint16_t*>(values_out), meta_out, bad_blocks);
}

extern "C" cudaError_t spmm24_pack_a_fp8_device(cudaStream_t stream, const void* dense_a, int M, int K, int prune,
                                                void* values_out, void* meta_out, int* bad_blocks) {
    using namespace spmm24;
    clear_last_error();
    if (!dense_a || !values_out || !meta_out) return record_invalid("null pointer");
    if (M <= 0 || K <= 0 || M % 16 || K % 128) return record_invalid("M must be a multiple of 16 and K of 128");
    if (misaligned16(dense_a) || misaligned16(values_out) || misaligned16(meta_out))
        return record_invalid("dense A, values and metadata must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(bad_blocks) & 3u) return record_invalid("bad_blocks must be 4-byte aligned");
    if (prune < 0 || prune > 2) return record_invalid("prune: 0 none, 1 E4M3, 2 E5M2");
    const int nbc = K / 32;
    dim3 grid((unsigned)((nbc + kTileBlocks - 1) / kTileBlocks), (unsigned)((M / 16 + kPackBands - 1) / kPackBands));
    if (grid.y > 65535) return record_invalid("M too large");
    const uint32_t top = prune == 1 ? 0x7eu : prune == 2 ? 0x7cu : 0u;
    return launch_pdl(pack_a_fp8_kernel, grid, stream, static_cast<const uint8_t*>(dense_a), M, K, top,
                      static_cast<uint8_t*>(values_out), static_cast<uint8_t*>(meta_out), bad_blocks);
}

namespace spmm24 {
namespace {
cudaError_t prune_device(cudaStream_t stream, void* dense_a, int M, int K, uint32_t inf) {
    clear_last_error();
    if (!dense_a) return record_invalid("null pointer");
    if (M <= 0 || K <= 0 || K % 4) return record_invalid("M must be positive and K a multiple of 4");
    if (reinterpret_cast<uintptr_t>(dense_a) & 7u) return record_invalid("dense A must be 8-byte aligned");
    const long long groups = (long long)M * K / 4;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long want = (groups + kPackThreads - 1) / kPackThreads;
    const unsigned blocks = (unsigned)(want < (long long)sms * 16 ? want : (long long)sms * 16);
    prune_kernel<<<blocks, kPackThreads, 0, stream>>>(static_cast<uint16_t*>(dense_a), groups, inf);
    return cudaGetLastError();
}
}  // namespace
}  // namespace spmm24

extern "C" cudaError_t spmm24_prune_2of4_device(cudaStream_t stream, void* dense_a, int M, int K) {
    return spmm24::prune_device(stream, dense_a, M, K, 0x7c00u);
}

extern "C" cudaError_t spmm24_prune_2of4_bf16_device(cudaStream_t stream, void* dense_a, int M, int K) {
    return spmm24::prune_device(stream, dense_a, M, K, 0x7f80u);
}

extern "C" cudaError_t spmm24_pack_b_device(cudaStream_t stream, const void* b_rowmajor, int K, int N,
                                            void* b_packed_out) {
    using namespace spmm24;
    clear_last_error();
    if (!b_rowmajor || !b_packed_out) return record_invalid("null pointer");
    if (K <= 0 || N <= 0 || K % 64) return record_invalid("K must be a positive multiple of 64");
    if (misaligned16(b_packed_out)) return record_invalid("packed B must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(b_rowmajor) & 1u) return record_invalid("B must be 2-byte aligned");
    if (K / kBTileRows > 65535) return record_invalid("K too large");
    dim3 grid((unsigned)((N + kBTileCols - 1) / kBTileCols), (unsigned)(K / kBTileRows));
    return launch_pdl(pack_b_kernel, grid, stream, static_cast<const uint16_t*>(b_rowmajor), K, N,
                      static_cast<uint16_t*>(b_packed_out));
}
