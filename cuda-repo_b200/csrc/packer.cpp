// packer.cpp -- host-side 2:4 prune / compress / metadata / B-packing.
//
// Bit-exact with the reference's host packer (SpeakOutLoudly/CUDA-Repo
// test/utils.h:91-229) for every valid 2:4-sparse input; large matrices are
// processed band-parallel on the host threads.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include <cuda_fp16.h>

#include "spmm24/SpMM_API.h"

namespace {

// Runs fn(begin, end) over [0, n) split across host threads when the work is
// large enough to amortise thread start-up.
template <class F>
void parallel_for(int n, long work_per_item, F fn) {
    unsigned hw = std::thread::hardware_concurrency();
    long total = (long)n * work_per_item;
    int nthreads = (int)std::min<long>(std::max(1u, hw), std::max(1L, total / (1L << 20)));
    nthreads = std::min(nthreads, n);
    if (nthreads <= 1) {
        fn(0, n);
        return;
    }
    std::vector<std::thread> pool;
    int chunk = (n + nthreads - 1) / nthreads;
    for (int t = 0; t < nthreads; ++t) {
        int b = t * chunk, e = std::min(n, b + chunk);
        if (b >= e) break;
        pool.emplace_back(fn, b, e);
    }
    for (auto& th : pool) th.join();
}

inline bool is_zero(uint16_t h) { return (h & 0x7fffu) == 0; }

inline float h2f(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

// One 16x16 block row: the reference's per-row walk (test/utils.h:124-146).
// Returns false when a group of four holds fewer than two zeros.
inline bool compress_row16(const uint16_t* src, uint16_t* vals, uint16_t* meta_word) {
    uint32_t md = 0;
    int kept = 0;
    for (int g = 0; g < 16; g += 4) {
        int zeros = 0, kept_here = 0;
        for (int o = 0; o < 4; ++o) {
            uint16_t v = src[g + o];
            if (zeros < 2 && is_zero(v)) {
                ++zeros;
                continue;
            }
            if (kept_here == 2) return false;
            vals[kept] = v;
            md |= (uint32_t)o << (2 * kept);
            ++kept;
            ++kept_here;
        }
    }
    *meta_word = (uint16_t)md;
    return true;
}

}  // namespace

extern "C" int spmm24_compress_a(const uint16_t* dense, int M, int K, uint16_t* vals, uint16_t* meta) {
    if (!dense || !vals || !meta || M <= 0 || K <= 0 || M % 16 || K % 16) return -1;
    const int nbc = K / 16;
    std::vector<char> bad((size_t)(M / 16), 0);
    parallel_for(M / 16, (long)16 * K, [&](int b0, int b1) {
        for (int br = b0; br < b1; ++br)
            for (int bc = 0; bc < nbc; ++bc)
                for (int r = 0; r < 16; ++r) {
                    size_t blk = ((size_t)br * nbc + bc) * 16 + r;
                    const uint16_t* src = dense + (size_t)(br * 16 + r) * K + (size_t)bc * 16;
                    if (!compress_row16(src, vals + blk * 8, meta + blk)) {
                        bad[br] = 1;
                        return;
                    }
                }
    });
    for (char b : bad)
        if (b) return -2;
    return (int)((size_t)M * K / 2);
}

extern "C" int spmm24_reorder_metadata(const uint16_t* in, int M, int K, uint16_t* out) {
    if (!in || !out || M <= 0 || K <= 0 || M % 16 || K % 64) return -1;
    const size_t groups = (size_t)M / 16 * (K / 64);
    // Per 64 words: out[i*8+j] = in[(j%2)*8 + (j/2)*16 + i] (test/utils.h:179-180).
    for (size_t g = 0; g < groups; ++g) {
        const uint16_t* s = in + g * 64;
        uint16_t* d = out + g * 64;
        for (int i = 0; i < 8; ++i)
            for (int j = 0; j < 8; ++j) d[i * 8 + j] = s[(j & 1) * 8 + (j >> 1) * 16 + i];
    }
    return 0;
}

extern "C" int spmm24_compress_reordered(const uint16_t* dense, int M, int K, uint16_t* vals, uint16_t* meta) {
    if (!dense || !vals || !meta || M <= 0 || K <= 0 || M % 16 || K % 64) return -1;
    std::vector<uint16_t> raw((size_t)M * K / 16);
    int n = spmm24_compress_a(dense, M, K, vals, raw.data());
    if (n < 0) return n;
    spmm24_reorder_metadata(raw.data(), M, K, meta);
    return n;
}

extern "C" int spmm24_pack_b(const uint16_t* b, int K, int N, uint16_t* out) {
    if (!b || !out || K <= 0 || N <= 0 || K % 64) return -1;
    const int strips = (N + 7) / 8;
    parallel_for(strips, (long)8 * K, [&](int s0, int s1) {
        for (int s = s0; s < s1; ++s) {
            uint16_t* d = out + (size_t)s * K * 8;
            for (int k = 0; k < K; ++k)
                for (int c = 0; c < 8; ++c) {
                    int n = s * 8 + c;
                    d[(size_t)k * 8 + c] = (n < N) ? b[(size_t)k * N + n] : (uint16_t)0;
                }
        }
    });
    return 0;
}

namespace {

inline float bf2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

template <float (*Decode)(uint16_t)>
int prune_rows(uint16_t* a, int M, int K) {
    if (!a || M <= 0 || K <= 0 || K % 4) return -1;
    parallel_for(M, K, [&](int m0, int m1) {
        for (int m = m0; m < m1; ++m) {
            uint16_t* row = a + (size_t)m * K;
            for (int g = 0; g < K; g += 4) {
                float v[4];
                for (int i = 0; i < 4; ++i) v[i] = std::fabs(Decode(row[g + i]));
                int k0 = 0;
                for (int i = 1; i < 4; ++i)
                    if (v[i] > v[k0]) k0 = i;
                int k1 = -1;
                for (int i = 0; i < 4; ++i) {
                    if (i == k0) continue;
                    if (k1 < 0 || v[i] > v[k1]) k1 = i;
                }
                for (int i = 0; i < 4; ++i)
                    if (i != k0 && i != k1) row[g + i] = 0;
            }
        }
    });
    return 0;
}

}  // namespace

extern "C" int spmm24_prune_2of4(uint16_t* a, int M, int K) { return prune_rows<h2f>(a, M, K); }

extern "C" int spmm24_prune_2of4_bf16(uint16_t* a, int M, int K) { return prune_rows<bf2f>(a, M, K); }

// ------------------------------------------------------------------- fp8
// OCP fp8 bytes (E4M3: fmt 0, E5M2: fmt 1).  For both, |x| of a non-NaN
// byte orders like the 7-bit integer b & 0x7f; NaN is every magnitude above
// the largest non-NaN pattern (0x7e for E4M3, whose only NaN is 0x7f; the
// infinity 0x7c for E5M2) and compares false with everything, as the float
// comparisons of the 16-bit prune do.
namespace {

inline bool fp8_gt(uint32_t a, uint32_t b, uint32_t top) { return a <= top && b <= top && a > b; }

int prune_rows_fp8(uint8_t* a, int M, int K, int fmt) {
    if (!a || M <= 0 || K <= 0 || K % 4 || (fmt != 0 && fmt != 1)) return -1;
    const uint32_t top = fmt == 0 ? 0x7eu : 0x7cu;
    parallel_for(M, K, [&](int m0, int m1) {
        for (int m = m0; m < m1; ++m) {
            uint8_t* row = a + (size_t)m * K;
            for (int g = 0; g < K; g += 4) {
                uint32_t v[4];
                for (int i = 0; i < 4; ++i) v[i] = row[g + i] & 0x7fu;
                int k0 = 0;
                for (int i = 1; i < 4; ++i)
                    if (fp8_gt(v[i], v[k0], top)) k0 = i;
                int k1 = -1;
                for (int i = 0; i < 4; ++i) {
                    if (i == k0) continue;
                    if (k1 < 0 || fp8_gt(v[i], v[k1], top)) k1 = i;
                }
                for (int i = 0; i < 4; ++i)
                    if (i != k0 && i != k1) row[g + i] = 0;
            }
        }
    });
    return 0;
}

}  // namespace

extern "C" int spmm24_prune_2of4_fp8(uint8_t* a, int M, int K, int fmt) { return prune_rows_fp8(a, M, K, fmt); }

// Values: band b, 32-K block q, row r -> 16 bytes at ((b*K/32 + q)*16 + r)*16.
// Metadata: band b, 128-K group g, row r -> 16 bytes at ((b*K/128 + g)*16 +
// r)*16, nibble c = group of four at K 128g + 4c (i0 | i1 << 2, i0 < i1).
// Compress rule of the 16-bit packer (test/utils.h:124-146) on bytes.
extern "C" int spmm24_compress_a_fp8(const uint8_t* dense, int M, int K, uint8_t* vals, uint8_t* meta) {
    if (!dense || !vals || !meta || M <= 0 || K <= 0 || M % 16 || K % 128) return -1;
    const int blocks = K / 32, groups = K / 128;
    std::vector<char> bad((size_t)(M / 16), 0);
    parallel_for(M / 16, (long)16 * K, [&](int b0, int b1) {
        for (int band = b0; band < b1 && !bad[band]; ++band)
            for (int r = 0; r < 16; ++r) {
                const uint8_t* src = dense + (size_t)(band * 16 + r) * K;
                for (int g = 0; g < groups; ++g) {
                    uint8_t md[16] = {};
                    for (int c = 0; c < 32; ++c) {
                        const int k = g * 128 + 4 * c;
                        int zeros = 0, kept = 0;
                        uint32_t nib = 0;
                        uint8_t* dst = vals + (((size_t)band * blocks + k / 32) * 16 + r) * 16 + (k % 32) / 2;
                        for (int o = 0; o < 4; ++o) {
                            const uint8_t x = src[k + o];
                            if (zeros < 2 && (x & 0x7fu) == 0) {
                                ++zeros;
                                continue;
                            }
                            if (kept == 2) {
                                bad[band] = 1;
                                return;
                            }
                            dst[kept] = x;
                            nib |= (uint32_t)o << (2 * kept);
                            ++kept;
                        }
                        md[c / 2] |= (uint8_t)(nib << (4 * (c & 1)));
                    }
                    std::memcpy(meta + (((size_t)band * groups + g) * 16 + r) * 16, md, 16);
                }
            }
    });
    for (char b : bad)
        if (b) return -2;
    return (int)((size_t)M * K / 2);
}

// ------------------------------------------------- C++ reference drop-ins
int toolCompressMatrixA(half* denseMatrixA, int Global_M, int Global_K, int Block_M, int Block_K,
                        half** compressedMatrixA, uint16_t** matadata) {
    if (!compressedMatrixA || !matadata) return -1;
    *compressedMatrixA = nullptr;
    *matadata = nullptr;
    if (Block_M != 16 || Block_K != 16 || Global_M <= 0 || Global_K <= 0 || Global_M % 16 || Global_K % 16)
        return -1;
    auto* v = static_cast<uint16_t*>(std::malloc(sizeof(uint16_t) * (size_t)Global_M * Global_K / 2));
    auto* m = static_cast<uint16_t*>(std::malloc(sizeof(uint16_t) * (size_t)Global_M * Global_K / 16));
    if (!v || !m) {
        std::free(v);
        std::free(m);
        return -1;
    }
    int n = spmm24_compress_a(reinterpret_cast<const uint16_t*>(denseMatrixA), Global_M, Global_K, v, m);
    if (n < 0) {
        std::free(v);
        std::free(m);
        return n;
    }
    *compressedMatrixA = reinterpret_cast<half*>(v);
    *matadata = m;
    return n;
}

void toolReorderMetadata(uint16_t* matadata, int Global_M, int Global_K, int Block_M, int Block_K,
                         uint16_t** reorderMatadata) {
    if (!reorderMatadata) return;
    *reorderMatadata = nullptr;
    if (Block_M != 16 || Block_K != 16 || Global_M <= 0 || Global_K <= 0 || Global_M % 16 || Global_K % 64) return;
    auto* o = static_cast<uint16_t*>(std::malloc(sizeof(uint16_t) * (size_t)Global_M * Global_K / 16));
    if (!o) return;
    spmm24_reorder_metadata(matadata, Global_M, Global_K, o);
    *reorderMatadata = o;
}

void toolPackMatrixB(half* MatrixB, int Global_K, int Global_N, int Block_K, int Block_N, half** packMatrixB) {
    if (!packMatrixB) return;
    *packMatrixB = nullptr;
    if (Block_K != 64 || Block_N != 8 || Global_K <= 0 || Global_N <= 0 || Global_K % 64 || Global_N % 8) return;
    auto* o = static_cast<uint16_t*>(std::malloc(sizeof(uint16_t) * (size_t)Global_K * Global_N));
    if (!o) return;
    spmm24_pack_b(reinterpret_cast<const uint16_t*>(MatrixB), Global_K, Global_N, o);
    *packMatrixB = reinterpret_cast<half*>(o);
}

extern "C" int spmm24_shard_rows(int M, int parts, int index, int align, int* row_begin, int* row_end) {
    if (!row_begin || !row_end || M <= 0 || M % 16 || parts <= 0 || index < 0 || index >= parts || align <= 0 ||
        align % 16)
        return -1;
    // Whole `align`-row units, spread as evenly as possible.  The final unit
    // may be partial (M need only be a multiple of 16), so the shards that
    // take one unit more are the last ones, the partial unit among them.
    const long long units = ((long long)M + align - 1) / align;
    const long long base = units / parts, rem = units % parts;
    const long long first_big = parts - rem;  // shards [first_big, parts) get base + 1 units
    const long long u0 = index * base + std::max<long long>(0, index - first_big);
    const long long u1 = u0 + base + (index >= first_big ? 1 : 0);
    *row_begin = (int)std::min<long long>(u0 * align, M);
    *row_end = (int)std::min<long long>(u1 * align, M);
    return 0;
}
