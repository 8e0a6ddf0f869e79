// packed_io.cpp -- a file format for packed 2:4 weights, so a model's layers
// are pruned and packed once and loaded directly in the SpMM's formats.
//
// Layout (little-endian, 64-byte header, then the payload):
//   0  char[8]  magic "SPMM24W" + NUL
//   8  u32      version (1)
//  12  u32      dtype (0 fp16, 1 bf16, 2 fp8 E4M3, 3 fp8 E5M2)
//  16  u32      M
//  20  u32      K
//  24  u64      values_bytes  (16-bit: M*K/2 elements * 2 bytes = M*K; fp8: M*K/2)
//  32  u64      meta_bytes    (M*K/8 for every dtype)
//  40  u64      checksum      (FNV-1a 64 over values then metadata)
//  48  u8[16]   reserved (zero)
//  64  values (compressed, 16x8 blocks, band-major), then metadata (reordered;
//      fp8: the fp8 SpMM's value and metadata formats)
// The reference has no file format (its packer runs per process,
// test/utils.h:91-185).
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "spmm24/SpMM_API.h"

namespace {

constexpr char kMagic[8] = {'S', 'P', 'M', 'M', '2', '4', 'W', '\0'};
constexpr uint32_t kVersion = 1;
constexpr size_t kHeaderBytes = 64;

// FNV-1a, 64-bit (Fowler, Noll, Vo): offset basis and prime of the
// published algorithm.
uint64_t fnv1a64(uint64_t h, const void* data, size_t n) {
    const uint8_t* p = static_cast<const uint8_t*>(data);
    for (size_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}
constexpr uint64_t kFnvBasis = 14695981039346656037ull;

void put32(uint8_t* p, uint32_t v) {
    for (int i = 0; i < 4; ++i) p[i] = (uint8_t)(v >> (8 * i));
}
void put64(uint8_t* p, uint64_t v) {
    for (int i = 0; i < 8; ++i) p[i] = (uint8_t)(v >> (8 * i));
}
uint32_t get32(const uint8_t* p) {
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) v |= (uint32_t)p[i] << (8 * i);
    return v;
}
uint64_t get64(const uint8_t* p) {
    uint64_t v = 0;
    for (int i = 0; i < 8; ++i) v |= (uint64_t)p[i] << (8 * i);
    return v;
}

bool is_fp8(long long dtype) { return dtype == 2 || dtype == 3; }

bool shape_ok(long long dtype, long long M, long long K) {
    return dtype >= 0 && dtype <= 3 && M > 0 && K > 0 && M % 16 == 0 && K % (is_fp8(dtype) ? 128 : 64) == 0;
}

uint64_t values_bytes(long long dtype, long long M, long long K) {
    return is_fp8(dtype) ? (uint64_t)M * K / 2 : (uint64_t)M * K;
}

int read_header(FILE* f, spmm24_packed_header* h) {
    uint8_t b[kHeaderBytes];
    if (std::fread(b, 1, kHeaderBytes, f) != kHeaderBytes) return SPMM24_PACKED_EIO;
    if (std::memcmp(b, kMagic, 8) != 0) return SPMM24_PACKED_EFORMAT;
    h->version = get32(b + 8);
    h->dtype = get32(b + 12);
    h->M = get32(b + 16);
    h->K = get32(b + 20);
    h->values_bytes = get64(b + 24);
    h->meta_bytes = get64(b + 32);
    h->checksum = get64(b + 40);
    if (h->version != kVersion || !shape_ok((int)h->dtype, h->M, h->K)) return SPMM24_PACKED_EFORMAT;
    if (h->values_bytes != values_bytes(h->dtype, h->M, h->K) || h->meta_bytes != (uint64_t)h->M * h->K / 8)
        return SPMM24_PACKED_EFORMAT;
    return 0;
}

}  // namespace

extern "C" int spmm24_save_packed(const char* path, int dtype, int M, int K, const void* values, const void* meta) {
    if (!path || !values || !meta || !shape_ok(dtype, M, K)) return SPMM24_PACKED_EARG;
    const uint64_t vb = values_bytes(dtype, M, K), mb = (uint64_t)M * K / 8;
    uint64_t sum = fnv1a64(kFnvBasis, values, vb);
    sum = fnv1a64(sum, meta, mb);
    uint8_t b[kHeaderBytes] = {};
    std::memcpy(b, kMagic, 8);
    put32(b + 8, kVersion);
    put32(b + 12, (uint32_t)dtype);
    put32(b + 16, (uint32_t)M);
    put32(b + 20, (uint32_t)K);
    put64(b + 24, vb);
    put64(b + 32, mb);
    put64(b + 40, sum);
    FILE* f = std::fopen(path, "wb");
    if (!f) return SPMM24_PACKED_EIO;
    const bool ok = std::fwrite(b, 1, kHeaderBytes, f) == kHeaderBytes && std::fwrite(values, 1, vb, f) == vb &&
                    std::fwrite(meta, 1, mb, f) == mb;
    const bool closed = std::fclose(f) == 0;
    return ok && closed ? 0 : SPMM24_PACKED_EIO;
}

extern "C" int spmm24_load_packed_header(const char* path, spmm24_packed_header* out) {
    if (!path || !out) return SPMM24_PACKED_EARG;
    FILE* f = std::fopen(path, "rb");
    if (!f) return SPMM24_PACKED_EIO;
    const int rc = read_header(f, out);
    std::fclose(f);
    return rc;
}

extern "C" int spmm24_load_packed(const char* path, void* values, size_t values_capacity, void* meta,
                                  size_t meta_capacity) {
    if (!path || !values || !meta) return SPMM24_PACKED_EARG;
    FILE* f = std::fopen(path, "rb");
    if (!f) return SPMM24_PACKED_EIO;
    spmm24_packed_header h;
    int rc = read_header(f, &h);
    // The payload sizes come from the header read here, which may differ from
    // an earlier spmm24_load_packed_header call if the file was replaced in
    // between: nothing is read unless both buffers can hold it.
    if (rc == 0 && (h.values_bytes > values_capacity || h.meta_bytes > meta_capacity)) rc = SPMM24_PACKED_ECAPACITY;
    if (rc == 0) {
        if (std::fread(values, 1, h.values_bytes, f) != h.values_bytes ||
            std::fread(meta, 1, h.meta_bytes, f) != h.meta_bytes)
            rc = SPMM24_PACKED_EIO;
        else if (std::fgetc(f) != EOF)
            rc = SPMM24_PACKED_EFORMAT;  // trailing bytes
    }
    std::fclose(f);
    if (rc != 0) return rc;
    uint64_t sum = fnv1a64(kFnvBasis, values, h.values_bytes);
    sum = fnv1a64(sum, meta, h.meta_bytes);
    return sum == h.checksum ? 0 : SPMM24_PACKED_ECHECKSUM;
}
