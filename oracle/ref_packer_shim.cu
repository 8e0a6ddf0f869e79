// Shim that exposes the reference's own host packer and data generator
// (SpeakOutLoudly/CUDA-Repo test/utils.h:38-66, :91-150, :155-185, :188-229)
// through plain extern "C" entry points, so tests can compare the oracle's
// restatement with the reference byte for byte.
//
// TEST INFRASTRUCTURE ONLY.  It is compiled by oracle/Makefile directly
// against the reference's header where it lies (-I<reference>/test); the
// output goes to oracle/_ref/ and nothing of the reference is copied here.
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <cublas_v2.h>
#include "utils.h"

extern "C" int ref_compress_a(const uint16_t* dense, int M, int K, uint16_t* vals_out, uint16_t* meta_out) {
    half* v = nullptr;
    uint16_t* m = nullptr;
    // toolCompressMatrixA takes a non-const pointer but only reads it.
    int count = toolCompressMatrixA(reinterpret_cast<half*>(const_cast<uint16_t*>(dense)), M, K, 16, 16, &v, &m);
    if (count >= 0) {
        std::memcpy(vals_out, v, sizeof(uint16_t) * (size_t)count);
        std::memcpy(meta_out, m, sizeof(uint16_t) * (size_t)M * K / 16);
    }
    std::free(v);
    std::free(m);
    return count;
}

extern "C" void ref_reorder_metadata(const uint16_t* meta, int M, int K, uint16_t* out) {
    uint16_t* o = nullptr;
    toolReorderMetadata(const_cast<uint16_t*>(meta), M, K, 16, 16, &o);
    std::memcpy(out, o, sizeof(uint16_t) * (size_t)M * K / 16);
    std::free(o);
}

extern "C" void ref_pack_b(const uint16_t* b, int K, int N, uint16_t* out) {
    half* o = nullptr;
    toolPackMatrixB(reinterpret_cast<half*>(const_cast<uint16_t*>(b)), K, N, 64, 8, &o);
    std::memcpy(out, o, sizeof(uint16_t) * (size_t)K * N);
    std::free(o);
}

// The reference generator draws its 2:4 mask from glibc rand() in its default
// state; srand(1) restores that state so repeated calls give the same matrix.
extern "C" void ref_init_pruned(uint16_t* a, int M, int K) {
    srand(1);
    init_host_matrices_pruned(reinterpret_cast<half*>(a), M, K);
}
