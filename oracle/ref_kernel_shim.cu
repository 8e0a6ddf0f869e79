// Shim that exposes the reference's own SpMM launcher (SpeakOutLoudly/CUDA-Repo
// src/SpMM_API.cu:61-171, kernel src/SpMM_Kernel.cuh:301-492) compiled for
// sm_100a, as a GPU parity target and a same-box comparator.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile from the reference
// sources where they lie (-I<reference>/src); output goes to oracle/_ref/.
// The reference kernel only dispatches N in {8,16,32,64,128} and reads past
// its K range when (Split_K-1)*ceil(K/64/Split_K) > K/64, so callers must
// stay inside those limits (ref_spmm_supported checks them).
#include <cstdint>
#include "SpMM_API.cu"

extern "C" int ref_spmm_supported(int M, int N, int K, int split_k) {
    if (split_k < 1 || K % 64) return 0;
    int tile_m;
    switch (N) {
        case 8: case 16: case 32: case 64: tile_m = 64; break;
        case 128: tile_m = 128; break;
        default: return 0;
    }
    if (M % tile_m) return 0;
    int kt = K / 64;
    int avg = (kt - 1) / split_k + 1;
    if ((split_k - 1) * avg > kt) return 0;
    if (split_k > 1 && ((long)M * N) % 256) return 0;
    return 1;
}

extern "C" int ref_spmm_launch(void* stream, const void* a, const void* b, const uint16_t* meta, void* c, int M, int N,
                               int K, void* ws, int split_k) {
    if (!ref_spmm_supported(M, N, K, split_k)) return (int)cudaErrorInvalidValue;
    return (int)SpMM_N2M4_Launch((cudaStream_t)stream, (const half*)a, (const half*)b, meta, (half*)c, M, N, K,
                                 (half*)ws, split_k);
}
