/*
 * SpMM_API.h -- public interface of libspmm24, the sm_100a (B200) 2:4
 * structured-sparse fp16 SpMM library: C = A_sparse * B.
 *
 * Drop-in for SpeakOutLoudly/CUDA-Repo's SpMM_N2M4_Launch path.  Every entry
 * point below names the reference interface it replaces (file:line within
 * that project).  Two bindings are provided:
 *
 *   - extern "C" entry points (spmm24_*) with plain pointers and sizes, for
 *     C, ctypes, cgo, JNI or any other FFI;
 *   - C++ declarations with exactly the reference's names and parameter
 *     types, so existing C++ callers link against the same mangled symbols
 *     (e.g. _Z16SpMM_N2M4_LaunchP11CUstream_stPK6__halfS3_PKtPS1_iiiS6_i).
 *
 * Data formats (identical to the reference's):
 *   compressed A   M*K/2 fp16 values in 16x8 blocks: band b (16 rows), 16-K
 *                  block q, row r -> 8 values at ((b*(K/16)+q)*16+r)*8
 *                  (test/utils.h:114-147)
 *   metadata       M*K/16 uint16 words, the reference's reordered layout
 *                  (test/utils.h:155-185): per band and 64-K group, word
 *                  [i*8+j] holds row i+8*(j%2), 16-K block j/2; each word
 *                  has eight 2-bit in-group indices, lowest bits first
 *   packed B       ceil(N/8) strips, each K x 8 fp16 row-major
 *                  (test/utils.h:188-229); for N % 8 != 0 the last strip is
 *                  padded (pad values never reach C)
 *   C              M x N fp16, row-major
 * Shape rules: M % 16 == 0, K % 64 == 0, N >= 1.  A, B and metadata must be
 * 16-byte aligned device pointers; C must be 2-byte aligned.
 */
#ifndef SPMM24_SPMM_API_H
#define SPMM24_SPMM_API_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Launches C = A_sparse * B on `stream`, asynchronously.
 * Replaces SpMM_N2M4_Launch (src/SpMM_API.cu:61-171).
 *   split_k   0 lets the library choose the decomposition from the shape;
 *             1..8 requests that many K slices (clamped to the number of
 *             128-wide K stages).  Values above 8 are treated as 8.  The K
 *             slices of a tile run as one thread-block cluster and their fp32
 *             partial sums are reduced on chip.  The result does not depend
 *             on split_k beyond fp32 summation order, and is bitwise
 *             reproducible for a fixed split_k on a fixed GPU.
 *   split_reduction  accepted for ABI compatibility and never touched, so it
 *             may be NULL.
 * Memory: this call allocates nothing and keeps no workspace.  Encoded TMA
 * descriptors are cached per host thread (64 entries), so repeated calls on
 * the same buffers skip the driver's encoder.
 * The kernel is launched with programmatic stream serialization: it may
 * start its set-up while the previous kernel in the stream finishes, and
 * waits for that kernel before touching global memory.
 * Returns cudaSuccess, cudaErrorInvalidValue (bad pointer, alignment or
 * shape -- the reference silently did nothing for unsupported N), or the
 * CUDA error of the allocation or launch. */
cudaError_t spmm24_launch(cudaStream_t stream, const void* compressed_a, const void* b_packed,
                          const uint16_t* metadata, void* c, int M, int N, int K, void* split_reduction,
                          int split_k);

/* Flags of spmm24_launch_ex. */
enum {
    /* Nothing earlier in the stream writes A or the metadata: the kernel may
     * start streaming the weights before the previous kernel has finished
     * (the activations B are still read only after it). */
    SPMM24_STATIC_WEIGHTS = 1u,
    /* Launch without programmatic stream serialization. */
    SPMM24_NO_PDL = 2u,
    /* A, B and C (and the epilogue's bias and residual) hold bf16 instead of
     * fp16; same layouts (the packer's formats are type-agnostic, prune with
     * spmm24_prune_2of4_bf16 or SPMM24_PRUNE_BF16).  fp32 accumulation. */
    SPMM24_BF16 = 4u
};

/* spmm24_launch with flags (no split_reduction argument).  Same contract
 * otherwise; unknown flag bits give cudaErrorInvalidValue. */
cudaError_t spmm24_launch_ex(cudaStream_t stream, const void* compressed_a, const void* b_packed,
                             const uint16_t* metadata, void* c, int M, int N, int K, int split_k, unsigned flags);

/* Several independent narrow-N SpMMs in one launch (no counterpart in the
 * reference, which launches one SpMM_N2M4_Launch per layer,
 * test/kernelTest.cu:193).  Each problem has the formats and shape rules of
 * spmm24_launch, with N <= 32 (decode: a few tokens per layer), and its
 * own buffers; problems must not write each other's inputs.  One CTA per
 * SM walks whole 128-row tiles of all problems, balanced by K, so the
 * weight stream does not stop between problems (per-call launches stop it
 * at the end of every call).  Each output is summed in one fp32
 * accumulator in increasing K (the result of spmm24_launch with
 * split_k = 1), except when the group has too few tiles to occupy the SMs:
 * then a cluster of 2 (or 4) CTAs shares each tile, each summing one share
 * of its K stages, and the shares are added in a fixed order (the result of
 * spmm24_launch with split_k = 2, or 4).  count: 1..16; at most 2048 tiles of
 * 128 rows in all; flags: SPMM24_STATIC_WEIGHTS, SPMM24_NO_PDL,
 * SPMM24_BF16.  Allocates nothing; the encoded launch is cached per host
 * thread and reused when the same problem array is launched again.
 * Returns cudaErrorInvalidValue (reason in spmm24_last_error) for a bad
 * problem, count or flag.
 * gather (optional): the problem is one M-shard of a layer split across the
 * GPUs of a node, and its output rows go straight into row
 * gather->row_offset + m of every rank's full C (as for
 * spmm24_launch_gather; c may then be NULL); complete on the peers after
 * spmm24_gather_barrier on every rank.
 * epilogue (optional): the problem's own fused epilogue, as for
 * spmm24_launch_fused (alpha, bias, activation, residual, packed-B output;
 * not packed with a gather).  spmm24_gather and spmm24_epilogue are
 * declared below. */
struct spmm24_gather;
struct spmm24_epilogue;
typedef struct spmm24_problem {
    const void* compressed_a;
    const void* b_packed;
    const uint16_t* metadata;
    void* c;
    int M, N, K;
    const struct spmm24_gather* gather;
    const struct spmm24_epilogue* epilogue;
} spmm24_problem;
cudaError_t spmm24_launch_grouped(cudaStream_t stream, const spmm24_problem* problems, int count, unsigned flags);
/* The same for fp8 operands in spmm24_launch_fp8's formats (values,
 * N x K row-major B, fp8 metadata; K % 128 == 0): compressed_a, b_packed
 * and metadata point at those, C is fp16 (bf16 with SPMM24_BF16), and each
 * problem's epilogue alpha carries its dequantisation scale (no epilogue:
 * alpha 1).  flags additionally take SPMM24_FP8_A_E5M2 / SPMM24_FP8_B_E5M2
 * (for every problem of the launch). */
cudaError_t spmm24_launch_grouped_fp8(cudaStream_t stream, const spmm24_problem* problems, int count,
                                      unsigned flags);

/* Epilogue of spmm24_launch_fused (no counterpart in the reference, whose
 * epilogue only rounds to fp16, src/LoadAndStore.cuh:385-429).  Applied
 * after the split-K reduction, before the output is rounded:
 *     C[m, n] = act(alpha * acc[m, n] + bias[m]) + residual[m, n]
 * bias: M elements of C's type (per output row = per output feature of the
 * layer), or NULL.  residual: C's type and layout, or NULL (it may be C
 * itself: each element is read before it is written).  */
enum {
    SPMM24_ACT_NONE = 0,
    SPMM24_ACT_RELU = 1,
    SPMM24_ACT_SILU = 2, /* y * sigmoid(y) */
    SPMM24_ACT_GELU = 3  /* tanh form: 0.5 y (1 + tanh(sqrt(2/pi) (y + 0.044715 y^3))) */
};
enum {
    SPMM24_OUT_ROW_MAJOR = 0, /* C is M x N row-major */
    /* C is written as the next layer's packed B (toolPackMatrixB's layout,
     * test/utils.h:188-229, with K' = M): ceil(N/8) strips of M x 8, element
     * (m, n) at ((n / 8) * M + m) * 8 + n % 8, pad columns zero; C must be
     * 16-byte aligned and hold ceil(N/8) * 8 * M elements. */
    SPMM24_OUT_PACKED_B = 1
};
typedef struct spmm24_epilogue {
    const void* bias;
    const void* residual;
    float alpha;    /* 1.0f for none */
    int activation; /* SPMM24_ACT_* */
    int out_layout; /* SPMM24_OUT_* */
} spmm24_epilogue;

/* spmm24_launch_ex with a fused epilogue; epilogue == NULL is the plain
 * launch.  flags as for spmm24_launch_ex (SPMM24_BF16 included). */
cudaError_t spmm24_launch_fused(cudaStream_t stream, const void* compressed_a, const void* b_packed,
                                const uint16_t* metadata, void* c, int M, int N, int K, int split_k, unsigned flags,
                                const spmm24_epilogue* epilogue);

/* Fused SpMM + all-gather across the GPUs of one node (no counterpart in
 * the reference, which runs on one GPU).  For an M-sharded layer each rank
 * launches its shard (compressed_a / metadata = the shard's rows, M = the
 * shard's row count) and the epilogue writes every output row straight into
 * row row_offset + m of every rank's full C (row-major, m_full x N) over
 * NVLink -- no separate collective.  c_full[r] is rank r's buffer as seen
 * from this process (this rank's own buffer, and the peers' buffers opened
 * with spmm24_ipc_import); all 16-byte aligned.  flags: as for
 * spmm24_launch_ex.  The peers' rows are complete only after
 * spmm24_gather_barrier on every rank. */
#define SPMM24_MAX_GATHER_RANKS 8
typedef struct spmm24_gather {
    void* c_full[SPMM24_MAX_GATHER_RANKS];
    int n_ranks;
    int row_offset;
    int m_full;
    /* Optional: the full C's NVLink multicast address (a multicast object
     * bound to every rank's c_full, e.g. a symmetric-memory buffer's
     * multicast pointer).  Each output chunk is then stored once with
     * multimem.st and replicated by the switch, instead of once per rank.
     * Requires N % 8 == 0.  NULL: unicast stores to c_full[]. */
    void* c_multicast;
} spmm24_gather;
cudaError_t spmm24_launch_gather(cudaStream_t stream, const void* compressed_a, const void* b_packed,
                                 const uint16_t* metadata, int M, int N, int K, int split_k, unsigned flags,
                                 const spmm24_gather* gather);

/* Cross-GPU barrier on `stream` after spmm24_launch_gather: rank `rank`
 * writes `epoch` into slot `rank` of every rank's flag array
 * (flag_arrays[r]: n_ranks u32 of rank r, peers' opened with
 * spmm24_ipc_import, zero-initialised once), then waits until all n_ranks
 * slots of its own array have reached `epoch` (use a counter that grows by
 * one per call).  epoch = 0 takes one past this rank's last published epoch
 * from its own flag array on the device, so the call needs no host-side
 * counter and can be captured in a CUDA graph and replayed; use either
 * form, or both, as long as every rank passes the same sequence of epochs.
 * The wait is bounded by limit_us; a barrier that gives up
 * sets bit 8 of the device status word (spmm24_device_status) instead of
 * hanging. */
cudaError_t spmm24_gather_barrier(cudaStream_t stream, uint32_t* const* flag_arrays, int n_ranks, int rank,
                                  uint32_t epoch, unsigned limit_us);

/* spmm24_launch_grouped with the cross-GPU barrier folded into the end of
 * the same kernel, for a step whose problems all carry gather descriptors
 * (no counterpart in the reference): when the launch has completed on
 * every rank, every rank's full C holds every rank's rows, with no
 * separate barrier launch.  flag_arrays[r]: rank r's array of n_ranks + 1
 * u32 (this process's own one, the peers' opened with spmm24_ipc_import),
 * zeroed once; slots 0..n_ranks-1 are spmm24_gather_barrier's, counted on
 * the device as with its epoch 0 (the two can be mixed on one array), and
 * word n_ranks counts this grid's finished CTAs (back to zero after every
 * launch).  The last CTA to finish publishes the epoch and waits, bounded
 * by limit_us; a barrier that gives up sets bit 8 of the device status
 * word.  Same problems, formats and flags as spmm24_launch_grouped (16-bit
 * operands). */
typedef struct spmm24_group_barrier {
    uint32_t* flag_arrays[SPMM24_MAX_GATHER_RANKS];
    int n_ranks;
    int rank;
    unsigned limit_us;
} spmm24_group_barrier;
cudaError_t spmm24_launch_grouped_gather(cudaStream_t stream, const spmm24_problem* problems, int count,
                                         unsigned flags, const spmm24_group_barrier* barrier);

/* CUDA IPC for the peer buffers: spmm24_ipc_export describes a device
 * pointer (any address inside an allocation, e.g. a tensor of a caching
 * allocator) for another process of the node; spmm24_ipc_import maps it
 * there (peer access over NVLink) and spmm24_ipc_close unmaps it. */
typedef struct spmm24_ipc_handle {
    unsigned char handle[64];
    uint64_t offset;
} spmm24_ipc_handle;
cudaError_t spmm24_ipc_export(const void* dev_ptr, spmm24_ipc_handle* out);
cudaError_t spmm24_ipc_import(const spmm24_ipc_handle* handle, void** dev_ptr);
cudaError_t spmm24_ipc_close(void* dev_ptr);

/* Allocation-free launch (no counterpart in the reference).  For callers
 * that cannot let a library call cudaMalloc: applications whose device
 * memory is owned by their own pool or arena (a framework allocator, a
 * pre-planned serving engine), and latency-critical loops where an
 * allocation, which can synchronise the device, is not acceptable.
 * Computes the same C = A_sparse * B as spmm24_launch (same formats and
 * shape rules, fp32 summation order may differ) with the stream-K kernel,
 * whose scratch is a fixed array inside the library: 4 MB + 1 KB of device
 * memory held by every GPU that loads the library, until process exit.
 *   Limit: N <= 32 (the scratch holds up to 256 partial tiles of 128 x 32
 *   fp32); wider N returns cudaErrorInvalidValue with the reason in
 *   spmm24_last_error().
 *   The first call on a device looks up the scratch array's device address
 *   (cudaGetSymbolAddress, with that device current); make that first call
 *   before any stream capture.  The address is kept for the life of the
 *   process: do not call this entry point on a device after
 *   cudaDeviceReset on it (the module is loaded again and the array may
 *   move).
 *   All calls share the one scratch array and every call starts by clearing
 *   the flag words it uses: calls that overlap on the GPU (different
 *   streams, or different host threads) race and must be serialised by the
 *   caller.
 * Calls no cudaMalloc, cudaFree or allocating library routine. */
cudaError_t spmm24_launch_noalloc(cudaStream_t stream, const void* compressed_a, const void* b_packed,
                                  const uint16_t* metadata, void* c, int M, int N, int K);

/* Caller-allocated form of toolCompressMatrixA (test/utils.h:91-150) with
 * its Block_M = Block_K = 16: dense row-major fp16 (as raw bits) ->
 * compressed values (M*K/2) and raw metadata (M*K/16).  Bit-exact with the
 * reference for every 2:4-sparse input (at least two zeros -- +0 or -0 --
 * in each group of four along K).  Returns the value count, -1 for a bad
 * shape (M % 16 or K % 16 nonzero) and -2 for a group with fewer than two
 * zeros (the reference would write past its buffers). */
int spmm24_compress_a(const uint16_t* dense_a, int M, int K, uint16_t* values_out, uint16_t* meta_out);

/* Caller-allocated form of toolReorderMetadata (test/utils.h:155-185).
 * Returns 0, or -1 when M % 16 or K % 64 is nonzero. */
int spmm24_reorder_metadata(const uint16_t* meta_in, int M, int K, uint16_t* meta_out);

/* compress + reorder in one pass: the on-device metadata directly. */
int spmm24_compress_reordered(const uint16_t* dense_a, int M, int K, uint16_t* values_out, uint16_t* meta_out);

/* Caller-allocated form of toolPackMatrixB (test/utils.h:188-229) with its
 * Block_K = 64, Block_N = 8.  Writes ceil(N/8)*8*K values; for N % 8 != 0
 * the pad columns are zero.  Returns 0, or -1 when K % 64 != 0. */
int spmm24_pack_b(const uint16_t* b_rowmajor, int K, int N, uint16_t* b_packed_out);

/* Magnitude 2:4 pruning along K, in place: keeps the two largest |x| of
 * each group of four (ties prefer the lower index).  The reference only
 * generates random masks (test/utils.h:38-66); this is the pruning step of
 * its host prune/compress/metadata pipeline.  Returns 0, or -1 if K % 4. */
int spmm24_prune_2of4(uint16_t* dense_a, int M, int K);

/* The same prune on bf16 bit patterns (for SPMM24_BF16 weights). */
int spmm24_prune_2of4_bf16(uint16_t* dense_a, int M, int K);

/* On-device packer (no counterpart in the reference, whose packer runs on
 * the host only): one pass over a dense row-major M x K 16-bit matrix in
 * device memory that optionally applies a magnitude 2:4 prune (prune =
 * SPMM24_PRUNE_F16: spmm24_prune_2of4; SPMM24_PRUNE_BF16:
 * spmm24_prune_2of4_bf16; SPMM24_PRUNE_NONE: none), then writes the
 * compressed values (M*K/2 elements) and the REORDERED metadata (M*K/16
 * u16) -- bit-exact with the prune + spmm24_compress_reordered.  M % 16 == 0, K % 64 == 0;
 * dense and values 16-byte aligned.  If bad_blocks (device int, optional)
 * is given, the kernel adds 1 for every row of a 16x16 block holding a
 * group of four with fewer than two zeros (the outputs of those rows are
 * unspecified); the caller zeroes it first.  Asynchronous on `stream`. */
enum { SPMM24_PRUNE_NONE = 0, SPMM24_PRUNE_F16 = 1, SPMM24_PRUNE_BF16 = 2 };
cudaError_t spmm24_pack_a_device(cudaStream_t stream, const void* dense_a, int M, int K, int prune,
                                 void* values_out, uint16_t* meta_out, int* bad_blocks);

/* spmm24_prune_2of4 on a device matrix, in place (K % 4 == 0, 8-byte
 * aligned).  Asynchronous on `stream`. */
cudaError_t spmm24_prune_2of4_device(cudaStream_t stream, void* dense_a, int M, int K);
/* spmm24_prune_2of4_bf16 on a device matrix, in place. */
cudaError_t spmm24_prune_2of4_bf16_device(cudaStream_t stream, void* dense_a, int M, int K);

/* spmm24_pack_b on the device: row-major K x N fp16 -> ceil(N/8) strips of
 * K x 8 (pad columns zero), bit-exact with the host form; the producer of a
 * layer's activations can pack them in place of toolPackMatrixB
 * (test/utils.h:188-229).  K % 64 == 0, output 16-byte aligned.
 * Asynchronous on `stream`. */
cudaError_t spmm24_pack_b_device(cudaStream_t stream, const void* b_rowmajor, int K, int N, void* b_packed_out);

/* ---------------------------------------------------------------- fp8
 * fp8 extension (no counterpart in the reference, which is fp16 only):
 * A and B hold OCP 8-bit floats, E4M3 (no infinities) or E5M2, and the
 * tensor cores run tcgen05.mma.sp kind::f8f6f4 with fp32 accumulation; C,
 * bias and residual are fp16 (bf16 with SPMM24_BF16).  Half the weight
 * bytes of the 16-bit path.  Formats (K % 128 == 0, M % 16 == 0):
 *   values   M*K/2 bytes: band b (16 rows), 32-K block q, row r -> the 16
 *            kept bytes of that row's eight groups of four, in K order, at
 *            ((b*K/32 + q)*16 + r)*16 -- the 16-bit layout's 16x8 blocks
 *            with bytes in place of halves
 *   metadata M*K/8 bytes: band b, 128-K group g, row r -> 16 bytes at
 *            ((b*K/128 + g)*16 + r)*16; nibble c (bits 4c..4c+3 of the
 *            little-endian 128-bit row) describes the group of four at
 *            K = 128g + 4c: i0 | i1 << 2, i0 < i1 the kept positions
 *   B        N x K row-major (the activations as a layer produces them: no
 *            B packing step)
 * The compress rule is the 16-bit one (test/utils.h:124-146) on bytes: the
 * first two zeros (+0 or -0) of each group are dropped. */
enum { SPMM24_FP8_E4M3 = 0, SPMM24_FP8_E5M2 = 1 };
enum {
    SPMM24_FP8_A_E5M2 = 8u,  /* spmm24_launch_fp8 flag: A holds E5M2 (default E4M3) */
    SPMM24_FP8_B_E5M2 = 16u  /* B holds E5M2 (default E4M3) */
};
/* Magnitude 2:4 prune of a row-major M x K fp8 matrix in place (the
 * selection of spmm24_prune_2of4; NaN compares false).  fmt: SPMM24_FP8_*.
 * Returns 0 or -1. */
int spmm24_prune_2of4_fp8(uint8_t* dense_a, int M, int K, int fmt);
/* Dense M x K fp8 (host) -> values (M*K/2 bytes) + metadata (M*K/8 bytes).
 * Returns M*K/2, -1 for bad arguments, -2 when a group of four holds more
 * than two non-zeros. */
int spmm24_compress_a_fp8(const uint8_t* dense_a, int M, int K, uint8_t* values_out, uint8_t* meta_out);
/* spmm24_compress_a_fp8 (after an optional spmm24_prune_2of4_fp8: prune 0 =
 * none, 1 = E4M3, 2 = E5M2) on a dense M x K fp8 matrix in device memory,
 * bit-exact with the host functions.  dense, values and metadata 16-byte
 * aligned.  If bad_blocks (device int, optional; the caller zeroes it) is
 * given, the kernel adds 1 for every row of a 16 x 32 block holding a group
 * of four with more than two non-zeros (those outputs are unspecified).
 * Asynchronous on `stream`. */
cudaError_t spmm24_pack_a_fp8_device(cudaStream_t stream, const void* dense_a, int M, int K, int prune,
                                     void* values_out, void* meta_out, int* bad_blocks);
/* C = A_sparse * B^T-layout B, with the same split_k, flags
 * (SPMM24_STATIC_WEIGHTS, SPMM24_NO_PDL, SPMM24_BF16 for the output type,
 * SPMM24_FP8_A_E5M2, SPMM24_FP8_B_E5M2) and epilogue (alpha doubles as the
 * product of the per-tensor dequantisation scales) as spmm24_launch_fused.
 * values, b_nk and metadata 16-byte aligned.  Asynchronous on `stream`. */
cudaError_t spmm24_launch_fp8(cudaStream_t stream, const void* values, const void* b_nk, const void* metadata, void* c,
                              int M, int N, int K, int split_k, unsigned flags, const spmm24_epilogue* epilogue);

/* Packed-weight files (no counterpart in the reference): a 64-byte header
 * (magic "SPMM24W", version 1, dtype 0 = fp16 / 1 = bf16 / 2 = fp8 E4M3 /
 * 3 = fp8 E5M2, M, K, payload sizes, FNV-1a-64 checksum of the payload),
 * then the compressed values and the metadata exactly as spmm24_launch
 * (16-bit: M*K bytes of values, reordered metadata, K % 64 == 0) or
 * spmm24_launch_fp8 (M*K/2 bytes of values, fp8 metadata, K % 128 == 0)
 * consumes them; M*K/8 bytes of metadata either way.  Host buffers.
 * Return 0 or a negative SPMM24_PACKED_E* code. */
enum {
    SPMM24_PACKED_EARG = -1,     /* bad argument or shape (M % 16, K % 64) */
    SPMM24_PACKED_EIO = -2,      /* open / read / write failed, or short file */
    SPMM24_PACKED_EFORMAT = -3,  /* not a packed-weight file, unknown version, or trailing bytes */
    SPMM24_PACKED_ECHECKSUM = -4, /* payload does not match its checksum */
    SPMM24_PACKED_ECAPACITY = -5  /* the payload is larger than the buffers passed to spmm24_load_packed */
};
typedef struct spmm24_packed_header {
    uint32_t version, dtype, M, K;
    uint64_t values_bytes, meta_bytes, checksum;
} spmm24_packed_header;
int spmm24_save_packed(const char* path, int dtype, int M, int K, const void* values, const void* meta);
int spmm24_load_packed_header(const char* path, spmm24_packed_header* out);
/* Reads the payload into values (values_capacity bytes) and meta
 * (meta_capacity bytes), normally sized from spmm24_load_packed_header.  The
 * header is read again inside this call; if its payload sizes exceed either
 * capacity (the file was replaced or grew after the header was read),
 * nothing is read and SPMM24_PACKED_ECAPACITY is returned. */
int spmm24_load_packed(const char* path, void* values, size_t values_capacity, void* meta, size_t meta_capacity);

/* Workspace the caller must pass as split_reduction: always 0 bytes (the
 * split-K reduction runs on chip; no launch path keeps a workspace).
 * Replaces the Split_K*M*N halves contract of test/kernelTest.cu:136. */
size_t spmm24_workspace_bytes(int M, int N, int K, int split_k);

/* The tile / stage / split configuration spmm24_launch would use.
 * Replaces the compile-time N switch of src/SpMM_API.cu:128-154 and
 * N2M4TilingConfig (src/TileConfig.h:60-94).  Returns 0 or -1. */
typedef struct spmm24_config {
    int tile_m;      /* rows per tile (128; 256 or 512 for a CTA pair) */
    int tile_n;      /* columns per tile */
    int stage_k;     /* logical K per pipeline stage (128) */
    int stages;      /* pipeline depth */
    int split_k;     /* CTAs per cluster along K */
    int grid_ctas;   /* CTAs launched */
    int smem_bytes;  /* dynamic shared memory per CTA */
    int stream_k;    /* always 0: spmm24_launch never picks the stream-K kernel (spmm24_launch_noalloc's) */
    int cta_pair;    /* 1: CTA-pair tiles (cta_group::2 MMAs): 256 x 256, 256 x 128 or 512 x 240 */
} spmm24_config;
int spmm24_select_config(int M, int N, int K, int split_k, spmm24_config* out);
/* Process-wide override of the kernel picker (no counterpart in the
 * reference, whose tile configuration is fixed at compile time,
 * src/TileConfig.h:60-94, src/SpMM_API.cu:128-154).  For tests and tuning
 * sweeps that must reach one specific kernel; production callers never
 * need it, and the library reads no environment variables.  Applies to the
 * launches that follow on every thread; NULL restores the automatic choice.
 * Returns cudaErrorInvalidValue for an out-of-range field. */
typedef struct spmm24_tuning {
    int pair;       /* -1 auto; 0 never use the CTA-pair kernels; 1 whenever legal (K % 128 == 0, split_k <= 1) */
    int pair2;      /* -1 auto; 0 never use the two-M-half pair kernel; 1 whenever the pair path allows it */
    int pair_split; /* 0 auto; 1 or 2 K halves per pair tile */
    int tile_n;     /* 0 auto; 16, 32, 64, 128 or 256: the cluster kernel's tile width; on the pair
                       path 128 forces 256 x 128 tiles and 256 the 256 x 256 ones */
    int deep_ring;  /* 0 auto (a shallow ring, two CTAs per SM, for tile_n <= 32); 1 the deepest ring */
    int group_split; /* grouped launches: 0 auto; 1 whole K per tile; 2 or 4: each tile's K split over a cluster of 2 or 4 CTAs */
} spmm24_tuning;
cudaError_t spmm24_set_tuning(const spmm24_tuning* t);
/* The schedule spmm24_launch_grouped would build for `count` problems of
 * M[i] rows and K[i] (fp8: K % 128 == 0, else K % 64 == 0) on a device of
 * `sms` SMs where `max_clusters4` clusters of four CTAs fit at once,
 * computed on the host without a GPU (N does not enter it): *split = CTAs
 * per 128-row tile along K (1, 2 or 4), *units = CTAs (or clusters) the
 * launch would use, *makespan = the busiest unit's cost in stages (a tile
 * costs its stages + 1; split: its share + 1, + 1 more for four).  Follows
 * spmm24_set_tuning's group_split.  For tests and tuning; any output may
 * be NULL.  Returns 0, or -1 for bad arguments. */
int spmm24_group_schedule(const int* M, const int* K, int count, int fp8, int sms, int max_clusters4, int* split,
                          int* units, long long* makespan);

/* The same for spmm24_launch_fp8 (stage_k 256: a stage carries 256 logical
 * K of fp8 operands; K % 128 == 0), for an epilogue without a residual or a
 * packed output. */
int spmm24_select_config_fp8(int M, int N, int K, int split_k, spmm24_config* out);

/* Row range of shard `index` of `parts` when an M x K layer is split along
 * M across devices (no reduction needed: each shard is a contiguous slice
 * of the compressed A, of the metadata and of the rows of C).  Boundaries
 * are multiples of `align` rows (align a positive multiple of 16; 128
 * keeps whole 128-row tiles on one device); the last shard takes the
 * remainder.  Element offsets of the shard: compressed A row_begin*K/2,
 * metadata row_begin*K/16, C row_begin*N.  The reference runs on one GPU
 * only (test/build/kernelTest.sh:37); this is the partition its multi-GPU
 * use needs.  Returns 0, or -1 for bad arguments. */
int spmm24_shard_rows(int M, int parts, int index, int align, int* row_begin, int* row_end);

/* Reads and clears this process's sticky device status word on `device`
 * (0 = no kernel gave up a bounded wait).  Synchronises the device. */
cudaError_t spmm24_device_status(int device, uint32_t* status_out);

/* Self test of the failure detection: runs a one-block kernel that waits,
 * with the library's bounded wait and a limit of `limit_us` microseconds,
 * on an mbarrier (which = 0) or a global flag (which = 1) that nothing ever
 * completes, then reports the status the kernel recorded (non-zero: the wait
 * gave up as designed) and whether the device is still usable.  Nothing
 * faults, traps or hangs.  The reference has no failure detection
 * (checkLastCudaError, test/utils.h:21-28, only exits the process). */
cudaError_t spmm24_selftest_bounded_wait(int which, unsigned limit_us, uint32_t* status_out);

/* Human-readable reason for the last cudaErrorInvalidValue returned on the
 * calling thread ("" if none). */
const char* spmm24_last_error(void);

const char* spmm24_version(void);

#ifdef __cplusplus
} /* extern "C" */

#include <cuda_fp16.h>

/* C++ drop-ins with the reference's exact names and types. */

/* src/SpMM_API.cu:61-70 (the stale 7-argument declaration of
 * build/SpMM_API.cuh:15-22 is replaced by the 9-argument definition).
 * Same call as spmm24_launch, with two differences from the reference a
 * migrating caller should know:
 *   Split_Reduction is never read or written (the split-K partial sums are
 *     reduced on chip), so it may be NULL; the reference used it as the
 *     Split_K * M * N fp16 scratch of its second, reduction launch.
 *   Split_K is a request, not a guarantee of the launch shape: 0 lets the
 *     library choose, 1..8 asks for that many K slices (clamped to the number
 *     of 128-wide K stages; above 8 means 8), and a wide-N shape on the
 *     CTA-pair kernels runs unsplit.  The result differs only in fp32
 *     summation order.
 * Unsupported shapes return cudaErrorInvalidValue (the reference returned
 * success without launching). */
cudaError_t SpMM_N2M4_Launch(cudaStream_t stream, const half* Compressed_A, const half* B, const uint16_t* metadata,
                             half* C, const int M_Global, const int N_Global, const int K_Global,
                             half* Split_Reduction, const int Split_K);

/* test/utils.h:91-150; outputs are malloc'ed, the caller frees them.
 * Only Block_M = Block_K = 16 is supported (-1 otherwise). */
int toolCompressMatrixA(half* denseMatrixA, int Global_M, int Global_K, int Block_M, int Block_K,
                        half** compressedMatrixA, uint16_t** matadata);

/* test/utils.h:155-185; output malloc'ed (NULL on failure). */
void toolReorderMetadata(uint16_t* matadata, int Global_M, int Global_K, int Block_M, int Block_K,
                         uint16_t** reorderMatadata);

/* test/utils.h:188-229; output malloc'ed (NULL on failure). */
void toolPackMatrixB(half* MatrixB, int Global_K, int Global_N, int Block_K, int Block_N, half** packMatrixB);

#endif /* __cplusplus */

#endif /* SPMM24_SPMM_API_H */
