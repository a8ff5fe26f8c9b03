/*
 * b2sq.h — C ABI of the B200 (sm_100a) smoothquant -> int8 GEMM hot path.
 *
 * This is the drop-in boundary for the quantized-inference path of
 * optimized_rocwmma_samples.  In the reference every operator is a HIP
 * __global__ kernel launched by the host driver of the same sample file; the
 * entry points below replace those launches one for one, keep the argument
 * order and meaning (M/N/K, layouts, leading dimensions, scale tensors,
 * quant_max, output dtype) and add only:
 *   - an explicit stream (the reference launches on the default stream),
 *   - a status return in place of CHECK_HIP -> exit(1)
 *     (reference common.hpp:33-46, rocwmma_smoothquant.cpp:35-37),
 *   - UNSUPPORTED in place of "print and return" for shapes the kernels do
 *     not take (reference rocwmma_gemm_quantized.cpp:199-203).
 *
 * Ownership: the caller owns every device buffer (the reference drivers
 * hipMalloc all of them).  No entry point allocates device memory.
 * Calls are stream-ordered, never synchronise the device and are reentrant.
 *
 * Element types: x is IEEE fp16 (the reference's __half); outputs of the GEMM
 * are fp16, bf16 or raw int32 accumulators.
 */
#ifndef B2SQ_H
#define B2SQ_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2SQ_API __attribute__((visibility("default")))
#else
#define B2SQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream; declared here so the header needs
 * no CUDA include.  NULL means the legacy default stream. */
struct CUstream_st;
typedef struct CUstream_st* b2sq_stream_t;

typedef enum {
    B2SQ_OK = 0,
    B2SQ_ERR_INVALID_ARG = 1,  /* null pointer, zero-size or inconsistent ld */
    B2SQ_ERR_UNSUPPORTED = 2,  /* valid request the kernels do not take (alignment) */
    B2SQ_ERR_CUDA = 3,         /* a CUDA runtime/driver call failed */
    B2SQ_ERR_TIMEOUT = 4       /* a bounded device-side wait ran out */
} b2sq_status;

typedef enum { B2SQ_ROW_MAJOR = 0, B2SQ_COL_MAJOR = 1 } b2sq_layout;

typedef enum {
    B2SQ_F16 = 0,
    B2SQ_BF16 = 1,
    B2SQ_I32 = 2  /* raw int32 accumulators, no dequantisation (debug / parity) */
} b2sq_dtype;

/* ------------------------------------------------------------------------ */
/* SmoothQuant                                                              */
/* ------------------------------------------------------------------------ */

/*
 * Replaces kernel_smoothquant (reference rocwmma_smoothquant.cpp:58-63,
 * launch :153-155).  For every row m of x[M,N] (row-major, ld = N):
 *   xs[n]        = float(x[m,n]) * smooth_scale[n]
 *   row_scale[m] = max_n |xs[n]| / quant_max
 *   inv          = row_scale[m] > 0 ? 1 / row_scale[m] : 0
 *   y[m,n]       = int8(clamp(rint(xs[n] * inv), -quant_max, quant_max))
 * with the reference's fp32 operation order (:83-84, :95, :98, :110-113).
 * Any N is accepted (the reference's scalar tail, :87-89 / :118-121).
 * M == 0 is a no-op.
 */
B2SQ_API b2sq_status b2sq_smoothquant(const void* x_f16, const float* smooth_scale,
                             int8_t* y, float* row_scale,
                             uint32_t M, uint32_t N, float quant_max,
                             b2sq_stream_t stream);

/*
 * Replaces kernel_moe_smoothquant (reference rocwmma_moe_smoothquant.cpp:69-76,
 * launch :179-182).  For token t and slot k < topk with e = topk_ids[t*topk+k]:
 *   output row r = row_perm ? row_perm[t*topk+k] : t*topk+k
 *   qy[r,:], row_scale[r] = smoothquant(x[t,:], smooth_scale[e,:])
 * An expert id outside [0, experts) leaves row r unwritten (reference :86-87);
 * so does a negative row_perm entry.  row_perm lets a caller write rows
 * straight into expert-sorted order; NULL gives the reference's order.
 */
B2SQ_API b2sq_status b2sq_moe_smoothquant(const void* x_f16, const float* smooth_scale,
                                 const int32_t* topk_ids, int8_t* qy,
                                 float* row_scale, uint32_t tokens,
                                 uint32_t hidden, uint32_t topk,
                                 uint32_t experts, float quant_max,
                                 const int32_t* row_perm,
                                 b2sq_stream_t stream);

/* ------------------------------------------------------------------------ */
/* int8 x int8 -> int32 GEMM with fused dequant epilogue                    */
/* ------------------------------------------------------------------------ */

/*
 * Replaces gemm_quant_tensor_scale (reference rocwmma_gemm_quantized.cpp:127-132)
 * and implements its documented, unimplemented "Mode 2 (row-col-scale)"
 * (:20, :26):
 *   acc[m,n] = sum_k int32(a[m,k]) * int32(b[k,n])            (exact int32)
 *   c[m,n]   = cvt_rn(float(acc[m,n]) * (sa * sb))             (c_type F16/BF16)
 *   c[m,n]   = acc[m,n]                                        (c_type I32)
 * where sa = scale_a_row ? scale_a_row[m] : scale_a and
 *       sb = scale_b_col ? scale_b_col[n] : scale_b
 * (the scale product first, mirroring :189-193).
 *
 * Layouts: a is [M,K], row-major (lda >= K) or column-major (lda >= M, the
 * reference's layout :92); b is [K,N], column-major (ldb >= K, i.e. K-major
 * weights) or row-major (ldb >= N, the reference's layout :93); c is row-major
 * [M,N] with ldc >= N (reference :94).
 * Requirements (else UNSUPPORTED): a, b 16-byte aligned, lda and ldb
 * multiples of 16.  M, N, K need not be tile multiples.
 *
 * workspace: optional scratch for stream-K splitting of tiles across SMs
 * (per-CTA int32 partial tiles + per-tile counters).  Query its size with
 * b2sq_gemm_i8_workspace_size; it must be 256-byte aligned and zero filled
 * before its first use; every completed call leaves its counters zero again,
 * so it can be reused without clearing by stream-ordered calls (concurrent
 * calls need separate workspaces).  NULL (or too small) disables stream-K;
 * results are identical either way (int32 sums are exact and order
 * independent).
 */
B2SQ_API b2sq_status b2sq_gemm_i8(uint32_t m, uint32_t n, uint32_t k,
                         const int8_t* a, b2sq_layout la, uint32_t lda,
                         const int8_t* b, b2sq_layout lb, uint32_t ldb,
                         void* c, b2sq_dtype c_type, uint32_t ldc,
                         const float* scale_a_row, const float* scale_b_col,
                         float scale_a, float scale_b,
                         void* workspace, size_t workspace_bytes,
                         b2sq_stream_t stream);

/*
 * b2sq_gemm_i8 without a caller-provided workspace (no counterpart in the
 * reference): for callers that cannot allocate device memory, e.g. a host
 * bound over a plain C FFI with no device allocator, or a serving process
 * that has given all of HBM to its own pool and must not call cudaMalloc on
 * the request path.  The stream-K scratch comes from a fixed 24 MiB array
 * compiled into the library, resident on every GPU that loads it until the
 * process exits; nothing is allocated.  Shapes whose schedule needs more
 * scratch than that return B2SQ_ERR_UNSUPPORTED (b2sq_gemm_i8 with a null
 * workspace runs them whole-tile, allocating nothing either); every shape whose tiles are at most 128 wide fits, and so
 * does every shape whose schedule needs no stream-K.  Arguments and results are those of b2sq_gemm_i8.
 * The first call on a device looks up the array's device address (once per
 * device); make that first call before any stream capture.  Every call
 * shares the array and clears its counters itself: calls that overlap on the
 * GPU (other streams or unordered host threads) race on it.  The cached
 * address belongs to the device's current context: after cudaDeviceReset
 * this entry point must not be called again in the same process.
 */
B2SQ_API b2sq_status b2sq_gemm_i8_no_alloc(uint32_t m, uint32_t n, uint32_t k,
                                           const int8_t* a, b2sq_layout la, uint32_t lda,
                                           const int8_t* b, b2sq_layout lb, uint32_t ldb,
                                           void* c, b2sq_dtype c_type, uint32_t ldc,
                                           const float* scale_a_row, const float* scale_b_col,
                                           float scale_a, float scale_b,
                                           b2sq_stream_t stream);

/*
 * The whole hot path in one call: b2sq_smoothquant of x [m, k] (fp16) into
 * xq / row_scale (caller-owned, [m, k] int8 and [m] fp32), then
 *   c = cvt_rn(float(xq @ w) * (row_scale[i] * sw))
 * with w [k, n] (column-major = K-major [n, k] weights, or row-major) and
 * sw = scale_w_col ? scale_w_col[j] : scale_w; c f16 or bf16, row-major.
 * Results are identical to the two separate calls.  The GEMM is enqueued
 * with programmatic dependent launch: its prologue and the streaming of the
 * weights overlap the smoothquant kernel, which matters for decode-sized m,
 * where the quantisation would otherwise be a separate step of its own.
 * k % 16 == 0.
 */
B2SQ_API b2sq_status b2sq_smoothquant_gemm_i8(const void* x_f16, const float* smooth_scale, float quant_max,
                                              int8_t* xq, float* row_scale, uint32_t m, uint32_t k,
                                              const int8_t* w, b2sq_layout lw, uint32_t ldw, uint32_t n,
                                              void* c, b2sq_dtype c_type, uint32_t ldc,
                                              const float* scale_w_col, float scale_w,
                                              void* workspace, size_t workspace_bytes,
                                              b2sq_stream_t stream);

/*
 * The quantized GEMM for operands and result in HOST memory (replaces the
 * reference driver's copy-in / kernel / copy-back sequence,
 * rocwmma_gemm_quantized.cpp:214-218):
 *   h_c[m, n] = cvt(float(h_a @ h_w^T) * (sa_i * sb_j))
 * with h_a int8 [m, k] row-major, h_w int8 [n, k] (K-major weights = B
 * column-major), scales as in b2sq_gemm_i8 (vectors may be null), h_c
 * row-major.  The problem is cut into row_chunks x col_chunks output blocks
 * (0 = chosen from the shape); the host->device copies, the block GEMMs and
 * the device->host copies of finished blocks overlap on three streams the
 * library keeps per device; the caller's stream waits for the last copy
 * back.  dev_buffer (256-byte aligned, b2sq_gemm_i8_host_buffer_size bytes) holds the device copies;
 * nothing is allocated.  Host memory should be pinned for the copies to
 * overlap.  Enqueues only: h_c is complete once `stream` has been
 * synchronised.  k % 16 == 0.  The copies into dev_buffer are ordered after
 * this function's previous call on the same buffer, not after other work
 * queued on `stream`: alternate two buffers to overlap consecutive calls
 * (the next inputs go up while the previous result comes down), and do not
 * use dev_buffer for anything else.  Calls are enqueued one at a time per
 * device (host lock).
 */
B2SQ_API b2sq_status b2sq_gemm_i8_host(uint32_t m, uint32_t n, uint32_t k,
                                       const int8_t* h_a, const int8_t* h_w,
                                       const float* h_scale_a_row, const float* h_scale_b_col,
                                       float scale_a, float scale_b,
                                       void* h_c, b2sq_dtype c_type,
                                       void* dev_buffer, size_t dev_buffer_bytes,
                                       uint32_t row_chunks, uint32_t col_chunks,
                                       b2sq_stream_t stream);

/* Device buffer bytes b2sq_gemm_i8_host needs for a shape. */
B2SQ_API b2sq_status b2sq_gemm_i8_host_buffer_size(uint32_t m, uint32_t n, uint32_t k, b2sq_dtype c_type,
                                                   size_t* bytes);

/* Bytes of workspace that let b2sq_gemm_i8 use stream-K for this shape
 * (0 when the chosen schedule never splits a tile).  Host only. */
B2SQ_API b2sq_status b2sq_gemm_i8_workspace_size(uint32_t m, uint32_t n, uint32_t k,
                                        b2sq_layout la, b2sq_layout lb,
                                        size_t* bytes);

/*
 * The schedule b2sq_gemm_i8 would run for a shape (host only, no CUDA call):
 * tile, operand swap, number of persistent CTAs and the stream-K split.
 * Exposed so the scheduler's coverage can be checked without a GPU.
 */
typedef struct {
    uint32_t swap_ab;        /* 1: computes C^T = B^T A^T (skinny M) */
    uint32_t tile_m;         /* MMA M of one tile (rows of the A operand) */
    uint32_t tile_n;         /* MMA N of one tile */
    uint32_t tile_k;         /* K elements per pipeline stage */
    uint32_t stages;
    uint32_t tiles_m, tiles_n, k_blocks;
    uint32_t ctas;           /* persistent CTAs launched */
    uint32_t dp_tiles;       /* tiles computed whole, in data-parallel order */
    uint32_t sk_iters_per_cta_floor; /* stream-K k-blocks per CTA (floor) */
    uint64_t sk_iters;       /* total stream-K k-blocks over the tail tiles */
    uint32_t cta_pair;       /* 1: tiles are computed by CTA pairs (two SMs, 256-row tiles);
                                ctas counts CTAs, i.e. twice the number of pairs */
} b2sq_gemm_plan;

B2SQ_API b2sq_status b2sq_gemm_i8_plan(uint32_t m, uint32_t n, uint32_t k,
                              b2sq_layout la, b2sq_layout lb,
                              int use_stream_k, uint32_t num_sms,
                              b2sq_gemm_plan* plan);

/* ------------------------------------------------------------------------ */
/* Multi-GPU: the N-sharded GEMM fused with the output all-gather           */
/* ------------------------------------------------------------------------ */

/*
 * Column-parallel GEMM whose epilogue performs the all-gather of the output
 * (no counterpart in the reference, which is single-GPU; it replaces the
 * GEMM + ncclAllGather pair of an N-sharded layer).  This rank computes its
 * shard C_r = dequant(A x B) of n columns, exactly as b2sq_gemm_i8, and
 * stores every output value into each rank's full output buffer:
 *   c_ranks[j] + (row * ldc + col_offset + col) elements, for j < world,
 * where c_ranks[rank] is this rank's own buffer and the others are peer
 * buffers mapped into this process (b2sq_ipc_open).  The stores are plain
 * stores over NVLink from the epilogue, overlapped with the next tiles'
 * math; no multicast is used.  The caller orders the exchange: every rank
 * must be done with the previous contents before any rank calls, and the
 * gathered result is complete once every rank's call has completed (a
 * barrier after the call, e.g. a one-element ncclAllReduce on the stream).
 * world <= 8; all buffers share their 16-byte alignment.
 */
B2SQ_API b2sq_status b2sq_gemm_i8_allgather(uint32_t m, uint32_t n, uint32_t k,
                                  const int8_t* a, b2sq_layout la, uint32_t lda,
                                  const int8_t* b, b2sq_layout lb, uint32_t ldb,
                                  void* const* c_ranks, uint32_t world, uint32_t rank,
                                  uint32_t col_offset, b2sq_dtype c_type, uint32_t ldc,
                                  const float* scale_a_row, const float* scale_b_col,
                                  float scale_a, float scale_b,
                                  void* workspace, size_t workspace_bytes,
                                  b2sq_stream_t stream);

/*
 * The same fused GEMM + all-gather through NVSwitch multicast: c_multicast is
 * an NVLink multicast address (a cuMulticast object every rank bound its
 * own copy of the [m, N] output buffer to, e.g. torch symmetric memory's
 * multicast_ptr) and c_local this rank's own mapping of its buffer.  Each
 * output piece is stored once with multimem.st and the switch writes it to
 * every rank, so a GPU sends its shard across NVLink once instead of once per
 * peer.  Requires m > 128, row-major a, n a multiple of 64 and 16-byte
 * aligned rows; the caller orders the exchange with barriers as above.
 */
B2SQ_API b2sq_status b2sq_gemm_i8_allgather_mc(uint32_t m, uint32_t n, uint32_t k,
                                     const int8_t* a, b2sq_layout la, uint32_t lda,
                                     const int8_t* b, b2sq_layout lb, uint32_t ldb,
                                     void* c_local, void* c_multicast, uint32_t col_offset,
                                     b2sq_dtype c_type, uint32_t ldc,
                                     const float* scale_a_row, const float* scale_b_col,
                                     float scale_a, float scale_b,
                                     void* workspace, size_t workspace_bytes,
                                     b2sq_stream_t stream);

/* CUDA IPC for the all-gather buffers: export a device pointer (memory from
 * cudaMalloc, any offset inside it) as a 64-byte handle plus offset, open a
 * peer's handle in this process (the returned base + offset is the peer's
 * pointer), and close it again. */
typedef struct { unsigned char bytes[64]; } b2sq_ipc_handle;
B2SQ_API b2sq_status b2sq_ipc_export(const void* dev_ptr, b2sq_ipc_handle* handle, uint64_t* offset);
B2SQ_API b2sq_status b2sq_ipc_open(const b2sq_ipc_handle* handle, void** base);
B2SQ_API b2sq_status b2sq_ipc_close(void* base);

/* ------------------------------------------------------------------------ */
/* MoE: grouping by expert and the grouped (per-expert) GEMM                */
/* ------------------------------------------------------------------------ */

/*
 * MoE router, replacing kernel_topk_softmax / kernel_topk_softmax_large
 * (rocwmma_topk_softmax.cpp:58-131, :137-187; launch :222-231).  For fp16
 * logits [tokens, experts] (row-major, ld = experts):
 *   topk_weights[t, k]  softmax probability of the k-th choice (fp32)
 *   topk_indices[t, k]  its expert id (int32)
 * Same selection rules as the reference: equal probabilities resolve in the
 * order of its wave64 shfl_down arg-max tree (lane l takes lane l + off only
 * when strictly greater: the first pick is the lowest id, later picks follow
 * the tree, e.g. 0, 4, 2 for eight equal logits); for experts <= 64, min(topk, experts) slots are written (the rest are left
 * untouched); for experts > 64 only experts 0..63 are candidates and all topk
 * slots are written, (-1.0f, -1) once no candidate is left.  The exp-sum is
 * accumulated in the reference's wave64 order; exp() itself is the library's
 * own fp32 evaluation (within 1 ulp), so probabilities match any platform
 * expf to a few ulp.  topk_indices may feed b2sq_moe_sorting directly.
 */
B2SQ_API b2sq_status b2sq_topk_softmax(const void* logits_f16, float* topk_weights,
                                       int32_t* topk_indices, uint32_t tokens,
                                       uint32_t experts, uint32_t topk,
                                       b2sq_stream_t stream);

/*
 * Replaces the histogram / padded prefix / scatter kernels of
 * rocwmma_moe_sorting.cpp (:53-77, :82-101, :107-125).  For topk_ids
 * [tokens, topk]:
 *   expert_count[e]     valid (token, slot) pairs routed to expert e
 *   expert_start[e]     start of e's segment, segments padded to unit_size;
 *                       expert_start[experts] = padded total
 *   sorted_token_ids    token id of each pair in its expert's segment
 *                       (capacity tokens*topk + experts*unit_size); padding
 *                       slots hold the sentinel `tokens`
 *   row_perm (nullable) sorted position of every flat index t*topk+k, -1 for
 *                       an expert id outside [0, experts)
 * The order inside a segment is stable (increasing flat index): one of the
 * orders the reference's atomic scatter can produce, but reproducible.
 * experts <= 1024, unit_size >= 1.
 */
B2SQ_API b2sq_status b2sq_moe_sorting(const int32_t* topk_ids, uint32_t tokens, uint32_t topk,
                                      uint32_t experts, uint32_t unit_size,
                                      int32_t* expert_count, int32_t* expert_start,
                                      int32_t* sorted_token_ids, int32_t* row_perm,
                                      b2sq_stream_t stream);

/*
 * Grouped int8 GEMM over expert segments (the grouped GEMM of
 * rocwmma_grouped_gemm.cpp:104-122, with the per-group descriptors replaced
 * by the sorting outputs, which stay on the device).  For every group g:
 *   rows r in [group_start[g], group_start[g] + group_count[g]):
 *   c[r, n] = cvt_rn(float(sum_k a[r,k] * w[g][n][k]) * (sa * sb))
 * with sa = scale_a_row ? scale_a_row[r] : scale_a and
 *      sb = scale_b_col ? scale_b_col[g*n_cols + n] : scale_b.
 * a: int8 [rows, k] row-major (lda >= k, lda % 16 == 0): the activations in
 *    expert-sorted order (b2sq_moe_smoothquant with row_perm writes them so);
 * w: int8 [groups][n][k] K-major weights, row pitch ldb (>= k, % 16 == 0);
 * c: row-major [rows, n] (ldc >= n); rows outside every segment are not
 * written.  groups <= 1024; rows = capacity of a / c in rows.
 */
B2SQ_API b2sq_status b2sq_gemm_i8_grouped(uint32_t groups, uint32_t rows, uint32_t n, uint32_t k,
                                          const int8_t* a, uint32_t lda,
                                          const int8_t* w, uint32_t ldb,
                                          void* c, b2sq_dtype c_type, uint32_t ldc,
                                          const float* scale_a_row, const float* scale_b_col,
                                          float scale_a, float scale_b,
                                          const int32_t* group_start, const int32_t* group_count,
                                          b2sq_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Diagnostics                                                              */
/* ------------------------------------------------------------------------ */

/* Static string for a status code. */
B2SQ_API const char* b2sq_status_string(b2sq_status s);

/* Detail of the last failing call on this host thread ("" if none). */
B2SQ_API const char* b2sq_last_error_message(void);

/*
 * Reads and clears the device status word that bounded device-side waits set
 * when they give up (synchronises `stream`).  B2SQ_OK if no wait ran out,
 * B2SQ_ERR_TIMEOUT otherwise; *where (nullable) receives the site code.
 */
B2SQ_API b2sq_status b2sq_last_device_error(b2sq_stream_t stream, uint32_t* where);

/*
 * Test hook for the timeout path: launches one CTA that waits on an mbarrier
 * nothing ever arrives on, with a wait limit of timeout_us microseconds, and
 * returns what b2sq_last_device_error reports afterwards (B2SQ_ERR_TIMEOUT
 * when the limit worked).  Touches no caller memory.
 */
B2SQ_API b2sq_status b2sq_debug_bounded_wait(uint32_t timeout_us, b2sq_stream_t stream);

/* Library version string. */
B2SQ_API const char* b2sq_version(void);

#ifdef __cplusplus
}
#endif

#endif /* B2SQ_H */
