// kernels.h — internal launch interface between the C ABI (api.cu) and the
// kernel translation units.  Not installed; the public surface is b2sq.h.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/b2sq.h"

namespace b2sq {

cudaError_t launch_smoothquant(const void* x, const float* s, int8_t* y, float* rs, uint32_t M, uint32_t N,
                               float qmax, cudaStream_t st, int* used_vector_path);

cudaError_t launch_moe_smoothquant(const void* x, const float* s, const int32_t* ids, int8_t* qy, float* rs,
                                   uint32_t T, uint32_t H, uint32_t K, uint32_t E, float qmax,
                                   const int32_t* perm, cudaStream_t st, int* used_vector_path);

// GEMM problem after the host has mapped the user's (A, B, layouts) onto the
// kernel's operands: kernel A has Mk rows, kernel B has Nk rows, both K long.
constexpr uint32_t kMaxExtraOut = 7;  // all-gather over at most 8 GPUs

struct GemmProblem {
    uint32_t Mk, Nk, K;
    const int8_t* a;  // kernel A operand
    uint32_t a_mn_major, lda;
    const int8_t* b;  // kernel B operand
    uint32_t b_mn_major, ldb;
    void* c;
    uint32_t ldc;
    int c_type;         // 0 f16, 1 bf16, 2 i32
    int transpose_out;  // 1: element (i, j) of the kernel result goes to c[j * ldc + i]
    const float* row_scale_vec;  // per kernel-row scale (nullable)
    const float* col_scale_vec;  // per kernel-column scale (nullable)
    float row_scale, col_scale;  // used when the vector is null
    int pdl_dep;                 // 1 / 2: A / B (and row scales) come from the previous kernel (PDL)
    // Extra output buffers (the all-gather entry): every value stored to c is
    // also stored, at the same offset, to each of these (peer GPUs' buffers
    // mapped into this process; plain stores over NVLink).
    void* extra_c[kMaxExtraOut];
    uint32_t n_extra;
    // Multicast all-gather: when set, every 16-byte output store goes once to
    // this NVSwitch multicast address (mapping every rank's buffer at the
    // offset of c) with multimem.st, instead of to c.
    void* mc_c;
};


struct GemmSchedule {
    uint32_t swap_ab;
    uint32_t tile_n;
    uint32_t tile_k;
    uint32_t cta_pair;  // 1: CTA-pair kernel, 256-row tiles
    uint32_t stages;
    uint32_t tiles_m, tiles_n, k_blocks;
    uint32_t ctas;
    uint32_t dp_tiles;
    uint64_t sk_iters;
    size_t workspace_bytes;  // bytes of workspace the schedule needs (0 without stream-K)
};

// Stream-K is used only when whole-tile rounds would leave more than this
// fraction of the last round's SM time idle.
constexpr double kStreamKMinTailLoss = 0.05;
// ... and only while each split tile has at most about this many contributing CTAs.
constexpr uint64_t kStreamKMaxContributors = 3;

// Stream-K workspace layout: a fixed header of per-tile k-block counters at
// offset 0 (zero before the first call; every call leaves them zero), then
// per-CTA partial-tile slots (scratch).  Keeping the counters at a fixed
// place means calls of different shapes can share one workspace.
constexpr uint32_t kWsCounters = 4096;
constexpr size_t kWsCounterBytes = kWsCounters * sizeof(uint32_t);

constexpr uint32_t kTileM = 128;

// Chooses tile_n, stages and the persistent/stream-K split (host only).
void plan_gemm_schedule(uint32_t Mk, uint32_t Nk, uint32_t K, uint32_t a_mn_major, uint32_t b_mn_major,
                        bool allow_stream_k, uint32_t num_sms, GemmSchedule& s);

// Launches the tcgen05 GEMM.  workspace may be null only if
// s.workspace_bytes == 0.  Returns a CUDA error or cudaSuccess; *detail gets
// a static explanation on failure.
cudaError_t launch_gemm_i8(const GemmProblem& p, const GemmSchedule& s, void* workspace, cudaStream_t st,
                           const char** detail);

// Grouped (MoE) GEMM: group g multiplies A rows [group_start[g], +group_count[g])
// (K-major, row-major [rows, K]) by B_g = rows [g*N, (g+1)*N) of a K-major
// [groups*N, K] weight array; C rows follow A rows.  Counts live on the device.
constexpr uint32_t kMaxGroups = 1024;
struct GroupedProblem {
    uint32_t groups, rows, N, K;
    const int8_t* a;
    uint32_t lda;
    const int8_t* b;
    uint32_t ldb;
    void* c;
    uint32_t ldc;
    int c_type;
    const float* row_scale_vec;
    const float* col_scale_vec;  // [groups * N] or null
    float row_scale, col_scale;
    const int32_t* group_start;
    const int32_t* group_count;
};
cudaError_t launch_gemm_i8_grouped(const GroupedProblem& g, uint32_t num_sms, cudaStream_t st, const char** detail);

// MoE sorting (one CTA); shared memory it needs for `experts`.
size_t moe_sort_smem(uint32_t experts);
cudaError_t launch_moe_sort(const int32_t* ids, uint32_t tokens, uint32_t topk, uint32_t experts, uint32_t unit_size,
                            int32_t* expert_count, int32_t* expert_start, int32_t* sorted_ids, int32_t* row_perm,
                            cudaStream_t st);

// MoE router: softmax over expert logits + top-k (moe_route.cu).
cudaError_t launch_topk_softmax(const void* logits, float* topk_w, int32_t* topk_i, uint32_t tokens,
                                uint32_t experts, uint32_t topk, cudaStream_t st);

// Debug: a kernel that waits for an mbarrier nobody arrives on, with a limit.
cudaError_t launch_debug_bounded_wait(uint64_t limit_ns, cudaStream_t st);

// Device status words: every translation unit that includes common.cuh has
// its own copy and registers a reader for it at load time (common.cuh);
// b2sq_last_device_error() calls every registered reader (api.cu).
using StatusReader = cudaError_t (*)(cudaStream_t st, uint32_t* value);
void register_status_reader(StatusReader reader);
cudaError_t read_and_clear_all_status(cudaStream_t st, uint32_t* first_site);

// Sets the calling thread's message returned by b2sq_last_error_message()
// and returns s (defined in api.cu).
b2sq_status set_last_error(b2sq_status s, const char* msg);

}  // namespace b2sq
