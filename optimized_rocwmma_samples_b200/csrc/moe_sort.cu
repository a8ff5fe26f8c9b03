// moe_sort.cu — MoE token grouping by expert for sm_100a.
//
// Replaces the three kernels of rocwmma_moe_sorting.cpp: histogram (:53-77),
// single-thread prefix sum padded to unit_size (:82-101) and the atomic
// scatter (:107-125).  Same outputs — expert_count[E], expert_start[E+1]
// (padded segments, expert_start[E] = total) and sorted_token_ids (the token
// id of every valid (token, slot) in its expert's segment) — plus row_perm:
// the sorted position of every flat (token, slot) index (-1 for an invalid
// expert id), which MoE smoothquant uses to write its rows directly in
// expert order for the grouped GEMM.
//
// Differences by design: the reference's scatter order inside a segment
// depends on atomic arrival order; here the order is stable (increasing flat
// index), one of the reference's possible outcomes and reproducible.  Padding
// slots of sorted_token_ids are written with the sentinel `tokens`.
//
// One CTA of 1024 threads: a shared-memory histogram, then chunks of 1024
// flat indices ranked per expert with warp match/ballot operations and a
// per-warp, per-expert prefix.  The routing tables are tiny (tokens * topk
// int32), so one SM suffices and the launch is the dominant cost.
#include "common.cuh"
#include "kernels.h"

namespace b2sq {

namespace {

constexpr int kSortThreads = 1024;
constexpr int kSortWarps = kSortThreads / 32;

__global__ void __launch_bounds__(kSortThreads) moe_sort_kernel(const int32_t* __restrict__ ids, uint32_t tokens,
                                                                uint32_t topk, uint32_t experts, uint32_t unit_size,
                                                                int32_t* __restrict__ expert_count,
                                                                int32_t* __restrict__ expert_start,
                                                                int32_t* __restrict__ sorted_ids,
                                                                int32_t* __restrict__ row_perm)
{
    griddep_wait();  // topk ids may come from the previous kernel (PDL launch)
    griddep_launch_dependents();
    extern __shared__ int32_t sh[];
    int32_t* count = sh;                      // [E]
    int32_t* base = count + experts;          // [E] next free position per expert
    int32_t* wcnt = base + experts;           // [warps][E] counts of the current chunk
    const uint32_t total = tokens * topk;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    for (uint32_t e = threadIdx.x; e < experts; e += kSortThreads) count[e] = 0;
    for (uint32_t i = threadIdx.x; i < kSortWarps * experts; i += kSortThreads) wcnt[i] = 0;
    __syncthreads();
    for (uint32_t f = threadIdx.x; f < total; f += kSortThreads) {
        const int32_t e = ids[f];
        if (e >= 0 && (uint32_t)e < experts) atomicAdd(&count[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // padded exclusive prefix, rocwmma_moe_sorting.cpp:88-99
        int32_t off = 0;
        for (uint32_t e = 0; e < experts; ++e) {
            expert_start[e] = off;
            base[e] = off;
            expert_count[e] = count[e];
            off += (int32_t)(((uint32_t)count[e] + unit_size - 1) / unit_size * unit_size);
        }
        expert_start[experts] = off;
        count[0] = off;  // total, read below before the scatter
    }
    __syncthreads();
    const int32_t padded_total = count[0];
    for (int32_t i = threadIdx.x; i < padded_total; i += kSortThreads) sorted_ids[i] = (int32_t)tokens;
    __syncthreads();

    for (uint32_t c0 = 0; c0 < total; c0 += kSortThreads) {
        const uint32_t f = c0 + threadIdx.x;
        int32_t e = f < total ? ids[f] : -1;
        const bool valid = e >= 0 && (uint32_t)e < experts;
        if (!valid) e = -1;
        const uint32_t same = __match_any_sync(0xffffffffu, e);
        const uint32_t rank = __popc(same & ((1u << lane) - 1));
        if (valid && rank == 0) wcnt[warp * experts + e] = __popc(same);
        __syncthreads();
        // Per expert: exclusive prefix over warps, then advance the base.
        for (uint32_t x = threadIdx.x; x < experts; x += kSortThreads) {
            int32_t run = base[x];
            for (int w = 0; w < kSortWarps; ++w) {
                const int32_t n = wcnt[w * experts + x];
                wcnt[w * experts + x] = run;  // becomes this warp's first position
                run += n;
            }
            base[x] = run;
        }
        __syncthreads();
        if (f < total) {
            if (valid) {
                const int32_t pos = wcnt[warp * experts + e] + (int32_t)rank;
                sorted_ids[pos] = (int32_t)(f / topk);
                if (row_perm) row_perm[f] = pos;
            } else if (row_perm) {
                row_perm[f] = -1;
            }
        }
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < kSortWarps * experts; i += kSortThreads) wcnt[i] = 0;
        __syncthreads();
    }
}

}  // namespace

size_t moe_sort_smem(uint32_t experts) { return sizeof(int32_t) * (size_t)experts * (2 + kSortWarps); }

cudaError_t launch_moe_sort(const int32_t* ids, uint32_t tokens, uint32_t topk, uint32_t experts, uint32_t unit_size,
                            int32_t* expert_count, int32_t* expert_start, int32_t* sorted_ids, int32_t* row_perm,
                            cudaStream_t st)
{
    const size_t smem = moe_sort_smem(experts);
    cudaError_t e = cudaFuncSetAttribute(moe_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(moe_sort_kernel, dim3(1), dim3(kSortThreads), smem, st, ids, tokens, topk, experts, unit_size,
                      expert_count, expert_start, sorted_ids, row_perm);
}

}  // namespace b2sq
