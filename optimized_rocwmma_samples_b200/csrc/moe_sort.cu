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
// One thread-block cluster of kSortCtas CTAs (1024 threads each, one SM
// each).  CTA c owns the contiguous flat range [c*C, (c+1)*C) and its warp w
// the sub-range [w*L, (w+1)*L) of it, so "increasing flat index" is "CTA
// order, warp order, then position".  Pass 1: each warp counts its range per
// expert (one ballot per key bit gives the lanes sharing an expert; the
// lowest of them adds to the warp's own shared-memory row of counters, no
// atomics).  One thread per expert then sums the warp rows into the CTA's
// totals; after a cluster barrier every CTA reads all CTAs' totals through
// distributed shared memory, so each derives, without a second kernel or any
// global scratch, the padded expert starts (block-wide scan, identical in
// every CTA) and its own first position in every segment.  Pass 2 walks the
// ranges again and scatters.  A single SM was issue-bound on these
// per-element steps (about 130 instructions per 32 ids); the cluster spreads
// them over kSortCtas SMs.
#include "common.cuh"
#include "kernels.h"

namespace b2sq {

namespace {

constexpr int kSortThreads = 1024;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortCtas = 8;  // cluster size (portable maximum)
constexpr int kSortBatch = 4;  // id loads in flight per lane

// Lanes of the warp holding the same value as this lane, from one ballot per
// bit of the value (nbits ballots whatever the number of distinct values).
__device__ __forceinline__ uint32_t same_lanes(uint32_t v, uint32_t nbits)
{
    uint32_t m = 0xffffffffu;
    for (uint32_t b = 0; b < nbits; ++b) {
        const uint32_t bal = __ballot_sync(0xffffffffu, (v >> b) & 1u);
        m &= ((v >> b) & 1u) ? bal : ~bal;
    }
    return m;
}

// ids[f + 32 b] for b < kSortBatch, -1 past `end` or for an id outside [0, experts).
__device__ __forceinline__ void load_batch(const int32_t* __restrict__ ids, uint32_t f, uint32_t end,
                                           uint32_t experts, int32_t (&out)[kSortBatch])
{
#pragma unroll
    for (int b = 0; b < kSortBatch; ++b) {
        const uint32_t g = f + 32 * b;
        const int32_t e = g < end ? __ldg(ids + g) : -1;
        out[b] = (e >= 0 && (uint32_t)e < experts) ? e : -1;
    }
}

__device__ __forceinline__ int32_t ld_dsmem_s32(uint32_t cluster_addr)
{
    int32_t v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
    return v;
}

}  // namespace

namespace {

__global__ void __launch_bounds__(kSortThreads) __cluster_dims__(kSortCtas, 1, 1)
    moe_sort_kernel(const int32_t* __restrict__ ids, uint32_t tokens, uint32_t topk, uint32_t experts,
                    uint32_t unit_size, int32_t* __restrict__ expert_count, int32_t* __restrict__ expert_start,
                    int32_t* __restrict__ sorted_ids, int32_t* __restrict__ row_perm)
{
    griddep_wait();  // topk ids may come from the previous kernel (PDL launch)
    griddep_launch_dependents();
    extern __shared__ int32_t sh[];
    int32_t* wc = sh;                           // [warps][E]: counts, then first positions
    int32_t* ctot = wc + kSortWarps * experts;  // [E] this CTA's totals (read by the whole cluster)
    int32_t* wsum = ctot + experts;             // [warps] block-scan partials
    const uint32_t rank = cluster_ctarank();
    const uint32_t total = tokens * topk;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t cspan = (total + kSortCtas - 1) / kSortCtas;
    const uint32_t c_0 = min(total, rank * cspan), c_1 = min(total, c_0 + cspan);
    const uint32_t span = (c_1 - c_0 + kSortWarps - 1) / kSortWarps;
    const uint32_t f0 = min(c_1, c_0 + warp * span), f1 = min(c_1, f0 + span);
    const uint32_t below = (1u << lane) - 1;
    // keys: expert ids 0..experts-1; an invalid slot (-1) maps to the
    // all-ones key, which no expert id reaches, and is never counted
    const uint32_t key_bits = 32 - __clz(experts);  // experts < 2^key_bits
    const uint32_t key_mask = (1u << key_bits) - 1;

    for (uint32_t i = threadIdx.x; i < kSortWarps * experts; i += kSortThreads) wc[i] = 0;
    __syncthreads();
    int32_t* mine = wc + warp * experts;
    for (uint32_t c0 = f0; c0 < f1; c0 += 32 * kSortBatch) {  // pass 1: per-warp counts
        int32_t idb[kSortBatch];
        load_batch(ids, c0 + lane, f1, experts, idb);
#pragma unroll
        for (int b = 0; b < kSortBatch; ++b) {
            const int32_t e = idb[b];
            const uint32_t same = same_lanes((uint32_t)e & key_mask, key_bits);
            if (e >= 0 && (same & below) == 0) mine[e] += __popc(same);
            __syncwarp();  // the next leader of the same expert may be another lane
        }
    }
    __syncthreads();

    const uint32_t e = threadIdx.x;  // one thread per expert (experts <= 1024)
    int32_t mycnt = 0;
    if (e < experts) {
        for (int w = 0; w < kSortWarps; ++w) mycnt += wc[w * experts + e];
        ctot[e] = mycnt;
    }
    cluster_sync();  // every CTA's totals are written
    int32_t cnt = 0, before = 0;  // all CTAs' count, and the count of the CTAs ahead of this one
    if (e < experts) {
        const uint32_t local = smem_u32(ctot + e);
#pragma unroll
        for (uint32_t c = 0; c < (uint32_t)kSortCtas; ++c) {
            const int32_t n = c == rank ? mycnt : ld_dsmem_s32(mapa_shared(local, c));
            cnt += n;
            if (c < rank) before += n;
        }
    }
    cluster_sync();  // no CTA leaves (or reuses ctot) while another still reads it

    // padded exclusive prefix over experts: block-wide scan (the same in every CTA)
    const int32_t padded = e < experts ? (int32_t)(((uint32_t)cnt + unit_size - 1) / unit_size * unit_size) : 0;
    int32_t incl = padded;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int32_t o = __shfl_up_sync(0xffffffffu, incl, off);
        if ((int)lane >= off) incl += o;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int32_t v = wsum[lane], x = v;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int32_t o = __shfl_up_sync(0xffffffffu, x, off);
            if ((int)lane >= off) x += o;
        }
        wsum[lane] = x - v;  // exclusive prefix of the warp totals
    }
    __syncthreads();
    const int32_t start = wsum[warp] + incl - padded;
    if (e < experts) {
        if (rank == 0) {
            expert_count[e] = cnt;
            expert_start[e] = start;
            if (e == experts - 1) expert_start[experts] = start + padded;
            for (int32_t p = start + cnt; p < start + padded; ++p) sorted_ids[p] = (int32_t)tokens;  // padding
        }
        int32_t run = start + before;
        for (int w = 0; w < kSortWarps; ++w) {
            const int32_t n = wc[w * experts + e];
            wc[w * experts + e] = run;
            run += n;
        }
    }
    __syncthreads();

    for (uint32_t c0 = f0; c0 < f1; c0 += 32 * kSortBatch) {  // pass 2: scatter in flat order
        int32_t idb[kSortBatch];
        load_batch(ids, c0 + lane, f1, experts, idb);
#pragma unroll
        for (int b = 0; b < kSortBatch; ++b) {
            const uint32_t f = c0 + 32 * b + lane;
            const int32_t ex = idb[b];
            const uint32_t same = same_lanes((uint32_t)ex & key_mask, key_bits);
            if (ex >= 0) {
                const int32_t pos = mine[ex] + __popc(same & below);
                sorted_ids[pos] = (int32_t)(f / topk);
                if (row_perm) row_perm[f] = pos;
            } else if (f < f1 && row_perm) {
                row_perm[f] = -1;
            }
            __syncwarp();
            if (ex >= 0 && (same & below) == 0) mine[ex] += __popc(same);
            __syncwarp();
        }
    }
}

}  // namespace

size_t moe_sort_smem(uint32_t experts)
{
    return sizeof(int32_t) * ((size_t)experts * (kSortWarps + 1) + kSortWarps);
}

cudaError_t launch_moe_sort(const int32_t* ids, uint32_t tokens, uint32_t topk, uint32_t experts, uint32_t unit_size,
                            int32_t* expert_count, int32_t* expert_start, int32_t* sorted_ids, int32_t* row_perm,
                            cudaStream_t st)
{
    const size_t smem = moe_sort_smem(experts);
    cudaError_t e = cudaFuncSetAttribute(moe_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(moe_sort_kernel, dim3(kSortCtas), dim3(kSortThreads), smem, st, ids, tokens, topk, experts, unit_size,
                      expert_count, expert_start, sorted_ids, row_perm);
}

}  // namespace b2sq
