// Compiles the reference's three sorting kernels (rocwmma_moe_sorting.cpp:53-125)
// unchanged against the HIP host emulation; one C entry runs the reference
// driver's sequence (rocwmma_moe_sorting.cpp:171-189): clear the counters and
// the sorted array (-1), histogram, prefix sum, scatter.  Test infrastructure.
#define main rocwmma_moe_sorting_sample_main
#include "rocwmma_moe_sorting.cpp"
#undef main

// The histogram's dynamic shared memory (extern __shared__ in the kernel).
thread_local IdxT smem_hist[1 << 16];

extern "C" void ref_moe_sorting(const int32_t* ids, uint32_t tokens, uint32_t topk, uint32_t experts,
                                uint32_t unit_size, int32_t* expert_count, int32_t* expert_start,
                                int32_t* padded_count, int32_t* sorted_ids, uint32_t sorted_len)
{
    const uint32_t total = tokens * topk;
    std::vector<IdxT> scatter(experts, 0);
    std::memset(expert_count, 0, experts * sizeof(IdxT));
    std::memset(sorted_ids, 0xff, (size_t)sorted_len * sizeof(IdxT));
    const dim3 blockH(TBLOCK), gridH((total + TBLOCK - 1) / TBLOCK);
    hipLaunchKernelGGL(kernel_moe_histogram, gridH, blockH, experts * sizeof(IdxT), 0, ids, expert_count, total,
                       experts);
    hipLaunchKernelGGL(kernel_prefix_sum, dim3(1), dim3(1), 0, 0, expert_count, expert_start, padded_count, experts,
                       unit_size);
    hipLaunchKernelGGL(kernel_moe_scatter, gridH, blockH, 0, 0, ids, expert_start, sorted_ids, scatter.data(), tokens,
                       topk, experts);
}
