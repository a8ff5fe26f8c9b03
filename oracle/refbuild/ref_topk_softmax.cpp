// Compiles the reference's kernel_topk_softmax and kernel_topk_softmax_large
// (rocwmma_topk_softmax.cpp:58-187) unchanged against the HIP host emulation;
// one C entry picks and launches them as the reference driver does
// (rocwmma_topk_softmax.cpp:222-230).  expf is the host C library's.  Test
// infrastructure.
#define main rocwmma_topk_softmax_sample_main
#include "rocwmma_topk_softmax.cpp"
#undef main

extern "C" void ref_topk_softmax(const void* logits, float* topk_w, int32_t* topk_i, uint32_t tokens,
                                 uint32_t experts, uint32_t topk)
{
    const dim3 block(TBLOCK), grid((tokens + WARPS_PER_BLOCK - 1) / WARPS_PER_BLOCK);
    if (experts <= WARP_SIZE)
        hipLaunchKernelGGL(kernel_topk_softmax, grid, block, 0, 0, static_cast<const __half*>(logits), topk_w, topk_i,
                           tokens, experts, topk);
    else
        hipLaunchKernelGGL(kernel_topk_softmax_large, grid, block, 0, 0, static_cast<const __half*>(logits), topk_w,
                           topk_i, tokens, experts, topk);
}
