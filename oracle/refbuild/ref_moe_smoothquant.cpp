// Compiles the reference's kernel_moe_smoothquant
// (rocwmma_moe_smoothquant.cpp:69-131) unchanged against the HIP host
// emulation; one C entry launches it as the reference driver does
// (rocwmma_moe_smoothquant.cpp:176-179).  Test infrastructure.
#define main rocwmma_moe_smoothquant_sample_main
#include "rocwmma_moe_smoothquant.cpp"
#undef main

extern "C" void ref_moe_smoothquant(const void* x, const float* smooth, const int32_t* topk_ids, int8_t* qy,
                                    float* row_scale, uint32_t tokens, uint32_t hidden, uint32_t topk,
                                    uint32_t experts, float quant_max)
{
    hipLaunchKernelGGL(kernel_moe_smoothquant, dim3(tokens * topk), dim3(TBLOCK), 0, 0,
                       static_cast<const __half*>(x), smooth, topk_ids, qy, row_scale, tokens, hidden, topk, experts,
                       quant_max);
}
