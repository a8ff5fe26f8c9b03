// Compiles the reference's kernel_smoothquant (rocwmma_smoothquant.cpp:58-122)
// unchanged, from its source where it lies, against the host emulation of
// HIP in hip_emu/, and exposes one C entry that launches it exactly as the
// reference driver does (rocwmma_smoothquant.cpp:147-149).  Test
// infrastructure: pins the oracle to the reference's own code.
#define main rocwmma_smoothquant_sample_main
#include "rocwmma_smoothquant.cpp"
#undef main

extern "C" void ref_smoothquant(const void* x, const float* smooth, int8_t* y, float* row_scale, uint32_t M,
                                uint32_t N, float quant_max)
{
    hipLaunchKernelGGL(kernel_smoothquant, dim3(M), dim3(TBLOCK), 0, 0, static_cast<const __half*>(x), smooth, y,
                       row_scale, M, N, quant_max);
}
