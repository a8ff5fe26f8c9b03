// sq_math.cuh — the per-element arithmetic of smoothquant (dense and MoE
// kernels).  Reference operation order (rocwmma_smoothquant.cpp:83-120), fp32:
//   xs = float(x) * s;  rs = amax / qmax;  inv = rs > 0 ? 1 / rs : 0;
//   q = int8(fminf(fmaxf(rintf(xs * inv), -qmax), qmax))
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace b2sq {

// fp16 pair -> two fp32, exactly.  Blackwell's mixed-precision add (fp16
// operand, fp32 addend and result) of -0.0 runs on the FMA pipe; the plain
// cvt.f32.f16 runs on the narrow conversion pipe, which would otherwise bound
// this HBM kernel.  x + (-0.0) == x for every x (signed zeros included); NaN
// payloads may differ, which no output observes.
__device__ __forceinline__ void h2_to_f2(uint32_t w, float& lo, float& hi)
{
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "add.rn.f32.f16 %0, l, %3;\n\tadd.rn.f32.f16 %1, h, %3;\n\t}"
        : "=f"(lo), "=f"(hi)
        : "r"(w), "f"(-0.0f));
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8])
{
    h2_to_f2(v.x, f[0], f[1]);
    h2_to_f2(v.y, f[2], f[3]);
    h2_to_f2(v.z, f[4], f[5]);
    h2_to_f2(v.w, f[6], f[7]);
}

__device__ __forceinline__ int8_t quant1(float xs, float inv, float qmax)
{
    float v = __fmul_rn(xs, inv);
    return static_cast<int8_t>(fminf(fmaxf(rintf(v), -qmax), qmax));
}

// Fast form of quant1 for an integer qmax (<= 127), bit-identical to it for
// every input including NaN and +-inf: clamp first (fmaxf maps NaN to -qmax,
// as fmaxf(rintf(NaN), -qmax) does), then round to nearest even by adding
// 1.5 * 2^23, which leaves rint(c) in the low mantissa bits in two's
// complement.  Clamping before rounding equals rounding before clamping
// because qmax is an integer.  Only FMA/ALU-pipe instructions, no
// conversion-pipe (rint / float->int) work.
__device__ __forceinline__ uint32_t quant_bits(float xs, float inv, float qmax)
{
    const float v = __fmul_rn(xs, inv);
    const float c = fminf(fmaxf(v, -qmax), qmax);
    return __float_as_uint(__fadd_rn(c, 12582912.0f));  // low byte = int8(rint(c))
}

__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3)
{
    return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

__device__ __forceinline__ uint32_t pack4(int8_t a, int8_t b, int8_t c, int8_t d)
{
    return (uint32_t)(uint8_t)a | ((uint32_t)(uint8_t)b << 8) | ((uint32_t)(uint8_t)c << 16) |
           ((uint32_t)(uint8_t)d << 24);
}

// row_scale and its reciprocal, reference :95 and :98 (IEEE divisions).
__device__ __forceinline__ float row_scale_of(float amax, float qmax) { return amax / qmax; }
__device__ __forceinline__ float inv_scale_of(float rs) { return (rs > 0.f) ? (1.f / rs) : 0.f; }

}  // namespace b2sq
