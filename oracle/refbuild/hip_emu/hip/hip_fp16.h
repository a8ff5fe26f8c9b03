// hip_fp16.h — host emulation of HIP's fp16 type and the conversions the
// reference kernels use (exact half -> float; float -> half rounded to
// nearest even).  Test infrastructure only.
#pragma once

#include <cstdint>
#include <cstring>

// HIP's vector types the kernels use (shared with hip_runtime.h).  float4
// carries no 16-byte alignment here: the kernels load rows of any length as
// float4 (rows of N % 8 != 0 start unaligned), which the GPU allows and x86
// does too as long as the compiler emits unaligned vector moves.
#ifndef HIPEMU_VECTOR_TYPES
#define HIPEMU_VECTOR_TYPES
struct float2 {
    float x, y;
};
struct float4 {
    float x, y, z, w;
};
#endif

struct __half {
    uint16_t bits;
};
struct __half2 {
    __half x, y;
};

inline float __half2float(__half h)
{
    const uint32_t s = (uint32_t)(h.bits & 0x8000u) << 16;
    const uint32_t e = (h.bits >> 10) & 0x1fu;
    const uint32_t m = h.bits & 0x3ffu;
    uint32_t f;
    if (e == 0x1f) {
        f = s | 0x7f800000u | (m << 13);
    } else if (e != 0) {
        f = s | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        f = s;
    } else {  // subnormal: m * 2^-24, exact in float
        float v = (float)m * 0x1p-24f;
        std::memcpy(&f, &v, 4);
        f |= s;
    }
    float out;
    std::memcpy(&out, &f, 4);
    return out;
}

inline __half __float2half(float v)
{
    uint32_t x;
    std::memcpy(&x, &v, 4);
    const uint32_t s = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    uint16_t r;
    if (ax >= 0x7f800000u) {  // inf / nan
        r = (uint16_t)(s | 0x7c00u | (ax > 0x7f800000u ? 0x200u | ((ax >> 13) & 0x3ffu) : 0u));
    } else if (ax >= 0x477ff000u) {  // rounds to >= 65520: overflow to inf
        r = (uint16_t)(s | 0x7c00u);
    } else if (ax >= 0x38800000u) {  // normal half
        const uint32_t mant = ax & 0x7fffffu;
        const uint32_t e = (ax >> 23) - 112u;
        uint32_t h = (e << 10) | (mant >> 13);
        const uint32_t rem = mant & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
        r = (uint16_t)(s | h);
    } else {  // subnormal half or zero: round ax * 2^24 to an integer, ties to even
        float a;
        std::memcpy(&a, &ax, 4);
        const double q = (double)a * 16777216.0;
        double fl = (double)(uint32_t)q;
        const double rem = q - fl;
        uint32_t h = (uint32_t)fl;
        if (rem > 0.5 || (rem == 0.5 && (h & 1u))) ++h;
        r = (uint16_t)(s | h);
    }
    return __half{r};
}

inline float2 __half22float2(__half2 h) { return float2{__half2float(h.x), __half2float(h.y)}; }
inline __half2 __floats2half2_rn(float a, float b) { return __half2{__float2half(a), __float2half(b)}; }
inline __half __float2half_rn(float v) { return __float2half(v); }
