// smoothquant.cu — per-token dynamic int8 quantisation with a per-channel
// smooth scale (dense and MoE per-expert variants) for sm_100a.
//
// Arithmetic follows the reference kernels operation for operation, in fp32:
//   kernel_smoothquant      rocwmma_smoothquant.cpp:74-121
//   kernel_moe_smoothquant  rocwmma_moe_smoothquant.cpp:81-130
//   xs = float(x) * s;  amax = max|xs|;  rs = amax / qmax;
//   inv = rs > 0 ? 1/rs : 0;  q = int8(fminf(fmaxf(rintf(xs * inv), -qmax), qmax))
// (IEEE division and round-to-nearest-even rint; the build has no fast-math.)
//
// Design (B200): the reference reads every row twice (pass 1 for the absmax,
// pass 2 to quantise).  Here a group of G threads owns a row, loads it ONCE
// with 128-bit non-allocating loads into registers, reduces the absmax with
// warp shuffles (+ one shared-memory exchange when G > 32) and quantises from
// registers with 64-bit int8 stores: one HBM read of x and one write of y.
// The MoE kernel reads each token row once for all of its top-k slots (the
// reference re-reads it per slot).
#include "common.cuh"
#include "kernels.h"

#include <cuda_fp16.h>

namespace b2sq {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint4 ld_stream_v4(const void* p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8])
{
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
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

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// Group-wide max for a group of G threads (G a power of two, 32..256) that
// share the block with other groups.  `red` holds kThreads/32 floats; `buf`
// selects one of two halves so consecutive calls need only one barrier.
template <int G>
__device__ __forceinline__ float group_max(float v, float* red)
{
    v = warp_max(v);
    if constexpr (G > 32) {
        const int warp = threadIdx.x >> 5;
        if ((threadIdx.x & 31) == 0) red[warp] = v;
        __syncthreads();
        const int first = (threadIdx.x / G) * (G / 32);
        float m = red[first];
#pragma unroll
        for (int i = 1; i < G / 32; ++i) m = fmaxf(m, red[first + i]);
        v = m;
    }
    return v;
}

// Smooth-scale product for one 8-wide vector: xs[i] = x[i] * s[i] (rounded fp32 multiply).
__device__ __forceinline__ void scale8(const float (&xf)[8], const float* s, float (&xs)[8])
{
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(s));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(s) + 1);
    xs[0] = __fmul_rn(xf[0], s0.x);
    xs[1] = __fmul_rn(xf[1], s0.y);
    xs[2] = __fmul_rn(xf[2], s0.z);
    xs[3] = __fmul_rn(xf[3], s0.w);
    xs[4] = __fmul_rn(xf[4], s1.x);
    xs[5] = __fmul_rn(xf[5], s1.y);
    xs[6] = __fmul_rn(xf[6], s1.z);
    xs[7] = __fmul_rn(xf[7], s1.w);
}

// Quantises one register-resident row slice and stores it.  Called by all
// G threads of a row group.
template <int G, int VPT>
__device__ __forceinline__ void quantize_store(const float (&xs)[VPT][8], float amax, int8_t* yrow, float* rs_out,
                                               uint32_t nvec, float qmax, bool row_ok, int lane_in_group)
{
    const float rs = amax / qmax;  // IEEE division, reference :95
    if (row_ok && lane_in_group == 0) *rs_out = rs;
    const float inv = (rs > 0.f) ? (1.f / rs) : 0.f;  // reference :98
    const bool integral_qmax = (qmax == truncf(qmax));
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const uint32_t v = j * G + lane_in_group;
        if (row_ok && v < nvec) {
            uint2 o;
            if (integral_qmax) {
                o.x = pack_low_bytes(quant_bits(xs[j][0], inv, qmax), quant_bits(xs[j][1], inv, qmax),
                                     quant_bits(xs[j][2], inv, qmax), quant_bits(xs[j][3], inv, qmax));
                o.y = pack_low_bytes(quant_bits(xs[j][4], inv, qmax), quant_bits(xs[j][5], inv, qmax),
                                     quant_bits(xs[j][6], inv, qmax), quant_bits(xs[j][7], inv, qmax));
            } else {
                o.x = pack4(quant1(xs[j][0], inv, qmax), quant1(xs[j][1], inv, qmax), quant1(xs[j][2], inv, qmax),
                            quant1(xs[j][3], inv, qmax));
                o.y = pack4(quant1(xs[j][4], inv, qmax), quant1(xs[j][5], inv, qmax), quant1(xs[j][6], inv, qmax),
                            quant1(xs[j][7], inv, qmax));
            }
            *reinterpret_cast<uint2*>(yrow + (size_t)v * 8) = o;
        }
    }
}

// Dense smoothquant, register-resident rows.  Requires N % 8 == 0, x 16-byte
// and y 8-byte aligned, N <= G * VPT * 8.
template <int G, int VPT>
__global__ void __launch_bounds__(kThreads) sq_vec_kernel(const __half* __restrict__ x,
                                                          const float* __restrict__ smooth,
                                                          int8_t* __restrict__ y, float* __restrict__ row_scale,
                                                          uint32_t M, uint32_t N, float qmax)
{
    __shared__ float red[kThreads / 32];
    constexpr int R = kThreads / G;
    const int lane_in_group = threadIdx.x % G;
    const uint64_t row = (uint64_t)blockIdx.x * R + threadIdx.x / G;
    const bool row_ok = row < M;
    const uint32_t nvec = N / 8;
    const __half* xrow = x + row * N;

    uint4 raw[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const uint32_t v = j * G + lane_in_group;
        raw[j] = (row_ok && v < nvec) ? ld_stream_v4(xrow + (size_t)v * 8) : make_uint4(0, 0, 0, 0);
    }
    float xs[VPT][8];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const uint32_t v = j * G + lane_in_group;
        float xf[8];
        unpack8(raw[j], xf);
        if (row_ok && v < nvec) {
            scale8(xf, smooth + (size_t)v * 8, xs[j]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) xs[j][i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(xs[j][i]));
    }
    amax = group_max<G>(amax, red);
    quantize_store<G, VPT>(xs, amax, y + row * N, row_scale + row, nvec, qmax, row_ok, lane_in_group);
}

// MoE smoothquant, one row group per token, the token row read once and
// quantised for each of its top-k slots with that slot's expert scale.
template <int G, int VPT>
__global__ void __launch_bounds__(kThreads) moe_sq_vec_kernel(const __half* __restrict__ x,
                                                              const float* __restrict__ smooth,
                                                              const int32_t* __restrict__ topk_ids,
                                                              int8_t* __restrict__ qy, float* __restrict__ row_scale,
                                                              uint32_t tokens, uint32_t hidden, uint32_t topk,
                                                              uint32_t experts, float qmax,
                                                              const int32_t* __restrict__ row_perm)
{
    __shared__ float red[2][kThreads / 32];
    constexpr int R = kThreads / G;
    const int lane_in_group = threadIdx.x % G;
    const uint64_t tok = (uint64_t)blockIdx.x * R + threadIdx.x / G;
    const bool tok_ok = tok < tokens;
    const uint32_t nvec = hidden / 8;
    const __half* xrow = x + tok * hidden;

    uint4 raw[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const uint32_t v = j * G + lane_in_group;
        raw[j] = (tok_ok && v < nvec) ? ld_stream_v4(xrow + (size_t)v * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll 1
    for (uint32_t k = 0; k < topk; ++k) {
        const uint64_t flat = tok * topk + k;
        int32_t eid = tok_ok ? __ldg(topk_ids + flat) : -1;
        int64_t r = (int64_t)flat;
        if (row_perm != nullptr && tok_ok) r = __ldg(row_perm + flat);
        const bool ok = tok_ok && eid >= 0 && (uint32_t)eid < experts && r >= 0;  // reference :86-87
        const float* srow = smooth + (size_t)(ok ? eid : 0) * hidden;
        float xs[VPT][8];
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
            const uint32_t v = j * G + lane_in_group;
            float xf[8];
            unpack8(raw[j], xf);
            if (ok && v < nvec) {
                scale8(xf, srow + (size_t)v * 8, xs[j]);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) xs[j][i] = 0.f;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(xs[j][i]));
        }
        amax = group_max<G>(amax, red[k & 1]);
        quantize_store<G, VPT>(xs, amax, qy + (size_t)r * hidden, row_scale + r, nvec, qmax, ok, lane_in_group);
    }
}

// Generic fallback: one block per output row, two passes over the row (the
// reference's own structure), any N and any alignment.  Used for N % 8 != 0,
// unaligned pointers and rows longer than the register-resident limit.
__device__ __forceinline__ float block_max(float v, float* red)
{
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = red[0];
#pragma unroll
    for (int i = 1; i < kThreads / 32; ++i) m = fmaxf(m, red[i]);
    __syncthreads();
    return m;
}

__device__ __forceinline__ void sq_row_generic(const __half* xrow, const float* srow, int8_t* yrow, float* rs_out,
                                               uint32_t N, float qmax, float* red)
{
    float amax = 0.f;
    for (uint32_t c = threadIdx.x; c < N; c += kThreads)
        amax = fmaxf(amax, fabsf(__fmul_rn(__half2float(xrow[c]), srow[c])));
    amax = block_max(amax, red);
    const float rs = amax / qmax;
    if (threadIdx.x == 0) *rs_out = rs;
    const float inv = (rs > 0.f) ? (1.f / rs) : 0.f;
    for (uint32_t c = threadIdx.x; c < N; c += kThreads)
        yrow[c] = quant1(__fmul_rn(__half2float(xrow[c]), srow[c]), inv, qmax);
}

__global__ void __launch_bounds__(kThreads) sq_generic_kernel(const __half* __restrict__ x,
                                                              const float* __restrict__ smooth,
                                                              int8_t* __restrict__ y, float* __restrict__ row_scale,
                                                              uint32_t M, uint32_t N, float qmax)
{
    __shared__ float red[kThreads / 32];
    for (uint64_t row = blockIdx.x; row < M; row += gridDim.x)
        sq_row_generic(x + row * N, smooth, y + row * N, row_scale + row, N, qmax, red);
}

__global__ void __launch_bounds__(kThreads) moe_sq_generic_kernel(const __half* __restrict__ x,
                                                                  const float* __restrict__ smooth,
                                                                  const int32_t* __restrict__ topk_ids,
                                                                  int8_t* __restrict__ qy,
                                                                  float* __restrict__ row_scale, uint32_t tokens,
                                                                  uint32_t hidden, uint32_t topk, uint32_t experts,
                                                                  float qmax, const int32_t* __restrict__ row_perm)
{
    __shared__ float red[kThreads / 32];
    const uint64_t total = (uint64_t)tokens * topk;
    for (uint64_t flat = blockIdx.x; flat < total; flat += gridDim.x) {
        const uint64_t tok = flat / topk;
        const int32_t eid = topk_ids[flat];
        if (eid < 0 || (uint32_t)eid >= experts) continue;  // block-uniform
        const int64_t r = row_perm ? (int64_t)row_perm[flat] : (int64_t)flat;
        if (r < 0) continue;
        sq_row_generic(x + tok * hidden, smooth + (size_t)eid * hidden, qy + (size_t)r * hidden, row_scale + r,
                       hidden, qmax, red);
    }
}

// --------------------------------------------------------------------------
// Host-side dispatch over the (G, VPT) instantiations.
// --------------------------------------------------------------------------
struct VecCfg {
    int G;
    int VPT;
};

// Smallest register-resident configuration holding nvec 16-byte vectors per row.
bool pick_cfg(uint32_t nvec, VecCfg& cfg)
{
    if (nvec <= 256) {
        int g = 32;
        while ((uint32_t)g < nvec) g <<= 1;
        cfg = {g, 1};
        return true;
    }
    const uint32_t vpt = (nvec + 255) / 256;
    if (vpt > 8) return false;
    cfg = {256, (int)vpt};
    return true;
}

template <int G, int VPT>
cudaError_t launch_sq(const __half* x, const float* s, int8_t* y, float* rs, uint32_t M, uint32_t N, float qmax,
                      cudaStream_t st)
{
    constexpr int R = kThreads / G;
    const uint64_t blocks = ((uint64_t)M + R - 1) / R;
    sq_vec_kernel<G, VPT><<<(unsigned)blocks, kThreads, 0, st>>>(x, s, y, rs, M, N, qmax);
    return cudaGetLastError();
}

template <int G, int VPT>
cudaError_t launch_moe(const __half* x, const float* s, const int32_t* ids, int8_t* qy, float* rs, uint32_t T,
                       uint32_t H, uint32_t K, uint32_t E, float qmax, const int32_t* perm, cudaStream_t st)
{
    constexpr int R = kThreads / G;
    const uint64_t blocks = ((uint64_t)T + R - 1) / R;
    moe_sq_vec_kernel<G, VPT><<<(unsigned)blocks, kThreads, 0, st>>>(x, s, ids, qy, rs, T, H, K, E, qmax, perm);
    return cudaGetLastError();
}

#define B2SQ_VEC_DISPATCH(FN, ...)                                        \
    switch (cfg.G * 16 + cfg.VPT) {                                       \
        case 32 * 16 + 1: return FN<32, 1>(__VA_ARGS__);                  \
        case 64 * 16 + 1: return FN<64, 1>(__VA_ARGS__);                  \
        case 128 * 16 + 1: return FN<128, 1>(__VA_ARGS__);                \
        case 256 * 16 + 1: return FN<256, 1>(__VA_ARGS__);                \
        case 256 * 16 + 2: return FN<256, 2>(__VA_ARGS__);                \
        case 256 * 16 + 3: return FN<256, 3>(__VA_ARGS__);                \
        case 256 * 16 + 4: return FN<256, 4>(__VA_ARGS__);                \
        case 256 * 16 + 5: return FN<256, 5>(__VA_ARGS__);                \
        case 256 * 16 + 6: return FN<256, 6>(__VA_ARGS__);                \
        case 256 * 16 + 7: return FN<256, 7>(__VA_ARGS__);                \
        case 256 * 16 + 8: return FN<256, 8>(__VA_ARGS__);                \
        default: return cudaErrorInvalidValue;                            \
    }

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

unsigned generic_grid(uint64_t rows)
{
    const uint64_t cap = 148ull * 16;
    return (unsigned)(rows < cap ? (rows ? rows : 1) : cap);
}

}  // namespace

cudaError_t launch_smoothquant(const void* x, const float* s, int8_t* y, float* rs, uint32_t M, uint32_t N, float qmax,
                               cudaStream_t st, int* used_vector_path)
{
    const __half* xh = static_cast<const __half*>(x);
    VecCfg cfg;
    const bool vec_ok = (N % 8 == 0) && aligned(x, 16) && aligned(y, 8) && aligned(s, 16) && pick_cfg(N / 8, cfg);
    if (used_vector_path) *used_vector_path = vec_ok ? 1 : 0;
    if (!vec_ok) {
        sq_generic_kernel<<<generic_grid(M), kThreads, 0, st>>>(xh, s, y, rs, M, N, qmax);
        return cudaGetLastError();
    }
    B2SQ_VEC_DISPATCH(launch_sq, xh, s, y, rs, M, N, qmax, st)
}

cudaError_t launch_moe_smoothquant(const void* x, const float* s, const int32_t* ids, int8_t* qy, float* rs,
                                   uint32_t T, uint32_t H, uint32_t K, uint32_t E, float qmax, const int32_t* perm,
                                   cudaStream_t st, int* used_vector_path)
{
    const __half* xh = static_cast<const __half*>(x);
    VecCfg cfg;
    const bool vec_ok = (H % 8 == 0) && aligned(x, 16) && aligned(qy, 8) && aligned(s, 16) && pick_cfg(H / 8, cfg);
    if (used_vector_path) *used_vector_path = vec_ok ? 1 : 0;
    if (!vec_ok) {
        moe_sq_generic_kernel<<<generic_grid((uint64_t)T * K), kThreads, 0, st>>>(xh, s, ids, qy, rs, T, H, K, E,
                                                                                  qmax, perm);
        return cudaGetLastError();
    }
    B2SQ_VEC_DISPATCH(launch_moe, xh, s, ids, qy, rs, T, H, K, E, qmax, perm, st)
}

}  // namespace b2sq
