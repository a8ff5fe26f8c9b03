// moe_route.cu — MoE router (softmax over expert logits + top-k) for sm_100a.
//
// Replaces kernel_topk_softmax (rocwmma_topk_softmax.cpp:58-131, experts <=
// 64) and kernel_topk_softmax_large (:137-187, experts > 64), with the same
// outputs: topk_weights[t, k] (fp32 probability) and topk_indices[t, k].
//
// The reference runs one wave64 per token.  Its results depend on the wave's
// reduction order (the exp-sum) and on its tie rules (the arg-max), so this
// kernel reproduces that order exactly on 32-wide warps: virtual lane l of
// the wave (l = 0..63) owns experts l, l+64, ...; the shfl_down tree
// (offsets 32..1, lane l takes lane l+off for l < off) is evaluated with the
// offsets >= G inside a thread and the offsets < G across the G threads of a
// token's group.  Offsets >= the padded expert count P only meet padding
// (sum 0, probability -1), which leaves every value unchanged, so a token
// with P experts needs just log2(P) levels.
//
//   experts <= 64:  P = next power of two >= experts, V = min(P, 8) virtual
//                   lanes per thread (lanes j, j+G, ..., strided so the
//                   in-thread levels come first), G = P / V threads per
//                   token, 128 / G tokens per CTA.  min(topk, experts)
//                   rounds of the tree arg-max; "other > self" keeps lane
//                   l over lane l+off on ties and a NaN where it is
//                   (:112-116), so later picks among equal values follow
//                   the tree (0, 4, 2 for eight equal logits), not the id.
//   experts > 64:   one warp per token, virtual lanes t and t + 32; the
//                   per-lane sums run over e = l + 64 j in order (:146-148);
//                   only experts 0..63 are candidates and each of the topk
//                   rounds takes the first maximum greater than -1 (the
//                   reference's sequential scan, :165-175), (-1, -1) if none.
//
// exp() is route_exp below, a Cody-Waite + Taylor evaluation from IEEE
// add/mul/fma only, so the CPU checker computes the same bits.  The data are
// tiny (tokens * experts fp16 in, tokens * topk * 8 bytes out); the kernel is
// launch-bound and sized to finish in one wave of CTAs for the reference's
// token counts.
#include "common.cuh"
#include "kernels.h"

#include <cuda_fp16.h>

namespace b2sq {

namespace {

constexpr int kRouteThreads = 128;

// exp(a) from IEEE fp32 operations only.  a = k ln2 + r with k = rint(a
// log2 e) and ln2 split into a 16-bit head (k * head exact for |k| <= 256)
// plus an fp32 tail; e^r by its degree-8 Taylor polynomial (coefficients
// 1/n! rounded to fp32, truncation < 3e-10 relative on |r| <= 0.35) in
// Horner form with fma; 2^k applied as two normal power-of-two factors so a
// subnormal result is rounded exactly once.  Measured within 1 ulp of the
// exact exponential.  Clamping to [-104, 89] maps everything below to 0 and
// above to +inf, as the exact function rounds; NaN passes through.
__device__ __forceinline__ float route_exp(float a)
{
    if (a != a) return a;
    a = fminf(fmaxf(a, -104.0f), 89.0f);
    const float k = rintf(__fmul_rn(a, 0x1.715476p+0f));
    float r = __fmaf_rn(-k, 0x1.62e4p-1f, a);
    r = __fmaf_rn(-k, 0x1.7f7d1cp-20f, r);
    float p = 0x1.a01a02p-16f;
    p = __fmaf_rn(p, r, 0x1.a01a02p-13f);
    p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
    p = __fmaf_rn(p, r, 0x1.111112p-7f);
    p = __fmaf_rn(p, r, 0x1.555556p-5f);
    p = __fmaf_rn(p, r, 0x1.555556p-3f);
    p = __fmaf_rn(p, r, 0x1.0p-1f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ki = (int)k;
    const int k1 = ki / 2, k2 = ki - k1;
    return __fmul_rn(__fmul_rn(p, __int_as_float((k1 + 127) << 23)), __int_as_float((k2 + 127) << 23));
}

__device__ __forceinline__ float half_at(const __half* p) { return __half2float(*p); }

// experts <= 64.  P: padded expert count (power of two).
template <int P>
__global__ void __launch_bounds__(kRouteThreads) topk_softmax_kernel(const __half* __restrict__ logits,
                                                                     float* __restrict__ topk_w,
                                                                     int32_t* __restrict__ topk_i, uint32_t tokens,
                                                                     uint32_t experts, uint32_t topk)
{
    griddep_wait();  // logits may come from the previous kernel (PDL launch)
    griddep_launch_dependents();
    constexpr int V = P < 8 ? P : 8;  // virtual lanes per thread
    constexpr int G = P / V;          // threads per token
    const uint64_t gtid = (uint64_t)blockIdx.x * kRouteThreads + threadIdx.x;
    const uint64_t tok = gtid / G;
    const int j = (int)(threadIdx.x % G);
    if (tok >= tokens) return;  // whole groups leave together (G divides 32)
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t gmask = G == 32 ? 0xffffffffu : (((1u << G) - 1u) << (lane & ~(uint32_t)(G - 1)));

    const __half* row = logits + tok * experts;
    float x[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const uint32_t l = (uint32_t)(j + G * i);
        x[i] = l < experts ? half_at(row + l) : -INFINITY;
    }
    // max (:74-80): order-free, fmaxf drops NaN
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < V; ++i) mx = fmaxf(mx, x[i]);
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(gmask, mx, off, G));

    // exp-sum (:83-90) in the wave's tree order
    float e[V], s[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const uint32_t l = (uint32_t)(j + G * i);
        e[i] = l < experts ? route_exp(__fsub_rn(x[i], mx)) : 0.0f;
        s[i] = e[i];
    }
#pragma unroll
    for (int off = P / 2; off >= G; off >>= 1) {
#pragma unroll
        for (int i = 0; i < off / G; ++i) s[i] = __fadd_rn(s[i], s[i + off / G]);
    }
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) s[0] = __fadd_rn(s[0], __shfl_down_sync(gmask, s[0], off, G));
    const float sum = __shfl_sync(gmask, s[0], 0, G);
    const float inv = sum > 0.0f ? __frcp_rn(sum) : 0.0f;

    float prob[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const uint32_t l = (uint32_t)(j + G * i);
        prob[i] = l < experts ? __fmul_rn(e[i], inv) : -1.0f;
    }

    float* ow = topk_w + tok * topk;
    int32_t* oi = topk_i + tok * topk;
    const uint32_t rounds = topk < experts ? topk : experts;
    for (uint32_t k = 0; k < rounds; ++k) {
        float v[V];
        int who[V];
#pragma unroll
        for (int i = 0; i < V; ++i) {
            v[i] = prob[i];
            who[i] = j + G * i;
        }
#pragma unroll
        for (int off = P / 2; off >= G; off >>= 1) {
#pragma unroll
            for (int i = 0; i < off / G; ++i)
                if (v[i + off / G] > v[i]) {
                    v[i] = v[i + off / G];
                    who[i] = who[i + off / G];
                }
        }
#pragma unroll
        for (int off = G / 2; off > 0; off >>= 1) {
            const float ov = __shfl_down_sync(gmask, v[0], off, G);
            const int ow_ = __shfl_down_sync(gmask, who[0], off, G);
            if (ov > v[0]) {
                v[0] = ov;
                who[0] = ow_;
            }
        }
        const float best = __shfl_sync(gmask, v[0], 0, G);
        const int at = __shfl_sync(gmask, who[0], 0, G);
        if (j == 0) {
            ow[k] = best;
            oi[k] = (uint32_t)at < experts ? at : 0;  // lanes >= experts carry index 0 (:104-106)
        }
#pragma unroll
        for (int i = 0; i < V; ++i)
            if (j + G * i == at) prob[i] = -1.0f;
    }
}

// Scan order of the wide variant: candidate (b, ib) replaces (a, ia) when b
// qualifies (> -1, not NaN) and a does not, or b is larger, or equal with a
// lower index.
__device__ __forceinline__ bool takes(float b, int ib, float a, int ia)
{
    if (!(b > -1.0f)) return false;
    if (!(a > -1.0f)) return true;
    return b > a || (b == a && ib < ia);
}

// experts > 64: one warp per token.
__global__ void __launch_bounds__(kRouteThreads) topk_softmax_wide_kernel(const __half* __restrict__ logits,
                                                                          float* __restrict__ topk_w,
                                                                          int32_t* __restrict__ topk_i,
                                                                          uint32_t tokens, uint32_t experts,
                                                                          uint32_t topk)
{
    griddep_wait();
    griddep_launch_dependents();
    const uint64_t tok = ((uint64_t)blockIdx.x * kRouteThreads + threadIdx.x) >> 5;
    const uint32_t t = threadIdx.x & 31;
    if (tok >= tokens) return;
    const __half* row = logits + tok * experts;

    float mx = -INFINITY;
    for (uint32_t e = t; e < experts; e += 32) mx = fmaxf(mx, half_at(row + e));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));

    float lo = 0.0f, hi = 0.0f;  // virtual lanes t and t + 32
    for (uint32_t e = t; e < experts; e += 64) {
        lo = __fadd_rn(lo, route_exp(__fsub_rn(half_at(row + e), mx)));
        if (e + 32 < experts) hi = __fadd_rn(hi, route_exp(__fsub_rn(half_at(row + e + 32), mx)));
    }
    float s = __fadd_rn(lo, hi);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, off));
    const float sum = __shfl_sync(0xffffffffu, s, 0);
    const float inv = sum > 0.0f ? __frcp_rn(sum) : 0.0f;

    // candidates: experts 0..63 only (:160-164)
    float p0 = __fmul_rn(route_exp(__fsub_rn(half_at(row + t), mx)), inv);
    float p1 = __fmul_rn(route_exp(__fsub_rn(half_at(row + t + 32), mx)), inv);

    float* ow = topk_w + tok * topk;
    int32_t* oi = topk_i + tok * topk;
    for (uint32_t k = 0; k < topk; ++k) {
        // first index of the maximum among values > -1 (NaN never qualifies);
        // the tree meets interleaved lanes, so equal values compare indices
        float v = p0;
        int at = (int)t;
        if (takes(p1, (int)t + 32, v, at)) {
            v = p1;
            at = (int)t + 32;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_down_sync(0xffffffffu, v, off);
            const int oa = __shfl_down_sync(0xffffffffu, at, off);
            if (takes(ov, oa, v, at)) {
                v = ov;
                at = oa;
            }
        }
        v = __shfl_sync(0xffffffffu, v, 0);
        at = __shfl_sync(0xffffffffu, at, 0);
        if (!(v > -1.0f)) {
            v = -1.0f;
            at = -1;
        }
        if (t == 0) {
            ow[k] = v;
            oi[k] = at;
        }
        if (at == (int)t) p0 = -1.0f;
        if (at == (int)t + 32) p1 = -1.0f;
    }
}

template <int P>
cudaError_t launch_small(const __half* x, float* w, int32_t* idx, uint32_t tokens, uint32_t experts, uint32_t topk,
                         cudaStream_t st)
{
    constexpr int G = P / (P < 8 ? P : 8);
    const uint64_t threads = (uint64_t)tokens * G;
    const unsigned grid = (unsigned)((threads + kRouteThreads - 1) / kRouteThreads);
    return launch_pdl(topk_softmax_kernel<P>, dim3(grid), dim3(kRouteThreads), 0, st, x, w, idx, tokens, experts, topk);
}

}  // namespace

cudaError_t launch_topk_softmax(const void* logits, float* topk_w, int32_t* topk_i, uint32_t tokens,
                                uint32_t experts, uint32_t topk, cudaStream_t st)
{
    const __half* x = static_cast<const __half*>(logits);
    if (experts > 64) {
        const unsigned grid = (unsigned)(((uint64_t)tokens * 32 + kRouteThreads - 1) / kRouteThreads);
        return launch_pdl(topk_softmax_wide_kernel, dim3(grid), dim3(kRouteThreads), 0, st, x, topk_w, topk_i, tokens,
                          experts, topk);
    }
    if (experts <= 1) return launch_small<1>(x, topk_w, topk_i, tokens, experts, topk, st);
    if (experts <= 2) return launch_small<2>(x, topk_w, topk_i, tokens, experts, topk, st);
    if (experts <= 4) return launch_small<4>(x, topk_w, topk_i, tokens, experts, topk, st);
    if (experts <= 8) return launch_small<8>(x, topk_w, topk_i, tokens, experts, topk, st);
    if (experts <= 16) return launch_small<16>(x, topk_w, topk_i, tokens, experts, topk, st);
    if (experts <= 32) return launch_small<32>(x, topk_w, topk_i, tokens, experts, topk, st);
    return launch_small<64>(x, topk_w, topk_i, tokens, experts, topk, st);
}

}  // namespace b2sq
