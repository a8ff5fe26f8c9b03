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
// pass 2 to quantise).  Here every row is read from HBM once: small inputs by
// register-resident row groups (128-bit non-allocating loads, warp-shuffle
// absmax), large inputs by a persistent kernel that stages whole rows in
// shared memory with bulk TMA copies and writes whole int8 rows with bulk TMA
// stores.
// The MoE kernel reads each token row once for all of its top-k slots (the
// reference re-reads it per slot).
#include "common.cuh"
#include "kernels.h"
#include "sq_math.cuh"

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

// Packed pair multiply of sm_100 (mul.rn.f32x2): each lane is rounded exactly
// like the scalar .rn multiply, at half the issue cost.  Used only where the
// product feeds a max, never an add (an add could be contracted with it).
__device__ __forceinline__ uint64_t f2_pack(float a, float b)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b)
{
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b)
{
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// xs[i] = x[i] * s[i] for one 8-wide vector, in pairs.
__device__ __forceinline__ void scale8_pairs(const float (&xf)[8], const float (&sv)[8], float (&xs)[8])
{
#pragma unroll
    for (int i = 0; i < 8; i += 2)
        f2_unpack(f2_mul(f2_pack(xf[i], xf[i + 1]), f2_pack(sv[i], sv[i + 1])), xs[i], xs[i + 1]);
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

// Eight quantised values of one 16-byte input vector, packed into 8 bytes.
__device__ __forceinline__ uint2 quantize8(const float (&xs)[8], float inv, float qmax, bool integral_qmax)
{
    uint2 o;
    if (integral_qmax) {
        o.x = pack_low_bytes(quant_bits(xs[0], inv, qmax), quant_bits(xs[1], inv, qmax), quant_bits(xs[2], inv, qmax),
                             quant_bits(xs[3], inv, qmax));
        o.y = pack_low_bytes(quant_bits(xs[4], inv, qmax), quant_bits(xs[5], inv, qmax), quant_bits(xs[6], inv, qmax),
                             quant_bits(xs[7], inv, qmax));
    } else {
        o.x = pack4(quant1(xs[0], inv, qmax), quant1(xs[1], inv, qmax), quant1(xs[2], inv, qmax),
                    quant1(xs[3], inv, qmax));
        o.y = pack4(quant1(xs[4], inv, qmax), quant1(xs[5], inv, qmax), quant1(xs[6], inv, qmax),
                    quant1(xs[7], inv, qmax));
    }
    return o;
}

// quantize8 for rows row_absmax() marked fast: |xs * inv| <= qmax(1 + 3 ulp),
// so round-to-nearest-even by the 1.5 * 2^23 addition alone gives
// clamp(rint(v)) exactly (qmax is an integer, so rint(v) never passes it).
__device__ __forceinline__ uint2 quantize8_fast(const float (&xs)[8], float inv)
{
    // Scalar __fmul_rn / __fadd_rn: they are never contracted into an FMA,
    // whose single rounding would differ from the reference's two on
    // near-ties (packed f32x2 pairs are not safe here).
    uint32_t b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = __float_as_uint(__fadd_rn(__fmul_rn(xs[i], inv), 12582912.0f));
    return make_uint2(pack_low_bytes(b[0], b[1], b[2], b[3]), pack_low_bytes(b[4], b[5], b[6], b[7]));
}

// Quantises one register-resident row slice and stores it.  Called by all
// G threads of a row group.
template <int G, int VPT>
__device__ __forceinline__ void quantize_store(const float (&xs)[VPT][8], float amax, int8_t* yrow, float* rs_out,
                                               uint32_t nvec, float qmax, bool row_ok, int lane_in_group)
{
    const float rs = row_scale_of(amax, qmax);
    if (row_ok && lane_in_group == 0) *rs_out = rs;
    const float inv = inv_scale_of(rs);
    const bool integral_qmax = (qmax == truncf(qmax));
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const uint32_t v = j * G + lane_in_group;
        if (row_ok && v < nvec) *reinterpret_cast<uint2*>(yrow + (size_t)v * 8) = quantize8(xs[j], inv, qmax, integral_qmax);
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
    griddep_wait();               // the previous kernel's writes are visible from here on
    griddep_launch_dependents();  // then a PDL-launched consumer may start its prologue
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
    griddep_wait();               // the previous kernel's writes are visible from here on
    griddep_launch_dependents();  // then a PDL-launched consumer may start its prologue
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

// ---------------------------------------------------------------------------
// Streaming variant for large inputs: persistent CTAs; whole fp16 rows are
// staged into a ring of shared-memory buffers by 1-D bulk TMA copies
// (cp.async.bulk) that a producer warp keeps several rows ahead, so HBM
// always has rows in flight while eight consumer warps reduce and quantise.
// Each consumer thread owns the same columns of every row, so its smooth
// scales live in registers.  Quantised rows are assembled in one of two
// shared-memory rows and written by a single bulk store (whole-row writes).
// ---------------------------------------------------------------------------
constexpr int kTmaConsumers = 256;  // 8 warps
constexpr int kTmaThreads = kTmaConsumers + 32;
constexpr int kTmaMaxStages = 8;
constexpr uint32_t kTmaReserved = 512;  // barriers, reduction slots, abort flag

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void bulk_store(void* dst, uint32_t src, uint32_t bytes)
{
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most one bulk store group still reads shared memory.
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's shared-memory writes before later async-proxy (TMA) reads.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void sts64(uint32_t addr, uint2 v)
{
    asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(addr), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t addr)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

struct TmaRing {
    uint32_t data;   // smem address of stage 0
    uint32_t full;   // kTmaMaxStages barriers
    uint32_t empty;  // kTmaMaxStages barriers
    float* red;      // [2 parities][2 reductions][8 warps] per-warp maxima
    volatile int* abort;
};

__device__ __forceinline__ TmaRing tma_ring(uint8_t* smem, uint32_t stages, uint32_t stage_bytes)
{
    TmaRing r;
    r.data = smem_u32(smem);
    const uint32_t bars = r.data + stages * stage_bytes;
    r.full = bars;
    r.empty = bars + 8 * kTmaMaxStages;
    r.red = reinterpret_cast<float*>(smem + stages * stage_bytes + 16 * kTmaMaxStages);
    r.abort = reinterpret_cast<volatile int*>(smem + stages * stage_bytes + 16 * kTmaMaxStages + 128);
    return r;
}

__device__ __forceinline__ void tma_ring_init(const TmaRing& r, uint32_t stages)
{
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < stages; ++s) {
            mbar_init(r.full + 8 * s, 1);
            mbar_init(r.empty + 8 * s, kTmaConsumers / 32);
        }
        *r.abort = 0;
        fence_barrier_init();
    }
    __syncthreads();
}

// Producer loop: row i of this CTA is global row blockIdx.x + i * gridDim.x.
__device__ __forceinline__ void tma_produce(const TmaRing& r, const __half* x, uint64_t rows, uint32_t row_elems,
                                            uint32_t stages, uint32_t stage_bytes)
{
    const uint32_t bytes = row_elems * 2;
    uint32_t i = 0;
    for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x, ++i) {
        const uint32_t s = i % stages, ph = (i / stages) & 1;
        if (!mbar_wait(r.empty + 8 * s, ph ^ 1, SITE_SQ_PRODUCER, r.abort)) return;
        mbar_arrive_expect_tx(r.full + 8 * s, bytes);
        bulk_load(r.data + s * stage_bytes, x + row * row_elems, bytes, r.full + 8 * s);
    }
    // Drain the copies still in flight before the CTA may exit.
    for (uint32_t k = i > stages ? i - stages : 0; k < i; ++k)
        mbar_wait(r.full + 8 * (k % stages), (k / stages) & 1, SITE_SQ_DRAIN, nullptr);
}

// Consumer side: wait for row i, copy this thread's vectors to registers and
// release the stage.  Returns false if the wait gave up.
template <int VPT>
__device__ __forceinline__ bool tma_consume(const TmaRing& r, uint32_t i, uint32_t stages, uint32_t stage_bytes,
                                            uint32_t nvec, uint4 (&raw)[VPT])
{
    const uint32_t s = i % stages, ph = (i / stages) & 1;
    if (!mbar_wait(r.full + 8 * s, ph, SITE_SQ_CONSUMER, r.abort)) return false;
    const uint32_t base = r.data + s * stage_bytes;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const uint32_t v = j * kTmaConsumers + threadIdx.x;
        raw[j] = v < nvec ? lds128(base + v * 16) : make_uint4(0, 0, 0, 0);
    }
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(r.empty + 8 * s);
    return true;
}

// max that returns NaN if either operand is NaN (fmaxf ignores NaN).
__device__ __forceinline__ float max_nan(float a, float b)
{
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// Block-wide max over the 8 consumer warps.  slot selects one of four 8-float
// areas, (row parity, reduction), so each reduction of a row needs a single
// barrier.  kNanProp chooses max.NaN (propagating) or fmaxf (ignoring).
template <bool kNanProp>
__device__ __forceinline__ float consumers_max(float v, float* red, uint32_t slot)
{
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float o = __shfl_xor_sync(0xffffffffu, v, off);
        v = kNanProp ? max_nan(v, o) : fmaxf(v, o);
    }
    if ((threadIdx.x & 31) == 0) red[slot * 8 + (threadIdx.x >> 5)] = v;
    named_bar_sync(1, kTmaConsumers);
    float m = red[slot * 8];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = kNanProp ? max_nan(m, red[slot * 8 + w]) : fmaxf(m, red[slot * 8 + w]);
    return m;
}

// Row absmax with the reference's NaN-ignoring fmaxf (:83-84), computed the
// cheap way: a NaN-propagating max first; only a row holding a NaN pays a
// second, NaN-ignoring reduction.  *fast tells the caller that the row is
// free of NaN and +-inf products and its reciprocal scale is finite, so every
// x*s*inv lies within qmax*(1 + 3 ulp) and needs no clamping.
template <int VPT>
__device__ __forceinline__ float row_absmax(const float (&xs)[VPT][8], float* red, uint32_t parity, float qmax,
                                            bool* fast)
{
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j)
#pragma unroll
        for (int k = 0; k < 8; ++k) a = max_nan(a, fabsf(xs[j][k]));
    float amax = consumers_max<true>(a, red, parity * 2);
    const bool has_nan = amax != amax;
    if (has_nan) {  // block-uniform
        a = 0.f;
#pragma unroll
        for (int j = 0; j < VPT; ++j)
#pragma unroll
            for (int k = 0; k < 8; ++k) a = fmaxf(a, fabsf(xs[j][k]));
        amax = consumers_max<false>(a, red, parity * 2 + 1);
    }
    const float inv = inv_scale_of(row_scale_of(amax, qmax));
    *fast = !has_nan && isfinite(amax) && isfinite(inv) && qmax == truncf(qmax);
    return amax;
}

// Quantises a row held by the 256 consumer threads and writes it out.  With
// out_bytes != 0 (row length a multiple of 16 bytes, y 16-byte aligned) the
// int8 row is assembled in one of two shared-memory rows and written by one
// bulk store; otherwise each thread stores its 8-byte pieces.
template <int VPT>
__device__ __forceinline__ void tma_quantize_out(const float (&xs)[VPT][8], float amax, bool fast, int8_t* yrow,
                                                 float* rs_out, uint32_t nvec, float qmax, bool ok, uint32_t out_buf,
                                                 uint32_t out_bytes)
{
    if (out_bytes == 0) {
        quantize_store<kTmaConsumers, VPT>(xs, amax, yrow, rs_out, nvec, qmax, ok, threadIdx.x);
        return;
    }
    const float rs = row_scale_of(amax, qmax);
    const float inv = inv_scale_of(rs);
    const bool integral_qmax = (qmax == truncf(qmax));
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const uint32_t v = j * kTmaConsumers + threadIdx.x;
        if (v < nvec) sts64(out_buf + v * 8, fast ? quantize8_fast(xs[j], inv) : quantize8(xs[j], inv, qmax, integral_qmax));
    }
    fence_proxy_async_smem();
    named_bar_sync(2, kTmaConsumers);
    if (threadIdx.x == 0) {
        if (ok) {
            *rs_out = rs;
            bulk_store(yrow, out_buf, out_bytes);
        }
        // The other buffer is rewritten for the next row only after this
        // thread reaches that row's first barrier, i.e. after this wait.
        bulk_wait_read_1();
    }
}

template <int VPT>
__global__ void __launch_bounds__(kTmaThreads) sq_tma_kernel(const __half* __restrict__ x,
                                                             const float* __restrict__ smooth,
                                                             int8_t* __restrict__ y, float* __restrict__ row_scale,
                                                             uint32_t M, uint32_t N, float qmax, uint32_t stages,
                                                             uint32_t stage_bytes, uint32_t out_bytes)
{
    griddep_wait();               // the previous kernel's writes are visible from here on
    griddep_launch_dependents();  // then a PDL-launched consumer may start its prologue
    extern __shared__ __align__(128) uint8_t smem[];
    const TmaRing r = tma_ring(smem, stages, stage_bytes);
    const uint32_t out_base = r.data + stages * stage_bytes + kTmaReserved;
    const uint32_t out_stride = (out_bytes + 127) & ~127u;
    tma_ring_init(r, stages);
    const uint32_t nvec = N / 8;
    if (threadIdx.x >= kTmaConsumers) {
        if (threadIdx.x == kTmaConsumers) tma_produce(r, x, M, N, stages, stage_bytes);
        return;
    }
    float sv[VPT][8];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const uint32_t v = j * kTmaConsumers + threadIdx.x;
        if (v < nvec) {
            const float4 s0 = __ldg(reinterpret_cast<const float4*>(smooth + (size_t)v * 8));
            const float4 s1 = __ldg(reinterpret_cast<const float4*>(smooth + (size_t)v * 8) + 1);
            sv[j][0] = s0.x, sv[j][1] = s0.y, sv[j][2] = s0.z, sv[j][3] = s0.w;
            sv[j][4] = s1.x, sv[j][5] = s1.y, sv[j][6] = s1.z, sv[j][7] = s1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) sv[j][i] = 0.f;
        }
    }
    uint32_t i = 0;
    for (uint64_t row = blockIdx.x; row < M; row += gridDim.x, ++i) {
        uint4 raw[VPT];
        if (!tma_consume<VPT>(r, i, stages, stage_bytes, nvec, raw)) break;
        float xs[VPT][8];
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
            float xf[8];
            unpack8(raw[j], xf);
            scale8_pairs(xf, sv[j], xs[j]);
        }
        bool fast;
        const float amax = row_absmax<VPT>(xs, r.red, i & 1, qmax, &fast);
        tma_quantize_out<VPT>(xs, amax, fast, y + row * N, row_scale + row, nvec, qmax, true,
                              out_base + (i & 1) * out_stride, out_bytes);
    }
    if (threadIdx.x == 0) bulk_wait_all();
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
    griddep_wait();               // the previous kernel's writes are visible from here on
    griddep_launch_dependents();  // then a PDL-launched consumer may start its prologue
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
    griddep_wait();               // the previous kernel's writes are visible from here on
    griddep_launch_dependents();  // then a PDL-launched consumer may start its prologue
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

// Register-resident configuration for rows of nvec 16-byte vectors: the
// smallest group G (a power of two in [32, 256]) that covers the row with at
// most 4 vectors per thread, more only when G = 256 is not enough.  Four
// 16-byte loads in flight per thread measured best on B200 at the
// reference's sizes (3328 rows of 1024..4096, MoE 3328 x 4096): fewer
// threads per row, fewer CTAs and waves, and no block barrier below G = 64.
bool pick_cfg(uint32_t nvec, VecCfg& cfg)
{
    uint32_t g = 32;
    while (g < 256 && g * 4 < nvec) g <<= 1;
    const uint32_t vpt = (nvec + g - 1) / g;
    if (vpt > 8) return false;
    cfg = {(int)g, (int)(vpt ? vpt : 1)};
    return true;
}

template <int G, int VPT>
cudaError_t launch_sq(const __half* x, const float* s, int8_t* y, float* rs, uint32_t M, uint32_t N, float qmax,
                      cudaStream_t st)
{
    constexpr int R = kThreads / G;
    const uint64_t blocks = ((uint64_t)M + R - 1) / R;
    return launch_pdl(sq_vec_kernel<G, VPT>, dim3((unsigned)blocks), dim3(kThreads), 0, st, x, s, y, rs, M, N, qmax);
}

template <int G, int VPT>
cudaError_t launch_moe(const __half* x, const float* s, const int32_t* ids, int8_t* qy, float* rs, uint32_t T,
                       uint32_t H, uint32_t K, uint32_t E, float qmax, const int32_t* perm, cudaStream_t st)
{
    constexpr int R = kThreads / G;
    const uint64_t blocks = ((uint64_t)T + R - 1) / R;
    return launch_pdl(moe_sq_vec_kernel<G, VPT>, dim3((unsigned)blocks), dim3(kThreads), 0, st, x, s, ids, qy, rs, T, H,
                      K, E, qmax, perm);
}

#define B2SQ_VEC_DISPATCH(FN, ...)                                        \
    switch (cfg.G * 16 + cfg.VPT) {                                       \
        case 32 * 16 + 1: return FN<32, 1>(__VA_ARGS__);              \
        case 32 * 16 + 2: return FN<32, 2>(__VA_ARGS__);              \
        case 32 * 16 + 3: return FN<32, 3>(__VA_ARGS__);              \
        case 32 * 16 + 4: return FN<32, 4>(__VA_ARGS__);              \
        case 64 * 16 + 3: return FN<64, 3>(__VA_ARGS__);              \
        case 64 * 16 + 4: return FN<64, 4>(__VA_ARGS__);              \
        case 128 * 16 + 3: return FN<128, 3>(__VA_ARGS__);            \
        case 128 * 16 + 4: return FN<128, 4>(__VA_ARGS__);            \
        case 256 * 16 + 3: return FN<256, 3>(__VA_ARGS__);            \
        case 256 * 16 + 4: return FN<256, 4>(__VA_ARGS__);            \
        case 256 * 16 + 5: return FN<256, 5>(__VA_ARGS__);            \
        case 256 * 16 + 6: return FN<256, 6>(__VA_ARGS__);            \
        case 256 * 16 + 7: return FN<256, 7>(__VA_ARGS__);            \
        case 256 * 16 + 8: return FN<256, 8>(__VA_ARGS__);            \
        default: return cudaErrorInvalidValue;                            \
    }

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

unsigned generic_grid(uint64_t rows)
{
    const uint64_t cap = 148ull * 16;
    return (unsigned)(rows < cap ? (rows ? rows : 1) : cap);
}

}  // namespace

// ------------------------------------------------------------- streaming path
namespace {

// Inputs of at least this many elements (rows of 8192+) take the streaming
// kernel (crossover measured on B200: at 3328 x 4096 the register-resident
// kernel is faster, from 3328 x 8192 up the streaming one).
constexpr uint64_t kTmaMinElems = 1ull << 24;
constexpr uint32_t kTmaRingBytes = 110 * 1024;   // rows up to half of this take the streaming kernel
constexpr uint32_t kTmaRingTarget = 52 * 1024;   // input ring per CTA

struct TmaCfg {
    uint32_t stages, stage_bytes, out_bytes, smem;
};

// Input ring of whole fp16 rows, plus two int8 output rows when the output
// can be written by bulk stores (row bytes a multiple of 16, y 16-B aligned).
TmaCfg tma_cfg(uint32_t row_elems, const void* y)
{
    TmaCfg c;
    c.stage_bytes = (row_elems * 2 + 127) & ~127u;
    // About 52 KiB of ring, at least three rows: the consumers' per-row
    // latency, not the loads, bounds this kernel, so more resident CTAs (rows
    // being consumed at once) beat a deeper ring (measured at 16384 x 8192:
    // three 16 KiB stages, 3 CTAs per SM, 2.5% faster than six, 2 per SM).
    const uint32_t s = kTmaRingTarget / c.stage_bytes;
    c.stages = s < 3 ? 3 : (s > (uint32_t)kTmaMaxStages ? (uint32_t)kTmaMaxStages : s);
    c.out_bytes = (row_elems % 16 == 0 && aligned(y, 16)) ? row_elems : 0;
    c.smem = c.stages * c.stage_bytes + kTmaReserved + 2 * ((c.out_bytes + 127) & ~127u);
    return c;
}

// Grid of a persistent kernel: SM count x resident CTAs per SM, capped by the work.
template <typename Kern>
cudaError_t persistent_grid(Kern kern, uint32_t smem, uint64_t work, unsigned* grid)
{
    int dev = 0, sms = 0, per_sm = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTmaThreads, smem);
    if (e != cudaSuccess) return e;
    const uint64_t cap = (uint64_t)sms * (per_sm > 0 ? per_sm : 1);
    *grid = (unsigned)(work < cap ? work : cap);
    return cudaSuccess;
}

template <int VPT>
cudaError_t launch_sq_tma(const __half* x, const float* s, int8_t* y, float* rs, uint32_t M, uint32_t N, float qmax,
                          cudaStream_t st)
{
    const TmaCfg c = tma_cfg(N, y);
    unsigned grid = 0;
    cudaError_t e = persistent_grid(sq_tma_kernel<VPT>, c.smem, M, &grid);
    if (e != cudaSuccess) return e;
    return launch_pdl(sq_tma_kernel<VPT>, dim3(grid), dim3(kTmaThreads), c.smem, st, x, s, y, rs, M, N, qmax, c.stages,
                      c.stage_bytes, c.out_bytes);
}

#define B2SQ_TMA_DISPATCH(FN, VPT, ...)        \
    switch (VPT) {                             \
        case 1: return FN<1>(__VA_ARGS__);     \
        case 2: return FN<2>(__VA_ARGS__);     \
        case 3: return FN<3>(__VA_ARGS__);     \
        case 4: return FN<4>(__VA_ARGS__);     \
        case 5: return FN<5>(__VA_ARGS__);     \
        case 6: return FN<6>(__VA_ARGS__);     \
        case 7: return FN<7>(__VA_ARGS__);     \
        case 8: return FN<8>(__VA_ARGS__);     \
        default: return cudaErrorInvalidValue; \
    }

bool use_tma(uint64_t rows, uint32_t row_elems, uint32_t& vpt)
{
    const uint32_t nvec = row_elems / 8;
    vpt = (nvec + kTmaConsumers - 1) / kTmaConsumers;
    // Rows of 8192+ elements stream from 2^24 elements on; 4096-element rows
    // only from 2^27 (16384 x 4096: register-resident 47 us vs 51 streaming;
    // 65536 x 4096: 190 vs 178); shorter rows never (32768 x 2048: 45 vs 70).
    const uint64_t elems = rows * row_elems;
    const bool big = row_elems >= 8192 ? elems >= kTmaMinElems : row_elems >= 4096 && elems >= (kTmaMinElems << 3);
    return big && vpt >= 1 && vpt <= 8 && row_elems * 2 <= kTmaRingBytes / 2;
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
        return launch_pdl(sq_generic_kernel, dim3(generic_grid(M)), dim3(kThreads), 0, st, xh, s, y, rs, M, N, qmax);
    }
    uint32_t vpt = 0;
    if (use_tma(M, N, vpt)) {
        if (used_vector_path) *used_vector_path = 2;
        B2SQ_TMA_DISPATCH(launch_sq_tma, vpt, xh, s, y, rs, M, N, qmax, st)
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
        return launch_pdl(moe_sq_generic_kernel, dim3(generic_grid((uint64_t)T * K)), dim3(kThreads), 0, st, xh, s, ids, qy,
                          rs, T, H, K, E, qmax, perm);
    }
    // MoE uses the register-resident row groups at every size: a streaming
    // (TMA-staged) variant measured slower at every configuration tried (its
    // per-slot reductions are latency-bound; many tokens in flight win).
    B2SQ_VEC_DISPATCH(launch_moe, xh, s, ids, qy, rs, T, H, K, E, qmax, perm, st)
}

}  // namespace b2sq
