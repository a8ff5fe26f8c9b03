/*
 * oracle.c — CPU restatement of the reference's smoothquant -> quantized GEMM
 * path.  TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU
 * baseline.  Nothing in the product links, loads or calls this file.
 *
 * The reference (zhangnju/optimized_rocwmma_samples) is HIP + rocWMMA and
 * cannot be built here (no hipcc / rocWMMA), and its samples carry no CPU
 * check for this path.  This file restates, in plain C with the same fp32
 * operation order, what the reference kernels compute:
 *
 *   oracle_smoothquant      <- kernel_smoothquant, rocwmma_smoothquant.cpp:58-122
 *   oracle_moe_smoothquant  <- kernel_moe_smoothquant, rocwmma_moe_smoothquant.cpp:69-131
 *   oracle_gemm_i8_acc      <- gemm_cpu_h, common.hpp:307-345, instantiated with
 *                              InputT=int8, ComputeT=int32, alpha=1, beta=0
 *   oracle_dequant          <- the epilogue of gemm_quant_tensor_scale,
 *                              rocwmma_gemm_quantized.cpp:188-194, generalised to the
 *                              per-row x per-column mode of its header (:20, :26)
 *   oracle_topk_softmax     <- kernel_topk_softmax / kernel_topk_softmax_large,
 *                              rocwmma_topk_softmax.cpp:58-131 / :137-187
 *
 * Parity pins: the reference's own driver inputs (x = 0.5, s = 1 ->
 * y = 127, row_scale = 0.5f/127; rocwmma_smoothquant.cpp:140-141,
 * rocwmma_moe_smoothquant.cpp:152-153) are the only known answers the
 * reference holds; the GEMM has no reference-held vector ("parity unpinned"
 * for the GEMM beyond exact integer arithmetic).
 *
 * Build: gcc -O3 -fopenmp -ffp-contract=off (no -ffast-math), see Makefile.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- fp16 / bf16 conversions ------------------------------------------- */

/* IEEE binary16 -> binary32, exact (the reference's __half2float). */
float oracle_half_to_float(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; ++e; } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* binary32 -> binary16, round to nearest even (the epilogue's cvt.rn.f16.f32). */
uint16_t oracle_float_to_half(float f)
{
    _Float16 h = (_Float16)f; /* IEEE conversion, current rounding mode (RNE) */
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

/* binary32 -> bfloat16, round to nearest even (cvt.rn.bf16.f32). */
uint16_t oracle_float_to_bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* ---- smoothquant ------------------------------------------------------- */

/* One row: rocwmma_smoothquant.cpp:74-121 (and moe :93-130) in order. */
static void sq_row(const uint16_t* xrow, const float* srow, int8_t* yrow,
                   float* rs_out, uint32_t n, float qmax)
{
    float amax = 0.f;
    for (uint32_t c = 0; c < n; ++c)                       /* :83-84, :88 */
        amax = fmaxf(amax, fabsf(oracle_half_to_float(xrow[c]) * srow[c]));
    float rs = amax / qmax;                                /* :95 */
    *rs_out = rs;
    float inv = (rs > 0.f) ? (1.f / rs) : 0.f;             /* :98 */
    for (uint32_t c = 0; c < n; ++c) {                     /* :110-113, :119-120 */
        float v = oracle_half_to_float(xrow[c]) * srow[c] * inv;
        yrow[c] = (int8_t)fminf(fmaxf(rintf(v), -qmax), qmax);
    }
}

void oracle_smoothquant(const uint16_t* x, const float* smooth, int8_t* y,
                        float* row_scale, uint32_t M, uint32_t N, float qmax)
{
    long long m;
#pragma omp parallel for schedule(static)
    for (m = 0; m < (long long)M; ++m)
        sq_row(x + (size_t)m * N, smooth, y + (size_t)m * N, row_scale + m, N, qmax);
}

/* rocwmma_moe_smoothquant.cpp:81-130: output row flat = t*topk + k (optionally
 * permuted), invalid expert id -> row untouched (:86-87). */
void oracle_moe_smoothquant(const uint16_t* x, const float* smooth,
                            const int32_t* topk_ids, int8_t* qy, float* row_scale,
                            uint32_t tokens, uint32_t hidden, uint32_t topk,
                            uint32_t experts, float qmax, const int32_t* row_perm)
{
    long long flat;
#pragma omp parallel for schedule(static)
    for (flat = 0; flat < (long long)tokens * topk; ++flat) {
        uint32_t tok = (uint32_t)(flat / topk);
        int32_t eid = topk_ids[flat];
        if (eid < 0 || (uint32_t)eid >= experts) continue;
        long long r = row_perm ? row_perm[flat] : flat;
        if (r < 0) continue;
        sq_row(x + (size_t)tok * hidden, smooth + (size_t)eid * hidden,
               qy + (size_t)r * hidden, row_scale + r, hidden, qmax);
    }
}

/* ---- int8 GEMM --------------------------------------------------------- */

/*
 * acc[i*ldacc + j] = sum_h a(i,h) * b(h,j), exact int32 (wrapping, like the
 * hardware's non-saturating accumulate).  la/lb: 0 = row-major, 1 = col-major,
 * with gemm_cpu_h's index maps (common.hpp:325-331): row-major (r,c) -> r*ld+c,
 * col-major (r,c) -> c*ld+r.  Operands are first packed K-contiguous so the
 * inner loop is a plain dot product.
 */
void oracle_gemm_i8_acc(uint32_t M, uint32_t N, uint32_t K,
                        const int8_t* a, int la, uint32_t lda,
                        const int8_t* b, int lb, uint32_t ldb,
                        int32_t* acc, uint32_t ldacc)
{
    int8_t* ap = (int8_t*)malloc((size_t)M * K + 1);
    int8_t* bp = (int8_t*)malloc((size_t)N * K + 1);
    long long i;
#pragma omp parallel for schedule(static)
    for (i = 0; i < (long long)M; ++i)
        for (uint32_t h = 0; h < K; ++h)
            ap[(size_t)i * K + h] = la == 0 ? a[(size_t)i * lda + h] : a[(size_t)h * lda + i];
    long long j;
#pragma omp parallel for schedule(static)
    for (j = 0; j < (long long)N; ++j)
        for (uint32_t h = 0; h < K; ++h)
            bp[(size_t)j * K + h] = lb == 0 ? b[(size_t)h * ldb + j] : b[(size_t)j * ldb + h];
#pragma omp parallel for schedule(dynamic, 4)
    for (i = 0; i < (long long)M; ++i) {
        const int8_t* ar = ap + (size_t)i * K;
        for (uint32_t jj = 0; jj < N; ++jj) {
            const int8_t* br = bp + (size_t)jj * K;
            int32_t s = 0;
            for (uint32_t h = 0; h < K; ++h)
                s += (int32_t)ar[h] * (int32_t)br[h];
            acc[(size_t)i * ldacc + jj] = s;
        }
    }
    free(ap);
    free(bp);
}

/*
 * Epilogue, rocwmma_gemm_quantized.cpp:189-193: out = cvt_rn(float(acc) * (sa*sb))
 * with sa = sa_row ? sa_row[i] : scale_a, sb = sb_col ? sb_col[j] : scale_b.
 * out_dtype: 0 = fp16, 1 = bf16 (16-bit outputs, row-major, ld = ldc).
 */
void oracle_dequant(uint32_t M, uint32_t N, const int32_t* acc, uint32_t ldacc,
                    const float* sa_row, const float* sb_col,
                    float scale_a, float scale_b, uint16_t* out, int out_dtype,
                    uint32_t ldc)
{
    long long i;
#pragma omp parallel for schedule(static)
    for (i = 0; i < (long long)M; ++i) {
        float sa = sa_row ? sa_row[i] : scale_a;
        for (uint32_t j = 0; j < N; ++j) {
            float sb = sb_col ? sb_col[j] : scale_b;
            float ab = sa * sb;
            float v = (float)acc[(size_t)i * ldacc + j] * ab;
            out[(size_t)i * ldc + j] = out_dtype == 0 ? oracle_float_to_half(v)
                                                      : oracle_float_to_bf16(v);
        }
    }
}

/* ---- MoE routing: softmax + top-k --------------------------------------- */

/*
 * exp(a) for the router, evaluated with IEEE fp32 adds, multiplies and fmas
 * only, so that this file and the device kernel (moe_route.cu) produce the
 * same bits.  Method: Cody-Waite range reduction a = k*ln2 + r, |r| <= ~ln2/2,
 * with ln2 split into a 16-bit head (k*head exact for |k| <= 256) and an fp32
 * tail; e^r by its Taylor series to degree 8 (coefficients 1/n! rounded to
 * fp32; truncation error < 3e-10 relative), Horner with fma; then 2^k applied
 * as two exact power-of-two factors so a subnormal result is rounded once.
 * Accuracy: within 1 ulp of the exact exponential (0.84 ulp worst over 450k
 * samples of [-104, 88.7] against double precision).
 * The reference calls the platform expf (rocwmma_topk_softmax.cpp:84, :101),
 * which is itself not correctly rounded; probabilities therefore agree with
 * any reference build to a few ulp, and with the device kernel bit for bit.
 */
float oracle_route_exp(float a)
{
    if (a != a) return a;
    a = fminf(fmaxf(a, -104.0f), 89.0f);
    float k = rintf(a * 0x1.715476p+0f);
    float r = fmaf(-k, 0x1.62e4p-1f, a);
    r = fmaf(-k, 0x1.7f7d1cp-20f, r);
    float p = 0x1.a01a02p-16f;
    p = fmaf(p, r, 0x1.a01a02p-13f);
    p = fmaf(p, r, 0x1.6c16c2p-10f);
    p = fmaf(p, r, 0x1.111112p-7f);
    p = fmaf(p, r, 0x1.555556p-5f);
    p = fmaf(p, r, 0x1.555556p-3f);
    p = fmaf(p, r, 0x1.0p-1f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ki = (int)k;
    int k1 = ki / 2, k2 = ki - k1;
    uint32_t b1 = (uint32_t)(k1 + 127) << 23, b2 = (uint32_t)(k2 + 127) << 23;
    float s1, s2;
    memcpy(&s1, &b1, 4);
    memcpy(&s2, &b2, 4);
    return (p * s1) * s2;
}

/*
 * rocwmma_topk_softmax.cpp:58-131 (experts <= 64) and :137-187 (experts > 64),
 * restated for one token at a time with the reference's wave64 arithmetic
 * order made explicit: virtual lane l (0..63) owns experts l, l+64, ...; the
 * cross-lane max / sum / arg-max use the shfl_down tree (offsets 32..1), in
 * which lane 0 combines lane l with lane l+off for l < off.
 *   max:   fmaxf over all experts (:74-80)
 *   sum:   per-lane running sum of exp(x - max) from 0, then the tree (:83-90)
 *   inv:   sum > 0 ? 1/sum : 0 (:92)
 *   prob:  exp(x - max) * inv (:103)
 *   top-k, experts <= 64 (:108-129): min(topk, experts) rounds of the tree
 *          arg-max ("other > self" keeps lane l over lane l+off on ties and a
 *          NaN in place; with lanes masked, a tie can go to a higher id, e.g.
 *          picks 0, 4, 2 for eight equal logits), the winner written and masked to -1; lanes >= experts
 *          hold -1.  Slots beyond min(topk, experts) are left unwritten.
 *   top-k, experts > 64 (:160-186): only experts 0..63 are candidates; each of
 *          the topk rounds scans them in order for the first value > the
 *          running best (start -1), writes (-1, -1) when none qualifies, and
 *          masks the winner.
 */
void oracle_topk_softmax(const uint16_t* logits, float* topk_w, int32_t* topk_i,
                         uint32_t tokens, uint32_t experts, uint32_t topk)
{
    long long t;
#pragma omp parallel for schedule(static)
    for (t = 0; t < (long long)tokens; ++t) {
        const uint16_t* row = logits + (size_t)t * experts;
        float* ow = topk_w + (size_t)t * topk;
        int32_t* oi = topk_i + (size_t)t * topk;
        float mx = -INFINITY;
        for (uint32_t e = 0; e < experts; ++e) mx = fmaxf(mx, oracle_half_to_float(row[e]));
        float lane[64];
        for (int l = 0; l < 64; ++l) lane[l] = 0.0f;
        for (uint32_t e = 0; e < experts; ++e)
            lane[e % 64] = lane[e % 64] + oracle_route_exp(oracle_half_to_float(row[e]) - mx);
        for (int off = 32; off > 0; off >>= 1)
            for (int l = 0; l < off; ++l) lane[l] = lane[l] + lane[l + off];
        float sum = lane[0];
        float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
        uint32_t cand = experts < 64 ? experts : 64;
        float prob[64];
        for (uint32_t l = 0; l < 64; ++l)
            prob[l] = l < cand ? oracle_route_exp(oracle_half_to_float(row[l]) - mx) * inv : -1.0f;
        if (experts <= 64) {
            for (uint32_t k = 0; k < topk && k < experts; ++k) {
                float v[64];
                int who[64];
                for (int l = 0; l < 64; ++l) { v[l] = prob[l]; who[l] = l; }
                for (int off = 32; off > 0; off >>= 1)
                    for (int l = 0; l < off; ++l)
                        if (v[l + off] > v[l]) { v[l] = v[l + off]; who[l] = who[l + off]; }
                ow[k] = v[0];
                oi[k] = who[0] < (int)experts ? who[0] : 0;
                prob[who[0]] = -1.0f;
            }
        } else {
            for (uint32_t k = 0; k < topk; ++k) {
                float best = -1.0f;
                int at = -1;
                for (int l = 0; l < 64; ++l)
                    if (prob[l] > best) { best = prob[l]; at = l; }
                ow[k] = best;
                oi[k] = at;
                if (at >= 0) prob[at] = -1.0f;
            }
        }
    }
}

/* Thread count of the parallel loops started from the calling thread
 * (torchrun sets OMP_NUM_THREADS=1 in every rank; the timed CPU baseline
 * sets it back to the host's core count). */
void oracle_set_num_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int oracle_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
