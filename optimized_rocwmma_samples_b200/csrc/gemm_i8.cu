// gemm_i8.cu — int8 x int8 -> int32 GEMM with a fused per-row x per-column
// dequant epilogue, for sm_100a (tcgen05 kind::i8, TMEM accumulators, TMA).
//
// Replaces gemm_quant_tensor_scale (reference rocwmma_gemm_quantized.cpp:127-195).
// The reference kernel is a 128x128 macro tile, 2-stage LDS ping-pong, one
// CTA per output tile, with the epilogue fp16(float(acc) * (scale_a*scale_b))
// (:188-194).  This kernel keeps that arithmetic and generalises the scales
// to per-row / per-column vectors (the reference header's Mode 2, :20, :26);
// the machinery is Blackwell's:
//
//  * persistent CTAs (one per SM), warp specialised:
//      warp 0      TMA producer: 128-byte-swizzled A/B tiles into a ring of
//                  shared-memory stages (mbarrier full/empty pairs);
//      warp 1      MMA issuer: one thread issues tcgen05.mma.kind::i8
//                  (M=128, N=tile_n, K=32 per instruction) into an int32
//                  accumulator in tensor memory; tcgen05.commit frees stages;
//      warps 2..5  epilogue: tcgen05.ld of the accumulator, fp32 dequant,
//                  cvt.rn to fp16/bf16, stores.  Two TMEM accumulators
//                  alternate so the epilogue of tile i overlaps the main loop
//                  of tile i+1.
//  * a stage holds BK elements of K: 128 for square tiles, up to 512 for the
//    skinny (decode) tiles so every weight row is streamed in >= 256-byte
//    runs per stage.
//  * tile schedule: whole tiles in data-parallel rounds over the CTAs; when
//    the last round would leave many SMs idle, the tail tiles' k-blocks are
//    instead split evenly over all CTAs (stream-K, the scheme of
//    rocwmma_streamk_gemm.cpp:102-143).  A CTA stores each partial tile to
//    its own workspace slot (plain coalesced stores), then bumps the tile's
//    k-block counter; the CTA whose contribution completes the tile sums the
//    contributors' slots (int32, exact, order independent) and runs the
//    epilogue.  No CTA ever waits on another CTA, so the fix-up cannot hang.
//  * no TMA multicast anywhere (every CTA loads its own tiles).
#include "common.cuh"
#include "kernels.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>
#include <cstring>
#include <mutex>

namespace b2sq {

namespace {

#ifndef B2SQ_PAIR_TMA_STORE
#define B2SQ_PAIR_TMA_STORE 1  // pair-kernel output blocks leave by TMA bulk-tensor stores
#endif
#ifndef B2SQ_RASTER_GROUP
#define B2SQ_RASTER_GROUP 16  // M tiles per raster group
#endif

constexpr uint32_t kThreads = 192;  // 6 warps
constexpr uint32_t kEpiThreads = 128;
constexpr uint32_t kSmemBudget = 232448;  // 227 KiB opt-in limit per CTA
constexpr uint32_t kBarrierBytes = 256;
constexpr uint32_t kEpiStageBytes = 4 * 4096;  // 4 epilogue warps x (32 rows x 128 B)

// K depth of a pipeline stage for a tile width.
__host__ __device__ constexpr uint32_t tile_k_for(uint32_t bn) { return bn <= 32 ? 512 : bn <= 64 ? 256 : 128; }
__host__ __device__ constexpr uint32_t stage_bytes(uint32_t bn, uint32_t bk) { return (kTileM + bn) * bk; }
__host__ __device__ constexpr uint32_t num_stages(uint32_t bn, uint32_t bk)
{
    return ((kSmemBudget - 1024 - kBarrierBytes) / stage_bytes(bn, bk)) > 8
               ? 8
               : ((kSmemBudget - 1024 - kBarrierBytes) / stage_bytes(bn, bk));
}
__host__ __device__ constexpr uint32_t tmem_cols(uint32_t bn)
{
    return (2 * bn <= 32) ? 32 : (2 * bn <= 64) ? 64 : (2 * bn <= 128) ? 128 : (2 * bn <= 256) ? 256 : 512;
}

struct KParams {
    uint32_t Mk, Nk, K;
    uint32_t tiles_m, tiles_n, k_blocks;
    uint32_t dp_tiles, ctas;
    uint64_t sk_iters;
    uint32_t a_mn_major, b_mn_major;
    void* c;
    uint32_t ldc;
    int c_type;
    int transpose_out;
    int vec_store_ok;
    void* extra_c[kMaxExtraOut];  // further destinations of every store (all-gather)
    uint32_t n_extra;
    uint8_t* mc_c;  // multicast view of c (all-gather through NVSwitch), or null
    uint32_t tma_store;  // 1: the pair kernel's staged output pieces leave by TMA bulk-tensor stores
    const float* row_scale_vec;
    const float* col_scale_vec;
    float row_scale, col_scale;
    uint32_t* ws_cnt;   // [tail tiles] k-blocks accumulated so far (zero between calls)
    int32_t* ws_slots;  // [ctas][2][tile_n][128] int32 partial tiles (scratch)
    uint32_t raster_group;
    // Grouped (MoE) mode: group g owns rows [grp_start[g], grp_start[g] + grp_count[g])
    // of A and C, rows [g * Nk, (g + 1) * Nk) of B and entries [g * Nk, ...) of
    // the column scales.
    const int32_t* grp_start;
    const int32_t* grp_count;
    uint32_t groups;
    // Programmatic dependent launch: 0 none, 1 / 2 = the A / B operand (and the
    // row scales) are written by the kernel launched just before this one.
    uint32_t pdl_dep;
};

constexpr uint32_t kTileK_Grouped = tile_k_for(256);

// Where one tile reads and writes.
struct TileGeom {
    uint32_t a_row;    // first A row (TMA coordinate)
    uint32_t b_row;    // first B row
    uint32_t c_row;    // first C row of the tile
    uint32_t row_end;  // C rows at or beyond this are not written
    uint32_t col0;     // first C column
    uint32_t cs_off;   // offset of this tile's group in the column scales
};

struct Unit {
    uint32_t tile, k0, k1;
    uint32_t slot;  // 0: first stream-K unit of this CTA, 1: a later one
};

__host__ __device__ __forceinline__ uint64_t sk_start(uint64_t c, uint64_t S, uint64_t P) { return c * S / P; }

// Work list of one CTA: its data-parallel tiles, then its contiguous range of
// stream-K k-block iterations over the tail tiles.
struct UnitIter {
    uint32_t dp_next;
    uint64_t sk_pos, sk_begin, sk_end;

    uint32_t dp_total;

    __device__ __forceinline__ void init(const KParams& p) { init(p, p.dp_tiles); }
    __device__ __forceinline__ void init(const KParams& p, uint32_t dp_tiles)
    {
        dp_total = dp_tiles;
        dp_next = blockIdx.x;
        sk_begin = sk_pos = sk_start(blockIdx.x, p.sk_iters, p.ctas);
        sk_end = sk_start(blockIdx.x + 1, p.sk_iters, p.ctas);
    }
    __device__ __forceinline__ bool next(const KParams& p, Unit& u)
    {
        if (dp_next < dp_total) {
            u = {dp_next, 0, p.k_blocks, 0};
            dp_next += p.ctas;
            return true;
        }
        if (sk_pos < sk_end) {
            const uint64_t t = sk_pos / p.k_blocks;
            const uint32_t k0 = (uint32_t)(sk_pos - t * p.k_blocks);
            const uint64_t rem = sk_end - sk_pos;
            const uint32_t k1 = (uint32_t)((k0 + rem < p.k_blocks) ? k0 + rem : p.k_blocks);
            u = {p.dp_tiles + (uint32_t)t, k0, k1, sk_pos == sk_begin ? 0u : 1u};
            sk_pos += k1 - k0;
            return true;
        }
        return false;
    }
};

// Tile index -> (tile_m, tile_n), grouped along M so that CTAs running at the
// same time share A and B panels in L2.
__device__ __forceinline__ void tile_coords(const KParams& p, uint32_t t, uint32_t& tm, uint32_t& tn)
{
    const uint32_t per_group = p.raster_group * p.tiles_n;
    const uint32_t g = t / per_group;
    const uint32_t first_m = g * p.raster_group;
    const uint32_t gsize = (p.tiles_m - first_m) < p.raster_group ? (p.tiles_m - first_m) : p.raster_group;
    const uint32_t r = t - g * per_group;
    tm = first_m + r % gsize;
    tn = r / gsize;
}

// Tile geometry.  Plain mode: raster-grouped (tm, tn).  Grouped mode: the
// group is found by binary search of the per-group tile prefix `gpre`
// (the scheme of rocwmma_grouped_gemm.cpp:111-122); inside a group the M
// tiles run fastest so a group's B panel is reused while it is in L2.
template <bool kGrouped, uint32_t BN>
__device__ __forceinline__ TileGeom tile_geom(const KParams& p, uint32_t t, const uint32_t* gpre)
{
    TileGeom g;
    if constexpr (kGrouped) {
        uint32_t lo = 0, hi = p.groups;  // gpre[lo] <= t < gpre[hi]
        while (hi - lo > 1) {
            const uint32_t mid = (lo + hi) >> 1;
            if (gpre[mid] <= t) lo = mid;
            else hi = mid;
        }
        const uint32_t tl = t - gpre[lo];
        const uint32_t cnt = (uint32_t)p.grp_count[lo];
        const uint32_t tme = (cnt + kTileM - 1) / kTileM;
        const uint32_t tm = tl % tme, tn = tl / tme;
        const uint32_t start = (uint32_t)p.grp_start[lo];
        g.a_row = start + tm * kTileM;
        g.c_row = g.a_row;
        g.row_end = start + cnt;
        g.b_row = lo * p.Nk + tn * BN;
        g.col0 = tn * BN;
        g.cs_off = lo * p.Nk;
    } else {
        uint32_t tm, tn;
        tile_coords(p, t, tm, tn);
        g.a_row = tm * kTileM;
        g.c_row = g.a_row;
        g.row_end = p.Mk;
        g.b_row = tn * BN;
        g.col0 = tn * BN;
        g.cs_off = 0;
    }
    return g;
}

template <uint32_t BN, uint32_t BK, bool G = false>
struct Smem {
    static constexpr uint32_t ST = num_stages(BN, BK);
    static constexpr uint32_t A_BYTES = kTileM * BK;
    static constexpr uint32_t SB = stage_bytes(BN, BK);
    static constexpr uint32_t bar_off = ST * SB;
    static constexpr uint32_t full_off = bar_off;
    static constexpr uint32_t empty_off = full_off + 8 * ST;
    static constexpr uint32_t tfull_off = empty_off + 8 * ST;
    static constexpr uint32_t tempty_off = tfull_off + 16;
    static constexpr uint32_t taddr_off = tempty_off + 16;
    static constexpr uint32_t abort_off = taddr_off + 4;
    static constexpr uint32_t flag_off = abort_off + 4;
    // 4 KiB per epilogue warp to re-shape output chunks for coalesced stores
    // to peer GPUs (all-gather), when the pipeline leaves room for it.
    static constexpr uint32_t epi_off = bar_off + kBarrierBytes;
    static constexpr uint32_t EPI =
        (bar_off + kBarrierBytes + kEpiStageBytes + 1024 <= kSmemBudget) ? kEpiStageBytes : 0;
    static constexpr uint32_t total = bar_off + kBarrierBytes + EPI + 1024;
    static_assert(ST >= 2, "pipeline needs at least two stages");
    static_assert(flag_off + 4 <= bar_off + kBarrierBytes, "barrier area overflow");
    static_assert(total <= kSmemBudget, "shared memory overflow");
    static_assert(A_BYTES % 1024 == 0 && SB % 1024 == 0, "stages must keep 1 KiB swizzle alignment");
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b)
{
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_f16(float a, float b)
{
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <uint32_t W>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, int32_t (&acc)[W])
{
    if constexpr (W == 32) tmem_ld_32x32b_x32(taddr, reinterpret_cast<uint32_t(&)[32]>(acc));
    else tmem_ld_32x32b_x16(taddr, reinterpret_cast<uint32_t(&)[16]>(acc));
}

// 16 bytes to every rank's buffer at once: a store to an NVSwitch multicast
// address is replicated by the switch to each GPU bound to the multicast
// object, so the data crosses this GPU's links once.
__device__ __forceinline__ void multimem_st16(void* mc_addr, uint4 v)
{
    asm volatile("multimem.st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr), "f"(__uint_as_float(v.x)),
                 "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)), "f"(__uint_as_float(v.w))
                 : "memory");
}

// 16-byte store of an output piece at byte offset `off` of c: plain, or
// through the multicast view.
template <bool G>
__device__ __forceinline__ void st16_out(const KParams& p, void* cbase, size_t off, uint4 v)
{
    if constexpr (G) {
        if (p.mc_c) {
            multimem_st16(p.mc_c + off, v);
            return;
        }
    }
    *reinterpret_cast<uint4*>(static_cast<uint8_t*>(cbase) + off) = v;
}

// Stores one dequantised chunk (v, or the raw acc for int32 output) of kernel
// row `row` into the output buffer at cbase.
template <uint32_t W, bool G>
__device__ __forceinline__ void store_to(const KParams& p, void* cbase, uint32_t row, uint32_t col0,
                                         const int32_t (&acc)[W], const float (&v)[W])
{
    if (p.c_type == 2) {  // raw int32
        int32_t* c = static_cast<int32_t*>(cbase);
        if (!p.transpose_out) {
            int32_t* dst = c + (size_t)row * p.ldc + col0;
            if (p.vec_store_ok && col0 + W <= p.Nk) {
#pragma unroll
                for (int j = 0; j < (int)W; j += 4)
                    st16_out<G>(p, cbase, ((size_t)row * p.ldc + col0 + j) * 4,
                             make_uint4((uint32_t)acc[j], (uint32_t)acc[j + 1], (uint32_t)acc[j + 2],
                                        (uint32_t)acc[j + 3]));
            } else {
#pragma unroll
                for (int j = 0; j < (int)W; ++j)
                    if (col0 + j < p.Nk) dst[j] = acc[j];
            }
        } else {
#pragma unroll
            for (int j = 0; j < (int)W; ++j)
                if (col0 + j < p.Nk) c[(size_t)(col0 + j) * p.ldc + row] = acc[j];
        }
        return;
    }
    uint16_t* c = static_cast<uint16_t*>(cbase);
    if (!p.transpose_out) {
        uint16_t* dst = c + (size_t)row * p.ldc + col0;
        if (p.vec_store_ok && col0 + W <= p.Nk) {
#pragma unroll
            for (int j = 0; j < (int)W; j += 8) {
                uint4 w;
                if (p.c_type == 1) {
                    w = make_uint4(pack_bf16(v[j], v[j + 1]), pack_bf16(v[j + 2], v[j + 3]),
                                   pack_bf16(v[j + 4], v[j + 5]), pack_bf16(v[j + 6], v[j + 7]));
                } else {
                    w = make_uint4(pack_f16(v[j], v[j + 1]), pack_f16(v[j + 2], v[j + 3]),
                                   pack_f16(v[j + 4], v[j + 5]), pack_f16(v[j + 6], v[j + 7]));
                }
                st16_out<G>(p, cbase, ((size_t)row * p.ldc + col0 + j) * 2, w);
            }
        } else {
#pragma unroll
            for (int j = 0; j < (int)W; ++j) {
                if (col0 + j < p.Nk) {
                    dst[j] = p.c_type == 1 ? __bfloat16_as_ushort(__float2bfloat16_rn(v[j]))
                                           : __half_as_ushort(__float2half_rn(v[j]));
                }
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < (int)W; ++j) {
            if (col0 + j < p.Nk) {
                c[(size_t)(col0 + j) * p.ldc + row] = p.c_type == 1 ? __bfloat16_as_ushort(__float2bfloat16_rn(v[j]))
                                                                    : __half_as_ushort(__float2half_rn(v[j]));
            }
        }
    }
}


// Dequantises and stores W consecutive kernel columns [col0, col0+W) of
// kernel row `row` (one thread = one row).  rsc is this row's scale;
// csc_lane is the scale of column col0 + (lane % W), so the warp holds the
// chunk's column scales in one register and shares them by shuffles.
// Called by all 32 lanes of a warp (the shuffles precede any early exit).
// G: the all-gather build of the epilogue (several destinations or a
// multicast view); plain GEMMs are compiled without it.
template <uint32_t W, bool G = false>
__device__ __forceinline__ void store_chunk(const KParams& p, uint32_t row, uint32_t col0, const int32_t (&acc)[W],
                                            float rsc, float csc_lane)
{
    float v[W];
    if (p.c_type != 2) {
#pragma unroll
        for (int j = 0; j < (int)W; ++j) {
            const float csc = __shfl_sync(0xffffffffu, csc_lane, j);
            v[j] = __fmul_rn(__int2float_rn(acc[j]), __fmul_rn(rsc, csc));
        }
    }
    if (row >= p.Mk) return;
    if constexpr (G) {
        if (p.c_type != 2 && !p.transpose_out && p.vec_store_ok && col0 + W <= p.Nk) {
            // pack once, then the same 16-byte pieces to every destination
            uint32_t pk[W / 2];
#pragma unroll
            for (int j = 0; j < (int)W; j += 2) pk[j / 2] = p.c_type == 1 ? pack_bf16(v[j], v[j + 1]) : pack_f16(v[j], v[j + 1]);
            const size_t off = ((size_t)row * p.ldc + col0) * 2;
            for (uint32_t d = 0; d <= p.n_extra; ++d) {
                void* const cbase = d == 0 ? p.c : p.extra_c[d - 1];
#pragma unroll
                for (int j = 0; j < (int)W / 8; ++j)
                    st16_out<G>(p, cbase, off + (size_t)j * 16,
                                make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]));
            }
            return;
        }
        for (uint32_t d = 0; d <= p.n_extra; ++d) {
            void* const cbase = d == 0 ? p.c : p.extra_c[d - 1];
            store_to<W, G>(p, cbase, row, col0, acc, v);
        }
    } else {
        store_to<W, G>(p, p.c, row, col0, acc, v);
    }
}


__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d)
{
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint4 lds128_epi(uint32_t addr)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
                 : "memory");
    return v;
}

// Two consecutive W-column chunks of the warp's 32 rows.  With a 16-bit
// output and room to stage (stage = this warp's 4 KiB of shared memory, 0 if
// none), the 32 x 64 values are re-shaped through shared memory so that
// every store instruction writes 4 rows x 128 contiguous bytes instead of 32
// rows x 16 bytes: 8x fewer L2 requests (8192^2 x 2048: 117 -> 105 us), and
// NVLink moves peer stores (the all-gather build) at full rate only from
// 128-byte runs (measured: 16-byte runs reach a quarter of it).  Same values
// as store_chunk in every case.
// TMA bulk-tensor store of one staged 32-row x 64-column (128-byte) block:
// the staging layout (16-byte pieces XOR-swizzled by row) is the 128-byte
// swizzle of a tensor map with box {64, 32}.  Issued by one lane after every
// lane's shared-memory writes are ordered for the async proxy.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int32_t x, int32_t y)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Output store of the staged path, marked evict-first (.cs): the output is
// written once and not re-read by this kernel, so it should not push operand
// tiles other CTAs still need out of L2 (measured 1-2% at 8192^2 x 2048).
__device__ __forceinline__ void st_out16(void* p, uint4 v)
{
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

template <uint32_t W, bool G>
__device__ __forceinline__ void store_pair(const KParams& p, uint32_t row, uint32_t col0, const int32_t (&a0)[W],
                                           const int32_t (&a1)[W], float rsc, float cs0, float cs1, uint32_t stage,
                                           const CUtensorMap* tmC = nullptr, uint32_t block_row0 = 0,
                                           bool block_whole = false)
{
    if constexpr (W == 32) {
        if (stage != 0 && p.c_type != 2 && !p.transpose_out && p.vec_store_ok &&
            col0 + 2 * W <= p.Nk) {
            const uint32_t lane = threadIdx.x & 31;
            const bool by_tma = !G && tmC != nullptr && block_whole;
            if (!G && tmC != nullptr) {
                if (lane == 0) bulk_wait_read0();  // the previous TMA store has read the staging area
                __syncwarp();
            }
            // row-major [32 rows][128 B], 16-byte pieces XOR-swizzled by row (conflict-free both
            // ways); pieces 0-3 from the first chunk, 4-7 from the second, each written as soon
            // as it is packed
            auto stage_chunk = [&](const int32_t (&acc)[W], float cs, uint32_t piece0) {
                uint32_t w[16];  // 32 outputs packed in pairs
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const float c0 = __shfl_sync(0xffffffffu, cs, j), c1 = __shfl_sync(0xffffffffu, cs, j + 1);
                    const float v0 = __fmul_rn(__int2float_rn(acc[j]), __fmul_rn(rsc, c0));
                    const float v1 = __fmul_rn(__int2float_rn(acc[j + 1]), __fmul_rn(rsc, c1));
                    w[j / 2] = p.c_type == 1 ? pack_bf16(v0, v1) : pack_f16(v0, v1);
                }
#pragma unroll
                for (uint32_t c = 0; c < 4; ++c)
                    sts128(stage + lane * 128 + (((piece0 + c) ^ (lane & 7)) << 4), w[4 * c], w[4 * c + 1],
                           w[4 * c + 2], w[4 * c + 3]);
            };
            stage_chunk(a0, cs0, 0);
            stage_chunk(a1, cs1, 4);
            if (by_tma) {
                fence_async_smem();
                __syncwarp();
                if (lane == 0) tma_store_2d(tmC, stage, (int32_t)col0, (int32_t)block_row0);
                return;
            }
            __syncwarp();
            const size_t ldc_bytes = (size_t)p.ldc * 2;
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k) {
                const uint32_t r = 4 * k + (lane >> 3), c = lane & 7;
                const uint4 val = lds128_epi(stage + r * 128 + ((c ^ (r & 7)) << 4));
                const uint32_t row_r = __shfl_sync(0xffffffffu, row, r);
                if (row_r < p.Mk) {
                    const size_t off = (size_t)row_r * ldc_bytes + (size_t)col0 * 2 + c * 16;
                    if constexpr (G) {
                        if (p.mc_c) {
                            multimem_st16(p.mc_c + off, val);
                        } else {
                            *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.c) + off) = val;
                            for (uint32_t d = 0; d < p.n_extra; ++d)
                                *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.extra_c[d]) + off) = val;
                        }
                    } else {
                        st_out16(static_cast<uint8_t*>(p.c) + off, val);
                    }
                }
            }
            __syncwarp();  // the next pair rewrites the staging area
            return;
        }
    }
    store_chunk<W, G>(p, row, col0, a0, rsc, cs0);
    store_chunk<W, G>(p, row, col0 + W, a1, rsc, cs1);
}

template <uint32_t BN, uint32_t BK, bool kGrouped, bool G = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const KParams p,
                   uint64_t wait_limit_ns)
{
    using L = Smem<BN, BK, G>;
    constexpr uint32_t ST = L::ST;
    constexpr uint32_t TMEM_COLS = tmem_cols(BN);
    constexpr uint32_t CW = BN < 32 ? BN : 32;  // columns per tcgen05.ld
    constexpr uint32_t NCH = BN / CW;
    constexpr uint32_t KATOMS = BK / 128;       // 128-byte swizzle atoms along K per stage
    constexpr uint32_t TILE_ELEMS = BN * kTileM;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full_bar = sbase + L::full_off;
    const uint32_t empty_bar = sbase + L::empty_off;
    const uint32_t tfull_bar = sbase + L::tfull_off;
    const uint32_t tempty_bar = sbase + L::tempty_off;
    volatile uint32_t* taddr_slot = reinterpret_cast<volatile uint32_t*>(smem + L::taddr_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::abort_off);
    volatile int* epi_flag = reinterpret_cast<volatile int*>(smem + L::flag_off);

    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < ST; ++s) {
            mbar_init(full_bar + 8 * s, 1);
            mbar_init(empty_bar + 8 * s, 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(tfull_bar + 8 * b, 1);
            mbar_init(tempty_bar + 8 * b, 4);  // one arrival per epilogue warp
        }
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(sbase + L::taddr_off, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    uint32_t* gpre = nullptr;  // grouped mode: tile prefix per group, [groups + 1]
    uint32_t tiles_total = p.dp_tiles;
    if constexpr (kGrouped) {
        __shared__ uint32_t s_gpre[kMaxGroups + 1];
        gpre = s_gpre;
        if (threadIdx.x == 0) {
            uint32_t acc = 0;
            for (uint32_t g = 0; g < p.groups; ++g) {
                s_gpre[g] = acc;
                const uint32_t cnt = p.grp_count[g] > 0 ? (uint32_t)p.grp_count[g] : 0u;
                acc += ((cnt + kTileM - 1) / kTileM) * p.tiles_n;
            }
            s_gpre[p.groups] = acc;
        }
        __syncthreads();
        tiles_total = s_gpre[p.groups];
    }
    const uint32_t tmem_base = *taddr_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            UnitIter it;
            it.init(p, tiles_total);
            Unit u;
            uint32_t stage = 0, phase = 0;
            uint32_t issued_phase[8];
            bool issued[8];
            for (uint32_t s = 0; s < 8; ++s) issued[s] = false, issued_phase[s] = 0;
            // One stage's A / B tiles (BK/128 swizzle atoms along K each).
            auto load_a = [&](uint32_t sa, uint32_t fb, uint32_t kb, int32_t a_row) {
#pragma unroll
                for (uint32_t i = 0; i < KATOMS; ++i) {
                    const int32_t kc = (int32_t)(kb * BK + i * 128);
                    // K-major: atom i is [128 rows][128 B]; MN-major: k rows are contiguous.
                    if (p.a_mn_major) tma_load_2d(sa + i * (128 * 128), &tmA, fb, a_row, kc);
                    else tma_load_2d(sa + i * (kTileM * 128), &tmA, fb, kc, a_row);
                }
            };
            auto load_b = [&](uint32_t sb, uint32_t fb, uint32_t kb, int32_t b_row) {
#pragma unroll
                for (uint32_t i = 0; i < KATOMS; ++i) {
                    const int32_t kc = (int32_t)(kb * BK + i * 128);
                    if (p.b_mn_major) {
#pragma unroll
                        for (uint32_t j = 0; j < BN / 128; ++j)
                            tma_load_2d(sb + j * (BK * 128) + i * (128 * 128), &tmB, fb, b_row + (int32_t)(j * 128), kc);
                    } else {
                        tma_load_2d(sb + i * (BN * 128), &tmB, fb, kc, b_row);
                    }
                }
            };
            // Programmatic dependent launch: the operand written by the
            // previous kernel (p.pdl_dep: 1 = A, 2 = B) is loaded only after
            // griddepcontrol.wait; the other operand of the first ring of
            // stages is already streaming meanwhile.
            bool pdl_pending = p.pdl_dep != 0;
            uint32_t ndef = 0, def_stage[8], def_kb[8];
            int32_t def_row[8];
            auto flush_deferred = [&]() {
                griddep_wait();
                for (uint32_t d = 0; d < ndef; ++d) {
                    const uint32_t sa = sbase + def_stage[d] * L::SB;
                    const uint32_t fb = full_bar + 8 * def_stage[d];
                    if (p.pdl_dep == 1) load_a(sa, fb, def_kb[d], def_row[d]);
                    else load_b(sa + L::A_BYTES, fb, def_kb[d], def_row[d]);
                }
                ndef = 0;
                pdl_pending = false;
            };
            bool ok = true;
            while (ok && it.next(p, u)) {
                const TileGeom tg = tile_geom<kGrouped, BN>(p, u.tile, gpre);
                const int32_t a_row = (int32_t)tg.a_row;
                const int32_t b_row = (int32_t)tg.b_row;
                for (uint32_t kb = u.k0; kb < u.k1; ++kb) {
                    if (pdl_pending && ndef == ST) flush_deferred();  // the ring is full of half-loaded stages
                    if (!mbar_wait(empty_bar + 8 * stage, phase ^ 1, SITE_PRODUCER_EMPTY, abort_flag, wait_limit_ns)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full_bar + 8 * stage;
                    mbar_arrive_expect_tx(fb, L::SB);
                    const uint32_t sa = sbase + stage * L::SB;
                    const uint32_t sb = sa + L::A_BYTES;
                    if (!pdl_pending) {
                        load_a(sa, fb, kb, a_row);
                        load_b(sb, fb, kb, b_row);
                    } else {
                        if (p.pdl_dep == 1) load_b(sb, fb, kb, b_row);
                        else load_a(sa, fb, kb, a_row);
                        def_stage[ndef] = stage;
                        def_kb[ndef] = kb;
                        def_row[ndef] = p.pdl_dep == 1 ? a_row : b_row;
                        ++ndef;
                    }
                    issued[stage] = true;
                    issued_phase[stage] = phase;
                    if (++stage == ST) stage = 0, phase ^= 1;
                }
            }
            if (pdl_pending) flush_deferred();
            // Drain: every TMA copy this thread issued lands before the CTA
            // exits (immediate on the normal path).
            for (uint32_t s = 0; s < ST; ++s)
                if (issued[s]) mbar_wait(full_bar + 8 * s, issued_phase[s], SITE_PRODUCER_DRAIN, nullptr, wait_limit_ns);
        }
        __syncwarp();  // reconverge before the CTA-wide barrier below
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_i8(kTileM, BN, p.a_mn_major, p.b_mn_major);
            const uint32_t a_lbo = p.a_mn_major ? 128 * BK : 16;
            const uint32_t b_lbo = p.b_mn_major ? 128 * BK : 16;
            UnitIter it;
            it.init(p, tiles_total);
            Unit u;
            uint32_t stage = 0, phase = 0, uidx = 0;
            bool ok = true;
            while (ok && it.next(p, u)) {
                const uint32_t buf = uidx & 1;
                const uint32_t use = uidx >> 1;
                if (!mbar_wait(tempty_bar + 8 * buf, (use & 1) ^ 1, SITE_MMA_TMEM_EMPTY, abort_flag, wait_limit_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * BN;
                for (uint32_t kb = u.k0; kb < u.k1; ++kb) {
                    if (!mbar_wait(full_bar + 8 * stage, phase, SITE_MMA_FULL, abort_flag, wait_limit_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = sbase + stage * L::SB;
                    const uint32_t sb = sa + L::A_BYTES;
#pragma unroll
                    for (uint32_t kk = 0; kk < BK / 32; ++kk) {
                        // K-major: atom kk/4, 32-byte step inside the swizzled row;
                        // MN-major: 32 k rows of 128 bytes.
                        const uint32_t a_off = p.a_mn_major ? kk * 32 * 128 : (kk / 4) * (kTileM * 128) + (kk % 4) * 32;
                        const uint32_t b_off = p.b_mn_major ? kk * 32 * 128 : (kk / 4) * (BN * 128) + (kk % 4) * 32;
                        const uint64_t ad = umma_desc_sw128(sa + a_off, a_lbo, 1024);
                        const uint64_t bd = umma_desc_sw128(sb + b_off, b_lbo, 1024);
                        mma_i8(d_tmem, ad, bd, idesc, (kb > u.k0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit(empty_bar + 8 * stage);
                    if (++stage == ST) stage = 0, phase ^= 1;
                }
                if (!ok) break;
                mma_commit(tfull_bar + 8 * buf);
                ++uidx;
            }
        }
        __syncwarp();  // reconverge before the CTA-wide barrier below
    } else {
        // ------------------------------------------------------------ epilogue
        if (p.pdl_dep) griddep_wait();  // row scales come from the previous kernel
        const uint32_t q = warp & 3;  // TMEM lane quarter this warp may access
        const uint32_t row_local = q * 32 + lane;
        const uint32_t epi_stage = L::EPI ? sbase + L::epi_off + q * 4096 : 0u;
        const uint32_t ethread = threadIdx.x - 64;
        UnitIter it;
        it.init(p, tiles_total);
        Unit u;
        uint32_t uidx = 0;
        bool ok = true;
        while (ok && it.next(p, u)) {
            const uint32_t buf = uidx & 1;
            const uint32_t use = uidx >> 1;
            if (!mbar_wait(tfull_bar + 8 * buf, use & 1, SITE_EPI_TMEM_FULL, abort_flag, wait_limit_ns)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const TileGeom tg = tile_geom<kGrouped, BN>(p, u.tile, gpre);
            const uint32_t tn_col0 = tg.col0;
            // Rows past the tile's limit (the matrix, or the group in grouped
            // mode) get an out-of-range index so store_chunk skips them.
            const uint32_t row = tg.c_row + row_local < tg.row_end ? tg.c_row + row_local : 0xffffffffu;
            const uint32_t taddr = tmem_base + ((q * 32) << 16) + buf * BN;
            const bool full = (u.k0 == 0 && u.k1 == p.k_blocks);
            // Scales of this tile, fetched once: the row's own scale, and per
            // lane the scale of column (chunk * CW + lane % CW) for every chunk.
            const float rsc = (p.row_scale_vec && row < p.Mk) ? __ldg(p.row_scale_vec + row) : p.row_scale;
            float csv[NCH];
#pragma unroll
            for (uint32_t ch = 0; ch < NCH; ++ch) {
                const uint32_t col = tn_col0 + ch * CW + (lane % CW);
                csv[ch] = p.col_scale_vec ? (col < p.Nk ? __ldg(p.col_scale_vec + tg.cs_off + col) : 0.f)
                                          : p.col_scale;
            }
            if (full) {
                if constexpr (NCH == 1) {
                    int32_t acc[CW];
                    tmem_ld_chunk<CW>(taddr, acc);
                    tmem_ld_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(tempty_bar + 8 * buf);
                    store_chunk<CW, G>(p, row, tn_col0, acc, rsc, csv[0]);
                } else {
                    // Two chunks per TMEM round trip.
#pragma unroll
                    for (uint32_t ch = 0; ch < NCH; ch += 2) {
                        int32_t acc0[CW], acc1[CW];
                        tmem_ld_chunk<CW>(taddr + ch * CW, acc0);
                        tmem_ld_chunk<CW>(taddr + (ch + 1) * CW, acc1);
                        tmem_ld_wait();
                        if (ch + 2 >= NCH) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(tempty_bar + 8 * buf);
                        }
                        store_pair<CW, G>(p, row, tn_col0 + ch * CW, acc0, acc1, rsc, csv[ch], csv[ch + 1], epi_stage);
                    }
                }
            } else {
                // Stream-K partial: store it to this CTA's slot ([BN][128],
                // column-major so a warp's stores are 128-byte coalesced).
                int32_t* my_slot = p.ws_slots + ((size_t)blockIdx.x * 2 + u.slot) * TILE_ELEMS;
#pragma unroll 1
                for (uint32_t ch = 0; ch < NCH; ++ch) {
                    int32_t acc[CW];
                    tmem_ld_chunk<CW>(taddr + ch * CW, acc);
                    tmem_ld_wait();
                    if (ch == NCH - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(tempty_bar + 8 * buf);
                    }
#pragma unroll
                    for (uint32_t j = 0; j < CW; ++j) __stcg(my_slot + (size_t)(ch * CW + j) * kTileM + row_local, acc[j]);
                }
                __threadfence();
                named_bar_sync(1, kEpiThreads);
                const uint32_t tail_idx = u.tile - p.dp_tiles;
                if (ethread == 0) {
                    const uint32_t add = u.k1 - u.k0;
                    const uint32_t old = atomicAdd(p.ws_cnt + tail_idx, add);
                    const int last = (old + add == p.k_blocks) ? 1 : 0;
                    if (last) p.ws_cnt[tail_idx] = 0;  // every contribution has arrived: reset for the next call
                    *epi_flag = last;
                }
                named_bar_sync(1, kEpiThreads);
                if (*epi_flag) {
                    // This contribution completed the tile: sum every
                    // contributor's slot and run the epilogue.
                    __threadfence();
                    const uint64_t it0 = (uint64_t)tail_idx * p.k_blocks;
                    const uint64_t it1 = it0 + p.k_blocks;
                    const uint64_t S = p.sk_iters, P = p.ctas;
                    const uint32_t c_first = (uint32_t)(((it0 + 1) * P - 1) / S);
                    const uint32_t c_last = (uint32_t)((it1 * P - 1) / S);
#pragma unroll 1
                    for (uint32_t ch = 0; ch < NCH; ++ch) {
                        int32_t acc[CW];
#pragma unroll
                        for (uint32_t j = 0; j < CW; ++j) acc[j] = 0;
#pragma unroll 1
                        for (uint32_t cc = c_first; cc <= c_last; ++cc) {
                            const uint64_t st = sk_start(cc, S, P);
                            if (sk_start(cc + 1, S, P) == st) continue;  // CTA without stream-K work
                            const uint32_t slot = st >= it0 ? 0u : 1u;
                            const int32_t* src = p.ws_slots + ((size_t)cc * 2 + slot) * TILE_ELEMS;
#pragma unroll
                            for (uint32_t j = 0; j < CW; ++j) acc[j] += __ldcg(src + (size_t)(ch * CW + j) * kTileM + row_local);
                        }
                        store_chunk<CW, G>(p, row, tn_col0 + ch * CW, acc, rsc, csv[ch]);
                    }
                }
            }
            ++uidx;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// CTA-pair kernel for large K-major problems: a cluster of two CTAs (two SMs)
// computes a 256 x 256 tile with tcgen05.mma.cta_group::2 (M = 256, N = 256).
// Each CTA loads its own 128 rows of A and its own 128 rows (columns of the
// product) of B per stage, so every SM streams half of the B panel a 1-CTA
// 128 x 256 tile would need; each CTA's TMEM holds its 128 x 256 half of the
// accumulator.  Only the leader (rank 0) issues MMAs; both CTAs' TMA copies
// signal the leader's "full" barrier; the leader's commits release "empty"
// stages and "accumulator full" in both CTAs; both CTAs' epilogue warps
// release an accumulator on the leader's "accumulator empty" barrier.
// Whole tiles only (data-parallel rounds), used when the last round leaves at
// most 5% of the pairs idle.
// ---------------------------------------------------------------------------
constexpr uint32_t kPairBN = 256;  // tile columns (MMA N)
constexpr uint32_t kPairBK = 128;
constexpr uint32_t kPairHalfBytes = 128 * kPairBK;          // 16 KiB: one operand half per stage
constexpr uint32_t kPairSB = 2 * kPairHalfBytes;            // A half + B half per CTA per stage
constexpr uint32_t kPairST = 6;
constexpr uint32_t kPairBarOff = kPairST * kPairSB;
// The staging area starts on a 1024-byte boundary: the TMA store's 128-byte
// swizzle is a function of the shared-memory address bits.
constexpr uint32_t kPairEpiOff = kPairBarOff + 1024;
static_assert(kBarrierBytes <= 1024 && kPairEpiOff % 1024 == 0, "pair staging alignment");
constexpr uint32_t pair_smem(bool) { return kPairEpiOff + kEpiStageBytes + 1024; }
constexpr uint32_t kPairSmem = pair_smem(true);
static_assert(kPairSmem <= kSmemBudget, "pair kernel shared memory overflow");

// One pair tile: 256 rows from a_row (rows from row_end on are not stored),
// 256 columns from col0 of the product, B rows from b_row, column scales
// offset by cs_off.  Grouped (MoE) mode: the tiles of group g are
// ceil(count_g / 256) x tiles_n, M fastest, found by binary search of `gpre`.
struct PairTile {
    uint32_t a_row, row_end, b_row, col0, cs_off;
};

template <bool kGrouped>
__device__ __forceinline__ PairTile pair_tile(const KParams& p, uint32_t t, const uint32_t* gpre)
{
    PairTile g;
    if constexpr (kGrouped) {
        uint32_t lo = 0, hi = p.groups;  // gpre[lo] <= t < gpre[hi]
        while (hi - lo > 1) {
            const uint32_t mid = (lo + hi) >> 1;
            if (gpre[mid] <= t) lo = mid;
            else hi = mid;
        }
        const uint32_t tl = t - gpre[lo];
        const uint32_t cnt = (uint32_t)p.grp_count[lo];
        const uint32_t tme = (cnt + 255) / 256;
        const uint32_t tm = tl % tme, tn = tl / tme;
        const uint32_t start = (uint32_t)p.grp_start[lo];
        g.a_row = start + tm * 256;
        g.row_end = start + cnt;
        g.b_row = lo * p.Nk + tn * kPairBN;
        g.col0 = tn * kPairBN;
        g.cs_off = lo * p.Nk;
    } else {
        uint32_t tm, tn;
        tile_coords(p, t, tm, tn);
        g.a_row = tm * 256;
        g.row_end = p.Mk;
        g.b_row = tn * kPairBN;
        g.col0 = tn * kPairBN;
        g.cs_off = 0;
    }
    return g;
}

template <bool kGrouped, bool G = false>
__global__ void __launch_bounds__(kThreads, 1) __cluster_dims__(2, 1, 1)
    gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const KParams p, uint64_t wait_limit_ns)
{
    constexpr uint32_t ST = kPairST;
    constexpr uint32_t TMEM_COLS = 512;  // two 256-column accumulators
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full_bar = sbase + kPairBarOff;
    const uint32_t empty_bar = full_bar + 8 * ST;
    const uint32_t tfull_bar = empty_bar + 8 * ST;
    const uint32_t tempty_bar = tfull_bar + 16;
    volatile uint32_t* taddr_slot = reinterpret_cast<volatile uint32_t*>(smem + kPairBarOff + 16 * ST + 32);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kPairBarOff + 16 * ST + 36);

    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t pair = blockIdx.x >> 1;
    const uint32_t npairs = gridDim.x >> 1;
    uint32_t T = p.tiles_m * p.tiles_n;
    const uint32_t* gpre = nullptr;  // grouped mode: pair-tile prefix per group, [groups + 1]
    if constexpr (kGrouped) {
        __shared__ uint32_t s_gpre[kMaxGroups + 1];
        if (threadIdx.x == 0) {
            uint32_t acc = 0;
            for (uint32_t g = 0; g < p.groups; ++g) {
                s_gpre[g] = acc;
                const uint32_t cnt = p.grp_count[g] > 0 ? (uint32_t)p.grp_count[g] : 0u;
                acc += ((cnt + 255) / 256) * p.tiles_n;
            }
            s_gpre[p.groups] = acc;
        }
        __syncthreads();
        gpre = s_gpre;
        T = s_gpre[p.groups];
    }

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < ST; ++s) {
            mbar_init(full_bar + 8 * s, 1);
            mbar_init(empty_bar + 8 * s, 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(tfull_bar + 8 * b, 1);
            mbar_init(tempty_bar + 8 * b, 8);  // four epilogue warps in each CTA of the pair
        }
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (!G && p.tma_store) tma_prefetch_desc(&tmC);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(const_cast<uint32_t*>(taddr_slot)), TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers initialised before any remote use
    tc_fence_after();
    const uint32_t tmem_base = *taddr_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer (both CTAs)
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            for (uint32_t t = pair; ok && t < T; t += npairs) {
                const PairTile tg = pair_tile<kGrouped>(p, t, gpre);
                const int32_t a_row = (int32_t)(tg.a_row + rank * 128);
                const int32_t b_row = (int32_t)(tg.b_row + rank * 128);
                for (uint32_t kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(empty_bar + 8 * stage, phase ^ 1, SITE_PRODUCER_EMPTY, abort_flag, wait_limit_ns)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full_bar + 8 * stage;
                    if (rank == 0) mbar_arrive_expect_tx(fb, 2 * kPairSB);  // both CTAs' bytes
                    const uint32_t fb_leader = mapa_shared(fb, 0);
                    const uint32_t sa = sbase + stage * kPairSB;
                    const int32_t kc = (int32_t)(kb * kPairBK);
                    // K-major: box {128 k, 128 rows}; MN-major: box {128 rows, 128 k} (one
                    // 128-byte swizzle atom along M or N: each CTA holds 128 of them)
                    if (p.a_mn_major) tma_load_2d_pair(sa, &tmA, fb_leader, a_row, kc);
                    else tma_load_2d_pair(sa, &tmA, fb_leader, kc, a_row);
                    if (p.b_mn_major) tma_load_2d_pair(sa + kPairHalfBytes, &tmB, fb_leader, b_row, kc);
                    else tma_load_2d_pair(sa + kPairHalfBytes, &tmB, fb_leader, kc, b_row);
                    if (++stage == ST) stage = 0, phase ^= 1;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader only)
        if (lane == 0 && rank == 0) {
            const uint32_t idesc = idesc_i8(256, kPairBN, p.a_mn_major, p.b_mn_major);
            // K-major: 32-byte steps inside the swizzled rows; MN-major: 32 k rows of 128 bytes
            const uint32_t a_step = p.a_mn_major ? 32 * 128 : 32, b_step = p.b_mn_major ? 32 * 128 : 32;
            const uint32_t a_lbo = p.a_mn_major ? 128 * kPairBK : 16, b_lbo = p.b_mn_major ? 128 * kPairBK : 16;
            uint32_t stage = 0, phase = 0, uidx = 0;
            bool ok = true;
            for (uint32_t t = pair; ok && t < T; t += npairs, ++uidx) {
                const uint32_t buf = uidx & 1, use = uidx >> 1;
                if (!mbar_wait(tempty_bar + 8 * buf, (use & 1) ^ 1, SITE_MMA_TMEM_EMPTY, abort_flag, wait_limit_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * kPairBN;
                for (uint32_t kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(full_bar + 8 * stage, phase, SITE_MMA_FULL, abort_flag, wait_limit_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = sbase + stage * kPairSB;
#pragma unroll
                    for (uint32_t kk = 0; kk < kPairBK / 32; ++kk) {
                        const uint64_t ad = umma_desc_sw128(sa + kk * a_step, a_lbo, 1024);
                        const uint64_t bd = umma_desc_sw128(sa + kPairHalfBytes + kk * b_step, b_lbo, 1024);
                        mma_i8_pair(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit_pair(empty_bar + 8 * stage, 0x3);
                    if (++stage == ST) stage = 0, phase ^= 1;
                }
                if (!ok) break;
                mma_commit_pair(tfull_bar + 8 * buf, 0x3);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const uint32_t q = warp & 3;
        const uint32_t row_local = q * 32 + lane;
        constexpr uint32_t CW = 32, NCH = kPairBN / CW;
        const uint32_t epi_stage = sbase + kPairEpiOff + q * 4096;
        const CUtensorMap* tmc = (!G && p.tma_store) ? &tmC : nullptr;
        uint32_t uidx = 0;
        for (uint32_t t = pair; t < T; t += npairs, ++uidx) {
            const uint32_t buf = uidx & 1, use = uidx >> 1;
            if (!mbar_wait(tfull_bar + 8 * buf, use & 1, SITE_EPI_TMEM_FULL, abort_flag, wait_limit_ns)) break;
            tc_fence_after();
            const PairTile tg = pair_tile<kGrouped>(p, t, gpre);
            // rows past the tile's limit (the matrix, or the group) get an
            // out-of-range index so the stores skip them
            const uint32_t row0 = tg.a_row + rank * 128 + row_local;
            const uint32_t row = row0 < tg.row_end ? row0 : 0xffffffffu;
            const uint32_t taddr = tmem_base + ((q * 32) << 16) + buf * kPairBN;
            const float rsc = (p.row_scale_vec && row < p.Mk) ? __ldg(p.row_scale_vec + row) : p.row_scale;
            float csv[NCH];
#pragma unroll
            for (uint32_t ch = 0; ch < NCH; ++ch) {
                const uint32_t col = tg.col0 + ch * CW + lane;
                csv[ch] = p.col_scale_vec ? (col < p.Nk ? __ldg(p.col_scale_vec + tg.cs_off + col) : 0.f) : p.col_scale;
            }
#pragma unroll
            for (uint32_t ch = 0; ch < NCH; ch += 2) {
                int32_t acc0[CW], acc1[CW];
                tmem_ld_chunk<CW>(taddr + ch * CW, acc0);
                tmem_ld_chunk<CW>(taddr + (ch + 1) * CW, acc1);
                tmem_ld_wait();
                if (ch + 2 >= NCH) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty_bar + 8 * buf, 0));
                }
                // TMA clips the matrix edges itself; a group's last block that
                // ends inside the matrix is stored row by row instead
                const uint32_t brow0 = tg.a_row + rank * 128 + q * 32;
                store_pair<CW, G>(p, row, tg.col0 + ch * CW, acc0, acc1, rsc, csv[ch], csv[ch + 1], epi_stage, tmc,
                                  brow0, brow0 + 32 <= tg.row_end || tg.row_end >= p.Mk);
            }
        }
        if (tmc != nullptr && lane == 0) bulk_wait_all();  // stores done before the CTA's shared memory goes
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while its peer may still signal its barriers
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
    }
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

// 2-D int8 operand map with a 128-byte swizzled box.  K-major: dims {K, rows},
// box {128, box_rows}; MN-major: dims {rows, K}, box {128, 128}.
bool make_operand_map(CUtensorMap* map, const int8_t* base, uint32_t rows, uint32_t K, uint32_t ld, bool mn_major,
                      uint32_t box_rows)
{
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2];
    cuuint32_t box[2];
    if (mn_major) {
        dims[0] = rows;
        dims[1] = K;
        box[0] = 128;
        box[1] = 128;
    } else {
        dims[0] = K;
        dims[1] = rows;
        box[0] = 128;
        box[1] = box_rows;
    }
    cuuint64_t strides[1] = {ld};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <uint32_t BN, uint32_t BK, bool kGrouped = false, bool G = false>
cudaError_t launch_tile(const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp, cudaStream_t st)
{
    using L = Smem<BN, BK, G>;
    // The shared-memory opt-in is a per-device function attribute.
    static std::atomic<uint64_t> done_mask{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(done_mask.load() & bit)) {
        e = cudaFuncSetAttribute(gemm_i8_kernel<BN, BK, kGrouped, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 L::total);
        if (e != cudaSuccess) return e;
        done_mask.fetch_or(bit);
    }
    if (kp.pdl_dep) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(kp.ctas);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = L::total;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, gemm_i8_kernel<BN, BK, kGrouped, G>, ta, tb, kp, (uint64_t)kWaitLimitNs);
    }
    gemm_i8_kernel<BN, BK, kGrouped, G><<<kp.ctas, kThreads, L::total, st>>>(ta, tb, kp, kWaitLimitNs);
    return cudaGetLastError();
}

// Output map of the pair kernel's TMA stores: 16-bit elements, dims {Nk, Mk},
// box {64 columns, 32 rows}, 128-byte swizzle (the staging layout).
bool make_output_map(CUtensorMap* map, void* c, uint32_t Mk, uint32_t Nk, uint32_t ldc)
{
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {Nk, Mk};
    cuuint64_t strides[1] = {(cuuint64_t)ldc * 2};
    cuuint32_t box[2] = {64, 32};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, c, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool kGrouped, bool G = false>
cudaError_t launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, KParams kp, cudaStream_t st)
{
    CUtensorMap tc;
    std::memset(&tc, 0, sizeof(tc));
    kp.tma_store = 0;
    if (!G && B2SQ_PAIR_TMA_STORE && kp.c_type != 2 && !kp.transpose_out && kp.vec_store_ok)
        kp.tma_store = make_output_map(&tc, kp.c, kp.Mk, kp.Nk, kp.ldc) ? 1u : 0u;
    static std::atomic<uint64_t> done_mask{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(done_mask.load() & bit)) {
        e = cudaFuncSetAttribute(gemm_i8_pair_kernel<kGrouped, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 pair_smem(G));
        if (e != cudaSuccess) return e;
        done_mask.fetch_or(bit);
    }
    gemm_i8_pair_kernel<kGrouped, G><<<kp.ctas, kThreads, pair_smem(G), st>>>(ta, tb, tc, kp, kWaitLimitNs);
    return cudaGetLastError();
}

}  // namespace

void plan_gemm_schedule(uint32_t Mk, uint32_t Nk, uint32_t K, uint32_t a_mn_major, uint32_t b_mn_major,
                        bool allow_stream_k, uint32_t num_sms, GemmSchedule& s)
{
    s = GemmSchedule{};
    const uint32_t P = num_sms ? num_sms : 148;
#ifndef B2SQ_DISABLE_PAIR
    // CTA-pair 256 x 256 tiles for every problem of more than 128 x 128 (either
    // operand K-major or MN-major): a 1-CTA 128 x 256 tile streams 1.5x the operand bytes per MMA and
    // is L2-bound (ncu: 57-60% against 84% tensor utilisation), so pairs win
    // even when most of their last round is idle, or most of their tile rows
    // or columns lie past the matrix (measured on B200, in us, pairs vs 1-CTA
    // tiles: 4096^3 57.9 vs 82.4; 512 x 8192 x 8192 37.3 vs 76.3; 1280 x 4096
    // x 8192 53.8 vs 57.8; 200 x 8192 x 4096 31.6 vs 51.2; 160 x 28672 x 8192
    // 61.3 vs 108.6; 129 x 8192 x 8192 41.0 vs 57.3; 8192 x 200 x 8192 47.1 vs
    // 55.3; 16384 x 192 x 2048 32.8 vs 45.1).
    if (Mk > kTileM && Nk > kTileM && P >= 2) {
        const uint64_t tm2 = (Mk + 255) / 256, tn2 = (Nk + kPairBN - 1) / kPairBN, T2 = tm2 * tn2;
        const uint64_t pairs = P / 2;
        s.cta_pair = 1;
        s.tile_n = kPairBN;
        s.tile_k = kPairBK;
        s.stages = kPairST;
        s.tiles_m = (uint32_t)tm2;
        s.tiles_n = (uint32_t)tn2;
        s.k_blocks = (K + kPairBK - 1) / kPairBK;
        s.dp_tiles = (uint32_t)T2;
        s.ctas = (uint32_t)(2 * (T2 < pairs ? T2 : pairs));
        return;
    }
#endif
    uint32_t bn = 16;
    while (bn < Nk && bn < 256) bn <<= 1;
    if (b_mn_major && bn < 128) bn = 128;  // MN-major B tiles are 128-element swizzle rows
    s.tile_n = bn;
    s.tile_k = tile_k_for(bn);
    s.stages = num_stages(bn, s.tile_k);
    s.tiles_m = (Mk + kTileM - 1) / kTileM;
    s.tiles_n = (Nk + bn - 1) / bn;
    s.k_blocks = (K + s.tile_k - 1) / s.tile_k;
    const uint64_t T = (uint64_t)s.tiles_m * s.tiles_n;
    const uint64_t rounds = (T + P - 1) / P;
    const double tail_loss = (double)(rounds * P - T) / (double)(rounds * P);
    // Skinny tiles (tile_n <= 64, the decode shapes) are bound by HBM: when
    // part of the SMs run out of tiles the others take over the bandwidth, so
    // splitting tiles gains nothing and its fix-up costs a few microseconds
    // (measured).  Stream-K is for compute-bound tails.
    const bool hbm_bound = bn <= 64;
    // A split tile is summed by the CTA whose slice completes it, which reads
    // every contributor's slot in turn, so stream-K pays only while a tile has
    // at most ~3 contributors (measured, us, stream-K vs whole tiles: 128 x 8192
    // x 8192 (64 tiles) 41.0 vs 45.0; 100 x 4096 x 4096 (32 tiles) 38.9 vs 34.8;
    // 120 x 640 x 4096 (5 tiles) 100.5 vs 34.8; 100 x 200 x 8192 (1 tile) 354.5
    // vs 57.4; 96 x 28672 x 8192 (224 tiles, 1.5 rounds) 68.5 vs 59.4).
    const uint64_t tail_tiles = T % P;
    const bool few_contributors = tail_tiles * kStreamKMaxContributors >= P;
    if (!allow_stream_k || hbm_bound || s.k_blocks < 2 || tail_loss <= kStreamKMinTailLoss || !few_contributors ||
        (T > P && T < 4ull * P)) {
        s.dp_tiles = (uint32_t)T;
        s.sk_iters = 0;
        s.ctas = (uint32_t)(T < P ? T : P);
    } else if (T >= 4ull * P) {
        // Whole rounds data-parallel, the partial last round split by k-blocks.
        s.dp_tiles = (uint32_t)((T / P) * P);
        s.sk_iters = (T - s.dp_tiles) * (uint64_t)s.k_blocks;
        s.ctas = P;
    } else {
        // Less than one round: stream-K over everything keeps every SM busy to the end.
        s.dp_tiles = 0;
        s.sk_iters = T * (uint64_t)s.k_blocks;
        s.ctas = (uint32_t)(s.sk_iters < P ? s.sk_iters : P);
    }
    const uint64_t tail = T - s.dp_tiles;
    if (tail > kWsCounters) {  // more tail tiles than counters: whole tiles only
        s.dp_tiles = (uint32_t)T;
        s.sk_iters = 0;
        s.ctas = (uint32_t)(T < P ? T : P);
    } else if (tail) {
        s.workspace_bytes = kWsCounterBytes + (size_t)s.ctas * 2 * bn * kTileM * 4;
    }
}

cudaError_t launch_gemm_i8(const GemmProblem& p, const GemmSchedule& s, void* workspace, cudaStream_t st,
                           const char** detail)
{
    const uint32_t bn = s.tile_n;
    CUtensorMap ta, tb;
    if (!make_operand_map(&ta, p.a, p.Mk, p.K, p.lda, p.a_mn_major != 0, kTileM) ||
        !make_operand_map(&tb, p.b, p.Nk, p.K, p.ldb, p.b_mn_major != 0, s.cta_pair ? 128 : bn)) {
        if (detail) *detail = "cuTensorMapEncodeTiled rejected an operand (alignment / stride)";
        return cudaErrorInvalidValue;
    }
    KParams kp{};
    kp.Mk = p.Mk;
    kp.Nk = p.Nk;
    kp.K = p.K;
    kp.tiles_m = s.tiles_m;
    kp.tiles_n = s.tiles_n;
    kp.k_blocks = s.k_blocks;
    kp.dp_tiles = s.dp_tiles;
    kp.ctas = s.ctas;
    kp.sk_iters = s.sk_iters;
    kp.a_mn_major = p.a_mn_major;
    kp.b_mn_major = p.b_mn_major;
    kp.c = p.c;
    kp.n_extra = p.n_extra;
    kp.mc_c = static_cast<uint8_t*>(p.mc_c);
    for (uint32_t d = 0; d < p.n_extra && d < kMaxExtraOut; ++d) kp.extra_c[d] = p.extra_c[d];
    kp.ldc = p.ldc;
    kp.c_type = p.c_type;
    kp.transpose_out = p.transpose_out;
    const uint32_t esz = p.c_type == 2 ? 4 : 2;
    kp.vec_store_ok = ((reinterpret_cast<uintptr_t>(p.c) & 15) == 0) && ((p.ldc * esz) % 16 == 0);
    kp.row_scale_vec = p.row_scale_vec;
    kp.col_scale_vec = p.col_scale_vec;
    kp.row_scale = p.row_scale;
    kp.col_scale = p.col_scale;
    if (s.workspace_bytes) {
        kp.ws_cnt = static_cast<uint32_t*>(workspace);
        kp.ws_slots = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + kWsCounterBytes);
    }
    kp.raster_group = B2SQ_RASTER_GROUP;
    kp.pdl_dep = s.cta_pair ? 0u : (uint32_t)p.pdl_dep;  // the pair kernel is launched without PDL
    if (kp.ctas == 0) return cudaSuccess;
    // The all-gather epilogue (extra destinations / multicast) is a separate
    // build of each kernel, so plain GEMMs carry none of its code.
    const bool gather = p.n_extra > 0 || p.mc_c != nullptr;
    if (s.cta_pair) return gather ? launch_pair<false, true>(ta, tb, kp, st) : launch_pair<false>(ta, tb, kp, st);
    if (gather) {
        switch (bn) {
            case 16: return launch_tile<16, tile_k_for(16), false, true>(ta, tb, kp, st);
            case 32: return launch_tile<32, tile_k_for(32), false, true>(ta, tb, kp, st);
            case 64: return launch_tile<64, tile_k_for(64), false, true>(ta, tb, kp, st);
            case 128: return launch_tile<128, tile_k_for(128), false, true>(ta, tb, kp, st);
            case 256: return launch_tile<256, tile_k_for(256), false, true>(ta, tb, kp, st);
            default: break;
        }
    }
    switch (bn) {
        case 16: return launch_tile<16, tile_k_for(16)>(ta, tb, kp, st);
        case 32: return launch_tile<32, tile_k_for(32)>(ta, tb, kp, st);
        case 64: return launch_tile<64, tile_k_for(64)>(ta, tb, kp, st);
        case 128: return launch_tile<128, tile_k_for(128)>(ta, tb, kp, st);
        case 256: return launch_tile<256, tile_k_for(256)>(ta, tb, kp, st);
        default:
            if (detail) *detail = "internal: unsupported tile_n";
            return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemm_i8_grouped(const GroupedProblem& g, uint32_t num_sms, cudaStream_t st, const char** detail)
{
    constexpr uint32_t BN = 256;
    // CTA pairs (256 x 256 tiles) whenever there are two SMs: a 1-CTA 128 x
    // 256 tile streams 1.5x the operand bytes per MMA and was L2-bound at
    // config 5 (57% tensor utilisation, against 84% for pairs).
    const bool pairs = num_sms != 1;
    CUtensorMap ta, tb;
    if (!make_operand_map(&ta, g.a, g.rows, g.K, g.lda, false, kTileM) ||
        !make_operand_map(&tb, g.b, g.groups * g.N, g.K, g.ldb, false, pairs ? 128 : BN)) {
        if (detail) *detail = "cuTensorMapEncodeTiled rejected an operand (alignment / stride)";
        return cudaErrorInvalidValue;
    }
    KParams kp{};
    kp.Mk = g.rows;
    kp.Nk = g.N;
    kp.K = g.K;
    kp.tiles_m = 0;  // per group, from the device counts
    kp.tiles_n = (g.N + BN - 1) / BN;
    kp.k_blocks = (g.K + kTileK_Grouped - 1) / kTileK_Grouped;
    kp.dp_tiles = 0;
    kp.ctas = num_sms ? num_sms : 148;
    kp.sk_iters = 0;
    kp.c = g.c;
    kp.ldc = g.ldc;
    kp.c_type = g.c_type;
    const uint32_t esz = g.c_type == 2 ? 4 : 2;
    kp.vec_store_ok = ((reinterpret_cast<uintptr_t>(g.c) & 15) == 0) && ((g.ldc * esz) % 16 == 0);
    kp.row_scale_vec = g.row_scale_vec;
    kp.col_scale_vec = g.col_scale_vec;
    kp.row_scale = g.row_scale;
    kp.col_scale = g.col_scale;
    kp.raster_group = 1;
    kp.grp_start = g.group_start;
    kp.grp_count = g.group_count;
    kp.groups = g.groups;
    if (pairs) {
        kp.k_blocks = (g.K + kPairBK - 1) / kPairBK;
        kp.ctas = 2 * ((num_sms ? num_sms : 148) / 2);
        return launch_pair<true>(ta, tb, kp, st);
    }
    return launch_tile<BN, kTileK_Grouped, true>(ta, tb, kp, st);
}

// --------------------------------------------------------------------------
// Device status + debug bounded wait
// --------------------------------------------------------------------------
namespace {
__global__ void debug_wait_kernel(uint64_t limit_ns)
{
    __shared__ alignas(8) uint64_t bar;
    const uint32_t b = smem_u32(&bar);
    if (threadIdx.x == 0) {
        mbar_init(b, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // Nothing ever arrives on this barrier: the wait must give up.
        mbar_wait(b, 0, SITE_DEBUG, nullptr, limit_ns);
    }
    __syncthreads();
}
}  // namespace

cudaError_t launch_debug_bounded_wait(uint64_t limit_ns, cudaStream_t st)
{
    debug_wait_kernel<<<1, 32, 0, st>>>(limit_ns);
    return cudaGetLastError();
}

}  // namespace b2sq
