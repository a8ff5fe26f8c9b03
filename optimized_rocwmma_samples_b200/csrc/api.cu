// api.cu — the extern "C" boundary declared in include/b2sq.h.
//
// Every entry point validates its arguments on the host before any CUDA call
// (so argument errors are reported without a device), maps the request onto
// the kernels and returns a status.  Nothing here allocates device memory,
// synchronises the device or exits the process (the reference's CHECK_HIP
// exits, common.hpp:33-46; its GEMM driver prints and returns on shapes it
// does not take, rocwmma_gemm_quantized.cpp:199-203).
#include "../../include/b2sq.h"
#include "kernels.h"

#include <cuda.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

namespace {

thread_local char g_msg[256] = "";

b2sq_status fail(b2sq_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
b2sq_status fail(b2sq_status s, const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return s;
}

b2sq_status ok()
{
    g_msg[0] = '\0';
    return B2SQ_OK;
}

b2sq_status cuda_fail(cudaError_t e, const char* where)
{
    return fail(B2SQ_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

bool qmax_ok(float q) { return std::isfinite(q) && q > 0.f && q <= 127.f; }

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Streaming multiprocessor count of the current device (cached per device).
cudaError_t current_sm_count(uint32_t* out)
{
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && cache[dev] > 0) {
        *out = (uint32_t)cache[dev];
        return cudaSuccess;
    }
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) cache[dev] = n;
    *out = (uint32_t)n;
    return cudaSuccess;
}

// Skinny M (decode): compute C^T = B^T A^T so the long N dimension fills the
// 128-row MMA and the few tokens become a 16..128-wide MMA N.
bool want_swap(uint32_t m, uint32_t n, b2sq_layout la)
{
    return m <= 128 && n >= 2 * m && n >= 256 && la == B2SQ_ROW_MAJOR;
}

struct Mapped {
    uint32_t swap;
    uint32_t Mk, Nk, a_mn, b_mn;
};

Mapped map_operands(uint32_t m, uint32_t n, b2sq_layout la, b2sq_layout lb)
{
    Mapped r{};
    r.swap = want_swap(m, n, la) ? 1u : 0u;
    if (r.swap) {
        r.Mk = n;
        r.Nk = m;
        r.a_mn = (lb == B2SQ_ROW_MAJOR) ? 1u : 0u;  // B [K,N] row-major: n contiguous
        r.b_mn = (la == B2SQ_COL_MAJOR) ? 1u : 0u;
    } else {
        r.Mk = m;
        r.Nk = n;
        r.a_mn = (la == B2SQ_COL_MAJOR) ? 1u : 0u;  // A [M,K] col-major: m contiguous
        r.b_mn = (lb == B2SQ_ROW_MAJOR) ? 1u : 0u;
    }
    return r;
}

b2sq_status validate_gemm(uint32_t m, uint32_t n, uint32_t k, const int8_t* a, b2sq_layout la, uint32_t lda,
                          const int8_t* b, b2sq_layout lb, uint32_t ldb, void* c, b2sq_dtype c_type, uint32_t ldc,
                          const float* sa, const float* sb)
{
    if (la != B2SQ_ROW_MAJOR && la != B2SQ_COL_MAJOR) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8: bad layout of a");
    if (lb != B2SQ_ROW_MAJOR && lb != B2SQ_COL_MAJOR) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8: bad layout of b");
    if (c_type != B2SQ_F16 && c_type != B2SQ_BF16 && c_type != B2SQ_I32)
        return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8: bad output dtype %d", (int)c_type);
    if (m == 0 || n == 0) return ok();
    if (!c) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8: c is null");
    if (ldc < n) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8: ldc %u < n %u", ldc, n);
    if (!aligned(c, c_type == B2SQ_I32 ? 4 : 2)) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8: c misaligned");
    if (k == 0) return ok();
    if (!a || !b) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8: a or b is null");
    const uint32_t min_lda = la == B2SQ_ROW_MAJOR ? k : m;
    const uint32_t min_ldb = lb == B2SQ_COL_MAJOR ? k : n;
    if (lda < min_lda) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8: lda %u < %u", lda, min_lda);
    if (ldb < min_ldb) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8: ldb %u < %u", ldb, min_ldb);
    if ((sa && !aligned(sa, 4)) || (sb && !aligned(sb, 4)))
        return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8: scale vector misaligned");
    if (!aligned(a, 16) || !aligned(b, 16))
        return fail(B2SQ_ERR_UNSUPPORTED, "gemm_i8: a and b must be 16-byte aligned (TMA)");
    if (lda % 16 || ldb % 16)
        return fail(B2SQ_ERR_UNSUPPORTED, "gemm_i8: lda (%u) and ldb (%u) must be multiples of 16 (TMA)", lda, ldb);
    return ok();
}

}  // namespace

b2sq_status b2sq::set_last_error(b2sq_status s, const char* msg) { return fail(s, "%s", msg); }

namespace {
std::mutex& status_mu()
{
    static std::mutex mu;
    return mu;
}
std::vector<b2sq::StatusReader>& status_readers()
{
    static std::vector<b2sq::StatusReader> v;  // constructed on first use, before any registration
    return v;
}
}  // namespace

void b2sq::register_status_reader(StatusReader reader)
{
    std::lock_guard<std::mutex> lock(status_mu());
    status_readers().push_back(reader);
}

// Reads and clears every translation unit's status word; *first_site gets the
// first non-zero site code found (0 if none).
cudaError_t b2sq::read_and_clear_all_status(cudaStream_t st, uint32_t* first_site)
{
    std::vector<StatusReader> rs;
    {
        std::lock_guard<std::mutex> lock(status_mu());
        rs = status_readers();
    }
    *first_site = 0;
    for (StatusReader r : rs) {
        uint32_t v = 0;
        cudaError_t e = r(st, &v);
        if (e != cudaSuccess) return e;
        if (*first_site == 0) *first_site = v;
    }
    return cudaSuccess;
}

extern "C" {

const char* b2sq_version(void) { return "b2sq 0.1.0 (sm_100a)"; }

const char* b2sq_status_string(b2sq_status s)
{
    switch (s) {
        case B2SQ_OK: return "ok";
        case B2SQ_ERR_INVALID_ARG: return "invalid argument";
        case B2SQ_ERR_UNSUPPORTED: return "unsupported";
        case B2SQ_ERR_CUDA: return "CUDA error";
        case B2SQ_ERR_TIMEOUT: return "device wait timed out";
    }
    return "unknown status";
}

const char* b2sq_last_error_message(void) { return g_msg; }

b2sq_status b2sq_smoothquant(const void* x_f16, const float* smooth_scale, int8_t* y, float* row_scale, uint32_t M,
                             uint32_t N, float quant_max, b2sq_stream_t stream)
{
    if (!qmax_ok(quant_max)) return fail(B2SQ_ERR_INVALID_ARG, "smoothquant: quant_max must be in (0, 127]");
    if (M == 0) return ok();
    if (!row_scale || (N > 0 && (!x_f16 || !smooth_scale || !y)))
        return fail(B2SQ_ERR_INVALID_ARG, "smoothquant: null pointer");
    if (!aligned(x_f16, 2) || !aligned(smooth_scale, 4) || !aligned(row_scale, 4))
        return fail(B2SQ_ERR_INVALID_ARG, "smoothquant: misaligned pointer");
    cudaError_t e = b2sq::launch_smoothquant(x_f16, smooth_scale, y, row_scale, M, N, quant_max,
                                             reinterpret_cast<cudaStream_t>(stream), nullptr);
    if (e != cudaSuccess) return cuda_fail(e, "smoothquant launch");
    return ok();
}

b2sq_status b2sq_moe_smoothquant(const void* x_f16, const float* smooth_scale, const int32_t* topk_ids, int8_t* qy,
                                 float* row_scale, uint32_t tokens, uint32_t hidden, uint32_t topk, uint32_t experts,
                                 float quant_max, const int32_t* row_perm, b2sq_stream_t stream)
{
    if (!qmax_ok(quant_max)) return fail(B2SQ_ERR_INVALID_ARG, "moe_smoothquant: quant_max must be in (0, 127]");
    if (tokens == 0 || topk == 0) return ok();
    if (!topk_ids || !row_scale || (hidden > 0 && (!x_f16 || !qy)) || (experts > 0 && hidden > 0 && !smooth_scale))
        return fail(B2SQ_ERR_INVALID_ARG, "moe_smoothquant: null pointer");
    if (!aligned(x_f16, 2) || !aligned(smooth_scale, 4) || !aligned(row_scale, 4) || !aligned(topk_ids, 4) ||
        !aligned(row_perm, 4))
        return fail(B2SQ_ERR_INVALID_ARG, "moe_smoothquant: misaligned pointer");
    if ((uint64_t)tokens * topk > 0xffffffffull)
        return fail(B2SQ_ERR_INVALID_ARG, "moe_smoothquant: tokens*topk overflows 32 bits");
    cudaError_t e = b2sq::launch_moe_smoothquant(x_f16, smooth_scale, topk_ids, qy, row_scale, tokens, hidden, topk,
                                                 experts, quant_max, row_perm,
                                                 reinterpret_cast<cudaStream_t>(stream), nullptr);
    if (e != cudaSuccess) return cuda_fail(e, "moe_smoothquant launch");
    return ok();
}

b2sq_status b2sq_gemm_i8_plan(uint32_t m, uint32_t n, uint32_t k, b2sq_layout la, b2sq_layout lb, int use_stream_k,
                              uint32_t num_sms, b2sq_gemm_plan* plan)
{
    if (!plan) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_plan: plan is null");
    if ((la != B2SQ_ROW_MAJOR && la != B2SQ_COL_MAJOR) || (lb != B2SQ_ROW_MAJOR && lb != B2SQ_COL_MAJOR))
        return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_plan: bad layout");
    if (num_sms == 0) {
        cudaError_t e = current_sm_count(&num_sms);
        if (e != cudaSuccess) return cuda_fail(e, "gemm_i8_plan: SM count");
    }
    const Mapped mp = map_operands(m, n, la, lb);
    b2sq::GemmSchedule s;
    b2sq::plan_gemm_schedule(mp.Mk, mp.Nk, k, mp.a_mn, mp.b_mn, use_stream_k != 0, num_sms, s);
    std::memset(plan, 0, sizeof(*plan));
    plan->swap_ab = mp.swap;
    plan->tile_m = s.cta_pair ? 2 * b2sq::kTileM : b2sq::kTileM;
    plan->cta_pair = s.cta_pair;
    plan->tile_n = s.tile_n;
    plan->tile_k = s.tile_k;
    plan->stages = s.stages;
    plan->tiles_m = s.tiles_m;
    plan->tiles_n = s.tiles_n;
    plan->k_blocks = s.k_blocks;
    plan->ctas = s.ctas;
    plan->dp_tiles = s.dp_tiles;
    plan->sk_iters = s.sk_iters;
    plan->sk_iters_per_cta_floor = s.ctas ? (uint32_t)(s.sk_iters / s.ctas) : 0;
    return ok();
}

b2sq_status b2sq_gemm_i8_workspace_size(uint32_t m, uint32_t n, uint32_t k, b2sq_layout la, b2sq_layout lb,
                                        size_t* bytes)
{
    if (!bytes) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_workspace_size: bytes is null");
    if ((la != B2SQ_ROW_MAJOR && la != B2SQ_COL_MAJOR) || (lb != B2SQ_ROW_MAJOR && lb != B2SQ_COL_MAJOR))
        return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_workspace_size: bad layout");
    *bytes = 0;
    if (m == 0 || n == 0 || k == 0) return ok();
    uint32_t sms = 0;
    cudaError_t e = current_sm_count(&sms);
    if (e != cudaSuccess) return cuda_fail(e, "gemm_i8_workspace_size: SM count");
    const Mapped mp = map_operands(m, n, la, lb);
    b2sq::GemmSchedule s;
    b2sq::plan_gemm_schedule(mp.Mk, mp.Nk, k, mp.a_mn, mp.b_mn, true, sms, s);
    *bytes = s.workspace_bytes;
    return ok();
}

}  // extern "C"

namespace {
// Body of b2sq_gemm_i8.  a_from_prev_kernel: the A operand and scale_a_row
// are written by the kernel enqueued just before on the same stream; the GEMM
// is then launched with programmatic dependent launch.
b2sq_status gemm_i8_impl(uint32_t m, uint32_t n, uint32_t k, const int8_t* a, b2sq_layout la, uint32_t lda,
                         const int8_t* b, b2sq_layout lb, uint32_t ldb, void* c, b2sq_dtype c_type, uint32_t ldc,
                         const float* scale_a_row, const float* scale_b_col, float scale_a, float scale_b,
                         void* workspace, size_t workspace_bytes, b2sq_stream_t stream, bool a_from_prev_kernel,
                         void* const* extra_c = nullptr, uint32_t n_extra = 0, void* mc_c = nullptr)
{
    b2sq_status st = validate_gemm(m, n, k, a, la, lda, b, lb, ldb, c, c_type, ldc, scale_a_row, scale_b_col);
    if (st != B2SQ_OK || m == 0 || n == 0) return st;
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    const size_t esz = c_type == B2SQ_I32 ? 4 : 2;
    if (k == 0) {  // empty sum: every output is +0
        for (uint32_t d = 0; d <= n_extra; ++d) {
            cudaError_t e = cudaMemset2DAsync(d == 0 ? c : extra_c[d - 1], (size_t)ldc * esz, 0, (size_t)n * esz, m, cs);
            if (e != cudaSuccess) return cuda_fail(e, "gemm_i8: zero fill");
        }
        return ok();
    }
    uint32_t sms = 0;
    cudaError_t e = current_sm_count(&sms);
    if (e != cudaSuccess) return cuda_fail(e, "gemm_i8: SM count");

    const Mapped mp = map_operands(m, n, la, lb);
    b2sq::GemmProblem p{};
    p.Mk = mp.Mk;
    p.Nk = mp.Nk;
    p.K = k;
    p.a_mn_major = mp.a_mn;
    p.b_mn_major = mp.b_mn;
    p.c = c;
    p.ldc = ldc;
    p.c_type = (int)c_type;
    p.transpose_out = (int)mp.swap;
    p.pdl_dep = a_from_prev_kernel ? (mp.swap ? 2 : 1) : 0;
    p.n_extra = n_extra;
    for (uint32_t d = 0; d < n_extra; ++d) p.extra_c[d] = extra_c[d];
    p.mc_c = mc_c;
    if (mp.swap) {
        p.a = b;
        p.lda = ldb;
        p.b = a;
        p.ldb = lda;
        p.row_scale_vec = scale_b_col;
        p.col_scale_vec = scale_a_row;
        p.row_scale = scale_b;
        p.col_scale = scale_a;
    } else {
        p.a = a;
        p.lda = lda;
        p.b = b;
        p.ldb = ldb;
        p.row_scale_vec = scale_a_row;
        p.col_scale_vec = scale_b_col;
        p.row_scale = scale_a;
        p.col_scale = scale_b;
    }
    b2sq::GemmSchedule s;
    b2sq::plan_gemm_schedule(p.Mk, p.Nk, k, p.a_mn_major, p.b_mn_major, workspace != nullptr, sms, s);
    if (s.workspace_bytes > 0 && (workspace == nullptr || workspace_bytes < s.workspace_bytes))
        b2sq::plan_gemm_schedule(p.Mk, p.Nk, k, p.a_mn_major, p.b_mn_major, false, sms, s);
    if (s.workspace_bytes > 0 && !aligned(workspace, 256))
        return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8: workspace must be 256-byte aligned");
    const char* detail = nullptr;
    e = b2sq::launch_gemm_i8(p, s, workspace, cs, &detail);
    if (e != cudaSuccess) {
        if (detail) return fail(B2SQ_ERR_UNSUPPORTED, "gemm_i8: %s", detail);
        return cuda_fail(e, "gemm_i8 launch");
    }
    return ok();
}
// Driver-API entry points used by the IPC helpers (no link-time libcuda dependency).
typedef CUresult (*MemGetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
MemGetAddressRangeFn get_address_range_fn()
{
    static MemGetAddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<MemGetAddressRangeFn>(ptr);
    });
    return fn;
}
}  // namespace

extern "C" {

b2sq_status b2sq_gemm_i8_allgather(uint32_t m, uint32_t n, uint32_t k, const int8_t* a, b2sq_layout la, uint32_t lda,
                                   const int8_t* b, b2sq_layout lb, uint32_t ldb, void* const* c_ranks,
                                   uint32_t world, uint32_t rank, uint32_t col_offset, b2sq_dtype c_type,
                                   uint32_t ldc, const float* scale_a_row, const float* scale_b_col, float scale_a,
                                   float scale_b, void* workspace, size_t workspace_bytes, b2sq_stream_t stream)
{
    if (world == 0 || world > b2sq::kMaxExtraOut + 1)
        return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_allgather: world must be in [1, %u]", b2sq::kMaxExtraOut + 1);
    if (rank >= world) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_allgather: rank %u >= world %u", rank, world);
    if (!c_ranks) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_allgather: c_ranks is null");
    if ((uint64_t)col_offset + n > ldc)
        return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_allgather: col_offset + n exceeds ldc");
    const size_t esz = c_type == B2SQ_I32 ? 4 : 2;
    void* dst[b2sq::kMaxExtraOut + 1];
    for (uint32_t r = 0; r < world; ++r) {
        if (!c_ranks[r]) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_allgather: c_ranks[%u] is null", r);
        dst[r] = static_cast<uint8_t*>(c_ranks[r]) + (size_t)col_offset * esz;
    }
    // Every destination gets the same stores: they must share their alignment.
    for (uint32_t r = 1; r < world; ++r)
        if ((reinterpret_cast<uintptr_t>(dst[r]) & 15) != (reinterpret_cast<uintptr_t>(dst[0]) & 15))
            return fail(B2SQ_ERR_UNSUPPORTED, "gemm_i8_allgather: the output buffers differ in 16-byte alignment");
    void* extra[b2sq::kMaxExtraOut];
    uint32_t ne = 0;
    for (uint32_t r = 0; r < world; ++r)
        if (r != rank) extra[ne++] = dst[r];
    return gemm_i8_impl(m, n, k, a, la, lda, b, lb, ldb, dst[rank], c_type, ldc, scale_a_row, scale_b_col, scale_a,
                        scale_b, workspace, workspace_bytes, stream, false, extra, ne);
}

b2sq_status b2sq_gemm_i8_allgather_mc(uint32_t m, uint32_t n, uint32_t k, const int8_t* a, b2sq_layout la,
                                      uint32_t lda, const int8_t* b, b2sq_layout lb, uint32_t ldb, void* c_local,
                                      void* c_multicast, uint32_t col_offset, b2sq_dtype c_type, uint32_t ldc,
                                      const float* scale_a_row, const float* scale_b_col, float scale_a,
                                      float scale_b, void* workspace, size_t workspace_bytes, b2sq_stream_t stream)
{
    if (!c_local || !c_multicast) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_allgather_mc: null output pointer");
    if ((uint64_t)col_offset + n > ldc)
        return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_allgather_mc: col_offset + n exceeds ldc");
    if (m == 0 || n == 0) return ok();
    // every output store must be a 16-byte vector store (multimem.st has no
    // narrower form here): no operand swap, whole 32-column chunks, aligned rows
    if (m <= 128 || la != B2SQ_ROW_MAJOR)
        return fail(B2SQ_ERR_UNSUPPORTED, "gemm_i8_allgather_mc: needs m > 128 and row-major a "
                                          "(use b2sq_gemm_i8_allgather for decode shapes)");
    const size_t esz = c_type == B2SQ_I32 ? 4 : 2;
    uint8_t* dst = static_cast<uint8_t*>(c_local) + (size_t)col_offset * esz;
    uint8_t* mc = static_cast<uint8_t*>(c_multicast) + (size_t)col_offset * esz;
    if (n % 64 || !aligned(dst, 16) || !aligned(mc, 16) || ((size_t)ldc * esz) % 16)
        return fail(B2SQ_ERR_UNSUPPORTED, "gemm_i8_allgather_mc: n a multiple of 64 and 16-byte aligned output rows");
    return gemm_i8_impl(m, n, k, a, la, lda, b, lb, ldb, dst, c_type, ldc, scale_a_row, scale_b_col, scale_a, scale_b,
                        workspace, workspace_bytes, stream, false, nullptr, 0, mc);
}

b2sq_status b2sq_ipc_export(const void* dev_ptr, b2sq_ipc_handle* handle, uint64_t* offset)
{
    if (!dev_ptr || !handle || !offset) return fail(B2SQ_ERR_INVALID_ARG, "ipc_export: null pointer");
    MemGetAddressRangeFn range = get_address_range_fn();
    if (!range) return fail(B2SQ_ERR_CUDA, "ipc_export: cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
        return fail(B2SQ_ERR_INVALID_ARG, "ipc_export: not a device allocation");
    static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(handle->bytes), "IPC handle size");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return cuda_fail(e, "ipc_export: cudaIpcGetMemHandle (memory from cudaMalloc is required)");
    std::memcpy(handle->bytes, &h, sizeof(h));
    *offset = reinterpret_cast<uint64_t>(dev_ptr) - (uint64_t)base;
    return ok();
}

b2sq_status b2sq_ipc_open(const b2sq_ipc_handle* handle, void** base)
{
    if (!handle || !base) return fail(B2SQ_ERR_INVALID_ARG, "ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle->bytes, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "ipc_open: cudaIpcOpenMemHandle");
    return ok();
}

b2sq_status b2sq_ipc_close(void* base)
{
    if (!base) return fail(B2SQ_ERR_INVALID_ARG, "ipc_close: null pointer");
    cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) return cuda_fail(e, "ipc_close: cudaIpcCloseMemHandle");
    return ok();
}

b2sq_status b2sq_gemm_i8(uint32_t m, uint32_t n, uint32_t k, const int8_t* a, b2sq_layout la, uint32_t lda,
                         const int8_t* b, b2sq_layout lb, uint32_t ldb, void* c, b2sq_dtype c_type, uint32_t ldc,
                         const float* scale_a_row, const float* scale_b_col, float scale_a, float scale_b,
                         void* workspace, size_t workspace_bytes, b2sq_stream_t stream)
{
    return gemm_i8_impl(m, n, k, a, la, lda, b, lb, ldb, c, c_type, ldc, scale_a_row, scale_b_col, scale_a, scale_b,
                        workspace, workspace_bytes, stream, false);
}

b2sq_status b2sq_smoothquant_gemm_i8(const void* x_f16, const float* smooth_scale, float quant_max, int8_t* xq,
                                     float* row_scale, uint32_t m, uint32_t k, const int8_t* w, b2sq_layout lw,
                                     uint32_t ldw, uint32_t n, void* c, b2sq_dtype c_type, uint32_t ldc,
                                     const float* scale_w_col, float scale_w, void* workspace, size_t workspace_bytes,
                                     b2sq_stream_t stream)
{
    if (c_type == B2SQ_I32) return fail(B2SQ_ERR_INVALID_ARG, "smoothquant_gemm_i8: output must be f16 or bf16");
    if (m == 0 || n == 0) return ok();
    if (k % 16) return fail(B2SQ_ERR_UNSUPPORTED, "smoothquant_gemm_i8: k must be a multiple of 16 (TMA)");
    if (!aligned(xq, 16)) return fail(B2SQ_ERR_UNSUPPORTED, "smoothquant_gemm_i8: xq must be 16-byte aligned");
    b2sq_status st = b2sq_smoothquant(x_f16, smooth_scale, xq, row_scale, m, k, quant_max, stream);
    if (st != B2SQ_OK) return st;
    return gemm_i8_impl(m, n, k, xq, B2SQ_ROW_MAJOR, k, w, lw, ldw, c, c_type, ldc, row_scale, scale_w_col, 1.f,
                        scale_w, workspace, workspace_bytes, stream, true);
}

b2sq_status b2sq_topk_softmax(const void* logits_f16, float* topk_weights, int32_t* topk_indices, uint32_t tokens,
                              uint32_t experts, uint32_t topk, b2sq_stream_t stream)
{
    if (tokens == 0 || experts == 0 || topk == 0) return ok();  // the reference writes nothing
    if ((uint64_t)tokens * experts > 0x7fffffffffffull || (uint64_t)tokens * topk > 0x7fffffffffffull)
        return fail(B2SQ_ERR_INVALID_ARG, "topk_softmax: tokens * experts too large");
    if ((uint64_t)tokens * (experts > 64 ? 32 : 8) / 128 >= 0x7fffffffull)
        return fail(B2SQ_ERR_INVALID_ARG, "topk_softmax: too many tokens for one launch");
    if (!logits_f16 || !topk_weights || !topk_indices) return fail(B2SQ_ERR_INVALID_ARG, "topk_softmax: null pointer");
    if (!aligned(logits_f16, 2) || !aligned(topk_weights, 4) || !aligned(topk_indices, 4))
        return fail(B2SQ_ERR_INVALID_ARG, "topk_softmax: misaligned pointer");
    cudaError_t e = b2sq::launch_topk_softmax(logits_f16, topk_weights, topk_indices, tokens, experts, topk,
                                              reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "topk_softmax launch");
    return ok();
}

b2sq_status b2sq_moe_sorting(const int32_t* topk_ids, uint32_t tokens, uint32_t topk, uint32_t experts,
                             uint32_t unit_size, int32_t* expert_count, int32_t* expert_start,
                             int32_t* sorted_token_ids, int32_t* row_perm, b2sq_stream_t stream)
{
    if (experts == 0 || experts > 1024) return fail(B2SQ_ERR_INVALID_ARG, "moe_sorting: experts must be in [1, 1024]");
    if (unit_size == 0) return fail(B2SQ_ERR_INVALID_ARG, "moe_sorting: unit_size must be >= 1");
    if ((uint64_t)tokens * topk > 0x7fffffffull) return fail(B2SQ_ERR_INVALID_ARG, "moe_sorting: too many rows");
    if (!expert_count || !expert_start || ((uint64_t)tokens * topk > 0 && (!topk_ids || !sorted_token_ids)))
        return fail(B2SQ_ERR_INVALID_ARG, "moe_sorting: null pointer");
    cudaError_t e = b2sq::launch_moe_sort(topk_ids, tokens, topk, experts, unit_size, expert_count, expert_start,
                                          sorted_token_ids, row_perm, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "moe_sorting launch");
    return ok();
}

b2sq_status b2sq_gemm_i8_grouped(uint32_t groups, uint32_t rows, uint32_t n, uint32_t k, const int8_t* a,
                                 uint32_t lda, const int8_t* w, uint32_t ldb, void* c, b2sq_dtype c_type,
                                 uint32_t ldc, const float* scale_a_row, const float* scale_b_col, float scale_a,
                                 float scale_b, const int32_t* group_start, const int32_t* group_count,
                                 b2sq_stream_t stream)
{
    if (c_type != B2SQ_F16 && c_type != B2SQ_BF16 && c_type != B2SQ_I32)
        return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_grouped: bad output dtype %d", (int)c_type);
    if (groups == 0 || rows == 0 || n == 0) return ok();
    if (groups > b2sq::kMaxGroups) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_grouped: groups must be <= 1024");
    if (k == 0) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_grouped: k must be >= 1");
    if (!a || !w || !c || !group_start || !group_count)
        return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_grouped: null pointer");
    if (lda < k || ldb < k || ldc < n) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_grouped: leading dimension too small");
    if ((uint64_t)groups * n > 0xffffffffull) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_grouped: groups*n too large");
    if (!aligned(c, c_type == B2SQ_I32 ? 4 : 2)) return fail(B2SQ_ERR_INVALID_ARG, "gemm_i8_grouped: c misaligned");
    if (!aligned(a, 16) || !aligned(w, 16) || lda % 16 || ldb % 16)
        return fail(B2SQ_ERR_UNSUPPORTED, "gemm_i8_grouped: a, w 16-byte aligned and lda, ldb multiples of 16 (TMA)");
    uint32_t sms = 0;
    cudaError_t e = current_sm_count(&sms);
    if (e != cudaSuccess) return cuda_fail(e, "gemm_i8_grouped: SM count");
    b2sq::GroupedProblem g{};
    g.groups = groups;
    g.rows = rows;
    g.N = n;
    g.K = k;
    g.a = a;
    g.lda = lda;
    g.b = w;
    g.ldb = ldb;
    g.c = c;
    g.ldc = ldc;
    g.c_type = (int)c_type;
    g.row_scale_vec = scale_a_row;
    g.col_scale_vec = scale_b_col;
    g.row_scale = scale_a;
    g.col_scale = scale_b;
    g.group_start = group_start;
    g.group_count = group_count;
    const char* detail = nullptr;
    e = b2sq::launch_gemm_i8_grouped(g, sms, reinterpret_cast<cudaStream_t>(stream), &detail);
    if (e != cudaSuccess) {
        if (detail) return fail(B2SQ_ERR_UNSUPPORTED, "gemm_i8_grouped: %s", detail);
        return cuda_fail(e, "gemm_i8_grouped launch");
    }
    return ok();
}

b2sq_status b2sq_last_device_error(b2sq_stream_t stream, uint32_t* where)
{
    uint32_t v = 0;
    cudaError_t e = b2sq::read_and_clear_all_status(reinterpret_cast<cudaStream_t>(stream), &v);
    if (e != cudaSuccess) return cuda_fail(e, "last_device_error");
    if (where) *where = v;
    if (v != 0) return fail(B2SQ_ERR_TIMEOUT, "device wait gave up at site %u", v);
    return ok();
}

b2sq_status b2sq_debug_bounded_wait(uint32_t timeout_us, b2sq_stream_t stream)
{
    if (timeout_us == 0 || timeout_us > 10u * 1000u * 1000u)
        return fail(B2SQ_ERR_INVALID_ARG, "debug_bounded_wait: timeout_us must be in (0, 10 s]");
    cudaError_t e = b2sq::launch_debug_bounded_wait((uint64_t)timeout_us * 1000ull,
                                                    reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "debug_bounded_wait launch");
    return b2sq_last_device_error(stream, nullptr);
}

}  // extern "C"
