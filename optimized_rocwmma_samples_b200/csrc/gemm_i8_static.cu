// gemm_i8_static.cu — b2sq_gemm_i8 for callers that cannot allocate device
// memory.
//
// b2sq_gemm_i8 takes its stream-K scratch from the caller.  Some callers have
// no way to provide it: a host bound over a plain C FFI with no device
// allocator of its own, or a serving process that has handed all of HBM to
// its own pool and forbids cudaMalloc on the request path (cudaMalloc can also
// synchronise the device, which such a process cannot afford mid-request).
// This entry point takes the scratch from a fixed array compiled into the
// library instead, so it allocates nothing.
//
// The array lives in every GPU that loads the library, for the life of the
// process.  Calls share it: overlapping calls on the GPU (different streams,
// or different host threads without ordering) race on it.
#include "../../include/b2sq.h"
#include "kernels.h"

#include <cstdio>
#include <mutex>

namespace {

// Largest stream-K scratch a call may need.  24 MiB covers every shape whose
// tiles are at most 128 wide (148 SMs) and every shape whose schedule needs
// no stream-K; larger needs (256-wide stream-K tiles) are rejected.
constexpr size_t kStaticScratchBytes = 24u << 20;

static __device__ __align__(256) unsigned char g_gemm_scratch[kStaticScratchBytes];

// Device address of g_gemm_scratch on the current device.  In host code the
// name g_gemm_scratch is only a host-side stand-in, so the address is looked
// up once per device, with that device current.  The cache assumes the
// device's context lives as long as the process: after cudaDeviceReset the
// address is stale and the entry point must not be called again.
cudaError_t scratch_address(void** out)
{
    static std::mutex mu;
    static void* addr[64] = {nullptr};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_gemm_scratch);
        if (e != cudaSuccess) return e;
        addr[dev] = p;
    }
    *out = addr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" {

B2SQ_API b2sq_status b2sq_gemm_i8_no_alloc(uint32_t m, uint32_t n, uint32_t k, const int8_t* a, b2sq_layout la,
                                           uint32_t lda, const int8_t* b, b2sq_layout lb, uint32_t ldb, void* c,
                                           b2sq_dtype c_type, uint32_t ldc, const float* scale_a_row,
                                           const float* scale_b_col, float scale_a, float scale_b,
                                           b2sq_stream_t stream)
{
    size_t need = 0;
    b2sq_status st = B2SQ_OK;
    if (m != 0 && n != 0 && k != 0) {
        st = b2sq_gemm_i8_workspace_size(m, n, k, la, lb, &need);
        if (st != B2SQ_OK) return st;
        if (need > kStaticScratchBytes) {
            char msg[224];
            std::snprintf(msg, sizeof(msg),
                          "gemm_i8_no_alloc: this shape needs %zu bytes of scratch, more than the library's "
                          "fixed %zu; b2sq_gemm_i8 with a null workspace runs it without scratch (whole tiles)",
                          need, kStaticScratchBytes);
            return b2sq::set_last_error(B2SQ_ERR_UNSUPPORTED, msg);
        }
    }
    void* scratch = nullptr;
    if (need > 0) {
        cudaError_t e = scratch_address(&scratch);
        if (e != cudaSuccess) return b2sq::set_last_error(B2SQ_ERR_CUDA, cudaGetErrorString(e));
        // The per-tile counters at the head of the scratch must start at zero;
        // the previous call normally leaves them so, but clear them anyway (an
        // interrupted call may not have).
        e = cudaMemsetAsync(scratch, 0, b2sq::kWsCounterBytes, reinterpret_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return b2sq::set_last_error(B2SQ_ERR_CUDA, cudaGetErrorString(e));
    }
    return b2sq_gemm_i8(m, n, k, a, la, lda, b, lb, ldb, c, c_type, ldc, scale_a_row, scale_b_col, scale_a, scale_b,
                        scratch, need > 0 ? kStaticScratchBytes : 0, stream);
}

}  // extern "C"
