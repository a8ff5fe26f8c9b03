// host_gemm.cu — b2sq_gemm_i8_host: the quantized GEMM for operands and
// result in host memory.
//
// Replaces the host side of the reference's GEMM driver (rocwmma_gemm_quantized.cpp:
// 214-218 and its copy back): copy A and B to the device, run the kernel,
// copy C back, one step after another.  Here the problem is cut into
// row_chunks x col_chunks output blocks and the transfers are pipelined
// against each other and against the GEMMs on three streams:
//
//   copy-in stream   A_0, B_0, A_1, B_1, ...   (+ scales)
//   GEMM stream      on each arrival, one GEMM over the strip of blocks it
//                    completes (A_i: blocks (i, j) of the B chunks already
//                    in; B_j: blocks (i, j) of the A chunks already in)
//   copy-out stream  each strip back to the host (pitched copy) once computed
//
// so the first block leaves the device after 1/row_chunks of A and
// 1/col_chunks of B have arrived, and host->device and device->host traffic
// overlap for most of the call (PCIe is full duplex).  The caller's stream
// waits for the last copy back.  Consecutive calls on two alternating device
// buffers overlap as well: a call's copies in and GEMMs wait only for the
// previous call on the same buffer.  Nothing is allocated:
// the caller passes one device buffer of b2sq_gemm_i8_host_buffer_size bytes.
// The copy streams and events are created once per device and reused.
#include "../../include/b2sq.h"
#include "kernels.h"

#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

namespace {

constexpr size_t kAlign = 256;
inline size_t up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

struct Layout {
    size_t a, w, sa, sb, c, total;
};

Layout layout(uint32_t m, uint32_t n, uint32_t k, b2sq_dtype c_type)
{
    const size_t esz = c_type == B2SQ_I32 ? 4 : 2;
    Layout l{};
    l.a = 0;
    l.w = l.a + up((size_t)m * k);
    l.sa = l.w + up((size_t)n * k);
    l.sb = l.sa + up((size_t)m * 4);
    l.c = l.sb + up((size_t)n * 4);
    l.total = l.c + up((size_t)m * n * esz);
    return l;
}

// Chunk boundaries: multiples of 256 rows (whole CTA-pair tiles), as even as that allows.
std::vector<uint32_t> cuts(uint32_t len, uint32_t chunks)
{
    const uint32_t units = (len + 255) / 256;
    if (chunks > units) chunks = units;
    if (chunks == 0) chunks = 1;
    std::vector<uint32_t> c(chunks + 1);
    for (uint32_t i = 0; i <= chunks; ++i) {
        const uint64_t u = (uint64_t)units * i / chunks;
        c[i] = (uint32_t)(u * 256 < len ? u * 256 : len);
    }
    return c;
}

// Measured at 8192^3 (bf16 out, B200, PCIe 5), one call / ten back-to-back
// calls on alternating buffers, ms per call: 1x1 5.18 / 3.17, 2x2 4.13 / 3.20,
// 3x3 3.77 / 3.19, 4x4 3.70 / 3.31, 8x8 3.72 / 3.29.  Finer blocks start the
// copy back sooner within one call; between calls the overlap of one call's
// copy back with the next call's copies in does that already, and finer
// pitched copies cost bandwidth.
uint32_t auto_chunks(uint32_t len) { return len >= 2048 ? 3 : len >= 1024 ? 2 : 1; }

struct DeviceCtx {
    bool ready = false;
    cudaStream_t s_in = nullptr, s_out = nullptr, s_mm = nullptr;
    // Per device buffer: the event after the last copy-back of the previous
    // call that used it (its GEMMs precede that copy-back).
    std::vector<std::pair<void*, cudaEvent_t>> buf_done;
    std::vector<cudaEvent_t> ev;  // grown on demand
    std::mutex mu;                 // one call at a time per device
};

DeviceCtx g_ctx[64];
std::mutex g_ctx_mu;

cudaError_t events(DeviceCtx& d, size_t n)
{
    while (d.ev.size() < n) {
        cudaEvent_t e;
        cudaError_t r = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
        if (r != cudaSuccess) return r;
        d.ev.push_back(e);
    }
    return cudaSuccess;
}

b2sq_status cuda_err(cudaError_t e, const char* where)
{
    char msg[200];
    std::snprintf(msg, sizeof(msg), "gemm_i8_host: %s: %s", where, cudaGetErrorString(e));
    return b2sq::set_last_error(B2SQ_ERR_CUDA, msg);
}

}  // namespace

extern "C" {

B2SQ_API b2sq_status b2sq_gemm_i8_host_buffer_size(uint32_t m, uint32_t n, uint32_t k, b2sq_dtype c_type,
                                                   size_t* bytes)
{
    if (!bytes) return b2sq::set_last_error(B2SQ_ERR_INVALID_ARG, "gemm_i8_host_buffer_size: bytes is null");
    if (c_type != B2SQ_F16 && c_type != B2SQ_BF16 && c_type != B2SQ_I32)
        return b2sq::set_last_error(B2SQ_ERR_INVALID_ARG, "gemm_i8_host_buffer_size: bad output dtype");
    *bytes = layout(m, n, k, c_type).total;
    return B2SQ_OK;
}

B2SQ_API b2sq_status b2sq_gemm_i8_host(uint32_t m, uint32_t n, uint32_t k, const int8_t* h_a, const int8_t* h_w,
                                       const float* h_scale_a_row, const float* h_scale_b_col, float scale_a,
                                       float scale_b, void* h_c, b2sq_dtype c_type, void* dev_buffer,
                                       size_t dev_buffer_bytes, uint32_t row_chunks, uint32_t col_chunks,
                                       b2sq_stream_t stream)
{
    if (c_type != B2SQ_F16 && c_type != B2SQ_BF16 && c_type != B2SQ_I32)
        return b2sq::set_last_error(B2SQ_ERR_INVALID_ARG, "gemm_i8_host: bad output dtype");
    if (m == 0 || n == 0) return B2SQ_OK;
    if (!h_c || !dev_buffer || (k > 0 && (!h_a || !h_w)))
        return b2sq::set_last_error(B2SQ_ERR_INVALID_ARG, "gemm_i8_host: null pointer");
    if (k % 16) return b2sq::set_last_error(B2SQ_ERR_UNSUPPORTED, "gemm_i8_host: k must be a multiple of 16 (TMA)");
    const Layout L = layout(m, n, k, c_type);
    if (dev_buffer_bytes < L.total)
        return b2sq::set_last_error(B2SQ_ERR_INVALID_ARG, "gemm_i8_host: device buffer smaller than "
                                                          "b2sq_gemm_i8_host_buffer_size");
    if (reinterpret_cast<uintptr_t>(dev_buffer) % kAlign)
        return b2sq::set_last_error(B2SQ_ERR_INVALID_ARG, "gemm_i8_host: device buffer must be 256-byte aligned");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return b2sq::set_last_error(B2SQ_ERR_UNSUPPORTED, "gemm_i8_host: device index >= 64");
    DeviceCtx& d = g_ctx[dev];
    std::lock_guard<std::mutex> call_lock(d.mu);
    if (!d.ready) {
        std::lock_guard<std::mutex> lock(g_ctx_mu);
        if ((e = cudaStreamCreateWithFlags(&d.s_in, cudaStreamNonBlocking)) != cudaSuccess) return cuda_err(e, "stream");
        if ((e = cudaStreamCreateWithFlags(&d.s_out, cudaStreamNonBlocking)) != cudaSuccess) return cuda_err(e, "stream");
        if ((e = cudaStreamCreateWithFlags(&d.s_mm, cudaStreamNonBlocking)) != cudaSuccess) return cuda_err(e, "stream");
        d.ready = true;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const std::vector<uint32_t> rc = cuts(m, row_chunks ? row_chunks : auto_chunks(m));
    const std::vector<uint32_t> cc = cuts(n, col_chunks ? col_chunks : auto_chunks(n));
    const size_t mi = rc.size() - 1, nj = cc.size() - 1;
    // events: [0] unused, [1, 1+mi) A_i in, [1+mi, 1+mi+nj) B_j in, then one per strip, then copy-out done
    const size_t ev_a = 1, ev_w = ev_a + mi, ev_c = ev_w + nj, ev_done = ev_c + mi + nj;
    if ((e = events(d, ev_done + 1)) != cudaSuccess) return cuda_err(e, "events");
    uint8_t* base = static_cast<uint8_t*>(dev_buffer);
    int8_t* d_a = reinterpret_cast<int8_t*>(base + L.a);
    int8_t* d_w = reinterpret_cast<int8_t*>(base + L.w);
    float* d_sa = h_scale_a_row ? reinterpret_cast<float*>(base + L.sa) : nullptr;
    float* d_sb = h_scale_b_col ? reinterpret_cast<float*>(base + L.sb) : nullptr;
    uint8_t* d_c = base + L.c;
    const size_t esz = c_type == B2SQ_I32 ? 4 : 2;

#define B2SQ_TRY(expr, where)                       \
    do {                                            \
        cudaError_t r_ = (expr);                    \
        if (r_ != cudaSuccess) return cuda_err(r_, where); \
    } while (0)

    // the copies start after whatever the caller enqueued before (earlier use of the buffer)
    // The copies into dev_buffer wait only for this library's previous call on
    // the same buffer (its GEMMs and copy-back), not for everything queued on
    // `stream`: calls on two alternating buffers overlap, the next call's
    // inputs going up while the previous call's result comes down.
    cudaEvent_t done = nullptr;
    for (auto& bd : d.buf_done)
        if (bd.first == dev_buffer) done = bd.second;
    const bool first_use = done == nullptr;
    if (first_use) {
        B2SQ_TRY(cudaEventCreateWithFlags(&done, cudaEventDisableTiming), "events");
        d.buf_done.emplace_back(dev_buffer, done);
    } else {
        B2SQ_TRY(cudaStreamWaitEvent(d.s_in, done, 0), "wait");
        B2SQ_TRY(cudaStreamWaitEvent(d.s_mm, done, 0), "wait");
    }
    if (d_sb) B2SQ_TRY(cudaMemcpyAsync(d_sb, h_scale_b_col, (size_t)n * 4, cudaMemcpyHostToDevice, d.s_in), "copy in");
    // Input chunks arrive alternately (A_0, B_0, A_1, B_1, ...): every block
    // needs one chunk of each, so after f of the input bytes about f^2 of the
    // output can be computed and sent back -- the most any order allows.
    struct Arrival {
        bool is_a;
        size_t idx;
    };
    std::vector<Arrival> order;
    for (size_t t = 0; t < mi || t < nj; ++t) {
        if (t < mi) order.push_back({true, t});
        if (t < nj) order.push_back({false, t});
    }
    for (const Arrival& ar : order) {
        cudaError_t r = cudaSuccess;
        if (ar.is_a) {
            const size_t r0 = rc[ar.idx], r1 = rc[ar.idx + 1];
            if (k) r = cudaMemcpyAsync(d_a + r0 * k, h_a + r0 * k, (r1 - r0) * k, cudaMemcpyHostToDevice, d.s_in);
            if (r == cudaSuccess && d_sa)
                r = cudaMemcpyAsync(d_sa + r0, h_scale_a_row + r0, (r1 - r0) * 4, cudaMemcpyHostToDevice, d.s_in);
            if (r == cudaSuccess) r = cudaEventRecord(d.ev[ev_a + ar.idx], d.s_in);
        } else {
            const size_t c0 = cc[ar.idx], c1 = cc[ar.idx + 1];
            if (k) r = cudaMemcpyAsync(d_w + c0 * k, h_w + c0 * k, (c1 - c0) * k, cudaMemcpyHostToDevice, d.s_in);
            if (r == cudaSuccess) r = cudaEventRecord(d.ev[ev_w + ar.idx], d.s_in);
        }
        if (r != cudaSuccess) return cuda_err(r, "copy in");
    }
    // Each arrival completes one strip of blocks: A_i the blocks (i, j < B's
    // arrived), B_j the blocks (i < A's arrived, j).  The strip is one GEMM
    // (its A rows or B rows are contiguous) and one pitched copy back.
    size_t na = 0, nb = 0, strip = 0;
    for (const Arrival& ar : order) {
        B2SQ_TRY(cudaStreamWaitEvent(d.s_mm, d.ev[ar.is_a ? ev_a + ar.idx : ev_w + ar.idx], 0), "wait");
        uint32_t r0, r1, c0, c1;
        if (ar.is_a) {
            r0 = rc[ar.idx], r1 = rc[ar.idx + 1], c0 = 0, c1 = cc[nb];
            ++na;
        } else {
            r0 = 0, r1 = rc[na], c0 = cc[ar.idx], c1 = cc[ar.idx + 1];
            ++nb;
        }
        if (r1 <= r0 || c1 <= c0) continue;  // nothing to pair with yet
        uint8_t* cblk = d_c + ((size_t)r0 * n + c0) * esz;
        b2sq_status s = b2sq_gemm_i8(r1 - r0, c1 - c0, k, d_a + (size_t)r0 * k, B2SQ_ROW_MAJOR, k,
                                     d_w + (size_t)c0 * k, B2SQ_COL_MAJOR, k, cblk, c_type, n,
                                     d_sa ? d_sa + r0 : nullptr, d_sb ? d_sb + c0 : nullptr, scale_a, scale_b,
                                     nullptr, 0, reinterpret_cast<b2sq_stream_t>(d.s_mm));
        if (s != B2SQ_OK) return s;
        B2SQ_TRY(cudaEventRecord(d.ev[ev_c + strip], d.s_mm), "record");
        B2SQ_TRY(cudaStreamWaitEvent(d.s_out, d.ev[ev_c + strip], 0), "wait");
        B2SQ_TRY(cudaMemcpy2DAsync(static_cast<uint8_t*>(h_c) + ((size_t)r0 * n + c0) * esz, (size_t)n * esz, cblk,
                                   (size_t)n * esz, (size_t)(c1 - c0) * esz, r1 - r0, cudaMemcpyDeviceToHost,
                                   d.s_out),
                 "copy out");
        ++strip;
    }
    // the caller's stream completes when the result is in host memory
    B2SQ_TRY(cudaEventRecord(d.ev[ev_done], d.s_out), "record");
    B2SQ_TRY(cudaEventRecord(done, d.s_out), "record");
    B2SQ_TRY(cudaStreamWaitEvent(st, d.ev[ev_done], 0), "wait");
#undef B2SQ_TRY
    return B2SQ_OK;
}

}  // extern "C"
