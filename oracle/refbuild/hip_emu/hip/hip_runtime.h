// hip_runtime.h — host emulation of the HIP device model, so that the
// reference's own kernel sources (HIP, AMD-only) compile with g++ and run on
// the CPU as a parity checker.  Test infrastructure only: nothing here is
// part of the library.
//
// Model: every GPU thread of a block is a fiber (ucontext) on one OS thread;
// blocks run one after another on that OS thread (blocks of one launch may be
// spread over several OS threads).  Barriers (__syncthreads, __syncwarp) and
// lane exchanges (__shfl*) are cooperative switch points; a barrier completes
// when every thread of its scope that has not returned has arrived, which is
// what the hardware does for exited threads.  Wavefronts are 64 lanes, the
// warp size the reference kernels are written for.  __shared__ variables are
// thread_local, i.e. one copy per block in flight.
#pragma once

#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <tuple>
#include <type_traits>

#include "hip_fp16.h"

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __launch_bounds__(...)
#define __shared__ thread_local
#define __restrict__ __restrict

struct dim3 {
    uint32_t x, y, z;
    constexpr dim3(uint32_t x_ = 1, uint32_t y_ = 1, uint32_t z_ = 1) : x(x_), y(y_), z(z_) {}
};


namespace hipemu {

constexpr int kWave = 64;

struct Coords {
    dim3 thread, block, block_dim, grid_dim;
};
// Coordinates of the fiber that is running on this OS thread.
extern thread_local Coords* g_cur;

void sync_block();
void sync_wave();
// Publishes 8 bytes from this lane, waits for the wave, returns the 8 bytes
// published by lane `src` of this wave (src outside [0, 64): own value).
uint64_t exchange(uint64_t mine, int src);
int lane_id();

// Runs fn(block) for every block of the grid with fibers for its threads.
using BlockBody = void (*)(void* ctx);
void run_grid(dim3 grid, dim3 block, void* ctx, BlockBody body);

template <typename T>
T shfl_src(T v, int src)
{
    static_assert(sizeof(T) <= 8 && std::is_trivially_copyable<T>::value, "shuffle of a scalar");
    uint64_t bits = 0;
    std::memcpy(&bits, &v, sizeof(T));
    uint64_t r = exchange(bits, src);
    T out;
    std::memcpy(&out, &r, sizeof(T));
    return out;
}

}  // namespace hipemu

#define threadIdx (hipemu::g_cur->thread)
#define blockIdx (hipemu::g_cur->block)
#define blockDim (hipemu::g_cur->block_dim)
#define gridDim (hipemu::g_cur->grid_dim)
#define warpSize 64

inline void __syncthreads() { hipemu::sync_block(); }
inline void __syncwarp() { hipemu::sync_wave(); }
inline void __syncwarp(uint64_t) { hipemu::sync_wave(); }

// Lane exchanges with HIP's width argument: segments of `width` lanes.
template <typename T>
inline T __shfl(T v, int src_lane, int width = warpSize)
{
    const int lane = hipemu::lane_id();
    const int base = (lane / width) * width;
    return hipemu::shfl_src(v, base + ((src_lane % width) + width) % width);
}
template <typename T>
inline T __shfl_down(T v, unsigned int delta, int width = warpSize)
{
    const int lane = hipemu::lane_id();
    const int in_seg = lane % width;
    const int src = (in_seg + (int)delta < width) ? lane + (int)delta : lane;
    return hipemu::shfl_src(v, src);
}
template <typename T>
inline T __shfl_up(T v, unsigned int delta, int width = warpSize)
{
    const int lane = hipemu::lane_id();
    const int in_seg = lane % width;
    const int src = (in_seg - (int)delta >= 0) ? lane - (int)delta : lane;
    return hipemu::shfl_src(v, src);
}
template <typename T>
inline T __shfl_xor(T v, int mask, int width = warpSize)
{
    const int lane = hipemu::lane_id();
    const int dst = lane ^ mask;
    const int src = (dst / width == lane / width) ? dst : lane;
    return hipemu::shfl_src(v, src);
}

// Blocks of one launch may run on several OS threads at once, so atomics
// on global memory are real atomics.
template <typename T>
inline T atomicAdd(T* p, T v)
{
    static_assert(std::is_integral<T>::value, "integer atomics only");
    return __atomic_fetch_add(p, v, __ATOMIC_SEQ_CST);
}
template <typename T>
inline T atomicMax(T* p, T v)
{
    static_assert(std::is_integral<T>::value, "integer atomics only");
    T old = __atomic_load_n(p, __ATOMIC_SEQ_CST);
    while (v > old && !__atomic_compare_exchange_n(p, &old, v, false, __ATOMIC_SEQ_CST, __ATOMIC_SEQ_CST)) {
    }
    return old;
}

// ---------------------------------------------------------------- host API
typedef int hipError_t;
constexpr hipError_t hipSuccess = 0;
enum hipMemcpyKind { hipMemcpyHostToHost, hipMemcpyHostToDevice, hipMemcpyDeviceToHost, hipMemcpyDeviceToDevice };
struct hipDeviceProp_t {
    char name[256] = "host emulation";
    char gcnArchName[256] = "host";
    int multiProcessorCount = 1;
};
typedef struct hipemu_event* hipEvent_t;
typedef struct hipemu_stream* hipStream_t;

inline const char* hipGetErrorString(hipError_t) { return "hip emulation error"; }
inline hipError_t hipGetDeviceProperties(hipDeviceProp_t* p, int) { *p = hipDeviceProp_t{}; return hipSuccess; }
inline hipError_t hipGetDevice(int* d) { *d = 0; return hipSuccess; }
inline hipError_t hipDeviceSynchronize() { return hipSuccess; }
template <typename T>
inline hipError_t hipMalloc(T** p, size_t n)
{
    *p = static_cast<T*>(std::calloc(n ? n : 1, 1));
    return *p ? hipSuccess : 1;
}
inline hipError_t hipFree(void* p) { std::free(p); return hipSuccess; }
inline hipError_t hipMemcpy(void* d, const void* s, size_t n, hipMemcpyKind) { std::memcpy(d, s, n); return hipSuccess; }
inline hipError_t hipMemset(void* d, int v, size_t n) { std::memset(d, v, n); return hipSuccess; }
inline hipError_t hipEventCreate(hipEvent_t* e) { *e = nullptr; return hipSuccess; }
inline hipError_t hipEventDestroy(hipEvent_t) { return hipSuccess; }
inline hipError_t hipEventRecord(hipEvent_t, hipStream_t = nullptr) { return hipSuccess; }
inline hipError_t hipEventSynchronize(hipEvent_t) { return hipSuccess; }
inline hipError_t hipEventElapsedTime(float* ms, hipEvent_t, hipEvent_t) { *ms = 1.f; return hipSuccess; }

namespace hipemu {
template <typename K, typename... A>
void launch(K kernel, dim3 grid, dim3 block, A... args)
{
    struct Ctx {
        K k;
        std::tuple<A...> a;
    } ctx{kernel, std::tuple<A...>(args...)};
    run_grid(grid, block, &ctx, [](void* c) {
        Ctx* x = static_cast<Ctx*>(c);
        std::apply(x->k, x->a);
    });
}
}  // namespace hipemu

#define hipLaunchKernelGGL(kernel, grid, block, shmem, stream, ...) \
    hipemu::launch(kernel, dim3(grid), dim3(block), __VA_ARGS__)
