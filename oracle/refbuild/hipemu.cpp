// hipemu.cpp — the fiber scheduler behind hip_emu/hip/hip_runtime.h (test
// infrastructure: runs the reference's HIP kernels on the CPU).
#include "hip/hip_runtime.h"

#include <ucontext.h>

#include <algorithm>
#include <atomic>
#include <thread>
#include <vector>

namespace hipemu {

thread_local Coords* g_cur = nullptr;

namespace {

constexpr size_t kStackBytes = 64 * 1024;

struct Barrier {
    int arrived = 0;
    unsigned gen = 0;
};

struct Fiber {
    ucontext_t ctx;
    Coords co;
    int tid = 0, wave = 0, lane = 0;
    bool done = false;
    bool waiting = false;
    Barrier* wait_bar = nullptr;
    unsigned wait_gen = 0;
};

struct Block {
    std::vector<Fiber> f;
    std::vector<char> stacks;
    ucontext_t sched;
    Barrier block_bar;
    std::vector<Barrier> wave_bar;
    std::vector<int> wave_size, wave_exited;
    std::vector<uint64_t> xbuf;
    int nthreads = 0, exited = 0, cur = -1;
    void* ctx = nullptr;
    BlockBody body = nullptr;
};

thread_local Block* t_blk = nullptr;

// Releases a barrier whose arrivals plus exited threads cover its scope.
bool try_release(Barrier& b, int scope, int exited)
{
    if (b.arrived > 0 && b.arrived + exited == scope) {
        b.arrived = 0;
        ++b.gen;
        return true;
    }
    return false;
}

void arrive(Barrier& b, int scope, int exited)
{
    Block* B = t_blk;
    Fiber& me = B->f[B->cur];
    ++b.arrived;
    if (try_release(b, scope, exited)) return;
    me.waiting = true;
    me.wait_bar = &b;
    me.wait_gen = b.gen;
    swapcontext(&me.ctx, &B->sched);
}

void fiber_entry()
{
    Block* B = t_blk;
    B->body(B->ctx);
    Fiber& me = B->f[B->cur];
    me.done = true;
    ++B->exited;
    ++B->wave_exited[me.wave];
    try_release(B->block_bar, B->nthreads, B->exited);
    try_release(B->wave_bar[me.wave], B->wave_size[me.wave], B->wave_exited[me.wave]);
    // returns to B->sched through uc_link
}

void run_block(Block& B, dim3 grid, dim3 bdim, uint32_t bid)
{
    const dim3 bi(bid % grid.x, (bid / grid.x) % grid.y, bid / (grid.x * grid.y));
    const int n = B.nthreads;
    B.exited = 0;
    B.block_bar = Barrier{};
    std::fill(B.wave_bar.begin(), B.wave_bar.end(), Barrier{});
    std::fill(B.wave_exited.begin(), B.wave_exited.end(), 0);
    for (int t = 0; t < n; ++t) {
        Fiber& f = B.f[t];
        f = Fiber{};
        f.tid = t;
        f.wave = t / kWave;
        f.lane = t % kWave;
        f.co.thread = dim3(t % bdim.x, (t / bdim.x) % bdim.y, t / (bdim.x * bdim.y));
        f.co.block = bi;
        f.co.block_dim = bdim;
        f.co.grid_dim = grid;
        getcontext(&f.ctx);
        f.ctx.uc_stack.ss_sp = B.stacks.data() + (size_t)t * kStackBytes;
        f.ctx.uc_stack.ss_size = kStackBytes;
        f.ctx.uc_link = &B.sched;
        makecontext(&f.ctx, fiber_entry, 0);
    }
    int done = 0;
    while (done < n) {
        bool progressed = false;
        done = 0;
        for (int t = 0; t < n; ++t) {
            Fiber& f = B.f[t];
            if (f.done) {
                ++done;
                continue;
            }
            if (f.waiting && f.wait_bar->gen == f.wait_gen) continue;
            f.waiting = false;
            B.cur = t;
            g_cur = &f.co;
            swapcontext(&B.sched, &f.ctx);
            progressed = true;
            if (f.done) ++done;
        }
        if (!progressed && done < n) {
            std::fprintf(stderr, "hipemu: barrier deadlock in block %u\n", bid);
            std::abort();
        }
    }
    g_cur = nullptr;
}

}  // namespace

void sync_block()
{
    Block* B = t_blk;
    arrive(B->block_bar, B->nthreads, B->exited);
}

void sync_wave()
{
    Block* B = t_blk;
    const int w = B->f[B->cur].wave;
    arrive(B->wave_bar[w], B->wave_size[w], B->wave_exited[w]);
}

int lane_id() { return t_blk->f[t_blk->cur].lane; }

uint64_t exchange(uint64_t mine, int src)
{
    Block* B = t_blk;
    const Fiber& me = B->f[B->cur];
    const int w = me.wave;
    B->xbuf[me.tid] = mine;
    sync_wave();
    const uint64_t r = (src >= 0 && src < B->wave_size[w]) ? B->xbuf[(size_t)w * kWave + src] : mine;
    sync_wave();
    return r;
}

void run_grid(dim3 grid, dim3 block, void* ctx, BlockBody body)
{
    const uint32_t nblocks = grid.x * grid.y * grid.z;
    const int nthreads = (int)(block.x * block.y * block.z);
    if (nblocks == 0 || nthreads == 0) return;
    unsigned hw = std::thread::hardware_concurrency();
    if (const char* e = std::getenv("HIPEMU_THREADS")) hw = (unsigned)std::atoi(e);
    const unsigned workers = std::max(1u, std::min<unsigned>(hw ? hw : 1, nblocks));
    std::atomic<uint32_t> next{0};
    auto work = [&]() {
        Block B;
        B.nthreads = nthreads;
        B.f.resize(nthreads);
        B.stacks.resize((size_t)nthreads * kStackBytes);
        const int waves = (nthreads + kWave - 1) / kWave;
        B.wave_bar.resize(waves);
        B.wave_exited.resize(waves);
        B.wave_size.resize(waves);
        for (int w = 0; w < waves; ++w) B.wave_size[w] = std::min(kWave, nthreads - w * kWave);
        B.xbuf.resize((size_t)waves * kWave);
        B.ctx = ctx;
        B.body = body;
        t_blk = &B;
        for (uint32_t b; (b = next.fetch_add(1)) < nblocks;) run_block(B, grid, block, b);
        t_blk = nullptr;
    };
    std::vector<std::thread> pool;
    for (unsigned i = 1; i < workers; ++i) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
}

}  // namespace hipemu
