// Fiber runtime of the CPU stand-in for the HIP device environment — TEST INFRASTRUCTURE ONLY.
//
// A block of T GPU threads runs as T fibers on one OS thread: each fiber runs until it reaches a barrier (block or
// wave), a cross-lane operation or its end, then control returns to the block's scheduler, which releases a barrier
// once every fiber of the block (or wave) that has not finished is waiting at it. Fibers switch with a
// callee-saved-register swap (x86-64 System V). Blocks are spread over a pool of OS threads; __shared__ arrays are
// thread_local, so the fibers of one block see one copy.
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <sys/mman.h>

#include <algorithm>
#include <atomic>
#include <functional>
#include <thread>
#include <vector>

#include "hipemu_core.h"

extern "C" void hipemu_switch(void** save_sp, void* load_sp);
asm(R"(
    .text
    .globl hipemu_switch
    .hidden hipemu_switch
    .type hipemu_switch, @function
hipemu_switch:
    pushq %rbp
    pushq %rbx
    pushq %r12
    pushq %r13
    pushq %r14
    pushq %r15
    movq %rsp, (%rdi)
    movq %rsi, %rsp
    popq %r15
    popq %r14
    popq %r13
    popq %r12
    popq %rbx
    popq %rbp
    ret
    .size hipemu_switch, .-hipemu_switch
)");

namespace hipemu {

enum State { RUNNABLE, WAIT_BLOCK, WAIT_WAVE, DONE };

struct Fiber {
    void* sp;
    Dim3 tid;
    int lane, wave;
    State state;
};

constexpr int MAX_THREADS = 1024;
constexpr size_t STACK_BYTES = 256 * 1024;

thread_local Fiber* current = nullptr;
thread_local Dim3 block_index{0, 0, 0}, block_dim{1, 1, 1}, grid_dim{1, 1, 1};
static thread_local void* sched_sp = nullptr;
static thread_local Fiber fibers[MAX_THREADS];
static thread_local char* stacks = nullptr;
static thread_local const std::function<void()>* body = nullptr;
static thread_local uint64_t exchange_table[MAX_THREADS / 32][32];

const Dim3& thread_index() { return current->tid; }
int lane_of_current() { return current->lane; }
int wave_of_current() { return current->wave; }

static void yield(State s) {
    Fiber* f = current;
    f->state = s;
    hipemu_switch(&f->sp, sched_sp);
}

void block_barrier() { yield(WAIT_BLOCK); }
void wave_barrier() { yield(WAIT_WAVE); }

const uint64_t* wave_exchange(uint64_t mine) {
    exchange_table[current->wave][current->lane] = mine;
    wave_barrier();
    return exchange_table[current->wave];
}

bool any(bool p) {
    const uint64_t* all = wave_exchange(p ? 1 : 0);
    bool r = false;
    const int base = current->wave * 32;
    for (int l = 0; l < 32; ++l) {
        const int t = base + l;
        const int n = (int)(block_dim.x * block_dim.y * block_dim.z);
        if (t < n && fibers[t].state != DONE && all[l]) r = true;
    }
    wave_barrier();
    return r;
}

static void fiber_entry() {
    (*body)();
    Fiber* f = current;
    f->state = DONE;
    hipemu_switch(&f->sp, sched_sp);
    abort();  // a finished fiber is never resumed
}

static void run_block(int n) {
    if (!stacks) {
        void* p = mmap(nullptr, STACK_BYTES * MAX_THREADS, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE,
                       -1, 0);
        if (p == MAP_FAILED) {
            fprintf(stderr, "hipemu: cannot map fiber stacks\n");
            abort();
        }
        stacks = static_cast<char*>(p);
    }
    for (int t = 0; t < n; ++t) {
        Fiber& f = fibers[t];
        f.tid = Dim3{(unsigned)(t % block_dim.x), (unsigned)((t / block_dim.x) % block_dim.y),
                     (unsigned)(t / (block_dim.x * block_dim.y))};
        f.lane = t & 31;
        f.wave = t >> 5;
        f.state = RUNNABLE;
        // Initial frame: six callee-saved registers, then the "return address" fiber_entry; fiber_entry starts with
        // rsp = 8 (mod 16) like any called function.
        uintptr_t top = reinterpret_cast<uintptr_t>(stacks + STACK_BYTES * (size_t)(t + 1)) & ~uintptr_t(15);
        void** sp = reinterpret_cast<void**>(top);
        *--sp = nullptr;                                        // fiber_entry's own return address (never used)
        *--sp = reinterpret_cast<void*>(&fiber_entry);
        for (int r = 0; r < 6; ++r) *--sp = nullptr;
        f.sp = sp;
    }
    int live = n;
    while (live > 0) {
        for (int t = 0; t < n; ++t) {
            if (fibers[t].state != RUNNABLE) continue;
            current = &fibers[t];
            hipemu_switch(&sched_sp, fibers[t].sp);
        }
        current = nullptr;
        live = 0;
        int at_block = 0;
        for (int t = 0; t < n; ++t) {
            if (fibers[t].state != DONE) ++live;
            if (fibers[t].state == WAIT_BLOCK) ++at_block;
        }
        if (live == 0) break;
        bool released = false;
        if (at_block == live) {
            for (int t = 0; t < n; ++t)
                if (fibers[t].state == WAIT_BLOCK) fibers[t].state = RUNNABLE;
            released = true;
        }
        for (int w = 0; w * 32 < n; ++w) {
            int waiting = 0, alive = 0;
            for (int t = w * 32; t < std::min(n, w * 32 + 32); ++t) {
                if (fibers[t].state != DONE) ++alive;
                if (fibers[t].state == WAIT_WAVE) ++waiting;
            }
            if (alive > 0 && waiting == alive) {
                for (int t = w * 32; t < std::min(n, w * 32 + 32); ++t)
                    if (fibers[t].state == WAIT_WAVE) fibers[t].state = RUNNABLE;
                released = true;
            }
        }
        if (!released) {
            fprintf(stderr, "hipemu: block (%u, %u, %u) deadlocked (%d threads waiting, none runnable)\n", block_index.x,
                    block_index.y, block_index.z, live);
            abort();
        }
    }
}

// Runs `kernel` (one call per GPU thread) over the grid.
void launch(Dim3 grid, Dim3 block, const std::function<void()>& kernel) {
    const int n = (int)(block.x * block.y * block.z);
    if (n <= 0 || n > MAX_THREADS) {
        fprintf(stderr, "hipemu: block of %d threads\n", n);
        abort();
    }
    const long blocks = (long)grid.x * grid.y * grid.z;
    std::atomic<long> next{0};
    auto worker = [&]() {
        body = &kernel;
        block_dim = block;
        grid_dim = grid;
        for (long b = next++; b < blocks; b = next++) {
            block_index = Dim3{(unsigned)(b % grid.x), (unsigned)((b / grid.x) % grid.y), (unsigned)(b / ((long)grid.x * grid.y))};
            run_block(n);
        }
    };
    const int threads = (int)std::min<long>(blocks, std::max(1u, std::min(32u, std::thread::hardware_concurrency())));
    std::vector<std::thread> pool;
    for (int i = 1; i < threads; ++i) pool.emplace_back(worker);
    worker();
    for (auto& t : pool) t.join();
}

}  // namespace hipemu

// Dynamic shared memory of the reference kernels (extern __shared__), sized for their largest launches.
thread_local __attribute__((aligned(16))) _Float16 rotated[16384];      // int8_gemm.hip rot_quant: K <= 16384
// g++ calls the TLS init function of `rotated` unconditionally from rot_quant (its extern declaration sits in a
// function template), while a definition without a dynamic initializer provides none: an empty one here.
extern "C" void _ZTH7rotated() {}
thread_local __attribute__((aligned(16))) hipemu::Vec<float, 4> xs[4096];  // int8_gemv.hip gemv_*: K <= 16384
thread_local __attribute__((aligned(16))) float s[65536];                // int8_gemv.hip rotate: group floats
