// One token of the int8 text decoder as ONE persistent kernel (b2_decode_step): for every layer, RMSNorm, the q|k|v
// GEMV, q/k RMSNorm + rope + KV-cache write, split-position attention and its merge, the output projection with the
// residual, RMSNorm, the gate|up GEMV with silu(gate) * up, and the down projection with the residual.
//
// The arithmetic is the reference's decode route, stage for stage: gemv_i8 (int8_gemv.hip:55-85: fp32 x, int8 row,
// one scale per output row), attn_decode + attn_merge (int8_gemv.hip:124-195: per split a running max / sum /
// weighted V, merged with exp(m_s - max) weights), and linear_forward / init_kv_cache around them
// (int8_gemv.py:48-64, 117-126). What differs is the schedule and the GEMV's inner arithmetic:
//
//   * One CTA per SM, launched cooperatively (all CTAs resident). One producer thread streams the int8 weight rows
//     the CTA owns, layer after layer, into a ring of four 40 KB shared-memory slots with 1-D bulk copies
//     (cp.async.bulk, L2 evict-first). The rows of a GEMV that a CTA owns are contiguous in memory, so each slot is
//     one copy of whole rows. Weights do not depend on activations, so the stream never waits for a stage boundary:
//     it runs ahead by the ring while the consumers wait at a grid barrier (at most two copies in flight).
//   * Eight consumer warps. Each GEMV input (RMSNorm of the residual stream, the merged attention output, or
//     silu(gate) * up) is formed once per CTA and written as three signed int8 digits per value under one power-of-
//     two scale (x = 2^-q (d0 + d1 2^-7 + d2 2^-14)); every weight word then costs three dp4a (exact int32 sums) and
//     each weight byte is read once from shared memory. The digits keep 20 bits of the input's largest value, the
//     accuracy of fp32 accumulation over a few thousand terms.
//   * Stages are separated by a grid barrier: an arrival counter in global memory (zeroed before each launch),
//     release on arrival, acquire on the poll, every wait bounded.
//   * Attention: CTA c < kv_heads * S takes one (kv head, position split) item for the group of query heads sharing
//     that kv head; the producer brings the split's K rows and V rows into two ring slots while the q|k|v GEMV runs.
//     The CTA normalises and rotates its q heads itself from the q|k|v output; the CTA whose split holds the new
//     position also forms k and v of that position, writes them into the caches and into its slots. The last CTA of
//     a kv head to finish (an arrival counter per kv head) merges the S partial results of its q heads.
//   * gate|up: CTA c owns gate rows [a, b) AND up rows [F + a, F + b), so it forms silu(gate) * up for [a, b)
//     itself; the down projection reads that product as its input.
//
// Every wait (ring slots, grid barrier) gives up after a time limit, records a code in *err and makes the whole
// grid stop at its next wait; the producer drains its copies in flight before the CTA exits. A launch that finds
// *err already set does nothing, so one failed token leaves the flag for the host to read.
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <stdint.h>

#include "common.cuh"
#include "host.hpp"

namespace b2 {
namespace {

constexpr int DS_CWARPS = 16;                  // consumer warps (four warpgroups)
constexpr int DS_CTHREADS = DS_CWARPS * 32;    // consumer threads (named barrier 1)
constexpr int DS_THREADS = DS_CTHREADS + 128;  // + the producer warpgroup (one thread works)
// Register split (setmaxnreg): launched with DS_REGS_LAUNCH per thread, the producer warpgroup gives back down to
// DS_REGS_PRODUCER and the consumers take DS_REGS_CONSUMER: 512 * 104 + 128 * 56 = 60416 <= 640 * 96 = 61440.
constexpr int DS_REGS_LAUNCH = 96, DS_REGS_CONSUMER = 104, DS_REGS_PRODUCER = 56;
static_assert(DS_CTHREADS * DS_REGS_CONSUMER + 128 * DS_REGS_PRODUCER <= DS_THREADS * DS_REGS_LAUNCH, "register split");
constexpr int DS_SLOT = 40960;                 // bytes per ring slot
constexpr int DS_SLOTS = 4;
constexpr int DS_INFLIGHT = 4;                 // bulk copies a producer keeps in flight (the rest of the ring holds
                                               // data that has landed); more would only queue the SM's other loads
constexpr int DS_MAXU = 3;                     // 16-value units of the input a consumer thread holds
constexpr int DS_RPG = 2;                      // rows per row group per slot
static_assert(DS_RPG == 2, "gemv_stage's finishing lanes pick v[0] / v[1]");
constexpr int DS_HD = 128;                     // head dim
constexpr int DS_MAX_SPLITS = 20;
constexpr int DS_MAX_GATE = 1024;              // gate rows one CTA may own
constexpr int DS_MAX_ROWS = 2 * DS_MAX_GATE;   // rows one CTA finishes in one stage
constexpr int DS_MAX_K = 10240;                // widest GEMV input, staged in shared memory
constexpr int DS_DIGITS = 3;                   // signed int8 digits of the GEMV input (base 2^7)
constexpr int DS_MAX_GROUP = 4;                // query heads per kv head
constexpr int DS_LINE = 32;                    // words per 128-byte line: one counter per line
constexpr int DS_SYNC_WORDS = 2048;            // arrival counters (one per line) cleared before each launch
constexpr int DS_O_ROWS = 64;                  // out-projection rows one CTA may own

// Error codes written to *err.
constexpr int DS_ERR_BARRIER = 1;  // a grid barrier ran out of time
constexpr int DS_ERR_FULL = 2;     // a consumer waited too long for a slot
constexpr int DS_ERR_EMPTY = 3;    // the producer waited too long for a free slot
constexpr int DS_ERR_POS = 4;      // position outside the cache

// Layer table: DS_FIELDS device pointers per layer, in this order.
enum {
    F_NORM_IN, F_NORM_POST, F_Q_NORM, F_K_NORM, F_W_QKV, F_S_QKV, F_W_O, F_S_O, F_W_GU, F_S_GU, F_W_DOWN, F_S_DOWN,
    F_K_CACHE, F_V_CACHE, DS_FIELDS
};

struct StepArgs {
    const uint64_t* layers;
    int n_layers;
    float* x;        // [D] residual stream: input of layer 0, output of the last layer
    float* x2;       // [D] residual after attention
    float* qkv;      // [(H + 2 Hk) * 128]
    float* att;      // [H * 128] floats of scratch: the merged attention output as 3 int8 digit planes of H * 128
                     // bytes (kv group g's values at g * GW of each plane) and then one fp32 scale 2^-q per kv head
    float* act;      // [F] silu(gate) * up
    float* partial;  // [H][S][128]
    float* stats;    // [H][S][2]
    const float* inv_freq;  // [64]
    const int64_t* pos;
    const int32_t* lengths;
    unsigned* sync;  // DS_SYNC_WORDS counters, one per 128-byte line (sync_barrier and the ones after it), all
                     // zeroed per launch
    int* err;
    int D, H, Hk, F, cap, S;
    float eps, scale;
    uint64_t timeout_ns;
};

// Where a CTA's rows of one GEMV lie and how the consumers split them.
struct Geo {
    int K, U, kw, rg, upl, rows;  // K bytes per row, U = K / 16 units, kw warps per row, rg row groups, units per
                                  // lane, rows per slot
};

__host__ __device__ inline Geo geometry(int K) {
    Geo g;
    g.K = K;
    g.U = K / 16;
    g.kw = 1;
    while (g.kw < DS_CWARPS && (g.U + 32 * g.kw - 1) / (32 * g.kw) > DS_MAXU) g.kw *= 2;
    g.rg = DS_CWARPS / g.kw;
    g.upl = (g.U + 32 * g.kw - 1) / (32 * g.kw);
    g.rows = g.rg * DS_RPG;
    return g;
}

__host__ __device__ inline int64_t split_lo(int64_t n, int c, int G) { return n * c / G; }

// The GEMVs of a layer: 0 q|k|v, 1 o, 2 gate (rows [a, b)) + up (rows [F + a, F + b)), 3 down.
struct Range {
    const int8_t* w;
    int64_t lo, hi;  // rows
};

__device__ inline int stage_ranges(const StepArgs& a, const uint64_t* L, int st, int c, int G, Range (&r)[3], int& K) {
    switch (st) {
        case 0: {
            const int64_t QKV = (int64_t)(a.H + 2 * a.Hk) * DS_HD;
            K = a.D;
            r[0] = {reinterpret_cast<const int8_t*>(L[F_W_QKV]), split_lo(QKV, c, G), split_lo(QKV, c + 1, G)};
            return 1;
        }
        case 1:
            K = a.H * DS_HD;
            r[0] = {reinterpret_cast<const int8_t*>(L[F_W_O]), split_lo(a.D, c, G), split_lo(a.D, c + 1, G)};
            return 1;
        case 2: {
            K = a.D;
            const int64_t lo = split_lo(a.F, c, G), hi = split_lo(a.F, c + 1, G);
            r[0] = {reinterpret_cast<const int8_t*>(L[F_W_GU]), lo, hi};
            r[1] = {reinterpret_cast<const int8_t*>(L[F_W_GU]), a.F + lo, a.F + hi};
            return 2;
        }
        default:
            K = a.F;
            r[0] = {reinterpret_cast<const int8_t*>(L[F_W_DOWN]), split_lo(a.D, c, G), split_lo(a.D, c + 1, G)};
            return 1;
    }
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(DS_CTHREADS) : "memory"); }

__device__ __forceinline__ void set_err(int* err, int code) { atomicCAS(err, 0, code); }

// The counters, each on its own 128-byte line so that the pollers of one do not slow the others: the grid barrier's
// arrivals; per kv head g its attention splits' arrivals and the flag that its merged output is published.
__device__ __forceinline__ unsigned* sync_barrier(const StepArgs& a) { return a.sync; }
__device__ __forceinline__ unsigned* sync_split(const StepArgs& a, int g) { return a.sync + DS_LINE * (1 + g); }
__device__ __forceinline__ unsigned* sync_published(const StepArgs& a, int g) {
    return a.sync + DS_LINE * (1 + a.Hk + g);
}


__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile_i32(const int* p) {
    int v;
    asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Bounded mbarrier wait that also gives up when another role or CTA has failed.
__device__ __forceinline__ bool ring_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code,
                                          uint64_t timeout_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*abort) return false;
            if (ld_volatile_i32(err)) {
                *abort = 1;
                return false;
            }
            if (global_timer() - start > timeout_ns) {
                set_err(err, code);
                *abort = 1;
                return false;
            }
        }
    }
}


struct AttnScratch {
    float4 acc[DS_CWARPS][DS_MAX_GROUP][32];
    float mx[DS_CWARPS][DS_MAX_GROUP], sum[DS_CWARPS][DS_MAX_GROUP];
    float q[DS_MAX_GROUP][DS_HD];
    float2 split[DS_MAX_GROUP][DS_MAX_SPLITS];  // merge: (max, sum) of each split
    float keep[DS_MAX_GROUP][DS_MAX_SPLITS];    // merge: exp(m_s - max) of each split
    float wkeep[DS_CWARPS][DS_MAX_GROUP];       // warp combine: exp(m_w - max) of each warp
    float top[DS_MAX_GROUP], total[DS_MAX_GROUP];
};

struct Smem {
    alignas(128) uint8_t ring[DS_SLOTS][DS_SLOT];
    uint64_t full[DS_SLOTS], empty[DS_SLOTS];
    float red[2][DS_CWARPS][DS_RPG];  // per-slot row partials of each warp
    float part[DS_CWARPS], pmax[DS_CWARPS];  // block sum / max
    union {
        uint32_t dig[DS_DIGITS][DS_MAX_K / 4];  // a stage's input as digit planes while it is handed out
        AttnScratch attn;                      // attention stage
        float gate[DS_MAX_GATE];               // gate rows of the gate|up stage (the input is in registers by then)
        float opart[DS_O_ROWS][DS_CWARPS];     // out-projection: each row's partial sum per kv group
    } u;
    float row_scale[DS_MAX_ROWS], row_res[DS_MAX_ROWS];  // the stage's per-row scales and residual values
    float rope_c[DS_HD / 2], rope_s[DS_HD / 2];  // cos / sin of the position's rotary angles
    int abort;
    int last;                         // this CTA merges its kv head
    int64_t pos;
    int length;
};

__device__ __forceinline__ Smem& smem_struct() {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    return *reinterpret_cast<Smem*>(smem_raw);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Consumer-wide AND of a predicate; doubles as the consumers' barrier.
__device__ __forceinline__ bool consumer_all(bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred q, d;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "barrier.cta.red.and.pred d, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, d;\n\t}\n"
        : "=r"(r)
        : "r"((uint32_t)p), "n"(DS_CTHREADS)
        : "memory");
    return r != 0;
}

// silu(g) * u in fp32 as torch forms silu(gate) * up: g / (1 + exp(-g)), then the product.
__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
}

// A GEMV row against the staged input: the input x (K fp32 values) is written as x = 2^-q (d0 + d1 2^-7 + d2 2^-14)
// with signed int8 digits d (|d| <= 64; q puts max|x| 2^q in [32, 64)), so that w . x = 2^-q (w . d0 + (w . d1)
// 2^-7 + (w . d2) 2^-14) with each w . d an exact int32 dot product (dp4a: four int8 products per instruction).
// The truncation left after the third digit is below 2^-20 max|x|, the size of fp32 accumulation error over a
// few thousand terms; the int32 sums themselves are exact.
__device__ __forceinline__ void dot_unit(const uint4 w, const uint4 (&x)[DS_DIGITS], int (&acc)[DS_DIGITS]) {
#pragma unroll
    for (int d = 0; d < DS_DIGITS; ++d) {
        acc[d] = __dp4a((int)w.x, (int)x[d].x, acc[d]);
        acc[d] = __dp4a((int)w.y, (int)x[d].y, acc[d]);
        acc[d] = __dp4a((int)w.z, (int)x[d].z, acc[d]);
        acc[d] = __dp4a((int)w.w, (int)x[d].w, acc[d]);
    }
}

__device__ __forceinline__ float combine_digits(const int (&acc)[DS_DIGITS]) {
    return __fadd_rn(__fadd_rn((float)acc[0], __fmul_rn((float)acc[1], 0.0078125f)),
                     __fmul_rn((float)acc[2], 6.103515625e-05f));
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}

// The consumer thread's place in a GEMV: row group, warp within the group, lane index within the group.
struct Lane {
    int grp, kwi, gl;
};
__device__ __forceinline__ Lane lane_of(const Geo& g) {
    const int w = threadIdx.x >> 5;
    return {w / g.kw, w % g.kw, (w % g.kw) * 32 + (int)(threadIdx.x & 31)};
}
__device__ __forceinline__ int unit_of(const Geo& g, const Lane& l, int j) { return l.gl + j * 32 * g.kw; }

// Forms a stage's input vector once per CTA and gives every consumer thread its units as int8 digit words.
// Pass 1: the consumers read v (and w) with coalesced 16-byte loads through L2, all issued before any is used
// (addresses clamped). With w (RMSNorm): y = v * rsqrt(mean(v^2) + eps) * w, the sum of squares accumulated in a
// fixed order and the fp32 products rounded in that order. Every CTA forms the same values in the same order, so
// all hold the same vector and the same digits. Pass 2: max|y| over the CTA, then each thread writes the digits of
// its values into the three planes (one byte per value; rounding to an integer by adding 1.5 * 2^23, ties to even,
// every step exact). Pass 3: each thread reads its units' digit words. Returns 2^-q, or NaN when the input holds a
// NaN or an infinity (every output of the GEMV is then NaN).
constexpr int DS_STAGE_PER_THREAD = DS_MAX_K / 4 / DS_CTHREADS;  // float4 per consumer thread

// xv[i] for a runtime i without sending the array to local memory.
__device__ __forceinline__ float4 sm_pick(const float4 (&xv)[DS_STAGE_PER_THREAD], int i) {
    float4 r = xv[0];
#pragma unroll
    for (int k = 1; k < DS_STAGE_PER_THREAD; ++k)
        if (i == k) r = xv[k];
    return r;
}

__device__ __forceinline__ uint32_t digit_byte_word(float a, float b, float c, float d) {
    const uint32_t lo = __byte_perm(__float_as_uint(a), __float_as_uint(b), 0x0040u);
    const uint32_t hi = __byte_perm(__float_as_uint(c), __float_as_uint(d), 0x0040u);
    return __byte_perm(lo, hi, 0x5410u);
}

// The power of two that puts max|x| = m in [32, 64): up = 2^q multiplies the values before their digits are taken,
// inv = 2^-q undoes it on the dot products; inv is NaN when m is not finite.
__device__ __forceinline__ void digit_scale(float m, float& up, float& inv) {
    int q = 0;
    if (m > 0.f && m <= 3.4e38f) {
        const int e = (int)((__float_as_uint(m) >> 23) & 0xff) - 127;  // floor(log2 m) for normal m
        q = min(max(5 - (e < -126 ? -127 : e), -126), 127);
    }
    up = ldexpf(1.f, q);
    inv = m <= 3.4e38f ? ldexpf(1.f, -q) : __int_as_float(0x7fffffff);
}

__device__ __forceinline__ float stage_input(Smem& sm, const float* v, const float* w, float eps, const Geo& g,
                                             const Lane& l, uint4 (&xd)[DS_MAXU][DS_DIGITS]) {
    const int t = threadIdx.x, n4 = g.K / 4;
    const float4* v4 = reinterpret_cast<const float4*>(v);
    float4 xv[DS_STAGE_PER_THREAD], wv[DS_STAGE_PER_THREAD];
#pragma unroll
    for (int i = 0; i < DS_STAGE_PER_THREAD; ++i) xv[i] = __ldcg(v4 + min(t + i * DS_CTHREADS, n4 - 1));
    if (w) {
        const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
        for (int i = 0; i < DS_STAGE_PER_THREAD; ++i) wv[i] = __ldg(w4 + min(t + i * DS_CTHREADS, n4 - 1));
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < DS_STAGE_PER_THREAD; ++i)
            if (t + i * DS_CTHREADS < n4) {
                ss = fmaf(xv[i].x, xv[i].x, ss);
                ss = fmaf(xv[i].y, xv[i].y, ss);
                ss = fmaf(xv[i].z, xv[i].z, ss);
                ss = fmaf(xv[i].w, xv[i].w, ss);
            }
        ss = warp_sum(ss);
        if ((t & 31) == 0) sm.part[t >> 5] = ss;
        consumer_sync();
        ss = sm.part[0];
#pragma unroll
        for (int i = 1; i < DS_CWARPS; ++i) ss += sm.part[i];
        const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)g.K), eps));
#pragma unroll
        for (int i = 0; i < DS_STAGE_PER_THREAD; ++i)
            xv[i] = make_float4(__fmul_rn(__fmul_rn(xv[i].x, r), wv[i].x), __fmul_rn(__fmul_rn(xv[i].y, r), wv[i].y),
                                __fmul_rn(__fmul_rn(xv[i].z, r), wv[i].z), __fmul_rn(__fmul_rn(xv[i].w, r), wv[i].w));
    }
    // max |y| (an infinity or NaN makes it +inf)
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < DS_STAGE_PER_THREAD; ++i)
        if (t + i * DS_CTHREADS < n4) {
            const float4 q = xv[i];
            const float a = fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w)));
            const bool finite = fabsf(q.x) <= 3.4e38f && fabsf(q.y) <= 3.4e38f && fabsf(q.z) <= 3.4e38f &&
                                fabsf(q.w) <= 3.4e38f;
            m = finite ? fmaxf(m, a) : __int_as_float(0x7f800000);
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((t & 31) == 0) sm.pmax[t >> 5] = m;
    consumer_sync();
    m = sm.pmax[0];
#pragma unroll
    for (int i = 1; i < DS_CWARPS; ++i) m = fmaxf(m, sm.pmax[i]);
    float up, inv;
    digit_scale(m, up, inv);
    const float M = 12582912.f;  // 1.5 * 2^23
    // Rolled loop: this code runs once per stage, and a compact body keeps it in the instruction cache.
#pragma unroll 1
    for (int i = 0; i < DS_STAGE_PER_THREAD; ++i) {
        if (t + i * DS_CTHREADS >= n4) break;
        const float4 q4 = sm_pick(xv, i);
        const float y[4] = {q4.x, q4.y, q4.z, q4.w};
        float tq[DS_DIGITS][4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float r = __fmul_rn(y[e], up);
#pragma unroll
            for (int d = 0; d < DS_DIGITS; ++d) {
                const float tt = __fadd_rn(r, M);
                tq[d][e] = tt;
                r = __fmul_rn(__fsub_rn(r, __fsub_rn(tt, M)), 128.f);
            }
        }
#pragma unroll
        for (int d = 0; d < DS_DIGITS; ++d)
            sm.u.dig[d][t + i * DS_CTHREADS] = digit_byte_word(tq[d][0], tq[d][1], tq[d][2], tq[d][3]);
    }
    consumer_sync();
#pragma unroll
    for (int j = 0; j < DS_MAXU; ++j) {
        const int u = unit_of(g, l, j);
        const bool ok = j < g.upl && u < g.U;
        const int uc = min(u, g.U - 1);
#pragma unroll
        for (int d = 0; d < DS_DIGITS; ++d) {
            const uint4 dw = *reinterpret_cast<const uint4*>(&sm.u.dig[d][uc * 4]);
            xd[j][d] = ok ? dw : make_uint4(0u, 0u, 0u, 0u);
        }
    }
    consumer_sync();  // the planes are free again (the gate rows and the attention scratch share their space)
    return inv;
}

// How a GEMV's output row is finished: y = dot * scale[n], then stored, added to a residual, or (gate|up) kept in
// shared memory for the gate rows and combined as silu(gate) * up for the up rows.
enum { FIN_STORE, FIN_RESIDUAL, FIN_GATE_UP };

struct Fin {
    int kind;
    const float* scale;
    const float* residual;
    float* out;
    int64_t gate_lo;
    int F;
};

// AND of a predicate over the kw warps of row group grp (named barrier 2 + grp); also their barrier.
__device__ __forceinline__ bool group_all(bool p, int grp, int nthreads) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred q, d;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "barrier.cta.red.and.pred d, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, d;\n\t}\n"
        : "=r"(r)
        : "r"((uint32_t)p), "r"(2 + grp), "r"(nthreads)
        : "memory");
    return r != 0;
}

// Consumes this CTA's slots of one GEMV. Each warp takes DS_RPG rows of every slot (rows grp + rr * rg) over its
// K slice; with one warp per row (kw = 1) the warp finishes its rows itself, otherwise the kw warps of a row group
// meet at their own named barrier and the group's first warp adds their partial sums. No CTA-wide barrier inside;
// the consumers agree once at the end. Returns false (on every consumer thread alike) when a wait gave up.
__device__ bool gemv_stage(Smem& sm, const StepArgs& a, const Range (&r)[3], int nr, const Geo& g,
                           const uint4 (&xd)[DS_MAXU][DS_DIGITS], float inv, uint32_t& it, const Fin& f) {
    const Lane l = lane_of(g);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool finisher = l.kwi == 0 && lane < DS_RPG;  // finishes row grp + lane * rg of every slot
    bool ok = true;
    for (int ri = 0; ri < nr && ok; ++ri) {
        for (int64_t n = r[ri].lo; n < r[ri].hi && ok; n += g.rows) {
            const int rows = (int)min((int64_t)g.rows, r[ri].hi - n);
            const int slot = it % DS_SLOTS;
            const uint32_t ph = (it / DS_SLOTS) & 1;
            const int buf = it & 1;
            ++it;
            const int my_row = l.grp + lane * g.rg;
            const bool finishes = finisher && my_row < rows;
            ok = ring_wait(&sm.full[slot], ph, &sm.abort, a.err, DS_ERR_FULL, a.timeout_ns);
            ok = __all_sync(0xffffffffu, ok);
            float v[DS_RPG];
            if (ok) {
                // All of the warp's shared-memory reads first (rows past the slot's last and units past the row's
                // end read clamped addresses: their digits are zero or their result is dropped), then dp4a.
                const uint8_t* base = sm.ring[slot];
                uint4 wv[DS_RPG][DS_MAXU];
#pragma unroll
                for (int rr = 0; rr < DS_RPG; ++rr) {
                    const uint8_t* wr = base + min(l.grp + rr * g.rg, rows - 1) * g.K;
#pragma unroll
                    for (int j = 0; j < DS_MAXU; ++j) wv[rr][j] = lds128(wr + min(unit_of(g, l, j), g.U - 1) * 16);
                }
#pragma unroll
                for (int rr = 0; rr < DS_RPG; ++rr) {
                    int acc[DS_DIGITS] = {};
#pragma unroll
                    for (int j = 0; j < DS_MAXU; ++j) dot_unit(wv[rr][j], xd[j], acc);
                    v[rr] = warp_sum(combine_digits(acc));
                }
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&sm.empty[slot]);
                    if (g.kw > 1) {
#pragma unroll
                        for (int rr = 0; rr < DS_RPG; ++rr) sm.red[buf][w][rr] = v[rr];
                    }
                }
            }
            if (g.kw > 1) ok = group_all(ok, l.grp, g.kw * 32);
            if (!ok || !finishes) continue;
            float sum;
            if (g.kw == 1) {
                sum = lane == 0 ? v[0] : v[1];
            } else {
                sum = sm.red[buf][l.grp * g.kw][lane];
                for (int i = 1; i < g.kw; ++i) sum = __fadd_rn(sum, sm.red[buf][l.grp * g.kw + i][lane]);
            }
            const int64_t row = n + my_row;
            int at = (int)(row - r[ri].lo);  // row of the stage: the ranges' rows in order
            for (int q = 0; q < ri; ++q) at += (int)(r[q].hi - r[q].lo);
            const float y = __fmul_rn(__fmul_rn(sum, inv), sm.row_scale[at]);
            if (f.kind == FIN_STORE) {
                f.out[row] = y;
            } else if (f.kind == FIN_RESIDUAL) {
                f.out[row] = __fadd_rn(sm.row_res[at], y);
            } else if (ri == 0) {
                sm.u.gate[row - f.gate_lo] = y;
            } else {
                const int64_t k = row - f.F;
                f.out[k] = silu_mul(sm.u.gate[k - f.gate_lo], y);
            }
        }
    }
    return consumer_all(ok);
}

// Grid barrier among the consumers of all CTAs: arrival counter in global memory, bounded poll by one thread.
// Returns false (on every consumer thread alike) when it gave up or another CTA failed.
__device__ bool grid_barrier(Smem& sm, const StepArgs& a, unsigned target) {
    consumer_sync();
    if (threadIdx.x == 0) {
        red_release_add(sync_barrier(a), 1u);  // orders the CTA's writes (seen through the barrier above) first
        const uint64_t start = global_timer();
        for (uint32_t i = 0;; ++i) {
            if (ld_acquire_u32(sync_barrier(a)) >= target) break;
            if ((i & 15) == 15) {
                if (ld_volatile_i32(a.err)) {
                    sm.abort = 1;
                    break;
                }
                if (global_timer() - start > a.timeout_ns) {
                    set_err(a.err, DS_ERR_BARRIER);
                    sm.abort = 1;
                    break;
                }
            }
        }
    }
    return consumer_all(*reinterpret_cast<volatile int*>(&sm.abort) == 0);
}

// Bounded wait (one thread) until *flag reaches target; on a timeout or another CTA's failure it raises the CTA's
// abort flag and returns false.
__device__ bool wait_flag(Smem& sm, const StepArgs& a, const unsigned* flag, unsigned target) {
    const uint64_t start = global_timer();
    for (uint32_t i = 0;; ++i) {
        if (ld_acquire_u32(flag) >= target) return true;
        if ((i & 15) == 15) {
            if (*reinterpret_cast<volatile int*>(&sm.abort)) return false;
            if (ld_volatile_i32(a.err)) {
                sm.abort = 1;
                return false;
            }
            if (global_timer() - start > a.timeout_ns) {
                set_err(a.err, DS_ERR_BARRIER);
                sm.abort = 1;
                return false;
            }
        }
    }
}

__device__ __forceinline__ const float* scale_of(const uint64_t* L, int st) {
    return reinterpret_cast<const float*>(L[st == 0 ? F_S_QKV : st == 1 ? F_S_O : st == 2 ? F_S_GU : F_S_DOWN]);
}

// The attention of one layer. CTA c < Hk * S takes kv head g = c / S and positions [s0, s1) of split s = c % S.
// Warps 0..GROUP-1 normalise and rotate the group's q heads (decode_qk_rope's arithmetic: RMSNorm over the head,
// then the half-split rotary embedding at position p); if the split holds p, warp GROUP does the same for k and
// writes it into the cache, warp GROUP+1 copies v. Then each warp runs attn_decode's online softmax over every
// eighth position of the split, the warps combine, and the split's partial result and (max, sum) are stored. The
// CTA that completes kv head g's arrivals merges the S splits of its q heads as attn_merge does.
template <int GROUP>
__device__ __noinline__ bool attn_stage(Smem& sm, const StepArgs& a, const uint64_t* L, int layer, uint32_t* it_io) {
    const int c = blockIdx.x, t = threadIdx.x, w = t >> 5, lane = t & 31;
    if (c >= a.Hk * a.S) return true;
    AttnScratch& as = sm.u.attn;
    // The split's K rows and V rows arrive in the next two ring slots (row j - s0 at (j - s0) * 512 bytes).
    const uint32_t it_k = *it_io, it_v = it_k + 1;
    *it_io = it_k + 2;
    const int slot_k = it_k % DS_SLOTS, slot_v = it_v % DS_SLOTS;
    const int g = c / a.S, s = c % a.S;
    const int64_t p = sm.pos;
    const int length = sm.length;
    const int chunk = (length + a.S - 1) / a.S;
    const int s0 = min(s * chunk, length), s1 = min(s0 + chunk, length);
    const bool holds = p >= s0 && p < s1;
    float* kc = reinterpret_cast<float*>(L[F_K_CACHE]);
    float* vc = reinterpret_cast<float*>(L[F_V_CACHE]);
    float4 fresh = make_float4(0.f, 0.f, 0.f, 0.f);  // warp GROUP: k of position p; warp GROUP + 1: its v
    if (w < GROUP || (holds && w < GROUP + 2)) {
        const bool is_v = w == GROUP + 1;
        const int head = w < GROUP ? g * GROUP + w : (is_v ? a.H + a.Hk + g : a.H + g);
        const float* nw = reinterpret_cast<const float*>(L[w < GROUP ? F_Q_NORM : F_K_NORM]);
        const float4 nv = __ldg(reinterpret_cast<const float4*>(nw) + lane);
        const float4 xv = __ldcg(reinterpret_cast<const float4*>(a.qkv + (int64_t)head * DS_HD) + lane);
        if (is_v) {
            fresh = xv;
        } else {
            float ss = __fadd_rn(__fadd_rn(__fmul_rn(xv.x, xv.x), __fmul_rn(xv.y, xv.y)),
                                 __fadd_rn(__fmul_rn(xv.z, xv.z), __fmul_rn(xv.w, xv.w)));
            ss = warp_sum(ss);
            const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)DS_HD), a.eps));
            const float y[4] = {__fmul_rn(__fmul_rn(xv.x, r), nv.x), __fmul_rn(__fmul_rn(xv.y, r), nv.y),
                                __fmul_rn(__fmul_rn(xv.z, r), nv.z), __fmul_rn(__fmul_rn(xv.w, r), nv.w)};
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float other = __shfl_xor_sync(0xffffffffu, y[e], 16);  // the value 64 places away
                const int i = (4 * lane + e) & 63;
                const float cs = sm.rope_c[i], sn = sm.rope_s[i];
                o[e] = lane < 16 ? __fsub_rn(__fmul_rn(y[e], cs), __fmul_rn(other, sn))
                                 : __fadd_rn(__fmul_rn(other, sn), __fmul_rn(y[e], cs));
            }
            if (w < GROUP)
                reinterpret_cast<float4*>(as.q[w])[lane] = make_float4(o[0], o[1], o[2], o[3]);
            else
                fresh = make_float4(o[0], o[1], o[2], o[3]);
        }
    }
    bool ok = ring_wait(&sm.full[slot_k], (it_k / DS_SLOTS) & 1, &sm.abort, a.err, DS_ERR_FULL, a.timeout_ns);
    ok = ok && ring_wait(&sm.full[slot_v], (it_v / DS_SLOTS) & 1, &sm.abort, a.err, DS_ERR_FULL, a.timeout_ns);
    if (!consumer_all(ok)) return false;
    // Position p: the slots hold the cache's old row; the fresh k and v replace it there and in the caches.
    if (holds && (w == GROUP || w == GROUP + 1)) {
        float* cache = w == GROUP ? kc : vc;
        reinterpret_cast<float4*>(cache + (p * a.Hk + g) * DS_HD)[lane] = fresh;
        reinterpret_cast<float4*>(sm.ring[w == GROUP ? slot_k : slot_v] + (p - s0) * DS_HD * 4)[lane] = fresh;
        fence_proxy_async_smem();  // before the slot is handed back to the bulk copies
    }
    consumer_sync();

    float4 qv[GROUP], acc[GROUP];
    float mx[GROUP], sum[GROUP];
#pragma unroll
    for (int gi = 0; gi < GROUP; ++gi) {
        const float4 q = reinterpret_cast<const float4*>(as.q[gi])[lane];
        qv[gi] = make_float4(q.x * a.scale, q.y * a.scale, q.z * a.scale, q.w * a.scale);
        acc[gi] = make_float4(0.f, 0.f, 0.f, 0.f);
        mx[gi] = -1e30f;
        sum[gi] = 0.f;
    }
    const float4* ks = reinterpret_cast<const float4*>(sm.ring[slot_k]);
    const float4* vs = reinterpret_cast<const float4*>(sm.ring[slot_v]);
#pragma unroll 1
    for (int r = w; r < s1 - s0; r += DS_CWARPS) {
        {
            const float4 kv = ks[r * 32 + lane], vv = vs[r * 32 + lane];
#pragma unroll
            for (int gi = 0; gi < GROUP; ++gi) {
                float d = qv[gi].x * kv.x + qv[gi].y * kv.y + qv[gi].z * kv.z + qv[gi].w * kv.w;
                d = warp_sum(d);
                const float next = fmaxf(mx[gi], d);
                const float keep = expf(mx[gi] - next), pr = expf(d - next);
                sum[gi] = sum[gi] * keep + pr;
                acc[gi].x = acc[gi].x * keep + vv.x * pr;
                acc[gi].y = acc[gi].y * keep + vv.y * pr;
                acc[gi].z = acc[gi].z * keep + vv.z * pr;
                acc[gi].w = acc[gi].w * keep + vv.w * pr;
                mx[gi] = next;
            }
        }
    }
    __syncwarp();
    if (lane == 0) {
        mbar_arrive(&sm.empty[slot_k]);
        mbar_arrive(&sm.empty[slot_v]);
    }
#pragma unroll
    for (int gi = 0; gi < GROUP; ++gi) {
        as.acc[w][gi][lane] = acc[gi];
        if (lane == 0) {
            as.mx[w][gi] = mx[gi];
            as.sum[w][gi] = sum[gi];
        }
    }
    consumer_sync();
    // The warps' weights exp(m_w - max) per head, once each; then every output value from them.
    if (t < DS_CWARPS * GROUP) {
        const int ww = t / GROUP, gi = t % GROUP;
        float top = as.mx[0][gi];
        for (int k = 1; k < DS_CWARPS; ++k) top = fmaxf(top, as.mx[k][gi]);
        as.wkeep[ww][gi] = expf(as.mx[ww][gi] - top);
        if (ww == 0) as.top[gi] = top;
    }
    consumer_sync();
    for (int i = t; i < GROUP * DS_HD; i += DS_CTHREADS) {
        const int gi = i / DS_HD, d = i % DS_HD;
        const float top = as.top[gi];
        float value = 0.f, total = 0.f;
#pragma unroll
        for (int ww = 0; ww < DS_CWARPS; ++ww) {
            const float keep = as.wkeep[ww][gi];
            value += reinterpret_cast<const float*>(&as.acc[ww][gi][0])[d] * keep;
            total += as.sum[ww][gi] * keep;
        }
        const int64_t at = (int64_t)(g * GROUP + gi) * a.S + s;
        a.partial[at * DS_HD + d] = value;
        if (d == 0) {
            a.stats[at * 2] = top;
            a.stats[at * 2 + 1] = total;
        }
    }
    consumer_sync();
    if (t == 0) {
        // acq_rel: releases this CTA's partial result (ordered before by the barrier above) and, for the last
        // arrival, acquires every other split's.
        unsigned old;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(sync_split(a, g)) : "memory");
        sm.last = old == (unsigned)((layer + 1) * a.S - 1);
    }
    consumer_sync();
    if (!*reinterpret_cast<volatile int*>(&sm.last)) return true;
    // The (max, sum) pairs of the group's heads into shared memory and every partial value this thread merges, all
    // loads in one round trip; then the weights exp(m_s - max), the sums and the division as attn_merge forms them,
    // in split order.
    constexpr int OUTS = (DS_MAX_GROUP * DS_HD + DS_CTHREADS - 1) / DS_CTHREADS;
    if (t < GROUP * a.S)
        as.split[t / a.S][t % a.S] =
            __ldcg(reinterpret_cast<const float2*>(a.stats) + (int64_t)(g * GROUP + t / a.S) * a.S + t % a.S);
    float pv[OUTS][DS_MAX_SPLITS];
#pragma unroll
    for (int o = 0; o < OUTS; ++o) {
        const int i = min(t + o * DS_CTHREADS, GROUP * DS_HD - 1);
        const int64_t head = g * GROUP + i / DS_HD;
#pragma unroll
        for (int k = 0; k < DS_MAX_SPLITS; ++k)
            pv[o][k] = __ldcg(a.partial + (head * a.S + min(k, a.S - 1)) * DS_HD + i % DS_HD);
    }
    consumer_sync();
    if (t < GROUP) {
        float top = as.split[t][0].x;
        for (int k = 1; k < a.S; ++k) top = fmaxf(top, as.split[t][k].x);
        float total = 0.f;
        for (int k = 0; k < a.S; ++k) {
            const float keep = expf(as.split[t][k].x - top);
            as.keep[t][k] = keep;
            total += as.split[t][k].y * keep;
        }
        as.total[t] = total;
    }
    consumer_sync();
    static_assert(OUTS == 1, "one merged value per consumer thread");
    const bool mine = t < GROUP * DS_HD;
    float v = 0.f;
    if (mine) {
        const int gi = t / DS_HD;
        float value = 0.f;
#pragma unroll
        for (int k = 0; k < DS_MAX_SPLITS; ++k)
            if (k < a.S) value += pv[0][k] * as.keep[gi][k];
        v = value / as.total[gi];
    }
    // The kv head's merged values go out as the out-projection's input: three int8 digit planes under one power of
    // two (as stage_input forms them), then the flag that kv head g's output is published for this layer.
    float m = mine ? (fabsf(v) <= 3.4e38f ? fabsf(v) : __int_as_float(0x7f800000)) : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) sm.pmax[w] = m;
    consumer_sync();
    m = sm.pmax[0];
#pragma unroll
    for (int i = 1; i < DS_CWARPS; ++i) m = fmaxf(m, sm.pmax[i]);
    float up, inv;
    digit_scale(m, up, inv);
    const int GW = GROUP * DS_HD;
    uint8_t* planes = reinterpret_cast<uint8_t*>(a.att);
    float r = __fmul_rn(v, up);
#pragma unroll
    for (int d = 0; d < DS_DIGITS; ++d) {
        const float M = 12582912.f;  // 1.5 * 2^23
        const float tt = __fadd_rn(r, M);
        r = __fmul_rn(__fsub_rn(r, __fsub_rn(tt, M)), 128.f);
        const uint32_t b0 = __float_as_uint(tt) & 0xffu;
        const uint32_t b1 = __shfl_down_sync(0xffffffffu, b0, 1), b2 = __shfl_down_sync(0xffffffffu, b0, 2),
                       b3 = __shfl_down_sync(0xffffffffu, b0, 3);
        if (mine && (t & 3) == 0)
            *reinterpret_cast<uint32_t*>(planes + (int64_t)d * a.H * DS_HD + g * GW + t) =
                b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
    if (t == 0) reinterpret_cast<float*>(planes + (int64_t)DS_DIGITS * a.H * DS_HD)[g] = inv;
    consumer_sync();
    if (t == 0) red_release_add(sync_published(a, g), 1u);
    return true;
}


// The out-projection with its residual, x2 = x + W_o . att, taken kv head by kv head without a grid barrier after
// the attention: warp w works on kv head g = w % Hk (its K slice of GROUP * 128 columns) and on every (16 / Hk)-th
// row of each slot; it waits only for that kv head's merged output (the merging CTA's flag) and reads it as the
// digit planes the merge published. Each (row, kv head) partial sum lands in shared memory; after the slots, the
// CTA adds them up per row in kv-head order and finishes x2 = x + s_o * sum. The weight slots are the same as for
// a whole-row GEMV (rows of H * 128 bytes).
__device__ __noinline__ bool o_stage(const StepArgs& a, const uint64_t* L, int layer, uint32_t* it_io) {
    Smem& sm = smem_struct();
    Range r[3];
    int K;
    stage_ranges(a, L, 1, blockIdx.x, gridDim.x, r, K);
    const Geo geo = geometry(K);
    const int64_t n0 = r[0].lo;
    const int nrows = (int)(r[0].hi - r[0].lo);
    const int t = threadIdx.x, w = t >> 5, lane = t & 31;
    const float* s_o = scale_of(L, 1);
    for (int i = t; i < nrows; i += DS_CTHREADS) {
        sm.row_scale[i] = __ldg(s_o + n0 + i);
        sm.row_res[i] = __ldcg(a.x + n0 + i);
    }
    const int GW = (a.H / a.Hk) * DS_HD, units = GW / 16, per = DS_CWARPS / a.Hk;
    const int grp = w % a.Hk, part = w / a.Hk;
    const uint8_t* planes = reinterpret_cast<const uint8_t*>(a.att);
    bool ok = true;
    if (lane == 0) ok = wait_flag(sm, a, sync_published(a, grp), (unsigned)layer + 1);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();  // the flag's acquire (lane 0) orders the whole warp's reads of the planes
    uint4 xd[DS_DIGITS];
    float inv = 0.f;
    {
        const int uc = min(lane, units - 1);
#pragma unroll
        for (int d = 0; d < DS_DIGITS; ++d) {
            const uint4 dw = __ldcg(reinterpret_cast<const uint4*>(planes + (int64_t)d * a.H * DS_HD + grp * GW) + uc);
            xd[d] = (ok && lane < units) ? dw : make_uint4(0u, 0u, 0u, 0u);
        }
        inv = __ldcg(reinterpret_cast<const float*>(planes + (int64_t)DS_DIGITS * a.H * DS_HD) + grp);
    }
    uint32_t it = *it_io;
    for (int64_t n = n0; n < n0 + nrows && ok; n += geo.rows) {
        const int rows = (int)min((int64_t)geo.rows, n0 + nrows - n);
        const int slot = it % DS_SLOTS;
        const uint32_t ph = (it / DS_SLOTS) & 1;
        ++it;
        ok = ring_wait(&sm.full[slot], ph, &sm.abort, a.err, DS_ERR_FULL, a.timeout_ns);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        const uint8_t* base = sm.ring[slot] + grp * GW + min(lane, units - 1) * 16;
        for (int rr = part; rr < rows; rr += per) {
            int acc[DS_DIGITS] = {};
            dot_unit(lds128(base + rr * K), xd, acc);
            const float y = __fmul_rn(warp_sum(combine_digits(acc)), inv);
            if (lane == 0) sm.u.opart[(int)(n - n0) + rr][grp] = y;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);
    }
    *it_io = it;
    if (!consumer_all(ok)) return false;
    for (int i = t; i < nrows; i += DS_CTHREADS) {
        float sum = sm.u.opart[i][0];
        for (int gg = 1; gg < a.Hk; ++gg) sum = __fadd_rn(sum, sm.u.opart[i][gg]);
        a.x2[n0 + i] = __fadd_rn(sm.row_res[i], __fmul_rn(sum, sm.row_scale[i]));
    }
    return true;
}


// Before the producer issues slot `it`: slot it - DS_INFLIGHT has landed. At about 45 GB/s per SM and a microsecond
// of latency, two 40 KB copies in flight keep the SM's share of HBM busy; every further byte in flight would only
// sit in the SM's response queue ahead of the consumers' own loads, barriers and atomics.
__device__ __forceinline__ bool throttle(Smem& sm, const StepArgs& a, uint32_t it) {
    if (it < (uint32_t)DS_INFLIGHT) return true;
    const uint32_t j = it - DS_INFLIGHT;
    return ring_wait(&sm.full[j % DS_SLOTS], (j / DS_SLOTS) & 1, &sm.abort, a.err, DS_ERR_EMPTY, a.timeout_ns);
}

// The producer's view of a layer: part 0 the q|k|v rows, 1 the attention item's K and V rows, 2 the o rows, 3 the
// gate|up rows, 4 the down rows (GEMV stages 0, 1, 2, 3 for parts 0, 2, 3, 4).
constexpr int DS_PARTS = 5;
// Parts requested into L2 ahead of the part being copied into the ring. The ring holds 160 KB per SM, a few
// microseconds of the SM's share of HBM, while attention, barriers and stage-ins leave the GEMV slots idle for about
// twenty; requesting the rows two parts ahead (at most about 85 MB, within the 126 MB L2) keeps HBM streaming through
// those gaps, and the ring then fills from L2.
constexpr int DS_L2_AHEAD = 2;

__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint64_t bytes) {
    const char* b = reinterpret_cast<const char*>(p);
    for (uint64_t o = 0; o < bytes; o += (1u << 30)) {  // pieces below 2^32 bytes
        const uint32_t n = (uint32_t)min(bytes - o, (uint64_t)1 << 30);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b + o), "r"(n) : "memory");
    }
}

__device__ void l2_request(const StepArgs& a, int q, bool has_item, int g, int s0, int s1) {
    const int l = q / DS_PARTS, part = q % DS_PARTS, c = blockIdx.x, G = gridDim.x;
    if (l >= a.n_layers) return;
    const uint64_t* L = a.layers + (int64_t)l * DS_FIELDS;
    if (part == 1) {
        if (!has_item) return;
        for (int kvs = 0; kvs < 2; ++kvs) {
            const float* cache = reinterpret_cast<const float*>(L[kvs == 0 ? F_K_CACHE : F_V_CACHE]);
            for (int j = s0; j < s1; ++j) prefetch_l2_bulk(cache + ((int64_t)j * a.Hk + g) * DS_HD, DS_HD * 4);
        }
        return;
    }
    const int st = part == 0 ? 0 : part - 1;
    Range r[3];
    int K;
    const int nr = stage_ranges(a, L, st, c, G, r, K);
    const float* sc = scale_of(L, st);
    for (int ri = 0; ri < nr; ++ri) {
        if (r[ri].hi > r[ri].lo) prefetch_l2_bulk(r[ri].w + r[ri].lo * K, (uint64_t)(r[ri].hi - r[ri].lo) * K);
        const char* b = reinterpret_cast<const char*>(sc + r[ri].lo);
        const int64_t bytes = (r[ri].hi - r[ri].lo) * 4;
        for (int64_t o = 0; o < bytes; o += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(b + o));
    }
    if (part == 0) {
        // The layer's norm weights (read by every CTA): this CTA asks for every G-th 128-byte line.
        for (int f = F_NORM_IN; f <= F_K_NORM; ++f) {
            const char* b = reinterpret_cast<const char*>(L[f]);
            const int64_t bytes = (f <= F_NORM_POST ? a.D : DS_HD) * 4;
            for (int64_t o = (int64_t)c * 128; o < bytes; o += (int64_t)G * 128)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(b + o));
        }
    }
}

// One lane of the producer warpgroup: every slot of every stage of every layer, in the consumers' order.
__device__ void producer(Smem& sm, const StepArgs& a) {
    const int c = blockIdx.x, G = gridDim.x;
    const uint64_t policy = l2_policy_evict_first();
    uint32_t it = 0;
    bool ok = true;
    const bool has_item = c < a.Hk * a.S;
    const int g = has_item ? c / a.S : 0, s = has_item ? c % a.S : 0;
    const int chunk = (sm.length + a.S - 1) / a.S;
    const int s0 = min(s * chunk, sm.length), s1 = min(s0 + chunk, sm.length);
    for (int q = 0; q < DS_L2_AHEAD; ++q) l2_request(a, q, has_item, g, s0, s1);
    for (int l = 0; l < a.n_layers && ok; ++l) {
        const uint64_t* L = a.layers + (int64_t)l * DS_FIELDS;
        for (int part = 0; part < DS_PARTS && ok; ++part) {
            l2_request(a, l * DS_PARTS + part + DS_L2_AHEAD, has_item, g, s0, s1);
            if (part == 1) {
                if (!has_item) continue;
                // The attention item's K rows, then its V rows, one slot each.
                for (int kvs = 0; kvs < 2 && ok; ++kvs) {
                    const float* cache = reinterpret_cast<const float*>(L[kvs == 0 ? F_K_CACHE : F_V_CACHE]);
                    const int slot = it % DS_SLOTS;
                    const uint32_t ph = (it / DS_SLOTS) & 1;
                    if (!ring_wait(&sm.empty[slot], ph ^ 1, &sm.abort, a.err, DS_ERR_EMPTY, a.timeout_ns) ||
                        !throttle(sm, a, it)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&sm.full[slot], (uint32_t)(s1 - s0) * DS_HD * 4);
                    for (int j = s0; j < s1; ++j)
                        bulk_g2s(sm.ring[slot] + (j - s0) * DS_HD * 4, cache + ((int64_t)j * a.Hk + g) * DS_HD,
                                 DS_HD * 4, &sm.full[slot], policy);
                    ++it;
                }
                continue;
            }
            Range r[3];
            int K;
            const int nr = stage_ranges(a, L, part == 0 ? 0 : part - 1, c, G, r, K);
            const Geo geo = geometry(K);
            for (int ri = 0; ri < nr && ok; ++ri) {
                for (int64_t n = r[ri].lo; n < r[ri].hi; n += geo.rows) {
                    const uint32_t rows = (uint32_t)min((int64_t)geo.rows, r[ri].hi - n);
                    const int slot = it % DS_SLOTS;
                    const uint32_t ph = (it / DS_SLOTS) & 1;
                    if (!ring_wait(&sm.empty[slot], ph ^ 1, &sm.abort, a.err, DS_ERR_EMPTY, a.timeout_ns) ||
                        !throttle(sm, a, it)) {
                        ok = false;
                        break;
                    }
                    const uint32_t bytes = rows * (uint32_t)K;
                    mbar_arrive_expect_tx(&sm.full[slot], bytes);
                    bulk_g2s(sm.ring[slot], r[ri].w + n * K, bytes, &sm.full[slot], policy);
                    ++it;
                }
            }
        }
    }
    // Copies still in flight land before the CTA's shared memory goes away.
    for (int sl = 0; sl < DS_SLOTS; ++sl) {
        if (it <= (uint32_t)sl) break;
        const uint32_t last = sl + DS_SLOTS * ((it - 1 - sl) / DS_SLOTS);
        mbar_wait_drain(&sm.full[sl], (last / DS_SLOTS) & 1, 100000000ull);
    }
}

// One GEMV stage of a layer (0 q|k|v, 2 gate|up, 3 down; the o rows are o_stage's): its input formed, then the CTA's rows. One copy of
// this code serves all four stages (it is not inlined), which keeps the kernel's instruction footprint small: the
// code outside the slot loop runs once per stage and is fetched again each time.
__device__ __noinline__ bool layer_gemv(const StepArgs& a, const uint64_t* L, int st, uint32_t* it_io) {
    Smem& sm = smem_struct();
    Range r[3];
    int K;
    const int nr = stage_ranges(a, L, st, blockIdx.x, gridDim.x, r, K);
    const Geo g = geometry(K);
    const float* src = st == 0 ? a.x : st == 2 ? a.x2 : a.act;
    const float* nw = reinterpret_cast<const float*>(st == 0 ? L[F_NORM_IN] : st == 2 ? L[F_NORM_POST] : 0);
    Fin f;
    f.scale = scale_of(L, st);
    f.gate_lo = r[0].lo;
    f.F = a.F;
    f.residual = st == 1 ? a.x : st == 3 ? a.x2 : nullptr;
    // The scales (and residual values) of every row the CTA finishes in this stage, into shared memory, in the same
    // round trip as the stage's input; stage_input's barriers publish them.
    for (int ri = 0, at0 = 0; ri < nr; at0 += (int)(r[ri].hi - r[ri].lo), ++ri)
        for (int i = threadIdx.x; i < (int)(r[ri].hi - r[ri].lo); i += DS_CTHREADS) {
            sm.row_scale[at0 + i] = __ldg(f.scale + r[ri].lo + i);
            if (f.residual) sm.row_res[at0 + i] = __ldcg(f.residual + r[ri].lo + i);
        }
    if (nr == 0) return true;  // no rows here (fewer rows than SMs)
    uint4 xd[DS_MAXU][DS_DIGITS];
    const float inv = stage_input(sm, src, nw, a.eps, g, lane_of(g), xd);
    f.kind = st == 0 ? FIN_STORE : st == 2 ? FIN_GATE_UP : FIN_RESIDUAL;
    f.out = st == 0 ? a.qkv : st == 1 ? a.x2 : st == 2 ? a.act : a.x;
    uint32_t it = *it_io;
    const bool ok = gemv_stage(sm, a, r, nr, g, xd, inv, it, f);
    *it_io = it;
    return ok;
}

template <int GROUP>
__device__ void consumers(Smem& sm, const StepArgs& a) {
    const int G = gridDim.x;
    // The rotary angles of this token's position (the same in every layer): fp32(p * inv_freq[i]).
    if (threadIdx.x < DS_HD / 2) {
        const float ang = __fmul_rn((float)sm.pos, __ldg(a.inv_freq + threadIdx.x));
        sm.rope_c[threadIdx.x] = cosf(ang);
        sm.rope_s[threadIdx.x] = sinf(ang);
    }
    consumer_sync();
    uint32_t it = 0;
    unsigned nb = 0;
    for (int l = 0; l < a.n_layers; ++l) {
        const uint64_t* L = a.layers + (int64_t)l * DS_FIELDS;
        // q|k|v = W_qkv . rms(x) * norm_in
        if (!layer_gemv(a, L, 0, &it) || !grid_barrier(sm, a, ++nb * G)) return;
        // attention -> att
        if (!attn_stage<GROUP>(sm, a, L, l, &it)) return;
        // x2 = x + W_o . att, kv head by kv head as their merged outputs appear (no grid barrier before it)
        if (!o_stage(a, L, l, &it) || !grid_barrier(sm, a, ++nb * G)) return;
        // act = silu(gate) * up of W_gu . rms(x2) * norm_post
        if (!layer_gemv(a, L, 2, &it) || !grid_barrier(sm, a, ++nb * G)) return;
        // x = x2 + W_down . act
        if (!layer_gemv(a, L, 3, &it)) return;
        if (l + 1 < a.n_layers && !grid_barrier(sm, a, ++nb * G)) return;
    }
}

template <int GROUP>
__global__ void __launch_bounds__(DS_THREADS, 1) decode_step_kernel(const __grid_constant__ StepArgs a) {
    Smem& sm = smem_struct();
    const int t = threadIdx.x;
    // Every table entry present and 16-byte aligned (bulk copies and float4 loads need it).
    bool bad = false;
    for (int i = t; i < a.n_layers * DS_FIELDS; i += DS_THREADS) {
        const uint64_t v = a.layers[i];
        bad |= v == 0 || (v & 15) != 0;
    }
    bad = __syncthreads_or(bad);
    if (t == 0) {
        int dead = ld_volatile_i32(a.err);
        const int64_t p = a.pos[0];
        const int len = min(a.lengths[0], a.cap);
        if (!dead && (bad || p < 0 || p >= a.cap || len < 1)) {
            set_err(a.err, DS_ERR_POS);
            dead = 1;
        }
        sm.abort = dead;
        sm.pos = p;
        sm.length = len;
        sm.last = 0;
        for (int s = 0; s < DS_SLOTS; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], DS_CWARPS);
        }
        fence_mbar_init();
    }
    __syncthreads();
    const bool dead = sm.abort != 0;
    __syncthreads();  // nothing writes abort before every thread has read it
    if (dead) return;
    if (t >= DS_CTHREADS) {
        regs_dec<DS_REGS_PRODUCER>();
        if (t == DS_CTHREADS) producer(sm, a);
        return;
    }
    regs_inc<DS_REGS_CONSUMER>();
    consumers<GROUP>(sm, a);
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" int b2_decode_step(const uint64_t* layers, int n_layers, float* x, float* x2, float* qkv, float* att,
                              float* act, float* partial, float* stats, const float* inv_freq, const int64_t* pos,
                              const int32_t* lengths, unsigned int* sync, int* err, int hidden, int heads,
                              int kv_heads, int mlp, int capacity, float eps, long long timeout_ns, void* stream) {
    if (!layers || n_layers <= 0 || !x || !x2 || !qkv || !att || !act || !partial || !stats || !inv_freq || !pos ||
        !lengths || !sync || !err || hidden <= 0 || heads <= 0 || kv_heads <= 0 || mlp <= 0 || capacity <= 0 ||
        timeout_ns <= 0)
        return fail(B2_ERR_INVALID, "decode_step: bad arguments");
    if (heads % kv_heads) return fail(B2_ERR_INVALID, "decode_step: heads %d not a multiple of kv_heads %d", heads, kv_heads);
    if (kv_heads > DS_CWARPS || DS_CWARPS % kv_heads)
        return fail(B2_ERR_UNSUPPORTED, "decode_step: %d kv heads (1, 2, 4, 8 or 16)", kv_heads);
    const int group = heads / kv_heads;
    if (group != 1 && group != 2 && group != 4)
        return fail(B2_ERR_UNSUPPORTED, "decode_step: %d query heads per kv head (1, 2 or 4)", group);
    if (DS_LINE * (1 + 2 * kv_heads) > DS_SYNC_WORDS) return fail(B2_ERR_UNSUPPORTED, "decode_step: too many kv heads");
    const int Ks[3] = {hidden, heads * DS_HD, mlp};
    for (int K : Ks) {
        if (K % 16) return fail(B2_ERR_UNSUPPORTED, "decode_step: GEMV width %d is not a multiple of 16", K);
        if (K > DS_MAX_K || geometry(K).upl > DS_MAXU)
            return fail(B2_ERR_UNSUPPORTED, "decode_step: GEMV width %d above %d", K, DS_MAX_K);
    }
    for (const void* p : {(const void*)x, (const void*)x2, (const void*)qkv, (const void*)att, (const void*)act,
                          (const void*)partial})
        if (!aligned16(p)) return fail(B2_ERR_UNSUPPORTED, "decode_step: activation buffers must be 16-byte aligned");
    const int G = sm_count();
    const int S = std::min(DS_MAX_SPLITS, G / kv_heads);
    if (S < 1) return fail(B2_ERR_UNSUPPORTED, "decode_step: %d kv heads on %d SMs", kv_heads, G);
    if ((mlp + G - 1) / G > DS_MAX_GATE) return fail(B2_ERR_UNSUPPORTED, "decode_step: MLP width %d too large", mlp);
    if ((hidden + G - 1) / G > DS_O_ROWS)
        return fail(B2_ERR_UNSUPPORTED, "decode_step: hidden %d gives more than %d output rows per SM", hidden, DS_O_ROWS);
    if (((heads + 2 * kv_heads) * DS_HD + G - 1) / G > DS_MAX_ROWS || (hidden + G - 1) / G > DS_MAX_ROWS)
        return fail(B2_ERR_UNSUPPORTED, "decode_step: more than %d rows per SM in one GEMV", DS_MAX_ROWS);
    if ((capacity + S - 1) / S * DS_HD * 4 > DS_SLOT)
        return fail(B2_ERR_UNSUPPORTED, "decode_step: capacity %d above %d (%d position splits of at most %d rows)",
                    capacity, S * (DS_SLOT / (DS_HD * 4)), S, DS_SLOT / (DS_HD * 4));
    const int smem = (int)sizeof(Smem);
    StepArgs a;
    a.layers = layers;
    a.n_layers = n_layers;
    a.x = x;
    a.x2 = x2;
    a.qkv = qkv;
    a.att = att;
    a.act = act;
    a.partial = partial;
    a.stats = stats;
    a.inv_freq = inv_freq;
    a.pos = pos;
    a.lengths = lengths;
    a.sync = sync;
    a.err = err;
    a.D = hidden;
    a.H = heads;
    a.Hk = kv_heads;
    a.F = mlp;
    a.cap = capacity;
    a.S = S;
    a.eps = eps;
    a.scale = (float)(1.0 / sqrt((double)DS_HD));  // the float nearest 128^-0.5, as the callers' d ** -0.5
    a.timeout_ns = (uint64_t)timeout_ns;
    void (*kernel)(StepArgs) = group == 4 ? decode_step_kernel<4> : group == 2 ? decode_step_kernel<2> : decode_step_kernel<1>;
    if (int rc = set_smem(kernel, smem)) return rc;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, DS_THREADS, smem) != cudaSuccess || per_sm < 1)
        return fail(B2_ERR_CUDA, "decode_step: the kernel does not fit on an SM");
    // The register split adds up only for the launch register count it was made for.
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess || fa.numRegs != DS_REGS_LAUNCH)
        return fail(B2_ERR_CUDA, "decode_step: kernel built with %d registers per thread, the split needs %d", fa.numRegs,
                    DS_REGS_LAUNCH);
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemsetAsync(sync, 0, DS_SYNC_WORDS * sizeof(unsigned), st) != cudaSuccess)
        return check_launch("decode_step: clearing the arrival counters");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(DS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, a);
    if (e != cudaSuccess) return fail(B2_ERR_CUDA, "decode_step_kernel: %s", cudaGetErrorString(e));
    return B2_OK;
}

extern "C" int b2_decode_step_splits(int kv_heads) {
    if (kv_heads <= 0) return 0;
    return std::min(DS_MAX_SPLITS, sm_count() / kv_heads);
}
