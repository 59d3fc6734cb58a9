// W4A8 GEMM with group-128 weight scales for sm_100a:
//   C[m, n] = fp16( F[m, n] * as[m] (+ bias[n]) ),  F = fma(acc_g, s[g, n], F) over groups g in order,
//   acc_g = sum over the g-th 128 k of A[m, k] * W[n, k]  (int8 x int4 -> int32, exact).
// The reference's int4 path is per-channel W4A4 (int8_gemm.hip:62-91 quant_row_i4, :412 gemm_i4; int8_gemm.py:90-103);
// the configuration asks for W4A8 with fp16 scales per 128 values along K, so this kernel follows the configuration.
//
// Layout: A int8 [M, K] (from the pre-pass), W packed uint8 [N, K/2] (low nibble = even k, two's-complement
// nibbles in [-8, 7]), group scales fp32 [K/128, N] (the fp16 scales widened once at load time, exact).
//
// Design. 256 x 128 output tiles on CTA pairs (clusters of two), persistent over tiles: one
// tcgen05.mma.cta_group::2.kind::i8 (M = 256, N = 128, K = 32) issued by CTA 0 reads A rows [128 r, 128 r + 128)
// and W rows [n0 + 64 r, n0 + 64 r + 64) of the tile from CTA r's shared memory and accumulates CTA r's 128 rows x
// 128 columns in its own TMEM. Per SM a k-block draws 16 KB of A and 4 KB of packed W from L2 for 361 tensor
// cycles; single-CTA 128 x 128 tiles with a widened weight draw 32 KB, which measured L2-bound on the
// configuration-3 shape. The fp32 sums of a CTA's 128 x 128 outputs fill a quarter of its register file, which is
// what bounds the tile's width.
// The weight reaches shared memory packed: TMA brings 64 rows x 64 bytes into a staging slot, and four converter
// warps (one per SM sub-partition) widen it into the 128-byte-swizzled K-major int8 tile the MMA reads, so no int8
// copy of the weight is ever written to memory.
// A k-block is one group. Its int32 partial goes to one of four 128-column TMEM buffers seeded with 0x4B400000 (the
// bits of 1.5 * 2^23), so the accumulator read back as fp32 minus 1.5 * 2^23 is acc_g exactly: one FADD instead of
// an int -> float conversion. Sixteen epilogue warps (four per TMEM lane quarter, 32 columns each, so that four
// warps per SM sub-partition hide each other's TMEM-load latency) fold each group into fp32 registers,
// F = fma(acc_g, s_g, F) on packed pairs, and re-seed the buffer while the MMA runs up to three groups ahead.
//
// Warps (768 threads; warpgroups 0-1 hand registers to the epilogue warpgroups 2-5 with setmaxnreg):
//   0       TMA producer: the A half into the stage (counted on CTA 0's full barrier), the packed W half into the
//           staging slot (counted on this CTA's loaded barrier)
//   1       TMEM owner; in CTA 0 also the MMA issuer
//   2..5    converters, 16 rows of this CTA's W half each; they arrive on CTA 0's full barrier
//   6, 7    idle
//   8..23   epilogue
#include "common.cuh"
#include "host.hpp"

namespace b2 {
namespace {

__device__ unsigned int g_status;

constexpr int GK = 128;                         // k per group and per k-block
constexpr int TN = 128;                         // tile columns (MMA N); each CTA holds TN / 2 rows of W
constexpr int STAGES = 6;
constexpr int A_BYTES = 128 * GK;               // 16 KB: 128 rows x 128 bytes
constexpr int B_BYTES = (TN / 2) * GK;          // 8 KB: 64 widened W rows x 128 bytes
constexpr int P_BYTES = (TN / 2) * GK / 2;      // 4 KB: 64 rows x 64 packed bytes
constexpr int S_BYTES = TN * 4;                 // the group's fp32 scales of the tile's columns
constexpr int OFF_B = A_BYTES, OFF_P = A_BYTES + B_BYTES, OFF_S = OFF_P + P_BYTES;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + P_BYTES + 1024;  // 29 KB with the scales, a multiple of 1024
constexpr int NPB = 4;                          // TMEM partial buffers of TN columns
constexpr int W4_THREADS = 768;
constexpr int EPI_WARPS = 16;
constexpr int EPI_COLS = TN / (EPI_WARPS / 4);  // 32 columns per epilogue warp
constexpr int REGS_CTRL = 32, REGS_EPI = 104;     // 256 x 32 + 512 x 104 = 61440 = 768 x 80 (the launch)
constexpr int SMEM = STAGES * STAGE_BYTES + 256 + 1024;
constexpr uint32_t SEED = 0x4B400000u;
constexpr float SEED_F = 12582912.0f;

struct W4Args {
    const float* as;
    const float* gs;  // [K / 128, N]
    const __half* bias;
    __half* C;
    int M, N, K;
};

// A 16-byte shared-memory load kept in program order with the TMEM loads around it (asm volatile with a memory
// clobber): issued just before a chunk's TMEM load, its latency hides under that load's; the compiler would otherwise
// hoist every scale load of a group ahead of the first TMEM load and run out of registers.
__device__ __forceinline__ float4 lds_ordered(const void* p) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(smem_u32(p))
                 : "memory");
    return v;
}

// Sign-extends four 4-bit fields held one per byte (low nibbles) into bytes: ((n ^ 8) + 0x78) ^ 0x80 per byte
// (no carry leaves a byte: n ^ 8 <= 15).
__device__ __forceinline__ uint32_t sext4(uint32_t v) { return ((v ^ 0x08080808u) + 0x78787878u) ^ 0x80808080u; }

// 8 packed bytes (16 int4, low nibble first) -> 16 int8 in k order.
__device__ __forceinline__ uint4 unpack16(uint32_t w0, uint32_t w1) {
    const uint32_t l0 = sext4(w0 & 0x0F0F0F0Fu), h0 = sext4((w0 >> 4) & 0x0F0F0F0Fu);
    const uint32_t l1 = sext4(w1 & 0x0F0F0F0Fu), h1 = sext4((w1 >> 4) & 0x0F0F0F0Fu);
    return make_uint4(__byte_perm(l0, h0, 0x5140), __byte_perm(l0, h0, 0x7362), __byte_perm(l1, h1, 0x5140),
                      __byte_perm(l1, h1, 0x7362));
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(W4_THREADS, 1)
    gemm_w4a8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                          const __grid_constant__ CUtensorMap tmS, const W4Args g) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* full = bars;                  // [STAGES] A halves landed, both W halves widened (CTA 0)
    uint64_t* loaded = bars + STAGES;       // [STAGES] packed W half and the group's scales landed (each CTA)
    uint64_t* empty = bars + 2 * STAGES;    // [STAGES] MMA and this CTA's epilogue done with the stage (each CTA)
    uint64_t* pready = bars + 3 * STAGES;   // [NPB] partial complete in TMEM (each CTA)
    uint64_t* pfree = pready + NPB;         // [NPB] partial folded and re-seeded by both CTAs (CTA 0)
    uint64_t* drain = pfree + NPB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
    const int num_m = (g.M + 255) / 256, num_n = (g.N + TN - 1) / TN;
    const int num_tiles = num_m * num_n;
    const int G = g.K / GK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 2 + 8);  // two producers (A bytes) and four converter warps per CTA
            mbar_init(&loaded[s], 1);
            mbar_init(&empty[s], 1 + EPI_WARPS);  // the MMA commit and each epilogue warp (scales read)
        }
        for (int b = 0; b < NPB; ++b) {
            mbar_init(&pready[b], 1);
            mbar_init(&pfree[b], 2 * EPI_WARPS);  // every epilogue warp of both CTAs
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmS);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before any remote arrival
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // the operands may come from the kernel launched before this one

    if (warp == 0) {
        regs_dec<REGS_CTRL>();
        if (lane == 0) {
            const uint64_t keep = l2_policy_evict_last(), normal = l2_policy_evict_normal();
            const uint32_t full0 = map_to_rank(smem_u32(full), 0);
            int stage = 0;
            uint32_t phase = 0, issued = 0, issued_ph = 0;
            bool ok = true;
            for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
                const int m0 = (tile % num_m) * 256, n0 = (tile / num_m) * TN;
                for (int kb = 0; kb < G; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, &g_status, B2_DEV_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    unsigned char* st = smem + stage * STAGE_BYTES;
                    const uint32_t bar = full0 + stage * 8;
                    mbar_arrive_expect_tx_remote(bar, A_BYTES);
                    tma_load_2d_pair(st, &tmA, bar, kb * GK, m0 + 128 * rank, normal);
                    mbar_arrive_expect_tx(&loaded[stage], P_BYTES + S_BYTES);
                    tma_load_2d_hint(st + OFF_P, &tmW, &loaded[stage], kb * (GK / 2), n0 + (TN / 2) * rank, keep);
                    tma_load_2d(st + OFF_S, &tmS, &loaded[stage], n0, kb);
                    issued |= 1u << stage;
                    issued_ph = (issued_ph & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok)  // let this CTA's own copies land before the CTA can exit
                for (int s = 0; s < STAGES; ++s)
                    if ((issued >> s) & 1)
                        if (!mbar_wait_drain(&loaded[s], (issued_ph >> s) & 1, 100000000ull))
                            atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
        }
    } else if (warp == 1) {
        regs_dec<REGS_CTRL>();
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_make(2, 1, 0, 0, 256, TN);
            const uint32_t empty_own = smem_u32(empty), empty_peer = map_to_rank(smem_u32(empty), 1);
            const uint32_t pready_own = smem_u32(pready), pready_peer = map_to_rank(smem_u32(pready), 1);
            int stage = 0;
            uint32_t phase = 0, q = 0;
            bool ok = true;
            for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
                for (int kb = 0; kb < G; ++kb, ++q) {
                    const uint32_t b = q % NPB;
                    if (!mbar_wait(&pfree[b], (q / NPB) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA) ||
                        !mbar_wait(&full[stage], phase, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
                    const uint64_t a_desc = sdesc_sw128(a_addr, 16, 1024);
                    const uint64_t b_desc = sdesc_sw128(a_addr + OFF_B, 16, 1024);
#pragma unroll
                    for (int k = 0; k < GK / 32; ++k)
                        mma_i8_ss_pair(tmem + b * TN, a_desc + (uint64_t)(k * 2), b_desc + (uint64_t)(k * 2), idesc, 1);
                    tc_commit_pair(empty_own + stage * 8);
                    tc_commit_pair(empty_peer + stage * 8);
                    tc_commit_pair(pready_own + b * 8);
                    tc_commit_pair(pready_peer + b * 8);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            tc_commit_pair(smem_u32(drain));
            if (!mbar_wait_drain(drain, 0, 100000000ull)) atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
        }
    } else if (warp < 6) {
        regs_dec<REGS_CTRL>();
        // Converters: warp cw widens rows 16 cw .. 16 cw + 15 of the stage's W half, four rows per step: lane ->
        // (row 4 i + lane / 8, 16-byte output chunk lane % 8, i.e. k 16 c .. 16 c + 15 from packed bytes 8 c .. 8 c + 7).
        const int cw = warp - 2;
        const uint32_t full0 = map_to_rank(smem_u32(full), 0);
        const int c = lane & 7;
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
            for (int kb = 0; kb < G; ++kb) {
                if (!mbar_wait(&loaded[stage], phase, abort_flag, &g_status, B2_DEV_TIMEOUT_PRODUCER)) {
                    ok = false;
                    break;
                }
                unsigned char* st = smem + stage * STAGE_BYTES;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = cw * 16 + i * 4 + (lane >> 3);
                    const uint2 p = *reinterpret_cast<const uint2*>(st + OFF_P + r * 64 + c * 8);
                    *reinterpret_cast<uint4*>(st + OFF_B + r * 128 + ((c ^ (r & 7)) << 4)) = unpack16(p.x, p.y);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote_release(full0 + stage * 8);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
    } else if (warp < 8) {
        regs_dec<REGS_CTRL>();
    } else {
        regs_inc<REGS_EPI>();
        // Epilogue: warp -> (32-lane TMEM quarter, 32-column slice); thread -> one row, 32 fp32 sums in 16 pairs.
        const int quarter = warp & 3;
        const int slice = (warp - 8) >> 2;
        const uint32_t pfree0 = map_to_rank(smem_u32(pfree), 0);
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const uint32_t col0 = tmem + lane_base + slice * EPI_COLS;
#pragma unroll
        for (int b = 0; b < NPB; ++b) tmem_fill32(col0 + b * TN, SEED);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int b = 0; b < NPB; ++b) mbar_arrive_remote(pfree0 + b * 8);
        const uint64_t nseed = pk2(-SEED_F, -SEED_F);
        uint32_t q = 0;
        bool ok = true;
        for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
            const int m0 = (tile % num_m) * 256, n0 = (tile / num_m) * TN + slice * EPI_COLS;
            uint64_t F[EPI_COLS / 2];
#pragma unroll
            for (int i = 0; i < EPI_COLS / 2; ++i) F[i] = 0ull;
            for (int kb = 0; kb < G; ++kb, ++q) {
                const uint32_t b = q % NPB, stage = q % STAGES;
                if (!mbar_wait(&pready[b], (q / NPB) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_EPILOGUE) ||
                    !mbar_wait(&loaded[stage], (q / STAGES) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_EPILOGUE)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const unsigned char* ss = smem + stage * STAGE_BYTES + OFF_S + slice * EPI_COLS * 4;
#pragma unroll
                for (int c = 0; c < EPI_COLS / 16; ++c) {
                    float4 s4[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) s4[i] = lds_ordered(ss + c * 64 + i * 16);
                    uint32_t v[16];
                    tmem_ld16_wait(col0 + b * TN + c * 16, v);
                    // Re-seed once the last chunk is read, so that the store runs under the last chunk's arithmetic.
                    if (c == EPI_COLS / 16 - 1) tmem_fill32(col0 + b * TN, SEED);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint64_t a0 = add2(pk2(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1])), nseed);
                        const uint64_t a1 = add2(pk2(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])), nseed);
                        F[c * 8 + 2 * i] = fma2(a0, pk2(s4[i].x, s4[i].y), F[c * 8 + 2 * i]);
                        F[c * 8 + 2 * i + 1] = fma2(a1, pk2(s4[i].z, s4[i].w), F[c * 8 + 2 * i + 1]);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive_remote(pfree0 + b * 8);
                    mbar_arrive(&empty[stage]);
                }
            }
            if (!ok) break;
            const int m = m0 + 128 * (int)rank + quarter * 32 + lane;
            if (m < g.M) {
                const float sa = g.as[m];
                __half* dst = g.C + (int64_t)m * g.N + n0;
#pragma unroll
                for (int j = 0; j < EPI_COLS / 8; ++j) {
                    if (n0 + 8 * j >= g.N) continue;  // (not break: F must stay register-indexed)
                    float y[8];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = upk2(F[4 * j + e]);
                        y[2 * e] = __fmul_rn(f.x, sa);
                        y[2 * e + 1] = __fmul_rn(f.y, sa);
                    }
                    if (g.bias) {
                        const uint4 braw = *reinterpret_cast<const uint4*>(g.bias + n0 + 8 * j);
                        const __half2* bh = reinterpret_cast<const __half2*>(&braw);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 bf = __half22float2(bh[e]);
                            y[2 * e] = __fadd_rn(y[2 * e], bf.x);
                            y[2 * e + 1] = __fadd_rn(y[2 * e + 1], bf.y);
                        }
                    }
                    uint4 o;
                    __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
                    for (int e = 0; e < 4; ++e) oh[e] = __floats2half2_rn(y[2 * e], y[2 * e + 1]);
                    *reinterpret_cast<uint4*>(dst + 8 * j) = o;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer's shared memory, barriers and TMEM stay alive until the pair is done with them
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, 512);
}

// ---------------------------------------------------------------- W4A8 on a widened weight
// The same arithmetic on a weight already widened to int8 [N, K] (values in [-8, 7]): the Int4 loader's
// convrot_w4a4_forward call shape carries such a copy (qweight_unpacked, int8_gemm.py:91), and b2_unpack_int4 makes
// one. With no conversion on the chip the tile can be 256 x 256 (M = 256, N = 256 pair MMAs, each CTA's B half 128
// rows, the full MMA rate), fed by TMA like the W8A8 pair kernel. The CTA's 128 x 256 fp32 sums then take half of
// its register file: sixteen epilogue warps (four per lane quarter, 64 columns each) hold them, with registers
// moved to them from the producer/MMA warpgroup by setmaxnreg; two 256-column TMEM buffers alternate groups.
//   warp 0 TMA producer, warp 1 TMEM owner + MMA issuer (CTA 0), warps 2-3 idle, warps 4..19 epilogue.
constexpr int WIDE_STAGES = 6;
constexpr int WIDE_HALF = 128 * GK;                          // 16 KB: 128 rows x 128 bytes
constexpr int WIDE_OFF_S = 2 * WIDE_HALF;                    // the group's scales of the tile's 256 columns (1 KB)
constexpr int WIDE_STAGE_BYTES = 2 * WIDE_HALF + 1024;       // A half + W half + scales
constexpr int WIDE_THREADS = 640;
constexpr int WIDE_EPI_WARPS = 16;
constexpr int WIDE_COLS = 256 / (WIDE_EPI_WARPS / 4);        // 64 columns per epilogue warp
constexpr int WIDE_REGS_CTRL = 32, WIDE_REGS_EPI = 112;      // 128 x 32 + 512 x 112 = 61440 = 640 x 96 (the launch)
constexpr int WIDE_SMEM = WIDE_STAGES * WIDE_STAGE_BYTES + 256 + 1024;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(WIDE_THREADS, 1)
    gemm_w4a8_wide_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                          const __grid_constant__ CUtensorMap tmS, const W4Args g) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + WIDE_STAGES * WIDE_STAGE_BYTES);
    uint64_t* full = bars;                       // [STAGES] both CTAs' halves landed (CTA 0)
    uint64_t* empty = bars + WIDE_STAGES;        // [STAGES] MMA and this CTA's epilogue done with the stage (each CTA)
    uint64_t* sload = bars + 2 * WIDE_STAGES;    // [STAGES] the group's scales landed (each CTA)
    uint64_t* pready = bars + 3 * WIDE_STAGES;   // [2] partial complete in TMEM (each CTA)
    uint64_t* pfree = pready + 2;                // [2] partial folded and re-seeded by both CTAs (CTA 0)
    uint64_t* drain = pfree + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
    const int num_m = (g.M + 255) / 256, num_n = (g.N + 255) / 256;
    const int num_tiles = num_m * num_n;
    const int G = g.K / GK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < WIDE_STAGES; ++s) {
            mbar_init(&full[s], 2);
            mbar_init(&empty[s], 1 + WIDE_EPI_WARPS);
            mbar_init(&sload[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&pready[b], 1);
            mbar_init(&pfree[b], 2 * WIDE_EPI_WARPS);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmS);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // the operands may come from the kernel launched before this one

    if (warp < 4) {
        regs_dec<WIDE_REGS_CTRL>();
        if (warp == 0 && lane == 0) {
            const uint64_t keep = l2_policy_evict_last(), normal = l2_policy_evict_normal();
            const uint32_t full0 = map_to_rank(smem_u32(full), 0);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
                const int m0 = (tile % num_m) * 256, n0 = (tile / num_m) * 256;
                for (int kb = 0; kb < G; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, &g_status, B2_DEV_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    unsigned char* st = smem + stage * WIDE_STAGE_BYTES;
                    const uint32_t bar = full0 + stage * 8;
                    mbar_arrive_expect_tx_remote(bar, 2 * WIDE_HALF);
                    tma_load_2d_pair(st, &tmA, bar, kb * GK, m0 + 128 * rank, normal);
                    tma_load_2d_pair(st + WIDE_HALF, &tmW, bar, kb * GK, n0 + 128 * rank, keep);
                    mbar_arrive_expect_tx(&sload[stage], 1024);
                    tma_load_2d(st + WIDE_OFF_S, &tmS, &sload[stage], n0, kb);
                    if (++stage == WIDE_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        } else if (warp == 1 && lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_make(2, 1, 0, 0, 256, 256);
            const uint32_t empty_own = smem_u32(empty), empty_peer = map_to_rank(smem_u32(empty), 1);
            const uint32_t pready_own = smem_u32(pready), pready_peer = map_to_rank(smem_u32(pready), 1);
            int stage = 0;
            uint32_t phase = 0, q = 0;
            bool ok = true;
            for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
                for (int kb = 0; kb < G; ++kb, ++q) {
                    const uint32_t b = q & 1;
                    if (!mbar_wait(&pfree[b], (q >> 1) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA) ||
                        !mbar_wait(&full[stage], phase, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * WIDE_STAGE_BYTES);
                    const uint64_t a_desc = sdesc_sw128(a_addr, 16, 1024);
                    const uint64_t b_desc = sdesc_sw128(a_addr + WIDE_HALF, 16, 1024);
#pragma unroll
                    for (int k = 0; k < GK / 32; ++k)
                        mma_i8_ss_pair(tmem + b * 256, a_desc + (uint64_t)(k * 2), b_desc + (uint64_t)(k * 2), idesc, 1);
                    tc_commit_pair(empty_own + stage * 8);
                    tc_commit_pair(empty_peer + stage * 8);
                    tc_commit_pair(pready_own + b * 8);
                    tc_commit_pair(pready_peer + b * 8);
                    if (++stage == WIDE_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            tc_commit_pair(smem_u32(drain));
            if (!mbar_wait_drain(drain, 0, 100000000ull)) atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
        }
    } else {
        regs_inc<WIDE_REGS_EPI>();
        // Epilogue: warp -> (32-lane TMEM quarter, 64-column slice); thread -> one row, 64 fp32 sums in 32 pairs.
        const int quarter = warp & 3;
        const int slice = (warp - 4) >> 2;
        const uint32_t pfree0 = map_to_rank(smem_u32(pfree), 0);
        const uint32_t col0 = tmem + ((uint32_t)(quarter * 32) << 16) + slice * WIDE_COLS;
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int c = 0; c < WIDE_COLS / 32; ++c) tmem_fill32(col0 + b * 256 + c * 32, SEED);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive_remote(pfree0);
            mbar_arrive_remote(pfree0 + 8);
        }
        const uint64_t nseed = pk2(-SEED_F, -SEED_F);
        uint32_t q = 0;
        bool ok = true;
        for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
            const int m0 = (tile % num_m) * 256, n0 = (tile / num_m) * 256 + slice * WIDE_COLS;
            uint64_t F[WIDE_COLS / 2];
#pragma unroll
            for (int i = 0; i < WIDE_COLS / 2; ++i) F[i] = 0ull;
            for (int kb = 0; kb < G; ++kb, ++q) {
                const uint32_t b = q & 1, stage = q % WIDE_STAGES;
                if (!mbar_wait(&pready[b], (q >> 1) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_EPILOGUE) ||
                    !mbar_wait(&sload[stage], (q / WIDE_STAGES) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_EPILOGUE)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const unsigned char* ss = smem + stage * WIDE_STAGE_BYTES + WIDE_OFF_S + slice * WIDE_COLS * 4;
#pragma unroll
                for (int c = 0; c < WIDE_COLS / 16; ++c) {
                    float4 s4[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) s4[i] = lds_ordered(ss + c * 64 + i * 16);
                    uint32_t v[16];
                    tmem_ld16_wait(col0 + b * 256 + c * 16, v);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint64_t a0 = add2(pk2(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1])), nseed);
                        const uint64_t a1 = add2(pk2(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])), nseed);
                        F[c * 8 + 2 * i] = fma2(a0, pk2(s4[i].x, s4[i].y), F[c * 8 + 2 * i]);
                        F[c * 8 + 2 * i + 1] = fma2(a1, pk2(s4[i].z, s4[i].w), F[c * 8 + 2 * i + 1]);
                    }
                }
#pragma unroll
                for (int c = 0; c < WIDE_COLS / 32; ++c) tmem_fill32(col0 + b * 256 + c * 32, SEED);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive_remote(pfree0 + b * 8);
                    mbar_arrive(&empty[stage]);
                }
            }
            if (!ok) break;
            const int m = m0 + 128 * (int)rank + quarter * 32 + lane;
            if (m < g.M) {
                const float sa = g.as[m];
                __half* dst = g.C + (int64_t)m * g.N + n0;
#pragma unroll
                for (int j = 0; j < WIDE_COLS / 8; ++j) {
                    if (n0 + 8 * j >= g.N) continue;  // (not break: F must stay register-indexed)
                    float y[8];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = upk2(F[4 * j + e]);
                        y[2 * e] = __fmul_rn(f.x, sa);
                        y[2 * e + 1] = __fmul_rn(f.y, sa);
                    }
                    if (g.bias) {
                        const uint4 braw = *reinterpret_cast<const uint4*>(g.bias + n0 + 8 * j);
                        const __half2* bh = reinterpret_cast<const __half2*>(&braw);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 bf = __half22float2(bh[e]);
                            y[2 * e] = __fadd_rn(y[2 * e], bf.x);
                            y[2 * e + 1] = __fadd_rn(y[2 * e + 1], bf.y);
                        }
                    }
                    uint4 o;
                    __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
                    for (int e = 0; e < 4; ++e) oh[e] = __floats2half2_rn(y[2 * e], y[2 * e + 1]);
                    *reinterpret_cast<uint4*>(dst + 8 * j) = o;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer's shared memory, barriers and TMEM stay alive until the pair is done with them
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, 512);
}

}  // namespace

unsigned int read_status_gemm_w4a8() {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    if (v) cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
    return v;
}

}  // namespace b2

using namespace b2;

// Launches a W4A8 kernel with programmatic stream serialization: its CTAs may set up while the pre-pass that made
// its activations finishes, and read them after pdl_wait().
template <class Kern>
int launch_pdl(Kern kernel, int grid, int threads, int smem, void* stream, const char* name, const CUtensorMap& ta,
               const CUtensorMap& tw, const CUtensorMap& ts, const W4Args& g) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ta, tw, ts, g);
    if (e != cudaSuccess) return fail(B2_ERR_CUDA, "%s launch: %s", name, cudaGetErrorString(e));
    return check_launch(name);
}

extern "C" int b2_gemm_w4a8(const int8_t* A, const uint8_t* Wp, const float* as, const float* gscale, const uint16_t* bias,
                            uint16_t* C, int M, int N, int K, void* stream) {
    if (!A || !Wp || !as || !gscale || !C) return fail(B2_ERR_INVALID, "gemm_w4a8: null pointer");
    if (M < 0 || N <= 0 || K <= 0) return fail(B2_ERR_INVALID, "gemm_w4a8: bad shape M=%d N=%d K=%d", M, N, K);
    if (K % GK) return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8: K=%d must be a multiple of 128", K);
    if (N % 8) return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8: N=%d must be a multiple of 8", N);
    if (!aligned16(A) || !aligned16(Wp) || !aligned16(gscale) || !aligned16(C) || (bias && !aligned16(bias)))
        return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8: operands must be 16-byte aligned");
    if (M == 0) return B2_OK;
    CUtensorMap ta, tw;
    if (int rc = make_map_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, K, GK, 128)) return rc;
    if (int rc = make_map_2d(&tw, Wp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, K / 2, GK / 2, TN / 2,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
        return rc;
    CUtensorMap ts;  // group scales [K / 128, N]: one row of the tile's TN columns per group (zero past N)
    if (int rc = make_map_2d(&ts, gscale, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, K / GK, (uint64_t)N * 4, TN, 1,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
        return rc;
    static int clusters[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8: device index %d out of range", dev);
    if (!clusters[dev]) {
        // The setmaxnreg split needs the CTA launched with at least 80 registers per thread.
        cudaFuncAttributes attr;
        if (cudaFuncGetAttributes(&attr, gemm_w4a8_pair_kernel) != cudaSuccess)
            return fail(B2_ERR_CUDA, "gemm_w4a8: cudaFuncGetAttributes failed");
        if (attr.numRegs * W4_THREADS < 256 * REGS_CTRL + 512 * REGS_EPI)
            return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8: kernel built with %d registers per thread, below its split",
                        attr.numRegs);
        if (int rc = set_smem(gemm_w4a8_pair_kernel, SMEM)) return rc;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
        cfg.blockDim = dim3(W4_THREADS, 1, 1);
        cfg.dynamicSmemBytes = SMEM;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_w4a8_pair_kernel, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = sm_count() / 2;
        }
        clusters[dev] = n;
    }
    W4Args g{as, gscale, reinterpret_cast<const __half*>(bias), reinterpret_cast<__half*>(C), M, N, K};
    const int tiles = ((M + 255) / 256) * ((N + TN - 1) / TN);
    const int nc = tiles < clusters[dev] ? tiles : clusters[dev];
    return launch_pdl(gemm_w4a8_pair_kernel, 2 * nc, W4_THREADS, SMEM, stream, "gemm_w4a8_pair_kernel", ta, tw, ts, g);
}

extern "C" int b2_gemm_w4a8_wide(const int8_t* A, const int8_t* W, const float* as, const float* gscale,
                                 const uint16_t* bias, uint16_t* C, int M, int N, int K, void* stream) {
    if (!A || !W || !as || !gscale || !C) return fail(B2_ERR_INVALID, "gemm_w4a8_wide: null pointer");
    if (M < 0 || N <= 0 || K <= 0) return fail(B2_ERR_INVALID, "gemm_w4a8_wide: bad shape M=%d N=%d K=%d", M, N, K);
    if (K % GK) return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8_wide: K=%d must be a multiple of 128", K);
    if (N % 8) return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8_wide: N=%d must be a multiple of 8", N);
    if (!aligned16(A) || !aligned16(W) || !aligned16(gscale) || !aligned16(C) || (bias && !aligned16(bias)))
        return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8_wide: operands must be 16-byte aligned");
    if (M == 0) return B2_OK;
    CUtensorMap ta, tw;
    if (int rc = make_map_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, K, GK, 128)) return rc;
    if (int rc = make_map_2d(&tw, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, K, GK, 128)) return rc;
    CUtensorMap ts;  // group scales [K / 128, N]: one row of the tile's 256 columns per group (zero past N)
    if (int rc = make_map_2d(&ts, gscale, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, K / GK, (uint64_t)N * 4, 256, 1,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
        return rc;
    static int clusters[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8_wide: device index %d out of range", dev);
    if (!clusters[dev]) {
        // The setmaxnreg split needs the CTA launched with at least 96 registers per thread.
        cudaFuncAttributes attr;
        if (cudaFuncGetAttributes(&attr, gemm_w4a8_wide_kernel) != cudaSuccess)
            return fail(B2_ERR_CUDA, "gemm_w4a8_wide: cudaFuncGetAttributes failed");
        if (attr.numRegs * WIDE_THREADS < 128 * WIDE_REGS_CTRL + 512 * WIDE_REGS_EPI)
            return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8_wide: kernel built with %d registers per thread, below its split",
                        attr.numRegs);
        if (int rc = set_smem(gemm_w4a8_wide_kernel, WIDE_SMEM)) return rc;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
        cfg.blockDim = dim3(WIDE_THREADS, 1, 1);
        cfg.dynamicSmemBytes = WIDE_SMEM;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_w4a8_wide_kernel, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = sm_count() / 2;
        }
        clusters[dev] = n;
    }
    W4Args g{as, gscale, reinterpret_cast<const __half*>(bias), reinterpret_cast<__half*>(C), M, N, K};
    const int tiles = ((M + 255) / 256) * ((N + 255) / 256);
    const int nc = tiles < clusters[dev] ? tiles : clusters[dev];
    return launch_pdl(gemm_w4a8_wide_kernel, 2 * nc, WIDE_THREADS, WIDE_SMEM, stream, "gemm_w4a8_wide_kernel", ta, tw, ts,
                      g);
}

// ---------------------------------------------------------------- per-channel W4A4
// The reference's own int4 path (int8_gemm.hip:412 gemm_i4, int8_gemm.py:90-103): activations with int4 values
// (b2_quant_pack_a_i4), int4 weights with one fp32 scale per output channel, int32 accumulation over all of K and
// the W8A8 epilogue y = (float)acc * as[m] * ws[n] (+ bias[n]). tcgen05 has no integer int4 kind, so the packed
// weight is widened to int8 into a caller-provided workspace by one streaming pass (as the reference re-packs its
// weights per call, pack_b, int8_gemm.hip:270-276) and the W8A8 kernel runs on it; int32 sums are exact in any
// order, so the result is the reference's bit for bit.
namespace b2 {
namespace {

// Four nibble values b in [0, 15] (one per byte) -> two's-complement int8 bytes: (b ^ 8) - 8 per byte.
__device__ __forceinline__ uint32_t sext_nibbles(uint32_t b) { return __vsub4(b ^ 0x08080808u, 0x08080808u); }

// Packed byte j holds k = 2j (low nibble) and k = 2j + 1 (high nibble). Each thread widens 16 packed bytes (32
// values) into two 16-byte stores.
__global__ void __launch_bounds__(256) unpack_int4_kernel(const uint4* __restrict__ wp, uint4* __restrict__ w, int64_t n16) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
        const uint4 p = __ldg(wp + i);
        const uint32_t in[4] = {p.x, p.y, p.z, p.w};
        uint32_t o[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t lo = in[j] & 0x0F0F0F0Fu, hi = (in[j] >> 4) & 0x0F0F0F0Fu;
            o[2 * j] = sext_nibbles(__byte_perm(lo, hi, 0x5140));      // k = 8j .. 8j + 3
            o[2 * j + 1] = sext_nibbles(__byte_perm(lo, hi, 0x7362));  // k = 8j + 4 .. 8j + 7
        }
        w[2 * i] = make_uint4(o[0], o[1], o[2], o[3]);
        w[2 * i + 1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

}  // namespace
}  // namespace b2

extern "C" int b2_unpack_int4(const uint8_t* Wp, int8_t* W, int N, int K, void* stream) {
    if (!Wp || !W || N < 0 || K <= 0) return fail(B2_ERR_INVALID, "unpack_int4: bad arguments");
    if (K % 32) return fail(B2_ERR_UNSUPPORTED, "unpack_int4: K=%d must be a multiple of 32", K);
    if (!aligned16(Wp) || !aligned16(W)) return fail(B2_ERR_UNSUPPORTED, "unpack_int4: Wp and W must be 16-byte aligned");
    const int64_t n16 = (int64_t)N * (K / 32);
    if (n16 == 0) return B2_OK;
    const int64_t blocks = (n16 + 255) / 256;
    const int cap = sm_count() * 8;
    unpack_int4_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint4*>(Wp), reinterpret_cast<uint4*>(W), n16);
    return check_launch("unpack_int4_kernel");
}

extern "C" int b2_gemm_w4a4(const int8_t* A, const uint8_t* Wp, const float* as, const float* ws, const uint16_t* bias,
                            uint16_t* C, int M, int N, int K, int8_t* workspace, void* stream) {
    if (!A || !Wp || !as || !ws || !C || !workspace) return fail(B2_ERR_INVALID, "gemm_w4a4: null pointer");
    if (M < 0 || N <= 0 || K <= 0) return fail(B2_ERR_INVALID, "gemm_w4a4: bad shape M=%d N=%d K=%d", M, N, K);
    if (K % 32) return fail(B2_ERR_UNSUPPORTED, "gemm_w4a4: K=%d must be a multiple of 32", K);
    if (N % 8) return fail(B2_ERR_UNSUPPORTED, "gemm_w4a4: N=%d must be a multiple of 8", N);
    if (M == 0) return B2_OK;
    if (int rc = b2_unpack_int4(Wp, workspace, N, K, stream)) return rc;
    return b2_gemm(A, workspace, as, ws, bias, C, M, N, K, nullptr, nullptr, 1, stream);
}
