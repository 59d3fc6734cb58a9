// W8A8 GEMM for sm_100a: C[M,N] = epilogue(A[M,K] int8 . B[N,K]^T int8), int32 accumulation in TMEM.
//
// Replaces int8_gemm.hip gemm_body (:315-406) and pack_b (:271-276). The weight is read as stored
// (int8 [N, K], K-major) by TMA, so there is no per-call re-layout. Epilogue semantics (:371-405):
//   y = (float)acc * as[m] * ws[n] (+ (float)bias[n]) -> fp16
//   residual: out = fp16(R[m,n] + fp16(G[m / L, n] * y))
//
// Structure: a persistent kernel, one CTA per SM, 14 warps; tiles 128 x BN (BN = 128, 192 or 256, whichever needs the
// fewest waves x width) or, for large problems, 256 x 256 on CTA pairs (gemm_w8a8_pair_kernel below).
//   warp 0      TMA producer: 128x128 A tiles and BNx128 B tiles (128-byte swizzle) into a STAGES-deep ring
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer (M=128, N=BN, K=32 per instruction)
//   warps 2..13 epilogue: tcgen05.ld of the int32 accumulator (three warps per 32-lane quarter, every third
//               16-column box), dequant, bias, residual, fp16 through a swizzled shared-memory box and one TMA store
//               per 32 x 16 box. One warp per quarter left the epilogue latency-bound (a 128-row tile's 192 columns
//               took 5 us on one wave, 3.4 us with two warps per quarter); more warps per scheduler overlap each
//               other's waits.
// Two TMEM accumulators (BN columns each) let the epilogue of tile i overlap the main loop of tile i+1.
#include "common.cuh"
#include "host.hpp"

namespace b2 {
namespace {

__device__ unsigned int g_status;

constexpr int BM = 128;
constexpr int BK = 128;  // bytes = int8 values per k-block (one 128-byte swizzle atom)
constexpr int EPI_WARPS = 12;  // warps 2..13
constexpr int EPI_SPLIT = EPI_WARPS / 4;  // epilogue warps per TMEM lane quarter
constexpr int GEMM_THREADS = 64 + 32 * EPI_WARPS;

// Epilogue staging: per epilogue warp EPI_BUFS boxes of 32 rows x 32 bytes (16 fp16 columns).
constexpr int EPI_BUFS = 2;
constexpr int EPI_BUF_BYTES = 32 * 32;
constexpr int EPI_WARP_BYTES = EPI_BUFS * EPI_BUF_BYTES;
constexpr int EPI_BYTES = EPI_WARPS * EPI_WARP_BYTES;

template <int BN>
struct Cfg {
    static constexpr int STAGES = BN == 256 ? 4 : BN == 192 ? 5 : 6;
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int ACC_STRIDE = BN == 192 ? 256 : BN;  // TMEM columns between the two accumulators
    static constexpr int TMEM_COLS = 2 * ACC_STRIDE;          // allocations are powers of two
    static constexpr int BAR_BYTES = 512;
    static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES + BN * 8 + 1024;
};

struct GemmArgs {
    const float* as;
    const float* ws;
    const __half* bias;
    __half* C;
    int32_t* C32;
    const __half* R;
    const __half* G;
    int L;
    int M, N, K;
    int swiglu;  // gate/up GEMM with rows interleaved in blocks of 128: C[M, N/2] = SwiGLU(gate, up)
};

// 32 raw int32 accumulator columns of one row (the debugging output C32), stored from registers.
__device__ __forceinline__ void epilogue_chunk_i32(const GemmArgs& g, uint32_t taddr, int m, bool row_ok, int nb) {
    uint32_t r[32];
    tmem_ld32_wait(taddr, r);
    if (!row_ok || nb >= g.N) return;
    int32_t* dst = g.C32 + (int64_t)m * g.N + nb;
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (nb + 4 * j < g.N)
            *reinterpret_cast<uint4*>(dst + 4 * j) = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
}

// One epilogue warp's share of a tile: 32 accumulator rows (TMEM lanes of the warp's quarter) x the tile's 16-column
// boxes part, part + EPI_SPLIT, ... (the EPI_SPLIT warps of a quarter take turns). Row `lane` of a box is dequantized in
// registers and written into a staging box of 32 rows x 32 bytes with the 32-byte swizzle (16-byte piece j of row r
// at piece j ^ ((r >> 2) & 1): the row-per-lane writes are free of bank conflicts), and lane 0 stores the box with
// one TMA store (TMA clips rows >= M and columns >= N). With a residual, lane 0 brings the warp's next box of R in by
// TMA one box ahead into the other staging box. The warp's n-th box uses staging box n % 2; a staging box is refilled
// only after the store that last read it is done reading (bulk_wait_read), and every R load is waited for before the
// function returns.
struct EpiCtx {
    unsigned char* buf;  // EPI_BUFS boxes
    uint64_t* rbar;      // EPI_BUFS barriers for the residual loads
    uint32_t n;          // chunks this warp has processed
    uint32_t inflight;   // bit b: a residual load into box b is in flight; bit 8 + b: its phase parity
};

__device__ __forceinline__ void epi_load_r(const CUtensorMap* tmR, EpiCtx& e, uint32_t chunk, int col, int row0) {
    const uint32_t b = chunk % EPI_BUFS;
    mbar_arrive_expect_tx(&e.rbar[b], EPI_BUF_BYTES);
    tma_load_2d(e.buf + b * EPI_BUF_BYTES, tmR, &e.rbar[b], col, row0);
    e.inflight = (e.inflight & ~(0x101u << b)) | (1u << b) | ((((chunk / EPI_BUFS) & 1u)) << (8 + b));
}

__device__ __noinline__ void epi_drain(EpiCtx& e) {
    for (int b = 0; b < EPI_BUFS; ++b)
        if (e.inflight & (1u << b))
            if (!mbar_wait_drain(&e.rbar[b], (e.inflight >> (8 + b)) & 1, 100000000ull))
                atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
    e.inflight = 0;
}

// The tile's per-column weight scales and bias (as fp32), staged in shared memory by the 128 epilogue threads
// (t = 0..127) while the k-loop still runs: no chunk of the epilogue waits on an L2 round trip for them, and the
// bias is converted once per tile instead of once per row. Columns past N are clamped to the last group of 4 or 8
// (N % 8 == 0); their results are never stored.
template <int BN>
__device__ __forceinline__ void epi_stage_cols(const GemmArgs& g, float* cw, float* cb, int n0, int t) {
    if (!g.ws) return;  // raw int32 output: no epilogue parameters
    if (t < BN / 4) {
        reinterpret_cast<float4*>(cw)[t] = __ldg(reinterpret_cast<const float4*>(g.ws + min(n0 + 4 * t, g.N - 4)));
    } else if (t < BN / 4 + BN / 8) {
        const int i = t - BN / 4;
        const uint4 h = g.bias ? __ldg(reinterpret_cast<const uint4*>(g.bias + min(n0 + 8 * i, g.N - 8)))
                               : make_uint4(0, 0, 0, 0);
        const float2 f0 = upk2(h2_to_f2(h.x)), f1 = upk2(h2_to_f2(h.y)), f2 = upk2(h2_to_f2(h.z)),
                     f3 = upk2(h2_to_f2(h.w));
        reinterpret_cast<float4*>(cb)[2 * i] = make_float4(f0.x, f0.y, f1.x, f1.y);
        reinterpret_cast<float4*>(cb)[2 * i + 1] = make_float4(f2.x, f2.y, f3.x, f3.y);
    }
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// The per-row gate of 16 columns from global memory (columns past N clamped to the last group of 8, their results
// never stored).
struct EpiParams {
    uint4 gt[2];
};

__device__ __forceinline__ void epi_params(const GemmArgs& g, const __half* gate_row, int nb, EpiParams& p) {
#pragma unroll
    for (int j = 0; j < 2; ++j)
        p.gt[j] = gate_row ? __ldg(reinterpret_cast<const uint4*>(gate_row + min(nb + 8 * j, g.N - 8)))
                           : make_uint4(0, 0, 0, 0);
}

// The dequant of one box runs on fp32 pairs: v = fp32(acc) * as * ws (two roundings, as the scalar form), + bias,
// then fp16; the residual fp16(R + fp16(G * y)) uses fp16 pair operations, which round exactly like the fp32 form
// (fp32 holds the exact sum or product of two fp16 values to within a rounding that cannot move the fp16 result).
// The gate of the warp's next box loads while this one computes; sa is the row's activation scale, read before the
// accumulator was ready. NB = 16-column boxes in a full tile.
template <int NB>
__device__ __forceinline__ bool epilogue_tile(const GemmArgs& g, const CUtensorMap* tmC, const CUtensorMap* tmR,
                                              EpiCtx& e, uint32_t taddr, int row0, int n0, int part, const float* cw,
                                              const float* cb, float sa, volatile int* abort) {
    const int lane = threadIdx.x & 31;
    const int m = row0 + lane;
    const bool row_ok = m < g.M;
    const uint64_t sa2 = splat2(sa);
    const int nc = min(NB, (g.N - n0 + 15) / 16);
    const bool res = g.R != nullptr;
    const __half* gate_row = (res && row_ok && g.G) ? g.G + (int64_t)(m / g.L) * g.N : nullptr;  // G null: gate 1
    const int sw = (lane >> 2) & 1;
    bool ok = true;
    EpiParams P[2];
    epi_params(g, gate_row, n0 + 16 * part, P[0]);
    if (res && lane == 0 && part < nc) {
        bulk_wait_read<EPI_BUFS - 1>();
        epi_load_r(tmR, e, e.n, n0 + 16 * part, row0);
    }
#pragma unroll
    for (int i = 0; i < (NB + EPI_SPLIT - 1) / EPI_SPLIT; ++i) {
        const int c = EPI_SPLIT * i + part;
        if (c >= nc) break;
        EpiParams& p = P[i & 1];
        if (c + EPI_SPLIT < nc) epi_params(g, gate_row, n0 + 16 * (c + EPI_SPLIT), P[(i + 1) & 1]);
        const uint32_t b = e.n % EPI_BUFS;
        unsigned char* box = e.buf + b * EPI_BUF_BYTES;
        if (res) {
            if (lane == 0 && c + EPI_SPLIT < nc) {
                bulk_wait_read<EPI_BUFS - 2>();
                epi_load_r(tmR, e, e.n + 1, n0 + 16 * (c + EPI_SPLIT), row0);
            }
            if (!mbar_wait(&e.rbar[b], (e.n / EPI_BUFS) & 1, abort, &g_status, B2_DEV_TIMEOUT_EPILOGUE)) {
                ok = false;
                break;
            }
            if (lane == 0) e.inflight &= ~(1u << b);
        } else {
            if (lane == 0) bulk_wait_read<EPI_BUFS - 1>();
            __syncwarp();
        }
        uint32_t r[16];
        tmem_ld16_wait(taddr + 16 * c, r);
        unsigned char* row = box + lane * 32;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            float wv[8], bv[8];
            *reinterpret_cast<float4*>(wv) = *reinterpret_cast<const float4*>(cw + 16 * c + 8 * j);
            *reinterpret_cast<float4*>(wv + 4) = *reinterpret_cast<const float4*>(cw + 16 * c + 8 * j + 4);
            *reinterpret_cast<float4*>(bv) = *reinterpret_cast<const float4*>(cb + 16 * c + 8 * j);
            *reinterpret_cast<float4*>(bv + 4) = *reinterpret_cast<const float4*>(cb + 16 * c + 8 * j + 4);
            const uint32_t* gw = reinterpret_cast<const uint32_t*>(&p.gt[j]);
            uint4* slot = reinterpret_cast<uint4*>(row + ((j ^ sw) << 4));
            uint4 rr = make_uint4(0, 0, 0, 0);
            if (res) rr = *slot;
            const uint32_t* rw = reinterpret_cast<const uint32_t*>(&rr);
            uint4 o;
            uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint64_t v = mul2(mul2(pk2((float)(int32_t)r[8 * j + 2 * q], (float)(int32_t)r[8 * j + 2 * q + 1]), sa2),
                                  pk2(wv[2 * q], wv[2 * q + 1]));
                if (g.bias) {
                    // Scalar adds: a packed add after the packed multiply was fused into one rounding by the
                    // compiler, which moved some results by an fp16 step.
                    const float2 f = upk2(v);
                    v = pk2(__fadd_rn(f.x, bv[2 * q]), __fadd_rn(f.y, bv[2 * q + 1]));
                }
                uint32_t y = f2_to_h2(v);
                if (res)  // with no gate, fp16(1 * y) = y: the same bits without the gate rows
                    y = h2_as_u32(g.G ? __hadd2_rn(u32_as_h2(rw[q]), __hmul2_rn(u32_as_h2(gw[q]), u32_as_h2(y)))
                                      : __hadd2_rn(u32_as_h2(rw[q]), u32_as_h2(y)));
                ow[q] = y;
            }
            *slot = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_2d(tmC, box, n0 + 16 * c, row0);
            bulk_commit();
        }
        ++e.n;
    }
    if (!ok && lane == 0) epi_drain(e);
    return ok;
}

// SwiGLU epilogue of a 256-wide tile whose weight rows hold gate features [f, f + 128) in columns 0..127 and the
// matching up features in columns 128..255 (rows interleaved in blocks of 128). Output box ob (16 features) pairs
// accumulator columns 16 ob (gate) and 128 + 16 ob (up): g and u are the epilogue's fp16 values, then
// fp16(fp16(g sigmoid(g)) u) with the same arithmetic as the pre-pass's SwiGLU, written as one 32 x 16 box of
// C[M, N/2] at feature column n0 / 2 + 16 ob; the EPI_SPLIT warps of a quarter take turns. The per-column scales
// come from the tile's staged columns.
__device__ __forceinline__ void epilogue_tile_swiglu(const GemmArgs& g, const CUtensorMap* tmC, EpiCtx& e,
                                                     uint32_t taddr, int row0, int n0, int part, const float* cw,
                                                     float sa) {
    const int lane = threadIdx.x & 31;
    const uint64_t sa2 = splat2(sa);
    const int sw = (lane >> 2) & 1;
#pragma unroll
    for (int i = 0; i < (8 + EPI_SPLIT - 1) / EPI_SPLIT; ++i) {
        const int ob = EPI_SPLIT * i + part;
        if (ob >= 8) break;
        float wg[16], wu[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            *reinterpret_cast<float4*>(wg + 4 * j) = reinterpret_cast<const float4*>(cw + 16 * ob)[j];
            *reinterpret_cast<float4*>(wu + 4 * j) = reinterpret_cast<const float4*>(cw + 128 + 16 * ob)[j];
        }
        unsigned char* box = e.buf + (e.n % EPI_BUFS) * EPI_BUF_BYTES;
        if (lane == 0) bulk_wait_read<EPI_BUFS - 1>();
        __syncwarp();
        uint32_t rg[16], ru[16];
        tmem_ld16_wait(taddr + 16 * ob, rg);
        tmem_ld16_wait(taddr + 128 + 16 * ob, ru);
        unsigned char* row = box + lane * 32;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            uint4 o;
            uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int k = 8 * j + 2 * q;
                const uint32_t gh = f2_to_h2(mul2(mul2(pk2((float)(int32_t)rg[k], (float)(int32_t)rg[k + 1]), sa2),
                                                  pk2(wg[k], wg[k + 1])));
                const uint32_t uh = f2_to_h2(mul2(mul2(pk2((float)(int32_t)ru[k], (float)(int32_t)ru[k + 1]), sa2),
                                                  pk2(wu[k], wu[k + 1])));
                ow[q] = swiglu_h2(gh, uh);
            }
            *reinterpret_cast<uint4*>(row + ((j ^ sw) << 4)) = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_2d(tmC, box, n0 / 2 + 16 * ob, row0);
            bulk_commit();
        }
        ++e.n;
    }
}

template <int BN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_w8a8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR, const GemmArgs g) {
    using C_ = Cfg<BN>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* staging = smem + C_::STAGES * C_::STAGE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + EPI_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + C_::STAGES;
    uint64_t* tfull = bars + 2 * C_::STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint64_t* rbars = drain + 1;  // [EPI_WARPS][EPI_BUFS]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbars + EPI_WARPS * EPI_BUFS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_m = (g.M + BM - 1) / BM, num_n = (g.N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int KB = (g.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C_::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 32 * EPI_WARPS);
        }
        mbar_init(drain, 1);
        for (int i = 0; i < EPI_WARPS * EPI_BUFS; ++i) mbar_init(&rbars[i], 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C_::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // the operands may come from the kernel launched before this one

    if (warp == 0) {
        if (lane == 0) {
            const uint64_t keep = l2_policy_evict_last();
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;  // bit s: stage s has a load in flight that nobody consumed yet (for draining)
            uint32_t issued_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const int m0 = (tile % num_m) * BM, n0 = (tile / num_m) * BN;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, &g_status, B2_DEV_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    unsigned char* sa = smem + stage * C_::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[stage], C_::STAGE_BYTES);
                    tma_load_2d(sa, &tmA, &full[stage], kb * BK, m0);
                    tma_load_2d_hint(sa + C_::A_BYTES, &tmB, &full[stage], kb * BK, n0, keep);
                    issued |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == C_::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok) {
                // Let every copy this thread started land before the CTA leaves.
                for (int s = 0; s < C_::STAGES; ++s)
                    if (issued & (1u << s))
                        if (!mbar_wait_drain(&full[s], (issued_phase >> s) & 1, 100000000ull))
                            atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_make(2, 1, 0, 0, BM, BN);  // S32 <- INT8 x INT8, both K-major
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int it = 0;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
                const int acc = it & 1;
                const uint32_t acc_phase = (it >> 1) & 1;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * C_::ACC_STRIDE;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * C_::STAGE_BYTES);
                    const uint64_t a_desc = sdesc_sw128(a_addr, 16, 1024);
                    const uint64_t b_desc = sdesc_sw128(a_addr + C_::A_BYTES, 16, 1024);
#pragma unroll
                    for (int k = 0; k < BK / 32; ++k)
                        mma_i8_ss(d_tmem, a_desc + (uint64_t)(k * 2), b_desc + (uint64_t)(k * 2), idesc,
                                  (kb | k) != 0);
                    tc_commit(&empty[stage]);
                    if (++stage == C_::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                tc_commit(&tfull[acc]);
            }
            // Every MMA issued above completes before TMEM is released.
            tc_commit(drain);
            if (!mbar_wait_drain(drain, 0, 100000000ull)) atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
        }
    } else {
        const int ew = warp - 2, quarter = warp & 3, part = ew >> 2;  // part: the warp's turn within its quarter
        const int row_local = quarter * 32 + lane;
        EpiCtx e{staging + ew * EPI_WARP_BYTES, rbars + ew * EPI_BUFS, 0u, 0u};
        float* cw = reinterpret_cast<float*>(staging + EPI_BYTES + C_::BAR_BYTES);
        float* cb = cw + BN;
        bool ok = true;
        int it = 0;
        // Every epilogue thread passes both named barriers of every tile, after a failed wait too, so that none is
        // left waiting at one.
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
            const int acc = it & 1;
            const uint32_t acc_phase = (it >> 1) & 1;
            const int m0 = (tile % num_m) * BM, n0 = (tile / num_m) * BN;
            named_bar_sync(1, 32 * EPI_WARPS);  // the epilogue warps are done with the previous tile's columns
            if (ok) epi_stage_cols<BN>(g, cw, cb, n0, threadIdx.x - 64);
            named_bar_sync(1, 32 * EPI_WARPS);
            if (!ok) continue;
            const float sa = (g.as && m0 + row_local < g.M) ? g.as[m0 + row_local] : 0.f;
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, &g_status, B2_DEV_TIMEOUT_EPILOGUE)) {
                ok = false;
                continue;
            }
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * C_::ACC_STRIDE;
            if (g.C32) {
                const int m = m0 + row_local;
                const bool row_ok = m < g.M;
#pragma unroll 1
                for (int c = part; c < BN / 32; c += EPI_SPLIT) epilogue_chunk_i32(g, taddr + c * 32, m, row_ok, n0 + c * 32);
            } else if (BN == 256 && g.swiglu) {
                epilogue_tile_swiglu(g, &tmC, e, taddr, m0 + quarter * 32, n0, part, cw, sa);
            } else {
                ok = epilogue_tile<BN / 16>(g, &tmC, &tmR, e, taddr, m0 + quarter * 32, n0, part, cw, cb, sa,
                                            abort_flag);
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
        }
        if (lane == 0) bulk_wait<0>();
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, C_::TMEM_COLS);
}


// ---------------------------------------------------------------- CTA-pair kernel
// Two CTAs of a cluster compute a 256 x 256 tile with cta_group::2 MMAs (M = 256, N = 256, K = 32): CTA r loads rows
// [128 r, 128 r + 128) of the A tile and of the B tile, the MMA issued by CTA 0 reads both CTAs' shared memory and
// writes each CTA's 128 accumulator rows x 256 columns into its own TMEM. Per SM this halves the B tile in shared
// memory (32 KB per k-block instead of 48 KB) for the same tensor work. Completion crosses the pair as ordinary
// barrier arrivals: TMA of both CTAs completes on CTA 0's full barrier, CTA 0's MMA commits to both CTAs' empty and
// tfull barriers, and both epilogues arrive on CTA 0's tempty barrier.
constexpr int PAIR_STAGES = 6;
constexpr int PAIR_HALF = 128 * BK;                    // 16 KB: 128 rows x 128 bytes
constexpr int PAIR_STAGE_BYTES = 2 * PAIR_HALF;        // A half + B half
constexpr int PAIR_SMEM = PAIR_STAGES * PAIR_STAGE_BYTES + EPI_BYTES + 512 + 256 * 8 + 1024;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    gemm_w8a8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR,
                          const GemmArgs g) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* staging = smem + PAIR_STAGES * PAIR_STAGE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + EPI_BYTES);
    uint64_t* full = bars;                      // [STAGES] (CTA 0)
    uint64_t* empty = bars + PAIR_STAGES;       // [STAGES] (each CTA)
    uint64_t* tfull = bars + 2 * PAIR_STAGES;   // [2] (each CTA)
    uint64_t* tempty = tfull + 2;               // [2] (CTA 0)
    uint64_t* drain = tempty + 2;
    uint64_t* rbars = drain + 1;                // [EPI_WARPS][EPI_BUFS] (each CTA)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbars + EPI_WARPS * EPI_BUFS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
    const int num_m = (g.M + 255) / 256, num_n = (g.N + 255) / 256;
    const int num_tiles = num_m * num_n;
    const int KB = (g.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < PAIR_STAGES; ++s) {
            mbar_init(&full[s], 2);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 2 * EPI_WARPS);  // one arrival per epilogue warp of each CTA
        }
        mbar_init(drain, 1);
        for (int i = 0; i < EPI_WARPS * EPI_BUFS; ++i) mbar_init(&rbars[i], 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before any remote arrival
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // the operands may come from the kernel launched before this one

    if (warp == 0) {
        if (lane == 0) {
            // Weights are re-read by every row tile and activations by every column tile: both stay in L2
            // (evict_last for the weights, the default for the activations).
            const uint64_t keep = l2_policy_evict_last(), normal = l2_policy_evict_normal();
            const uint32_t full0 = map_to_rank(smem_u32(full), 0);
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = cluster; tile < num_tiles; tile += nclusters) {
                const int m0 = (tile % num_m) * 256, n0 = (tile / num_m) * 256;
                bool ok = true;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, &g_status, B2_DEV_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    unsigned char* st = smem + stage * PAIR_STAGE_BYTES;
                    const uint32_t bar = full0 + stage * 8;
                    mbar_arrive_expect_tx_remote(bar, PAIR_STAGE_BYTES);
                    tma_load_2d_pair(st, &tmA, bar, kb * BK, m0 + 128 * rank, normal);
                    tma_load_2d_pair(st + PAIR_HALF, &tmB, bar, kb * BK, n0 + 128 * rank, keep);
                    if (++stage == PAIR_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_make(2, 1, 0, 0, 256, 256);
            const uint32_t empty_own = smem_u32(empty), empty_peer = map_to_rank(smem_u32(empty), 1);
            const uint32_t tfull_own = smem_u32(tfull), tfull_peer = map_to_rank(smem_u32(tfull), 1);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int it = 0;
            for (int tile = cluster; tile < num_tiles && ok; tile += nclusters, ++it) {
                const int acc = it & 1;
                const uint32_t acc_phase = (it >> 1) & 1;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * 256;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * PAIR_STAGE_BYTES);
                    const uint64_t a_desc = sdesc_sw128(a_addr, 16, 1024);
                    const uint64_t b_desc = sdesc_sw128(a_addr + PAIR_HALF, 16, 1024);
#pragma unroll
                    for (int k = 0; k < BK / 32; ++k)
                        mma_i8_ss_pair(d_tmem, a_desc + (uint64_t)(k * 2), b_desc + (uint64_t)(k * 2), idesc, (kb | k) != 0);
                    tc_commit_pair(empty_own + stage * 8);
                    tc_commit_pair(empty_peer + stage * 8);
                    if (++stage == PAIR_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                tc_commit_pair(tfull_own + acc * 8);
                tc_commit_pair(tfull_peer + acc * 8);
            }
            tc_commit_pair(smem_u32(drain));
            if (!mbar_wait_drain(drain, 0, 100000000ull)) atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
        }
    } else {
        const int ew = warp - 2, quarter = warp & 3, part = ew >> 2;  // part: the warp's turn within its quarter
        const int row_local = quarter * 32 + lane;
        const uint32_t tempty0 = map_to_rank(smem_u32(tempty), 0);
        EpiCtx e{staging + ew * EPI_WARP_BYTES, rbars + ew * EPI_BUFS, 0u, 0u};
        float* cw = reinterpret_cast<float*>(staging + EPI_BYTES + 512);
        float* cb = cw + 256;
        bool ok = true;
        int it = 0;
        // Every epilogue thread passes both named barriers of every tile, after a failed wait too.
        for (int tile = cluster; tile < num_tiles; tile += nclusters, ++it) {
            const int acc = it & 1;
            const uint32_t acc_phase = (it >> 1) & 1;
            const int m0 = (tile % num_m) * 256, n0 = (tile / num_m) * 256;
            named_bar_sync(1, 32 * EPI_WARPS);  // the epilogue warps are done with the previous tile's columns
            if (ok) epi_stage_cols<256>(g, cw, cb, n0, threadIdx.x - 64);
            named_bar_sync(1, 32 * EPI_WARPS);
            if (!ok) continue;
            const int mrow = m0 + 128 * rank + row_local;
            const float sa = (g.as && mrow < g.M) ? g.as[mrow] : 0.f;
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, &g_status, B2_DEV_TIMEOUT_EPILOGUE)) {
                ok = false;
                continue;
            }
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * 256;
            if (g.C32) {
                const int m = m0 + 128 * rank + row_local;
                const bool row_ok = m < g.M;
#pragma unroll 1
                for (int c = part; c < 8; c += EPI_SPLIT) epilogue_chunk_i32(g, taddr + c * 32, m, row_ok, n0 + c * 32);
            } else if (g.swiglu) {
                epilogue_tile_swiglu(g, &tmC, e, taddr, m0 + 128 * rank + quarter * 32, n0, part, cw, sa);
            } else {
                ok = epilogue_tile<16>(g, &tmC, &tmR, e, taddr, m0 + 128 * rank + quarter * 32, n0, part, cw, cb, sa,
                                       abort_flag);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(tempty0 + acc * 8);
        }
        if (lane == 0) bulk_wait<0>();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer's shared memory and barriers stay alive until the pair is done with them
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, 512);
}

// Launches a GEMM kernel with programmatic stream serialization: its CTAs may start (barrier set-up, TMEM
// allocation, descriptor prefetch) while the previous kernel of the stream finishes, and wait in pdl_wait() for its
// results.
template <class Kern>
int launch_pdl(Kern kernel, dim3 grid, int smem, cudaStream_t stream, const char* name, const CUtensorMap& ta,
               const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& tr, const GemmArgs& g) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, tr, g);
    if (e != cudaSuccess) return fail(B2_ERR_CUDA, "%s launch: %s", name, cudaGetErrorString(e));
    return check_launch(name);
}

// Output (and residual) maps: fp16 [M, N] row-major, 16-column x 32-row boxes with the 32-byte swizzle of the staging
// boxes.
// The raw int32 path stores from registers and gets the A map as a placeholder.
int make_out_maps(const GemmArgs& g, const CUtensorMap& fallback, CUtensorMap* tc, CUtensorMap* tr) {
    *tc = fallback;
    *tr = fallback;
    if (g.C32) return B2_OK;
    const int nc = g.swiglu ? g.N / 2 : g.N;
    if (int rc = make_map_2d(tc, g.C, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, nc, g.M, (uint64_t)nc * 2, 16, 32,
                             CU_TENSOR_MAP_SWIZZLE_32B))
        return rc;
    if (g.R)
        if (int rc = make_map_2d(tr, g.R, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, g.N, g.M, (uint64_t)g.N * 2, 16, 32,
                                 CU_TENSOR_MAP_SWIZZLE_32B))
            return rc;
    return B2_OK;
}

int launch_pair(const int8_t* A, const int8_t* B, const GemmArgs& g, cudaStream_t stream) {
    CUtensorMap ta, tb, tc, tr;
    if (int rc = make_map_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.K, g.M, g.K, BK, 128)) return rc;
    if (int rc = make_map_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.K, g.N, g.K, BK, 128)) return rc;
    if (int rc = make_out_maps(g, ta, &tc, &tr)) return rc;
    static int clusters[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !clusters[dev]) {
        if (int rc = set_smem(gemm_w8a8_pair_kernel, PAIR_SMEM)) return rc;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
        cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
        cfg.dynamicSmemBytes = PAIR_SMEM;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_w8a8_pair_kernel, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = sm_count() / 2;
        }
        clusters[dev] = n;
    }
    const int tiles = ((g.M + 255) / 256) * ((g.N + 255) / 256);
    const int nc = tiles < clusters[dev] ? tiles : clusters[dev];
    return launch_pdl(gemm_w8a8_pair_kernel, dim3(2 * nc), PAIR_SMEM, stream, "gemm_w8a8_pair_kernel", ta, tb, tc, tr, g);
}

template <int BN>
int launch_bn(const int8_t* A, const int8_t* B, const GemmArgs& g, cudaStream_t stream) {
    CUtensorMap ta, tb, tc, tr;
    if (int rc = make_map_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.K, g.M, g.K, BK, BM)) return rc;
    if (int rc = make_map_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.K, g.N, g.K, BK, BN)) return rc;
    if (int rc = make_out_maps(g, ta, &tc, &tr)) return rc;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (int rc = set_smem(gemm_w8a8_kernel<BN>, Cfg<BN>::SMEM)) return rc;
        configured[dev] = true;
    }
    const int tiles = ((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN);
    const int grid = tiles < sm_count() ? tiles : sm_count();
    return launch_pdl(gemm_w8a8_kernel<BN>, dim3(grid), Cfg<BN>::SMEM, stream, "gemm_w8a8_kernel", ta, tb, tc, tr, g);
}

int run(const int8_t* A, const int8_t* B, GemmArgs& g, cudaStream_t stream) {
    if (!A || !B) return fail(B2_ERR_INVALID, "gemm: null operand");
    if (g.M < 0 || g.N <= 0 || g.K <= 0) return fail(B2_ERR_INVALID, "gemm: bad shape M=%d N=%d K=%d", g.M, g.N, g.K);
    if (g.K % 16) return fail(B2_ERR_UNSUPPORTED, "gemm: K=%d must be a multiple of 16", g.K);
    if (g.N % 8) return fail(B2_ERR_UNSUPPORTED, "gemm: N=%d must be a multiple of 8", g.N);
    if (!aligned16(A) || !aligned16(B)) return fail(B2_ERR_UNSUPPORTED, "gemm: A and B must be 16-byte aligned");
    if (g.M == 0) return B2_OK;
    // CTA pairs on 256 x 256 tiles when they fill the machine; single-CTA tiles for small problems.
    // Otherwise the tile width with the least estimated time: waves of single-CTA tiles x tile width.
    auto cost = [&](int bn) {
        const int64_t tiles = (int64_t)((g.M + BM - 1) / BM) * ((g.N + bn - 1) / bn);
        return ((tiles + sm_count() - 1) / sm_count()) * bn;
    };
    if (g.M >= 256 && g.N >= 256 && ((g.M + 255) / 256) * ((g.N + 255) / 256) >= sm_count() / 2)
        return launch_pair(A, B, g, stream);
    if (g.swiglu) return launch_bn<256>(A, B, g, stream);  // the SwiGLU epilogue pairs the two halves of 256 columns
    const int64_t c128 = cost(128), c192 = cost(192), c256 = cost(256);
    if (c256 <= c192 && c256 <= c128) return launch_bn<256>(A, B, g, stream);
    if (c192 < c128) return launch_bn<192>(A, B, g, stream);
    return launch_bn<128>(A, B, g, stream);
}

}  // namespace

unsigned int read_status_gemm() {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    if (v) cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
    return v;
}

}  // namespace b2

using namespace b2;

extern "C" int b2_gemm(const int8_t* A, const int8_t* B, const float* as, const float* ws, const uint16_t* bias,
                       uint16_t* C, int M, int N, int K, const uint16_t* R, const uint16_t* G, int L, void* stream) {
    if (!as || !ws || !C) return fail(B2_ERR_INVALID, "gemm: null scale or output");
    if (G && (!R || L <= 0)) return fail(B2_ERR_INVALID, "gemm: a gate needs a residual and L > 0");
    if (!aligned16(C) || !aligned16(ws) || (bias && !aligned16(bias)) || (R && !aligned16(R)) || (G && !aligned16(G)))
        return fail(B2_ERR_UNSUPPORTED, "gemm: C, ws, bias, R, G must be 16-byte aligned");
    GemmArgs g{};
    g.as = as;
    g.ws = ws;
    g.bias = reinterpret_cast<const __half*>(bias);
    g.C = reinterpret_cast<__half*>(C);
    g.R = reinterpret_cast<const __half*>(R);
    g.G = reinterpret_cast<const __half*>(G);
    g.L = L > 0 ? L : 1;
    g.M = M;
    g.N = N;
    g.K = K;
    return run(A, B, g, (cudaStream_t)stream);
}

extern "C" int b2_gemm_swiglu(const int8_t* A, const int8_t* B, const float* as, const float* ws, uint16_t* C, int M,
                              int N, int K, void* stream) {
    if (!as || !ws || !C) return fail(B2_ERR_INVALID, "gemm_swiglu: null scale or output");
    if (N <= 0 || N % 256) return fail(B2_ERR_UNSUPPORTED, "gemm_swiglu: N=%d must be a multiple of 256", N);
    if (!aligned16(C) || !aligned16(ws)) return fail(B2_ERR_UNSUPPORTED, "gemm_swiglu: C and ws must be 16-byte aligned");
    GemmArgs g{};
    g.as = as;
    g.ws = ws;
    g.C = reinterpret_cast<__half*>(C);
    g.L = 1;
    g.M = M;
    g.N = N;
    g.K = K;
    g.swiglu = 1;
    return run(A, B, g, (cudaStream_t)stream);
}

extern "C" int b2_gemm_i32(const int8_t* A, const int8_t* B, int32_t* C32, int M, int N, int K, void* stream) {
    if (!C32) return fail(B2_ERR_INVALID, "gemm_i32: null output");
    if (!aligned16(C32)) return fail(B2_ERR_UNSUPPORTED, "gemm_i32: output must be 16-byte aligned");
    GemmArgs g{};
    g.C32 = C32;
    g.L = 1;
    g.M = M;
    g.N = N;
    g.K = K;
    return run(A, B, g, (cudaStream_t)stream);
}
