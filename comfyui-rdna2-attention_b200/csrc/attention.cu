// Fused attention for head dim 128 on sm_100a, fp16 QK or int8 QK, fp16 PV, fp32 softmax.
//
// Semantics follow hip_attention.hip:
//   fp16 (attn, :280-373): s = q.k (fp32 accumulate); log2-domain online softmax with c = scale*log2(e);
//     rows of a 32-row warp rescale together, and only when some row's block max exceeds m + 8 (:333-340);
//     p = exp2(s*c - m) rounded to fp16 for PV, l sums the fp32 p (:343-347); out = fp16(o * (1/l)).
//   int8 QK (pack_kv_i8 :56-103, attn_i8 :160-278): per-row q and per-key k scales max(|x|max/127, 1e-30),
//     values rint(x/scale) (half-even); s = ((float)int_dot * (qs*c)) * ks; p = exp2(s - m); PV stays fp16.
// Keys past Lk are masked (score -inf), queries past Lq are not stored.
//
// One CTA computes two 128-row Q tiles of one (batch, head) with two softmax warpgroups in ping-pong; S, P and O
// live in TMEM (P overwrites the consumed S columns and is the A operand of the PV MMA). V is the MN-major B operand
// of the PV MMA in its natural [keys][d] layout. See attention_kernel for the roles.
#include "common.cuh"
#include "host.hpp"

namespace b2 {
namespace {

__device__ unsigned int g_status;

constexpr int TQ = 128;   // query rows per tile; a CTA computes two tiles (A and B) of one (batch, head)
constexpr int TK = 128;   // keys per tile
constexpr int HD = 128;   // head dim
constexpr int ATT_THREADS = 576;  // TMA warp, MMA warp, 16 softmax warps
constexpr float LOG2E = 1.4426950408889634f;

template <bool I8>
struct AttCfg {
    static constexpr int Q_BYTES = I8 ? TQ * HD : TQ * HD * 2;  // per tile
    static constexpr int K_BYTES = I8 ? TK * HD : TK * HD * 2;
    static constexpr int V_BYTES = TK * HD * 2;
    static constexpr int KS_BYTES = I8 ? TK * 4 : 0;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;
    static constexpr int OFF_V = OFF_K + 2 * K_BYTES;
    static constexpr int OFF_KS = OFF_V + 2 * V_BYTES;
    static constexpr int OFF_RED = OFF_KS + 2 * KS_BYTES;  // row max halves [parity][tile][row][half], l halves
    static constexpr int RED_BYTES = 2 * 2 * TQ * 2 * 4 + 2 * TQ * 2 * 4;
    static constexpr int OFF_BAR = OFF_RED + RED_BYTES;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;
};

constexpr int MAX_PEERS = 7;

struct AttArgs {
    __half* out;
    int64_t sob, soh, sol;
    // Head-group gather: the same output tile also goes to these peers' buffers at the same offsets (their memory
    // mapped into this GPU's address space), and each finished CTA adds 1 to every peer's arrival counter.
    __half* peer_out[MAX_PEERS];
    unsigned long long* peer_cnt[MAX_PEERS];
    int npeer;
    const float* qscale;  // int8: [B*H, Lq]
    int Lq, Lk, H, rep;
    float scale_log2;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Meeting point of the two softmax warps that share 32 rows: an mbarrier of count 2 (one arrival per warp after
// __syncwarp, so the warp's shared-memory writes are ordered before it), waited with the bounded wait.
__device__ __forceinline__ bool pair_sync(uint64_t* bar, uint32_t parity, volatile int* abort) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
    return mbar_wait(bar, parity, abort, &g_status, B2_DEV_TIMEOUT_EPILOGUE);
}

// One CTA: 2 x 128 query rows of one (batch, head).
//   warp 0      TMA: both Q tiles once, then K/V tiles of 128 keys into a 2-deep ring
//   warp 1      TMEM owner and single-thread tcgen05.mma issuer. TMEM columns: S_A [0,128), S_B [128,256),
//               O_A [256,384), O_B [384,512). Issue order per key tile j:
//                 PV_A(j-1) ... S_A(j) ... PV_B(j-1) ... S_B(j)
//               so the softmax of tile A on S_A(j) overlaps the tensor work for tile B and vice versa.
//   warps 2..9  softmax of tile A, warps 10..17 softmax of tile B. A warp owns 32 query rows (its TMEM lane
//               quarter, thread = row) and one half of the 128 key columns; its partner (4 warps away) owns the
//               other half of the same rows. Two passes over the half (row max, then p = exp2); the two halves'
//               maxima meet through shared memory and a 64-thread barrier, so both take the same rescale decision.
//               P is written back as fp16 into the half's consumed S columns, where the PV MMA reads it as its A
//               operand (TMEM); lazy, warp-uniform rescale of the half's O columns in TMEM.
template <bool I8>
__global__ void __launch_bounds__(ATT_THREADS, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKS, const AttArgs a) {
    using C_ = AttCfg<I8>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C_::OFF_BAR);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;   // [2] stages
    uint64_t* v_full = bars + 3;   // [2]
    uint64_t* k_empty = bars + 5;  // [2]
    uint64_t* v_empty = bars + 7;  // [2]
    uint64_t* s_full = bars + 9;   // [2] tiles A, B
    uint64_t* p_full = bars + 11;  // [2]
    uint64_t* o_done = bars + 13;  // [2]
    uint64_t* drain = bars + 15;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
    uint64_t* pair_bar = bars + 17;  // [2 tiles][4 quarters]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * (2 * TQ);
    const int bh = blockIdx.y;
    const int b = bh / a.H, h = bh % a.H;
    const int hkv = h / a.rep;
    const int bkv = b * (a.H / a.rep) + hkv;
    const int n_tiles = (a.Lk + TK - 1) / TK;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&v_full[i], 1);
            // int8: the key scales in the K stage are read by both softmax warpgroups too.
            mbar_init(&k_empty[i], I8 ? 1 + 16 : 1);  // MMA commit (+ one arrival per softmax warp)
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 8);  // one arrival per softmax warp of the tile
            mbar_init(&o_done[i], 1);
        }
        mbar_init(drain, 1);
        for (int i = 0; i < 8; ++i) mbar_init(&pair_bar[i], 2);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        if (I8) tma_prefetch_desc(&tmKS);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    unsigned char* sQ = smem + C_::OFF_Q;
    unsigned char* sK = smem + C_::OFF_K;
    unsigned char* sV = smem + C_::OFF_V;
    float* sKS = reinterpret_cast<float*>(smem + C_::OFF_KS);

    if (warp == 0) {
        if (lane == 0) {
            uint32_t k_issued = 0, v_issued = 0, k_ph = 0, v_ph = 0;
            bool ok = true;
            mbar_arrive_expect_tx(q_full, 2 * C_::Q_BYTES);
            for (int t = 0; t < 2; ++t) {
                unsigned char* dst = sQ + t * C_::Q_BYTES;
                if (I8) {
                    tma_load_3d(dst, &tmQ, q_full, 0, q0 + t * TQ, bh);
                } else {
                    tma_load_4d(dst, &tmQ, q_full, 0, q0 + t * TQ, h, b);
                    tma_load_4d(dst + TQ * 128, &tmQ, q_full, 64, q0 + t * TQ, h, b);
                }
            }
            auto load_k = [&](int j) -> bool {
                const int st = j & 1;
                if (!mbar_wait(&k_empty[st], ((j >> 1) & 1) ^ 1, abort_flag, &g_status, B2_DEV_TIMEOUT_PRODUCER)) return false;
                mbar_arrive_expect_tx(&k_full[st], C_::K_BYTES + C_::KS_BYTES);
                unsigned char* dst = sK + st * C_::K_BYTES;
                if (I8) {
                    tma_load_3d(dst, &tmK, &k_full[st], 0, j * TK, bkv);
                    tma_load_2d(sKS + st * TK, &tmKS, &k_full[st], j * TK, bkv);
                } else {
                    tma_load_4d(dst, &tmK, &k_full[st], 0, j * TK, hkv, b);
                    tma_load_4d(dst + TK * 128, &tmK, &k_full[st], 64, j * TK, hkv, b);
                }
                k_issued |= 1u << st;
                k_ph = (k_ph & ~(1u << st)) | (((j >> 1) & 1u) << st);
                return true;
            };
            auto load_v = [&](int j) -> bool {
                const int st = j & 1;
                if (!mbar_wait(&v_empty[st], ((j >> 1) & 1) ^ 1, abort_flag, &g_status, B2_DEV_TIMEOUT_PRODUCER)) return false;
                mbar_arrive_expect_tx(&v_full[st], C_::V_BYTES);
                unsigned char* dst = sV + st * C_::V_BYTES;
                tma_load_4d(dst, &tmV, &v_full[st], 0, j * TK, hkv, b);
                tma_load_4d(dst + TK * 128, &tmV, &v_full[st], 64, j * TK, hkv, b);
                v_issued |= 1u << st;
                v_ph = (v_ph & ~(1u << st)) | (((j >> 1) & 1u) << st);
                return true;
            };
            ok = load_k(0);
            for (int j = 0; j < n_tiles && ok; ++j) {
                if (j + 1 < n_tiles && !load_k(j + 1)) ok = false;
                if (ok && !load_v(j)) ok = false;
            }
            if (!ok) {
                mbar_wait_drain(q_full, 0, 100000000ull);
                for (int s = 0; s < 2; ++s) {
                    if ((k_issued >> s) & 1)
                        if (!mbar_wait_drain(&k_full[s], (k_ph >> s) & 1, 100000000ull)) atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
                    if ((v_issued >> s) & 1)
                        if (!mbar_wait_drain(&v_full[s], (v_ph >> s) & 1, 100000000ull)) atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_qk = I8 ? idesc_make(2, 1, 0, 0, TQ, TK) : idesc_make(1, 0, 0, 0, TQ, TK);
            constexpr uint32_t idesc_pv = idesc_make(1, 0, 0, 1, TQ, HD);
            const uint32_t q_addr = smem_u32(sQ);
            auto issue_s = [&](int t, int j) {
                const uint32_t k_addr = smem_u32(sK + (j & 1) * C_::K_BYTES);
                const uint32_t qa = q_addr + t * C_::Q_BYTES;
                const uint32_t d = tmem + t * TK;
                if (I8) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_i8_ss(d, sdesc_sw128(qa + kk * 32, 16, 1024), sdesc_sw128(k_addr + kk * 32, 16, 1024), idesc_qk,
                                  kk != 0);
                } else {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t off = (kk >> 2) * (TQ * 128) + (kk & 3) * 32;
                        mma_f16_ss(d, sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(k_addr + off, 16, 1024), idesc_qk,
                                   kk != 0);
                    }
                }
                tc_commit(&s_full[t]);
            };
            auto issue_pv = [&](int t, int j) {
                const uint32_t v_addr = smem_u32(sV + (j & 1) * C_::V_BYTES);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    // P of keys [64 h, 64 h + 64) sits in columns [64 h, 64 h + 32) of the tile's S region
                    mma_f16_ts(tmem + 256 + t * HD, tmem + t * TK + 64 * (kk >> 2) + 8 * (kk & 3),
                               sdesc_sw128(v_addr + kk * 2048, TK * 128, 1024),
                               idesc_pv, (j | kk) != 0);
                tc_commit(&o_done[t]);
            };
            bool ok = mbar_wait(q_full, 0, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA) &&
                      mbar_wait(&k_full[0], 0, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA);
            if (ok) {
                tc_fence_after();
                issue_s(0, 0);
                issue_s(1, 0);
                tc_commit(&k_empty[0]);
            }
            for (int j = 0; j < n_tiles && ok; ++j) {
                const int st = j & 1;
                if (!mbar_wait(&p_full[0], j & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA) ||
                    !mbar_wait(&v_full[st], (j >> 1) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA))
                    break;
                tc_fence_after();
                issue_pv(0, j);
                const bool more = j + 1 < n_tiles;
                if (more) {
                    if (!mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA)) break;
                    tc_fence_after();
                    issue_s(0, j + 1);
                }
                if (!mbar_wait(&p_full[1], j & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA)) break;
                tc_fence_after();
                issue_pv(1, j);
                tc_commit(&v_empty[st]);
                if (more) {
                    issue_s(1, j + 1);
                    tc_commit(&k_empty[(j + 1) & 1]);
                }
            }
            tc_commit(drain);
            if (!mbar_wait_drain(drain, 0, 100000000ull)) atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
        }
    } else {
        // Softmax: tile t, key half hh, lane quarter (TMEM lanes 32 quarter .. + 31); thread -> query row r.
        const int sw = warp - 2;
        const int t = sw >> 3, hh = (sw >> 2) & 1;
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        uint64_t* pbar = &pair_bar[t * 4 + quarter];
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const uint32_t tS = tmem + lane_base + t * TK + 64 * hh;  // this half's 64 score columns
        const uint32_t tO = tmem + lane_base + 256 + t * HD + 64 * hh;  // this half's 64 output columns
        const int qrow = q0 + t * TQ + r;
        float* red = reinterpret_cast<float*>(smem + C_::OFF_RED);  // [2][2][TQ][2] maxima, then [2][TQ][2] sums
        float m = -1e30f, l = 0.f;
        float qs_c = 0.f;
        if (I8) qs_c = __fmul_rn(a.qscale[(int64_t)bh * a.Lq + min(qrow, a.Lq - 1)], a.scale_log2);
        bool ok = true;
        for (int j = 0; j < n_tiles; ++j) {
            if (!mbar_wait(&s_full[t], j & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_EPILOGUE)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int valid = a.Lk - j * TK - 64 * hh;  // valid keys of this half (may be <= 0 or >= 64)
            const float* ks = sKS + (j & 1) * TK + 64 * hh;
            const bool full = valid >= 64;
            // Pass 1: the half's row max, four independent chains. int8 scores are exact small integers
            // (|dot| < 2^22) that become fp32 without the conversion pipe and are scaled by q_scale * c and
            // k_scale (hip_attention.hip:238-246); they go back to TMEM as fp32 for pass 2. fp16 scores enter the
            // log2 domain after the max (the scale is applied to the max).
            float mm[4] = {-1e30f, -1e30f, -1e30f, -1e30f};
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t v[32];
                tmem_ld32_wait(tS + c * 32, v);
                if (I8) {
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float2 k2 = *reinterpret_cast<const float2*>(ks + c * 32 + i);
                        const float2 y = upk2(mul2(mul2(pk2(small_i2f(v[i]), small_i2f(v[i + 1])), pk2(qs_c, qs_c)),
                                                   pk2(k2.x, k2.y)));
                        v[i] = __float_as_uint(y.x);
                        v[i + 1] = __float_as_uint(y.y);
                    }
                    tmem_st32(tS + c * 32, v);
                }
                if (full) {
#pragma unroll
                    for (int i = 0; i < 32; i += 8)
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            mm[q] = max3(mm[q], __uint_as_float(v[i + 2 * q]), __uint_as_float(v[i + 2 * q + 1]));
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c * 32 + i < valid) mm[i & 3] = fmaxf(mm[i & 3], __uint_as_float(v[i]));
                }
            }
            if (I8) {
                tmem_wait_st();
                __syncwarp();
                if (lane == 0) mbar_arrive(&k_empty[j & 1]);  // the key scales of this stage are consumed
            }
            // The two halves' maxima meet (slot by tile parity, so a fast warp never overwrites a slot its partner
            // still reads).
            float* rm = red + (((j & 1) * 2 + t) * TQ + r) * 2;
            rm[hh] = max3(mm[0], mm[1], fmaxf(mm[2], mm[3]));
            if (!pair_sync(pbar, j & 1, abort_flag)) {
                ok = false;
                break;
            }
            float mx = fmaxf(rm[0], rm[1]);
            if (!I8) mx *= a.scale_log2;
            if (__any_sync(0xffffffffu, mx > m + 8.f)) {
                const float mn = fmaxf(m, mx);
                const float alpha = ex2(m - mn);
                m = mn;
                l *= alpha;
                if (j > 0) {
                    // O holds PV of the previous tiles; it must be complete before it is rescaled.
                    if (!mbar_wait(&o_done[t], (j - 1) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_EPILOGUE)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < 2; ++c) {
                        uint32_t o[32];
                        tmem_ld32_wait(tO + c * 32, o);
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(tO + c * 32, o);
                    }
                }
            }
            // Pass 2: p = exp2(s*c - m) (fp16 path) or exp2(s - m) (int8); l sums the fp32 p (two running partial
            // sums); P (fp16 pairs) goes into the half's columns already read: 32 scores -> columns [16c, 16c + 16).
            const uint64_t c2 = I8 ? pk2(1.f, 1.f) : pk2(a.scale_log2, a.scale_log2);
            const uint64_t nm2 = pk2(-m, -m);
            uint64_t l2 = pk2(0.f, 0.f);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t v[32], pk[16];
                tmem_ld32_wait(tS + c * 32, v);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int col = c * 32 + 2 * i;
                    const float2 e = upk2(fma2(pk2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])), c2, nm2));
                    float p0 = ex2(e.x), p1 = ex2(e.y);
                    if (!full) {
                        if (col >= valid) p0 = 0.f;
                        if (col + 1 >= valid) p1 = 0.f;
                    }
                    l2 = add2(l2, pk2(p0, p1));
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    pk[i] = *reinterpret_cast<const uint32_t*>(&hp);
                }
                tmem_st16(tS + c * 16, pk);
            }
            {
                const float2 lf = upk2(l2);
                l += lf.x + lf.y;
            }
            // Every lane's P stores complete before the warp's single arrival (serialized arrivals of 256 threads on
            // one barrier cost more than the whole handshake otherwise).
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t]);
        }
        // The row sum is the two halves' sums (half 0 first in both warps, so both use the same l).
        float* rl = red + 2 * 2 * TQ * 2 + (t * TQ + r) * 2;
        rl[hh] = l;
        if (ok) ok = pair_sync(pbar, n_tiles & 1, abort_flag);
        l = rl[0] + rl[1];
        if (ok && mbar_wait(&o_done[t], (n_tiles - 1) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_EPILOGUE)) {
            tc_fence_after();
            const float inv = 1.f / l;
            const bool row_ok = qrow < a.Lq;
            __half* dst = a.out + (int64_t)b * a.sob + (int64_t)h * a.soh + (int64_t)qrow * a.sol + 64 * hh;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                uint32_t o[32];
                tmem_ld32_wait(tO + c * 32, o);
                if (row_ok) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        uint4 u;
                        __half2* hu = reinterpret_cast<__half2*>(&u);
#pragma unroll
                        for (int z = 0; z < 4; ++z)
                            hu[z] = __floats2half2_rn(__uint_as_float(o[8 * e + 2 * z]) * inv,
                                                      __uint_as_float(o[8 * e + 2 * z + 1]) * inv);
                        *reinterpret_cast<uint4*>(dst + c * 32 + 8 * e) = u;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
    if (a.npeer) {
        // The CTA's finished output tile (its 2 TQ rows x 256 bytes of head h) to every peer of the head group:
        // coalesced plain stores (16 threads per row), read back from this GPU's L2, while other CTAs compute.
        const int rows = min(2 * TQ, a.Lq - q0);
        const __half* src0 = a.out + (int64_t)b * a.sob + (int64_t)h * a.soh + (int64_t)q0 * a.sol;
        for (int i = threadIdx.x; i < rows * 16; i += blockDim.x) {
            const int64_t off = (int64_t)(i >> 4) * a.sol + (i & 15) * 8;
            const uint4 u = __ldcg(reinterpret_cast<const uint4*>(src0 + off));
            for (int p = 0; p < a.npeer; ++p) *reinterpret_cast<uint4*>(a.peer_out[p] + (src0 - a.out) + off) = u;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            // The barrier orders every thread's peer stores before this system-scope fence; the arrivals follow it.
            __threadfence_system();
            for (int p = 0; p < a.npeer; ++p) atomicAdd_system(a.peer_cnt[p], 1ull);
        }
    }
}

// One thread waits until *cnt >= expected (acquire loads at system scope), sleeping between polls, for at most
// timeout_ns; if the count is not reached by then it sets *err and returns, so the stream moves on and the host reads
// the failure instead of a hung GPU.
__global__ void wait_count_kernel(const unsigned long long* cnt, unsigned long long expected, unsigned int* err,
                                  long long timeout_ns) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const uint64_t t0 = global_timer();
    for (;;) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(cnt) : "memory");
        if (v >= expected) return;
        if ((long long)(global_timer() - t0) > timeout_ns) {
            atomicOr(err, 1u);
            return;
        }
        __nanosleep(256);
    }
}

// Per-row int8 quantization of Q or K rows of 128 values (hip_attention.hip:67-93, :172-194):
// scale = max(absmax / 127, 1e-30), q = rint(x / scale). 16 threads per row, 8 values each.
__global__ void __launch_bounds__(256) quant_rows_i8_kernel(const __half* __restrict__ x, int64_t sb, int64_t sh,
                                                           int64_t sl, int H, int L, int rows, int8_t* __restrict__ q,
                                                           float* __restrict__ scale, int64_t scale_ld) {
    const int n = blockIdx.x * 16 + (threadIdx.x >> 4);
    const int t = threadIdx.x & 15;
    const bool valid = n < rows;
    const int nn = valid ? n : rows - 1;
    const int l = nn % L, bh = nn / L, h = bh % H, b = bh / H;
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + b * sb + h * sh + (int64_t)l * sl) + t);
    const __half2* hv = reinterpret_cast<const __half2*>(&raw);
    float f[8];
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = __half22float2(hv[i]);
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
        mx = fmaxf(mx, fmaxf(fabsf(v.x), fabsf(v.y)));
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o, 16));
    const float s = fmaxf(__fdiv_rn(mx, 127.f), 1e-30f);
    if (!valid) return;
    uint32_t w[2];
#pragma unroll
    for (int d = 0; d < 2; ++d) {
        uint32_t acc = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int v = (int)fminf(fmaxf(rintf(__fdiv_rn(f[4 * d + i], s)), -128.f), 127.f);
            acc |= (uint32_t)(v & 255) << (8 * i);
        }
        w[d] = acc;
    }
    *reinterpret_cast<uint2*>(q + (int64_t)n * HD + t * 8) = make_uint2(w[0], w[1]);
    if (t == 0) scale[(int64_t)bh * scale_ld + l] = s;
}

struct Views {
    const void* p;
    int64_t sb, sh, sl;
};

inline int64_t rup(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

struct I8Layout {
    int64_t q_off, k_off, qs_off, ks_off, total, ks_ld;
};

I8Layout i8_layout(int B, int H, int Hkv, int Lq, int Lk) {
    I8Layout o;
    o.ks_ld = rup(Lk, 4);
    o.q_off = 0;
    o.k_off = rup(o.q_off + (int64_t)B * H * Lq * HD, 1024);
    o.qs_off = rup(o.k_off + (int64_t)B * Hkv * Lk * HD, 1024);
    o.ks_off = rup(o.qs_off + (int64_t)B * H * Lq * 4, 1024);
    o.total = rup(o.ks_off + (int64_t)B * Hkv * o.ks_ld * 4, 1024);
    return o;
}

int map_heads(CUtensorMap* m, const Views& v, int B, int H, int L) {
    const uint64_t dims[4] = {(uint64_t)HD, (uint64_t)L, (uint64_t)H, (uint64_t)B};
    const uint64_t strides[3] = {(uint64_t)v.sl * 2, (uint64_t)v.sh * 2, (uint64_t)v.sb * 2};
    const uint32_t box[4] = {64, 128, 1, 1};
    return make_map_4d(m, v.p, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dims, strides, box);
}

int map_rows_i8(CUtensorMap* m, const void* base, int64_t rows_per_head, int heads) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(B2_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t d3[3] = {(cuuint64_t)HD, (cuuint64_t)rows_per_head, (cuuint64_t)heads};
    cuuint64_t s3[2] = {(cuuint64_t)HD, (cuuint64_t)rows_per_head * HD};
    cuuint32_t b3[3] = {128, 128, 1};
    cuuint32_t e3[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), d3, s3, b3, e3,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(B2_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled(3d int8) failed with %d", (int)r);
    return B2_OK;
}

template <bool I8>
int launch_attention(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tks,
                     const AttArgs& a, int B, cudaStream_t s) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (int rc = set_smem(attention_kernel<I8>, AttCfg<I8>::SMEM)) return rc;
        configured[dev] = true;
    }
    dim3 grid((a.Lq + 2 * TQ - 1) / (2 * TQ), B * a.H);
    attention_kernel<I8><<<grid, ATT_THREADS, AttCfg<I8>::SMEM, s>>>(tq, tk, tv, tks, a);
    return check_launch("attention_kernel");
}

}  // namespace

unsigned int read_status_attention() {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    if (v) cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
    return v;
}

}  // namespace b2

using namespace b2;

extern "C" int64_t b2_attention_workspace_bytes(int B, int H, int Hkv, int Lq, int Lk, int int8_qk) {
    if (!int8_qk) return 0;
    if (B <= 0 || H <= 0 || Hkv <= 0 || Lq <= 0 || Lk <= 0) return 0;
    return i8_layout(B, H, Hkv, Lq, Lk).total;
}

namespace b2 {
namespace {
int attention_impl(const uint16_t* q, int64_t sqb, int64_t sqh, int64_t sql, const uint16_t* k, int64_t skb,
                   int64_t skh, int64_t skl, const uint16_t* v, int64_t svb, int64_t svh, int64_t svl, uint16_t* out,
                   int64_t sob, int64_t soh, int64_t sol, int B, int H, int Hkv, int Lq, int Lk, float scale,
                   int int8_qk, void* workspace, int64_t workspace_bytes, uint16_t* const* peer_out,
                   unsigned long long* const* peer_cnt, int npeer, void* stream);
}  // namespace
}  // namespace b2

extern "C" int b2_attention(const uint16_t* q, int64_t sqb, int64_t sqh, int64_t sql, const uint16_t* k, int64_t skb,
                            int64_t skh, int64_t skl, const uint16_t* v, int64_t svb, int64_t svh, int64_t svl,
                            uint16_t* out, int64_t sob, int64_t soh, int64_t sol, int B, int H, int Hkv, int Lq, int Lk,
                            float scale, int int8_qk, void* workspace, int64_t workspace_bytes, void* stream) {
    return attention_impl(q, sqb, sqh, sql, k, skb, skh, skl, v, svb, svh, svl, out, sob, soh, sol, B, H, Hkv, Lq, Lk,
                          scale, int8_qk, workspace, workspace_bytes, nullptr, nullptr, 0, stream);
}

extern "C" int b2_attention_gather(const uint16_t* q, int64_t sqb, int64_t sqh, int64_t sql, const uint16_t* k,
                                   int64_t skb, int64_t skh, int64_t skl, const uint16_t* v, int64_t svb, int64_t svh,
                                   int64_t svl, uint16_t* out, int64_t sob, int64_t soh, int64_t sol, int B, int H,
                                   int Hkv, int Lq, int Lk, float scale, int int8_qk, void* workspace,
                                   int64_t workspace_bytes, uint16_t* const* peer_out,
                                   unsigned long long* const* peer_cnt, int npeer, void* stream) {
    if (npeer < 0 || npeer > MAX_PEERS) return fail(B2_ERR_UNSUPPORTED, "attention_gather: %d peers (at most %d)", npeer, MAX_PEERS);
    if (npeer && (!peer_out || !peer_cnt)) return fail(B2_ERR_INVALID, "attention_gather: null peer arrays");
    return attention_impl(q, sqb, sqh, sql, k, skb, skh, skl, v, svb, svh, svl, out, sob, soh, sol, B, H, Hkv, Lq, Lk,
                          scale, int8_qk, workspace, workspace_bytes, peer_out, peer_cnt, npeer, stream);
}

extern "C" int b2_attention_gather_ctas(int B, int H, int Lq) {
    if (B <= 0 || H <= 0 || Lq <= 0) return 0;
    return ((Lq + 2 * TQ - 1) / (2 * TQ)) * B * H;
}

extern "C" int b2_wait_count(const unsigned long long* cnt, unsigned long long expected, unsigned int* err,
                             long long timeout_ns, void* stream) {
    if (!cnt || !err || timeout_ns <= 0) return fail(B2_ERR_INVALID, "wait_count: bad arguments");
    wait_count_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(cnt, expected, err, timeout_ns);
    return check_launch("wait_count_kernel");
}

namespace b2 {
namespace {
int attention_impl(const uint16_t* q, int64_t sqb, int64_t sqh, int64_t sql, const uint16_t* k, int64_t skb,
                   int64_t skh, int64_t skl, const uint16_t* v, int64_t svb, int64_t svh, int64_t svl, uint16_t* out,
                   int64_t sob, int64_t soh, int64_t sol, int B, int H, int Hkv, int Lq, int Lk, float scale,
                   int int8_qk, void* workspace, int64_t workspace_bytes, uint16_t* const* peer_out,
                   unsigned long long* const* peer_cnt, int npeer, void* stream) {
    if (!q || !k || !v || !out) return fail(B2_ERR_INVALID, "attention: null pointer");
    if (B < 0 || H <= 0 || Hkv <= 0 || Lq < 0 || Lk <= 0 || H % Hkv)
        return fail(B2_ERR_INVALID, "attention: bad shape B=%d H=%d Hkv=%d Lq=%d Lk=%d", B, H, Hkv, Lq, Lk);
    if (!aligned16(out) || (sob * 2) % 16 || (soh * 2) % 16 || (sol * 2) % 16)
        return fail(B2_ERR_UNSUPPORTED, "attention: out must be 16-byte aligned with 16-byte strides");
    if (B == 0 || Lq == 0) return B2_OK;
    cudaStream_t s = (cudaStream_t)stream;
    AttArgs a{};
    a.out = reinterpret_cast<__half*>(out);
    a.sob = sob;
    a.soh = soh;
    a.sol = sol;
    a.Lq = Lq;
    a.Lk = Lk;
    a.H = H;
    a.rep = H / Hkv;
    a.scale_log2 = scale * LOG2E;
    for (int i = 0; i < npeer; ++i) {
        if (!peer_out[i] || !peer_cnt[i] || !aligned16(peer_out[i]))
            return fail(B2_ERR_INVALID, "attention_gather: peer %d buffer or counter", i);
        a.peer_out[i] = reinterpret_cast<__half*>(peer_out[i]);
        a.peer_cnt[i] = peer_cnt[i];
    }
    a.npeer = npeer;
    CUtensorMap tq, tk, tv, tks;
    const Views vq{q, sqb, sqh, sql}, vk{k, skb, skh, skl}, vv{v, svb, svh, svl};
    if (int rc = map_heads(&tv, vv, B, Hkv, Lk)) return rc;
    if (!int8_qk) {
        if (int rc = map_heads(&tq, vq, B, H, Lq)) return rc;
        if (int rc = map_heads(&tk, vk, B, Hkv, Lk)) return rc;
        tks = tk;
        return launch_attention<false>(tq, tk, tv, tks, a, B, s);
    }
    const I8Layout lay = i8_layout(B, H, Hkv, Lq, Lk);
    if (!workspace || workspace_bytes < lay.total)
        return fail(B2_ERR_INVALID, "attention: int8 QK needs %lld bytes of workspace", (long long)lay.total);
    if (!aligned16(workspace)) return fail(B2_ERR_UNSUPPORTED, "attention: workspace must be 16-byte aligned");
    if (!aligned16(q) || !aligned16(k) || (sqb | sqh | sql | skb | skh | skl) % 8)
        return fail(B2_ERR_UNSUPPORTED, "attention: q and k must be 16-byte aligned with 16-byte strides");
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    int8_t* q8 = reinterpret_cast<int8_t*>(ws + lay.q_off);
    int8_t* k8 = reinterpret_cast<int8_t*>(ws + lay.k_off);
    float* qs = reinterpret_cast<float*>(ws + lay.qs_off);
    float* ks = reinterpret_cast<float*>(ws + lay.ks_off);
    const int qrows = B * H * Lq, krows = B * Hkv * Lk;
    quant_rows_i8_kernel<<<(qrows + 15) / 16, 256, 0, s>>>(reinterpret_cast<const __half*>(q), sqb, sqh, sql, H, Lq, qrows,
                                                          q8, qs, Lq);
    if (int rc = check_launch("quant_rows_i8_kernel(q)")) return rc;
    quant_rows_i8_kernel<<<(krows + 15) / 16, 256, 0, s>>>(reinterpret_cast<const __half*>(k), skb, skh, skl, Hkv, Lk,
                                                          krows, k8, ks, lay.ks_ld);
    if (int rc = check_launch("quant_rows_i8_kernel(k)")) return rc;
    if (int rc = map_rows_i8(&tq, q8, Lq, B * H)) return rc;
    if (int rc = map_rows_i8(&tk, k8, Lk, B * Hkv)) return rc;
    if (int rc = make_map_2d(&tks, ks, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Lk, (uint64_t)B * Hkv, lay.ks_ld * 4, TK, 1,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
        return rc;
    a.qscale = qs;
    return launch_attention<true>(tq, tk, tv, tks, a, B, s);
}
}  // namespace
}  // namespace b2
