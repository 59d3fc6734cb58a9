// W4A8 GEMM with group-128 weight scales for sm_100a:
//   C[m, n] = fp16( F[m, n] * as[m] (+ bias[n]) ),  F = fma(acc_g, s[g, n], F) over groups g in order,
//   acc_g = sum over the g-th 128 k of A[m, k] * W[n, k]  (int8 x int4 -> int32, exact).
// The reference's int4 path is per-channel W4A4 (int8_gemm.hip:62-91 quant_row_i4, :412 gemm_i4; int8_gemm.py:90-103);
// the configuration asks for W4A8 with fp16 scales per 128 values along K, so this kernel follows the configuration.
//
// Layout: A int8 [M, K] (from the pre-pass), W packed uint8 [N, K/2] (low nibble = even k, two's-complement
// nibbles in [-8, 7]), group scales fp32 [K/128, N] (the fp16 scales widened once at load time, exact).
//
// One CTA per SM, persistent over 128x128 output tiles, 12 warps (three per SM sub-partition, so up to 168
// registers each):
//   warp 0      TMA: A tile (128 x 128 B, 128-byte swizzle), packed W tile (128 x 64 B, 64-byte swizzle) and the
//               group's 128 scales into a 4-deep ring
//   warp 1      TMEM owner + tcgen05.mma issuer (kind::i8, M=128, N=128, K=32): one group = one k-block of 128,
//               into one of 4 TMEM partial buffers, so the MMA runs up to three groups ahead of the epilogue
//   warps 2..3  converters: thread t unpacks rows t and t + 64 of the int4 tile to int8 in the 128-byte-swizzled
//               K-major layout
//   warps 4..11 epilogue: two warps per 32-lane TMEM quarter, 64 columns each; per group, read the int32 partial,
//               F = fma(acc, s, F) in packed fp32 pairs, re-seed the buffer; after the last group, scale by as[m],
//               add bias, store fp16
// Each group's partial accumulates on top of 0x4B400000 (the bits of 1.5 * 2^23), so the accumulator read back
// as fp32 minus 1.5 * 2^23 is acc_g exactly: one FADD instead of an int->float conversion.
#include "common.cuh"
#include "host.hpp"

namespace b2 {
namespace {

__device__ unsigned int g_status;

constexpr int BM = 128, BN = 128, GK = 128;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * GK;          // 16 KB
constexpr int B_BYTES = BN * GK;          // 16 KB unpacked
constexpr int WP_BYTES = BN * GK / 2;     // 8 KB packed
constexpr int S_BYTES = BN * 4;           // 512 B scales
constexpr int OFF_B = A_BYTES, OFF_WP = A_BYTES + B_BYTES, OFF_S = OFF_WP + WP_BYTES;
constexpr int STAGE_BYTES = 41 * 1024;    // 16 + 16 + 8 KB + 512 B, 1024-aligned stride
constexpr int W4_THREADS = 384;
constexpr int NPB = 4;  // TMEM partial buffers of 128 columns
constexpr int SMEM = STAGES * STAGE_BYTES + 256 + 1024;
constexpr uint32_t SEED = 0x4B400000u;
constexpr float SEED_F = 12582912.0f;

struct W4Args {
    const float* as;
    const __half* bias;
    __half* C;
    int M, N, K;
};

// Sign-extends eight 4-bit fields held one per byte (low nibbles) into bytes: ((n ^ 8) + 0x78) ^ 0x80.
__device__ __forceinline__ uint32_t sext4(uint32_t v) { return ((v ^ 0x08080808u) + 0x78787878u) ^ 0x80808080u; }

// 8 packed bytes (16 int4, low nibble first) -> 16 int8 in k order.
__device__ __forceinline__ uint4 unpack16(uint32_t w0, uint32_t w1) {
    const uint32_t l0 = sext4(w0 & 0x0F0F0F0Fu), h0 = sext4((w0 >> 4) & 0x0F0F0F0Fu);
    const uint32_t l1 = sext4(w1 & 0x0F0F0F0Fu), h1 = sext4((w1 >> 4) & 0x0F0F0F0Fu);
    return make_uint4(__byte_perm(l0, h0, 0x5140), __byte_perm(l0, h0, 0x7362), __byte_perm(l1, h1, 0x5140),
                      __byte_perm(l1, h1, 0x7362));
}

__global__ void __launch_bounds__(W4_THREADS, 1)
    gemm_w4a8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmS, const W4Args g) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* full = bars;                 // [STAGES] TMA landed
    uint64_t* conv = bars + STAGES;        // [STAGES] int8 B tile written
    uint64_t* empty = bars + 2 * STAGES;   // [STAGES] MMA done + epilogue read the scales
    uint64_t* pready = bars + 3 * STAGES;  // [NPB] partial complete in TMEM
    uint64_t* pfree = pready + NPB;        // [NPB] partial consumed and re-seeded
    uint64_t* drain = pfree + NPB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_m = (g.M + BM - 1) / BM, num_n = (g.N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int G = g.K / GK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 64);
            mbar_init(&empty[s], 1 + 8);  // the MMA commit and one arrival per epilogue warp (scales read)
        }
        for (int b = 0; b < NPB; ++b) {
            mbar_init(&pready[b], 1);
            mbar_init(&pfree[b], 8);
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
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, issued = 0, issued_ph = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const int m0 = (tile % num_m) * BM, n0 = (tile / num_m) * BN;
                for (int kb = 0; kb < G; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, &g_status, B2_DEV_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    unsigned char* st = smem + stage * STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[stage], A_BYTES + WP_BYTES + S_BYTES);
                    tma_load_2d(st, &tmA, &full[stage], kb * GK, m0);
                    tma_load_2d(st + OFF_WP, &tmW, &full[stage], kb * (GK / 2), n0);
                    tma_load_2d(st + OFF_S, &tmS, &full[stage], n0, kb);
                    issued |= 1u << stage;
                    issued_ph = (issued_ph & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok)
                for (int s = 0; s < STAGES; ++s)
                    if ((issued >> s) & 1)
                        if (!mbar_wait_drain(&full[s], (issued_ph >> s) & 1, 100000000ull)) atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_make(2, 1, 0, 0, BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t q = 0;  // group counter across tiles
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                for (int kb = 0; kb < G; ++kb, ++q) {
                    const uint32_t b = q % NPB;
                    if (!mbar_wait(&pfree[b], (q / NPB) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA) ||
                        !mbar_wait(&full[stage], phase, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA) ||
                        !mbar_wait(&conv[stage], phase, abort_flag, &g_status, B2_DEV_TIMEOUT_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t base = smem_u32(smem + stage * STAGE_BYTES);
#pragma unroll
                    for (int k = 0; k < GK / 32; ++k)
                        mma_i8_ss(tmem + b * BN, sdesc_sw128(base + k * 32, 16, 1024),
                                  sdesc_sw128(base + OFF_B + k * 32, 16, 1024), idesc, 1);
                    tc_commit(&empty[stage]);
                    tc_commit(&pready[b]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            tc_commit(drain);
            if (!mbar_wait_drain(drain, 0, 100000000ull)) atomicOr(&g_status, B2_DEV_TIMEOUT_DRAIN);
        }
    } else if (warp < 4) {
        // Converters: thread t unpacks rows t and t + 64 of every stage.
        const int t = threadIdx.x - 64;
        int stage = 0;
        uint32_t phase = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            bool ok = true;
            for (int kb = 0; kb < G; ++kb) {
                if (!mbar_wait(&full[stage], phase, abort_flag, &g_status, B2_DEV_TIMEOUT_EPILOGUE)) {
                    ok = false;
                    break;
                }
                unsigned char* st = smem + stage * STAGE_BYTES;
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const int r = t + 64 * hr;
                    const unsigned char* src = st + OFF_WP + r * 64;
                    unsigned char* dst = st + OFF_B + r * 128;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {  // 16-byte packed chunk c = k 32c .. 32c+31
                        const uint4 p = *reinterpret_cast<const uint4*>(src + ((c ^ ((r >> 1) & 3)) << 4));
                        *reinterpret_cast<uint4*>(dst + (((2 * c) ^ (r & 7)) << 4)) = unpack16(p.x, p.y);
                        *reinterpret_cast<uint4*>(dst + (((2 * c + 1) ^ (r & 7)) << 4)) = unpack16(p.z, p.w);
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(&conv[stage]);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) break;
        }
    } else {
        // Epilogue: warp -> (32-lane quarter, 64-column half); thread -> row, 64 fp32 accumulators in 32 pairs.
        const int quarter = warp & 3;
        const int half = (warp - 4) >> 2;
        const int r = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
#pragma unroll
        for (int b = 0; b < NPB; ++b)
#pragma unroll
            for (int c = 0; c < 2; ++c) tmem_fill32(tmem + lane_base + b * BN + half * 64 + c * 32, SEED);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int b = 0; b < NPB; ++b) mbar_arrive(&pfree[b]);
        const uint64_t nseed = pk2(-SEED_F, -SEED_F);
        int stage = 0;
        uint32_t q = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
            const int m0 = (tile % num_m) * BM, n0 = (tile / num_m) * BN + half * 64;
            uint64_t F[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) F[i] = 0ull;
            for (int kb = 0; kb < G; ++kb, ++q) {
                const uint32_t b = q % NPB;
                if (!mbar_wait(&pready[b], (q / NPB) & 1, abort_flag, &g_status, B2_DEV_TIMEOUT_EPILOGUE)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const float4* sc = reinterpret_cast<const float4*>(smem + stage * STAGE_BYTES + OFF_S) + half * 16;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t v[16];
                    tmem_ld16_wait(tmem + lane_base + b * BN + half * 64 + c * 16, v);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 s4 = sc[c * 4 + i];
                        const uint64_t a0 = add2(pk2(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1])), nseed);
                        const uint64_t a1 = add2(pk2(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])), nseed);
                        F[c * 8 + 2 * i] = fma2(a0, pk2(s4.x, s4.y), F[c * 8 + 2 * i]);
                        F[c * 8 + 2 * i + 1] = fma2(a1, pk2(s4.z, s4.w), F[c * 8 + 2 * i + 1]);
                    }
                }
#pragma unroll
                for (int c = 0; c < 2; ++c) tmem_fill32(tmem + lane_base + b * BN + half * 64 + c * 32, SEED);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&pfree[b]);
                    mbar_arrive(&empty[stage]);
                }
                if (++stage == STAGES) stage = 0;
            }
            if (!ok) break;
            const int m = m0 + r;
            if (m < g.M) {
                const float sa = g.as[m];
                __half* dst = g.C + (int64_t)m * g.N + n0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (n0 + 8 * j >= g.N) continue;  // (not break: F must stay register-indexed)
                    float y[8];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = upk2(F[4 * j + e]);
                        y[2 * e] = __fmul_rn(f.x, sa);
                        y[2 * e + 1] = __fmul_rn(f.y, sa);
                    }
                    if (g.bias) {
                        const uint4 braw = __ldg(reinterpret_cast<const uint4*>(g.bias + n0 + 8 * j));
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
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
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

extern "C" int b2_gemm_w4a8(const int8_t* A, const uint8_t* Wp, const float* as, const float* gscale, const uint16_t* bias,
                            uint16_t* C, int M, int N, int K, void* stream) {
    if (!A || !Wp || !as || !gscale || !C) return fail(B2_ERR_INVALID, "gemm_w4a8: null pointer");
    if (M < 0 || N <= 0 || K <= 0) return fail(B2_ERR_INVALID, "gemm_w4a8: bad shape M=%d N=%d K=%d", M, N, K);
    if (K % GK) return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8: K=%d must be a multiple of 128", K);
    if (N % 8) return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8: N=%d must be a multiple of 8", N);
    if (!aligned16(A) || !aligned16(Wp) || !aligned16(gscale) || !aligned16(C) || (bias && !aligned16(bias)))
        return fail(B2_ERR_UNSUPPORTED, "gemm_w4a8: operands must be 16-byte aligned");
    if (M == 0) return B2_OK;
    CUtensorMap ta, tw, ts;
    if (int rc = make_map_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, K, GK, BM)) return rc;
    if (int rc = make_map_2d(&tw, Wp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, K / 2, GK / 2, BN,
                             CU_TENSOR_MAP_SWIZZLE_64B))
        return rc;
    if (int rc = make_map_2d(&ts, gscale, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, K / GK, (uint64_t)N * 4, BN, 1,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
        return rc;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (int rc = set_smem(gemm_w4a8_kernel, SMEM)) return rc;
        configured[dev] = true;
    }
    W4Args g{as, reinterpret_cast<const __half*>(bias), reinterpret_cast<__half*>(C), M, N, K};
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int grid = tiles < sm_count() ? tiles : sm_count();
    gemm_w4a8_kernel<<<grid, W4_THREADS, SMEM, (cudaStream_t)stream>>>(ta, tw, ts, g);
    return check_launch("gemm_w4a8_kernel");
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
