// Activation pre-pass: [activation] -> [block Hadamard] -> fp16 -> per-row absmax int8.
//
// Semantics follow int8_gemm.hip:
//   quant        : scale = max(absmax / 127, 1e-30); q = clamp(floor(y / scale + 0.5), -128, 127)  (:38,:53)
//   ConvRot 256  : H4 (x) H4 (x) H4 (x) H4 applied one base-4 digit at a time, lowest digit first, with
//                  h4(a,b,c,d): s = ((a+b)+c)+d; (s-2d, s-2c, s-2b, s-2a); then y = fp16(v * 1/16)   (:105-116,:222-235)
//   SwiGLU       : fp16(fp16(g / (1 + exp(-g))) * u)                                                (:129-132)
//   sigmoid gate : fp16(x * fp16(1 / (1 + exp(-g))))                                                (:134-137)
//   modulate     : fp16(fp16(fp16(x * rstd * (w + 1)) * s) + t), no contraction                     (:139-143)
//   situ         : fp16(4 tanh(g / 4) sigmoid(g) 25 tanh(h / 25)) of a [h | g] row, tanh and sigmoid from
//                  base-2 exponentials, one rounding at the end                                       (:118-127,:202)
// The block-128 rotation (the configuration's normalised Hadamard) is Sylvester H2^(x)7, one bit at a
// time from bit 0, butterflies (a+b, a-b), then y = fp16(v * fp32(1/sqrt(128))).
//
// Layout on the device: one warp owns one row. Each lane loads 16 contiguous fp16 (two 16-byte loads,
// so a warp reads 1 KB contiguous per pass), applies the activation and the low index bits of the
// rotation in registers, swaps through a 2 KB shared-memory transpose so the high bits become lane-local,
// finishes the rotation and parks the fp16 row in shared memory. After a warp max, the row is read back
// contiguously and written as int8 with 16-byte stores. HBM traffic is one read of the inputs and one
// write of int8 + scale; nothing else touches DRAM.
#include "common.cuh"
#include "host.hpp"

namespace b2 {
namespace {

enum Act { ACT_NONE = 0, ACT_SWIGLU = 1, ACT_GATE = 2, ACT_MOD = 3, ACT_SITU = 4 };

template <int ACT>
__host__ __device__ constexpr bool two_inputs() { return ACT == ACT_SWIGLU || ACT == ACT_GATE || ACT == ACT_SITU; }

constexpr int PP_WARPS = 4;
constexpr int T_FLOATS = 576;  // 32 x 16 transpose plus bank padding
constexpr int T_BYTES = T_FLOATS * 4;
constexpr int MAX_K = 16384;
constexpr float INV_SQRT128 = 0.08838834764831845f;

struct PrepassArgs {
    const __half* x;
    int64_t ldx;
    int seg;
    int64_t seg_stride;
    const __half* u;
    int64_t ldu;
    const float* w;
    const __half* s;
    const __half* t;
    int L;
    float eps;
    int8_t* q;
    float* scale;
    __half* act_out;
    int M;
    int K;
};

__device__ __forceinline__ void h4(float& a, float& b, float& c, float& d) {
    const float s = __fadd_rn(__fadd_rn(__fadd_rn(a, b), c), d);
    const float a0 = a, b0 = b;
    a = __fsub_rn(s, __fmul_rn(2.f, d));
    b = __fsub_rn(s, __fmul_rn(2.f, c));
    c = __fsub_rn(s, __fmul_rn(2.f, b0));
    d = __fsub_rn(s, __fmul_rn(2.f, a0));
}

// Digits 0 and 1 of 16 values (int8_gemm.hip:111-116).
__device__ __forceinline__ void h16(float (&v)[16]) {
#pragma unroll
    for (int i = 0; i < 16; i += 4) h4(v[i], v[i + 1], v[i + 2], v[i + 3]);
#pragma unroll
    for (int i = 0; i < 4; i++) h4(v[i], v[i + 4], v[i + 8], v[i + 12]);
}

__device__ __forceinline__ void bfly(float& a, float& b) {
    const float x = a, y = b;
    a = __fadd_rn(x, y);
    b = __fsub_rn(x, y);
}

// Transpose-buffer index with a float4-granular XOR swizzle and row padding, conflict-free for the
// row writes and for the column reads of each rotation.
template <int ROT>
__device__ __forceinline__ int tidx(int r, int c) {
    const int pad = ROT == 256 ? (r >> 4) * 16 : (r >> 3) * 16;
    return r * 16 + pad + ((((c >> 2) ^ ((r >> 1) & 3))) << 2) + (c & 3);
}

__device__ __forceinline__ void load16(const __half* p, float (&f)[16]) {
    const uint4 lo = __ldg(reinterpret_cast<const uint4*>(p));
    const uint4 hi = __ldg(reinterpret_cast<const uint4*>(p) + 1);
    const __half2* a = reinterpret_cast<const __half2*>(&lo);
    const __half2* b = reinterpret_cast<const __half2*>(&hi);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 x = __half22float2(a[i]);
        const float2 y = __half22float2(b[i]);
        f[2 * i] = x.x;
        f[2 * i + 1] = x.y;
        f[8 + 2 * i] = y.x;
        f[8 + 2 * i + 1] = y.y;
    }
}

__device__ __forceinline__ void unpack16(const uint4 (&r)[2], float (&f)[16]) {
    const __half2* a = reinterpret_cast<const __half2*>(&r[0]);
    const __half2* b = reinterpret_cast<const __half2*>(&r[1]);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 x = __half22float2(a[i]);
        const float2 y = __half22float2(b[i]);
        f[2 * i] = x.x;
        f[2 * i + 1] = x.y;
        f[8 + 2 * i] = y.x;
        f[8 + 2 * i + 1] = y.y;
    }
}

__device__ __forceinline__ void store16(__half* p, const float (&f)[16]) {
    uint4 lo, hi;
    __half2* a = reinterpret_cast<__half2*>(&lo);
    __half2* b = reinterpret_cast<__half2*>(&hi);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        a[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        b[i] = __floats2half2_rn(f[8 + 2 * i], f[8 + 2 * i + 1]);
    }
    reinterpret_cast<uint4*>(p)[0] = lo;
    reinterpret_cast<uint4*>(p)[1] = hi;
}

// The exponential and the quotient use the hardware approximations (ex2-based __expf, rcp-based __fdividef, a few
// fp32 ulps); after the fp16 rounding of each stage the activation equals the exact formula's except for about one
// value in a thousand, by one fp16 step.
__device__ __forceinline__ float silu_mul(float g, float u) {
    const float silu = round_h(__fdividef(g, __fadd_rn(1.f, __expf(-g))));
    return round_h(__fmul_rn(silu, u));
}
__device__ __forceinline__ float sigmoid_gate(float x, float g) {
    const float sig = round_h(__fdividef(1.f, __fadd_rn(1.f, __expf(-g))));
    return round_h(__fmul_rn(x, sig));
}

// tanh(x) = (1 - t) / (1 + t) with t = 2^(-2 |x| log2(e)), and its odd series x (1 - x^2 (1/3 - x^2 2/15)) below
// |x| = 0.02, where 1 - t would cancel (int8_gemm.hip:118-122).
__device__ __forceinline__ float soft_tanh(float x) {
    const float ax = fabsf(x);
    float y;
    if (ax < 0.02f) {
        const float a2 = __fmul_rn(ax, ax);
        y = __fmul_rn(ax, __fsub_rn(1.f, __fmul_rn(a2, __fsub_rn(1.f / 3.f, __fmul_rn(a2, 2.f / 15.f)))));
    } else {
        const float t = ex2_approx(__fmul_rn(-2.885390082f, ax));
        y = __fdiv_rn(__fsub_rn(1.f, t), __fadd_rn(1.f, t));
    }
    return x < 0.f ? -y : y;
}

// The situ activation of a [hidden | gate] pair, soft-capped: fp16(4 tanh(g / 4) sigmoid(g) 25 tanh(h / 25)), the
// products taken left to right (int8_gemm.hip:124-127).
__device__ __forceinline__ float situ(float h, float g) {
    const float sig = __fdiv_rn(1.f, __fadd_rn(1.f, ex2_approx(__fmul_rn(-1.442695041f, g))));
    const float a = __fmul_rn(__fmul_rn(4.f, soft_tanh(__fmul_rn(g, 0.25f))), sig);
    return round_h(__fmul_rn(__fmul_rn(a, 25.f), soft_tanh(__fmul_rn(h, 0.04f))));
}

__device__ __forceinline__ uint32_t situ_h2(uint32_t h2, uint32_t g2) {
    const float2 h = __half22float2(u32_as_h2(h2)), g = __half22float2(u32_as_h2(g2));
    return h2_as_u32(__floats2half2_rn(situ(h.x, g.x), situ(h.y, g.y)));
}
__device__ __forceinline__ float modulate(float x, float rstd, float w, float s, float t) {
    const float n = round_h(__fmul_rn(__fmul_rn(x, rstd), __fadd_rn(w, 1.f)));
    return round_h(__fadd_rn(round_h(__fmul_rn(n, s)), t));
}

// y = fp16(v * c) (a power of two or 1/sqrt(128), one fp32 rounding then one fp16 rounding), parked as 16 fp16 at p;
// mx2 accumulates max |y| exactly in fp16.
__device__ __forceinline__ void park16(__half* p, const float (&v)[16], float c, __half2& mx2) {
    uint4 o[2];
    __half2* h = reinterpret_cast<__half2*>(o);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        h[i] = __floats2half2_rn(__fmul_rn(v[2 * i], c), __fmul_rn(v[2 * i + 1], c));
        mx2 = __hmax2(mx2, __habs2(h[i]));
    }
    reinterpret_cast<uint4*>(p)[0] = o[0];
    reinterpret_cast<uint4*>(p)[1] = o[1];
}

// floor(f / scale + 0.5) with the IEEE quotient, computed as f * (1/scale): |f / scale| <= 127 keeps that product
// within 2e-5 of the quotient, so unless f * inv + 0.5 lands within 1e-4 of an integer the floor is the same; those
// few values take the IEEE divide. The result is bit-identical to floorf(f / scale + 0.5f).
// W4A4 activations (int8_gemm.hip:62-91 quant_row_i4): q = clamp(rint(f / scale), -7, 7) with an IEEE divide,
// kept here as one int8 per value; a NaN quotient clamps to -7 like fminf(fmaxf(NaN, -7), 7).
__device__ __forceinline__ int quant1_i4(float f, float scale) {
    const float r = fminf(fmaxf(rintf(__fdiv_rn(f, scale)), -7.f), 7.f);
    return __float_as_int(__fadd_rn(r, 12582912.f)) - 0x4B400000;
}

__device__ __forceinline__ int quant1(float f, float scale, float inv) {
    const float u = __fmaf_rn(f, inv, 0.5f);
    float r = floorf(u);
    if (fabsf(__fsub_rn(__fsub_rn(u, r), 0.5f)) > 0.4999f) r = floorf(__fadd_rn(__fdiv_rn(f, scale), 0.5f));
    r = fminf(fmaxf(r, -128.f), 127.f);
    // r is an integer in [-128, 127]: adding 1.5 * 2^23 puts it in the low mantissa bits (exact).
    return __float_as_int(__fadd_rn(r, 12582912.f)) - 0x4B400000;
}

// ------------------------------------------------------------------------------------------- block-128, K % 1024
// Rows whose K is a multiple of 1024 under the block-128 rotation: a CTA of K/32 threads holds one row in
// registers (many CTAs per SM hide the load latency; a grid-stride walk with a prefetch of the next row needed so
// many registers that fewer rows were in flight). Thread t owns a
// quarter of 128-block t/4: with s = t%4 it loads the four 16-byte runs at 128 (t/4) + 32 o + 8 s (o = 0..3), so
// block index bits 0-2 (e) and 5-6 (o) are in registers and bits 3-4 (s) span the block's 4 threads. Bits 0-2 are
// rotated first; a per-warp 4 KB shared-memory transpose then trades bits 1-2 for the thread bits, and bits 3-6
// finish in registers. Butterflies run on packed fp32 pairs (bit 5 on the two halves of a pair) in the Sylvester
// order, bit 0 first, so every fp32 result equals the one-bit-at-a-time reference exactly. The fp16 row waits in
// registers for the CTA's absmax (one barrier), is quantized in place (quant_fast) and leaves through a 1 KB
// per-warp byte transpose as 16-byte stores. Both transposes are free of shared-memory bank conflicts.
constexpr int R128_WARP_BYTES = 4096 + 1024;
constexpr int R128_MAX_WARPS = MAX_K / 1024;

// max(a, |b|, |c|) with NaN propagation: any NaN operand gives NaN.
__device__ __forceinline__ float max3_abs_nan(float a, float b, float c) {
    float d;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(fabsf(b)), "f"(fabsf(c)));
    return d;
}
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}


__device__ __forceinline__ void bfly2(uint64_t& a, uint64_t& b) {
    const uint64_t x = a, y = b;
    a = add2(x, y);
    b = sub2(x, y);
}
// The butterfly between the two halves of one pair.
__device__ __forceinline__ void bfly_in(uint64_t& a) {
    const float2 f = upk2(a);
    a = pk2(__fadd_rn(f.x, f.y), __fsub_rn(f.x, f.y));
}

// Quantization with one fma per value: t = fma(y, 1/scale, 1.5 * 2^23) rounds y/scale to the nearest integer q (ties
// to even) and holds q in its low mantissa bits, so the int8 byte is t's low byte. That equals the reference's
// floor(y / scale + 0.5) unless y/scale lies within 1e-4 of a half-integer (|y/scale| <= 127 keeps the product within
// 8e-6 of the IEEE quotient): d = y/scale - q tells, and the caller sends a thread whose largest |d| exceeds 0.4999
// (or is NaN, from a non-finite y) through quant1. F is the fp32 pair of one fp16 pair; returns T, accumulates |d|.
__device__ __forceinline__ uint64_t quant_fast(uint64_t F, uint64_t inv2, float& dmax) {
    const uint64_t C = splat2(12582912.f);
    const uint64_t T = fma2(F, inv2, C);
    const float2 d = upk2(fma2(F, inv2, fma2(T, splat2(-1.f), C)));
    dmax = max3_abs_nan(dmax, d.x, d.y);
    return T;
}

template <int ACT>
__global__ void __launch_bounds__(512) prepass128_kernel(const PrepassArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float red[2][R128_MAX_WARPS];
    pdl_trigger();  // a GEMM launched after this kernel may run its set-up meanwhile; it waits for the data
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nwarps = blockDim.x >> 5;
    const int K = a.K;
    const int s = lane & 3, bw = lane >> 2;  // quarter within the block, block within the warp
    const int k0 = (tid >> 2) * 128 + s * 8;
    float* T = reinterpret_cast<float*>(smem + warp * R128_WARP_BYTES);
    unsigned char* B8 = smem + warp * R128_WARP_BYTES + 4096;
    constexpr bool TWO = two_inputs<ACT>();

    uint4 rx[4], ru[4];
    auto load_row = [&](int r) {
        const __half* xr = a.x + (int64_t)r * a.ldx;
#pragma unroll
        for (int o = 0; o < 4; ++o) {
            const int k = k0 + 32 * o;
            rx[o] = ldg_stream(a.seg ? xr + (int64_t)(k / a.seg) * a.seg_stride + (k % a.seg) : xr + k);
            if (TWO) ru[o] = ldg_stream(a.u + (int64_t)r * a.ldu + k);
        }
    };

    const int row = blockIdx.x;
    load_row(row);
    {
        // y[o][p]: the activation's fp16 pair at k0 + 32 o + 2 p.
        uint32_t y[4][4];
        if (ACT == ACT_MOD) {
            uint64_t X[4][4];
            uint64_t ss2 = splat2(0.f);
#pragma unroll
            for (int o = 0; o < 4; ++o) {
                const uint32_t* w = reinterpret_cast<const uint32_t*>(&rx[o]);
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    X[o][p] = h2_to_f2(w[p]);
                    ss2 = fma2(X[o][p], X[o][p], ss2);
                }
            }
            const float2 sp = upk2(ss2);
            float ss = sp.x + sp.y;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            if (lane == 0) red[0][warp] = ss;
            __syncthreads();
            ss = 0.f;
            for (int w = 0; w < nwarps; ++w) ss += red[0][w];
            const uint64_t R2 = splat2(rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
            // Without modulation rows (s = t = null) the result is the RMSNorm n itself.
            const bool modulate = a.s != nullptr;
            const __half* srow = modulate ? a.s + (int64_t)(row / a.L) * K : nullptr;
            const __half* trow = modulate ? a.t + (int64_t)(row / a.L) * K : nullptr;
#pragma unroll
            for (int o = 0; o < 4; ++o) {
                const int k = k0 + 32 * o;
                uint4 sv = make_uint4(0, 0, 0, 0), tv = make_uint4(0, 0, 0, 0);
                if (modulate) {
                    sv = __ldg(reinterpret_cast<const uint4*>(srow + k));
                    tv = __ldg(reinterpret_cast<const uint4*>(trow + k));
                }
                const float4 w0 = __ldg(reinterpret_cast<const float4*>(a.w + k));
                const float4 w1 = __ldg(reinterpret_cast<const float4*>(a.w + k) + 1);
                const uint64_t W[4] = {pk2(w0.x, w0.y), pk2(w0.z, w0.w), pk2(w1.x, w1.y), pk2(w1.z, w1.w)};
                const uint32_t* s2 = reinterpret_cast<const uint32_t*>(&sv);
                const uint32_t* t2 = reinterpret_cast<const uint32_t*>(&tv);
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    // n = fp16(x rstd (w + 1)); y = fp16(fp16(n s) + t) as exact fp16 pair operations (see
                    // prepass_kernel)
                    const uint32_t n = f2_to_h2(mul2(mul2(X[o][p], R2), add2(W[p], splat2(1.f))));
                    y[o][p] = modulate ? h2_as_u32(__hadd2_rn(__hmul2_rn(u32_as_h2(n), u32_as_h2(s2[p])), u32_as_h2(t2[p])))
                                       : n;
                }
            }
        } else {
#pragma unroll
            for (int o = 0; o < 4; ++o) {
                const uint32_t* xw = reinterpret_cast<const uint32_t*>(&rx[o]);
                const uint32_t* uw = reinterpret_cast<const uint32_t*>(&ru[o]);
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    if (ACT == ACT_SWIGLU) {
                        y[o][p] = swiglu_h2(xw[p], uw[p]);
                    } else if (ACT == ACT_GATE) {
                        const uint32_t sig = f2_to_h2(sigmoid2(h2_to_f2(uw[p])));
                        y[o][p] = h2_as_u32(__hmul2_rn(u32_as_h2(xw[p]), u32_as_h2(sig)));
                    } else if (ACT == ACT_SITU) {
                        y[o][p] = situ_h2(xw[p], uw[p]);
                    } else {
                        y[o][p] = xw[p];
                    }
                }
            }
        }
        if (ACT != ACT_NONE && a.act_out) {
#pragma unroll
            for (int o = 0; o < 4; ++o)
                *reinterpret_cast<uint4*>(a.act_out + (int64_t)row * K + k0 + 32 * o) =
                    make_uint4(y[o][0], y[o][1], y[o][2], y[o][3]);
        }

        // Bits 0-2 on pairs P[h][e] = (value of o = 2h, value of o = 2h + 1) at e.
        uint64_t P[2][8];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const float2 lo = __half22float2(u32_as_h2(y[2 * h][p]));
                const float2 hi = __half22float2(u32_as_h2(y[2 * h + 1][p]));
                P[h][2 * p] = pk2(lo.x, hi.x);
                P[h][2 * p + 1] = pk2(lo.y, hi.y);
            }
#pragma unroll
        for (int st = 1; st < 8; st <<= 1)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    if (!(e & st)) bfly2(P[h][e], P[h][e + st]);

        // Transpose: row R = 4 bw + e/2 of the warp's buffer receives the 4 values (o = 0..3) of (s, e) as its
        // logical 16-byte chunk 2 s + e%2; chunks are XOR-swizzled with g(R) = (R & 7) ^ ((R >> 2) & 1).
        __syncwarp();
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int R = 4 * bw + (e >> 1);
            const int chunk = (2 * s + (e & 1)) ^ ((R & 7) ^ ((R >> 2) & 1));
            const float2 lo = upk2(P[0][e]), hi = upk2(P[1][e]);
            *reinterpret_cast<float4*>(T + R * 32 + chunk * 4) = make_float4(lo.x, lo.y, hi.x, hi.y);
        }
        __syncwarp();
        // Q[j][i][h] = the pair (o = 2h, o = 2h + 1) of element 32 o + 8 j + 2 s + i of this thread's block:
        // bits 3-4 are j, bit 0 is i, bit 5 is inside the pair and bit 6 is h.
        uint64_t Q[4][2][2];
        {
            const int gl = (lane & 7) ^ ((lane >> 2) & 1);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float4 f = *reinterpret_cast<const float4*>(T + lane * 32 + ((c ^ gl) << 2));
                Q[c >> 1][c & 1][0] = pk2(f.x, f.y);
                Q[c >> 1][c & 1][1] = pk2(f.z, f.w);
            }
        }
#pragma unroll
        for (int st = 1; st < 4; st <<= 1)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int i = 0; i < 2; ++i)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        if (!(j & st)) bfly2(Q[j][i][h], Q[j + st][i][h]);
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                bfly_in(Q[j][i][0]);
                bfly_in(Q[j][i][1]);
                bfly2(Q[j][i][0], Q[j][i][1]);
            }

        // y = fp16(v / sqrt(128)); max |y| = fp16(max |v / sqrt(128)|) since rounding is monotonic (a NaN is skipped,
        // as the reference's fmaxf chain skips it).
        uint32_t yq[4][2][2];
        float mxf = 0.f;
        const uint64_t C2 = splat2(INV_SQRT128);
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint64_t V = mul2(Q[j][i][h], C2);
                    const float2 v = upk2(V);
                    mxf = max3(mxf, fabsf(v.x), fabsf(v.y));
                    yq[j][i][h] = f2_to_h2(V);
                }
        float mx = round_h(mxf);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        float* redm = red[1];
        if (lane == 0) redm[warp] = mx;
        __syncthreads();
        mx = 0.f;
        for (int w = 0; w < nwarps; ++w) mx = fmaxf(mx, redm[w]);
        const float scale = fmaxf(__fdiv_rn(mx, 127.f), 1e-30f);
        const float inv = __frcp_rn(scale);
        if (tid == 0) a.scale[row] = scale;

        // qb[o][j]: bytes of elements 32 o + 8 j + 2 s + {0, 1}.
        uint32_t qb[4][4];
        float dmax = 0.f;
        const uint64_t inv2 = splat2(inv);
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float2 t0 = upk2(quant_fast(h2_to_f2(yq[j][0][h]), inv2, dmax));
                const float2 t1 = upk2(quant_fast(h2_to_f2(yq[j][1][h]), inv2, dmax));
                qb[2 * h][j] = __byte_perm(__float_as_uint(t0.x), __float_as_uint(t1.x), 0x0040);
                qb[2 * h + 1][j] = __byte_perm(__float_as_uint(t0.y), __float_as_uint(t1.y), 0x0040);
            }
        if (!(dmax <= 0.4999f)) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float2 f0 = __half22float2(u32_as_h2(yq[j][0][h]));
                    const float2 f1 = __half22float2(u32_as_h2(yq[j][1][h]));
                    qb[2 * h][j] = (uint32_t)(quant1(f0.x, scale, inv) & 255) | ((uint32_t)(quant1(f1.x, scale, inv) & 255) << 8);
                    qb[2 * h + 1][j] =
                        (uint32_t)(quant1(f0.y, scale, inv) & 255) | ((uint32_t)(quant1(f1.y, scale, inv) & 255) << 8);
                }
        }

        // Byte transpose: logical byte 32 o + 8 j + 2 s of block bw, 16-byte chunks XOR-swizzled with f(bw).
        const int fb = ((bw & 1) << 2) | (bw >> 1);
#pragma unroll
        for (int o = 0; o < 4; ++o)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int L = 32 * o + 8 * j + 2 * s;
                *reinterpret_cast<uint16_t*>(B8 + bw * 128 + (((L >> 4) ^ fb) << 4) + (L & 15)) = (uint16_t)qb[o][j];
            }
        __syncwarp();
        int8_t* qrow = a.q + (int64_t)row * K + warp * 1024 + bw * 128;
#pragma unroll
        for (int h = 0; h < 2; ++h)
            *reinterpret_cast<uint4*>(qrow + h * 64 + s * 16) =
                *reinterpret_cast<const uint4*>(B8 + bw * 128 + (((4 * h + s) ^ fb) << 4));
    }
}

template <int ACT, int ROT, bool I4 = false>
__global__ void __launch_bounds__(PP_WARPS * 32, 5) prepass_kernel(const PrepassArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    pdl_trigger();  // a GEMM launched after this kernel may run its set-up meanwhile; it waits for the data
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * PP_WARPS + warp;
    if (row >= a.M) return;
    const int K = a.K;
    unsigned char* base = smem + warp * (K * 2 + T_BYTES);
    __half* rowbuf = reinterpret_cast<__half*>(base);
    float* T = reinterpret_cast<float*>(base + K * 2);

    const __half* xr = a.x + (int64_t)row * a.ldx;
    auto xptr = [&](int k) -> const __half* {
        return a.seg ? xr + (int64_t)(k / a.seg) * a.seg_stride + (k % a.seg) : xr + k;
    };

    float rstd = 0.f;
    if (ACT == ACT_MOD) {
        // Stage the raw row and sum its squares (the norm needs the whole row before any output).
        float ss = 0.f;
        for (int c0 = lane * 8; c0 < K; c0 += 8 * 256) {
            uint4 raw[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (c0 + j * 256 < K) raw[j] = __ldg(reinterpret_cast<const uint4*>(xptr(c0 + j * 256)));
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (c0 + j * 256 >= K) break;
                *reinterpret_cast<uint4*>(rowbuf + c0 + j * 256) = raw[j];
                const __half2* h = reinterpret_cast<const __half2*>(&raw[j]);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 f = __half22float2(h[i]);
                    ss = fmaf(f.x, f.x, ss);
                    ss = fmaf(f.y, f.y, ss);
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        rstd = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps));
        __syncwarp();
    }

    const __half* ur = two_inputs<ACT>() ? a.u + (int64_t)row * a.ldu : nullptr;
    // Without modulation rows (s = t = null) the MOD flavour's result is the RMSNorm n itself.
    const __half* srow = ACT == ACT_MOD && a.s ? a.s + (int64_t)(row / a.L) * K : nullptr;
    const __half* trow = ACT == ACT_MOD && a.s ? a.t + (int64_t)(row / a.L) * K : nullptr;

    __half2 mx2 = __float2half2_rn(0.f);  // running max of |y| over this lane's values (fp16, exact)
    const int npass = (K + 511) >> 9;
    // Loads for PF passes are issued together, so each warp keeps PF KB (x2 with a second input) in flight.
    constexpr bool TWO = two_inputs<ACT>();
    constexpr int PF = ACT == ACT_MOD ? 1 : (TWO ? 2 : 4);
    for (int p0 = 0; p0 < npass; p0 += PF) {
    uint4 rx[PF][2], ru[PF][2];
#pragma unroll
    for (int j = 0; j < PF; ++j) {
        const int kk = (p0 + j) * 512 + lane * 16;
        if (ACT != ACT_MOD && p0 + j < npass && kk < K) {
            const uint4* px = reinterpret_cast<const uint4*>(xptr(kk));
            rx[j][0] = __ldg(px);
            rx[j][1] = __ldg(px + 1);
            if (TWO) {
                const uint4* pu = reinterpret_cast<const uint4*>(ur + kk);
                ru[j][0] = __ldg(pu);
                ru[j][1] = __ldg(pu + 1);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < PF; ++j) {
        const int p = p0 + j;
        if (p >= npass) break;
        const int k0 = p * 512 + lane * 16;
        const bool active = k0 < K;
        float v[16];
        if (active) {
            if (ACT == ACT_MOD) {
                // n = fp16(x * rstd * (w + 1)) in fp32; then fp16(fp16(n * s) + t) as fp16 pairs: the product of two
                // fp16 values is exact before its single rounding, and a sum of two fp16 values rounded once to
                // fp16 equals the fp32 sum rounded to fp16, so the packed ops round exactly like the fp32 path.
                uint4 xr[2], sr[2] = {}, tr[2] = {};
                xr[0] = *reinterpret_cast<const uint4*>(rowbuf + k0);
                xr[1] = *reinterpret_cast<const uint4*>(rowbuf + k0 + 8);
                if (srow) {
                    sr[0] = __ldg(reinterpret_cast<const uint4*>(srow + k0));
                    sr[1] = __ldg(reinterpret_cast<const uint4*>(srow + k0) + 1);
                    tr[0] = __ldg(reinterpret_cast<const uint4*>(trow + k0));
                    tr[1] = __ldg(reinterpret_cast<const uint4*>(trow + k0) + 1);
                }
                const __half2* x2 = reinterpret_cast<const __half2*>(xr);
                const __half2* s2 = reinterpret_cast<const __half2*>(sr);
                const __half2* t2 = reinterpret_cast<const __half2*>(tr);
                const float4* wp = reinterpret_cast<const float4*>(a.w + k0);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float4 w4 = __ldg(wp + i);
                    const float2 xa = __half22float2(x2[2 * i]), xb = __half22float2(x2[2 * i + 1]);
                    const __half2 na = __floats2half2_rn(__fmul_rn(__fmul_rn(xa.x, rstd), __fadd_rn(w4.x, 1.f)),
                                                         __fmul_rn(__fmul_rn(xa.y, rstd), __fadd_rn(w4.y, 1.f)));
                    const __half2 nb = __floats2half2_rn(__fmul_rn(__fmul_rn(xb.x, rstd), __fadd_rn(w4.z, 1.f)),
                                                         __fmul_rn(__fmul_rn(xb.y, rstd), __fadd_rn(w4.w, 1.f)));
                    const float2 ya = __half22float2(srow ? __hadd2_rn(__hmul2_rn(na, s2[2 * i]), t2[2 * i]) : na);
                    const float2 yb = __half22float2(srow ? __hadd2_rn(__hmul2_rn(nb, s2[2 * i + 1]), t2[2 * i + 1]) : nb);
                    v[4 * i + 0] = ya.x;
                    v[4 * i + 1] = ya.y;
                    v[4 * i + 2] = yb.x;
                    v[4 * i + 3] = yb.y;
                }
            } else {
                unpack16(rx[j], v);
                if (TWO) {
                    float u[16];
                    unpack16(ru[j], u);
#pragma unroll
                    for (int i = 0; i < 16; i++)
                        v[i] = ACT == ACT_SWIGLU ? silu_mul(v[i], u[i])
                             : ACT == ACT_GATE   ? sigmoid_gate(v[i], u[i])
                                                 : situ(v[i], u[i]);
                }
            }
            if (ACT != ACT_NONE && a.act_out) store16(a.act_out + (int64_t)row * K + k0, v);
        }

        if (ROT == 0) {
            if (active) park16(rowbuf + k0, v, 1.f, mx2);
        } else {
            if (active) {
                if (ROT == 256) {
                    h16(v);
                } else {
#pragma unroll
                    for (int st = 1; st < 16; st <<= 1)
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            if ((i & st) == 0) bfly(v[i], v[i + st]);
                }
#pragma unroll
                for (int j = 0; j < 4; j++)
                    *reinterpret_cast<float4*>(T + tidx<ROT>(lane, 4 * j)) =
                        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
            __syncwarp();
            if (ROT == 256) {
                const int hw = lane >> 4, c = lane & 15;
                if (p * 512 + hw * 256 < K) {
#pragma unroll
                    for (int i = 0; i < 16; i++) v[i] = T[tidx<ROT>(16 * hw + i, c)];
                    h16(v);
                    // Parked in this lane's own slot (conflict-free); the quant phase knows the positions.
                    park16(rowbuf + k0, v, 0.0625f, mx2);
                }
            } else {
                const int q = lane >> 3, sub = lane & 7;
                if (p * 512 + q * 128 < K) {
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float2 f = *reinterpret_cast<const float2*>(T + tidx<ROT>(8 * q + j, 2 * sub));
                        v[2 * j] = f.x;
                        v[2 * j + 1] = f.y;
                    }
#pragma unroll
                    for (int st = 2; st < 16; st <<= 1)
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            if ((i & st) == 0) bfly(v[i], v[i + st]);
                    park16(rowbuf + k0, v, INV_SQRT128, mx2);
                }
            }
            __syncwarp();
        }
    }
    }

    float mx = fmaxf(__low2float(mx2), __high2float(mx2));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    // int8: max(absmax / 127, 1e-30) (int8_gemm.hip:38); int4 values: max(absmax, 1e-10) / 7 (:71).
    const float scale = I4 ? __fdiv_rn(fmaxf(mx, 1e-10f), 7.f) : fmaxf(__fdiv_rn(mx, 127.f), 1e-30f);
    const float inv = __frcp_rn(scale);
    if (lane == 0) a.scale[row] = scale;
    __syncwarp();
    auto qv = [&](float f) -> uint32_t { return (uint32_t)((I4 ? quant1_i4(f, scale) : quant1(f, scale, inv)) & 255); };

    // Each lane quantizes the 16 values it parked per pass. With a rotation they sit at transposed positions, so
    // the bytes go through a small shared-memory transpose (the float buffer, now free) and every lane then stores
    // 16 contiguous bytes: the warp writes 512 contiguous bytes per pass.
    int8_t* qr = a.q + (int64_t)row * K;
    unsigned char* T8 = reinterpret_cast<unsigned char*>(T);
    for (int p = 0; p < npass; ++p) {
        const int k0 = p * 512 + lane * 16;
        const bool active = k0 < K;
        uint32_t w[4] = {0, 0, 0, 0};
        if (active) {
            const uint4 r0 = *reinterpret_cast<const uint4*>(rowbuf + k0);
            const uint4 r1 = *reinterpret_cast<const uint4*>(rowbuf + k0 + 8);
            const __half2* h0 = reinterpret_cast<const __half2*>(&r0);
            const __half2* h1 = reinterpret_cast<const __half2*>(&r1);
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const float2 a0 = __half22float2(h0[2 * i]), a1 = __half22float2(h0[2 * i + 1]);
                const float2 b0 = __half22float2(h1[2 * i]), b1 = __half22float2(h1[2 * i + 1]);
                w[i] = qv(a0.x) | (qv(a0.y) << 8) | (qv(a1.x) << 16) | (qv(a1.y) << 24);
                w[2 + i] = qv(b0.x) | (qv(b0.y) << 8) | (qv(b1.x) << 16) | (qv(b1.y) << 24);
            }
        }
        if (ROT == 0) {
            if (active) *reinterpret_cast<uint4*>(qr + k0) = make_uint4(w[0], w[1], w[2], w[3]);
            continue;
        }
        if (active) {
            if (ROT == 256) {
                // value i of lane (hw, c) belongs to row 16 hw + i, column c of the pass's 32 x 16 byte block
                const int hw = lane >> 4, c = lane & 15;
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const int r = 16 * hw + i;
                    T8[r * 16 + (r >> 4) * 16 + c] = (unsigned char)(w[i >> 2] >> (8 * (i & 3)));
                }
            } else {
                // values 2j, 2j+1 of lane (q, sub) belong to row 8 q + j, columns 2 sub, 2 sub + 1
                const int q = lane >> 3, sub = lane & 7;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int r = 8 * q + j;
                    *reinterpret_cast<uint16_t*>(T8 + r * 16 + (r >> 3) * 16 + 2 * sub) =
                        (uint16_t)(w[j >> 1] >> (16 * (j & 1)));
                }
            }
        }
        __syncwarp();
        if (active) {
            const int pad = ROT == 256 ? (lane >> 4) * 16 : (lane >> 3) * 16;
            *reinterpret_cast<uint4*>(qr + k0) = *reinterpret_cast<const uint4*>(T8 + lane * 16 + pad);
        }
        __syncwarp();
    }
}

template <int ACT>
int launch_r128(const PrepassArgs& a, cudaStream_t stream) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        int rc = set_smem(prepass128_kernel<ACT>, R128_MAX_WARPS * R128_WARP_BYTES);
        if (rc) return rc;
        configured[dev] = true;
    }
    const int warps = a.K / 1024;
    prepass128_kernel<ACT><<<a.M, warps * 32, warps * R128_WARP_BYTES, stream>>>(a);
    return check_launch("prepass128_kernel");
}

template <int ACT, int ROT, bool I4 = false>
int launch_t(const PrepassArgs& a, cudaStream_t stream) {
    if (!I4 && ROT == 128 && a.K % 1024 == 0) return launch_r128<ACT>(a, stream);
    const int smem = PP_WARPS * (a.K * 2 + T_BYTES);
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        int rc = set_smem(prepass_kernel<ACT, ROT, I4>, PP_WARPS * (MAX_K * 2 + T_BYTES));
        if (rc) return rc;
        configured[dev] = true;
    }
    const int grid = (a.M + PP_WARPS - 1) / PP_WARPS;
    prepass_kernel<ACT, ROT, I4><<<grid, PP_WARPS * 32, smem, stream>>>(a);
    return check_launch("prepass_kernel");
}

template <int ACT>
int launch_rot(const PrepassArgs& a, int rot, cudaStream_t stream) {
    switch (rot) {
        case 0: return launch_t<ACT, 0>(a, stream);
        case 128: return launch_t<ACT, 128>(a, stream);
        case 256: return launch_t<ACT, 256>(a, stream);
        default: return fail(B2_ERR_UNSUPPORTED, "rot_group must be 0, 128 or 256 (got %d)", rot);
    }
}

int validate(const PrepassArgs& a, int rot) {
    if (a.M < 0 || a.K <= 0) return fail(B2_ERR_INVALID, "prepass: bad shape M=%d K=%d", a.M, a.K);
    if (!a.x || !a.q || !a.scale) return fail(B2_ERR_INVALID, "prepass: null pointer");
    if (a.K % 16) return fail(B2_ERR_UNSUPPORTED, "prepass: K=%d must be a multiple of 16", a.K);
    if (a.K > MAX_K) return fail(B2_ERR_UNSUPPORTED, "prepass: K=%d above %d", a.K, MAX_K);
    if (rot && a.K % rot) return fail(B2_ERR_UNSUPPORTED, "prepass: K=%d not a multiple of rot_group %d", a.K, rot);
    if (!aligned16(a.x) || (a.ldx * 2) % 16) return fail(B2_ERR_UNSUPPORTED, "prepass: x must be 16-byte aligned");
    if (a.seg && (a.seg % 16 || (a.seg_stride * 2) % 16))
        return fail(B2_ERR_UNSUPPORTED, "prepass: segments must be multiples of 16 values, 16-byte aligned");
    if (!aligned16(a.q)) return fail(B2_ERR_UNSUPPORTED, "prepass: q must be 16-byte aligned");
    if (a.u && (!aligned16(a.u) || (a.ldu * 2) % 16)) return fail(B2_ERR_UNSUPPORTED, "prepass: u must be 16-byte aligned");
    if (a.act_out && !aligned16(a.act_out)) return fail(B2_ERR_UNSUPPORTED, "prepass: act_out must be 16-byte aligned");
    return B2_OK;
}

PrepassArgs base_args(const uint16_t* x, int64_t ldx, int8_t* q, float* scale, int M, int K) {
    PrepassArgs a{};
    a.x = reinterpret_cast<const __half*>(x);
    a.ldx = ldx;
    a.q = q;
    a.scale = scale;
    a.M = M;
    a.K = K;
    a.L = 1;
    return a;
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" int b2_quant_pack_a_seg(const uint16_t* x, int64_t ldx, int seg, int64_t seg_stride, int8_t* q, float* scale,
                                   int M, int K, int rot_group, void* stream) {
    PrepassArgs a = base_args(x, ldx, q, scale, M, K);
    a.seg = seg;
    a.seg_stride = seg_stride;
    if (int rc = validate(a, rot_group)) return rc;
    if (M == 0) return B2_OK;
    return launch_rot<ACT_NONE>(a, rot_group, (cudaStream_t)stream);
}

extern "C" int b2_quant_pack_a(const uint16_t* x, int64_t ldx, int8_t* q, float* scale, int M, int K, int rot_group,
                               void* stream) {
    return b2_quant_pack_a_seg(x, ldx, 0, 0, q, scale, M, K, rot_group, stream);
}

extern "C" int b2_quant_pack_a_i4(const uint16_t* x, int64_t ldx, int8_t* q, float* scale, int M, int K, int rot_group,
                                  void* stream) {
    PrepassArgs a = base_args(x, ldx, q, scale, M, K);
    if (int rc = validate(a, rot_group)) return rc;
    if (M == 0) return B2_OK;
    switch (rot_group) {
        case 0: return launch_t<ACT_NONE, 0, true>(a, (cudaStream_t)stream);
        case 128: return launch_t<ACT_NONE, 128, true>(a, (cudaStream_t)stream);
        case 256: return launch_t<ACT_NONE, 256, true>(a, (cudaStream_t)stream);
        default: return fail(B2_ERR_UNSUPPORTED, "rot_group must be 0, 128 or 256 (got %d)", rot_group);
    }
}

extern "C" int b2_swiglu_quant_pack_a(const uint16_t* gate, const uint16_t* up, int64_t ld, int8_t* q, float* scale,
                                      int M, int K, int rot_group, uint16_t* act_out, void* stream) {
    PrepassArgs a = base_args(gate, ld, q, scale, M, K);
    a.u = reinterpret_cast<const __half*>(up);
    a.ldu = ld;
    a.act_out = reinterpret_cast<__half*>(act_out);
    if (!up) return fail(B2_ERR_INVALID, "swiglu: null up");
    if (int rc = validate(a, rot_group)) return rc;
    if (M == 0) return B2_OK;
    return launch_rot<ACT_SWIGLU>(a, rot_group, (cudaStream_t)stream);
}

extern "C" int b2_gate_quant_pack_a(const uint16_t* x, const uint16_t* gate, int64_t ld, int8_t* q, float* scale,
                                    int M, int K, int rot_group, uint16_t* act_out, void* stream) {
    PrepassArgs a = base_args(x, ld, q, scale, M, K);
    a.u = reinterpret_cast<const __half*>(gate);
    a.ldu = ld;
    a.act_out = reinterpret_cast<__half*>(act_out);
    if (!gate) return fail(B2_ERR_INVALID, "gate: null gate");
    if (int rc = validate(a, rot_group)) return rc;
    if (M == 0) return B2_OK;
    return launch_rot<ACT_GATE>(a, rot_group, (cudaStream_t)stream);
}

extern "C" int b2_situ_quant_pack_a(const uint16_t* x, int64_t ldx, int8_t* q, float* scale, int M, int K, int rot_group,
                                    uint16_t* act_out, void* stream) {
    // Row m is [hidden (K values) | gate (K values)] at x + m * ldx.
    PrepassArgs a = base_args(x, ldx, q, scale, M, K);
    a.u = x ? reinterpret_cast<const __half*>(x) + K : nullptr;
    a.ldu = ldx;
    a.act_out = reinterpret_cast<__half*>(act_out);
    if (int rc = validate(a, rot_group)) return rc;
    if (ldx < 2 * (int64_t)K) return fail(B2_ERR_INVALID, "situ: row stride %lld below 2K = %d", (long long)ldx, 2 * K);
    if (M == 0) return B2_OK;
    return launch_rot<ACT_SITU>(a, rot_group, (cudaStream_t)stream);
}

extern "C" int b2_mod_quant_pack_a(const uint16_t* x, int64_t ldx, const float* w, const uint16_t* s, const uint16_t* t,
                                   int L, float eps, int8_t* q, float* scale, int M, int K, int rot_group,
                                   uint16_t* act_out, void* stream) {
    PrepassArgs a = base_args(x, ldx, q, scale, M, K);
    a.w = w;
    a.s = reinterpret_cast<const __half*>(s);
    a.t = reinterpret_cast<const __half*>(t);
    a.L = L;
    a.eps = eps;
    a.act_out = reinterpret_cast<__half*>(act_out);
    if (!w || !s != !t || (s && L <= 0)) return fail(B2_ERR_INVALID, "mod: null weight, one of scale/shift null, or L <= 0");
    if (!aligned16(w) || (s && (!aligned16(s) || !aligned16(t))))
        return fail(B2_ERR_UNSUPPORTED, "mod: w, s, t must be 16-byte aligned");
    if (!s) a.L = 1;
    if (int rc = validate(a, rot_group)) return rc;
    if (M == 0) return B2_OK;
    return launch_rot<ACT_MOD>(a, rot_group, (cudaStream_t)stream);
}
