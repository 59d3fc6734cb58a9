// Activation pre-pass: [activation] -> [block Hadamard] -> fp16 -> per-row absmax int8.
//
// Semantics follow int8_gemm.hip:
//   quant        : scale = max(absmax / 127, 1e-30); q = clamp(floor(y / scale + 0.5), -128, 127)  (:38,:53)
//   ConvRot 256  : H4 (x) H4 (x) H4 (x) H4 applied one base-4 digit at a time, lowest digit first, with
//                  h4(a,b,c,d): s = ((a+b)+c)+d; (s-2d, s-2c, s-2b, s-2a); then y = fp16(v * 1/16)   (:105-116,:222-235)
//   SwiGLU       : fp16(fp16(g / (1 + exp(-g))) * u)                                                (:129-132)
//   sigmoid gate : fp16(x * fp16(1 / (1 + exp(-g))))                                                (:134-137)
//   modulate     : fp16(fp16(fp16(x * rstd * (w + 1)) * s) + t), no contraction                     (:139-143)
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

enum Act { ACT_NONE = 0, ACT_SWIGLU = 1, ACT_GATE = 2, ACT_MOD = 3 };

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
__device__ __forceinline__ int quant1(float f, float scale, float inv) {
    const float u = __fmaf_rn(f, inv, 0.5f);
    float r = floorf(u);
    if (fabsf(__fsub_rn(__fsub_rn(u, r), 0.5f)) > 0.4999f) r = floorf(__fadd_rn(__fdiv_rn(f, scale), 0.5f));
    r = fminf(fmaxf(r, -128.f), 127.f);
    // r is an integer in [-128, 127]: adding 1.5 * 2^23 puts it in the low mantissa bits (exact).
    return __float_as_int(__fadd_rn(r, 12582912.f)) - 0x4B400000;
}

template <int ACT, int ROT>
__global__ void __launch_bounds__(PP_WARPS * 32, 5) prepass_kernel(const PrepassArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
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

    const __half* ur = (ACT == ACT_SWIGLU || ACT == ACT_GATE) ? a.u + (int64_t)row * a.ldu : nullptr;
    const __half* srow = ACT == ACT_MOD ? a.s + (int64_t)(row / a.L) * K : nullptr;
    const __half* trow = ACT == ACT_MOD ? a.t + (int64_t)(row / a.L) * K : nullptr;

    __half2 mx2 = __float2half2_rn(0.f);  // running max of |y| over this lane's values (fp16, exact)
    const int npass = (K + 511) >> 9;
    // Loads for PF passes are issued together, so each warp keeps PF KB (x2 with a second input) in flight.
    constexpr bool TWO = ACT == ACT_SWIGLU || ACT == ACT_GATE;
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
                uint4 xr[2], sr[2], tr[2];
                xr[0] = *reinterpret_cast<const uint4*>(rowbuf + k0);
                xr[1] = *reinterpret_cast<const uint4*>(rowbuf + k0 + 8);
                sr[0] = __ldg(reinterpret_cast<const uint4*>(srow + k0));
                sr[1] = __ldg(reinterpret_cast<const uint4*>(srow + k0) + 1);
                tr[0] = __ldg(reinterpret_cast<const uint4*>(trow + k0));
                tr[1] = __ldg(reinterpret_cast<const uint4*>(trow + k0) + 1);
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
                    const float2 ya = __half22float2(__hadd2_rn(__hmul2_rn(na, s2[2 * i]), t2[2 * i]));
                    const float2 yb = __half22float2(__hadd2_rn(__hmul2_rn(nb, s2[2 * i + 1]), t2[2 * i + 1]));
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
                    for (int i = 0; i < 16; i++) v[i] = ACT == ACT_SWIGLU ? silu_mul(v[i], u[i]) : sigmoid_gate(v[i], u[i]);
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
    const float scale = fmaxf(__fdiv_rn(mx, 127.f), 1e-30f);
    const float inv = __frcp_rn(scale);
    if (lane == 0) a.scale[row] = scale;
    __syncwarp();

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
                w[i] = (uint32_t)(quant1(a0.x, scale, inv) & 255) | ((uint32_t)(quant1(a0.y, scale, inv) & 255) << 8) |
                       ((uint32_t)(quant1(a1.x, scale, inv) & 255) << 16) | ((uint32_t)(quant1(a1.y, scale, inv) & 255) << 24);
                w[2 + i] = (uint32_t)(quant1(b0.x, scale, inv) & 255) | ((uint32_t)(quant1(b0.y, scale, inv) & 255) << 8) |
                           ((uint32_t)(quant1(b1.x, scale, inv) & 255) << 16) | ((uint32_t)(quant1(b1.y, scale, inv) & 255) << 24);
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

template <int ACT, int ROT>
int launch_t(const PrepassArgs& a, cudaStream_t stream) {
    const int smem = PP_WARPS * (a.K * 2 + T_BYTES);
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        int rc = set_smem(prepass_kernel<ACT, ROT>, PP_WARPS * (MAX_K * 2 + T_BYTES));
        if (rc) return rc;
        configured[dev] = true;
    }
    const int grid = (a.M + PP_WARPS - 1) / PP_WARPS;
    prepass_kernel<ACT, ROT><<<grid, PP_WARPS * 32, smem, stream>>>(a);
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
    if (!w || !s || !t || L <= 0) return fail(B2_ERR_INVALID, "mod: null weight/scale/shift or L <= 0");
    if (!aligned16(w) || !aligned16(s) || !aligned16(t))
        return fail(B2_ERR_UNSUPPORTED, "mod: w, s, t must be 16-byte aligned");
    if (int rc = validate(a, rot_group)) return rc;
    if (M == 0) return B2_OK;
    return launch_rot<ACT_MOD>(a, rot_group, (cudaStream_t)stream);
}
