// RMSNorm with fp32 math for fp16 rows, optionally followed by rope on 128-wide attention heads.
//
// Arithmetic (the reference's rms_norm.hip:38,47 and :48-61):
//   rstd = rsqrt(sum(x^2) / D + eps);  y = fp16((x * rstd) * (w + 1)), each product rounded to fp32 (zero-centred w)
//   rope: per pair (x0, x1) of the fp16 result and its 2x2 fp32 matrix m = (m00, m01, m10, m11):
//         a = fma(m01, x1, m00 * x0), c = fma(m11, x1, m10 * x0), each rounded to fp32 and then to fp16.
// Input rows are strided: row (b, h, l) starts at b * sb + h * sh + l * sl. The output is contiguous [B, H, L, D].
//
// Both kernels are HBM-bound (every value read once and written once) and differ in how a row meets the threads:
//  - heads_kernel (D == 128: QK-norm, with or without rope): one CTA per token; the token's heads are dealt to the
//    CTA's four warps, and a head row is 32 lanes x 4 values (one 8-byte load per lane, 256 contiguous bytes per
//    warp). With rope, the token's 64 rotation matrices (1 KB) are staged in shared memory once for all its heads.
//  - rows_kernel (D > 128): each warp walks rows with a stride of the grid's warp count (the grid is a few waves of
//    the SM count); a row lives in registers as NV 16-byte pieces per lane (piece j * 32 + lane), all NV loads in
//    flight before the warp-wide reduction.
#include "common.cuh"
#include "host.hpp"

namespace b2 {
namespace {

struct NormArgs {
    const __half* x;
    const float* w;
    __half* y;
    int rows, D, L, H;
    int64_t sb, sh, sl;
    float eps;
    const float4* F;  // rope matrices, 64 per token, [batch (fb apart)][L][64]
    int64_t fb;       // float4 elements between batches of F (0: one set shared by the batch)
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float rstd_of(float sum, int D, float eps) {
    return rsqrtf(__fadd_rn(__fdiv_rn(sum, (float)D), eps));
}

// fp16((v * rstd) * (w + 1)) with both products rounded to fp32, returned as the fp32 value of the fp16 result.
__device__ __forceinline__ float scale_round(float v, float rstd, float w) {
    return round_h(__fmul_rn(__fmul_rn(v, rstd), __fadd_rn(w, 1.f)));
}

// One pair through its rotation matrix, each output rounded to fp32 (the fma) and then to fp16.
__device__ __forceinline__ __half2 rotate_pair(float x0, float x1, float4 m) {
    const float a = __fmaf_rn(m.y, x1, __fmul_rn(m.x, x0));
    const float c = __fmaf_rn(m.w, x1, __fmul_rn(m.z, x0));
    return __floats2half2_rn(a, c);
}

template <bool ROPE>
__global__ void __launch_bounds__(128) heads_kernel(const NormArgs a) {
    __shared__ float4 rot[64];
    const int tok = blockIdx.x;  // b * L + l
    const int b = tok / a.L, l = tok - b * a.L;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (ROPE) {
        if (threadIdx.x < 64) rot[threadIdx.x] = __ldg(a.F + b * a.fb + (int64_t)l * 64 + threadIdx.x);
        __syncthreads();
    }
    const float4 w = __ldg(reinterpret_cast<const float4*>(a.w) + lane);
    const __half* xt = a.x + b * a.sb + l * a.sl + lane * 4;
    for (int h = warp; h < a.H; h += 4) {
        const uint2 raw = __ldg(reinterpret_cast<const uint2*>(xt + h * a.sh));
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        float sum = __fmul_rn(v01.x, v01.x);
        sum = fmaf(v01.y, v01.y, sum);
        sum = fmaf(v23.x, v23.x, sum);
        sum = fmaf(v23.y, v23.y, sum);
        const float rstd = rstd_of(warp_sum(sum), 128, a.eps);
        const float y0 = scale_round(v01.x, rstd, w.x), y1 = scale_round(v01.y, rstd, w.y);
        const float y2 = scale_round(v23.x, rstd, w.z), y3 = scale_round(v23.y, rstd, w.w);
        __half2 o01, o23;
        if (ROPE) {
            o01 = rotate_pair(y0, y1, rot[2 * lane]);
            o23 = rotate_pair(y2, y3, rot[2 * lane + 1]);
        } else {
            o01 = __floats2half2_rn(y0, y1);
            o23 = __floats2half2_rn(y2, y3);
        }
        uint2 out;
        out.x = *reinterpret_cast<const uint32_t*>(&o01);
        out.y = *reinterpret_cast<const uint32_t*>(&o23);
        *reinterpret_cast<uint2*>(a.y + ((int64_t)(b * a.H + h) * a.L + l) * 128 + lane * 4) = out;
    }
}

template <int NV>
__global__ void __launch_bounds__(256) rows_kernel(const NormArgs a) {
    const int lane = threadIdx.x & 31;
    const int stride = gridDim.x * (blockDim.x >> 5);
    const int pieces = a.D >> 3;
    for (int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < a.rows; n += stride) {
        // Rows are numbered head-first: n = (b * L + l) * H + h.
        const int h = n % a.H, bl = n / a.H, l = bl % a.L, b = bl / a.L;
        const uint4* x = reinterpret_cast<const uint4*>(a.x + b * a.sb + h * a.sh + l * a.sl);
        uint4 v[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (j * 32 + lane < pieces) v[j] = __ldg(x + j * 32 + lane);
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            if (j * 32 + lane < pieces) {
                const __half2* hv = reinterpret_cast<const __half2*>(&v[j]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(hv[e]);
                    sum = fmaf(f.x, f.x, sum);
                    sum = fmaf(f.y, f.y, sum);
                }
            }
        }
        const float rstd = rstd_of(warp_sum(sum), a.D, a.eps);
        uint4* y = reinterpret_cast<uint4*>(a.y + ((int64_t)(b * a.H + h) * a.L + l) * a.D);
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int p = j * 32 + lane;
            if (p < pieces) {
                const float4 w0 = __ldg(reinterpret_cast<const float4*>(a.w) + 2 * p);
                const float4 w1 = __ldg(reinterpret_cast<const float4*>(a.w) + 2 * p + 1);
                const __half2* hv = reinterpret_cast<const __half2*>(&v[j]);
                const float2 f0 = __half22float2(hv[0]), f1 = __half22float2(hv[1]);
                const float2 f2 = __half22float2(hv[2]), f3 = __half22float2(hv[3]);
                uint4 o;
                __half2* oh = reinterpret_cast<__half2*>(&o);
                oh[0] = __floats2half2_rn(scale_round(f0.x, rstd, w0.x), scale_round(f0.y, rstd, w0.y));
                oh[1] = __floats2half2_rn(scale_round(f1.x, rstd, w0.z), scale_round(f1.y, rstd, w0.w));
                oh[2] = __floats2half2_rn(scale_round(f2.x, rstd, w1.x), scale_round(f2.y, rstd, w1.y));
                oh[3] = __floats2half2_rn(scale_round(f3.x, rstd, w1.z), scale_round(f3.y, rstd, w1.w));
                y[p] = o;
            }
        }
    }
}

template <int NV>
int launch_rows(const NormArgs& a, cudaStream_t s) {
    const int warps = 8;
    const int needed = (a.rows + warps - 1) / warps;
    const int grid = needed < sm_count() * 8 ? needed : sm_count() * 8;
    rows_kernel<NV><<<grid, warps * 32, 0, s>>>(a);
    return check_launch("rms_norm rows_kernel");
}

int run(NormArgs& a, cudaStream_t s) {
    if (!a.x || !a.w || !a.y || a.rows < 0 || a.D <= 0 || a.L <= 0 || a.H <= 0)
        return fail(B2_ERR_INVALID, "rms_norm: bad arguments");
    if (a.D % 8 || a.D > 8192) return fail(B2_ERR_UNSUPPORTED, "rms_norm: D=%d must be a multiple of 8, <= 8192", a.D);
    if (!aligned16(a.x) || !aligned16(a.y) || !aligned16(a.w) || (a.sb * 2) % 16 || (a.sh * 2) % 16 || (a.sl * 2) % 16)
        return fail(B2_ERR_UNSUPPORTED, "rms_norm: x, y, w and strides must be 16-byte aligned");
    if (a.rows == 0) return B2_OK;
    if (a.D == 128) {
        if ((int64_t)a.rows != (int64_t)a.H * a.L * (a.rows / ((int64_t)a.H * a.L)))
            return fail(B2_ERR_INVALID, "rms_norm: %d rows are not whole tokens of %d heads x %d positions", a.rows,
                        a.H, a.L);
        const int tokens = a.rows / a.H;  // B * L
        if (a.F) heads_kernel<true><<<tokens, 128, 0, s>>>(a);
        else heads_kernel<false><<<tokens, 128, 0, s>>>(a);
        return check_launch("rms_norm heads_kernel");
    }
    if (a.F) return fail(B2_ERR_UNSUPPORTED, "rms_norm: rope needs 128-wide heads");
    const int pieces = a.D / 8;
    if (pieces <= 32 * 4) return launch_rows<4>(a, s);
    if (pieces <= 32 * 8) return launch_rows<8>(a, s);
    if (pieces <= 32 * 16) return launch_rows<16>(a, s);
    return launch_rows<32>(a, s);
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" int b2_rms_norm(const uint16_t* x, const float* w, uint16_t* y, int rows, int D, int L, int H, int64_t sb,
                           int64_t sh, int64_t sl, float eps, void* stream) {
    NormArgs a{reinterpret_cast<const __half*>(x), w, reinterpret_cast<__half*>(y), rows, D, L, H, sb, sh, sl, eps, nullptr, 0};
    return run(a, (cudaStream_t)stream);
}

extern "C" int b2_rms_norm_rope(const uint16_t* x, const float* w, uint16_t* y, int rows, int D, int L, int H,
                                int64_t sb, int64_t sh, int64_t sl, float eps, const float* F, int64_t fb, void* stream) {
    if (!F) return fail(B2_ERR_INVALID, "rms_norm_rope: null freqs");
    if (D != 128) return fail(B2_ERR_UNSUPPORTED, "rms_norm_rope: head dim must be 128 (got %d)", D);
    if (!aligned16(F)) return fail(B2_ERR_UNSUPPORTED, "rms_norm_rope: freqs must be 16-byte aligned");
    NormArgs a{reinterpret_cast<const __half*>(x), w, reinterpret_cast<__half*>(y), rows, D, L, H, sb, sh, sl, eps,
               reinterpret_cast<const float4*>(F), fb};
    return run(a, (cudaStream_t)stream);
}
