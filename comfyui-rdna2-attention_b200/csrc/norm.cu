// RMSNorm with fp32 math for fp16 rows (+ optional rope on 128-wide heads).
//
// Semantics follow rms_norm.hip norm_row (:9-65):
//   rstd = rsqrt(sum(x^2) / D + eps);  y = fp16(x * rstd * (w + 1))   (zero-centred fp32 weight)
//   rope : per pair (x0, x1) of the normalised fp16 row and 2x2 fp32 matrix m:
//          a = fma(m1, x1, m0 * x0), c = fma(m3, x1, m2 * x0), rounded to fp32 and then to fp16 (:48-61)
// Rows are ordered head-first (:15-16): row n -> h = n % H, l = (n / H) % L, b = n / (H L); input is strided,
// output is contiguous [B, H, L, D].
//
// D <= 128: 16 threads per row, one 16-byte vector each. D > 128: one warp per row with the row held in
// registers (CH 16-byte vectors per lane), so every value is read once and written once.
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
    const float4* F;
    int64_t fb;
};

__device__ __forceinline__ void norm8(const uint4 raw, float rstd, const float* w, const float4* f, uint4& out) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(w));
    const float4 w1 = __ldg(reinterpret_cast<const float4*>(w) + 1);
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = __half22float2(h[i]);
        o[2 * i] = round_h(__fmul_rn(__fmul_rn(v.x, rstd), __fadd_rn(wv[2 * i], 1.f)));
        o[2 * i + 1] = round_h(__fmul_rn(__fmul_rn(v.y, rstd), __fadd_rn(wv[2 * i + 1], 1.f)));
    }
    if (f) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 m = __ldg(f + j);
            const float x0 = o[2 * j], x1 = o[2 * j + 1];
            const float a = __fmaf_rn(m.y, x1, __fmul_rn(m.x, x0));
            const float c = __fmaf_rn(m.w, x1, __fmul_rn(m.z, x0));
            o[2 * j] = round_h(a);
            o[2 * j + 1] = round_h(c);
        }
    }
    __half2* oh = reinterpret_cast<__half2*>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i) oh[i] = __floats2half2_rn(o[2 * i], o[2 * i + 1]);
}

// TPR threads per row, CH vectors of 8 values per thread.
template <int TPR, int CH>
__global__ void __launch_bounds__(256) rms_norm_kernel(const NormArgs a) {
    const int t = threadIdx.x % TPR;
    const int n = blockIdx.x * (256 / TPR) + threadIdx.x / TPR;
    const bool valid = n < a.rows;
    const int nn = valid ? n : a.rows - 1;
    const int h = nn % a.H, l = (nn / a.H) % a.L, b = nn / a.H / a.L;
    const __half* x = a.x + b * a.sb + h * a.sh + l * a.sl;
    uint4 v[CH];
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int i = t + c * TPR;
        if (i < a.D / 8) {
            v[c] = __ldg(reinterpret_cast<const uint4*>(x) + i);
            const __half2* hv = reinterpret_cast<const __half2*>(&v[c]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __half22float2(hv[j]);
                sum = fmaf(f.x, f.x, sum);
                sum = fmaf(f.y, f.y, sum);
            }
        }
    }
#pragma unroll
    for (int o = TPR / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o, TPR);
    const float rstd = rsqrtf(__fadd_rn(__fdiv_rn(sum, (float)a.D), a.eps));
    if (!valid) return;
    uint4* y = reinterpret_cast<uint4*>(a.y + ((int64_t)(b * a.H + h) * a.L + l) * a.D);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int i = t + c * TPR;
        if (i < a.D / 8) {
            const float4* f = a.F ? a.F + b * a.fb + (int64_t)l * (a.D / 2) + i * 4 : nullptr;
            uint4 o;
            norm8(v[c], rstd, a.w + i * 8, f, o);
            y[i] = o;
        }
    }
}

template <int TPR, int CH>
int launch(const NormArgs& a, cudaStream_t s) {
    const int per = 256 / TPR;
    rms_norm_kernel<TPR, CH><<<(a.rows + per - 1) / per, 256, 0, s>>>(a);
    return check_launch("rms_norm_kernel");
}

int run(NormArgs& a, cudaStream_t s) {
    if (!a.x || !a.w || !a.y || a.rows < 0 || a.D <= 0 || a.L <= 0 || a.H <= 0)
        return fail(B2_ERR_INVALID, "rms_norm: bad arguments");
    if (a.D % 8 || a.D > 8192) return fail(B2_ERR_UNSUPPORTED, "rms_norm: D=%d must be a multiple of 8, <= 8192", a.D);
    if (!aligned16(a.x) || !aligned16(a.y) || !aligned16(a.w) || (a.sb * 2) % 16 || (a.sh * 2) % 16 || (a.sl * 2) % 16)
        return fail(B2_ERR_UNSUPPORTED, "rms_norm: x, y, w and strides must be 16-byte aligned");
    if (a.rows == 0) return B2_OK;
    if (a.D <= 128) return launch<16, 1>(a, s);
    const int vec = a.D / 8;  // vectors per row, spread over 32 lanes
    if (vec <= 32 * 4) return launch<32, 4>(a, s);
    if (vec <= 32 * 8) return launch<32, 8>(a, s);
    if (vec <= 32 * 12) return launch<32, 12>(a, s);
    if (vec <= 32 * 16) return launch<32, 16>(a, s);
    return launch<32, 32>(a, s);
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
