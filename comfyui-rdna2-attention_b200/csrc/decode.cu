// Single-token decode kernels: fp32 Hadamard rotation, int8 GEMV, split-KV fp32 decode attention.
//
// Semantics follow int8_gemv.hip:
//   rotate      : radix-4 regular-Hadamard stages, stride x4, y[i] = sum - 2 x[3-i], then * rsqrt(group) (:32-52)
//   gemv_i8     : out[n] = scale[n] * sum_k w[n,k] x[k] (+ bias[n]), fp32                         (:55-85)
//   attn_decode : q * scale, online softmax with expf over a split of ceil(len/32) positions, merge (:124-195)
//
// The GEMV streams the int8 weight once from HBM with 16-byte non-allocating loads, several rows and
// several steps in flight per warp. int8 -> fp32 goes through a byte permute into the mantissa of
// 2^23 (exact), which keeps the conversion off the narrow conversion pipe.
#include "common.cuh"
#include "host.hpp"

namespace b2 {
namespace {

constexpr int DEC_SPLITS = 32;
constexpr int HEAD = 128;

// ---------------------------------------------------------------- rotate
// One regular 4-point Hadamard step on (a, b, c, d): s = ((a + b) + c) + d, then (s - 2d, s - 2c, s - 2b, s - 2a).
__device__ __forceinline__ void h4_step(float& a, float& b, float& c, float& d) {
    const float s = __fadd_rn(__fadd_rn(__fadd_rn(a, b), c), d);
    const float a0 = a, b0 = b;
    a = __fsub_rn(s, __fmul_rn(2.f, d));
    b = __fsub_rn(s, __fmul_rn(2.f, c));
    c = __fsub_rn(s, __fmul_rn(2.f, b0));
    d = __fsub_rn(s, __fmul_rn(2.f, a0));
}

// One CTA per group of `group` = 4^k values. The k base-4 digit stages (stride 1, 4, 16, ...) run two at a time in
// registers: a thread takes a 16-value tile (digits 2p and 2p+1 free, the others fixed), applies the stride-4^(2p)
// step to its four rows and then the stride-4^(2p+1) step to its four columns, which is the stage order of the
// reference, value for value. The first pass reads the input directly and the last one writes the output (times
// 1 / sqrt(group), an exact power of two); shared memory holds the group only between passes, so groups of at most
// 16 values never touch it.
__global__ void __launch_bounds__(256) rotate_kernel(const float* __restrict__ x, float* __restrict__ out, int group) {
    extern __shared__ float stage_buf[];
    const float* in = x + (int64_t)blockIdx.x * group;
    float* o = out + (int64_t)blockIdx.x * group;
    const int stages = __ffs(group) / 2;  // group = 4^stages
    const float norm = __fdiv_rn(1.f, sqrtf((float)group));
    for (int p = 0; 2 * p < stages; ++p) {
        const int st = 1 << (4 * p);
        const bool first = p == 0, last = 2 * p + 2 >= stages;
        const float* src = first ? in : stage_buf;
        if (2 * p + 1 < stages) {
            for (int q = threadIdx.x; q < group / 16; q += blockDim.x) {
                const int base = (q / st) * 16 * st + q % st;
                float v[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] = src[base + (e & 3) * st + (e >> 2) * 4 * st];
#pragma unroll
                for (int c = 0; c < 4; ++c) h4_step(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
#pragma unroll
                for (int a = 0; a < 4; ++a) h4_step(v[a], v[a + 4], v[a + 8], v[a + 12]);
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int i = base + (e & 3) * st + (e >> 2) * 4 * st;
                    if (last) o[i] = __fmul_rn(v[e], norm);
                    else stage_buf[i] = v[e];
                }
            }
        } else {
            for (int q = threadIdx.x; q < group / 4; q += blockDim.x) {
                const int base = (q / st) * 4 * st + q % st;
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) v[e] = src[base + e * st];
                h4_step(v[0], v[1], v[2], v[3]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    if (last) o[base + e * st] = __fmul_rn(v[e], norm);
                    else stage_buf[base + e * st] = v[e];
                }
            }
        }
        if (!last) __syncthreads();
    }
}

// ---------------------------------------------------------------- gemv_i8
__device__ __forceinline__ float i8f(uint32_t w_biased, int i) {
    // bytes of w_biased are b + 128; 0x4B0000uu is 2^23 + u exactly.
    return __int_as_float(__byte_perm(w_biased, 0x4B000000u, 0x7540u | i)) - 8388736.f;
}

__device__ __forceinline__ float dot16(const uint4 w, const float4 (&x)[4], float acc) {
    const uint32_t wv[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        acc = fmaf(i8f(wv[j], 0), x[j].x, acc);
        acc = fmaf(i8f(wv[j], 1), x[j].y, acc);
        acc = fmaf(i8f(wv[j], 2), x[j].z, acc);
        acc = fmaf(i8f(wv[j], 3), x[j].w, acc);
    }
    return acc;
}

__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_ROWS = 2;     // rows per warp
constexpr int GEMV_UNROLL = 4;   // 512-value steps in flight per row

// x is staged in shared memory in reading order: step s, sub-chunk j, lane l -> float4 index (s*4+j)*32+l,
// so each float4 read of a warp is conflict-free. K % 16 == 0; a partial last step is masked.
// silu(g) u in fp32 as torch computes silu(gate) * up: g / (1 + exp(-g)), then the product.
__device__ __forceinline__ float silu_mul_f32(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
}

// act 1: x holds [gate | up] (2K values) and the GEMV input is silu(gate) * up, formed while x is staged.
// residual: out[n] = residual[n] + y[n].
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_i8_kernel(const float* __restrict__ x, const int8_t* __restrict__ w,
                                                                 const float* __restrict__ scale,
                                                                 const float* __restrict__ bias,
                                                                 const float* __restrict__ residual, float* __restrict__ out,
                                                                 int N, int K, int act) {
    extern __shared__ float4 xs[];
    const int steps = (K + 511) / 512;
    for (int i = threadIdx.x; i < steps * 128; i += blockDim.x) {
        const int s = i >> 7, r = i & 127, l = r >> 2, j = r & 3;
        const int k = i * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k < K) {
            v = *reinterpret_cast<const float4*>(x + k);
            if (act) {
                const float4 u = *reinterpret_cast<const float4*>(x + K + k);
                v = make_float4(silu_mul_f32(v.x, u.x), silu_mul_f32(v.y, u.y), silu_mul_f32(v.z, u.z), silu_mul_f32(v.w, u.w));
            }
        }
        xs[(s * 4 + j) * 32 + l] = v;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * GEMV_WARPS + warp) * GEMV_ROWS;
    if (row0 >= N) return;
    float acc[GEMV_ROWS] = {};
    const int8_t* wr[GEMV_ROWS];
#pragma unroll
    for (int r = 0; r < GEMV_ROWS; ++r) wr[r] = w + (int64_t)min(row0 + r, N - 1) * K + lane * 16;
    const bool full_steps = (K % 512) == 0;
    int s = 0;
    for (; s + GEMV_UNROLL <= steps && (full_steps || s + GEMV_UNROLL < steps); s += GEMV_UNROLL) {
        uint4 v[GEMV_UNROLL][GEMV_ROWS];
#pragma unroll
        for (int u = 0; u < GEMV_UNROLL; ++u)
#pragma unroll
            for (int r = 0; r < GEMV_ROWS; ++r) v[u][r] = ld_stream(wr[r] + (s + u) * 512);
#pragma unroll
        for (int u = 0; u < GEMV_UNROLL; ++u) {
            float4 xv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) xv[j] = xs[((s + u) * 4 + j) * 32 + lane];
#pragma unroll
            for (int r = 0; r < GEMV_ROWS; ++r) acc[r] = dot16(v[u][r], xv, acc[r]);
        }
    }
    for (; s < steps; ++s) {
        if (s * 512 + lane * 16 >= K) break;
        float4 xv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[j] = xs[(s * 4 + j) * 32 + lane];
#pragma unroll
        for (int r = 0; r < GEMV_ROWS; ++r) acc[r] = dot16(ld_stream(wr[r] + s * 512), xv, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < GEMV_ROWS; ++r) {
        float v = acc[r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        const int n = row0 + r;
        if (lane == 0 && n < N) {
            float y = v * scale[n];
            if (bias) y += bias[n];
            out[n] = residual ? __fadd_rn(residual[n], y) : y;
        }
    }
}

// ---------------------------------------------------------------- gemv_bf16
// out[n] = sum_k w[n,k] x[k] for a bf16 table (the LM head of a decoder with tied embeddings). Same streaming
// scheme as gemv_i8: 16-byte non-allocating loads (8 bf16), GEMV_UNROLL steps of 256 values in flight for each of a
// warp's GEMV_ROWS rows. bf16 -> fp32 is exact: the high half of a word already is the fp32 pattern, the low half
// shifted up by 16 is.
__device__ __forceinline__ float dot8_bf16(const uint4 w, const float4 (&x)[2], float acc) {
    acc = fmaf(__uint_as_float(w.x << 16), x[0].x, acc);
    acc = fmaf(__uint_as_float(w.x & 0xffff0000u), x[0].y, acc);
    acc = fmaf(__uint_as_float(w.y << 16), x[0].z, acc);
    acc = fmaf(__uint_as_float(w.y & 0xffff0000u), x[0].w, acc);
    acc = fmaf(__uint_as_float(w.z << 16), x[1].x, acc);
    acc = fmaf(__uint_as_float(w.z & 0xffff0000u), x[1].y, acc);
    acc = fmaf(__uint_as_float(w.w << 16), x[1].z, acc);
    acc = fmaf(__uint_as_float(w.w & 0xffff0000u), x[1].w, acc);
    return acc;
}

// x staged in reading order: step s (256 values), half j, lane l -> float4 index (s*2+j)*32+l holds
// x[s*256 + l*8 + 4j .. +3]. K % 8 == 0; a partial last step is masked per lane.
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_bf16_kernel(const float* __restrict__ x,
                                                                   const uint16_t* __restrict__ w,
                                                                   float* __restrict__ out, int N, int K) {
    extern __shared__ float4 xs[];
    const int steps = (K + 255) / 256;
    for (int i = threadIdx.x; i < steps * 64; i += blockDim.x) {
        const int s = i >> 6, r = i & 63, l = r >> 1, j = r & 1;
        const int k = i * 4;
        xs[(s * 2 + j) * 32 + l] = k < K ? *reinterpret_cast<const float4*>(x + k) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * GEMV_WARPS + warp) * GEMV_ROWS;
    if (row0 >= N) return;
    float acc[GEMV_ROWS] = {};
    const uint16_t* wr[GEMV_ROWS];
#pragma unroll
    for (int r = 0; r < GEMV_ROWS; ++r) wr[r] = w + (int64_t)min(row0 + r, N - 1) * K + lane * 8;
    const bool full_steps = (K % 256) == 0;
    int s = 0;
    for (; s + GEMV_UNROLL <= steps && (full_steps || s + GEMV_UNROLL < steps); s += GEMV_UNROLL) {
        uint4 v[GEMV_UNROLL][GEMV_ROWS];
#pragma unroll
        for (int u = 0; u < GEMV_UNROLL; ++u)
#pragma unroll
            for (int r = 0; r < GEMV_ROWS; ++r) v[u][r] = ld_stream(wr[r] + (s + u) * 256);
#pragma unroll
        for (int u = 0; u < GEMV_UNROLL; ++u) {
            const float4 xv[2] = {xs[((s + u) * 2) * 32 + lane], xs[((s + u) * 2 + 1) * 32 + lane]};
#pragma unroll
            for (int r = 0; r < GEMV_ROWS; ++r) acc[r] = dot8_bf16(v[u][r], xv, acc[r]);
        }
    }
    for (; s < steps; ++s) {
        if (s * 256 + lane * 8 >= K) break;
        const float4 xv[2] = {xs[(s * 2) * 32 + lane], xs[(s * 2 + 1) * 32 + lane]};
#pragma unroll
        for (int r = 0; r < GEMV_ROWS; ++r) acc[r] = dot8_bf16(ld_stream(wr[r] + s * 256), xv, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < GEMV_ROWS; ++r) {
        float v = acc[r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        const int n = row0 + r;
        if (lane == 0 && n < N) out[n] = v;
    }
}

// ---------------------------------------------------------------- decode step glue
// y = x * rsqrt(mean(x^2) + eps) * w for one fp32 row (torch's rms(x, w) of the decode step), one CTA.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();  // red may still be read from a previous call
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t += red[i];
    return t;
}

__global__ void __launch_bounds__(1024) rms_norm_f32_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                           float* __restrict__ y, int D, float eps) {
    __shared__ float red[32];
    float ss = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = block_sum(ss, red);
    const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), eps));
    for (int i = threadIdx.x; i < D; i += blockDim.x) y[i] = __fmul_rn(__fmul_rn(x[i], r), w[i]);
}

// After the q|k|v GEMV of one token: per head of 128, q and k get RMSNorm (q_norm / k_norm weights) and the
// half-split rotary embedding at position *pos (angle pos * inv_freq[i], pairs (i, i + 64)); q goes to q_out, k and
// v into the caches' row *pos ([capacity][kv_heads][128] each). One CTA of 128 threads per head (q heads, then k,
// then v).
__global__ void __launch_bounds__(HEAD) decode_qk_rope_kernel(const float* __restrict__ qkv, const float* __restrict__ q_norm,
                                                             const float* __restrict__ k_norm,
                                                             const float* __restrict__ inv_freq,
                                                             const int64_t* __restrict__ pos, float* __restrict__ q_out,
                                                             float* __restrict__ k_cache, float* __restrict__ v_cache,
                                                             int heads, int kv_heads, float eps) {
    __shared__ float red[4];
    __shared__ float ys[HEAD];
    const int hd = blockIdx.x, t = threadIdx.x;
    const int64_t p = *pos;
    const float x = qkv[(int64_t)hd * HEAD + t];
    if (hd >= heads + kv_heads) {  // v: copied into the cache
        v_cache[(p * kv_heads + (hd - heads - kv_heads)) * HEAD + t] = x;
        return;
    }
    const bool is_q = hd < heads;
    const float ss = block_sum(__fmul_rn(x, x), red);
    const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)HEAD), eps));
    ys[t] = __fmul_rn(__fmul_rn(x, r), (is_q ? q_norm : k_norm)[t]);
    __syncthreads();
    const int i = t & 63;
    const float ang = __fmul_rn((float)p, inv_freq[i]);
    const float c = cosf(ang), sn = sinf(ang);
    const float a = ys[i], b = ys[i + 64];
    const float o = t < 64 ? __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn)) : __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
    if (is_q)
        q_out[(int64_t)hd * HEAD + t] = o;
    else
        k_cache[(p * kv_heads + (hd - heads)) * HEAD + t] = o;
}

// ---------------------------------------------------------------- decode attention
constexpr int DEC_WARPS = 8;

template <int GROUP>
__global__ void __launch_bounds__(DEC_WARPS * 32) attn_decode_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                                    const float* __restrict__ v,
                                                                    const int32_t* __restrict__ lengths,
                                                                    float* __restrict__ partial, float* __restrict__ stats,
                                                                    int capacity, int kv_heads, float scale) {
    __shared__ float4 acc_s[DEC_WARPS][GROUP][HEAD / 4];
    __shared__ float max_s[DEC_WARPS][GROUP], sum_s[DEC_WARPS][GROUP];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.y / kv_heads, kvh = blockIdx.y % kv_heads, split = blockIdx.x;
    const int length = min(lengths[b], capacity);
    const int chunk = (length + DEC_SPLITS - 1) / DEC_SPLITS;
    const int end = min((split + 1) * chunk, length);
    const int first_head = (b * kv_heads + kvh) * GROUP;

    float4 qv[GROUP], acc[GROUP];
    float mx[GROUP], sum[GROUP];
#pragma unroll
    for (int g = 0; g < GROUP; ++g) {
        const float4 t = reinterpret_cast<const float4*>(q + (int64_t)(first_head + g) * HEAD)[lane];
        qv[g] = make_float4(t.x * scale, t.y * scale, t.z * scale, t.w * scale);
        acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
        mx[g] = -1e30f;
        sum[g] = 0.f;
    }
    for (int j = split * chunk + warp; j < end; j += DEC_WARPS) {
        const int64_t row = ((int64_t)(b * capacity + j) * kv_heads + kvh) * HEAD;
        const float4 kv = __ldg(reinterpret_cast<const float4*>(k + row) + lane);
        const float4 vv = __ldg(reinterpret_cast<const float4*>(v + row) + lane);
#pragma unroll
        for (int g = 0; g < GROUP; ++g) {
            float d = qv[g].x * kv.x + qv[g].y * kv.y + qv[g].z * kv.z + qv[g].w * kv.w;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            const float next = fmaxf(mx[g], d);
            const float keep = expf(mx[g] - next), p = expf(d - next);
            sum[g] = sum[g] * keep + p;
            acc[g].x = acc[g].x * keep + vv.x * p;
            acc[g].y = acc[g].y * keep + vv.y * p;
            acc[g].z = acc[g].z * keep + vv.z * p;
            acc[g].w = acc[g].w * keep + vv.w * p;
            mx[g] = next;
        }
    }
#pragma unroll
    for (int g = 0; g < GROUP; ++g) {
        acc_s[warp][g][lane] = acc[g];
        if (lane == 0) {
            max_s[warp][g] = mx[g];
            sum_s[warp][g] = sum[g];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < GROUP * HEAD; i += DEC_WARPS * 32) {
        const int g = i / HEAD, d = i % HEAD;
        float top = max_s[0][g];
#pragma unroll
        for (int w = 1; w < DEC_WARPS; ++w) top = fmaxf(top, max_s[w][g]);
        float value = 0.f, total = 0.f;
#pragma unroll
        for (int w = 0; w < DEC_WARPS; ++w) {
            const float keep = expf(max_s[w][g] - top);
            value += reinterpret_cast<const float*>(&acc_s[w][g][0])[d] * keep;
            total += sum_s[w][g] * keep;
        }
        const int64_t at = (int64_t)(first_head + g) * DEC_SPLITS + split;
        partial[at * HEAD + d] = value;
        if (d == 0) {
            stats[at * 2] = top;
            stats[at * 2 + 1] = total;
        }
    }
}

__global__ void __launch_bounds__(HEAD) attn_merge_kernel(const float* __restrict__ partial, const float* __restrict__ stats,
                                                         float* __restrict__ out) {
    const int64_t head = blockIdx.x;
    const float* st = stats + head * DEC_SPLITS * 2;
    float top = st[0];
    for (int s = 1; s < DEC_SPLITS; ++s) top = fmaxf(top, st[s * 2]);
    float value = 0.f, total = 0.f;
    for (int s = 0; s < DEC_SPLITS; ++s) {
        const float keep = expf(st[s * 2] - top);
        value += partial[(head * DEC_SPLITS + s) * HEAD + threadIdx.x] * keep;
        total += st[s * 2 + 1] * keep;
    }
    out[head * HEAD + threadIdx.x] = value / total;
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" int b2_rotate(const float* x, float* out, int64_t n, int group, void* stream) {
    if (!x || !out || n < 0) return fail(B2_ERR_INVALID, "rotate: bad arguments");
    if (group < 4 || group > 16384 || (group & (group - 1)) || (__builtin_ctz(group) & 1))
        return fail(B2_ERR_UNSUPPORTED, "rotate: group %d must be a power of 4 in [4, 16384]", group);
    if (n % group) return fail(B2_ERR_UNSUPPORTED, "rotate: %lld values is not a multiple of group %d", (long long)n, group);
    if (n == 0) return B2_OK;
    const int smem = group > 16 ? group * 4 : 0;  // groups of at most 16 values stay in registers
    if (smem > 48 * 1024)
        if (int rc = set_smem(rotate_kernel, smem)) return rc;
    rotate_kernel<<<(unsigned)(n / group), 256, smem, (cudaStream_t)stream>>>(x, out, group);
    return check_launch("rotate_kernel");
}

extern "C" int b2_gemv_i8(const float* x, const int8_t* w, const float* scale, const float* bias, float* out, int N, int K,
                          void* stream) {
    if (!x || !w || !scale || !out || N < 0 || K <= 0) return fail(B2_ERR_INVALID, "gemv_i8: bad arguments");
    if (K % 16) return fail(B2_ERR_UNSUPPORTED, "gemv_i8: K=%d must be a multiple of 16", K);
    if (!aligned16(x) || !aligned16(w)) return fail(B2_ERR_UNSUPPORTED, "gemv_i8: x and w must be 16-byte aligned");
    if (N == 0) return B2_OK;
    const int steps = (K + 511) / 512;
    const int smem = steps * 512 * 4;
    if (smem > 200 * 1024) return fail(B2_ERR_UNSUPPORTED, "gemv_i8: K=%d too large", K);
    if (smem > 48 * 1024)
        if (int rc = set_smem(gemv_i8_kernel, smem)) return rc;
    const int rows_per_cta = GEMV_WARPS * GEMV_ROWS;
    gemv_i8_kernel<<<(N + rows_per_cta - 1) / rows_per_cta, GEMV_WARPS * 32, smem, (cudaStream_t)stream>>>(
        x, w, scale, bias, nullptr, out, N, K, 0);
    return check_launch("gemv_i8_kernel");
}

extern "C" int b2_gemv_i8_ex(const float* x, const int8_t* w, const float* scale, const float* bias, const float* residual,
                             float* out, int N, int K, int act, void* stream) {
    if (!x || !w || !scale || !out || N < 0 || K <= 0) return fail(B2_ERR_INVALID, "gemv_i8_ex: bad arguments");
    if (act != 0 && act != 1) return fail(B2_ERR_INVALID, "gemv_i8_ex: act %d (0: none, 1: silu(gate) * up)", act);
    if (K % 16) return fail(B2_ERR_UNSUPPORTED, "gemv_i8_ex: K=%d must be a multiple of 16", K);
    if (!aligned16(x) || !aligned16(w)) return fail(B2_ERR_UNSUPPORTED, "gemv_i8_ex: x and w must be 16-byte aligned");
    if (residual == out) return fail(B2_ERR_INVALID, "gemv_i8_ex: residual and out must not alias");
    if (N == 0) return B2_OK;
    const int steps = (K + 511) / 512;
    const int smem = steps * 512 * 4;
    if (smem > 200 * 1024) return fail(B2_ERR_UNSUPPORTED, "gemv_i8_ex: K=%d too large", K);
    if (smem > 48 * 1024)
        if (int rc = set_smem(gemv_i8_kernel, smem)) return rc;
    const int rows_per_cta = GEMV_WARPS * GEMV_ROWS;
    gemv_i8_kernel<<<(N + rows_per_cta - 1) / rows_per_cta, GEMV_WARPS * 32, smem, (cudaStream_t)stream>>>(
        x, w, scale, bias, residual, out, N, K, act);
    return check_launch("gemv_i8_kernel");
}

extern "C" int b2_gemv_bf16(const float* x, const uint16_t* w, float* out, int N, int K, void* stream) {
    if (!x || !w || !out || N < 0 || K <= 0) return fail(B2_ERR_INVALID, "gemv_bf16: bad arguments");
    if (K % 8) return fail(B2_ERR_UNSUPPORTED, "gemv_bf16: K=%d must be a multiple of 8", K);
    if (!aligned16(x) || !aligned16(w)) return fail(B2_ERR_UNSUPPORTED, "gemv_bf16: x and w must be 16-byte aligned");
    if (N == 0) return B2_OK;
    const int steps = (K + 255) / 256;
    const int smem = steps * 256 * 4;
    if (smem > 200 * 1024) return fail(B2_ERR_UNSUPPORTED, "gemv_bf16: K=%d too large", K);
    if (smem > 48 * 1024)
        if (int rc = set_smem(gemv_bf16_kernel, smem)) return rc;
    const int rows_per_cta = GEMV_WARPS * GEMV_ROWS;
    gemv_bf16_kernel<<<(N + rows_per_cta - 1) / rows_per_cta, GEMV_WARPS * 32, smem, (cudaStream_t)stream>>>(x, w, out, N,
                                                                                                            K);
    return check_launch("gemv_bf16_kernel");
}

extern "C" int b2_rms_norm_f32(const float* x, const float* w, float* y, int D, float eps, void* stream) {
    if (!x || !w || !y || D <= 0) return fail(B2_ERR_INVALID, "rms_norm_f32: bad arguments");
    rms_norm_f32_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(x, w, y, D, eps);
    return check_launch("rms_norm_f32_kernel");
}

extern "C" int b2_decode_qk_rope(const float* qkv, const float* q_norm, const float* k_norm, const float* inv_freq,
                                 const int64_t* pos, float* q_out, float* k_cache, float* v_cache, int heads,
                                 int kv_heads, float eps, void* stream) {
    if (!qkv || !q_norm || !k_norm || !inv_freq || !pos || !q_out || !k_cache || !v_cache || heads <= 0 || kv_heads <= 0)
        return fail(B2_ERR_INVALID, "decode_qk_rope: bad arguments");
    decode_qk_rope_kernel<<<heads + 2 * kv_heads, HEAD, 0, (cudaStream_t)stream>>>(qkv, q_norm, k_norm, inv_freq, pos, q_out,
                                                                                   k_cache, v_cache, heads, kv_heads, eps);
    return check_launch("decode_qk_rope_kernel");
}

namespace b2 {
namespace {

bool attn_decode_group_supported(int group) { return group == 1 || group == 2 || group == 4 || group == 8; }

// The split pass and the merge of one decode-attention call, with the partials and statistics at the given device
// addresses (the caller's scratch, or the library's fixed array). `group` = heads / kv_heads must be supported.
int launch_attn_decode(const float* q, const float* k, const float* v, const int32_t* lengths, float* out,
                       float* partial, float* stats, int batch, int heads, int kv_heads, int capacity, float scale,
                       cudaStream_t s) {
    const dim3 grid(DEC_SPLITS, batch * kv_heads);
    switch (heads / kv_heads) {
        case 1: attn_decode_kernel<1><<<grid, DEC_WARPS * 32, 0, s>>>(q, k, v, lengths, partial, stats, capacity, kv_heads, scale); break;
        case 2: attn_decode_kernel<2><<<grid, DEC_WARPS * 32, 0, s>>>(q, k, v, lengths, partial, stats, capacity, kv_heads, scale); break;
        case 4: attn_decode_kernel<4><<<grid, DEC_WARPS * 32, 0, s>>>(q, k, v, lengths, partial, stats, capacity, kv_heads, scale); break;
        case 8: attn_decode_kernel<8><<<grid, DEC_WARPS * 32, 0, s>>>(q, k, v, lengths, partial, stats, capacity, kv_heads, scale); break;
        default: return fail(B2_ERR_UNSUPPORTED, "attn_decode: %d query heads per KV head", heads / kv_heads);
    }
    if (int rc = check_launch("attn_decode_kernel")) return rc;
    attn_merge_kernel<<<batch * heads, HEAD, 0, s>>>(partial, stats, out);
    return check_launch("attn_merge_kernel");
}

}  // namespace
}  // namespace b2

extern "C" int b2_attn_decode(const float* q, const float* k, const float* v, const int32_t* lengths, float* out,
                              float* partial, float* stats, int batch, int heads, int kv_heads, int capacity, float scale,
                              void* stream) {
    if (!q || !k || !v || !lengths || !out || !partial || !stats) return fail(B2_ERR_INVALID, "attn_decode: null pointer");
    if (batch < 0 || heads <= 0 || kv_heads <= 0 || capacity <= 0 || heads % kv_heads)
        return fail(B2_ERR_INVALID, "attn_decode: bad shape");
    const int group = heads / kv_heads;
    if (!attn_decode_group_supported(group))
        return fail(B2_ERR_UNSUPPORTED, "attn_decode: %d query heads per KV head (supported: 1, 2, 4, 8)", group);
    if (batch == 0) return B2_OK;
    return launch_attn_decode(q, k, v, lengths, out, partial, stats, batch, heads, kv_heads, capacity, scale,
                              (cudaStream_t)stream);
}

// ---------------------------------------------------------------- decode attention without allocation
// Some callers cannot allocate device memory: a host whose device memory is owned by another allocator (a
// framework's caching pool) and which therefore has no scratch to hand out, or an FFI caller that only holds
// pointers to its own inputs and outputs. b2_attn_decode_noalloc serves them: the split partials and statistics
// that b2_attn_decode takes from the caller live here instead, in a file-scope device array of fixed size that every
// GPU loading this library holds until the process exits.
#include <mutex>

namespace b2 {
namespace {

constexpr int NOALLOC_MAX_ROWS = 128;  // batch x query heads
constexpr size_t NOALLOC_PARTIAL = (size_t)NOALLOC_MAX_ROWS * DEC_SPLITS * HEAD;
constexpr size_t NOALLOC_STATS = (size_t)NOALLOC_MAX_ROWS * DEC_SPLITS * 2;
static __device__ __align__(256) float g_decode_scratch[NOALLOC_PARTIAL + NOALLOC_STATS];  // 2.1 MB

// Device address of g_decode_scratch per device. The symbol's name in host code is only a host-side stand-in, so
// the address comes from cudaGetSymbolAddress, once per device with that device current.
float* g_scratch_addr[64] = {};
std::mutex g_scratch_mutex;

int scratch_for_current_device(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(B2_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return fail(B2_ERR_UNSUPPORTED, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess) return fail(B2_ERR_CUDA, "cudaGetSymbolAddress(decode scratch): %s", cudaGetErrorString(e));
        g_scratch_addr[dev] = static_cast<float*>(p);
    }
    *out = g_scratch_addr[dev];
    return B2_OK;
}

}  // namespace
}  // namespace b2

extern "C" int b2_attn_decode_noalloc(const float* q, const float* k, const float* v, const int32_t* lengths, float* out,
                                      int batch, int heads, int kv_heads, int capacity, float scale, void* stream) {
    if (!q || !k || !v || !lengths || !out) return fail(B2_ERR_INVALID, "attn_decode_noalloc: null pointer");
    if (batch < 0 || heads <= 0 || kv_heads <= 0 || capacity <= 0 || heads % kv_heads)
        return fail(B2_ERR_INVALID, "attn_decode_noalloc: bad shape");
    if ((int64_t)batch * heads > NOALLOC_MAX_ROWS)
        return fail(B2_ERR_UNSUPPORTED, "attn_decode_noalloc: batch x heads = %lld exceeds its fixed scratch of %d rows",
                    (long long)batch * heads, NOALLOC_MAX_ROWS);
    const int group = heads / kv_heads;
    if (!attn_decode_group_supported(group))
        return fail(B2_ERR_UNSUPPORTED, "attn_decode_noalloc: %d query heads per KV head (supported: 1, 2, 4, 8)", group);
    if (batch == 0) return B2_OK;
    float* scratch = nullptr;
    if (int rc = scratch_for_current_device(&scratch)) return rc;
    // Every (row, split) slot that attn_merge reads is written by attn_decode first, so the array's previous
    // contents never leak into a result and nothing needs clearing.
    return launch_attn_decode(q, k, v, lengths, out, scratch, scratch + NOALLOC_PARTIAL, batch, heads, kv_heads,
                              capacity, scale, (cudaStream_t)stream);
}
