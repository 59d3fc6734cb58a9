// C-ABI launchers of the reference's kernels on the CPU stand-in — TEST INFRASTRUCTURE ONLY.
//
// Each ref_<kernel> runs the reference kernel of that name (compiled from its .hip source by build.py) with the grid
// and block its Python caller launches it with: int8_gemm.py:56-80 (quantization, pack_b, gemm), :176-186 (the
// modulated pre-pass), hip_attention.py:48-66 (pack_kv, attn), int8_gemv.py:42-45,48-64,87-98,101-114 (rotate,
// gemv_i8, gemv_bf16, attn_decode + attn_merge), rms_norm.py:25-52 (rms_norm_head/_row/_rope). Pointers are host
// memory; sizes are the kernels' own int arguments.
#include <stdint.h>

#include "hipemu_core.h"

using hipemu::Dim3;
using hipemu::launch;

// The reference kernels (extern "C" in their sources); pointer parameters are passed through as addresses.
extern "C" {
void quant_pack_a(const void* X, void* Ap, float* as, int K);
void rot_quant_pack_a(const void* X, void* Ap, float* as, int K);
void situ_rot_quant_pack_a(const void* X, void* Ap, float* as, int K);
void swiglu_rot_quant_pack_a(const void* X, const void* U, void* Ap, float* as, int K);
void gate_rot_quant_pack_a(const void* X, const void* U, void* Ap, float* as, int K);
void mod_rot_quant_pack_a(const void* X, void* Ap, float* as, int K, const float* W, const void* S, const void* T, int L,
                          float eps);
void rot_quant_pack_a_i4(const void* X, void* Ap, float* as, int K);
void pack_b(const void* B, void* Bp, int K);
void gemm(const void* Ap, const void* Bp, const float* as, const float* ws, const void* bias, void* C, int M, int N, int KCs,
          const void* R, const void* G, int L);
void gemm_i4(const void* Ap, const void* Bp, const float* as, const float* ws, const void* bias, void* C, int M, int N,
             int KCs, const void* R, const void* G, int L);
void gemm_k6144(const void* Ap, const void* Bp, const float* as, const float* ws, const void* bias, void* C, int M, int N,
                int KCs, const void* R, const void* G, int L);

void pack_kv(const void* K, const void* V, void* P, int Lk, int groups, int H, int skb, int skh, int skl, int svb,
             int svh, int svl);
void pack_kv_i8(const void* K, const void* V, void* P, int Lk, int groups, int H, int skb, int skh, int skl, int svb,
                int svh, int svl);
void attn(const void* Q, const void* P, void* O, int Lq, int Lk, int groups, int H, int rep, int sqb, int sqh, int sql,
          int sob, int soh, int sol, float scale_log2);
void attn_i8(const void* Q, const void* P, void* O, int Lq, int Lk, int groups, int H, int rep, int sqb, int sqh, int sql,
             int sob, int soh, int sol, float scale_log2);

void rotate(const float* x, float* out, int group);
void gemv_i8(const float* x, const void* w, const float* scale, const float* bias, float* out, int K);
void gemv_bf16(const float* x, const void* w, float* out, int K);
void attn_decode(const float* q, const float* k, const float* v, const int* lengths, float* partial, float* stats,
                 int capacity, int kv_heads, float scale);
void attn_merge(const float* partial, const float* stats, float* out);

void rms_norm_head(const void* X, const float* W, void* Y, int rows, int D, int L, int H, int sb, int sh, int sl,
                   float eps);
void rms_norm_row(const void* X, const float* W, void* Y, int rows, int D, int L, int H, int sb, int sh, int sl,
                  float eps);
void rms_norm_rope(const void* X, const float* W, void* Y, int rows, int D, int L, int H, int sb, int sh, int sl,
                   float eps, const void* F, int fb);
}

#define EXPORT extern "C" __attribute__((visibility("default")))

static Dim3 d3(unsigned x, unsigned y = 1) { return Dim3{x, y, 1}; }

// ---------------------------------------------------------------- int8_gemm.hip
// Activation pre-passes: one block per row (int8_gemm.py:67: 128 threads for the rotating ones, 256 otherwise).
EXPORT void ref_quant_pack_a(const void* X, void* Ap, float* as, int M, int K) {
    launch(d3(M), d3(256), [=] { quant_pack_a(X, Ap, as, K); });
}
EXPORT void ref_rot_quant_pack_a(const void* X, void* Ap, float* as, int M, int K) {
    launch(d3(M), d3(128), [=] { rot_quant_pack_a(X, Ap, as, K); });
}
EXPORT void ref_situ_rot_quant_pack_a(const void* X, void* Ap, float* as, int M, int K) {
    launch(d3(M), d3(128), [=] { situ_rot_quant_pack_a(X, Ap, as, K); });
}
EXPORT void ref_swiglu_rot_quant_pack_a(const void* X, const void* U, void* Ap, float* as, int M, int K) {
    launch(d3(M), d3(128), [=] { swiglu_rot_quant_pack_a(X, U, Ap, as, K); });
}
EXPORT void ref_gate_rot_quant_pack_a(const void* X, const void* U, void* Ap, float* as, int M, int K) {
    launch(d3(M), d3(128), [=] { gate_rot_quant_pack_a(X, U, Ap, as, K); });
}
EXPORT void ref_mod_rot_quant_pack_a(const void* X, void* Ap, float* as, int M, int K, const float* W, const void* S,
                                     const void* T, int L, float eps) {
    launch(d3(M), d3(128), [=] { mod_rot_quant_pack_a(X, Ap, as, K, W, S, T, L, eps); });
}
EXPORT void ref_rot_quant_pack_a_i4(const void* X, void* Ap, float* as, int M, int K) {
    launch(d3(M), d3(128), [=] { rot_quant_pack_a_i4(X, Ap, as, K); });
}
// Weight stream: grid (row_bytes / 64, N / 64) (int8_gemm.py:74).
EXPORT void ref_pack_b(const void* B, void* Bp, int N, int row_bytes) {
    launch(d3(row_bytes / 64, N / 64), d3(256), [=] { pack_b(B, Bp, row_bytes); });
}
// GEMM: grid (ceil(M / 512), N / 64) (int8_gemm.py:76-79). variant 0 gemm, 1 gemm_i4, 2 gemm_k6144 (raw weight).
EXPORT void ref_gemm(int variant, const void* Ap, const void* Bp, const float* as, const float* ws, const void* bias,
                     void* C, int M, int N, int KCs, const void* R, const void* G, int L) {
    const Dim3 grid = d3((M + 511) / 512, N / 64);
    if (variant == 1) launch(grid, d3(256), [=] { gemm_i4(Ap, Bp, as, ws, bias, C, M, N, KCs, R, G, L); });
    else if (variant == 2) launch(grid, d3(256), [=] { gemm_k6144(Ap, Bp, as, ws, bias, C, M, N, KCs, R, G, L); });
    else launch(grid, d3(256), [=] { gemm(Ap, Bp, as, ws, bias, C, M, N, KCs, R, G, L); });
}

// ---------------------------------------------------------------- hip_attention.hip
// K/V packing: grid (groups, B * Hkv) (hip_attention.py:61-63); attention: grid (ceil(Lq / 256), B * H) (:64-66).
EXPORT void ref_pack_kv(int int8_qk, const void* K, const void* V, void* P, int B, int Lk, int groups, int H, int skb,
                        int skh, int skl, int svb, int svh, int svl) {
    if (int8_qk) launch(d3(groups, B * H), d3(256), [=] { pack_kv_i8(K, V, P, Lk, groups, H, skb, skh, skl, svb, svh, svl); });
    else launch(d3(groups, B * H), d3(256), [=] { pack_kv(K, V, P, Lk, groups, H, skb, skh, skl, svb, svh, svl); });
}
EXPORT void ref_attn(int int8_qk, const void* Q, const void* P, void* O, int B, int Lq, int Lk, int groups, int H, int rep,
                     int sqb, int sqh, int sql, int sob, int soh, int sol, float scale_log2) {
    const Dim3 grid = d3((Lq + 255) / 256, B * H);
    if (int8_qk)
        launch(grid, d3(256), [=] { attn_i8(Q, P, O, Lq, Lk, groups, H, rep, sqb, sqh, sql, sob, soh, sol, scale_log2); });
    else
        launch(grid, d3(256), [=] { attn(Q, P, O, Lq, Lk, groups, H, rep, sqb, sqh, sql, sob, soh, sol, scale_log2); });
}

// ---------------------------------------------------------------- int8_gemv.hip
EXPORT void ref_rotate(const float* x, float* out, long n, int group) {
    launch(d3((unsigned)(n / group)), d3(256), [=] { rotate(x, out, group); });
}
EXPORT void ref_gemv_i8(const float* x, const void* w, const float* scale, const float* bias, float* out, int N, int K) {
    launch(d3(N / 16), d3(256), [=] { gemv_i8(x, w, scale, bias, out, K); });
}
EXPORT void ref_gemv_bf16(const float* x, const void* w, float* out, int N, int K) {
    launch(d3(N / 16), d3(256), [=] { gemv_bf16(x, w, out, K); });
}
// Decode attention: grid (32 splits, B * Hkv), then the merge with one 128-thread block per query head
// (int8_gemv.py:111-113).
EXPORT void ref_attn_decode(const float* q, const float* k, const float* v, const int* lengths, float* partial,
                            float* stats, float* out, int B, int H, int Hkv, int capacity, float scale) {
    launch(d3(32, B * Hkv), d3(256), [=] { attn_decode(q, k, v, lengths, partial, stats, capacity, Hkv, scale); });
    launch(d3(B * H), d3(128), [=] { attn_merge(partial, stats, out); });
}

// ---------------------------------------------------------------- rms_norm.hip
// rms_norm.py:33-38: 16 threads per row when D <= 128 (rms_norm_head), a block per row otherwise (rms_norm_row);
// rms_norm_rope always 16 per row (:49-51).
EXPORT void ref_rms_norm(const void* X, const float* W, void* Y, int rows, int D, int L, int H, int sb, int sh, int sl,
                         float eps) {
    if (D <= 128) launch(d3((rows + 15) / 16), d3(256), [=] { rms_norm_head(X, W, Y, rows, D, L, H, sb, sh, sl, eps); });
    else launch(d3(rows), d3(256), [=] { rms_norm_row(X, W, Y, rows, D, L, H, sb, sh, sl, eps); });
}
EXPORT void ref_rms_norm_rope(const void* X, const float* W, void* Y, int rows, int D, int L, int H, int sb, int sh,
                              int sl, float eps, const void* F, int fb) {
    launch(d3((rows + 15) / 16), d3(256), [=] { rms_norm_rope(X, W, Y, rows, D, L, H, sb, sh, sl, eps, F, fb); });
}
