/*
 * rdna2_b200.h — C-ABI of the B200 (sm_100a) kernels behind the drop-in Python modules.
 *
 * The reference binds its gfx1030 kernels by name through ctypes + hipModuleLaunchKernel
 * (hip_attention.py:39-42): raw device pointers, int dims/strides and float scalars, launched on
 * torch's current stream; buffers are allocated by the Python caller. These entry points keep that
 * contract: plain pointers and sizes, a cudaStream_t passed as void*, no allocation inside, and an
 * int status instead of a launch-time HIP error (hip_attention.py:14-16 raises RuntimeError on a
 * non-zero code; the Python layer here does the same with b2_last_error()).
 *
 * All matrices are row-major. fp16 is IEEE binary16 passed as uint16_t bits.
 */
#ifndef RDNA2_B200_H
#define RDNA2_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Status codes. */
#define B2_OK 0
#define B2_ERR_INVALID 1     /* null pointer, negative size, inconsistent arguments */
#define B2_ERR_UNSUPPORTED 2 /* shape or alignment outside what the kernel handles */
#define B2_ERR_CUDA 3        /* CUDA runtime error at launch */
#define B2_ERR_DEVICE 4      /* a kernel reported a device-side error (bounded wait expired) */

/* Bits of the device status word returned by b2_device_status. */
#define B2_DEV_TIMEOUT_PRODUCER 1u
#define B2_DEV_TIMEOUT_MMA 2u
#define B2_DEV_TIMEOUT_EPILOGUE 4u
#define B2_DEV_TIMEOUT_DRAIN 8u

/* Library version (major * 100 + minor). */
int b2_version(void);

/* Message of the last failing call on this host thread (empty string if none). */
const char* b2_last_error(void);

/* Synchronizes the current device, then returns in *flags and clears the status bits that kernels
 * set when a bounded wait ran out. Returns B2_ERR_DEVICE if any bit was set. */
int b2_device_status(unsigned int* flags);

/* ------------------------------------------------------------------------------------------------
 * Activation pre-pass: optional activation, optional block-Hadamard rotation, per-row int8.
 * Replaces int8_gemm.hip quant_pack_a (:93), rot_quant_pack_a (:245), swiglu_rot_quant_pack_a
 * (:253), gate_rot_quant_pack_a (:257) and mod_rot_quant_pack_a (:261), launched from
 * int8_gemm.py:67 and :184. Output is plain row-major int8 [M, K] (ldq = K) and fp32 scale [M];
 * the reference's packed register layout (int8_gemm.hip:41-58) is internal to its GEMM and not kept.
 *
 *   rot_group 0   : no rotation (quant_pack_a)
 *   rot_group 256 : ConvRot H4^(x)4 / 16 over each 256 values (int8_gemm.hip:105-116,222-235)
 *   rot_group 128 : Sylvester H2^(x)7 / sqrt(128) over each 128 values (block-128 configuration)
 *
 * Rounding (int8_gemm.hip:38,53): scale = max(absmax/127, 1e-30); q = clamp(floor(y/scale + 0.5)).
 * act_out (nullable) receives the fp16 activation before rotation, for parity checks.
 * x rows are ldx elements apart; element k of a row is at (k / seg) * seg_stride + k % seg when
 * seg > 0 (a row gathered from per-rank segments), else at k.
 * ------------------------------------------------------------------------------------------------ */
int b2_quant_pack_a(const uint16_t* x, int64_t ldx, int8_t* q, float* scale, int M, int K, int rot_group,
                    void* stream);
int b2_quant_pack_a_seg(const uint16_t* x, int64_t ldx, int seg, int64_t seg_stride, int8_t* q, float* scale, int M,
                        int K, int rot_group, void* stream);
/* Activations with int4 values for the per-channel W4A4 path (int8_gemm.hip:62-91 quant_row_i4, :266
 * rot_quant_pack_a_i4; caller int8_gemm.py:90-103): after the rotation, scale = max(absmax, 1e-10) / 7 and
 * q = clamp(rint(y / scale), -7, 7) (IEEE divide, half-even). q holds one int8 per value (the reference packs eight
 * per dword for its dot8 instruction; the GEMM here reads bytes). rot_group 0, 128 or 256. */
int b2_quant_pack_a_i4(const uint16_t* x, int64_t ldx, int8_t* q, float* scale, int M, int K, int rot_group,
                       void* stream);
/* h = fp16(fp16(silu(gate)) * up), as F.silu(gate).mul_(up) (int8_gemm.hip:129-132). */
int b2_swiglu_quant_pack_a(const uint16_t* gate, const uint16_t* up, int64_t ld, int8_t* q, float* scale, int M,
                           int K, int rot_group, uint16_t* act_out, void* stream);
/* h = fp16(x * fp16(sigmoid(gate))), as x * F.sigmoid(gate) (int8_gemm.hip:134-137). */
int b2_gate_quant_pack_a(const uint16_t* x, const uint16_t* gate, int64_t ld, int8_t* q, float* scale, int M, int K,
                         int rot_group, uint16_t* act_out, void* stream);
/* h = fp16(4 tanh(g / 4) sigmoid(g) 25 tanh(h / 25)) of rows [h (K) | g (K)] at x + m * ldx, ldx >= 2K
 * (int8_gemm.hip:118-127 situ, situ_rot_quant_pack_a :249; caller int8_gemm.py:83-87,152-157). */
int b2_situ_quant_pack_a(const uint16_t* x, int64_t ldx, int8_t* q, float* scale, int M, int K, int rot_group,
                         uint16_t* act_out, void* stream);
/* h = fp16(fp16(fp16(x * rstd * (w + 1)) * s) + t), rstd = rsqrt(mean(x^2) + eps); s (= 1 + scale)
 * and t are fp16 [M / L, K] rows (int8_gemm.hip:139-143,167-191; caller int8_gemm.py:176-186). With s and t both
 * null there is no modulation: h = fp16(x * rstd * (w + 1)), the same int8 as s = 1, t = 0 without reading them. */
int b2_mod_quant_pack_a(const uint16_t* x, int64_t ldx, const float* w, const uint16_t* s, const uint16_t* t, int L,
                        float eps, int8_t* q, float* scale, int M, int K, int rot_group, uint16_t* act_out,
                        void* stream);

/* ------------------------------------------------------------------------------------------------
 * W8A8 GEMM with fused epilogue. Replaces int8_gemm.hip gemm / gemm_k6144 (:411,:414) and the
 * per-call pack_b (:271), launched from int8_gemm.py:70-79. B is the weight as stored, int8 [N, K].
 *   y = (float)acc * as[m] * ws[n] (+ bias[n])  -> fp16                     (int8_gemm.hip:382-383)
 *   with R: out = fp16(R[m,n] + fp16(G[m / L, n] * y))                      (int8_gemm.hip:394-400)
 *   with R and G null: out = fp16(R[m,n] + y), the same as a gate of ones (no gate rows read)
 * Needs K % 16 == 0, N % 8 == 0, 16-byte aligned A and B.
 * ------------------------------------------------------------------------------------------------ */
int b2_gemm(const int8_t* A, const int8_t* B, const float* as, const float* ws, const uint16_t* bias, uint16_t* C,
            int M, int N, int K, const uint16_t* R, const uint16_t* G, int L, void* stream);
/* Raw int32 accumulators C32[M, N] = A B^T of the same kernel, for bit-exact checks. */
int b2_gemm_i32(const int8_t* A, const int8_t* B, int32_t* C32, int M, int N, int K, void* stream);
/* Gate/up projection with the SwiGLU applied in the epilogue (no counterpart entry point in the reference: its
 * SwiGLU runs in the next layer's pre-pass, swiglu_rot_quant_pack_a, int8_gemm.hip:253, which this replaces for
 * callers that own the weight layout). B's rows hold the gate and up weights interleaved in blocks of 128: rows
 * [256 j, 256 j + 128) are gate features [128 j, 128 j + 128), rows [256 j + 128, 256 j + 256) the matching up
 * features; ws is ordered the same way. C[M, N/2] = fp16(fp16(g sigmoid(g)) u) with g and u the fp16 epilogue
 * values (as in b2_gemm without bias), the same SwiGLU arithmetic as b2_swiglu_quant_pack_a's act_out.
 * Needs N % 256 == 0 and K % 16 == 0. */
int b2_gemm_swiglu(const int8_t* A, const int8_t* B, const float* as, const float* ws, uint16_t* C, int M, int N,
                   int K, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Per-channel W4A4 GEMM, the reference's own int4 form (int8_gemm.hip:412 gemm_i4; int8_gemm.py:90-103):
 *   acc = sum_k A[m, k] W[n, k] (int32, all of K); C = fp16((float)acc * as[m] * ws[n] (+ bias[n])), the W8A8
 *   epilogue of b2_gemm. A: int8 [M, K] with values in [-7, 7] (b2_quant_pack_a_i4). Wp: packed uint8 [N, K/2],
 *   low nibble = even k, two's-complement nibbles. ws: fp32 [N]. workspace: N * K bytes of device scratch
 *   (16-byte aligned) that receives the widened weight, b2_unpack_int4 (as the reference re-packs its weight into a
 *   per-call buffer, pack_b, int8_gemm.hip:270-276). K % 32 == 0, N % 8 == 0.
 * ------------------------------------------------------------------------------------------------ */
int b2_unpack_int4(const uint8_t* Wp, int8_t* W, int N, int K, void* stream);
int b2_gemm_w4a4(const int8_t* A, const uint8_t* Wp, const float* as, const float* ws, const uint16_t* bias,
                 uint16_t* C, int M, int N, int K, int8_t* workspace, void* stream);

/* ------------------------------------------------------------------------------------------------
 * W4A8 GEMM with group-128 weight scales (the configuration's tuned-int4 form). The reference's int4 path is
 * per-channel W4A4 (int8_gemm.hip gemm_i4 :412, quant_row_i4 :62-91; int8_gemm.py wrap_w4a4 :90-103); this entry
 * point keeps that call's role (packed int4 weights read as stored, row-scaled int8 activations, fp16 out).
 *   acc_g = int32 dot of A[m, 128g..] and W[n, 128g..]; F = fma(acc_g, gscale[g, n], F) in group order;
 *   C = fp16(F * as[m] (+ bias[n])).
 * Wp: uint8 [N, K/2], low nibble = even k, nibbles two's complement in [-8, 7]. gscale: fp32 [K/128, N] (the fp16
 * group scales, transposed and widened). K % 128 == 0, N % 8 == 0, 16-byte aligned operands.
 * ------------------------------------------------------------------------------------------------ */
int b2_gemm_w4a8(const int8_t* A, const uint8_t* Wp, const float* as, const float* gscale, const uint16_t* bias,
                 uint16_t* C, int M, int N, int K, void* stream);
/* b2_gemm_w4a8 on a weight already widened to int8 W [N, K] (values in [-8, 7]), e.g. by b2_unpack_int4: the
 * unpacked-weight form that convrot_w4a4_forward's qweight_unpacked argument carries (int8_gemm.py:91). Same
 * arithmetic and result bit for bit; the tile no longer waits on on-chip widening. */
int b2_gemm_w4a8_wide(const int8_t* A, const int8_t* W, const float* as, const float* gscale, const uint16_t* bias,
                      uint16_t* C, int M, int N, int K, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Fused attention, head dim 128, no mask. Replaces hip_attention.hip pack_kv + attn (:32,:280) and
 * pack_kv_i8 + attn_i8 (:59,:161), launched from hip_attention.py:48-66 (called by attention.py:46-61).
 * q [B,H,Lq,128], k/v [B,Hkv,Lk,128], out [B,H,Lq,128], fp16, any element strides (b, h, l) that are
 * multiples of 8 with a contiguous last dimension; H % Hkv == 0 (grouped-query heads share K/V).
 * int8_qk != 0 selects per-row int8 Q and per-key int8 K with int32 dot products and fp16 PV; it needs
 * b2_attention_workspace_bytes() of caller-provided device scratch (16-byte aligned), else none.
 * ------------------------------------------------------------------------------------------------ */
int64_t b2_attention_workspace_bytes(int B, int H, int Hkv, int Lq, int Lk, int int8_qk);
int b2_attention(const uint16_t* q, int64_t sqb, int64_t sqh, int64_t sql, const uint16_t* k, int64_t skb,
                 int64_t skh, int64_t skl, const uint16_t* v, int64_t svb, int64_t svh, int64_t svl, uint16_t* out,
                 int64_t sob, int64_t soh, int64_t sol, int B, int H, int Hkv, int Lq, int Lk, float scale,
                 int int8_qk, void* workspace, int64_t workspace_bytes, void* stream);
/* b2_attention that also delivers its output to the other GPUs of a head group: the output store of
 * hip_attention.hip attn (:363-372) plus the all-gather the sharded block needs after it, in one kernel. Each CTA,
 * once its output tile is written to `out`, copies the tile to peer_out[p] (the same tensor offsets in peer p's
 * buffer, which must be mapped into this GPU's address space, e.g. symmetric memory) with plain coalesced stores,
 * fences at system scope and adds 1 to peer_cnt[p] (a 64-bit counter in peer p's memory). A launch makes
 * b2_attention_gather_ctas(B, H, Lq) arrivals on every peer counter. npeer <= 7. */
int b2_attention_gather(const uint16_t* q, int64_t sqb, int64_t sqh, int64_t sql, const uint16_t* k, int64_t skb,
                        int64_t skh, int64_t skl, const uint16_t* v, int64_t svb, int64_t svh, int64_t svl,
                        uint16_t* out, int64_t sob, int64_t soh, int64_t sol, int B, int H, int Hkv, int Lq, int Lk,
                        float scale, int int8_qk, void* workspace, int64_t workspace_bytes, uint16_t* const* peer_out,
                        unsigned long long* const* peer_cnt, int npeer, void* stream);
int b2_attention_gather_ctas(int B, int H, int Lq);
/* Stream-ordered wait for the gather: one thread polls *cnt (acquire, system scope) until it reaches `expected`;
 * after timeout_ns without it, sets *err (nonzero) and returns so that the stream and the GPU stay usable and the
 * host can report the failure. */
int b2_wait_count(const unsigned long long* cnt, unsigned long long expected, unsigned int* err, long long timeout_ns,
                  void* stream);

/* ------------------------------------------------------------------------------------------------
 * RMSNorm with fp32 math, zero-centred fp32 weight: y = fp16(x * rsqrt(mean(x^2) + eps) * (w + 1)).
 * Replaces rms_norm.hip rms_norm_head / rms_norm_row (:67,:71), launched from rms_norm.py:36.
 * Rows are ordered head-first: row n -> (h = n % H, l = (n / H) % L, b = n / (H L)), read from
 * x + b sb + h sh + l sl, written contiguous as [B, H, L, D]. D % 8 == 0, D <= 8192.
 * ------------------------------------------------------------------------------------------------ */
int b2_rms_norm(const uint16_t* x, const float* w, uint16_t* y, int rows, int D, int L, int H, int64_t sb, int64_t sh,
                int64_t sl, float eps, void* stream);
/* RMSNorm + rope over 128-wide heads (rms_norm.hip:48-61,75-77; rms_norm.py:42-52): F holds per token
 * 64 pairs of 2x2 fp32 rotations [fb-strided batch][L][64][2][2]. */
int b2_rms_norm_rope(const uint16_t* x, const float* w, uint16_t* y, int rows, int D, int L, int H, int64_t sb,
                     int64_t sh, int64_t sl, float eps, const float* F, int64_t fb, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Single-token decode (int8_gemv.hip, launched from int8_gemv.py).
 * ------------------------------------------------------------------------------------------------ */
/* fp32 regular-Hadamard rotation of each `group` values (power of 4), times rsqrt(group)
 * (int8_gemv.hip:32-52 rotate; int8_gemv.py:42-45). n % group == 0. */
int b2_rotate(const float* x, float* out, int64_t n, int group, void* stream);
/* out[n] = scale[n] * sum_k w[n,k] x[k] (+ bias[n]), fp32 (int8_gemv.hip:55-85 gemv_i8;
 * int8_gemv.py:62-63). K % 16 == 0. */
int b2_gemv_i8(const float* x, const int8_t* w, const float* scale, const float* bias, float* out, int N, int K,
               void* stream);
/* out[n] = sum_k w[n,k] x[k] in fp32 for a bf16 table w [N, K] (int8_gemv.hip:88-119 gemv_bf16; the logits of
 * int8_gemv.py:87-98). K % 8 == 0 (the reference: K % 256, N % 16); x and w 16-byte aligned. */
int b2_gemv_bf16(const float* x, const uint16_t* w, float* out, int N, int K, void* stream);
/* Decode-step glue of the configuration-5 driver (no counterpart entry points in the reference, whose decode step
 * runs these as torch ops around int8_gemv.py's kernels):
 *   b2_gemv_i8_ex: b2_gemv_i8 with act = 1 taking x = [gate | up] (2K values) and using silu(gate) * up as the input
 *     (torch's silu(g) * u in fp32), and an optional residual: out[n] = residual[n] + y[n] (residual != out).
 *   b2_rms_norm_f32: y = x * rsqrt(mean(x^2) + eps) * w for one fp32 row of D values.
 *   b2_decode_qk_rope: after the q|k|v GEMV, per head of 128: RMSNorm of q (q_norm) and k (k_norm), half-split
 *     rotary embedding at position *pos (angles *pos * inv_freq[0..63]), q to q_out [heads][128], k and v into row
 *     *pos of the caches [capacity][kv_heads][128]. */
int b2_gemv_i8_ex(const float* x, const int8_t* w, const float* scale, const float* bias, const float* residual,
                  float* out, int N, int K, int act, void* stream);
int b2_rms_norm_f32(const float* x, const float* w, float* y, int D, float eps, void* stream);
int b2_decode_qk_rope(const float* qkv, const float* q_norm, const float* k_norm, const float* inv_freq,
                      const int64_t* pos, float* q_out, float* k_cache, float* v_cache, int heads, int kv_heads,
                      float eps, void* stream);
/* One whole decode step of an int8 decoder in ONE persistent launch (one CTA per SM, cooperative): per layer
 * RMSNorm -> q|k|v GEMV -> q/k RMSNorm + rope + cache write -> split attention + merge -> o GEMV + residual ->
 * RMSNorm -> gate|up GEMV -> silu(gate) * up -> down GEMV + residual, with the arithmetic of gemv_i8
 * (int8_gemv.hip:55-85) and attn_decode / attn_merge (int8_gemv.hip:124-195) around linear_forward
 * (int8_gemv.py:48-64). It replaces the reference's per-layer sequence of those launches (and the torch ops between
 * them) for a whole token; the stages are separated by grid barriers inside the kernel, except the out-projection,
 * which takes each kv head's slice of its input as soon as that kv head's attention is merged.
 *   layers: device array of n_layers x 14 device pointers, in this order: norm_in [D], norm_post [D], q_norm [128],
 *     k_norm [128], w_qkv int8 [(H + 2 Hk) 128, D], s_qkv [(H + 2 Hk) 128], w_o int8 [D, H 128], s_o [D],
 *     w_gu int8 [2 F, D] (gate rows then up rows), s_gu [2 F], w_down int8 [D, F], s_down [D],
 *     k_cache [capacity, Hk, 128], v_cache [capacity, Hk, 128] (fp32 unless stated); every one 16-byte aligned.
 *   x [D]: the residual stream, read as the step's input and overwritten with its output. x2 [D], qkv
 *   [(H + 2 Hk) 128], att [H 128] (it holds the merged attention output as int8 digit planes and scales), act [F],
 *   partial [H, S, 128], stats [H, S, 2] are scratch, S = b2_decode_step_splits(Hk). inv_freq [64]; pos int64 [1] and lengths int32 [1] are read on the device (the
 *   position written, and the number of cache rows attended), so a captured graph replays for any position.
 *   sync: 2048 uint32 (8 KB) of arrival counters, cleared by this call (stream-ordered) before the launch.
 *   err: int32 flag; nonzero after a wait ran out (1 grid barrier, 2/3 weight ring), or 4 for a position outside
 *   the cache or a missing / misaligned table entry. A launch finding *err set does nothing.
 * H / Hk in {1, 2, 4}; Hk in {1, 2, 4, 8, 16}; D, H 128 and F multiples of 16 and at most 10240; at most 64 output
 * rows of D per SM; timeout_ns bounds every wait. */
int b2_decode_step(const uint64_t* layers, int n_layers, float* x, float* x2, float* qkv, float* att, float* act,
                   float* partial, float* stats, const float* inv_freq, const int64_t* pos, const int32_t* lengths,
                   unsigned int* sync, int* err, int hidden, int heads, int kv_heads, int mlp, int capacity, float eps,
                   long long timeout_ns, void* stream);
/* Position splits per kv head that b2_decode_step uses on the current device (sizes partial and stats). */
int b2_decode_step_splits(int kv_heads);
/* fp32 split-KV decode attention + merge (int8_gemv.hip:124-180 attn_decode, :183-195 attn_merge;
 * int8_gemv.py:101-114). q [B,1,H,128], k/v [B,capacity,Hkv,128], lengths int32 [B] read on the
 * device (graph-replayable), out [B,1,H,128]. partial: fp32 [B*H, 32, 128], stats: fp32 [B*H, 32, 2]
 * scratch from the caller. */
int b2_attn_decode(const float* q, const float* k, const float* v, const int32_t* lengths, float* out, float* partial,
                   float* stats, int batch, int heads, int kv_heads, int capacity, float scale, void* stream);
/* b2_attn_decode without the caller's scratch. It has no counterpart in the reference (whose attention_decode
 * allocates its partials with torch.empty, int8_gemv.py:108-110). It is for callers that cannot allocate device
 * memory: hosts whose device memory belongs to another allocator and FFI callers that hold only their own inputs
 * and outputs. The split partials live in a fixed device array inside this library, 2.1 MB on every GPU that loads
 * it, for at most batch x heads = 128 query rows; larger calls return B2_ERR_UNSUPPORTED. The first call on a
 * device looks up that array's address, so make it before any stream capture; the address is then kept for the
 * life of the process, so a device reset (cudaDeviceReset, a re-created primary context) is not supported after it.
 * All calls share the array: calls that overlap on the GPU (other streams, other threads) race on it. Nothing in it
 * needs to start at zero. */
int b2_attn_decode_noalloc(const float* q, const float* k, const float* v, const int32_t* lengths, float* out, int batch,
                           int heads, int kv_heads, int capacity, float scale, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* RDNA2_B200_H */
