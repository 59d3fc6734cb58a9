"""The reference's own kernels run on the host — TEST INFRASTRUCTURE ONLY.

oracle/hipemu/build.py compiles the reference's .hip kernels for the CPU (oracle/_ref/libref_hip.so); this module
launches them the way the reference's Python does (int8_gemm.py run / linear / wrap_w4a4 / quantize_block_input,
hip_attention.py attention, int8_gemv.py rotate / linear_forward / logits / attention_decode, rms_norm.py rms_norm /
rms_norm_rope) on numpy arrays, and undoes the reference's internal packed layouts so that results compare with the
oracle restatement and with this build's kernels. It pins the restatement to the reference's code: tests/
test_oracle_ref.py checks one against the other, and tests/golden/make_golden_ref.py stores outputs as fixtures.
Where the stand-in's arithmetic differs from the gfx1030 hardware (exp2/expf/rsqrt ulps, fdot2 rounding, no fp
contraction; see oracle/hipemu/hipemu_core.h) the comparisons carry a tolerance.
"""
import ctypes
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_ref", "libref_hip.so")
F16, F32 = np.float16, np.float32
_P, _I, _F, _L = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_long
_lib = None


def available():
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(LIB_PATH)
        sig = {
            "ref_quant_pack_a": [_P, _P, _P, _I, _I],
            "ref_rot_quant_pack_a": [_P, _P, _P, _I, _I],
            "ref_situ_rot_quant_pack_a": [_P, _P, _P, _I, _I],
            "ref_swiglu_rot_quant_pack_a": [_P, _P, _P, _P, _I, _I],
            "ref_gate_rot_quant_pack_a": [_P, _P, _P, _P, _I, _I],
            "ref_mod_rot_quant_pack_a": [_P, _P, _P, _I, _I, _P, _P, _P, _I, _F],
            "ref_rot_quant_pack_a_i4": [_P, _P, _P, _I, _I],
            "ref_pack_b": [_P, _P, _I, _I],
            "ref_gemm": [_I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _P, _I],
            "ref_pack_kv": [_I, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I],
            "ref_attn": [_I, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F],
            "ref_rotate": [_P, _P, _L, _I],
            "ref_gemv_i8": [_P, _P, _P, _P, _P, _I, _I],
            "ref_gemv_bf16": [_P, _P, _P, _I, _I],
            "ref_attn_decode": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F],
            "ref_rms_norm": [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F],
            "ref_rms_norm_rope": [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _P, _I],
        }
        for name, args in sig.items():
            fn = getattr(_lib, name)
            fn.argtypes = args
            fn.restype = None
    return _lib


def _p(a):
    return None if a is None else _P(a.ctypes.data)


def _c(a, dtype):
    return np.ascontiguousarray(np.asarray(a, dtype=dtype))


# ---------------------------------------------------------------- int8_gemm.hip
def _quantized(M, row_bytes):
    """The packed activation buffer and scales of int8_gemm.py:51-53 (rows rounded up to 512)."""
    blocks = (M + 511) // 512
    return np.zeros(blocks * 512 * row_bytes, np.uint8), np.zeros(M, F32)


def _chunk_index(M, K, values_per_chunk):
    """16-byte chunk index of (row, chunk) in the packed layout quant_row writes (int8_gemm.hip:41-58): rows in
    64-row wave tiles, two 32-lane halves, chunk g of a row at ((g / 4) * 256 + (g % 4) * 32) chunks from the row's
    base (wave tile * KCs * 256 + half * 128 + lane), KCs = K / (4 * values_per_chunk)."""
    kcs = K // (4 * values_per_chunk)
    m = np.arange(M)[:, None]
    g = np.arange(K // values_per_chunk)[None, :]
    return (m >> 6) * kcs * 256 + ((m >> 5) & 1) * 128 + (m & 31) + (g >> 2) * 256 + (g & 3) * 32


def unpack_a(packed, M, K):
    """Packed int8 activations -> int8 [M, K] (16 values per 16-byte chunk, in order)."""
    chunks = packed.reshape(-1, 16)[_chunk_index(M, K, 16)]
    return chunks.reshape(M, K).view(np.int8)


def unpack_a_i4(packed, M, K):
    """Packed int4 activations (quant_row_i4, int8_gemm.hip:74-90: eight nibbles per dword, low first) -> int8."""
    words = packed.view(np.uint32).reshape(-1, 4)[_chunk_index(M, K, 32)]  # [M, K/32, 4]
    shifts = np.arange(8, dtype=np.uint32) * 4
    nib = ((words[..., None] >> shifts) & 15).astype(np.int8)  # [M, K/32, 4, 8]
    nib = np.where(nib >= 8, nib - 16, nib).astype(np.int8)
    return nib.reshape(M, K)


def quant(x, kind="plain", u=None, w=None, s=None, t=None, L=1, eps=1e-6):
    """One pre-pass of int8_gemm.hip on fp16 rows x [M, K] ([M, 2K] for situ): kind is "plain" (quant_pack_a),
    "rotate" (ConvRot-256), "situ", "swiglu" / "gate" (with u), "mod" (with w, s, t, L, eps), or "i4" (ConvRot + int4
    values). Returns (int8 [M, K], fp32 scales [M])."""
    x = _c(x, F16)
    M = x.shape[0]
    K = x.shape[1] // 2 if kind == "situ" else x.shape[1]
    row_bytes = K // 2 if kind == "i4" else K
    ap, scale = _quantized(M, row_bytes)
    r = lib()
    if kind == "plain":
        r.ref_quant_pack_a(_p(x), _p(ap), _p(scale), M, K)
    elif kind == "rotate":
        r.ref_rot_quant_pack_a(_p(x), _p(ap), _p(scale), M, K)
    elif kind == "situ":
        r.ref_situ_rot_quant_pack_a(_p(x), _p(ap), _p(scale), M, K)
    elif kind in ("swiglu", "gate"):
        uu = _c(u, F16)
        fn = r.ref_swiglu_rot_quant_pack_a if kind == "swiglu" else r.ref_gate_rot_quant_pack_a
        fn(_p(x), _p(uu), _p(ap), _p(scale), M, K)
    elif kind == "mod":
        wf, sf, tf = _c(w, F32), _c(s, F16), _c(t, F16)
        r.ref_mod_rot_quant_pack_a(_p(x), _p(ap), _p(scale), M, K, _p(wf), _p(sf), _p(tf), L, F32(eps))
    elif kind == "i4":
        r.ref_rot_quant_pack_a_i4(_p(x), _p(ap), _p(scale), M, K)
        return unpack_a_i4(ap, M, K), scale
    else:
        raise ValueError(kind)
    return unpack_a(ap, M, K), scale


def linear(x, weight, weight_scale, bias=None, kind="plain", u=None, res=None, i4=False, **mod):
    """int8_gemm.py run(): pre-pass, pack_b (or the raw-weight gemm_k6144 for 6144-byte rows), gemm; weight int8
    [N, K] (packed uint8 [N, K/2] with i4), weight_scale fp32 [N], bias fp16 [N], res = (R [M, N], G [M/L, N], L)
    fp16 for the gated residual R + G * y. Returns fp16 [M, N]."""
    x = _c(x, F16)
    M = x.shape[0]
    wt = _c(weight, np.uint8 if i4 else np.int8)
    N, row_bytes = wt.shape
    K = row_bytes * 2 if i4 else row_bytes
    ap, scale = _quantized(M, row_bytes)
    r = lib()
    if i4:
        r.ref_rot_quant_pack_a_i4(_p(x), _p(ap), _p(scale), M, K)
    elif kind == "plain":
        r.ref_quant_pack_a(_p(x), _p(ap), _p(scale), M, K)
    elif kind == "rotate":
        r.ref_rot_quant_pack_a(_p(x), _p(ap), _p(scale), M, K)
    elif kind == "situ":
        r.ref_situ_rot_quant_pack_a(_p(x), _p(ap), _p(scale), M, K)
    elif kind in ("swiglu", "gate"):
        uu = _c(u, F16)
        fn = r.ref_swiglu_rot_quant_pack_a if kind == "swiglu" else r.ref_gate_rot_quant_pack_a
        fn(_p(x), _p(uu), _p(ap), _p(scale), M, K)
    elif kind == "mod":
        wf, sf, tf = _c(mod["w"], F32), _c(mod["s"], F16), _c(mod["t"], F16)
        r.ref_mod_rot_quant_pack_a(_p(x), _p(ap), _p(scale), M, K, _p(wf), _p(sf), _p(tf), mod["L"], F32(mod["eps"]))
    else:
        raise ValueError(kind)
    variant = 1 if i4 else (2 if row_bytes == 6144 else 0)
    if variant == 2:
        bp = wt
    else:
        bp = np.zeros(N * row_bytes, np.uint8)
        r.ref_pack_b(_p(wt), _p(bp), N, row_bytes)
    out = np.zeros((M, N), F16)
    ws = _c(weight_scale, F32)
    b = None if bias is None else _c(bias, F16)
    R = G = None
    L = 1
    if res is not None:
        R, G, L = _c(res[0], F16), _c(res[1], F16), int(res[2])
    r.ref_gemm(variant, _p(ap), _p(bp), _p(scale), _p(ws), _p(b), _p(out), M, N, row_bytes // 64, _p(R), _p(G), L)
    return out


# ---------------------------------------------------------------- hip_attention.hip
def attention(q, k, v, scale, int8_qk=False):
    """hip_attention.py attention(): pack_kv(_i8) then attn(_i8), on fp16 (B, H, L, 128) arrays (k, v may have fewer
    heads). Returns fp16 (B, H, Lq, 128)."""
    q, k, v = _c(q, F16), _c(k, F16), _c(v, F16)
    B, H, Lq, D = q.shape
    Hkv, Lk = k.shape[1], k.shape[2]
    assert D == 128
    groups = (Lk + 15) // 16
    packed = np.zeros(B * Hkv * (groups + 1) * (1552 if int8_qk else 2048), np.int32)
    out = np.zeros(q.shape, F16)
    r = lib()
    es = lambda a: [int(st // 2) for st in a.strides[:3]]  # noqa: E731  element strides (b, h, l)
    r.ref_pack_kv(int(int8_qk), _p(k), _p(v), _p(packed), B, Lk, groups, Hkv, *es(k), *es(v))
    r.ref_attn(int(int8_qk), _p(q), _p(packed), _p(out), B, Lq, Lk, groups, H, H // Hkv, *es(q), *es(out),
               F32(scale * math.log2(math.e)))
    return out


# ---------------------------------------------------------------- int8_gemv.hip
def rotate(x, group):
    """int8_gemv.py rotate(): fp32 regular-Hadamard rotation of every `group` values, times rsqrt(group)."""
    x = _c(x, F32)
    out = np.zeros_like(x)
    lib().ref_rotate(_p(x), _p(out), x.size, group)
    return out


def gemv_i8(x, w, scale, bias=None):
    """int8_gemv.py linear_forward's kernel: out[n] = scale[n] * dot(w[n], x) (+ bias[n]), fp32. K % 512 == 0 and
    N % 16 == 0 (int8_gemv.py:135)."""
    x, w, s = _c(x, F32).reshape(-1), _c(w, np.int8), _c(scale, F32)
    N, K = w.shape
    out = np.zeros(N, F32)
    b = None if bias is None else _c(bias, F32)
    lib().ref_gemv_i8(_p(x), _p(w), _p(s), _p(b), _p(out), N, K)
    return out


def gemv_bf16(x, w_bits):
    """int8_gemv.py logits()'s kernel: out[n] = dot(w[n], x) for a bf16 table given as uint16 bit patterns."""
    x, w = _c(x, F32).reshape(-1), _c(w_bits, np.uint16)
    N, K = w.shape
    out = np.zeros(N, F32)
    lib().ref_gemv_bf16(_p(x), _p(w), _p(out), N, K)
    return out


def attn_decode(q, k, v, lengths, scale=128 ** -0.5):
    """int8_gemv.py attention_decode(): q (B, 1, H, 128), k/v (B, capacity, Hkv, 128) fp32, lengths (B,) int32;
    split-32 attention then the merge. GQA of 4 query heads per KV head (GROUPS, int8_gemv.hip:12)."""
    q, k, v = _c(q, F32), _c(k, F32), _c(v, F32)
    ln = _c(lengths, np.int32)
    B, _, H, _ = q.shape
    cap, Hkv = k.shape[1], k.shape[2]
    assert H == 4 * Hkv, "the reference kernel serves 4 query heads per KV head"
    partial = np.zeros((B * H, 32, 128), F32)
    stats = np.zeros((B * H, 32, 2), F32)
    out = np.zeros_like(q)
    lib().ref_attn_decode(_p(q), _p(k), _p(v), _p(ln), _p(partial), _p(stats), _p(out), B, H, Hkv, cap, F32(scale))
    return out


# ---------------------------------------------------------------- rms_norm.hip
def rms_norm(x, w, eps):
    """rms_norm.py rms_norm() on a contiguous fp16 (B, L, D) or (B, H, L, D) array; w fp32 (D,) zero-centred."""
    x = _c(x, F16)
    v = x if x.ndim == 4 else x[:, None]
    B, H, L, D = v.shape
    sb, sh, sl = (int(st // 2) for st in v.strides[:3])
    out = np.zeros(x.shape, F16)
    wf = _c(w, F32)
    lib().ref_rms_norm(_p(x), _p(wf), _p(out), B * H * L, D, L, H, sb, sh, sl, F32(eps))
    return out


def rms_norm_rope(x, heads, w, eps, freqs):
    """rms_norm.py rms_norm_rope(): x fp16 (B, L, heads * 128) -> (B, heads, L, 128) with QK-norm and rope; freqs fp32
    (B or 1, 1, L, 64, 2, 2)."""
    x = _c(x, F16)
    B, L, _ = x.shape
    f = _c(freqs, F32)
    out = np.zeros((B, heads, L, 128), F16)
    wf = _c(w, F32)
    fb = L * 64 if f.shape[0] > 1 else 0
    lib().ref_rms_norm_rope(_p(x), _p(wf), _p(out), B * heads * L, 128, L, heads, x.shape[1] * x.shape[2], 128,
                            x.shape[2], F32(eps), _p(f), fb)
    return out
