"""Tensor-level wrappers of the C-ABI: shape/dtype checks, output allocation by the caller side (as the
reference allocates with torch.empty, e.g. int8_gemm.py:51-53,60), launch on torch's current stream."""
import math

import torch

from . import _lib
from ._lib import F, I, I64, call, ptr, require_cuda, stream

ROT_NONE, ROT_BLOCK128, ROT_CONVROT = 0, 128, 256


def _half2d(x, name):
    if x.dtype != torch.float16 or x.dim() != 2 or x.stride(-1) != 1:
        raise RuntimeError(f"{name} must be a 2D fp16 tensor with a contiguous last dimension")


def quant_pack_a(x, rot_group=ROT_NONE, out=None):
    """Per-row int8 of fp16 rows x [M, K] after an optional rotation. Returns (int8 [M, K], fp32 [M])."""
    require_cuda(x)
    _half2d(x, "x")
    M, K = x.shape
    q, s = out if out is not None else (torch.empty((M, K), dtype=torch.int8, device=x.device),
                                        torch.empty((M,), dtype=torch.float32, device=x.device))
    call("b2_quant_pack_a", ptr(x), I64(x.stride(0)), ptr(q), ptr(s), I(M), I(K), I(rot_group), stream())
    return q, s


def quant_pack_a_segments(x, K, rot_group, seg, seg_stride, M, ldx, out=None):
    """Rows gathered from segments: element k of row m sits at x[m*ldx + (k//seg)*seg_stride + k%seg]."""
    require_cuda(x)
    q, s = out if out is not None else (torch.empty((M, K), dtype=torch.int8, device=x.device),
                                        torch.empty((M,), dtype=torch.float32, device=x.device))
    call("b2_quant_pack_a_seg", ptr(x), I64(ldx), I(seg), I64(seg_stride), ptr(q), ptr(s), I(M), I(K), I(rot_group),
         stream())
    return q, s


def swiglu_quant_pack_a(gate, up, rot_group=ROT_NONE, act_out=None, out=None):
    """int8 of fp16(fp16(silu(gate)) * up) after an optional rotation. gate, up fp16 [M, K] with equal strides."""
    require_cuda(gate, up)
    _half2d(gate, "gate")
    _half2d(up, "up")
    if gate.shape != up.shape or gate.stride(0) != up.stride(0):
        raise RuntimeError("gate and up must have the same shape and row stride")
    M, K = gate.shape
    q, s = out if out is not None else (torch.empty((M, K), dtype=torch.int8, device=gate.device),
                                        torch.empty((M,), dtype=torch.float32, device=gate.device))
    call("b2_swiglu_quant_pack_a", ptr(gate), ptr(up), I64(gate.stride(0)), ptr(q), ptr(s), I(M), I(K), I(rot_group),
         ptr(act_out), stream())
    return q, s


def gate_quant_pack_a(x, gate, rot_group=ROT_NONE, act_out=None, out=None):
    """int8 of fp16(x * fp16(sigmoid(gate))) after an optional rotation."""
    require_cuda(x, gate)
    _half2d(x, "x")
    _half2d(gate, "gate")
    if x.shape != gate.shape or x.stride(0) != gate.stride(0):
        raise RuntimeError("x and gate must have the same shape and row stride")
    M, K = x.shape
    q, s = out if out is not None else (torch.empty((M, K), dtype=torch.int8, device=x.device),
                                        torch.empty((M,), dtype=torch.float32, device=x.device))
    call("b2_gate_quant_pack_a", ptr(x), ptr(gate), I64(x.stride(0)), ptr(q), ptr(s), I(M), I(K), I(rot_group),
         ptr(act_out), stream())
    return q, s


def situ_quant_pack_a(x, rot_group=ROT_NONE, act_out=None, out=None):
    """int8 of the situ activation fp16(4 tanh(g/4) sigmoid(g) 25 tanh(h/25)) after an optional rotation. x fp16
    [M, 2K] holds [h | g] per row; the result is [M, K]."""
    require_cuda(x)
    _half2d(x, "x")
    M, K2 = x.shape
    if K2 % 2:
        raise RuntimeError("situ input rows must be [hidden | gate], an even width")
    K = K2 // 2
    q, s = out if out is not None else (torch.empty((M, K), dtype=torch.int8, device=x.device),
                                        torch.empty((M,), dtype=torch.float32, device=x.device))
    call("b2_situ_quant_pack_a", ptr(x), I64(x.stride(0)), ptr(q), ptr(s), I(M), I(K), I(rot_group), ptr(act_out),
         stream())
    return q, s


def mod_quant_pack_a(x, weight, s_rows, t_rows, L, eps, rot_group=ROT_NONE, act_out=None, out=None):
    """int8 of the modulated RMSNorm fp16(fp16(fp16(x*rstd*(w+1)) * s) + t) after an optional rotation.
    x fp16 [M, K]; weight fp32 [K]; s_rows (= 1 + scale), t_rows fp16 [M // L, K]."""
    require_cuda(x, weight, s_rows, t_rows)
    _half2d(x, "x")
    M, K = x.shape
    for t, n in ((s_rows, "scale"), (t_rows, "shift")):
        if t.dtype != torch.float16 or not t.is_contiguous() or t.numel() < ((M + L - 1) // L) * K:
            raise RuntimeError(f"modulation {n} must be contiguous fp16 [M / L, K]")
    if weight.dtype != torch.float32 or not weight.is_contiguous() or weight.numel() != K:
        raise RuntimeError("norm weight must be contiguous fp32 [K]")
    q, s = out if out is not None else (torch.empty((M, K), dtype=torch.int8, device=x.device),
                                        torch.empty((M,), dtype=torch.float32, device=x.device))
    call("b2_mod_quant_pack_a", ptr(x), I64(x.stride(0)), ptr(weight), ptr(s_rows), ptr(t_rows), I(L), F(eps), ptr(q),
         ptr(s), I(M), I(K), I(rot_group), ptr(act_out), stream())
    return q, s


def gemm(a_q, a_scale, w_q, w_scale, bias=None, residual=None, gate=None, L=1, out=None):
    """fp16 [M, N] = (a_q . w_q^T) * a_scale[m] * w_scale[n] (+ bias) (, residual + gate * y)."""
    require_cuda(a_q, a_scale, w_q, w_scale, bias, residual, gate)
    M, K = a_q.shape
    N = w_q.shape[0]
    if a_q.dtype != torch.int8 or w_q.dtype != torch.int8 or w_q.shape[1] != K:
        raise RuntimeError("gemm operands must be int8 [M, K] and [N, K]")
    if not (a_q.is_contiguous() and w_q.is_contiguous()):
        raise RuntimeError("gemm operands must be contiguous")
    if a_scale.dtype != torch.float32 or w_scale.dtype != torch.float32:
        raise RuntimeError("gemm scales must be fp32")
    if bias is not None and (bias.dtype != torch.float16 or not bias.is_contiguous()):
        raise RuntimeError("gemm bias must be contiguous fp16")
    if residual is not None:
        if gate is None:
            gate = torch.ones((1, N), dtype=torch.float16, device=a_q.device)
            L = max(M, 1)
        if residual.dtype != torch.float16 or not residual.is_contiguous() or residual.shape != (M, N):
            raise RuntimeError("residual must be contiguous fp16 [M, N]")
        if gate.dtype != torch.float16 or not gate.is_contiguous() or gate.shape[-1] != N:
            raise RuntimeError("gate must be contiguous fp16 [M / L, N]")
        if L < 1 or gate.numel() // N < (M + L - 1) // L:
            raise RuntimeError(f"gate has {gate.numel() // N} rows, the {M} output rows need {(M + L - 1) // L} with L={L}")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=a_q.device)
    call("b2_gemm", ptr(a_q), ptr(w_q), ptr(a_scale), ptr(w_scale.contiguous()), ptr(bias), ptr(out), I(M), I(N), I(K),
         ptr(residual), ptr(gate if residual is not None else None), I(L), stream())
    return out


def gemm_i32(a_q, w_q):
    """Raw int32 accumulators of the W8A8 kernel, [M, N]."""
    require_cuda(a_q, w_q)
    M, K = a_q.shape
    N = w_q.shape[0]
    out = torch.empty((M, N), dtype=torch.int32, device=a_q.device)
    call("b2_gemm_i32", ptr(a_q.contiguous()), ptr(w_q.contiguous()), ptr(out), I(M), I(N), I(K), stream())
    return out


def swiglu_interleave(n2, device=None):
    """Row order of a gate/up weight [2F, K] for gemm_swiglu: gate rows and up rows alternate in blocks of 128
    (returns the natural row index of each interleaved row)."""
    F = n2 // 2
    if n2 % 256:
        raise RuntimeError(f"gemm_swiglu needs 2F % 256 == 0 (got {n2})")
    blk = torch.arange(F // 128).repeat_interleave(128) * 128 + torch.arange(128).repeat(F // 128)
    idx = torch.stack((blk.view(-1, 128), (blk + F).view(-1, 128)), 1).reshape(-1)
    return idx.to(device) if device is not None else idx


def gemm_swiglu(a_q, a_scale, w_q, w_scale, out=None):
    """fp16 [M, F] = SwiGLU(gate, up) of the gate/up projection, in the GEMM's epilogue. w_q int8 [2F, K] and
    w_scale fp32 [2F] in the order of swiglu_interleave."""
    require_cuda(a_q, a_scale, w_q, w_scale)
    M, K = a_q.shape
    N = w_q.shape[0]
    if a_q.dtype != torch.int8 or w_q.dtype != torch.int8 or w_q.shape[1] != K:
        raise RuntimeError("gemm_swiglu operands must be int8 [M, K] and [2F, K]")
    if not (a_q.is_contiguous() and w_q.is_contiguous()):
        raise RuntimeError("gemm_swiglu operands must be contiguous")
    if a_scale.dtype != torch.float32 or w_scale.dtype != torch.float32:
        raise RuntimeError("gemm_swiglu scales must be fp32")
    if out is None:
        out = torch.empty((M, N // 2), dtype=torch.float16, device=a_q.device)
    call("b2_gemm_swiglu", ptr(a_q), ptr(w_q), ptr(a_scale), ptr(w_scale.contiguous()), ptr(out), I(M), I(N), I(K),
         stream())
    return out


def w4a8_scales(scales_fp16):
    """fp16 group scales [N, K/128] -> the kernel's fp32 [K/128, N] (exact widening, done once per weight)."""
    return scales_fp16.to(torch.float32).t().contiguous()


def gemm_w4a8(a_q, a_scale, w_packed, gscale, bias=None, out=None):
    """fp16 [M, N] = sum over groups of int32 (a_q . w^T)_g * gscale[g, n], times a_scale[m] (+ bias).
    w_packed uint8 [N, K/2] (low nibble = even k); gscale fp32 [K/128, N] (see w4a8_scales)."""
    require_cuda(a_q, a_scale, w_packed, gscale, bias)
    M, K = a_q.shape
    N = w_packed.shape[0]
    if a_q.dtype != torch.int8 or w_packed.dtype != torch.uint8 or w_packed.shape[1] * 2 != K:
        raise RuntimeError("gemm_w4a8 operands must be int8 [M, K] and packed uint8 [N, K/2]")
    if gscale.dtype != torch.float32 or gscale.shape != (K // 128, N) or not gscale.is_contiguous():
        raise RuntimeError("gemm_w4a8 scales must be contiguous fp32 [K/128, N]")
    if bias is not None and (bias.dtype != torch.float16 or not bias.is_contiguous()):
        raise RuntimeError("gemm_w4a8 bias must be contiguous fp16")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=a_q.device)
    call("b2_gemm_w4a8", ptr(a_q.contiguous()), ptr(w_packed.contiguous()), ptr(a_scale), ptr(gscale), ptr(bias),
         ptr(out), I(M), I(N), I(K), stream())
    return out


def quant_pack_a_i4(x, rot_group=ROT_CONVROT, out=None):
    """Per-row int4-valued activations of fp16 rows x [M, K] after an optional rotation: scale = max(absmax, 1e-10)
    / 7, q = clamp(rint(y / scale), -7, 7), one int8 per value. Returns (int8 [M, K], fp32 [M])."""
    require_cuda(x)
    _half2d(x, "x")
    M, K = x.shape
    q, s = out if out is not None else (torch.empty((M, K), dtype=torch.int8, device=x.device),
                                        torch.empty((M,), dtype=torch.float32, device=x.device))
    call("b2_quant_pack_a_i4", ptr(x), I64(x.stride(0)), ptr(q), ptr(s), I(M), I(K), I(rot_group), stream())
    return q, s


def _packed_int4(w_packed, name):
    if w_packed.dtype not in (torch.uint8, torch.int8) or w_packed.dim() != 2 or not w_packed.is_contiguous():
        raise RuntimeError(f"{name}: the packed weight must be a contiguous 8-bit [N, K/2] tensor")


def unpack_int4(w_packed, out=None):
    """Packed int4 [N, K/2] (low nibble = even k, two's complement) -> int8 [N, K]."""
    require_cuda(w_packed)
    _packed_int4(w_packed, "unpack_int4")
    N, K = w_packed.shape[0], w_packed.shape[1] * 2
    out = torch.empty((N, K), dtype=torch.int8, device=w_packed.device) if out is None else out
    call("b2_unpack_int4", ptr(w_packed), ptr(out), I(N), I(K), stream())
    return out


def gemm_w4a4(a_q, a_scale, w_packed, w_scale, bias=None, out=None, workspace=None):
    """Per-channel W4A4: fp16 [M, N] = int32 (a_q . w^T) * a_scale[m] * w_scale[n] (+ bias), a_q int8 [M, K] with
    int4 values, w_packed [N, K/2]. ``workspace`` (int8, N * K bytes) receives the widened weight; allocated here
    when not given."""
    require_cuda(a_q, a_scale, w_packed, w_scale, bias)
    _packed_int4(w_packed, "gemm_w4a4")
    M, K = a_q.shape
    N = w_packed.shape[0]
    if a_q.dtype != torch.int8 or w_packed.shape[1] * 2 != K or not a_q.is_contiguous():
        raise RuntimeError("gemm_w4a4 operands must be contiguous int8 [M, K] and packed [N, K/2]")
    if w_scale.dtype != torch.float32 or w_scale.numel() != N or not w_scale.is_contiguous():
        raise RuntimeError("gemm_w4a4 weight scale must be contiguous fp32 [N]")
    if bias is not None and (bias.dtype != torch.float16 or not bias.is_contiguous()):
        raise RuntimeError("gemm_w4a4 bias must be contiguous fp16")
    if workspace is None:
        workspace = torch.empty((N * K,), dtype=torch.int8, device=a_q.device)
    elif workspace.dtype != torch.int8 or workspace.numel() < N * K or not workspace.is_contiguous():
        raise RuntimeError("gemm_w4a4 workspace must be contiguous int8 of at least N * K bytes")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=a_q.device)
    call("b2_gemm_w4a4", ptr(a_q), ptr(w_packed), ptr(a_scale), ptr(w_scale), ptr(bias), ptr(out), I(M), I(N), I(K),
         ptr(workspace), stream())
    return out


def attention(q, k, v, out, scale, int8_qk=False, workspace=None):
    """Fused attention on (B, H, L, 128) fp16 views with a contiguous last dimension; writes ``out``."""
    require_cuda(q, k, v, out)
    B, H, Lq, D = q.shape
    _, Hkv, Lk, _ = k.shape
    if D != 128 or k.shape[-1] != 128 or v.shape[-1] != 128 or out.shape != q.shape:
        raise RuntimeError("attention needs head dim 128 and out shaped like q")
    for t in (q, k, v, out):
        if t.dtype != torch.float16 or t.stride(-1) != 1:
            raise RuntimeError("attention tensors must be fp16 with a contiguous last dimension")
    ws_bytes = _lib.load().b2_attention_workspace_bytes(B, H, Hkv, Lq, Lk, int(bool(int8_qk)))
    if ws_bytes and (workspace is None or workspace.numel() < ws_bytes):
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    call("b2_attention", ptr(q), *map(I64, q.stride()[:3]), ptr(k), *map(I64, k.stride()[:3]), ptr(v),
         *map(I64, v.stride()[:3]), ptr(out), *map(I64, out.stride()[:3]), I(B), I(H), I(Hkv), I(Lq), I(Lk), F(scale),
         I(int(bool(int8_qk))), ptr(workspace if ws_bytes else None), I64(ws_bytes), stream())
    return out


def rms_norm_rows(x, weight, eps, rows, D, L, H, sb, sh, sl, out, freqs=None, fb=0):
    require_cuda(x, weight, out, freqs)
    if freqs is None:
        call("b2_rms_norm", ptr(x), ptr(weight), ptr(out), I(rows), I(D), I(L), I(H), I64(sb), I64(sh), I64(sl), F(eps),
             stream())
    else:
        call("b2_rms_norm_rope", ptr(x), ptr(weight), ptr(out), I(rows), I(D), I(L), I(H), I64(sb), I64(sh), I64(sl),
             F(eps), ptr(freqs), I64(fb), stream())
    return out


def rotate(x, group, out=None):
    require_cuda(x)
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise RuntimeError("rotate needs contiguous fp32")
    out = torch.empty_like(x) if out is None else out
    call("b2_rotate", ptr(x), ptr(out), I64(x.numel()), I(group), stream())
    return out


def gemv_i8(x, w, scale, bias=None, out=None):
    """fp32 [N] = scale * (w int8 [N, K] . x fp32 [K]) (+ bias)."""
    require_cuda(x, w, scale, bias)
    N, K = w.shape
    if x.dtype != torch.float32 or x.numel() != K or not x.is_contiguous():
        raise RuntimeError("gemv_i8 needs one contiguous fp32 row of K values")
    out = torch.empty((N,), dtype=torch.float32, device=x.device) if out is None else out
    call("b2_gemv_i8", ptr(x), ptr(w), ptr(scale), ptr(bias), ptr(out), I(N), I(K), stream())
    return out


def gemv_i8_ex(x, w, scale, bias=None, residual=None, silu_mul=False, out=None):
    """gemv_i8 for the decode step: with silu_mul, x = [gate | up] (2K values) and the input is silu(gate) * up;
    with a residual, the result is residual + y."""
    require_cuda(x, w, scale, bias, residual)
    N, K = w.shape
    if x.dtype != torch.float32 or x.numel() != (2 * K if silu_mul else K) or not x.is_contiguous():
        raise RuntimeError("gemv_i8_ex needs one contiguous fp32 row of K (2K with silu_mul) values")
    out = torch.empty((N,), dtype=torch.float32, device=x.device) if out is None else out
    call("b2_gemv_i8_ex", ptr(x), ptr(w), ptr(scale), ptr(bias), ptr(residual), ptr(out), I(N), I(K), I(1 if silu_mul else 0),
         stream())
    return out


def gemv_bf16(x, w, out=None):
    """fp32 [N] = w bf16 [N, K] . x fp32 [K] (the logits of a tied-embedding decoder)."""
    require_cuda(x, w)
    if w.dtype != torch.bfloat16 or w.dim() != 2 or not w.is_contiguous():
        raise RuntimeError("gemv_bf16 needs a contiguous bf16 [N, K] table")
    N, K = w.shape
    if x.dtype != torch.float32 or x.numel() != K or not x.is_contiguous():
        raise RuntimeError("gemv_bf16 needs one contiguous fp32 row of K values")
    out = torch.empty((N,), dtype=torch.float32, device=x.device) if out is None else out
    call("b2_gemv_bf16", ptr(x), ptr(w), ptr(out), I(N), I(K), stream())
    return out


def rms_norm_f32(x, w, eps, out=None):
    """One fp32 row: x * rsqrt(mean(x^2) + eps) * w."""
    require_cuda(x, w)
    out = torch.empty_like(x) if out is None else out
    call("b2_rms_norm_f32", ptr(x), ptr(w), ptr(out), I(x.numel()), F(eps), stream())
    return out


def decode_qk_rope(qkv, q_norm, k_norm, inv_freq, pos, q_out, k_cache, v_cache, heads, kv_heads, eps):
    """q/k RMSNorm + rotary at device position pos (int64 [1]) for one token; k and v into the caches' row pos."""
    require_cuda(qkv, q_norm, k_norm, inv_freq, pos, q_out, k_cache, v_cache)
    if pos.dtype != torch.int64 or not all(t.is_contiguous() for t in (qkv, q_out, k_cache, v_cache)):
        raise RuntimeError("decode_qk_rope needs contiguous fp32 buffers and an int64 position")
    call("b2_decode_qk_rope", ptr(qkv), ptr(q_norm), ptr(k_norm), ptr(inv_freq), ptr(pos), ptr(q_out), ptr(k_cache),
         ptr(v_cache), I(heads), I(kv_heads), F(eps), stream())
    return q_out


DECODE_SPLITS = 32


def attn_decode(q, k, v, lengths, scale, out=None, partial=None, stats=None):
    """q [B,1,H,128], k/v [B,cap,Hkv,128] fp32 contiguous, lengths int32 [B] on the device."""
    require_cuda(q, k, v, lengths)
    B, _, H, D = q.shape
    _, cap, Hkv, _ = k.shape
    q = q.contiguous()
    out = torch.empty_like(q) if out is None else out
    if partial is None:
        partial = torch.empty((B * H, DECODE_SPLITS, 128), dtype=torch.float32, device=q.device)
    if stats is None:
        stats = torch.empty((B * H, DECODE_SPLITS, 2), dtype=torch.float32, device=q.device)
    call("b2_attn_decode", ptr(q), ptr(k), ptr(v), ptr(lengths), ptr(out), ptr(partial), ptr(stats), I(B), I(H),
         I(Hkv), I(cap), F(scale), stream())
    return out


def default_scale():
    return 1.0 / math.sqrt(128)
