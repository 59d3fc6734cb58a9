"""Tensor-level wrappers of the C-ABI: shape/dtype checks, output allocation by the caller side (as the
reference allocates with torch.empty, e.g. int8_gemm.py:51-53,60), launch on torch's current stream.

The C-ABI receives bare pointers and sizes, so it cannot see how large a buffer is: every wrapper here checks that
each tensor it passes has the dtype, layout and element count the kernel will index (outputs included) before
anything reaches the device, and raises ``RuntimeError`` naming the tensor otherwise. These checks run before the
CUDA-tensor check, so they hold (and are tested) without a GPU.
"""
import ctypes
import math

import torch

from . import _lib
from ._lib import F, I, I64, call, ptr, require_cuda, stream

ROT_NONE, ROT_BLOCK128, ROT_CONVROT = 0, 128, 256
DECODE_SPLITS = 32
HEAD_DIM = 128


# ---------------------------------------------------------------- argument checks
def _fail(msg):
    raise RuntimeError(msg)


def _half2d(x, name):
    if x.dtype != torch.float16 or x.dim() != 2 or x.stride(-1) != 1:
        _fail(f"{name} must be a 2D fp16 tensor with a contiguous last dimension")


def _vec(t, n, dtype, name):
    """t (optional): contiguous ``dtype`` with at least n elements."""
    if t is not None and (t.dtype != dtype or not t.is_contiguous() or t.numel() < n):
        _fail(f"{name} must be contiguous {dtype} with at least {n} elements (got {t.dtype}, {t.numel()})")


def _exact(t, shape, dtype, name):
    """t (optional): contiguous ``dtype`` holding exactly prod(shape) elements (any view of that shape)."""
    n = math.prod(shape)
    if t is not None and (t.dtype != dtype or not t.is_contiguous() or t.numel() != n):
        _fail(f"{name} must be contiguous {dtype} of shape {tuple(shape)} (got {t.dtype}, {tuple(t.shape)})")


def _quant_out(out, M, K, device):
    """The (q [M, K] int8, scale [M] fp32) pair of a pre-pass: allocated when not given, else checked."""
    if out is None:
        return (torch.empty((M, K), dtype=torch.int8, device=device),
                torch.empty((M,), dtype=torch.float32, device=device))
    q, s = out
    _exact(q, (M, K), torch.int8, "quantized output")
    _vec(s, M, torch.float32, "scale output")
    return q, s


# ---------------------------------------------------------------- activation pre-pass
def quant_pack_a(x, rot_group=ROT_NONE, out=None):
    """Per-row int8 of fp16 rows x [M, K] after an optional rotation. Returns (int8 [M, K], fp32 [M])."""
    _half2d(x, "x")
    M, K = x.shape
    q, s = _quant_out(out, M, K, x.device)
    require_cuda(x, q, s)
    call("b2_quant_pack_a", ptr(x), I64(x.stride(0)), ptr(q), ptr(s), I(M), I(K), I(rot_group), stream())
    return q, s


def quant_pack_a_segments(x, K, rot_group, seg, seg_stride, M, ldx, out=None):
    """Rows gathered from segments: element k of row m sits at x[m*ldx + (k//seg)*seg_stride + k%seg]."""
    if x.dtype != torch.float16 or not x.is_contiguous():
        _fail("x must be contiguous fp16")
    if seg <= 0 or K % seg:
        _fail(f"segment width {seg} must divide K={K}")
    if M > 0 and (M - 1) * ldx + (K // seg - 1) * seg_stride + seg > x.numel():
        _fail(f"segments reach past the {x.numel()} values of x")
    q, s = _quant_out(out, M, K, x.device)
    require_cuda(x, q, s)
    call("b2_quant_pack_a_seg", ptr(x), I64(ldx), I(seg), I64(seg_stride), ptr(q), ptr(s), I(M), I(K), I(rot_group),
         stream())
    return q, s


def _two_inputs(a, b, an, bn):
    _half2d(a, an)
    _half2d(b, bn)
    if a.shape != b.shape or a.stride(0) != b.stride(0):
        _fail(f"{an} and {bn} must have the same shape and row stride")


def swiglu_quant_pack_a(gate, up, rot_group=ROT_NONE, act_out=None, out=None):
    """int8 of fp16(fp16(silu(gate)) * up) after an optional rotation. gate, up fp16 [M, K] with equal strides."""
    _two_inputs(gate, up, "gate", "up")
    M, K = gate.shape
    _exact(act_out, (M, K), torch.float16, "act_out")
    q, s = _quant_out(out, M, K, gate.device)
    require_cuda(gate, up, q, s, act_out)
    call("b2_swiglu_quant_pack_a", ptr(gate), ptr(up), I64(gate.stride(0)), ptr(q), ptr(s), I(M), I(K), I(rot_group),
         ptr(act_out), stream())
    return q, s


def gate_quant_pack_a(x, gate, rot_group=ROT_NONE, act_out=None, out=None):
    """int8 of fp16(x * fp16(sigmoid(gate))) after an optional rotation."""
    _two_inputs(x, gate, "x", "gate")
    M, K = x.shape
    _exact(act_out, (M, K), torch.float16, "act_out")
    q, s = _quant_out(out, M, K, x.device)
    require_cuda(x, gate, q, s, act_out)
    call("b2_gate_quant_pack_a", ptr(x), ptr(gate), I64(x.stride(0)), ptr(q), ptr(s), I(M), I(K), I(rot_group),
         ptr(act_out), stream())
    return q, s


def situ_quant_pack_a(x, rot_group=ROT_NONE, act_out=None, out=None):
    """int8 of the situ activation fp16(4 tanh(g/4) sigmoid(g) 25 tanh(h/25)) after an optional rotation. x fp16
    [M, 2K] holds [h | g] per row; the result is [M, K]."""
    _half2d(x, "x")
    M, K2 = x.shape
    if K2 % 2:
        _fail("situ input rows must be [hidden | gate], an even width")
    K = K2 // 2
    _exact(act_out, (M, K), torch.float16, "act_out")
    q, s = _quant_out(out, M, K, x.device)
    require_cuda(x, q, s, act_out)
    call("b2_situ_quant_pack_a", ptr(x), I64(x.stride(0)), ptr(q), ptr(s), I(M), I(K), I(rot_group), ptr(act_out),
         stream())
    return q, s


def mod_quant_pack_a(x, weight, s_rows, t_rows, L, eps, rot_group=ROT_NONE, act_out=None, out=None):
    """int8 of the modulated RMSNorm fp16(fp16(fp16(x*rstd*(w+1)) * s) + t) after an optional rotation.
    x fp16 [M, K]; weight fp32 [K]; s_rows (= 1 + scale), t_rows fp16 [M // L, K]; both None: the RMSNorm alone
    (the same int8 as s = 1, t = 0)."""
    _half2d(x, "x")
    M, K = x.shape
    if L < 1:
        _fail(f"L={L} must be at least 1")
    if (s_rows is None) != (t_rows is None):
        _fail("modulation scale and shift are both given or both None")
    for t, n in ((s_rows, "scale"), (t_rows, "shift")):
        if t is not None and (t.dtype != torch.float16 or not t.is_contiguous() or t.numel() < ((M + L - 1) // L) * K):
            _fail(f"modulation {n} must be contiguous fp16 [M / L, K]")
    if weight.dtype != torch.float32 or not weight.is_contiguous() or weight.numel() != K:
        _fail("norm weight must be contiguous fp32 [K]")
    _exact(act_out, (M, K), torch.float16, "act_out")
    q, s = _quant_out(out, M, K, x.device)
    require_cuda(x, weight, s_rows, t_rows, q, s, act_out)
    call("b2_mod_quant_pack_a", ptr(x), I64(x.stride(0)), ptr(weight), ptr(s_rows), ptr(t_rows), I(L), F(eps), ptr(q),
         ptr(s), I(M), I(K), I(rot_group), ptr(act_out), stream())
    return q, s


def quant_pack_a_i4(x, rot_group=ROT_CONVROT, out=None):
    """Per-row int4-valued activations of fp16 rows x [M, K] after an optional rotation: scale = max(absmax, 1e-10)
    / 7, q = clamp(rint(y / scale), -7, 7), one int8 per value. Returns (int8 [M, K], fp32 [M])."""
    _half2d(x, "x")
    M, K = x.shape
    q, s = _quant_out(out, M, K, x.device)
    require_cuda(x, q, s)
    call("b2_quant_pack_a_i4", ptr(x), I64(x.stride(0)), ptr(q), ptr(s), I(M), I(K), I(rot_group), stream())
    return q, s


# ---------------------------------------------------------------- W8A8 GEMM
def _gemm_operands(a_q, a_scale, w_q, w_scale, name):
    if a_q.dtype != torch.int8 or a_q.dim() != 2 or not a_q.is_contiguous():
        _fail(f"{name}: activations must be contiguous int8 [M, K]")
    if w_q.dtype != torch.int8 or w_q.dim() != 2 or not w_q.is_contiguous() or w_q.shape[1] != a_q.shape[1]:
        _fail(f"{name}: weight must be contiguous int8 [N, K] with the activations' K")
    M, K = a_q.shape
    N = w_q.shape[0]
    _vec(a_scale, M, torch.float32, f"{name}: activation scale")
    _vec(w_scale, N, torch.float32, f"{name}: weight scale")
    return M, N, K


def gemm(a_q, a_scale, w_q, w_scale, bias=None, residual=None, gate=None, L=1, out=None):
    """fp16 [M, N] = (a_q . w_q^T) * a_scale[m] * w_scale[n] (+ bias) (, residual + gate * y; without a gate,
    residual + y)."""
    M, N, K = _gemm_operands(a_q, a_scale, w_q, w_scale, "gemm")
    _vec(bias, N, torch.float16, "gemm bias")
    if gate is not None and residual is None:
        _fail("a gate needs a residual")
    if residual is not None:
        _exact(residual, (M, N), torch.float16, "residual")
    if gate is not None:
        if gate.dtype != torch.float16 or not gate.is_contiguous() or gate.shape[-1] != N:
            _fail("gate must be contiguous fp16 [M / L, N]")
        if L < 1 or gate.numel() // N < (M + L - 1) // L:
            _fail(f"gate has {gate.numel() // N} rows, the {M} output rows need {(M + L - 1) // L} with L={L}")
    _exact(out, (M, N), torch.float16, "gemm output")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=a_q.device)
    require_cuda(a_q, a_scale, w_q, w_scale, bias, residual, gate, out)
    call("b2_gemm", ptr(a_q), ptr(w_q), ptr(a_scale), ptr(w_scale), ptr(bias), ptr(out), I(M), I(N), I(K),
         ptr(residual), ptr(gate if residual is not None else None), I(L), stream())
    return out


def gemm_i32(a_q, w_q):
    """Raw int32 accumulators of the W8A8 kernel, [M, N]."""
    if a_q.dtype != torch.int8 or w_q.dtype != torch.int8 or a_q.dim() != 2 or w_q.dim() != 2 \
            or a_q.shape[1] != w_q.shape[1]:
        _fail("gemm_i32 operands must be int8 [M, K] and [N, K]")
    a_q, w_q = a_q.contiguous(), w_q.contiguous()
    M, K = a_q.shape
    N = w_q.shape[0]
    out = torch.empty((M, N), dtype=torch.int32, device=a_q.device)
    require_cuda(a_q, w_q, out)
    call("b2_gemm_i32", ptr(a_q), ptr(w_q), ptr(out), I(M), I(N), I(K), stream())
    return out


def swiglu_interleave(n2, device=None):
    """Row order of a gate/up weight [2F, K] for gemm_swiglu: gate rows and up rows alternate in blocks of 128
    (returns the natural row index of each interleaved row)."""
    F = n2 // 2
    if n2 % 256:
        _fail(f"gemm_swiglu needs 2F % 256 == 0 (got {n2})")
    blk = torch.arange(F // 128).repeat_interleave(128) * 128 + torch.arange(128).repeat(F // 128)
    idx = torch.stack((blk.view(-1, 128), (blk + F).view(-1, 128)), 1).reshape(-1)
    return idx.to(device) if device is not None else idx


def gemm_swiglu(a_q, a_scale, w_q, w_scale, out=None):
    """fp16 [M, F] = SwiGLU(gate, up) of the gate/up projection, in the GEMM's epilogue. w_q int8 [2F, K] and
    w_scale fp32 [2F] in the order of swiglu_interleave."""
    M, N, K = _gemm_operands(a_q, a_scale, w_q, w_scale, "gemm_swiglu")
    _exact(out, (M, N // 2), torch.float16, "gemm_swiglu output")
    if out is None:
        out = torch.empty((M, N // 2), dtype=torch.float16, device=a_q.device)
    require_cuda(a_q, a_scale, w_q, w_scale, out)
    call("b2_gemm_swiglu", ptr(a_q), ptr(w_q), ptr(a_scale), ptr(w_scale), ptr(out), I(M), I(N), I(K), stream())
    return out


# ---------------------------------------------------------------- int4 weights
def w4a8_scales(scales_fp16):
    """fp16 group scales [N, K/128] -> the kernel's fp32 [K/128, N] (exact widening, done once per weight)."""
    return scales_fp16.to(torch.float32).t().contiguous()


def _int8_rows(a_q, name):
    if a_q.dtype != torch.int8 or a_q.dim() != 2 or not a_q.is_contiguous():
        _fail(f"{name}: activations must be contiguous int8 [M, K]")
    return a_q.shape


def _packed_int4(w_packed, K, name):
    if w_packed.dtype not in (torch.uint8, torch.int8) or w_packed.dim() != 2 or not w_packed.is_contiguous():
        _fail(f"{name}: the packed weight must be a contiguous 8-bit [N, K/2] tensor")
    if K is not None and w_packed.shape[1] * 2 != K:
        _fail(f"{name}: the packed weight has {w_packed.shape[1] * 2} values per row, the activations {K}")


def gemm_w4a8(a_q, a_scale, w_packed, gscale, bias=None, out=None, w_wide=None):
    """fp16 [M, N] = sum over groups of int32 (a_q . w^T)_g * gscale[g, n], times a_scale[m] (+ bias).
    w_packed uint8 [N, K/2] (low nibble = even k); gscale fp32 [K/128, N] (see w4a8_scales). ``w_wide``, the same
    weight widened to int8 [N, K] (unpack_int4), selects the kernel that reads it instead; the result is the same
    bit for bit."""
    M, K = _int8_rows(a_q, "gemm_w4a8")
    _packed_int4(w_packed, K, "gemm_w4a8")
    N = w_packed.shape[0]
    if w_wide is not None and (w_wide.dtype != torch.int8 or tuple(w_wide.shape) != (N, K) or not w_wide.is_contiguous()):
        _fail(f"gemm_w4a8: the widened weight must be contiguous int8 [{N}, {K}]")
    _vec(a_scale, M, torch.float32, "gemm_w4a8 activation scale")
    if gscale.dtype != torch.float32 or tuple(gscale.shape) != (K // 128, N) or not gscale.is_contiguous():
        _fail("gemm_w4a8 scales must be contiguous fp32 [K/128, N]")
    _vec(bias, N, torch.float16, "gemm_w4a8 bias")
    _exact(out, (M, N), torch.float16, "gemm_w4a8 output")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=a_q.device)
    require_cuda(a_q, a_scale, w_packed, gscale, bias, out, w_wide)
    if w_wide is not None:
        call("b2_gemm_w4a8_wide", ptr(a_q), ptr(w_wide), ptr(a_scale), ptr(gscale), ptr(bias), ptr(out), I(M), I(N),
             I(K), stream())
    else:
        call("b2_gemm_w4a8", ptr(a_q), ptr(w_packed), ptr(a_scale), ptr(gscale), ptr(bias), ptr(out), I(M), I(N),
             I(K), stream())
    return out


def unpack_int4(w_packed, out=None):
    """Packed int4 [N, K/2] (low nibble = even k, two's complement) -> int8 [N, K]."""
    _packed_int4(w_packed, None, "unpack_int4")
    N, K = w_packed.shape[0], w_packed.shape[1] * 2
    _exact(out, (N, K), torch.int8, "unpack_int4 output")
    out = torch.empty((N, K), dtype=torch.int8, device=w_packed.device) if out is None else out
    require_cuda(w_packed, out)
    call("b2_unpack_int4", ptr(w_packed), ptr(out), I(N), I(K), stream())
    return out


def gemm_w4a4(a_q, a_scale, w_packed, w_scale, bias=None, out=None, workspace=None):
    """Per-channel W4A4: fp16 [M, N] = int32 (a_q . w^T) * a_scale[m] * w_scale[n] (+ bias), a_q int8 [M, K] with
    int4 values, w_packed [N, K/2]. ``workspace`` (int8, N * K bytes) receives the widened weight; allocated here
    when not given."""
    M, K = _int8_rows(a_q, "gemm_w4a4")
    _packed_int4(w_packed, K, "gemm_w4a4")
    N = w_packed.shape[0]
    _vec(a_scale, M, torch.float32, "gemm_w4a4 activation scale")
    _exact(w_scale, (N,), torch.float32, "gemm_w4a4 weight scale")
    _vec(bias, N, torch.float16, "gemm_w4a4 bias")
    _vec(workspace, N * K, torch.int8, "gemm_w4a4 workspace")
    _exact(out, (M, N), torch.float16, "gemm_w4a4 output")
    if workspace is None:
        workspace = torch.empty((N * K,), dtype=torch.int8, device=a_q.device)
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=a_q.device)
    require_cuda(a_q, a_scale, w_packed, w_scale, bias, workspace, out)
    call("b2_gemm_w4a4", ptr(a_q), ptr(w_packed), ptr(a_scale), ptr(w_scale), ptr(bias), ptr(out), I(M), I(N), I(K),
         ptr(workspace), stream())
    return out


# ---------------------------------------------------------------- attention
def attention(q, k, v, out, scale, int8_qk=False, workspace=None, gather=None):
    """Fused attention on (B, H, L, 128) fp16 views with a contiguous last dimension; writes ``out``. ``gather`` =
    (peer output addresses, peer counter addresses) also copies each finished tile to the peers' buffers at the
    same offsets and counts its arrival there (b2_attention_gather)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (out, "out")):
        if t.dim() != 4 or t.dtype != torch.float16 or t.stride(-1) != 1:
            _fail(f"attention {n} must be a 4D fp16 (B, H, L, 128) view with a contiguous last dimension")
    B, H, Lq, D = q.shape
    _, Hkv, Lk, _ = k.shape
    if D != HEAD_DIM or k.shape[-1] != HEAD_DIM or v.shape[-1] != HEAD_DIM or out.shape != q.shape:
        _fail("attention needs head dim 128 and out shaped like q")
    if k.shape[0] != B or v.shape != k.shape:
        _fail(f"attention k and v must be (B={B}, Hkv, Lk, 128) with equal shapes "
              f"(got {tuple(k.shape)}, {tuple(v.shape)})")
    if Hkv == 0 or H % Hkv:
        _fail(f"attention: {H} query heads do not group over {Hkv} KV heads")
    require_cuda(q, k, v, out, workspace)
    ws_bytes = _lib.load().b2_attention_workspace_bytes(B, H, Hkv, Lq, Lk, int(bool(int8_qk)))
    if ws_bytes and (workspace is None or not workspace.is_contiguous()
                     or workspace.numel() * workspace.element_size() < ws_bytes):
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    if gather is None:
        call("b2_attention", ptr(q), *map(I64, q.stride()[:3]), ptr(k), *map(I64, k.stride()[:3]), ptr(v),
             *map(I64, v.stride()[:3]), ptr(out), *map(I64, out.stride()[:3]), I(B), I(H), I(Hkv), I(Lq), I(Lk),
             F(scale), I(int(bool(int8_qk))), ptr(workspace if ws_bytes else None), I64(ws_bytes), stream())
    else:
        peer_out, peer_cnt = gather
        n = len(peer_out)
        if n != len(peer_cnt) or n > 7:
            _fail("attention gather needs one counter per peer buffer, at most 7 peers")
        po = (ctypes.c_void_p * max(n, 1))(*[ctypes.c_void_p(int(p)) for p in peer_out])
        pc = (ctypes.c_void_p * max(n, 1))(*[ctypes.c_void_p(int(c)) for c in peer_cnt])
        call("b2_attention_gather", ptr(q), *map(I64, q.stride()[:3]), ptr(k), *map(I64, k.stride()[:3]), ptr(v),
             *map(I64, v.stride()[:3]), ptr(out), *map(I64, out.stride()[:3]), I(B), I(H), I(Hkv), I(Lq), I(Lk),
             F(scale), I(int(bool(int8_qk))), ptr(workspace if ws_bytes else None), I64(ws_bytes), po, pc, I(n),
             stream())
    return out


def attention_gather_ctas(B, H, Lq):
    """Arrivals one attention_gather launch makes on each peer counter."""
    return _lib.load().b2_attention_gather_ctas(B, H, Lq)


def wait_count(cnt, expected, err, timeout_ns=2_000_000_000):
    """Stream-ordered wait until the int64 counter ``cnt`` (device) reaches ``expected``; sets ``err`` (int32,
    device) on timeout."""
    if cnt.dtype != torch.int64 or err.dtype != torch.int32:
        _fail("wait_count needs an int64 counter and an int32 error flag")
    require_cuda(cnt, err)
    call("b2_wait_count", ptr(cnt), ctypes.c_ulonglong(int(expected)), ptr(err), ctypes.c_longlong(int(timeout_ns)),
         stream())


# ---------------------------------------------------------------- RMSNorm
def rms_norm_rows(x, weight, eps, rows, D, L, H, sb, sh, sl, out, freqs=None, fb=0):
    """rows = B * H * L rows of D values, row (b, h, l) at x + b sb + h sh + l sl, into contiguous out. With freqs
    (fp32 (B or 1, 1, L, D/2, 2, 2)), the rope of position l follows the norm; fb = the batch stride of freqs in
    units of 4 values (0 when shared)."""
    if x.dtype != torch.float16 or x.stride(-1) != 1:
        _fail("rms_norm x must be fp16 with a contiguous last dimension")
    _vec(weight, D, torch.float32, "rms_norm weight")
    _vec(out, rows * D, torch.float16, "rms_norm output")
    if freqs is not None:
        batches = rows // max(H * L, 1)
        _vec(freqs, 4 * (max(batches - 1, 0) * fb + L * (D // 2)), torch.float32, "rope frequencies")
    require_cuda(x, weight, out, freqs)
    if freqs is None:
        call("b2_rms_norm", ptr(x), ptr(weight), ptr(out), I(rows), I(D), I(L), I(H), I64(sb), I64(sh), I64(sl), F(eps),
             stream())
    else:
        call("b2_rms_norm_rope", ptr(x), ptr(weight), ptr(out), I(rows), I(D), I(L), I(H), I64(sb), I64(sh), I64(sl),
             F(eps), ptr(freqs), I64(fb), stream())
    return out


# ---------------------------------------------------------------- single-token decode
def rotate(x, group, out=None):
    if x.dtype != torch.float32 or not x.is_contiguous():
        _fail("rotate needs contiguous fp32")
    _exact(out, tuple(x.shape), torch.float32, "rotate output")
    out = torch.empty_like(x) if out is None else out
    require_cuda(x, out)
    call("b2_rotate", ptr(x), ptr(out), I64(x.numel()), I(group), stream())
    return out


def _gemv_weight(w, dtype, name):
    if w.dtype != dtype or w.dim() != 2 or not w.is_contiguous():
        _fail(f"{name} needs a contiguous {dtype} [N, K] weight")
    return w.shape


def gemv_i8(x, w, scale, bias=None, out=None):
    """fp32 [N] = scale * (w int8 [N, K] . x fp32 [K]) (+ bias)."""
    N, K = _gemv_weight(w, torch.int8, "gemv_i8")
    if x.dtype != torch.float32 or x.numel() != K or not x.is_contiguous():
        _fail("gemv_i8 needs one contiguous fp32 row of K values")
    _vec(scale, N, torch.float32, "gemv_i8 scale")
    _vec(bias, N, torch.float32, "gemv_i8 bias")
    _vec(out, N, torch.float32, "gemv_i8 output")
    out = torch.empty((N,), dtype=torch.float32, device=x.device) if out is None else out
    require_cuda(x, w, scale, bias, out)
    call("b2_gemv_i8", ptr(x), ptr(w), ptr(scale), ptr(bias), ptr(out), I(N), I(K), stream())
    return out


def gemv_i8_ex(x, w, scale, bias=None, residual=None, silu_mul=False, out=None):
    """gemv_i8 for the decode step: with silu_mul, x = [gate | up] (2K values) and the input is silu(gate) * up;
    with a residual, the result is residual + y."""
    N, K = _gemv_weight(w, torch.int8, "gemv_i8_ex")
    if x.dtype != torch.float32 or x.numel() != (2 * K if silu_mul else K) or not x.is_contiguous():
        _fail("gemv_i8_ex needs one contiguous fp32 row of K (2K with silu_mul) values")
    _vec(scale, N, torch.float32, "gemv_i8_ex scale")
    _vec(bias, N, torch.float32, "gemv_i8_ex bias")
    _vec(residual, N, torch.float32, "gemv_i8_ex residual")
    _vec(out, N, torch.float32, "gemv_i8_ex output")
    out = torch.empty((N,), dtype=torch.float32, device=x.device) if out is None else out
    require_cuda(x, w, scale, bias, residual, out)
    call("b2_gemv_i8_ex", ptr(x), ptr(w), ptr(scale), ptr(bias), ptr(residual), ptr(out), I(N), I(K),
         I(1 if silu_mul else 0), stream())
    return out


def gemv_bf16(x, w, out=None):
    """fp32 [N] = w bf16 [N, K] . x fp32 [K] (the logits of a tied-embedding decoder)."""
    N, K = _gemv_weight(w, torch.bfloat16, "gemv_bf16")
    if x.dtype != torch.float32 or x.numel() != K or not x.is_contiguous():
        _fail("gemv_bf16 needs one contiguous fp32 row of K values")
    _vec(out, N, torch.float32, "gemv_bf16 output")
    out = torch.empty((N,), dtype=torch.float32, device=x.device) if out is None else out
    require_cuda(x, w, out)
    call("b2_gemv_bf16", ptr(x), ptr(w), ptr(out), I(N), I(K), stream())
    return out


def rms_norm_f32(x, w, eps, out=None):
    """One fp32 row: x * rsqrt(mean(x^2) + eps) * w."""
    if x.dtype != torch.float32 or not x.is_contiguous():
        _fail("rms_norm_f32 needs one contiguous fp32 row")
    D = x.numel()
    _vec(w, D, torch.float32, "rms_norm_f32 weight")
    _vec(out, D, torch.float32, "rms_norm_f32 output")
    out = torch.empty_like(x) if out is None else out
    require_cuda(x, w, out)
    call("b2_rms_norm_f32", ptr(x), ptr(w), ptr(out), I(D), F(eps), stream())
    return out


def decode_qk_rope(qkv, q_norm, k_norm, inv_freq, pos, q_out, k_cache, v_cache, heads, kv_heads, eps):
    """q/k RMSNorm + rotary at device position pos (int64 [1]) for one token; k and v into the caches' row pos.
    The position is read on the device: the caller keeps it below the caches' capacity."""
    d = HEAD_DIM
    if pos.dtype != torch.int64 or pos.numel() < 1:
        _fail("decode_qk_rope needs an int64 position")
    _vec(qkv, (heads + 2 * kv_heads) * d, torch.float32, "q|k|v row")
    _vec(q_norm, d, torch.float32, "q_norm")
    _vec(k_norm, d, torch.float32, "k_norm")
    _vec(inv_freq, d // 2, torch.float32, "inv_freq")
    _vec(q_out, heads * d, torch.float32, "q output")
    for c, n in ((k_cache, "k_cache"), (v_cache, "v_cache")):
        _vec(c, kv_heads * d, torch.float32, n)
        if c.numel() % (kv_heads * d):
            _fail(f"{n} must hold whole [kv_heads, 128] rows")
    require_cuda(qkv, q_norm, k_norm, inv_freq, pos, q_out, k_cache, v_cache)
    call("b2_decode_qk_rope", ptr(qkv), ptr(q_norm), ptr(k_norm), ptr(inv_freq), ptr(pos), ptr(q_out), ptr(k_cache),
         ptr(v_cache), I(heads), I(kv_heads), F(eps), stream())
    return q_out


def attn_decode(q, k, v, lengths, scale, out=None, partial=None, stats=None):
    """q [B,1,H,128], k/v [B,cap,Hkv,128] fp32 contiguous, lengths int32 [B] on the device."""
    if q.dim() != 4 or k.dim() != 4 or q.shape[1] != 1 or q.shape[-1] != HEAD_DIM or k.shape[-1] != HEAD_DIM:
        _fail("attn_decode needs q (B, 1, H, 128) and k, v (B, capacity, Hkv, 128)")
    B, _, H, _ = q.shape
    _, cap, Hkv, _ = k.shape
    if k.shape[0] != B or v.shape != k.shape:
        _fail(f"attn_decode k and v must be (B={B}, capacity, Hkv, 128) with equal shapes")
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        if t.dtype != torch.float32:
            _fail(f"attn_decode {n} must be fp32")
    if not (k.is_contiguous() and v.is_contiguous()):
        _fail("attn_decode k and v must be contiguous")
    _vec(lengths, B, torch.int32, "lengths")
    q = q.contiguous()
    _exact(out, tuple(q.shape), torch.float32, "attn_decode output")
    _vec(partial, B * H * DECODE_SPLITS * HEAD_DIM, torch.float32, "attn_decode partial")
    _vec(stats, B * H * DECODE_SPLITS * 2, torch.float32, "attn_decode stats")
    out = torch.empty_like(q) if out is None else out
    if partial is None:
        partial = torch.empty((B * H, DECODE_SPLITS, HEAD_DIM), dtype=torch.float32, device=q.device)
    if stats is None:
        stats = torch.empty((B * H, DECODE_SPLITS, 2), dtype=torch.float32, device=q.device)
    require_cuda(q, k, v, lengths, out, partial, stats)
    call("b2_attn_decode", ptr(q), ptr(k), ptr(v), ptr(lengths), ptr(out), ptr(partial), ptr(stats), I(B), I(H),
         I(Hkv), I(cap), F(scale), stream())
    return out


DECODE_STEP_FIELDS = ("norm_in", "norm_post", "q_norm", "k_norm", "w_qkv", "s_qkv", "w_o", "s_o", "w_gu", "s_gu",
                      "w_down", "s_down", "k_cache", "v_cache")
DECODE_STEP_SYNC_WORDS = 2048


def decode_step_splits(kv_heads):
    """Position splits per kv head of decode_step on the current device."""
    return int(_lib.load().b2_decode_step_splits(kv_heads))


def decode_step_table(layers, hidden, heads, kv_heads, mlp, capacity):
    """The device table of layer pointers decode_step reads: for each layer the 14 tensors of DECODE_STEP_FIELDS
    (attributes of the layer objects), each checked for shape, dtype, contiguity and 16-byte alignment."""
    d = HEAD_DIM
    shapes = {
        "norm_in": ((hidden,), torch.float32), "norm_post": ((hidden,), torch.float32),
        "q_norm": ((d,), torch.float32), "k_norm": ((d,), torch.float32),
        "w_qkv": (((heads + 2 * kv_heads) * d, hidden), torch.int8), "s_qkv": (((heads + 2 * kv_heads) * d,), torch.float32),
        "w_o": ((hidden, heads * d), torch.int8), "s_o": ((hidden,), torch.float32),
        "w_gu": ((2 * mlp, hidden), torch.int8), "s_gu": ((2 * mlp,), torch.float32),
        "w_down": ((hidden, mlp), torch.int8), "s_down": ((hidden,), torch.float32),
        "k_cache": (None, torch.float32), "v_cache": (None, torch.float32),
    }
    rows = []
    for i, L in enumerate(layers):
        row = []
        for name in DECODE_STEP_FIELDS:
            t = getattr(L, name)
            shape, dtype = shapes[name]
            if name.endswith("cache"):
                if t.dtype != dtype or tuple(t.shape[-3:]) != (capacity, kv_heads, d) or t.numel() != capacity * kv_heads * d:
                    _fail(f"decode_step layer {i} {name} must be fp32 [1, {capacity}, {kv_heads}, {d}]")
            elif t.dtype != dtype or tuple(t.shape) != shape:
                _fail(f"decode_step layer {i} {name} must be {dtype} {shape}, got {t.dtype} {tuple(t.shape)}")
            if not t.is_contiguous() or t.data_ptr() % 16:
                _fail(f"decode_step layer {i} {name} must be contiguous and 16-byte aligned")
            row.append(t.data_ptr())
        rows.append(row)
    require_cuda(*(getattr(L, n) for L in layers for n in DECODE_STEP_FIELDS))
    return torch.tensor(rows, dtype=torch.int64).to(layers[0].w_qkv.device)


def decode_step(table, x, x2, qkv, att, act, partial, stats, inv_freq, pos, lengths, sync, err, hidden, heads, kv_heads,
                mlp, capacity, eps, timeout_ns=2_000_000_000):
    """One token through every layer of the table in one persistent launch (b2_decode_step). x [hidden] fp32 is
    the residual stream in and out; the other buffers are scratch sized as the header states; sync is 2048 int32
    counters (cleared by the call), err an int32 flag the host reads after the step."""
    d = HEAD_DIM
    S = DECODE_SPLITS  # the kernel uses at most this many splits per kv head
    if table.dtype != torch.int64 or table.dim() != 2 or table.shape[1] != len(DECODE_STEP_FIELDS):
        _fail("decode_step table must be int64 [layers, 14]")
    _vec(x, hidden, torch.float32, "decode_step x")
    _vec(x2, hidden, torch.float32, "decode_step x2")
    _vec(qkv, (heads + 2 * kv_heads) * d, torch.float32, "decode_step qkv")
    _vec(att, heads * d, torch.float32, "decode_step att")
    if act is None or act.dtype != torch.float32 or not act.is_contiguous() or act.numel() < mlp:
        _fail("decode_step act must be contiguous fp32 with at least mlp values")
    for t, n, k in ((partial, "partial", heads * S * d), (stats, "stats", heads * S * 2)):
        if t is None or t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < k:
            _fail(f"decode_step {n} must be contiguous fp32 with at least {k} values")
    _vec(inv_freq, d // 2, torch.float32, "inv_freq")
    if pos.dtype != torch.int64 or lengths.dtype != torch.int32:
        _fail("decode_step needs an int64 position and int32 lengths")
    if sync.dtype != torch.int32 or sync.numel() < DECODE_STEP_SYNC_WORDS or err.dtype != torch.int32:
        _fail(f"decode_step needs int32 sync ({DECODE_STEP_SYNC_WORDS} words) and err")
    require_cuda(table, x, x2, qkv, att, act, partial, stats, inv_freq, pos, lengths, sync, err)
    call("b2_decode_step", ptr(table), I(table.shape[0]), ptr(x), ptr(x2), ptr(qkv), ptr(att), ptr(act), ptr(partial),
         ptr(stats), ptr(inv_freq), ptr(pos), ptr(lengths), ptr(sync), ptr(err), I(hidden), I(heads), I(kv_heads),
         I(mlp), I(capacity), F(eps), ctypes.c_longlong(int(timeout_ns)), stream())
    return x


def default_scale():
    return 1.0 / math.sqrt(HEAD_DIM)
