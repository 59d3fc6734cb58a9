"""W8A8 / W4A8 GEMM oracle: exact int32 accumulation and the dequant/bias/residual epilogue.

Restates int8_gemm.hip gemm_body (:315-406). The int32 product uses torch._int_mm on CPU (exact) for speed,
falling back to int64 numpy for shapes it does not take.
"""
import numpy as np
import torch

F32 = np.float32
F16 = np.float16


def int_mm(a, b):
    """acc[m, n] = sum_k a[m, k] * b[n, k] exactly (int8 x int8 -> int32), the MAC loop of int8_gemm.hip:338-368."""
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    M, K = a.shape
    N = b.shape[0]
    if M >= 17 and K % 8 == 0 and N % 8 == 0:
        return torch._int_mm(torch.from_numpy(a), torch.from_numpy(b).t().contiguous()).numpy()
    return (a.astype(np.int64) @ b.astype(np.int64).T).astype(np.int32)


def epilogue(acc, sa, sw, bias=None, R=None, G=None, L=1):
    """y = (float)acc * sa[m] * sw[n] (+ (float)bias[n]) -> fp16 (int8_gemm.hip:382-383);
    residual out = fp16(R + fp16(G[m // L] * y)) (:394-400)."""
    y = (np.asarray(acc).astype(F32) * np.asarray(sa, F32)[:, None]) * np.asarray(sw, F32)[None, :]
    if bias is not None:
        y = y + np.asarray(bias).astype(F32)[None, :]
    y16 = y.astype(F16)
    if R is None:
        return y16
    rows = np.arange(y16.shape[0]) // L
    g = np.asarray(G).astype(F32)[rows]
    return (np.asarray(R).astype(F32) + (g * y16.astype(F32)).astype(F16).astype(F32)).astype(F16)


def w4a8_grouped(a_q, a_scale, w_packed, w_scales, group=128, bias=None):
    """W4A8 with per-group int32 accumulation: out = fp16(sum_g (acc_g * sw[n, g]) * sa[m] (+ bias)).

    The configuration's grouped form has no reference kernel (the reference's gemm_i4 is per-channel W4A4,
    int8_gemm.hip:412, int8_gemm.py:90-103), so this is the specification: acc_g = int32 dot over the g-th 128 k
    (exact), converted to fp32 (exact, |acc_g| < 2^22), and combined in group order with one fused multiply-add per
    group, F = fma(acc_g, s[n, g], F) in fp32, then y = F * sa[m] (+ bias) with separate roundings, -> fp16.
    The fma is evaluated in extended precision (the product is exact there) and rounded once to fp32.
    """
    w = unpack_int4(w_packed)
    K = w.shape[1]
    sw = np.asarray(w_scales).astype(F32)
    out = np.zeros((a_q.shape[0], w.shape[0]), F32)
    for g in range(K // group):
        acc = int_mm(a_q[:, g * group:(g + 1) * group], w[:, g * group:(g + 1) * group])
        prod = acc.astype(np.longdouble) * sw[None, :, g].astype(np.longdouble)
        out = (prod + out.astype(np.longdouble)).astype(F32)
    y = out * np.asarray(a_scale, F32)[:, None]
    if bias is not None:
        y = y + np.asarray(bias).astype(F32)[None, :]
    return y.astype(F16)


def unpack_int4(packed):
    """uint8 [N, K/2] -> int8 [N, K], low nibble = even k, two's-complement nibbles in [-8, 7]."""
    p = np.asarray(packed, dtype=np.uint8)
    lo = (p & 0x0F).astype(np.int16)
    hi = (p >> 4).astype(np.int16)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    out = np.empty((p.shape[0], p.shape[1] * 2), np.int8)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    return out
