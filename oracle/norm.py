"""RMSNorm (+rope) oracle, restating rms_norm.hip norm_row (:9-65)."""
import numpy as np

F32 = np.float32
F16 = np.float16


def rms_norm(x, w, eps):
    """y = fp16(x * rstd * (w + 1)), rstd = rsqrt(sum(x^2) / D + eps) in fp32 (rms_norm.hip:38,47).
    x fp16 [..., D], w fp32 [D] zero-centred. The fp32 sum order of the kernel is not reproduced."""
    f = np.asarray(x).astype(F32)
    D = f.shape[-1]
    ss = (f * f).sum(axis=-1, dtype=F32)
    rstd = (F32(1) / np.sqrt(ss / F32(D) + F32(eps))).astype(F32)
    return ((f * rstd[..., None]) * (np.asarray(w, F32) + F32(1))).astype(F16)


def _fma32(a, b, c):
    """fp32 fma(a, b, c) with a single rounding (float64 holds a*b exactly; the add is then rounded once more,
    which can differ from a true fma only in rare double-rounding cases)."""
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(F32)


def rope(y16, freqs):
    """Per pair (x0, x1) of the normalised fp16 head and its 2x2 fp32 matrix m (rms_norm.hip:48-61):
    a = fma(m1, x1, m0 * x0), c = fma(m3, x1, m2 * x0), each rounded to fp32 then to fp16.
    y16 [..., L, 128]; freqs [..., L, 64, 2, 2] broadcastable."""
    x = np.asarray(y16).astype(F32)
    x0 = x[..., 0::2]
    x1 = x[..., 1::2]
    m = np.asarray(freqs, F32)
    m0, m1, m2, m3 = m[..., 0, 0], m[..., 0, 1], m[..., 1, 0], m[..., 1, 1]
    a = _fma32(m1, x1, (m0 * x0).astype(F32))
    c = _fma32(m3, x1, (m2 * x0).astype(F32))
    out = np.empty(x.shape, F16)
    out[..., 0::2] = a.astype(F16)
    out[..., 1::2] = c.astype(F16)
    return out


def rms_norm_rope(x, heads, w, eps, freqs):
    """rms_norm.py:42-52: x (B, L, heads*128) -> (B, heads, L, 128) with QK-norm then rope; freqs (B or 1, 1, L,
    64, 2, 2)."""
    x = np.asarray(x)
    B, L, _ = x.shape
    v = x.reshape(B, L, heads, 128).transpose(0, 2, 1, 3)
    y = rms_norm(v, w, eps)
    f = np.asarray(freqs, F32).reshape(freqs.shape[0], 1, L, 64, 2, 2)
    return rope(y, f)
