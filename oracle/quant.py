"""Activation pre-pass oracle: activations, block Hadamard rotations and per-row int8 quantization.

Restates int8_gemm.hip (reference file). All arithmetic is float32 numpy with one IEEE rounding per operation,
which is what the kernels do once contraction is ruled out (the reference disables it where it matters,
int8_gemm.hip:141,395).
"""
import numpy as np

F32 = np.float32
F16 = np.float16
INV_SQRT128 = F32(0.08838834764831845)


def quant_rows(y):
    """Per-row absmax int8 (int8_gemm.hip:29-60, quant_row).

    scale = fmaxf(mx / 127.f, 1e-30f) (:38); q = clamp(floorf(f / scale + 0.5f), -128, 127) (:53), i.e. round
    half up after an IEEE divide. ``y`` is the fp16 (or fp16-valued) activation [M, K]; returns (int8 [M, K],
    float32 [M]).
    """
    f = np.asarray(y).astype(F32)
    # The absmax is a chain of fmaxf starting at 0 (:96-100, :32-37): a NaN value never wins it.
    mx = np.fmax.reduce(np.abs(f), axis=1, initial=F32(0)) if f.shape[1] else np.zeros(f.shape[0], F32)
    scale = np.maximum(mx / F32(127), F32(1e-30)).astype(F32)
    with np.errstate(invalid="ignore", divide="ignore"):
        q = np.floor(f / scale[:, None] + F32(0.5))
    # fminf(fmaxf(q, -128), 127): IEEE maxNum/minNum drop a NaN operand (inf / inf after an fp16 overflow).
    return np.fmin(np.fmax(q, F32(-128)), F32(127)).astype(np.int8), scale


def quant_rows_i4(y):
    """Per-row int4-valued activations (int8_gemm.hip:62-91, quant_row_i4): scale = fmaxf(mx, 1e-10f) / 7.f (:71),
    q = clamp(rintf(f / scale), -7, 7) (:85), i.e. round half to even after an IEEE divide; one int8 per value here
    (the reference packs eight per dword, low nibble first, which only its dot8 instruction needs)."""
    f = np.asarray(y).astype(F32)
    mx = np.fmax.reduce(np.abs(f), axis=1, initial=F32(0)) if f.shape[1] else np.zeros(f.shape[0], F32)
    scale = (np.maximum(mx, F32(1e-10)) / F32(7)).astype(F32)
    with np.errstate(invalid="ignore", divide="ignore"):
        q = np.rint(f / scale[:, None])
    return np.fmin(np.fmax(q, F32(-7)), F32(7)).astype(np.int8), scale


def _h4(a, b, c, d):
    """One regular 4-point Hadamard step (int8_gemm.hip:106-109): s = ((a+b)+c)+d; (s-2d, s-2c, s-2b, s-2a)."""
    s = ((a + b) + c) + d
    two = F32(2)
    return s - two * d, s - two * c, s - two * b, s - two * a


def _apply_h4(v, axis):
    parts = [np.take(v, i, axis=axis) for i in range(4)]
    return np.stack(_h4(*parts), axis=axis)


def hadamard256(x):
    """ConvRot of each 256 values: H4^(x)4 one base-4 digit at a time, lowest first, then fp16(v * 0.0625).

    Digits 0 and 1 are the lane-local h16 (int8_gemm.hip:111-116, :222), digits 2 and 3 the h16 after the LDS
    transpose (:229-230); the result lands at the input's position (:233-234). ``x``: float32 [M, K], K % 256 == 0.
    Returns float16 [M, K].
    """
    x = np.asarray(x, dtype=F32)
    M, K = x.shape
    v = x.reshape(M, K // 256, 4, 4, 4, 4)  # axes: digit3, digit2, digit1, digit0
    for axis in (5, 4, 3, 2):
        v = _apply_h4(v, axis)
    return (v.reshape(M, K) * F32(0.0625)).astype(F16)


def hadamard128(x):
    """Block-128 normalised Hadamard (the configuration's rotation): Sylvester H2^(x)7 applied one index bit at a
    time from bit 0, butterflies (a+b, a-b), then fp16(v * fp32(1/sqrt(128))). float32 [M, K] -> float16."""
    x = np.asarray(x, dtype=F32)
    M, K = x.shape
    v = x.reshape(M, K // 128, 2, 2, 2, 2, 2, 2, 2)  # axes 2..8 = bits 6..0
    for axis in range(8, 1, -1):
        a = np.take(v, 0, axis=axis)
        b = np.take(v, 1, axis=axis)
        v = np.stack((a + b, a - b), axis=axis)
    with np.errstate(over="ignore"):
        return (v.reshape(M, K) * INV_SQRT128).astype(F16)


def rotate_rows(y16, rot_group):
    """fp16 rows -> fp16 rows after the pre-pass rotation (0: none, 256: ConvRot, 128: block-128)."""
    f = np.asarray(y16).astype(F32)
    if rot_group == 0:
        return np.asarray(y16).astype(F16)
    if rot_group == 256:
        return hadamard256(f)
    if rot_group == 128:
        return hadamard128(f)
    raise ValueError(rot_group)


def swiglu(gate, up):
    """fp16(fp16(g / (1 + exp(-g))) * u), the rounding of F.silu(gate).mul_(up) (int8_gemm.hip:129-132)."""
    g = np.asarray(gate).astype(F32)
    u = np.asarray(up).astype(F32)
    with np.errstate(over="ignore"):
        silu = (g / (F32(1) + np.exp(-g))).astype(F16).astype(F32)
    return (silu * u).astype(F16)


def sigmoid_gate(x, gate):
    """fp16(x * fp16(1 / (1 + exp(-g)))), the rounding of x * F.sigmoid(gate) (int8_gemm.hip:134-137)."""
    xf = np.asarray(x).astype(F32)
    g = np.asarray(gate).astype(F32)
    with np.errstate(over="ignore"):
        sig = (F32(1) / (F32(1) + np.exp(-g))).astype(F16).astype(F32)
    return (xf * sig).astype(F16)


def soft_tanh(x):
    """tanh through base-2 exponentials as int8_gemm.hip:118-122: ax = |x|, t = 2^(-2.885390082 ax),
    y = (1 - t) / (1 + t), or ax (1 - ax^2 (1/3 - ax^2 2/15)) below ax = 0.02; the sign of x restored."""
    x = np.asarray(x, F32)
    ax = np.abs(x)
    with np.errstate(over="ignore", invalid="ignore"):
        t = np.exp2(F32(-2.885390082) * ax).astype(F32)
        y = ((F32(1) - t) / (F32(1) + t)).astype(F32)
    a2 = ax * ax
    series = ax * (F32(1) - a2 * (F32(1) / F32(3) - a2 * (F32(2) / F32(15))))
    y = np.where(ax < F32(0.02), series, y).astype(F32)
    return np.where(x < 0, -y, y).astype(F32)


def situ(hidden, gate):
    """fp16(4 tanh(g / 4) sigmoid(g) 25 tanh(h / 25)), the products left to right and sigmoid through 2^x
    (int8_gemm.hip:124-127)."""
    h = np.asarray(hidden).astype(F32)
    g = np.asarray(gate).astype(F32)
    with np.errstate(over="ignore"):
        sig = (F32(1) / (F32(1) + np.exp2(F32(-1.442695041) * g))).astype(F32)
    a = (F32(4) * soft_tanh(g * F32(0.25))) * sig
    return ((a * F32(25)) * soft_tanh(h * F32(0.04))).astype(F16)


def rms_rstd(x):
    """rsqrt(sum(x^2) / K + eps) per row in fp32 (int8_gemm.hip:167-189; the sum order is not reproduced)."""
    f = np.asarray(x).astype(F32)
    return f, (f * f).sum(axis=1, dtype=F32)


def modulate(x, w, s, t, L, eps):
    """fp16(fp16(fp16(x * rstd * (w + 1)) * s) + t) per row, no contraction (int8_gemm.hip:139-143,167-191).

    x fp16 [M, K]; w fp32 [K] (zero-centred); s (= 1 + scale) and t fp16 [M / L, K]; row m uses s[m // L].
    """
    f, ss = rms_rstd(x)
    K = f.shape[1]
    rstd = (F32(1) / np.sqrt(ss / F32(K) + F32(eps))).astype(F32)
    rows = np.arange(f.shape[0]) // L
    sf = np.asarray(s).astype(F32)[rows]
    tf = np.asarray(t).astype(F32)[rows]
    n = ((f * rstd[:, None]) * (np.asarray(w, F32)[None, :] + F32(1))).astype(F16).astype(F32)
    return ((n * sf).astype(F16).astype(F32) + tf).astype(F16)


def prepass(x, rot_group, act="none", u=None, w=None, s=None, t=None, L=1, eps=1e-6):
    """The whole pre-pass of one row block: activation -> rotation -> quant. Returns (q, scale, act16)."""
    if act == "none":
        a16 = np.asarray(x).astype(F16)
    elif act == "swiglu":
        a16 = swiglu(x, u)
    elif act == "gate":
        a16 = sigmoid_gate(x, u)
    elif act == "mod":
        a16 = modulate(x, w, s, t, L, eps)
    elif act == "situ":
        xs = np.asarray(x)
        k = xs.shape[1] // 2
        a16 = situ(xs[:, :k], xs[:, k:])
    else:
        raise ValueError(act)
    y16 = rotate_rows(a16, rot_group)
    q, scale = quant_rows(y16)
    return q, scale, a16
