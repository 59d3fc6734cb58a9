"""Weight preparation used by tests and benchmarks: rotation and quantization of fp weights.

In the reference this happens in the third-party int8/int4 loader (ComfyUI-INT8-Fast-ROCM, un-vendored and
unpinned; int8_gemm.py:247-271 only patches it), so nothing here is pinned by the reference. The formats follow
the benchmark configurations: per-output-channel symmetric int8 with scale = absmax / 127 and round-half-even,
and int4 in [-8, 7] with fp16 scales per 128 values along K, packed low nibble first.
"""
import numpy as np

F32 = np.float32


def sylvester_rotate(w, block=128):
    """Rotate rows along K with the block-diagonal normalised Sylvester Hadamard (float64, exact enough for a
    weight that is quantized afterwards). The same transform applied to activations cancels in X W^T."""
    w = np.asarray(w, dtype=np.float64)
    N, K = w.shape
    v = w.reshape(N, K // block, *([2] * int(np.log2(block))))
    nb = int(np.log2(block))
    for axis in range(1 + nb, 1, -1):
        a = np.take(v, 0, axis=axis)
        b = np.take(v, 1, axis=axis)
        v = np.stack((a + b, a - b), axis=axis)
    return (v.reshape(N, K) / np.sqrt(block)).astype(F32)


def convrot_rotate(w):
    """Rotate rows along K with H4^(x)4 / 16 per 256 values (the reference ConvRot matrix, int8_gemm.hip:105-108)."""
    w = np.asarray(w, dtype=np.float64)
    N, K = w.shape
    h4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)
    h = h4
    for _ in range(3):
        h = np.kron(h, h4)
    return ((w.reshape(N, K // 256, 256) @ h.T) / 16.0).reshape(N, K).astype(F32)


def quantize_per_channel(w):
    """int8 per output channel: scale = absmax / 127, q = round_half_even(w / scale). Returns (int8, float32)."""
    w = np.asarray(w, dtype=F32)
    scale = (np.abs(w).max(axis=1) / F32(127)).astype(F32)
    scale = np.where(scale == 0, F32(1), scale).astype(F32)
    q = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale


def quantize_int4_groups(w, group=128):
    """int4 in [-8, 7] per 128 values along K with fp16 scales (absmax / 7, rounded to fp16 first), half-even.
    Returns (packed uint8 [N, K/2] low nibble = even k, fp16 scales [N, K/group])."""
    w = np.asarray(w, dtype=F32)
    N, K = w.shape
    g = w.reshape(N, K // group, group)
    s16 = (np.abs(g).max(axis=2) / F32(7)).astype(np.float16)
    s16 = np.where(s16 == 0, np.float16(1), s16)
    q = np.clip(np.rint(g / s16.astype(F32)[:, :, None]), -8, 7).astype(np.int8).reshape(N, K)
    packed = ((q[:, 0::2].astype(np.uint8) & 0x0F) | ((q[:, 1::2].astype(np.uint8) & 0x0F) << 4)).astype(np.uint8)
    return packed, s16
