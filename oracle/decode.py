"""Single-token decode oracle, restating int8_gemv.hip and the reference's non-GEMV fallback."""
import numpy as np

F32 = np.float32


def rotate(x, group):
    """int8_gemv.hip:32-52: radix-4 regular-Hadamard stages with stride 1, 4, 16, ... (the lowest base-4 digit
    first), y[i] = s - 2 x[3 - i] with s = ((a+b)+c)+d in fp32, then times rsqrt(group) (a power of two)."""
    x = np.asarray(x, F32)
    n = x.size
    v = x.reshape(n // group, group).copy()
    stride = 1
    two = F32(2)
    while stride < group:
        w = v.reshape(n // group, group // (4 * stride), 4, stride)
        a, b, c, d = (w[:, :, i, :] for i in range(4))
        s = ((a + b) + c) + d
        w = np.stack((s - two * d, s - two * c, s - two * b, s - two * a), axis=2)
        v = w.reshape(n // group, group)
        stride *= 4
    return (v * F32(1.0 / np.sqrt(group))).reshape(x.shape)


def gemv_i8(x, w, scale, bias=None):
    """out[n] = scale[n] * sum_k w[n, k] x[k] (+ bias[n]) (int8_gemv.hip:55-85), accumulated in float64 here;
    the reference's own fallback is F.linear(x, w.to(fp32) * scale, bias) (int8_gemv.py:58-59)."""
    acc = np.asarray(w, np.float64) @ np.asarray(x, np.float64).reshape(-1)
    y = acc * np.asarray(scale, np.float64)
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return y.astype(F32)


def bf16_to_f32(bits):
    """bf16 bit patterns (uint16) -> float32, exactly: the pattern is the high half of the float32."""
    return (np.asarray(bits, np.uint16).astype(np.uint32) << np.uint32(16)).view(F32)


def gemv_bf16(x, w_bits):
    """out[n] = sum_k w[n, k] x[k] for a bf16 table (int8_gemv.hip:88-119 gemv_bf16, the logits of
    int8_gemv.py:87-98), the table given as uint16 bit patterns, accumulated in float64 here."""
    w = bf16_to_f32(w_bits).astype(np.float64)
    return (w @ np.asarray(x, np.float64).reshape(-1)).astype(F32)


def linear_fallback(x, w, scale, bias=None):
    """The reference's non-GEMV path in fp32 torch semantics: F.linear(x, w.to(fp32) * scale, bias)
    (int8_gemv.py:58-59), used as the CPU baseline."""
    import torch
    import torch.nn.functional as F
    wt = torch.as_tensor(np.asarray(w)).to(torch.float32) * torch.as_tensor(np.asarray(scale, F32))[:, None]
    xt = torch.as_tensor(np.asarray(x, F32))
    bt = None if bias is None else torch.as_tensor(np.asarray(bias, F32))
    return F.linear(xt, wt, bt).numpy()


def attn_decode(q, k, v, lengths, scale):
    """float64 softmax decode attention, the value int8_gemv.hip:124-195 (split-32 online softmax + merge)
    approximates in fp32. q [B,1,H,128], k/v [B,cap,Hkv,128], lengths [B]."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    B, _, H, D = q.shape
    Hkv = k.shape[2]
    rep = H // Hkv
    out = np.zeros(q.shape, F32)
    for b in range(B):
        n = int(lengths[b])
        for h in range(H):
            s = (k[b, :n, h // rep] @ q[b, 0, h]) * scale
            s -= s.max()
            p = np.exp(s)
            out[b, 0, h] = (p @ v[b, :n, h // rep]) / p.sum()
    return out
