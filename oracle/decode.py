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


def _rms64(x, w, eps):
    x = np.asarray(x, np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * np.asarray(w, np.float64)


def decoder_step(x, layers, pos, length, heads, kv_heads, mlp, eps, inv_freq):
    """One token through an int8 decoder's layers in float64: the route int8_gemv.py's decode takes around its
    kernels, composed as the configuration-5 decoder does. Per layer
        h = RMSNorm(x) * norm_in;  q|k|v = gemv_i8(h)                       (int8_gemv.hip:55-85, int8_gemv.py:62-63)
        q, k = RMSNorm per head (q_norm / k_norm), half-split rotary at `pos` (angle fp32(pos * inv_freq[i]), pairs
               (i, i + 64)); k and v written into row `pos` of the caches
        att = softmax(q k^T / sqrt(128)) v over `length` cache rows, GQA  (int8_gemv.hip:124-195)
        x = x + gemv_i8(att);  h = RMSNorm(x) * norm_post;  g|u = gemv_i8(h)
        x = x + gemv_i8(silu(g) * u)
    layers: one dict per layer holding DECODE_STEP_FIELDS' arrays (int8 weights, fp32 scales / norms, caches
    [1, cap, kv_heads, 128]); the caches are updated in place (as float32). Returns x as float32."""
    d = 128
    x = np.asarray(x, np.float64).reshape(-1)
    ang = (np.float32(pos) * np.asarray(inv_freq, F32)).astype(np.float64)
    cos, sin = np.cos(ang), np.sin(ang)

    def rope(t):
        a, b = t[:, :64], t[:, 64:]
        return np.concatenate((a * cos - b * sin, a * sin + b * cos), axis=1)

    for L in layers:
        h = _rms64(x, L["norm_in"], eps)
        qkv = (np.asarray(L["w_qkv"], np.float64) @ h) * np.asarray(L["s_qkv"], np.float64)
        q = rope(_rms64(qkv[:heads * d].reshape(heads, d), L["q_norm"], eps))
        k = rope(_rms64(qkv[heads * d:(heads + kv_heads) * d].reshape(kv_heads, d), L["k_norm"], eps))
        v = qkv[(heads + kv_heads) * d:].reshape(kv_heads, d)
        kc, vc = L["k_cache"], L["v_cache"]
        kc[0, pos] = k.astype(F32)
        vc[0, pos] = v.astype(F32)
        att = attn_decode(q.reshape(1, 1, heads, d), kc, vc, np.array([length]), d ** -0.5).astype(np.float64)
        x = x + (np.asarray(L["w_o"], np.float64) @ att.reshape(-1)) * np.asarray(L["s_o"], np.float64)
        h = _rms64(x, L["norm_post"], eps)
        gu = (np.asarray(L["w_gu"], np.float64) @ h) * np.asarray(L["s_gu"], np.float64)
        g, u = gu[:mlp], gu[mlp:]
        a = g / (1.0 + np.exp(-g)) * u
        x = x + (np.asarray(L["w_down"], np.float64) @ a) * np.asarray(L["s_down"], np.float64)
    return x.astype(F32)
