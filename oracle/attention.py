"""Attention oracles.

* ``attention_bmm``: the reference's own pure-PyTorch path (attention.py:15-43: baddbmm(alpha=scale) -> softmax
  -> bmm, in the input dtype), restated for CPU. Golden outputs of the reference function itself pin it
  (tests/golden). It is also the timed CPU baseline for attention.
* ``attention_exact``: float64 softmax attention, the accuracy yardstick for the fp16 and int8-QK kernels.
* ``attention_semantics``: the fused kernel's arithmetic (hip_attention.hip attn :280-373 and attn_i8 :160-278):
  log2-domain online softmax over key tiles, warp-uniform lazy rescale at m + 8, fp16 P, fp32 l.
* ``quant_rows_rint``: the int8-QK operand quantization (hip_attention.hip:67-93, :172-194), bit-exact target.
"""
import math

import numpy as np
import torch

F32 = np.float32
F16 = np.float16
LOG2E = 1.4426950408889634


def attention_bmm(q, k, v, scale=None, chunk_bytes=128 * 1024 * 1024):
    """attention.py:15-43 for inputs (B, H, L, D) (skip_reshape=True, skip_output_reshape=True): chunks of
    the batch*heads dimension through baddbmm -> softmax -> bmm in q's dtype."""
    b, heads, q_len, dim_head = q.shape
    k_len = k.shape[2]
    batch = b * heads
    if scale is None:
        scale = dim_head ** -0.5
    qq = q.reshape(batch, q_len, dim_head).contiguous()
    kk = k.reshape(batch, k_len, dim_head).contiguous().transpose(1, 2).contiguous()
    vv = v.reshape(batch, k_len, -1)
    out = torch.empty((batch, q_len, vv.shape[-1]), dtype=q.dtype, device=q.device)
    step = min(batch, max(1, chunk_bytes // (q_len * k_len * q.element_size())))
    scores = torch.empty((step, q_len, k_len), dtype=q.dtype, device=q.device)
    for i in range(0, batch, step):
        s = scores[:min(step, batch - i)]
        torch.baddbmm(s, qq[i:i + step], kk[i:i + step], beta=0, alpha=scale, out=s)
        torch.softmax(s, -1, out=s)
        torch.bmm(s, vv[i:i + step], out=out[i:i + step])
    return out.view(b, heads, q_len, -1)


def expand_kv(k, heads):
    """Grouped-query heads: query head h reads KV head h // (H / Hkv) (hip_attention.py:59, rep = H / Hkv)."""
    rep = heads // k.shape[1]
    return np.repeat(k, rep, axis=1) if rep > 1 else k


def attention_exact(q, k, v, scale):
    """float64 softmax(q k^T * scale) v for numpy (B, H, L, 128) arrays (k/v may have fewer heads)."""
    q = np.asarray(q, np.float64)
    k = expand_kv(np.asarray(k, np.float64), q.shape[1])
    v = expand_kv(np.asarray(v, np.float64), q.shape[1])
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v)


def quant_rows_rint(x):
    """Per-row int8 with rint (half-even) and no +0.5: scale = fmaxf(max|x| / 127, 1e-30), q = rint(x / scale)
    (hip_attention.hip:85,91 for keys; :183,192-193 for queries). x fp16 [..., 128] -> (int8, float32 [...])."""
    f = np.asarray(x).astype(F32)
    mx = np.abs(f).max(axis=-1)
    scale = np.maximum(mx / F32(127), F32(1e-30)).astype(F32)
    q = np.fmin(np.fmax(np.rint(f / scale[..., None]), F32(-128)), F32(127)).astype(np.int8)
    return q, scale


def attention_semantics(q, k, v, scale, int8_qk=False, tile=128, warp_rows=32):
    """The fused kernel's arithmetic for one call on numpy fp16 (B, H, Lq, 128) inputs.

    For each key tile: scores s (fp32 dot products, or int8 dots scaled ((float)si * (qs*c)) * ks), block max
    (fp16 path: max(s) * c), warp-uniform rescale when any of the warp's rows exceeds m + 8, p = exp2(s*c - m)
    (fp16 path) or exp2(s - m) (int8), P rounded to fp16, o += P V (fp32), l += p (fp32); out = fp16(o * (1/l)).
    The reference steps keys by 16 (tile=16); the B200 kernel by 128.
    """
    q = np.asarray(q, F16)
    B, H, Lq, D = q.shape
    k = expand_kv(np.asarray(k, F16), H)
    v = expand_kv(np.asarray(v, F16), H)
    Lk = k.shape[2]
    c = F32(scale * LOG2E)
    out = np.zeros((B, H, Lq, D), F16)
    for b in range(B):
        for h in range(H):
            if int8_qk:
                qq, qs = quant_rows_rint(q[b, h])
                kq, ks = quant_rows_rint(k[b, h])
                si = (qq.astype(np.int64) @ kq.astype(np.int64).T).astype(np.int32)
                s_all = (si.astype(F32) * (qs * c)[:, None]) * ks[None, :]
            else:
                s_all = (q[b, h].astype(np.float64) @ k[b, h].astype(np.float64).T).astype(F32)
            m = np.full(Lq, F32(-1e30), F32)
            l = np.zeros(Lq, F32)
            o = np.zeros((Lq, D), F32)
            for j0 in range(0, Lk, tile):
                s = s_all[:, j0:j0 + tile]
                mx = s.max(axis=1)
                if not int8_qk:
                    mx = (mx * c).astype(F32)
                for w0 in range(0, Lq, warp_rows):
                    rows = slice(w0, w0 + warp_rows)
                    if np.any(mx[rows] > m[rows] + F32(8)):
                        mn = np.maximum(m[rows], mx[rows])
                        alpha = np.exp2((m[rows] - mn).astype(np.float64)).astype(F32)
                        m[rows] = mn
                        l[rows] *= alpha
                        o[rows] *= alpha[:, None]
                if int8_qk:
                    p = np.exp2((s - m[:, None]).astype(np.float64)).astype(F32)
                else:
                    p = np.exp2((s.astype(np.float64) * np.float64(c) - m[:, None])).astype(F32)
                l += p.sum(axis=1, dtype=F32)
                o += (p.astype(F16).astype(np.float64) @ v[b, h, j0:j0 + tile].astype(np.float64)).astype(F32)
            out[b, h] = (o * (F32(1) / l)[:, None]).astype(F16)
    return out


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def default_scale(dim_head=128):
    return dim_head ** -0.5 if dim_head else 1.0 / math.sqrt(128)
