"""ComfyUI ``optimized_attention`` override, the drop-in for the reference's attention.py:46-65.

``attention_hip`` keeps the reference's signature and reshaping. The reference falls back to its rocBLAS bmm path
for masks, an ``enable_gqa`` kwarg, head dims other than 128, differing v width or non-fp16 inputs
(attention.py:48-49); this build has no bmm path and no CPU fallback, so those inputs raise ``NotImplementedError``
naming the condition.
"""
import torch

from . import hip_attention

HEAD_DIM = 128


def to_heads(t, b, heads, dim_head):
    """(B, L, H*D) -> (B, H, L, D) view (attention.py:11-12)."""
    return t.reshape(b, -1, heads, dim_head).transpose(1, 2)


def eligible(q, k, v, heads, mask=None, skip_reshape=False, **kwargs):
    dim_head = q.shape[-1] if skip_reshape else q.shape[-1] // heads
    if mask is not None:
        return "attention masks are not supported"
    if kwargs.get("enable_gqa", False):
        return "the enable_gqa kwarg is not supported (pass (B, Hkv, L, D) k/v with skip_reshape instead)"
    if dim_head != HEAD_DIM:
        return f"head dim {dim_head} is not 128"
    if v.shape[-1] != q.shape[-1]:
        return "v and q widths differ"
    if q.dtype != torch.float16:
        return f"dtype {q.dtype} is not fp16"
    return None


def attention_hip(q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False, skip_output_reshape=False,
                  int8_qk=False, **kwargs):
    reason = eligible(q, k, v, heads, mask=mask, skip_reshape=skip_reshape, **kwargs)
    if reason:
        raise NotImplementedError(f"attention_hip: {reason}")
    dim_head = q.shape[-1] if skip_reshape else q.shape[-1] // heads
    b = q.shape[0]
    if not skip_reshape:
        q, k, v = (to_heads(t, b, heads, dim_head) for t in (q, k, v))
    q_len = q.shape[2]
    q, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (q, k, v))
    out = torch.empty((b, q_len, heads, dim_head), dtype=q.dtype, device=q.device).transpose(1, 2)
    hip_attention.attention(q, k, v, out, kwargs.get("scale", dim_head ** -0.5), int8_qk)
    if skip_output_reshape:
        return out
    return out.transpose(1, 2).reshape(b, q_len, heads * dim_head)


def attention_hip_int8(*args, **kwargs):
    return attention_hip(*args, int8_qk=True, **kwargs)
