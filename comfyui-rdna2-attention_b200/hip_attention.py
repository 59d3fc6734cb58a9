"""Low-level fused attention call, the drop-in for the reference's ``hip_attention.attention``
(hip_attention.py:45-66). The name is kept so that callers written against the reference import it unchanged;
the kernel behind it is the sm_100a tcgen05 attention of librdna2_b200.so (no HIP, no packing pass: TMA reads
K and V in place, so the reference's packed KV buffer, hip_attention.py:56-63, does not exist here)."""
import torch

from . import ops


def _tma_ready(t):
    return t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and all(s % 8 == 0 for s in t.stride()[:3])


def attention(q, k, v, out, scale, int8_qk=False):
    """q, k, v, out are (batch, heads, length, 128) fp16 tensors with a contiguous last dimension. k and v may
    have fewer heads than q, which then share them. ``out`` may be a strided view; it is written in place."""
    q, k, v = (t if _tma_ready(t) else t.contiguous() for t in (q, k, v))
    if _tma_ready(out):
        ops.attention(q, k, v, out, scale, int8_qk)
    else:
        tmp = torch.empty(out.shape, dtype=out.dtype, device=out.device)
        ops.attention(q, k, v, tmp, scale, int8_qk)
        out.copy_(tmp)
    return out
