"""Single-token decode, the drop-in for the reference's int8_gemv.py.

Same entry points: ``rotate(x, group)`` (:42-45), ``linear_forward(module, N, K, weight_dtype, group, x, ...)``
(:48-64), ``attention_decode(q, k, v, lengths)`` (:101-114, installed as ``comfy_kitchen.flash_attention_decode``),
``init_kv_cache`` (:117-126), ``generate`` (:78-84) and ``patch`` (:129-148). Modules are duck-typed: an int8 linear
is anything whose ``weight`` carries ``_qdata`` (int8 [N, K]) and ``_params.scale`` (fp32 [N]), as ComfyUI's
``int8_tensorwise`` MixedPrecisionOp does. Single-row fp32 steps run the HBM-streaming GEMV; other inputs raise
instead of falling back (:49-50).
"""
import collections
import functools

import torch

from . import ops

BLOCK_ROWS = 16
STEP = 16  # K granularity of the B200 GEMV (16-byte loads)
SPLITS = ops.DECODE_SPLITS
HEAD = 128

generating = False

FixedKVCache = collections.namedtuple("FixedKVCache", "key value index position length")


def patched(module):
    return bool(getattr(module, "weight_function", None) or getattr(module, "bias_function", None)
                or getattr(module, "weight_lowvram_function", None) is not None)


def rotate(x, group):
    """fp32 regular-Hadamard rotation of each ``group`` values (int8_gemv.py:42-45)."""
    return ops.rotate(x.contiguous(), group)


def linear_forward(module, N, K, weight_dtype, group, x, *args, **kwargs):
    """One decode step of an int8 linear: optional ConvRot of x, then out = scale * (W x) + bias in fp32."""
    if x.dtype != torch.float32 or patched(module) or x.numel() != K:
        raise NotImplementedError("linear_forward handles one unpatched fp32 row per call")
    weight = module.weight
    qdata = weight._qdata
    scale = weight._params.scale.to(device=x.device, dtype=torch.float32).reshape(N).contiguous()
    bias = getattr(module, "bias", None)
    if bias is not None:
        bias = bias.to(device=x.device, dtype=torch.float32).contiguous()
    x = x.contiguous()
    if group:
        x = rotate(x, group)
    out = ops.gemv_i8(x.reshape(K), qdata, scale, bias)
    return out.reshape(*x.shape[:-1], N)


def attention_decode(q, k, v, lengths):
    """q is (batch, 1, heads, 128), k and v are (batch, capacity, kv heads, 128) and lengths (batch,) int32, all but
    lengths fp32 (int8_gemv.py:101-114)."""
    return ops.attn_decode(q, k.contiguous(), v.contiguous(), lengths.to(torch.int32), HEAD ** -0.5)


def init_kv_cache(model, batch, capacity, device, dtype):
    """fp32 fixed-capacity KV cache per layer, so each layer can be replayed from a CUDA graph (int8_gemv.py:117-126).
    Uses ComfyUI's FixedKV when available."""
    try:
        from comfy.text_encoders.llama import FixedKV
    except ImportError:
        FixedKV = FixedKVCache
    config = model.config
    position = torch.empty((batch,), device=device, dtype=torch.int64)
    length = torch.zeros((batch,), device=device, dtype=torch.int32)
    caches = []
    for _ in range(config.num_hidden_layers):
        key = torch.empty((batch, capacity, config.num_key_value_heads, HEAD), device=device, dtype=dtype)
        caches.append(FixedKV(key, torch.empty_like(key), 0, position, length))
    return caches


def generate(transformer, *args, **kwargs):
    global generating
    generating = True
    try:
        return type(transformer).generate(transformer, *args, **kwargs)
    finally:
        generating = False


def patch(clip):
    """Single-token steps read the int8 weights directly (int8_gemv.py:129-148)."""
    for name, module in clip.patcher.model.named_modules():
        w = getattr(module, "weight", None)
        if type(module).__name__ == "Linear" and getattr(module, "quant_format", None) == "int8_tensorwise" and w is not None:
            N, K = w.shape
            params = w._params
            if K % STEP == 0 and params.scale.numel() == N and params.scale.dtype == torch.float32 and not params.transposed:
                group = params.convrot_groupsize if params.convrot else 0
                clip.patcher.add_object_patch(f"{name}.forward", functools.partial(linear_forward, module, N, K, w.dtype, group))
