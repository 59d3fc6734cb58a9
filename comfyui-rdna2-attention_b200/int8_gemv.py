"""Single-token decode, the drop-in for the reference's int8_gemv.py.

Same entry points: ``rotate(x, group)`` (:42-45), ``linear_forward(module, N, K, weight_dtype, group, x, ...)``
(:48-64), ``mlp_forward(module, weight_dtype, x, norm)`` (:67-75), ``logits(transformer, x)`` (:87-98),
``attention_decode(q, k, v, lengths)`` (:101-114, installed as ``comfy_kitchen.flash_attention_decode``),
``init_kv_cache`` (:117-126), ``generate`` (:78-84) and ``patch`` (:129-148). Modules are duck-typed: an int8 linear
is anything whose ``weight`` carries ``_qdata`` (int8 [N, K]) and ``_params.scale`` (fp32 [N]), as ComfyUI's
``int8_tensorwise`` MixedPrecisionOp does.

Which calls these kernels take follows the reference: one fp32 token of an unpatched layer runs the HBM-streaming
GEMV (``linear_forward``) or the bf16 logits GEMV (``logits``); a prefill while generating runs the ConvRot kernel
and a dequantized fp32 linear for ConvRot groups above 256 (:49-57) and the merged gate|up linear (``mlp_forward``).
Prompt encoding (multi-token, not generating) keeps the text encoder's own forward, because its rounding decides the
image (:23-24, :49-50); that path never reaches this library.
"""
import collections
import functools

import torch
import torch.nn.functional as F

from . import ops

BLOCK_ROWS = 16
STEP = 16  # K granularity of the B200 int8 GEMV (16-byte loads)
BF16_STEP = 8  # K granularity of the B200 bf16 GEMV
FAST_DEQUANT_GROUP = 256  # int8_gemv.py:20: prefills with larger ConvRot groups rotate here and run a dense fp32 linear
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


def _scale(module, N, device):
    return module.weight._params.scale.to(device=device, dtype=torch.float32).reshape(N).contiguous()


def _bias(module, device):
    bias = getattr(module, "bias", None)
    return None if bias is None else bias.to(device=device, dtype=torch.float32).contiguous()


def linear_forward(module, N, K, weight_dtype, group, x, *args, **kwargs):
    """An int8 linear of the decoder (int8_gemv.py:48-64). One fp32 token: optional ConvRot of x (fp32 kernel), then
    out = scale * (W x) + bias by the int8 GEMV. A prefill while generating with a ConvRot group above 256: the same
    rotation, then F.linear with the dequantized weight. Anything else is the module's own forward."""
    if x.dtype != torch.float32 or patched(module) or (x.numel() != K and (group <= FAST_DEQUANT_GROUP or not generating)):
        return type(module).forward(module, x, *args, **kwargs)
    x = x.contiguous()
    scale, bias = _scale(module, N, x.device), _bias(module, x.device)
    if group:
        x = rotate(x, group)
    qdata = module.weight._qdata
    if x.numel() != K:
        return F.linear(x, qdata.to(x.dtype) * scale[:, None], bias)
    out = ops.gemv_i8(x.reshape(K), qdata, scale, bias)
    return out.reshape(*x.shape[:-1], N)


def _dequantized(linear, dtype, device):
    w = linear.weight
    N = w._qdata.shape[0]
    return w._qdata.to(device=device, dtype=dtype) * _scale(linear, N, device)[:, None].to(dtype)


def mlp_forward(module, weight_dtype, x, norm=None):
    """Prefill of a gated MLP while generating (int8_gemv.py:67-75): one fp32 linear with the dequantized gate and up
    weights stacked (one GEMM of twice the width instead of two), then down_proj(activation(gate) * up). Single
    tokens, prompt encoding and patched layers use the module's own forward, whose linears are patched separately."""
    if (not generating or norm is not None or x.dtype != torch.float32 or x.numel() == x.shape[-1]
            or patched(module.gate_proj) or patched(module.up_proj)):
        return type(module).forward(module, x, norm)
    weight = torch.cat((_dequantized(module.gate_proj, x.dtype, x.device), _dequantized(module.up_proj, x.dtype, x.device)))
    gate, up = F.linear(x, weight).chunk(2, dim=-1)
    return module.down_proj(module.activation(gate) * up)


def logits(transformer, x):
    """Logits of the last position for one sequence from the tied bf16 embedding table (int8_gemv.py:87-98):
    out (1, 1, vocab) fp32 = embed . x[:, -1]. Other batches or dtypes use the transformer's own logits."""
    embed = transformer.model.embed_tokens
    if x.shape[0] != 1 or x.dtype != torch.float32 or patched(embed):
        return type(transformer).logits(transformer, x)
    x = x[:, -1:].contiguous()
    weight = embed.weight.to(device=x.device, dtype=torch.bfloat16)
    N, K = weight.shape
    return ops.gemv_bf16(x.reshape(K), weight.contiguous()).reshape(1, 1, N)


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


def _is(module, name):
    return any(c.__name__ == name for c in type(module).__mro__)


def patch(clip):
    """Single-token steps read the int8 and bf16 weights directly (int8_gemv.py:129-148): int8 linears, the gated
    MLPs' prefill, the logits of a tied-embedding Qwen3, and the fixed-capacity fp32 KV cache with its decode
    attention."""
    for name, module in clip.patcher.model.named_modules():
        w = getattr(module, "weight", None)
        if type(module).__name__ == "Linear" and getattr(module, "quant_format", None) == "int8_tensorwise" and w is not None:
            N, K = w.shape
            params = w._params
            if K % STEP == 0 and params.scale.numel() == N and params.scale.dtype == torch.float32 and not params.transposed:
                group = params.convrot_groupsize if params.convrot else 0
                clip.patcher.add_object_patch(f"{name}.forward", functools.partial(linear_forward, module, N, K, w.dtype, group))
        elif (_is(module, "MLP") and not getattr(module, "merged_mlp", False)
              and getattr(getattr(module, "gate_proj", None), "quant_format", None) == "int8_tensorwise"
              and getattr(getattr(module, "up_proj", None), "quant_format", None) == "int8_tensorwise"):
            clip.patcher.add_object_patch(f"{name}.forward", functools.partial(mlp_forward, module, module.gate_proj.weight.dtype))
        elif _is(module, "BaseQwen3") and not module.model.config.lm_head:
            embed = module.model.embed_tokens
            if embed.weight.dtype == torch.bfloat16 and embed.weight.shape[1] % BF16_STEP == 0:
                clip.patcher.add_object_patch(f"{name}.logits", functools.partial(logits, module))
            clip.patcher.add_object_patch(f"{name}.generate", functools.partial(generate, module))
            config = module.model.config
            if getattr(module.model, "fixed_kv", False) and config.head_dim == HEAD \
                    and config.num_attention_heads % config.num_key_value_heads == 0 \
                    and config.num_attention_heads // config.num_key_value_heads in (1, 2, 4, 8):
                try:
                    import comfy_kitchen
                    comfy_kitchen.flash_attention_decode = attention_decode
                except ImportError:
                    pass
                clip.patcher.add_object_patch(f"{name}.model.init_kv_cache", functools.partial(init_kv_cache, module.model))
