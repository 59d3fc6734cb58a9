"""Fused RMSNorm, the drop-in for the reference's rms_norm.py (:25-64).

Same functions and signatures: ``rms_norm(x, weight, eps)``, ``rms_norm_rope(x, heads, module, freqs)``,
``forward(module, x)`` and ``patch(model)``. ``module`` is anything with the attributes of ComfyUI's Krea-2
``RMSNorm``: ``scale`` (zero-centred weight) and ``eps``. Ineligible inputs raise instead of falling back to the
module's own forward (rms_norm.py:56-57).
"""
import functools

import torch

from . import ops

THREADS = 256
HEAD_DIM = 128
MAX_DIM = 8192


def _weight(module, device):
    w = module.scale
    return w.to(dtype=torch.float32, device=device).contiguous()


def rms_norm(x, weight, eps):
    """x is (B, L, D) or (B, H, L, D) fp16 with a contiguous last dimension, weight (D,) fp32 and zero-centered.
    Returns contiguous fp16 (rms_norm.py:25-39)."""
    v = x if x.ndim == 4 else x.unsqueeze(1)
    B, H, L, D = v.shape
    sb, sh, sl = v.stride()[:3]
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    return ops.rms_norm_rows(x, weight.float().contiguous(), eps, B * H * L, D, L, H, sb, sh, sl, out)


def rms_norm_rope(x, heads, module, freqs):
    """x is (B, L, heads * 128) fp16 and freqs (B or 1, 1, L, 64, 2, 2) fp32. Returns (B, heads, L, 128) with
    QK-norm and rope applied (rms_norm.py:42-52)."""
    B, L, _ = x.shape
    out = torch.empty((B, heads, L, HEAD_DIM), dtype=x.dtype, device=x.device)
    freqs = freqs.to(torch.float32).contiguous()
    fb = L * HEAD_DIM // 2 if freqs.shape[0] > 1 else 0
    return ops.rms_norm_rows(x, _weight(module, x.device), module.eps, B * heads * L, HEAD_DIM, L, heads,
                             x.stride(0), HEAD_DIM, x.stride(1), out, freqs=freqs, fb=fb)


def forward(module, x):
    if x.dtype != torch.float16 or x.ndim not in (3, 4) or x.stride(-1) != 1 or x.shape[-1] % 8 != 0 or x.shape[-1] > MAX_DIM:
        raise NotImplementedError("rms_norm.forward needs fp16 (B, L, D) or (B, H, L, D) with D % 8 == 0, D <= 8192")
    return rms_norm(x, _weight(module, x.device), module.eps)


def patch(model):
    """Patches every RMSNorm of a ComfyUI diffusion model (rms_norm.py:61-64)."""
    for name, module in model.get_model_object("diffusion_model").named_modules():
        if type(module).__name__ == "RMSNorm" and hasattr(module, "scale") and hasattr(module, "eps"):
            model.add_object_patch(f"diffusion_model.{name}.forward", functools.partial(forward, module))
