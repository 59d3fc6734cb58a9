"""W8A8 linear layers, the drop-in for the reference's int8_gemm.py.

It keeps the reference's entry points and its hand-off protocol with the Int8 loader (ComfyUI-INT8-Fast-ROCM):
``wrap`` returns the ``int8_linear`` that replaces the pack's ``triton_int8_linear(_per_row)`` (int8_gemm.py:105-129),
``rotate_activation`` leaves the ConvRot rotation to the pre-pass kernel by parking the tensor in ``pending``
(:132-142), ``swiglu_forward`` hands the up projection to the down layer's quantization (:160-167),
``quantize_block_input`` / ``block_forward`` fuse a Krea-2 block (:176-226), ``enable`` installs the patches (:247-271).
Module globals are the same side channels as the reference's (:25-41).

Differences, all by design of this build: every linear runs the sm_100a kernels (pre-pass + tcgen05 GEMM reading the
weight as stored: no pack_b), for any row count, so MIN_ROWS is 1; inputs the kernels cannot take raise instead of
falling back to the pack's Triton path; the rotation group is a parameter (256 = ConvRot as in the reference, 128 =
the block-128 configuration). ``wrap_w4a4`` runs the Int4 loader's per-channel W4A4 layers (int8_gemm.py:90-103) and
``linear_input_act`` hands situ activations to the pre-pass (:152-157), as in the reference; ``w4a8_forward`` is the
configuration-3 W4A8 (group-128 scales) in the same call shape.
"""
import functools
import logging
import sys

import torch
import torch.nn.functional as F

from . import hip_attention, ops, rms_norm

MIN_ROWS = 1
MAX_ROT_K = 16384
ROT_GROUP = 256

originals = {}
fusable = False
pending = None
situ_next = False
swiglu_up = None
sigmoid_gate = None
shared = None
residual = None
swiglu_fusable = False


def quantized(M, K, device):
    """(int8 [M, K], fp32 [M]) activation buffers (int8_gemm.py:51-53; plain row-major here)."""
    return (torch.empty((M, K), dtype=torch.int8, device=device), torch.empty((M,), dtype=torch.float32, device=device))


def run(x, weight, weight_scale, bias, rotate=False, up=None, gate=None, activations=None, res=None, rot_group=ROT_GROUP,
        situ=False):
    """Pre-pass (unless ``activations`` are given) then GEMM. x (M, K) fp16, or (M, 2K) [hidden | gate] with situ;
    weight (N, K) int8; weight_scale (N,) fp32; res = (R (M, N) fp16, G (M / L, N) fp16) adds R + G * y. Returns
    (M, N) fp16 (int8_gemm.py:56-80)."""
    M = x.shape[0] if activations is None else activations[0].shape[0]
    N, K = weight.shape
    group = rot_group if rotate or situ else 0
    if activations is None:
        out = quantized(M, K, x.device)
        if situ:
            if x.shape[1] != 2 * K:
                raise RuntimeError(f"situ input width {x.shape[1]} is not 2 x K = {2 * K}")
            activations = ops.situ_quant_pack_a(x, group, out=out)
        elif up is not None:
            activations = ops.swiglu_quant_pack_a(x, up, group, out=out)
        elif gate is not None:
            activations = ops.gate_quant_pack_a(x, gate, group, out=out)
        else:
            activations = ops.quant_pack_a(x, group, out=out)
    a_q, a_s = activations
    R, G, L = (None, None, 1)
    if res is not None:
        R = res[0].reshape(M, N).contiguous()
        G = res[1].reshape(-1, N).contiguous()
        L = M // G.shape[0]
    return ops.gemm(a_q, a_s, weight, weight_scale, bias, residual=R, gate=G, L=L)


def linear(x, weight, weight_scale, bias, rotate=False, situ=False, up=None, gate=None, activations=None, res=None,
           rot_group=ROT_GROUP):
    """x is (M, K) fp16, or (M, 2K) with situ, weight (N, K) int8 and weight_scale (N,) fp32. With up, x is the gate
    of a SwiGLU. With gate, x is multiplied by its sigmoid. With situ, x's rows are [hidden | gate] and the pre-pass
    applies the situ activation, then ConvRot (situ layers always rotate: int8_gemm.py:152-157 only hands over layers
    that do). Returns (M, N) fp16 (int8_gemm.py:83-87)."""
    return run(x, weight, weight_scale, bias, rotate, up, gate, activations, res, rot_group, situ)


def ineligible(x, weight, bias, compute_dtype, x_q):
    N, K = weight.shape
    if x_q is not None:
        return "pre-quantized x_q"
    if x.dtype != torch.float16 or compute_dtype != torch.float16:
        return "non-fp16 input or compute dtype"
    if bias is not None and bias.dtype != torch.float16:
        return "non-fp16 bias"
    if N % 8 or K % 16:
        return f"N={N} must be a multiple of 8 and K={K} of 16"
    return None


def wrap(original):
    def int8_linear(x, weight, weight_scale, bias=None, compute_dtype=torch.float16, x_q=None):
        global pending, situ_next, swiglu_up, sigmoid_gate, residual
        rotate, situ, up, gate, res = x is pending, situ_next, swiglu_up, sigmoid_gate, residual
        pending, situ_next, swiglu_up, sigmoid_gate, residual = None, False, None, None, None
        N, K = weight.shape
        reason = ineligible(x, weight, bias, compute_dtype, x_q)
        if reason:
            raise NotImplementedError(f"int8_linear: {reason}")
        if isinstance(weight_scale, torch.Tensor) and weight_scale.numel() == N:
            scale = weight_scale.reshape(N).float().contiguous()
        else:
            scale = torch.full((N,), float(weight_scale), dtype=torch.float32, device=x.device)
        out = linear(x.reshape(-1, x.shape[-1]).contiguous(), weight.contiguous(), scale, bias, rotate, situ,
                     None if up is None else up.reshape(-1, K).contiguous(), gate, shared, res)
        return out.reshape(x.shape[:-1] + (N,))
    return int8_linear


def w4a4_ineligible(x, qweight, wscales, bias, convrot_groupsize, compute_dtype, skip_rotation, x_rot):
    N, row_bytes = qweight.shape
    K = row_bytes * 2
    if x_rot is not None or skip_rotation:
        return "a pre-rotated input (x_rot / skip_rotation)"
    if convrot_groupsize != ROT_GROUP:
        return f"ConvRot group {convrot_groupsize} (the W4A4 pre-pass rotates by {ROT_GROUP})"
    if compute_dtype != torch.float16:
        return "non-fp16 compute dtype"
    if x.shape[-1] != K or K > MAX_ROT_K:
        return f"input width {x.shape[-1]} against K = {K} (at most {MAX_ROT_K})"
    if N % 8 or K % 256:
        return f"N={N} must be a multiple of 8 and K={K} of 256"
    if bias is not None and bias.dtype != torch.float16:
        return "non-fp16 bias"
    if wscales.numel() != N:
        return "weight scales that are not one per output channel"
    return None


def wrap_w4a4(original):
    """convrot_w4a4_forward of the Int4 loader on the sm_100a kernels (int8_gemm.py:90-103): ConvRot-256 and
    int4-valued per-token activations in one pre-pass, the packed weight widened to int8 and multiplied on the
    tcgen05 int8 GEMM with int32 accumulation, the per-channel epilogue. ``qweight_unpacked``, the weight widened to
    int8 [N, K] once at load time (as w4a8_forward takes it), feeds the GEMM directly; without it the packed weight
    is widened per call into a temporary, as the reference re-packs it (int8_gemm.py:73-75). Both give the same result
    bit for bit. Ineligible calls raise (no fallback)."""
    def convrot_w4a4_forward(x, qweight, wscales, bias, convrot_groupsize, compute_dtype, skip_rotation=False,
                             qweight_unpacked=None, x_rot=None, orig_shape=None):
        reason = w4a4_ineligible(x, qweight, wscales, bias, convrot_groupsize, compute_dtype, skip_rotation, x_rot)
        if reason:
            raise NotImplementedError(f"convrot_w4a4_forward: {reason}")
        N, K = qweight.shape[0], qweight.shape[1] * 2
        if qweight_unpacked is not None and (qweight_unpacked.dtype != torch.int8
                                             or tuple(qweight_unpacked.shape) != (N, K)):
            raise NotImplementedError(f"convrot_w4a4_forward: qweight_unpacked must be int8 [{N}, {K}]")
        x2d = x.reshape(-1, K).to(torch.float16).contiguous()
        a_q, a_s = ops.quant_pack_a_i4(x2d, ROT_GROUP)
        ws = wscales.reshape(N).float().contiguous()
        if qweight_unpacked is not None:
            out = ops.gemm(a_q, a_s, qweight_unpacked.contiguous(), ws, bias)
        else:
            out = ops.gemm_w4a4(a_q, a_s, qweight.contiguous(), ws, bias)
        return out.reshape(x.shape[:-1] + (N,))
    return convrot_w4a4_forward


def w4a8_forward(x, qweight, wscales, bias, convrot_groupsize, compute_dtype, skip_rotation=False,
                 qweight_unpacked=None, x_rot=None, orig_shape=None):
    """W4A8 with group-128 weight scales (the configuration-3 form) in the call shape of convrot_w4a4_forward
    (int8_gemm.py:91): x fp16 (..., K) is rotated by ``convrot_groupsize`` (128: block-128 Sylvester, 256: ConvRot)
    and quantized per token to int8 in one pre-pass; qweight is packed int4 [N, K/2] (low nibble = even k); wscales
    are fp16 [N, K/128], one scale per output channel and 128 values of K. The GEMM combines the int32 partial sum of
    each 128-value group with its scale in fp32, in group order, then scales by the token's scale (+ bias).
    ``qweight_unpacked``, the weight widened to int8 [N, K] once at load time, feeds the GEMM directly; without it
    the packed weight is widened into a temporary first (as the reference re-packs its weight per call,
    int8_gemm.py:73-75), which measured faster than widening inside the GEMM. Both give the same result bit for
    bit."""
    N, K = qweight.shape[0], qweight.shape[1] * 2
    if x_rot is not None or skip_rotation:
        raise NotImplementedError("w4a8_forward: a pre-rotated input (x_rot / skip_rotation)")
    if convrot_groupsize not in (ROT_GROUP, 128) or compute_dtype != torch.float16 or x.shape[-1] != K or K % 128:
        raise NotImplementedError(f"w4a8_forward: group {convrot_groupsize}, {compute_dtype}, K={K} (needs 128 or 256, "
                                  "fp16, K % 128 == 0)")
    if tuple(wscales.shape) != (N, K // 128):
        raise NotImplementedError(f"w4a8_forward: scales of shape {tuple(wscales.shape)}, expected ({N}, {K // 128})")
    qweight = qweight.contiguous()
    if qweight_unpacked is None:
        qweight_unpacked = ops.unpack_int4(qweight)
    elif qweight_unpacked.dtype != torch.int8 or tuple(qweight_unpacked.shape) != (N, K):
        raise NotImplementedError(f"w4a8_forward: qweight_unpacked must be int8 [{N}, {K}]")
    x2d = x.reshape(-1, K).to(torch.float16).contiguous()
    a_q, a_s = ops.quant_pack_a(x2d, convrot_groupsize)
    out = ops.gemm_w4a8(a_q, a_s, qweight, ops.w4a8_scales(wscales.to(torch.float16)), bias,
                        w_wide=qweight_unpacked.contiguous())
    return out.reshape(x.shape[:-1] + (N,))


def rotate_activation(x, H, group_size):
    """ConvRot hand-off (int8_gemm.py:132-142): the next int8_linear rotates inside its pre-pass."""
    global pending
    if shared is not None:
        return x
    if situ_next or swiglu_up is not None or sigmoid_gate is not None:
        pending = x
        return x
    if fusable and group_size == ROT_GROUP and x.dtype == torch.float16 and x.dim() == 2 and x.shape[1] % ROT_GROUP == 0 \
            and x.shape[1] <= MAX_ROT_K:
        pending = x
        return x
    return originals["rotate_activation"](x, H, group_size)


def fuse_act(layer, x, K):
    """Layers whose activation, ConvRot and quantization run as one pre-pass (int8_gemm.py:145-150)."""
    return (getattr(layer, "_is_quantized", False) and getattr(layer, "_use_convrot", False) and not getattr(layer, "_is_w4a8", False)
            and getattr(layer, "_convrot_groupsize", 0) == ROT_GROUP and not getattr(layer, "lora_patches", None)
            and x.dtype == torch.float16 and K == layer.in_features and layer.in_features % ROT_GROUP == 0
            and layer.in_features <= MAX_ROT_K)


def linear_input_act(linear, x, input_act, act_weight=None, act_eps=0.0, residual=None, residual_scale=None):
    """comfy.ops.linear_input_act for situ layers (int8_gemm.py:152-157): the raw [hidden | gate] input goes to the
    linear, whose pre-pass applies the activation, so the K-wide activation never goes through HBM."""
    global situ_next
    if input_act == "situ" and residual is None and fuse_act(linear, x, x.shape[-1] // 2):
        situ_next = True
        return linear(x)
    return originals["linear_input_act"](linear, x, input_act, act_weight, act_eps, residual, residual_scale)


def swiglu_forward(module, x):
    """SwiGLU with the activation folded into the down layer's quantization (int8_gemm.py:160-167)."""
    global swiglu_up
    gate, up = module.gate(x), module.up(x)
    if swiglu_fusable and isinstance(module.down, originals["layer"]) and fuse_act(module.down, gate, gate.shape[-1]):
        swiglu_up = up
        return module.down(gate)
    return module.down(F.silu(gate).mul_(up))


def patch_swiglu(model):
    for name, module in model.get_model_object("diffusion_model").named_modules():
        if type(module).__name__ == "SwiGLU":
            model.add_object_patch(f"diffusion_model.{name}.forward", functools.partial(swiglu_forward, module))


def quantize_block_input(x, norm, scale, shift, rot_group=ROT_GROUP):
    """Sets ``shared`` to the quantized (1 + scale) * norm(x) + shift that all of a block's input linears read
    (int8_gemm.py:176-186)."""
    global shared
    B, L, K = x.shape
    weight = norm.scale.to(dtype=torch.float32, device=x.device).contiguous()
    s = (1 + scale).to(torch.float16).reshape(-1, K).contiguous()
    t = shift.to(torch.float16).reshape(-1, K).contiguous()
    shared = ops.mod_quant_pack_a(x.reshape(B * L, K), weight, s, t, L, norm.eps, rot_group)


def block_forward(module, int8_qk, x, vec, freqs, mask=None, timestep_zero_index=None, transformer_options={}):
    """Krea-2 SingleStreamBlock.forward with everything between the matmuls fused (int8_gemm.py:189-226)."""
    global shared, swiglu_up, sigmoid_gate, residual
    attn, mlp = module.attn, module.mlp
    patches = transformer_options.get("patches", {})
    if (mask is not None or timestep_zero_index is not None or freqs is None or "attn1_patch" in patches
            or "attn1_output_patch" in patches or x.dtype != torch.float16 or attn.headdim != rms_norm.HEAD_DIM):
        raise NotImplementedError("block_forward: masks, patches, non-fp16 or head dim != 128 are not supported")
    B, L, D = x.shape
    prescale, preshift, pregate, postscale, postshift, postgate = module.mod(vec)
    try:
        quantize_block_input(x, module.prenorm, prescale, preshift)
        q, k, v, gate = attn.wq(x), attn.wk(x), attn.wv(x), attn.gate(x)
        shared = None

        q = rms_norm.rms_norm_rope(q, attn.heads, attn.qknorm.qnorm, freqs)
        k = rms_norm.rms_norm_rope(k, attn.kvheads, attn.qknorm.knorm, freqs)
        v = v.view(B, L, attn.kvheads, attn.headdim).transpose(1, 2)
        out = torch.empty((B, L, attn.heads, attn.headdim), dtype=x.dtype, device=x.device)
        hip_attention.attention(q, k, v, out.transpose(1, 2), attn.headdim ** -0.5, int8_qk)

        sigmoid_gate = gate.view(-1, D)
        residual = x, pregate.contiguous()
        x = attn.wo(out.view(B, L, D))

        quantize_block_input(x, module.postnorm, postscale, postshift)
        gate, up = mlp.gate(x), mlp.up(x)
        shared = None

        swiglu_up = up
        residual = x, postgate.contiguous()
        return mlp.down(gate)
    finally:
        shared = swiglu_up = sigmoid_gate = residual = None


def patch_block(model, int8_qk):
    for name, module in model.get_model_object("diffusion_model").named_modules():
        if type(module).__name__ == "SingleStreamBlock":
            model.add_object_patch(f"diffusion_model.{name}.forward", functools.partial(block_forward, module, int8_qk))


def wrap_forward(forward):
    def int8_forward(self, x):
        global fusable
        fusable = not getattr(self, "lora_patches", None)
        try:
            return forward(self, x)
        finally:
            fusable = False
    return int8_forward


def enable(on):
    """Installs (or removes) the patches in the loaded Int8/Int4 packs (int8_gemm.py:247-271)."""
    global swiglu_fusable
    pack = next((m for name, m in sys.modules.items() if name.endswith(".int8_quant") and hasattr(m, "triton_int8_linear_per_row")), None)
    int4 = next((m for name, m in sys.modules.items() if name.endswith(".int4_quant") and hasattr(m, "convrot_w4a4_forward")), None)
    if int4 is not None:
        originals.setdefault("convrot_w4a4_forward", int4.convrot_w4a4_forward)
        int4.convrot_w4a4_forward = wrap_w4a4(originals["convrot_w4a4_forward"]) if on else originals["convrot_w4a4_forward"]
    if pack is None:
        if on:
            logging.warning("rdna2_b200: int8_gemm skipped, ComfyUI-INT8-Fast-ROCM is not loaded.")
        return
    convrot = next(m for name, m in sys.modules.items() if name.endswith(".convrot") and hasattr(m, "rotate_activation"))
    layer = pack.Int8TensorwiseOps.Linear
    if "forward" not in originals:
        originals.update(layer=layer, triton_int8_linear=pack.triton_int8_linear,
                         triton_int8_linear_per_row=pack.triton_int8_linear_per_row,
                         rotate_activation=convrot.rotate_activation, build_hadamard=convrot.build_hadamard,
                         forward=layer.forward)
    comfy_ops = sys.modules.get("comfy.ops")
    if comfy_ops is not None and hasattr(comfy_ops, "linear_input_act"):
        originals.setdefault("linear_input_act", comfy_ops.linear_input_act)
        comfy_ops.linear_input_act = linear_input_act if on else originals["linear_input_act"]
    for name in ("triton_int8_linear", "triton_int8_linear_per_row"):
        setattr(pack, name, wrap(originals[name]) if on else originals[name])
    convrot.rotate_activation = rotate_activation if on else originals["rotate_activation"]
    layer.forward = wrap_forward(originals["forward"]) if on else originals["forward"]
    swiglu_fusable = on and getattr(pack, "_TRITON_AVAILABLE", True)
