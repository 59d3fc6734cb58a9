"""B200 (sm_100a) implementation of the ComfyUI-RDNA2-Attention quantized DiT/LLM inner loop.

Drop-in modules with the reference's names: ``attention`` (optimized_attention override), ``hip_attention`` (low-level
fused attention), ``int8_gemm`` (W8A8 linears, ConvRot/SwiGLU/modulation pre-pass, fused Krea-2 block), ``rms_norm``
and ``int8_gemv`` (single-token decode). ``ops`` holds the tensor-level wrappers of the C-ABI library
``librdna2_b200.so``; ``dit`` and ``decoder`` are the benchmark-configuration drivers.

Like a ComfyUI custom node, this directory is loaded as a package by path (its name has dashes).
"""
from . import _lib, ops  # noqa: F401
from . import attention, hip_attention, int8_gemm, int8_gemv, rms_norm  # noqa: F401

__version__ = "1.0"
