"""ctypes binding of librdna2_b200.so, the sm_100a C-ABI (declared in include/rdna2_b200.h).

The reference binds its HIP kernels the same way (hip_attention.py:11-42): ctypes, raw device pointers, int
dims and float scalars, launched on torch's current stream, ``RuntimeError`` on a non-zero status. There is no
CPU fallback: if the library is missing or no CUDA device is present, calls raise.
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librdna2_b200.so")

P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
F = ctypes.c_float

# name -> (restype, argtypes), mirroring include/rdna2_b200.h
SIGNATURES = {
    "b2_version": (I, []),
    "b2_last_error": (ctypes.c_char_p, []),
    "b2_device_status": (I, [P]),
    "b2_quant_pack_a": (I, [P, I64, P, P, I, I, I, P]),
    "b2_quant_pack_a_seg": (I, [P, I64, I, I64, P, P, I, I, I, P]),
    "b2_swiglu_quant_pack_a": (I, [P, P, I64, P, P, I, I, I, P, P]),
    "b2_gate_quant_pack_a": (I, [P, P, I64, P, P, I, I, I, P, P]),
    "b2_situ_quant_pack_a": (I, [P, I64, P, P, I, I, I, P, P]),
    "b2_mod_quant_pack_a": (I, [P, I64, P, P, P, I, F, P, P, I, I, I, P, P]),
    "b2_gemm": (I, [P, P, P, P, P, P, I, I, I, P, P, I, P]),
    "b2_gemm_i32": (I, [P, P, P, I, I, I, P]),
    "b2_gemm_swiglu": (I, [P, P, P, P, P, I, I, I, P]),
    "b2_gemm_w4a8": (I, [P, P, P, P, P, P, I, I, I, P]),
    "b2_gemm_w4a8_wide": (I, [P, P, P, P, P, P, I, I, I, P]),
    "b2_quant_pack_a_i4": (I, [P, I64, P, P, I, I, I, P]),
    "b2_unpack_int4": (I, [P, P, I, I, P]),
    "b2_gemm_w4a4": (I, [P, P, P, P, P, P, I, I, I, P, P]),
    "b2_attention_workspace_bytes": (I64, [I, I, I, I, I, I]),
    "b2_attention": (I, [P, I64, I64, I64, P, I64, I64, I64, P, I64, I64, I64, P, I64, I64, I64,
                         I, I, I, I, I, F, I, P, I64, P]),
    "b2_attention_gather": (I, [P, I64, I64, I64, P, I64, I64, I64, P, I64, I64, I64, P, I64, I64, I64,
                                I, I, I, I, I, F, I, P, I64, P, P, I, P]),
    "b2_attention_gather_ctas": (I, [I, I, I]),
    "b2_wait_count": (I, [P, ctypes.c_ulonglong, P, ctypes.c_longlong, P]),
    "b2_rms_norm": (I, [P, P, P, I, I, I, I, I64, I64, I64, F, P]),
    "b2_rms_norm_rope": (I, [P, P, P, I, I, I, I, I64, I64, I64, F, P, I64, P]),
    "b2_rotate": (I, [P, P, I64, I, P]),
    "b2_gemv_i8": (I, [P, P, P, P, P, I, I, P]),
    "b2_gemv_i8_ex": (I, [P, P, P, P, P, P, I, I, I, P]),
    "b2_gemv_bf16": (I, [P, P, P, I, I, P]),
    "b2_rms_norm_f32": (I, [P, P, P, I, F, P]),
    "b2_decode_qk_rope": (I, [P, P, P, P, P, P, P, P, I, I, F, P]),
    "b2_attn_decode": (I, [P, P, P, P, P, P, P, I, I, I, I, F, P]),
    "b2_attn_decode_noalloc": (I, [P, P, P, P, P, I, I, I, I, F, P]),
    "b2_decode_step": (I, [P, I, P, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, F, ctypes.c_longlong, P]),
    "b2_decode_step_splits": (I, [I]),
}

_lib = None


def load():
    """Loads the library once and declares every entry point. Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing; build it with build.py (nvcc, sm_100a). There is no CPU fallback.")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status, what=""):
    if status != 0:
        msg = load().b2_last_error().decode(errors="replace")
        raise RuntimeError(f"rdna2_b200 {what} failed with status {status}: {msg}")


def call(name, *args):
    check(getattr(load(), name)(*args), name)


def stream():
    return P(torch.cuda.current_stream().cuda_stream)


def ptr(t):
    return P(t.data_ptr()) if t is not None else P(None)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("rdna2_b200 kernels need CUDA tensors; there is no CPU fallback")


def device_status():
    """Synchronizes and returns the device status bits that bounded waits set when they ran out (0 = none)."""
    flags = ctypes.c_uint(0)
    load().b2_device_status(ctypes.byref(flags))
    return flags.value
