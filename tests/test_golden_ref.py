"""Outputs of the reference's own kernels (tests/golden/hip_ref.npz, made by tests/golden/make_golden_ref.py from
the reference's .hip sources compiled for the host) against the oracle (CPU) and against this build's CUDA kernels
(GPU). The fixture needs no reference checkout, so the GPU half runs on the GPU machine.

Bit-exact: quantizers with and without ConvRot (edge values included), int4 activations, the int32 GEMM with its
fp16 epilogue (bias, gated residual), the int4 GEMM, the decode rotation. With tolerances, each stated below: the
stages through exp/exp2/rsqrt/fdot2, whose last-ulp behaviour differs between the reference's hardware, the host
that ran it, and the B200.
"""
import os

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import decode as odec
from oracle import gemm as ogemm
from oracle import norm as onorm
from oracle import quant as oq

F16, F32 = np.float16, np.float32
REF = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "hip_ref.npz"))


def close_int8(q, s, q_ref, s_ref, rate=2e-3):
    # One exp or rsqrt ulp can move an fp16 activation by a step and an int8 value by one.
    d = np.abs(np.asarray(q).astype(np.int32) - q_ref.astype(np.int32))
    assert d.max() <= 1 and np.mean(d != 0) < rate, (d.max(), np.mean(d != 0))
    assert np.max(np.abs(np.asarray(s, np.float64) - s_ref) / s_ref) < 2e-3


def steps(got, ref, n, rate):
    got, ref = np.asarray(got), np.asarray(ref)
    d = np.abs(got.astype(F32) - ref.astype(F32))
    assert np.all(d <= n * np.abs(np.spacing(ref.astype(F16))).astype(F32)), np.max(d)
    assert np.mean(got != ref) < rate


# ---------------------------------------------------------------- oracle (CPU)
def test_oracle_quantizers_match_reference():
    x = REF["quant_x"]
    for kind, rot in (("plain", 0), ("rotate", 256)):
        q, s, _ = oq.prepass(x, rot)
        assert np.array_equal(q, REF[f"quant_{kind}_q"]) and np.array_equal(s, REF[f"quant_{kind}_s"]), kind
    q, s = oq.quant_rows_i4(oq.rotate_rows(x, 256))
    assert np.array_equal(q, REF["quant_i4_q"]) and np.array_equal(s, REF["quant_i4_s"])


def test_oracle_linears_match_reference():
    x, w, ws, b = REF["lin_x"], REF["lin_w"], REF["lin_ws"], REF["lin_b"]
    q, s, _ = oq.prepass(x, 256)
    assert np.array_equal(ogemm.epilogue(ogemm.int_mm(q, w), s, ws, b), REF["lin_bias_y"])
    q, s, _ = oq.prepass(x, 0)
    y = ogemm.epilogue(ogemm.int_mm(q, w), s, ws, None, R=REF["lin_R"], G=REF["lin_G"], L=36)
    assert np.array_equal(y, REF["lin_res_y"])
    q4, s4 = oq.quant_rows_i4(oq.rotate_rows(x, 256))
    y = ogemm.epilogue(ogemm.int_mm(q4, ogemm.unpack_int4(REF["w4a4_w"])), s4, REF["w4a4_ws"])
    assert np.array_equal(y, REF["w4a4_y"])


def test_oracle_activations_match_reference():
    g, u = REF["act_gate"], REF["act_up"]
    close_int8(*oq.quant_rows(oq.rotate_rows(oq.swiglu(g, u), 256)), REF["act_swiglu_q"], REF["act_swiglu_s"])
    close_int8(*oq.quant_rows(oq.rotate_rows(oq.sigmoid_gate(g, u), 256)), REF["act_gate_q"], REF["act_gate_s"])
    hs = REF["act_situ_x"]
    K = hs.shape[1] // 2
    close_int8(*oq.quant_rows(oq.rotate_rows(oq.situ(hs[:, :K], hs[:, K:]), 256)), REF["act_situ_q"], REF["act_situ_s"])
    m = oq.modulate(REF["act_mod_x"], REF["act_mod_w"], REF["act_mod_s"], REF["act_mod_t"], 8, 1e-6)
    close_int8(*oq.quant_rows(oq.rotate_rows(m, 256)), REF["act_mod_q"], REF["act_mod_sc"])


def test_oracle_attention_norms_decode_match_reference():
    q, k, v = REF["attn_q"], REF["attn_k"], REF["attn_v"]
    for i8, name in ((False, "attn_fp16_o"), (True, "attn_i8_o")):
        sem = oatt.attention_semantics(q, k, v, 128 ** -0.5, int8_qk=i8, tile=16)
        assert oatt.rel_l2(sem, REF[name]) < 2e-4, name
    steps(onorm.rms_norm(REF["norm_x"], REF["norm_w"], 1e-6), REF["norm_y"], 2, 2e-3)
    r = onorm.rms_norm_rope(REF["rope_x"], 2, REF["rope_w"], 1e-6, REF["rope_f"])
    assert np.mean(r != REF["rope_y"]) < 5e-3 and np.max(np.abs(r.astype(F32) - REF["rope_y"].astype(F32))) < 1e-2
    assert np.array_equal(odec.rotate(REF["rot_x"], 256), REF["rot_256"])
    assert np.array_equal(odec.rotate(REF["rot_x"], 1024), REF["rot_1024"])
    assert oatt.rel_l2(odec.gemv_i8(REF["gemv_x"], REF["gemv_w"], REF["gemv_s"], REF["gemv_b"]), REF["gemv_y"]) < 1e-6
    assert oatt.rel_l2(odec.gemv_bf16(REF["bf16_x"], REF["bf16_w"]), REF["bf16_y"]) < 1e-6
    o = odec.attn_decode(REF["dec_q"], REF["dec_k"], REF["dec_v"], REF["dec_len"], 128 ** -0.5)
    assert oatt.rel_l2(o, REF["dec_o"]) < 1e-6


# ---------------------------------------------------------------- CUDA kernels (GPU)
def _d(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _h(t):
    return t.detach().cpu().numpy()


@pytest.mark.gpu
def test_cuda_prepass_and_linears_match_reference(pkg, dev):
    ops = pkg.ops
    x = _d(REF["quant_x"], dev)
    for kind, rot in (("plain", 0), ("rotate", 256)):
        q, s = ops.quant_pack_a(x, rot)
        assert np.array_equal(_h(q), REF[f"quant_{kind}_q"]) and np.array_equal(_h(s), REF[f"quant_{kind}_s"]), kind
    q, s = ops.quant_pack_a_i4(x, 256)
    assert np.array_equal(_h(q), REF["quant_i4_q"]) and np.array_equal(_h(s), REF["quant_i4_s"])
    xl, w, ws = _d(REF["lin_x"], dev), _d(REF["lin_w"], dev), _d(REF["lin_ws"], dev)
    q, s = ops.quant_pack_a(xl, 256)
    assert np.array_equal(_h(ops.gemm(q, s, w, ws, _d(REF["lin_b"], dev))), REF["lin_bias_y"])
    q, s = ops.quant_pack_a(xl, 0)
    G = _d(REF["lin_G"], dev)
    y = ops.gemm(q, s, w, ws, residual=_d(REF["lin_R"], dev), gate=G, L=36)
    assert np.array_equal(_h(y), REF["lin_res_y"])
    q4, s4 = ops.quant_pack_a_i4(xl, 256)
    y = ops.gemm_w4a4(q4, s4, _d(REF["w4a4_w"], dev), _d(REF["w4a4_ws"], dev))
    assert np.array_equal(_h(y), REF["w4a4_y"])
    assert pkg._lib.device_status() == 0


@pytest.mark.gpu
def test_cuda_activations_match_reference(pkg, dev):
    ops = pkg.ops
    g, u = _d(REF["act_gate"], dev), _d(REF["act_up"], dev)
    close_int8(*map(_h, ops.swiglu_quant_pack_a(g, u, 256)), REF["act_swiglu_q"], REF["act_swiglu_s"])
    close_int8(*map(_h, ops.gate_quant_pack_a(g, u, 256)), REF["act_gate_q"], REF["act_gate_s"])
    close_int8(*map(_h, ops.situ_quant_pack_a(_d(REF["act_situ_x"], dev), 256)), REF["act_situ_q"], REF["act_situ_s"])
    q, s = ops.mod_quant_pack_a(_d(REF["act_mod_x"], dev), _d(REF["act_mod_w"], dev), _d(REF["act_mod_s"], dev),
                                _d(REF["act_mod_t"], dev), 8, 1e-6, 256)
    close_int8(_h(q), _h(s), REF["act_mod_q"], REF["act_mod_sc"])


@pytest.mark.gpu
def test_cuda_attention_norms_decode_match_reference(pkg, dev):
    ops = pkg.ops
    q, k, v = (_d(REF[n], dev) for n in ("attn_q", "attn_k", "attn_v"))
    for i8, name, tol in ((False, "attn_fp16_o", 2e-3), (True, "attn_i8_o", 1e-2)):
        out = torch.empty_like(q)
        ops.attention(q, k, v, out, 128 ** -0.5, i8)
        # 128-key tiles here against the reference's 16-key steps: different lazy-rescale points, fp16 P.
        assert oatt.rel_l2(_h(out), REF[name]) < tol, name
    steps(_h(pkg.rms_norm.rms_norm(_d(REF["norm_x"], dev), _d(REF["norm_w"], dev), 1e-6)), REF["norm_y"], 2, 2e-3)
    module = type("RMSNorm", (), {})()
    module.scale, module.eps = torch.from_numpy(REF["rope_w"]), 1e-6
    r = _h(pkg.rms_norm.rms_norm_rope(_d(REF["rope_x"], dev), 2, module, _d(REF["rope_f"], dev)))
    assert np.mean(r != REF["rope_y"]) < 5e-3 and np.max(np.abs(r.astype(F32) - REF["rope_y"].astype(F32))) < 1e-2
    assert np.array_equal(_h(ops.rotate(_d(REF["rot_x"], dev), 256)), REF["rot_256"])
    assert np.array_equal(_h(ops.rotate(_d(REF["rot_x"], dev), 1024)), REF["rot_1024"])
    y = ops.gemv_i8(_d(REF["gemv_x"], dev), _d(REF["gemv_w"], dev), _d(REF["gemv_s"], dev), _d(REF["gemv_b"], dev))
    assert oatt.rel_l2(_h(y), REF["gemv_y"]) < 1e-5
    assert oatt.rel_l2(_h(ops.gemv_bf16(_d(REF["bf16_x"], dev), _d(REF["bf16_w"].view(np.int16), dev).view(torch.bfloat16))), REF["bf16_y"]) < 1e-5
    o = ops.attn_decode(_d(REF["dec_q"], dev), _d(REF["dec_k"], dev), _d(REF["dec_v"], dev), _d(REF["dec_len"], dev),
                        128 ** -0.5)
    assert oatt.rel_l2(_h(o), REF["dec_o"]) < 1e-5
    assert pkg._lib.device_status() == 0
