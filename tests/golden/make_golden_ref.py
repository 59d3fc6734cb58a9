"""Generates tests/golden/hip_ref.npz: outputs of the reference's own kernels on seeded inputs.

The reference's int8_gemm.hip, hip_attention.hip, int8_gemv.hip and rms_norm.hip are compiled for the host by
oracle/hipemu/build.py (the reference checkout is named by REF_DIR) and launched through oracle/hipref.py the way
the reference's Python launches them. The fixture keeps inputs and outputs small (a few hundred KB) so that the
GPU tests can compare this build's kernels with the reference's results on a machine without the reference, and
the CPU tests can check the oracle against them. Cases:
  quant_*      quant_pack_a / rot_quant_pack_a / rot_quant_pack_a_i4 on random and edge-value rows
  act_*        swiglu / gate / situ / mod pre-passes (int8 + scales)
  lin_*        run(): pre-pass + pack_b + gemm with bias, and with the gated residual
  w4a4_*       wrap_w4a4's gemm_i4 path
  attn_*       pack_kv + attn and the int8-QK variant (grouped-query heads, ragged key count)
  norm_*, rope_*   rms_norm_row / rms_norm_head / rms_norm_rope
  rot_*, gemv_*, bf16_*, dec_*   the decode kernels
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import hipref as hr  # noqa: E402
from oracle.hipemu import build as hbuild  # noqa: E402

OUT = os.path.join(HERE, "hip_ref.npz")
F16, F32 = np.float16, np.float32


def edge_rows(K):
    x = np.zeros((8, K), F16)
    x[1, :] = 65504
    x[2, ::2] = 6e-8
    x[3, :8] = [127, 0.5, -0.5, 1.5, -1.5, 2.5, -2.5, -127]
    x[4] = np.linspace(-3, 3, K).astype(F16)
    x[6] = np.linspace(-1, 1, K).astype(F16)
    x[6, 130] = np.nan
    x[7] = np.linspace(-2, 2, K).astype(F16)
    x[7, 5] = -np.inf
    return x


def main():
    if hbuild.build() is None:
        sys.exit("set REF_DIR to the reference checkout (the directory holding int8_gemm.hip)")
    g = np.random.default_rng(20261202)
    c = {}
    # Pre-passes.
    x = g.standard_normal((16, 512)).astype(F32)
    x[:, g.choice(512, 5, replace=False)] *= 20
    x = np.concatenate([x.astype(F16), edge_rows(512)])
    c["quant_x"] = x
    for kind in ("plain", "rotate", "i4"):
        c[f"quant_{kind}_q"], c[f"quant_{kind}_s"] = hr.quant(x, kind)
    gate = (g.standard_normal((16, 512)) * 2).astype(F16)
    up = g.standard_normal((16, 512)).astype(F16)
    c["act_gate"], c["act_up"] = gate, up
    for kind in ("swiglu", "gate"):
        c[f"act_{kind}_q"], c[f"act_{kind}_s"] = hr.quant(gate, kind, u=up)
    hs = np.concatenate([(g.standard_normal((16, 256)) * 30).astype(F16), (g.standard_normal((16, 256)) * 3).astype(F16)], 1)
    c["act_situ_x"] = hs
    c["act_situ_q"], c["act_situ_s"] = hr.quant(hs, "situ")
    xm = g.standard_normal((16, 512)).astype(F16)
    wm = (g.standard_normal(512) * 0.02).astype(F32)
    sm = (1 + g.standard_normal((2, 512)) * 0.1).astype(F16)
    tm = (g.standard_normal((2, 512)) * 0.1).astype(F16)
    c.update(act_mod_x=xm, act_mod_w=wm, act_mod_s=sm, act_mod_t=tm)
    c["act_mod_q"], c["act_mod_sc"] = hr.quant(xm, "mod", w=wm, s=sm, t=tm, L=8, eps=1e-6)
    # Linears.
    xl = g.standard_normal((72, 256)).astype(F16)
    wl = g.integers(-127, 128, (64, 256), dtype=np.int8)
    sl = (g.random(64) * 1e-3).astype(F32)
    bl = (g.standard_normal(64) * 0.01).astype(F16)
    R = g.standard_normal((72, 64)).astype(F16)
    G = (g.standard_normal((2, 64)) * 0.5).astype(F16)
    c.update(lin_x=xl, lin_w=wl, lin_ws=sl, lin_b=bl, lin_R=R, lin_G=G)
    c["lin_bias_y"] = hr.linear(xl, wl, sl, bl, kind="rotate")
    c["lin_res_y"] = hr.linear(xl, wl, sl, None, kind="plain", res=(R, G, 36))
    wp = g.integers(0, 256, (64, 128), dtype=np.uint8)
    sp = (g.random(64) * 1e-2).astype(F32)
    c.update(w4a4_w=wp, w4a4_ws=sp)
    c["w4a4_y"] = hr.linear(xl, wp, sp, None, i4=True)
    # Attention.
    q = g.standard_normal((1, 2, 40, 128)).astype(F16)
    k = g.standard_normal((1, 1, 50, 128)).astype(F16)
    v = g.standard_normal((1, 1, 50, 128)).astype(F16)
    c.update(attn_q=q, attn_k=k, attn_v=v)
    c["attn_fp16_o"] = hr.attention(q, k, v, 128 ** -0.5, False)
    c["attn_i8_o"] = hr.attention(q, k, v, 128 ** -0.5, True)
    # Norms.
    xn = (g.standard_normal((2, 5, 512)) * 3).astype(F16)
    wn = (g.standard_normal(512) * 0.1).astype(F32)
    c.update(norm_x=xn, norm_w=wn)
    c["norm_y"] = hr.rms_norm(xn, wn, 1e-6)
    xr = g.standard_normal((2, 6, 2 * 128)).astype(F16)
    wr = (g.standard_normal(128) * 0.1).astype(F32)
    ang = g.random((2, 1, 6, 64)).astype(F32) * 6
    fr = np.stack([np.stack([np.cos(ang), -np.sin(ang)], -1), np.stack([np.sin(ang), np.cos(ang)], -1)], -2).astype(F32)
    c.update(rope_x=xr, rope_w=wr, rope_f=fr)
    c["rope_y"] = hr.rms_norm_rope(xr, 2, wr, 1e-6, fr)
    # Decode.
    xd = g.standard_normal(2048).astype(F32)
    c["rot_x"] = xd
    c["rot_256"], c["rot_1024"] = hr.rotate(xd, 256), hr.rotate(xd, 1024)
    wg = g.integers(-127, 128, (16, 1024), dtype=np.int8)
    sg = g.random(16).astype(F32)
    bg = g.standard_normal(16).astype(F32)
    xg = g.standard_normal(1024).astype(F32)
    c.update(gemv_x=xg, gemv_w=wg, gemv_s=sg, gemv_b=bg)
    c["gemv_y"] = hr.gemv_i8(xg, wg, sg, bg)
    bits = (g.standard_normal((16, 512)).astype(F32).view(np.uint32) >> 16).astype(np.uint16)
    xb = g.standard_normal(512).astype(F32)
    c.update(bf16_x=xb, bf16_w=bits)
    c["bf16_y"] = hr.gemv_bf16(xb, bits)
    qd = g.standard_normal((2, 1, 8, 128)).astype(F32)
    kd = g.standard_normal((2, 40, 2, 128)).astype(F32)
    vd = g.standard_normal((2, 40, 2, 128)).astype(F32)
    ld = np.array([37, 7], np.int32)
    c.update(dec_q=qd, dec_k=kd, dec_v=vd, dec_len=ld)
    c["dec_o"] = hr.attn_decode(qd, kd, vd, ld)
    np.savez_compressed(OUT, **c)
    print(OUT, os.path.getsize(OUT), "bytes,", len(c), "arrays")


if __name__ == "__main__":
    main()
