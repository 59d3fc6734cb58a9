"""The Krea-2 fused block, int8_gemm.block_forward (reference int8_gemm.py:189-226), on the GPU.

A duck-typed SingleStreamBlock at Krea-2 widths (hidden 3072, heads of 128, MLP 8192, ConvRot-256 W8A8 linears as the
Int8 loader's Linear calls them) runs through block_forward with real modulation vectors and QK-norm + rope. Every
hand-off inside the block is recorded and checked from the GPU's own input to that stage:

  quantize_block_input (x2)   modulated RMSNorm + ConvRot + int8, shared by the block's input linears: activation
                              within two fp16 steps of the oracle's modulate; int8 and scales bit-exact from it
  wq/wk/wv/gate, mlp gate/up  GEMMs on the shared activations: bit-exact
  rms_norm_rope (q and k)     within three fp16 steps of the larger normalised value of each rotated pair,
                              on < 5e-3 of the values
  attention                   relative L2 within 1e-3 (fp16 QK) / 1e-2 (int8 QK) of the kernel-semantics oracle
  wo                          sigmoid-gate pre-pass (activation within two steps, int8 bit-exact from it), then the
                              GEMM with the gated residual x + pregate * y: bit-exact
  down                        SwiGLU pre-pass (same rule), then the GEMM with x + postgate * y: bit-exact

and the block's output against an oracle chain that starts from x alone (relative L2 within 1e-2 / 2e-2).
"""
import types

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import gemm as ogemm
from oracle import norm as onorm
from oracle import quant as oq
from oracle import weights as ow

pytestmark = pytest.mark.gpu

F16 = np.float16
F32 = np.float32
D, F, HD = 3072, 8192, 128


def cpu(t):
    return t.detach().cpu().numpy()


def within_two_steps(got, ref, what, rate_max, mag=None):
    diff = np.abs(got.astype(F32) - ref.astype(F32))
    mag = np.abs(ref.astype(F32)) if mag is None else mag
    ulp = np.abs(np.spacing(mag.astype(F16))).astype(F32)
    assert np.all(diff <= 2 * ulp), f"{what}: off by {np.max(diff / ulp)} fp16 steps"
    rate = np.mean(got != ref)
    assert rate < rate_max, f"{what}: {rate:.2e} of the values differ"


class Linear:
    """What the Int8 loader's ConvRot Linear does in forward: the rotation hand-off, then the patched
    triton_int8_linear. It records its output and the side channels it was called with."""

    def __init__(self, gm, name, n, k, rng, dev, log):
        w = (rng.standard_normal((n, k)) * 0.02).astype(F32)
        self.wq, self.ws = ow.quantize_per_channel(ow.convrot_rotate(w))
        self.w_d, self.s_d = torch.from_numpy(self.wq).to(dev), torch.from_numpy(self.ws).to(dev)
        self.gm, self.name, self.log = gm, name, log
        self.in_features, self.bias = k, None
        self._is_quantized = self._use_convrot = True
        self._convrot_groupsize, self._is_w4a8, self.lora_patches = 256, False, None
        self.int8_linear = gm.wrap(None)

    def __call__(self, x):
        gm = self.gm
        seen = {"x": x, "shared": gm.shared, "sigmoid_gate": gm.sigmoid_gate, "swiglu_up": gm.swiglu_up,
                "residual": gm.residual}
        y = self.int8_linear(gm.rotate_activation(x, None, 256), self.w_d, self.s_d)
        seen["y"] = y
        self.log[self.name] = seen
        return y


def rope_freqs(B, L, rng):
    pos = np.arange(L, dtype=np.float64)[:, None]
    inv = 10000.0 ** (-np.arange(64, dtype=np.float64) / 64)
    ang = (pos * inv)[None, None] + rng.random((B, 1, 1, 64)) * 0.1
    c, s = np.cos(ang), np.sin(ang)
    return np.stack([np.stack([c, -s], -1), np.stack([s, c], -1)], -2).astype(F32)  # (B, 1, L, 64, 2, 2)


@pytest.mark.parametrize("int8_qk,heads,kvheads", [(False, 24, 24), (True, 24, 8)])
def test_krea2_block_forward(pkg, dev, monkeypatch, int8_qk, heads, kvheads):
    gm = pkg.int8_gemm
    B, L = 2, 512
    rng = np.random.default_rng(31 + kvheads)
    log = {}
    mk = lambda name, n, k: Linear(gm, name, n, k, rng, dev, log)  # noqa: E731
    nrm = lambda d: types.SimpleNamespace(scale=torch.from_numpy((rng.standard_normal(d) * 0.1).astype(F32)).to(dev),  # noqa: E731
                                          eps=1e-6)
    qk = types.SimpleNamespace(qnorm=nrm(HD), knorm=nrm(HD))
    attn = types.SimpleNamespace(wq=mk("wq", heads * HD, D), wk=mk("wk", kvheads * HD, D), wv=mk("wv", kvheads * HD, D),
                                 gate=mk("gate", D, D), wo=mk("wo", D, D), heads=heads, kvheads=kvheads, headdim=HD,
                                 qknorm=qk)
    mlp = types.SimpleNamespace(gate=mk("mlp_gate", F, D), up=mk("mlp_up", F, D), down=mk("down", D, F))
    # prescale, preshift, pregate, postscale, postshift, postgate: (B, 1, D) fp16 from the timestep vector
    spread = [0.1, 0.1, 0.5, 0.1, 0.1, 0.5]
    mods_np = [(rng.standard_normal((B, 1, D)) * s).astype(F16) for s in spread]
    mods = [torch.from_numpy(m).to(dev) for m in mods_np]
    module = types.SimpleNamespace(attn=attn, mlp=mlp, mod=lambda vec: mods, prenorm=nrm(D), postnorm=nrm(D))
    freqs_np = rope_freqs(B, L, rng)
    x_np = rng.standard_normal((B, L, D)).astype(F16)
    x = torch.from_numpy(x_np).to(dev)

    ropes, atts = [], []
    real_rope, real_att = pkg.rms_norm.rms_norm_rope, pkg.hip_attention.attention

    def rec_rope(t, h, m, f):
        out = real_rope(t, h, m, f)
        ropes.append((t, out))
        return out

    def rec_att(q, k, v, out, scale, i8=False):
        res = real_att(q, k, v, out, scale, i8)
        atts.append((q, k, v, out))
        return res

    monkeypatch.setattr(pkg.rms_norm, "rms_norm_rope", rec_rope)
    monkeypatch.setattr(pkg.hip_attention, "attention", rec_att)
    out = gm.block_forward(module, int8_qk, x, None, torch.from_numpy(freqs_np).to(dev))
    torch.cuda.synchronize()
    assert gm.shared is None and gm.swiglu_up is None and gm.sigmoid_gate is None and gm.residual is None
    M = B * L
    ops = pkg.ops

    def check_shared(x_in, norm, scale, shift, shared, what):
        s_rows = (1 + scale).to(torch.float16).reshape(B, D).contiguous()
        t_rows = shift.reshape(B, D).contiguous()
        act = torch.empty((M, D), dtype=torch.float16, device=dev)
        q8, sa = ops.mod_quant_pack_a(x_in.reshape(M, D), norm.scale.float(), s_rows, t_rows, L, norm.eps, 256,
                                      act_out=act)
        assert torch.equal(q8, shared[0]) and torch.equal(sa, shared[1]), f"{what}: not the block's activations"
        ref = oq.modulate(cpu(x_in).reshape(M, D), cpu(norm.scale), cpu(s_rows), cpu(t_rows), L, norm.eps)
        mag = np.abs(ref.astype(F32)) + np.abs(np.repeat(cpu(t_rows), L, axis=0).astype(F32))
        a = cpu(act)
        within_two_steps(a, ref, what, 5e-3, mag=mag)
        q_ref, s_ref = oq.quant_rows(oq.rotate_rows(a, 256))
        assert np.array_equal(q_ref, cpu(q8)) and np.array_equal(s_ref, cpu(sa)), f"{what}: int8 from the activation"
        return cpu(q8), cpu(sa)

    def gemm_ref(lin, q8, sa, res=None):
        R, G = (None, None) if res is None else (cpu(res[0]).reshape(M, -1), cpu(res[1]).reshape(B, -1))
        return ogemm.epilogue(ogemm.int_mm(q8, lin.wq), sa, lin.ws, R=R, G=G, L=L if res is not None else 1)

    # The block's input linears read one shared quantization of the modulated norm.
    q8, sa = check_shared(x, module.prenorm, mods[0], mods[1], log["wq"]["shared"], "pre-norm")
    for name, lin in (("wq", attn.wq), ("wk", attn.wk), ("wv", attn.wv), ("gate", attn.gate)):
        assert log[name]["shared"] is log["wq"]["shared"]
        assert np.array_equal(cpu(log[name]["y"]).reshape(M, -1), gemm_ref(lin, q8, sa)), name

    # QK-norm + rope on the wq / wk outputs.
    (q_in, q_rope), (k_in, k_rope) = ropes
    assert q_in is log["wq"]["y"] and k_in is log["wk"]["y"]
    for got, src, n, norm, what in ((q_rope, q_in, heads, qk.qnorm, "q"), (k_rope, k_in, kvheads, qk.knorm, "k")):
        ref = onorm.rms_norm_rope(cpu(src), n, cpu(norm.scale), norm.eps, freqs_np)
        # The normalised value may be a step off (rstd differs by an ulp); the rotation mixes the two values of a
        # pair and can cancel most of them, so steps are measured at the larger normalised value of the pair: at
        # most one step from each input and one from the final rounding.
        y = onorm.rms_norm(cpu(src).reshape(B, L, n, HD).transpose(0, 2, 1, 3), cpu(norm.scale), norm.eps)
        pair = np.maximum(np.abs(y[..., 0::2]), np.abs(y[..., 1::2])).astype(F32)
        mag = np.repeat(pair, 2, axis=-1)
        diff = np.abs(cpu(got).astype(F32) - ref.astype(F32))
        ulp = np.abs(np.spacing(mag.astype(F16))).astype(F32)
        assert np.all(diff <= 3 * ulp), f"rms_norm_rope {what}: off by {np.max(diff / ulp)} steps of the pair"
        assert np.mean(cpu(got) != ref) < 5e-3, f"rms_norm_rope {what}"

    # Attention on the GPU's own q, k, v.
    (qa, ka, va, oa), = atts
    assert qa is q_rope and ka is k_rope
    att = cpu(oa)
    sem = oatt.attention_semantics(cpu(qa), cpu(ka), cpu(va), HD ** -0.5, int8_qk=int8_qk, tile=128)
    assert oatt.rel_l2(att, sem) < (1e-2 if int8_qk else 1e-3)

    # wo: sigmoid gate in the pre-pass, gated residual x + pregate * y in the epilogue.
    rec = log["wo"]
    assert rec["sigmoid_gate"] is not None and rec["residual"][0] is x
    att_rows = oa.transpose(1, 2).reshape(M, D)
    gate_rows = log["gate"]["y"].reshape(M, D)
    assert torch.equal(rec["x"].reshape(M, D), att_rows)
    act = torch.empty((M, D), dtype=torch.float16, device=dev)
    q8, sa = ops.gate_quant_pack_a(att_rows.contiguous(), gate_rows.contiguous(), 256, act_out=act)
    within_two_steps(cpu(act), oq.sigmoid_gate(cpu(att_rows), cpu(gate_rows)), "sigmoid gate", 5e-3)
    q_ref, s_ref = oq.quant_rows(oq.rotate_rows(cpu(act), 256))
    assert np.array_equal(q_ref, cpu(q8)) and np.array_equal(s_ref, cpu(sa))
    x1 = rec["y"]
    assert np.array_equal(cpu(x1).reshape(M, D), gemm_ref(attn.wo, cpu(q8), cpu(sa), rec["residual"])), "wo"

    # MLP: second shared quantization, gate / up, SwiGLU in the down pre-pass, gated residual x1 + postgate * y.
    q8, sa = check_shared(x1, module.postnorm, mods[3], mods[4], log["mlp_gate"]["shared"], "post-norm")
    for name, lin in (("mlp_gate", mlp.gate), ("mlp_up", mlp.up)):
        assert np.array_equal(cpu(log[name]["y"]).reshape(M, -1), gemm_ref(lin, q8, sa)), name
    rec = log["down"]
    g_y, u_y = log["mlp_gate"]["y"].reshape(M, F), log["mlp_up"]["y"].reshape(M, F)
    assert rec["swiglu_up"] is log["mlp_up"]["y"] and rec["residual"][0] is x1
    act = torch.empty((M, F), dtype=torch.float16, device=dev)
    q8, sa = ops.swiglu_quant_pack_a(g_y.contiguous(), u_y.contiguous(), 256, act_out=act)
    within_two_steps(cpu(act), oq.swiglu(cpu(g_y), cpu(u_y)), "swiglu", 5e-3)
    q_ref, s_ref = oq.quant_rows(oq.rotate_rows(cpu(act), 256))
    assert np.array_equal(q_ref, cpu(q8)) and np.array_equal(s_ref, cpu(sa))
    assert np.array_equal(cpu(out).reshape(M, D), gemm_ref(mlp.down, cpu(q8), cpu(sa), rec["residual"])), "down"

    # The whole block against an oracle chain from x alone.
    def chain_shared(xin, norm, scale, shift):
        s = (F16(1) + scale.reshape(B, D)).astype(F16)
        h = oq.modulate(xin.reshape(M, D), cpu(norm.scale), s, shift.reshape(B, D), L, norm.eps)
        return oq.quant_rows(oq.rotate_rows(h, 256))

    q8, sa = chain_shared(x_np, module.prenorm, mods_np[0], mods_np[1])
    yq, yk, yv, yg = (gemm_ref(lin, q8, sa) for lin in (attn.wq, attn.wk, attn.wv, attn.gate))
    qh = onorm.rms_norm_rope(yq.reshape(B, L, -1), heads, cpu(qk.qnorm.scale), 1e-6, freqs_np)
    kh = onorm.rms_norm_rope(yk.reshape(B, L, -1), kvheads, cpu(qk.knorm.scale), 1e-6, freqs_np)
    vh = yv.reshape(B, L, kvheads, HD).transpose(0, 2, 1, 3)
    o = oatt.attention_semantics(qh, kh, vh, HD ** -0.5, int8_qk=int8_qk, tile=128).transpose(0, 2, 1, 3).reshape(M, D)
    qa8, sa8 = oq.quant_rows(oq.rotate_rows(oq.sigmoid_gate(o, yg), 256))
    x1r = ogemm.epilogue(ogemm.int_mm(qa8, attn.wo.wq), sa8, attn.wo.ws, R=x_np.reshape(M, D),
                         G=mods_np[2].reshape(B, D), L=L)
    q8, sa = chain_shared(x1r, module.postnorm, mods_np[3], mods_np[4])
    gy, uy = gemm_ref(mlp.gate, q8, sa), gemm_ref(mlp.up, q8, sa)
    qd, sd = oq.quant_rows(oq.rotate_rows(oq.swiglu(gy, uy), 256))
    ref = ogemm.epilogue(ogemm.int_mm(qd, mlp.down.wq), sd, mlp.down.ws, R=x1r, G=mods_np[5].reshape(B, D), L=L)
    # The chain re-quantizes activations that differ from the GPU's by fp16 steps (exp, rsqrt and attention
    # rounding), so some int8 values round the other way downstream; every stage above is exact from its own input.
    assert oatt.rel_l2(cpu(out).reshape(M, D), ref) < (2e-2 if int8_qk else 1e-2)
    assert pkg._lib.device_status() == 0
