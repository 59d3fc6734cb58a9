"""Fused attention parity on the GPU (hip_attention.hip attn / attn_i8 semantics).

Tolerances (relative L2 against float64 softmax attention): fp16 QK 2e-3, int8 QK 1e-2. Against the oracle's
restatement of the kernel arithmetic (fp16 P, lazy rescale, 128-key tiles) the fp16 path agrees to 1e-3. The
int8-QK operand quantization is bit-exact.
"""
import os

import numpy as np
import pytest
import torch

from oracle import attention as oatt

pytestmark = pytest.mark.gpu

F16 = np.float16
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "attention_bmm.npz")


def dev_(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def qkv(B, H, Hkv, Lq, Lk, seed):
    g = np.random.default_rng(seed)
    return (g.standard_normal((B, H, Lq, 128)).astype(F16), g.standard_normal((B, Hkv, Lk, 128)).astype(F16),
            g.standard_normal((B, Hkv, Lk, 128)).astype(F16))


CASES = [(1, 2, 2, 200, 300), (2, 4, 2, 128, 128), (1, 1, 1, 1, 1), (1, 2, 1, 77, 1000), (1, 3, 3, 129, 257),
         (1, 8, 2, 256, 511), (2, 1, 1, 1000, 17)]


@pytest.mark.parametrize("int8_qk", [False, True])
@pytest.mark.parametrize("B,H,Hkv,Lq,Lk", CASES)
def test_attention_matches_exact(pkg, dev, B, H, Hkv, Lq, Lk, int8_qk):
    q, k, v = qkv(B, H, Hkv, Lq, Lk, Lq + Lk)
    out = torch.empty((B, H, Lq, 128), dtype=torch.float16, device=dev)
    pkg.ops.attention(dev_(q, dev), dev_(k, dev), dev_(v, dev), out, 128 ** -0.5, int8_qk=int8_qk)
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    exact = oatt.attention_exact(q, k, v, 128 ** -0.5)
    assert oatt.rel_l2(got, exact) < (1e-2 if int8_qk else 2e-3)
    if B * H * Lq * Lk <= 4e6:
        sem = oatt.attention_semantics(q, k, v, 128 ** -0.5, int8_qk=int8_qk, tile=128)
        assert oatt.rel_l2(got, sem) < (5e-3 if int8_qk else 1e-3)


def test_int8_operands_bit_exact(pkg, dev):
    B, H, Hkv, Lq, Lk = 1, 2, 1, 70, 130
    q, k, v = qkv(B, H, Hkv, Lq, Lk, 3)
    lib = pkg._lib.load()
    n = lib.b2_attention_workspace_bytes(B, H, Hkv, Lq, Lk, 1)
    ws = torch.zeros(n, dtype=torch.uint8, device=dev)
    out = torch.empty((B, H, Lq, 128), dtype=torch.float16, device=dev)
    pkg.ops.attention(dev_(q, dev), dev_(k, dev), dev_(v, dev), out, 128 ** -0.5, int8_qk=True, workspace=ws)
    w = ws.cpu().numpy()
    qq, qs = oatt.quant_rows_rint(q.reshape(-1, 128))
    kq, ks = oatt.quant_rows_rint(k.reshape(-1, 128))
    r = lambda x, m: (x + m - 1) // m * m
    k_off = r(qq.size, 1024)
    qs_off = r(k_off + kq.size, 1024)
    ks_off = r(qs_off + qs.size * 4, 1024)
    assert np.array_equal(w[:qq.size].view(np.int8).reshape(qq.shape), qq)
    assert np.array_equal(w[k_off:k_off + kq.size].view(np.int8).reshape(kq.shape), kq)
    assert np.array_equal(w[qs_off:qs_off + qs.size * 4].view(np.float32), qs)
    ks_ld = r(Lk, 4)
    got_ks = w[ks_off:ks_off + Hkv * ks_ld * 4].view(np.float32).reshape(Hkv, ks_ld)[:, :Lk].reshape(-1)
    assert np.array_equal(got_ks, ks)


@pytest.mark.parametrize("int8_qk", [False, True])
def test_strided_views_and_drop_in(pkg, dev, int8_qk):
    # attention_hip with (B, L, H*D) inputs: q/k/v are transposed views and out is a strided view.
    B, L, H = 2, 333, 3
    g = np.random.default_rng(21)
    q, k, v = (g.standard_normal((B, L, H * 128)).astype(F16) for _ in range(3))
    got = pkg.attention.attention_hip(dev_(q, dev), dev_(k, dev), dev_(v, dev), H, int8_qk=int8_qk).cpu().numpy()
    heads = lambda t: t.reshape(B, L, H, 128).transpose(0, 2, 1, 3)
    exact = oatt.attention_exact(heads(q), heads(k), heads(v), 128 ** -0.5).transpose(0, 2, 1, 3).reshape(B, L, H * 128)
    assert oatt.rel_l2(got, exact) < (1e-2 if int8_qk else 2e-3)


def test_golden_reference_outputs(pkg, dev):
    data = np.load(GOLDEN)
    for name in ("self", "cross"):
        q, k, v = (dev_(data[f"{name}_{t}"], dev) for t in "qkv")
        got = pkg.attention.attention_hip(q, k, v, q.shape[1], skip_reshape=True, skip_output_reshape=True)
        assert oatt.rel_l2(got.cpu().numpy(), data[f"{name}_out"]) < 2e-3, name
    q, k, v = (dev_(data[f"flat_{t}"], dev) for t in "qkv")
    got = pkg.attention.attention_hip(q, k, v, 2)
    assert oatt.rel_l2(got.cpu().numpy(), data["flat_out"]) < 2e-3


@pytest.mark.parametrize("int8_qk", [False, True])
def test_config2_full_size(pkg, dev, int8_qk):
    """Configuration 2: B=2, H=24, S=4056, d=128, N(0,1), scale 1/sqrt(128); checked against an fp32 torch
    computation on the device, head by head."""
    B, H, S = 2, 24, 4056
    gen = torch.Generator(device="cpu").manual_seed(2)
    q, k, v = (torch.randn((B, H, S, 128), generator=gen).half().to(dev) for _ in range(3))
    out = torch.empty_like(q)
    pkg.ops.attention(q, k, v, out, 128 ** -0.5, int8_qk=int8_qk)
    num = den = 0.0
    for b in range(B):
        for h in (0, 7, 23):
            s = (q[b, h].float() @ k[b, h].float().t()) * 128 ** -0.5
            ref = torch.softmax(s, -1) @ v[b, h].float()
            num += (out[b, h].float() - ref).pow(2).sum().item()
            den += ref.pow(2).sum().item()
    assert (num / den) ** 0.5 < (1e-2 if int8_qk else 2e-3)
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("B,H,Hkv,Lq,Lk", [(2, 12, 12, 3321, 3321), (1, 40, 8, 1300, 1000), (1, 80, 80, 600, 70)])
def test_full_grid_shapes(pkg, dev, B, H, Hkv, Lq, Lk):
    """Grids of more than one CTA per SM: the DiT's 3321-row sequences (the last CTA's second tile partly past Lq),
    grouped-query heads and a partial key tile; checked against fp32 torch on a few heads."""
    gen = torch.Generator(device="cpu").manual_seed(B * 1000 + H)
    q = torch.randn((B, H, Lq, 128), generator=gen).half().to(dev)
    k, v = (torch.randn((B, Hkv, Lk, 128), generator=gen).half().to(dev) for _ in range(2))
    out = torch.full_like(q, float("nan"))
    pkg.ops.attention(q, k, v, out, 128 ** -0.5)
    assert torch.isfinite(out).all()
    num = den = 0.0
    rep = H // Hkv
    for b in range(B):
        for h in sorted({0, H // 2, H - 1}):
            s = (q[b, h].float() @ k[b, h // rep].float().t()) * 128 ** -0.5
            ref = torch.softmax(s, -1) @ v[b, h // rep].float()
            num += (out[b, h].float() - ref).pow(2).sum().item()
            den += ref.pow(2).sum().item()
    assert (num / den) ** 0.5 < 2e-3
