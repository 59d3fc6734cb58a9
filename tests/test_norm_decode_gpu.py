"""RMSNorm (+rope) and single-token decode parity on the GPU.

RMSNorm: within two fp16 steps of the oracle (the fp32 sum order and rsqrt differ from the reference's), with at
most 2e-3 of the values off. Decode: rotate bit-exact; GEMV and decode attention within 1e-5 relative L2 of float64.
"""
import types

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import decode as odec
from oracle import norm as onorm

pytestmark = pytest.mark.gpu

F16 = np.float16
F32 = np.float32


def dev_(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def close_fp16(got, ref):
    # rstd differs by an ulp (sum order, rsqrt); through the fp16 rounding(s) that is at most two fp16 steps.
    got = np.asarray(got)
    diff = np.abs(got.astype(F32) - ref.astype(F32))
    assert np.all(diff <= 2 * np.abs(np.spacing(ref.astype(F16))).astype(F32)), diff.max()
    assert np.mean(got != ref) < 2e-3


@pytest.mark.parametrize("shape", [(2, 77, 3072), (1, 5, 128), (1, 300, 64), (2, 13, 8192), (1, 9, 1000)])
def test_rms_norm_rows(pkg, dev, shape):
    if shape[-1] % 8:
        pytest.skip()
    g = np.random.default_rng(shape[-1])
    x = (g.standard_normal(shape) * 3).astype(F16)
    w = (g.standard_normal(shape[-1]) * 0.1).astype(F32)
    got = pkg.rms_norm.rms_norm(dev_(x, dev), dev_(w, dev), 1e-6).cpu().numpy()
    close_fp16(got, onorm.rms_norm(x, w, 1e-6))


def test_rms_norm_strided_heads(pkg, dev):
    # (B, H, L, D) view of a (B, L, H*D) tensor: rows are read head-first, output is contiguous (B, H, L, D).
    B, L, H = 2, 50, 6
    g = np.random.default_rng(1)
    x = g.standard_normal((B, L, H * 128)).astype(F16)
    w = (g.standard_normal(128) * 0.1).astype(F32)
    xv = dev_(x, dev).view(B, L, H, 128).transpose(1, 2)
    got = pkg.rms_norm.rms_norm(xv, dev_(w, dev), 1e-6)
    assert got.is_contiguous() and got.shape == (B, H, L, 128)
    close_fp16(got.cpu().numpy(), onorm.rms_norm(x.reshape(B, L, H, 128).transpose(0, 2, 1, 3), w, 1e-6))


@pytest.mark.parametrize("batched_freqs", [False, True])
def test_rms_norm_rope(pkg, dev, batched_freqs):
    B, L, H = 2, 40, 4
    g = np.random.default_rng(2)
    x = g.standard_normal((B, L, H * 128)).astype(F16)
    w = (g.standard_normal(128) * 0.1).astype(F32)
    ang = g.random((B if batched_freqs else 1, 1, L, 64)).astype(F32) * 6
    f = np.stack([np.stack([np.cos(ang), -np.sin(ang)], -1), np.stack([np.sin(ang), np.cos(ang)], -1)], -2).astype(F32)
    module = type("RMSNorm", (), {})()
    module.scale, module.eps = torch.from_numpy(w), 1e-6
    got = pkg.rms_norm.rms_norm_rope(dev_(x, dev), H, module, dev_(f, dev)).cpu().numpy()
    close_fp16(got, onorm.rms_norm_rope(x, H, w, 1e-6, f))


@pytest.mark.parametrize("group", [4, 256, 1024, 16384])
def test_rotate_bit_exact(pkg, dev, group):
    x = np.random.default_rng(group).standard_normal(max(group, 2560 if group <= 256 else group) * 2).astype(F32)
    x = x[: (x.size // group) * group]
    got = pkg.int8_gemv.rotate(dev_(x, dev), group).cpu().numpy()
    assert np.array_equal(got, odec.rotate(x, group))


C5_LINEARS = [(4096, 2560), (1024, 2560), (2560, 4096), (9728, 2560), (2560, 9728), (16, 512), (24, 80)]


@pytest.mark.parametrize("N,K", C5_LINEARS)
def test_gemv_i8(pkg, dev, N, K):
    g = np.random.default_rng(N + K)
    x = g.standard_normal(K).astype(F32)
    w = g.integers(-127, 128, (N, K), dtype=np.int8)
    s = (g.random(N) * 1e-3).astype(F32)
    b = g.standard_normal(N).astype(F32)
    for bias in (None, b):
        got = pkg.ops.gemv_i8(dev_(x, dev), dev_(w, dev), dev_(s, dev), None if bias is None else dev_(bias, dev))
        ref = odec.gemv_i8(x, w, s, bias)
        assert oatt.rel_l2(got.cpu().numpy(), ref) < 1e-5


@pytest.mark.parametrize("N,K", [(151936, 256), (4096, 2560), (16, 256), (37, 264), (5, 8), (1000, 1288)])
def test_gemv_bf16(pkg, dev, N, K):
    """The logits GEMV on a bf16 table, including ragged K (a partial last 256-value step) and N off the 16-row CTA."""
    g = np.random.default_rng(N * 7 + K)
    x = g.standard_normal(K).astype(F32)
    wt = torch.from_numpy((g.standard_normal((N, K)) * 0.05).astype(F32)).to(torch.bfloat16)
    got = pkg.ops.gemv_bf16(dev_(x, dev), wt.to(dev)).cpu().numpy()
    ref = odec.gemv_bf16(x, wt.view(torch.int16).numpy().view(np.uint16))
    assert oatt.rel_l2(got, ref) < 1e-5


def test_logits_drop_in(pkg, dev):
    """int8_gemv.logits: the last position of one fp32 sequence against the tied bf16 table, shape (1, 1, vocab)."""
    N, K = 4096, 2560
    g = np.random.default_rng(5)
    table = torch.from_numpy((g.standard_normal((N, K)) * 0.05).astype(F32)).to(torch.bfloat16)
    x = g.standard_normal((1, 7, K)).astype(F32)
    embed = types.SimpleNamespace(weight=table.to(dev), weight_function=[], bias_function=[])
    transformer = types.SimpleNamespace(model=types.SimpleNamespace(embed_tokens=embed))
    got = pkg.int8_gemv.logits(transformer, dev_(x, dev))
    assert got.shape == (1, 1, N) and got.dtype == torch.float32
    ref = odec.gemv_bf16(x[0, -1], table.view(torch.int16).numpy().view(np.uint16))
    assert oatt.rel_l2(got.cpu().numpy().reshape(-1), ref) < 1e-5


def _int8_linear(w, s, dev):
    weight = types.SimpleNamespace(_qdata=dev_(w, dev), _params=types.SimpleNamespace(scale=dev_(s, dev)))
    return types.SimpleNamespace(weight=weight, bias=None, weight_function=[], bias_function=[])


def test_prefill_paths_while_generating(pkg, dev):
    """While generating: a multi-token fp32 input of a linear with a ConvRot group above 256 is rotated by the kernel
    and multiplied by the dequantized weight (int8_gemv.py:49-57); a gated MLP runs one stacked gate|up linear
    (:67-75). Both against float64 restatements."""
    gv = pkg.int8_gemv
    g = np.random.default_rng(6)
    T, K, N, F_ = 5, 1024, 256, 512
    w = g.integers(-127, 128, (N, K), dtype=np.int8)
    s = (g.random(N) * 1e-3).astype(F32)
    x = g.standard_normal((1, T, K)).astype(F32)
    lin = _int8_linear(w, s, dev)
    wg = g.integers(-127, 128, (F_, K), dtype=np.int8)
    wu = g.integers(-127, 128, (F_, K), dtype=np.int8)
    sg, su = (g.random(F_) * 1e-3).astype(F32), (g.random(F_) * 1e-3).astype(F32)
    down_seen = []
    mlp = types.SimpleNamespace(gate_proj=_int8_linear(wg, sg, dev), up_proj=_int8_linear(wu, su, dev),
                                activation=torch.nn.functional.silu, down_proj=lambda h: down_seen.append(h) or h)
    gv.generating = True
    try:
        got = gv.linear_forward(lin, N, K, torch.int8, 1024, dev_(x, dev)).cpu().numpy()
        got_mlp = gv.mlp_forward(mlp, torch.int8, dev_(x, dev)).cpu().numpy()
    finally:
        gv.generating = False
    xr = odec.rotate(x.reshape(-1), 1024).reshape(T, K).astype(np.float64)
    ref = xr @ (w.astype(np.float64) * s[:, None]).T
    assert got.shape == (1, T, N) and oatt.rel_l2(got.reshape(T, N), ref) < 1e-5
    x64 = x.reshape(T, K).astype(np.float64)
    gate = x64 @ (wg.astype(np.float64) * sg[:, None]).T
    up = x64 @ (wu.astype(np.float64) * su[:, None]).T
    ref_h = gate / (1 + np.exp(-gate)) * up
    assert len(down_seen) == 1 and oatt.rel_l2(got_mlp.reshape(T, F_), ref_h) < 1e-5


def test_linear_forward_drop_in(pkg, dev):
    N, K = 1024, 2560
    g = np.random.default_rng(3)
    w = g.integers(-127, 128, (N, K), dtype=np.int8)
    s = (g.random(N) * 1e-3).astype(F32)
    x = g.standard_normal((1, 1, K)).astype(F32)
    weight = type("W", (), {})()
    weight._qdata = dev_(w, dev)
    weight._params = type("P", (), {"scale": dev_(s, dev)})()
    module = type("Linear", (), {"weight": weight, "bias": None, "weight_function": [], "bias_function": []})()
    got = pkg.int8_gemv.linear_forward(module, N, K, torch.int8, 256, dev_(x, dev)).cpu().numpy()
    ref = odec.linear_fallback(odec.rotate(x.reshape(-1), 256), w, s)
    assert got.shape == (1, 1, N)
    assert oatt.rel_l2(got.reshape(-1), ref) < 1e-5


@pytest.mark.parametrize("B,H,Hkv,cap,lengths", [(1, 32, 8, 1024, [1024]), (2, 32, 8, 1024, [17, 700]), (1, 8, 8, 64, [1]),
                                                 (3, 16, 4, 300, [299, 64, 33])])
def test_attn_decode(pkg, dev, B, H, Hkv, cap, lengths):
    g = np.random.default_rng(cap + B)
    q = g.standard_normal((B, 1, H, 128)).astype(F32)
    k = g.standard_normal((B, cap, Hkv, 128)).astype(F32)
    v = g.standard_normal((B, cap, Hkv, 128)).astype(F32)
    ln = np.array(lengths, np.int32)
    got = pkg.int8_gemv.attention_decode(dev_(q, dev), dev_(k, dev), dev_(v, dev), dev_(ln, dev)).cpu().numpy()
    ref = odec.attn_decode(q, k, v, ln, 128 ** -0.5)
    assert oatt.rel_l2(got, ref) < 1e-5


def test_decoder_fused_step_matches_torch_ops(pkg, dev):
    """The configuration-5 decode step on the fused kernels (9 launches per layer) against the same layer written
    with torch element-wise ops: two consecutive tokens, hidden state and KV caches."""
    import importlib

    decoder = importlib.import_module(pkg.__name__ + ".decoder")
    cfg = decoder.DecoderConfig(hidden=512, layers=3, heads=8, kv_heads=2, head_dim=128, mlp=1024, capacity=64)
    fused, ref = decoder.TextDecoder(cfg, dev, seed=1), decoder.TextDecoder(cfg, dev, seed=1)
    fused.mode = "layers"  # the persistent mode has its own tests (test_decode_step_gpu.py)
    ref.fused = False
    x0 = torch.randn((1, cfg.hidden), generator=torch.Generator(device=dev).manual_seed(5), device=dev)
    for dec in (fused, ref):
        dec.x.copy_(x0)
    for pos in (37, 38):
        for dec in (fused, ref):
            dec.set_position(pos)
            dec.step_eager()
        rel = ((fused.x - ref.x).norm() / ref.x.norm()).item()
        assert rel < 2e-5, (pos, rel)
    for lf, lr in zip(fused.layers, ref.layers):
        assert torch.allclose(lf.k_cache, lr.k_cache, rtol=1e-5, atol=1e-6)
        assert torch.equal(lf.v_cache, lr.v_cache) or torch.allclose(lf.v_cache, lr.v_cache, rtol=1e-5, atol=1e-6)


def test_decoder_graph_replay_matches_eager(pkg, dev):
    """A captured decode step replayed from its CUDA graph (position and cache length read on the device) gives the
    eager step's hidden state and caches bit for bit, token after token."""
    import importlib

    decoder = importlib.import_module(pkg.__name__ + ".decoder")
    cfg = decoder.DecoderConfig(hidden=512, layers=3, heads=8, kv_heads=2, head_dim=128, mlp=1024, capacity=64)
    eager, graphed = decoder.TextDecoder(cfg, dev, seed=2), decoder.TextDecoder(cfg, dev, seed=2)
    x0 = torch.randn((1, cfg.hidden), generator=torch.Generator(device=dev).manual_seed(6), device=dev)
    for dec in (eager, graphed):
        dec.mode = "layers"
        dec.x.copy_(x0)
        dec.set_position(20)
    eager.step_eager()
    graphed.capture()  # runs the step once (position 20) before recording it
    for pos in (21, 22):
        eager.set_position(pos)
        eager.step_eager()
        graphed.set_position(pos)
        graphed.step()
    torch.cuda.synchronize()
    assert torch.equal(eager.x, graphed.x)
    for le, lg in zip(eager.layers, graphed.layers):
        assert torch.equal(le.k_cache, lg.k_cache) and torch.equal(le.v_cache, lg.v_cache)
