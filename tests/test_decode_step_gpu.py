"""The whole-token persistent decode kernel (b2_decode_step, the decoder's default mode) on the GPU.

Checked against the float64 oracle (oracle.decode.decoder_step: the same layer route with every GEMV, norm, rope and
softmax in float64), against the decoder's 9-launches-per-layer mode, and against the torch-op layer; for 1, 2 and
4 query heads per kv head, several positions, and the configuration-5 shape. A captured step replays bit for bit.
The error paths end without touching the GPU's state: a flag already set, a position outside the cache, and waits
given a limit too short to be met all return with the flag set and leave the context usable.
"""
import importlib

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import decode as odec

pytestmark = pytest.mark.gpu


def _decoder(pkg):
    return importlib.import_module(pkg.__name__ + ".decoder")


def _oracle_layers(dec):
    ops = importlib.import_module(type(dec).__module__.rsplit(".", 1)[0] + ".ops")
    return [{n: getattr(L, n).detach().cpu().numpy().copy() for n in ops.DECODE_STEP_FIELDS} for L in dec.layers]


@pytest.mark.parametrize("heads,kv_heads", [(8, 2), (4, 2), (2, 2)])
def test_persistent_step_matches_float64_oracle(pkg, dev, heads, kv_heads):
    decoder = _decoder(pkg)
    cfg = decoder.DecoderConfig(hidden=512, layers=3, heads=heads, kv_heads=kv_heads, head_dim=128, mlp=1024,
                                capacity=64)
    dec = decoder.TextDecoder(cfg, dev, seed=1)
    x0 = torch.randn((1, cfg.hidden), generator=torch.Generator(device=dev).manual_seed(5), device=dev)
    dec.x.copy_(x0)
    layers = _oracle_layers(dec)
    x = x0.cpu().numpy()
    for pos in (0, 37, 38, 63):
        dec.set_position(pos)
        dec.step_eager()
        x = odec.decoder_step(x, layers, pos, pos + 1, heads, kv_heads, cfg.mlp, cfg.eps, dec.inv_freq.cpu().numpy())
        got = dec.x.cpu().numpy().reshape(-1)
        assert dec.failed() == 0
        assert oatt.rel_l2(got, x) < 2e-5, (pos, oatt.rel_l2(got, x))
        x = got.reshape(1, -1)  # continue from the GPU's state so that the comparison stays per token
    for L, ref in zip(dec.layers, layers):
        assert oatt.rel_l2(L.k_cache.cpu().numpy(), ref["k_cache"]) < 1e-5
        assert oatt.rel_l2(L.v_cache.cpu().numpy(), ref["v_cache"]) < 1e-5


def test_persistent_step_matches_layers_and_torch_modes(pkg, dev):
    decoder = _decoder(pkg)
    cfg = decoder.DecoderConfig(hidden=512, layers=3, heads=8, kv_heads=2, head_dim=128, mlp=1024, capacity=64)
    decs = [decoder.TextDecoder(cfg, dev, seed=1) for _ in range(3)]
    decs[1].mode = "layers"
    decs[2].fused = False
    x0 = torch.randn((1, cfg.hidden), generator=torch.Generator(device=dev).manual_seed(5), device=dev)
    for d in decs:
        d.x.copy_(x0)
    for pos in (37, 38):
        for d in decs:
            d.set_position(pos)
            d.step_eager()
        for other in decs[1:]:
            rel = ((decs[0].x - other.x).norm() / other.x.norm()).item()
            assert rel < 2e-5, (pos, rel)
    # The caches' new rows come from the q|k|v GEMV, whose sums the persistent kernel forms exactly over a 3-digit
    # int8 form of the input (error below 2^-20 of the input's largest value) and the other modes in fp32.
    for a, b in zip(decs[0].layers, decs[2].layers):
        for ca, cb in ((a.k_cache[0, 37:39], b.k_cache[0, 37:39]), (a.v_cache[0, 37:39], b.v_cache[0, 37:39])):
            rel = ((ca - cb).norm() / cb.norm()).item()
            worst = ((ca - cb).abs().max() / cb.abs().max()).item()
            assert rel < 1e-5 and worst < 1e-4, (rel, worst)
        assert torch.equal(a.k_cache[0, :37], b.k_cache[0, :37]) and torch.equal(a.v_cache[0, 39:], b.v_cache[0, 39:])


def test_persistent_step_configuration5_shape(pkg, dev):
    """Hidden 2560, 32/8 heads, MLP 9728, capacity 1024 (4 of the 36 layers), last position: against the
    9-launch mode token by token, and the caches' new rows against it."""
    decoder = _decoder(pkg)
    cfg = decoder.DecoderConfig(layers=4)
    a, b = decoder.TextDecoder(cfg, dev, seed=3), decoder.TextDecoder(cfg, dev, seed=3)
    b.mode = "layers"
    x0 = torch.randn((1, cfg.hidden), generator=torch.Generator(device=dev).manual_seed(8), device=dev)
    for d in (a, b):
        d.x.copy_(x0)
    for pos in (cfg.capacity - 2, cfg.capacity - 1):
        for d in (a, b):
            d.set_position(pos)
            d.step_eager()
        rel = ((a.x - b.x).norm() / b.x.norm()).item()
        assert rel < 2e-5, (pos, rel)
    assert a.failed() == 0
    rows = slice(cfg.capacity - 2, cfg.capacity)
    for la, lb in zip(a.layers, b.layers):
        for ca, cb in ((la.k_cache[0, rows], lb.k_cache[0, rows]), (la.v_cache[0, rows], lb.v_cache[0, rows])):
            rel = ((ca - cb).norm() / cb.norm()).item()
            worst = ((ca - cb).abs().max() / cb.abs().max()).item()
            assert rel < 1e-5 and worst < 1e-4, (rel, worst)


def test_persistent_graph_replay_matches_eager(pkg, dev):
    decoder = _decoder(pkg)
    cfg = decoder.DecoderConfig(hidden=512, layers=3, heads=8, kv_heads=2, head_dim=128, mlp=1024, capacity=64)
    eager, graphed = decoder.TextDecoder(cfg, dev, seed=2), decoder.TextDecoder(cfg, dev, seed=2)
    x0 = torch.randn((1, cfg.hidden), generator=torch.Generator(device=dev).manual_seed(6), device=dev)
    for d in (eager, graphed):
        d.x.copy_(x0)
        d.set_position(20)
    eager.step_eager()
    graphed.capture()
    for pos in (21, 22):
        eager.set_position(pos)
        eager.step_eager()
        graphed.set_position(pos)
        graphed.step()
    torch.cuda.synchronize()
    assert torch.equal(eager.x, graphed.x)
    for le, lg in zip(eager.layers, graphed.layers):
        assert torch.equal(le.k_cache, lg.k_cache) and torch.equal(le.v_cache, lg.v_cache)


def test_persistent_step_is_deterministic(pkg, dev):
    decoder = _decoder(pkg)
    cfg = decoder.DecoderConfig(hidden=1024, layers=2, heads=8, kv_heads=2, head_dim=128, mlp=2048, capacity=128)
    outs = []
    for _ in range(2):
        d = decoder.TextDecoder(cfg, dev, seed=4)
        d.x.copy_(torch.randn((1, cfg.hidden), generator=torch.Generator(device=dev).manual_seed(1), device=dev))
        d.set_position(100)
        d.step_eager()
        outs.append(d.x.clone())
    assert torch.equal(outs[0], outs[1])


def test_persistent_step_error_paths_leave_the_gpu_usable(pkg, dev):
    decoder = _decoder(pkg)
    cfg = decoder.DecoderConfig(hidden=512, layers=2, heads=8, kv_heads=2, head_dim=128, mlp=1024, capacity=64)
    d = decoder.TextDecoder(cfg, dev, seed=7)
    x0 = torch.randn((1, cfg.hidden), generator=torch.Generator(device=dev).manual_seed(2), device=dev)
    d.x.copy_(x0)
    # A position outside the cache: nothing is written, the flag says why.
    d.set_position(cfg.capacity)
    d.step_eager()
    assert d.failed() == 4 and torch.equal(d.x, x0)
    # A flag already set: the launch does nothing.
    d.set_position(5)
    d.step_eager()
    assert d.failed() == 4 and torch.equal(d.x, x0)
    # Waits whose limit cannot be met: every CTA gives up, drains its copies and returns.
    d.err.zero_()
    cfgs = (d.table, d.x.view(-1), d.xb, d.qkv, d.att.view(-1), d.act, d.partial, d.stats, d.inv_freq, d.pos,
            d.lengths, d.sync, d.err, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.mlp, cfg.capacity, cfg.eps)
    pkg.ops.decode_step(*cfgs, timeout_ns=1)
    torch.cuda.synchronize()
    assert d.failed() in (1, 2, 3)
    # The context still works: a normal step afterwards gives the right answer.
    d.err.zero_()
    d.x.copy_(x0)
    ref = decoder.TextDecoder(cfg, dev, seed=7)
    ref.mode = "layers"
    ref.x.copy_(x0)
    for dd in (d, ref):
        dd.set_position(5)
        dd.step_eager()
    assert d.failed() == 0
    assert ((d.x - ref.x).norm() / ref.x.norm()).item() < 2e-5
    assert np.isfinite(d.x.cpu().numpy()).all()
