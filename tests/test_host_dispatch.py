"""Host-side dispatch without a GPU: the drop-in modules and drivers run on CPU tensors with the C-ABI call replaced
by a recorder, so every tensor they hand to the library passes the wrappers' size/dtype checks and the sequence of
entry points is the documented one (the DiT block's 9 launches, the decode layer's 9, the Krea-2 fused block's
side-channel hand-offs, the W4A4 and situ paths). The numerics of the same paths are the GPU tests' job."""
import types

import pytest
import torch


@pytest.fixture
def calls(pkg, monkeypatch):
    log = []
    monkeypatch.setattr(pkg.ops, "call", lambda name, *args: log.append(name))
    monkeypatch.setattr(pkg.ops, "require_cuda", lambda *tensors: None)
    monkeypatch.setattr(pkg.ops, "stream", lambda: None)
    return log


def test_dit_block_is_nine_launches(pkg, calls):
    import importlib

    dit = importlib.import_module(pkg.__name__ + ".dit")
    cfg = dit.DiTConfig(hidden=256, heads=2, mlp=512, blocks=2, batch=2, tokens=40)
    stack = dit.DiTStack(cfg, dit.shard_plan(1, 0, cfg.batch, cfg.heads), "cpu")
    stack.forward(torch.randn((2, 40, 256)).half())
    block = ["b2_mod_quant_pack_a", "b2_gemm", "b2_attention", "b2_quant_pack_a", "b2_gemm", "b2_mod_quant_pack_a",
             "b2_gemm_swiglu", "b2_quant_pack_a", "b2_gemm"]
    assert calls == block * cfg.blocks


def test_dit_head_group_reads_the_gathered_segments(pkg, calls):
    import importlib

    dit = importlib.import_module(pkg.__name__ + ".dit")
    cfg = dit.DiTConfig(hidden=256, heads=2, mlp=512, blocks=1, batch=2, tokens=40)
    plan = dit.shard_plan(4, 1, cfg.batch, cfg.heads)
    gathered = []
    stack = dit.DiTStack(cfg, plan, "cpu", all_gather=lambda out, inp: gathered.append((out.numel(), inp.numel())))
    stack.forward(torch.randn((1, 40, 256)).half())
    assert "b2_quant_pack_a_seg" in calls and gathered == [(40 * 256, 40 * 128)]


def test_decoder_layer_is_nine_launches(pkg, calls):
    import importlib

    decoder = importlib.import_module(pkg.__name__ + ".decoder")
    cfg = decoder.DecoderConfig(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128, mlp=512, capacity=16)
    dec = decoder.TextDecoder(cfg, "cpu")
    dec.mode = "layers"
    dec.set_position(3)
    dec.step_eager()
    layer = ["b2_rms_norm_f32", "b2_gemv_i8", "b2_decode_qk_rope", "b2_attn_decode", "b2_gemv_i8_ex",
             "b2_rms_norm_f32", "b2_gemv_i8", "b2_gemv_i8_ex"]
    assert calls == layer * cfg.layers
    assert decoder.TextDecoder.launches_per_layer == len(layer) + 1  # attn_decode is two kernels (split, merge)


def test_decoder_persistent_step_is_one_launch(pkg, calls):
    """The default mode hands the whole token to b2_decode_step, with a table of every layer's 14 pointers."""
    import importlib

    decoder = importlib.import_module(pkg.__name__ + ".decoder")
    cfg = decoder.DecoderConfig(hidden=256, layers=3, heads=4, kv_heads=2, head_dim=128, mlp=512, capacity=16)
    dec = decoder.TextDecoder(cfg, "cpu")
    assert dec.mode == "persistent"
    for pos in (3, 4):
        dec.set_position(pos)
        dec.step_eager()
    assert calls == ["b2_decode_step"] * 2
    assert tuple(dec.table.shape) == (3, 14)
    assert dec.table[1, 4].item() == dec.layers[1].w_qkv.data_ptr()
    assert dec.table[2, 13].item() == dec.layers[2].v_cache.data_ptr()


def test_decode_step_table_refuses_bad_layers(pkg):
    import importlib

    decoder = importlib.import_module(pkg.__name__ + ".decoder")
    cfg = decoder.DecoderConfig(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128, mlp=512, capacity=16)
    dec = decoder.TextDecoder(cfg, "cpu")
    dec.layers[1].s_o = dec.layers[1].s_o.double()
    with pytest.raises(RuntimeError, match="layer 1 s_o"):
        pkg.ops.decode_step_table(dec.layers, 256, 4, 2, 512, 16)
    dec.layers[1].s_o = dec.layers[1].s_o.float()
    dec.layers[0].w_gu = dec.layers[0].w_gu.t()
    with pytest.raises(RuntimeError, match="layer 0 w_gu"):
        pkg.ops.decode_step_table(dec.layers, 256, 4, 2, 512, 16)


def _linear(pkg, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    s = torch.rand(N, generator=g) * 1e-3
    f = pkg.int8_gemm.wrap(None)

    def forward(x):
        # What the Int8 loader's Linear does: ConvRot hand-off, then the patched triton_int8_linear.
        return f(pkg.int8_gemm.rotate_activation(x, None, 256), w, s)
    return types.SimpleNamespace(__call__=forward, forward=forward, in_features=K)


class _Call:
    def __init__(self, fn):
        self.fn = fn

    def __call__(self, x):
        return self.fn(x)


def test_krea2_block_forward_hand_offs(pkg, calls):
    """int8_gemm.block_forward (int8_gemm.py:189-226): the modulated norm quantized once for wq/wk/wv/gate, QK-norm +
    rope, attention, the sigmoid gate in the out-projection's pre-pass with the gated residual, the second norm for
    gate/up, the SwiGLU in the down projection's pre-pass with the gated residual."""
    gm = pkg.int8_gemm
    B, L, D, H = 1, 24, 256, 2
    mk = lambda n, k, s: _Call(_linear(pkg, n, k, s).forward)  # noqa: E731
    norm = lambda: types.SimpleNamespace(scale=torch.randn(D) * 0.02, eps=1e-6)  # noqa: E731
    qk = types.SimpleNamespace(qnorm=types.SimpleNamespace(scale=torch.zeros(128), eps=1e-6),
                               knorm=types.SimpleNamespace(scale=torch.zeros(128), eps=1e-6))
    attn = types.SimpleNamespace(wq=mk(D, D, 1), wk=mk(D, D, 2), wv=mk(D, D, 3), gate=mk(D, D, 4), wo=mk(D, D, 5),
                                 heads=H, kvheads=H, headdim=128, qknorm=qk)
    mlp = types.SimpleNamespace(gate=mk(512, D, 6), up=mk(512, D, 7), down=mk(D, 512, 8))
    mods = [torch.randn((B, 1, D)).half() * 0.1 for _ in range(6)]
    module = types.SimpleNamespace(attn=attn, mlp=mlp, mod=lambda vec: mods, prenorm=norm(), postnorm=norm())
    freqs = torch.randn((1, 1, L, 64, 2, 2))
    out = gm.block_forward(module, False, torch.randn((B, L, D)).half(), None, freqs)
    assert out.shape == (B, L, D)
    assert calls == ["b2_mod_quant_pack_a", "b2_gemm", "b2_gemm", "b2_gemm", "b2_gemm", "b2_rms_norm_rope",
                     "b2_rms_norm_rope", "b2_attention", "b2_gate_quant_pack_a", "b2_gemm", "b2_mod_quant_pack_a",
                     "b2_gemm", "b2_gemm", "b2_swiglu_quant_pack_a", "b2_gemm"]
    assert gm.shared is None and gm.swiglu_up is None and gm.sigmoid_gate is None and gm.residual is None


def test_drop_in_entry_points_dispatch(pkg, calls):
    # attention_hip: (B, L, H*D) and (B, H, L, D) with skip_reshape
    q = torch.randn((2, 30, 2 * 128)).half()
    assert pkg.attention.attention_hip(q, q, q, 2).shape == q.shape
    qh = q.view(2, 30, 2, 128).transpose(1, 2)
    assert pkg.attention.attention_hip(qh, qh, qh, 2, skip_reshape=True, skip_output_reshape=True).shape == qh.shape
    # rms_norm drop-ins
    m = types.SimpleNamespace(scale=torch.zeros(256), eps=1e-6)
    pkg.rms_norm.forward(m, torch.randn((2, 5, 256)).half())
    mh = types.SimpleNamespace(scale=torch.zeros(128), eps=1e-6)
    pkg.rms_norm.rms_norm_rope(torch.randn((2, 7, 2 * 128)).half(), 2, mh, torch.randn((2, 1, 7, 64, 2, 2)))
    # int8 linears: plain, rotated, situ, SwiGLU and gate flavours of the pre-pass
    g = pkg.int8_gemm
    w, s = torch.randint(-127, 128, (64, 256), dtype=torch.int8), torch.rand(64)
    x = torch.randn((9, 256)).half()
    g.linear(x, w, s, None)
    g.linear(x, w, s, None, rotate=True)
    g.linear(torch.randn((9, 512)).half(), w, s, None, situ=True)
    g.linear(x, w, s, None, rotate=True, up=x.clone())
    g.linear(x, w, s, None, gate=x.clone())
    # per-channel W4A4
    g.wrap_w4a4(None)(torch.randn((3, 5, 512)).half(), torch.zeros((64, 256), dtype=torch.uint8), torch.ones(64), None,
                      256, torch.float16)
    # decode: GEMV with and without ConvRot, logits, decode attention
    gv = pkg.int8_gemv
    lin = types.SimpleNamespace(weight=types.SimpleNamespace(_qdata=torch.zeros((32, 256), dtype=torch.int8),
                                                             _params=types.SimpleNamespace(scale=torch.ones(32))),
                                bias=None, weight_function=[], bias_function=[])
    gv.linear_forward(lin, 32, 256, torch.int8, 0, torch.randn((1, 1, 256)))
    gv.linear_forward(lin, 32, 256, torch.int8, 256, torch.randn((1, 1, 256)))
    embed = types.SimpleNamespace(weight=torch.zeros((48, 256), dtype=torch.bfloat16), weight_function=[],
                                  bias_function=[])
    assert gv.logits(types.SimpleNamespace(model=types.SimpleNamespace(embed_tokens=embed)),
                     torch.randn((1, 4, 256))).shape == (1, 1, 48)
    gv.attention_decode(torch.randn((1, 1, 8, 128)), torch.randn((1, 16, 2, 128)), torch.randn((1, 16, 2, 128)),
                        torch.tensor([5], dtype=torch.int32))
    assert calls == ["b2_attention", "b2_attention", "b2_rms_norm", "b2_rms_norm_rope",
                     "b2_quant_pack_a", "b2_gemm", "b2_quant_pack_a", "b2_gemm", "b2_situ_quant_pack_a", "b2_gemm",
                     "b2_swiglu_quant_pack_a", "b2_gemm", "b2_gate_quant_pack_a", "b2_gemm",
                     "b2_quant_pack_a_i4", "b2_gemm_w4a4",
                     "b2_gemv_i8", "b2_rotate", "b2_gemv_i8", "b2_gemv_bf16", "b2_attn_decode"]


def test_wrappers_refuse_buffers_the_kernels_would_overrun(pkg, calls):
    ops = pkg.ops
    a, w = torch.zeros((8, 64), dtype=torch.int8), torch.zeros((16, 64), dtype=torch.int8)
    with pytest.raises(RuntimeError, match="activation scale"):
        ops.gemm(a, torch.ones(4), w, torch.ones(16))
    with pytest.raises(RuntimeError, match="weight scale"):
        ops.gemm(a, torch.ones(8), w, torch.ones(15))
    with pytest.raises(RuntimeError, match="gemm output"):
        ops.gemm(a, torch.ones(8), w, torch.ones(16), out=torch.empty((8, 8), dtype=torch.float16))
    with pytest.raises(RuntimeError, match="bias"):
        ops.gemm(a, torch.ones(8), w, torch.ones(16), bias=torch.zeros(16))
    with pytest.raises(RuntimeError, match="quantized output"):
        ops.quant_pack_a(torch.zeros((4, 64)).half(), out=(torch.empty((4, 32), dtype=torch.int8), torch.empty(4)))
    with pytest.raises(RuntimeError, match="act_out"):
        ops.swiglu_quant_pack_a(torch.zeros((4, 64)).half(), torch.zeros((4, 64)).half(),
                                act_out=torch.empty((4, 32)).half())
    q = torch.zeros((2, 2, 8, 128)).half()
    with pytest.raises(RuntimeError, match="k and v"):
        ops.attention(q, torch.zeros((1, 2, 8, 128)).half(), torch.zeros((1, 2, 8, 128)).half(), q, 1.0)
    with pytest.raises(RuntimeError, match="k and v"):
        ops.attention(q, q, torch.zeros((2, 2, 9, 128)).half(), q, 1.0)
    with pytest.raises(RuntimeError, match="gemv_i8 output"):
        ops.gemv_i8(torch.zeros(64), w, torch.ones(16), out=torch.empty(8))
    with pytest.raises(RuntimeError, match="gemv_i8 scale"):
        ops.gemv_i8(torch.zeros(64), w, torch.ones(16, dtype=torch.float64))
    with pytest.raises(RuntimeError, match="lengths"):
        ops.attn_decode(torch.zeros((2, 1, 4, 128)), torch.zeros((2, 8, 2, 128)), torch.zeros((2, 8, 2, 128)),
                        torch.zeros(2, dtype=torch.int64), 1.0)
    with pytest.raises(RuntimeError, match="segments reach past"):
        ops.quant_pack_a_segments(torch.zeros(4 * 10 * 128).half(), 512, 128, 128, 10 * 128, 11, 128)
    with pytest.raises(RuntimeError, match="workspace"):
        ops.gemm_w4a4(a, torch.ones(8), torch.zeros((16, 32), dtype=torch.uint8), torch.ones(16),
                      workspace=torch.empty(10, dtype=torch.int8))
    with pytest.raises(RuntimeError, match="rope frequencies"):
        ops.rms_norm_rows(torch.zeros((2, 3, 128)).half(), torch.zeros(128), 1e-6, 6, 128, 3, 1, 384, 0, 128,
                          torch.empty((2, 3, 128)).half(), freqs=torch.zeros((1, 1, 2, 64, 2, 2)))
    assert calls == []


def test_prefill_routes_while_generating(pkg, calls):
    """While generating, a multi-token fp32 input of a linear with a ConvRot group above 256 runs the rotation kernel
    and a dense fp32 linear on the dequantized weight (int8_gemv.py:49-57); a gated MLP runs one stacked gate|up
    linear (:67-75). With a group of 256 or less the layer's own forward runs (no launch)."""
    gv = pkg.int8_gemv
    qdata = torch.randint(-127, 128, (32, 1024), dtype=torch.int8)

    class Linear:
        weight = types.SimpleNamespace(_qdata=qdata, _params=types.SimpleNamespace(scale=torch.rand(32)))
        bias, weight_function, bias_function = None, [], []

        def forward(self, x):
            return "core"

    lin = Linear()
    x = torch.randn((1, 5, 1024))
    gv.generating = True
    try:
        y = gv.linear_forward(lin, 32, 1024, torch.int8, 1024, x)
        assert y.shape == (1, 5, 32) and calls == ["b2_rotate"]
        assert gv.linear_forward(lin, 32, 1024, torch.int8, 256, x) == "core"
        gate, up = Linear(), Linear()
        mlp = types.SimpleNamespace(gate_proj=gate, up_proj=up, activation=torch.nn.functional.silu,
                                    down_proj=lambda h: h)
        h = gv.mlp_forward(mlp, torch.int8, x)
        assert h.shape == (1, 5, 32) and calls == ["b2_rotate"]
    finally:
        gv.generating = False


def test_w4a8_forward_dispatch(pkg, calls):
    """int8_gemm.w4a8_forward: block-128 rotation + int8 pre-pass, then the group-128 W4A8 GEMM on the widened weight
    (widened per call, or the caller's qweight_unpacked as is)."""
    f = pkg.int8_gemm.w4a8_forward
    x = torch.randn((2, 7, 512)).half()
    out = f(x, torch.zeros((64, 256), dtype=torch.uint8), torch.ones((64, 4)).half(), None, 128, torch.float16)
    assert out.shape == (2, 7, 64) and calls == ["b2_unpack_int4", "b2_quant_pack_a", "b2_gemm_w4a8_wide"]
    calls.clear()
    out = f(x, torch.zeros((64, 256), dtype=torch.uint8), torch.ones((64, 4)).half(), None, 128, torch.float16,
            qweight_unpacked=torch.zeros((64, 512), dtype=torch.int8))
    assert out.shape == (2, 7, 64) and calls == ["b2_quant_pack_a", "b2_gemm_w4a8_wide"]
    with pytest.raises(NotImplementedError, match="qweight_unpacked"):
        f(x, torch.zeros((64, 256), dtype=torch.uint8), torch.ones((64, 4)).half(), None, 128, torch.float16,
          qweight_unpacked=torch.zeros((64, 256), dtype=torch.int8))
    with pytest.raises(NotImplementedError, match="scales of shape"):
        f(x, torch.zeros((64, 256), dtype=torch.uint8), torch.ones(64).half(), None, 128, torch.float16)


def test_dit_fused_gather_dispatch(pkg, calls):
    """Head-group mode with the fused gather: the attention delivers to the peers (b2_attention_gather), a bounded
    stream-ordered wait on the arrival counter precedes the out-projection pre-pass, which reads the parity buffer."""
    import importlib

    dit = importlib.import_module(pkg.__name__ + ".dit")
    cfg = dit.DiTConfig(hidden=256, heads=4, mlp=512, blocks=3, batch=2, tokens=40)
    plan = dit.shard_plan(4, 1, cfg.batch, cfg.heads)
    g, hl = plan.group_size, plan.head_hi - plan.head_lo
    buf = torch.zeros((2, g, 1, cfg.tokens, hl * 128), dtype=torch.float16)
    fg = dit.FusedGather(buf, [1 << 20], torch.zeros(8, dtype=torch.int64), [2 << 20], torch.zeros(1, dtype=torch.int32),
                         plan.group_index)
    stack = dit.DiTStack(cfg, plan, "cpu", fused_gather=fg)
    stack.forward(torch.randn((1, 40, 256)).half())
    block = ["b2_mod_quant_pack_a", "b2_gemm", "b2_attention_gather", "b2_wait_count", "b2_quant_pack_a_seg", "b2_gemm",
             "b2_mod_quant_pack_a", "b2_gemm_swiglu", "b2_quant_pack_a", "b2_gemm"]
    assert calls == block * cfg.blocks and fg.blocks_done == cfg.blocks
