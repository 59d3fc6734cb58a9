"""Host-side checks that need no GPU: the C-ABI library loads and exports every declared entry point, argument
validation returns the documented status codes before touching the device, and the drop-in modules' host logic
(eligibility, ConvRot hand-off, patch installation) behaves like the reference's."""
import ctypes
import os
import re
import sys
import types

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rdna2_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._lib.load()
    names = declared_symbols()
    assert len(names) >= 17
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(pkg._lib.SIGNATURES), "ctypes signatures and header disagree"
    assert lib.b2_version() == 100


def _status(pkg, name, *args):
    return getattr(pkg._lib.load(), name)(*args)


def test_validation_errors_before_any_launch(pkg):
    P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    fake = P(4096)
    # null pointers -> B2_ERR_INVALID
    assert _status(pkg, "b2_gemm", P(None), fake, fake, fake, P(None), fake, I(8), I(8), I(16), P(None), P(None), I(1), P(None)) == 1
    assert b"null" in pkg._lib.load().b2_last_error()
    # K not a multiple of 16 -> B2_ERR_UNSUPPORTED
    assert _status(pkg, "b2_gemm_i32", fake, fake, fake, I(8), I(8), I(24), P(None)) == 2
    assert _status(pkg, "b2_quant_pack_a", fake, I64(24), fake, fake, I(4), I(24), I(0), P(None)) == 2
    # rotation group must divide K
    assert _status(pkg, "b2_quant_pack_a", fake, I64(384), fake, fake, I(4), I(384), I(256), P(None)) == 2
    assert _status(pkg, "b2_quant_pack_a", fake, I64(512), fake, fake, I(4), I(512), I(64), P(None)) == 2
    # misaligned operand
    assert _status(pkg, "b2_gemm_i32", P(4097), fake, fake, I(8), I(8), I(16), P(None)) == 2
    # rotate: group must be a power of 4
    assert _status(pkg, "b2_rotate", fake, fake, I64(128), I(128), P(None)) == 2
    # decode attention: heads must be a multiple of kv heads
    assert _status(pkg, "b2_attn_decode", fake, fake, fake, fake, fake, fake, fake, I(1), I(6), I(4), I(16), F(1.0), P(None)) == 1
    # attention: head counts
    assert _status(pkg, "b2_attention", fake, I64(0), I64(0), I64(128), fake, I64(0), I64(0), I64(128), fake, I64(0), I64(0),
                   I64(128), fake, I64(0), I64(0), I64(128), I(1), I(3), I(2), I(4), I(4), F(1.0), I(0), P(None), I64(0), P(None)) == 1
    # rms_norm: D bound
    assert _status(pkg, "b2_rms_norm", fake, fake, fake, I(1), I(8200), I(1), I(1), I64(0), I64(0), I64(8200), F(1e-6), P(None)) == 2
    # SwiGLU GEMM: 2F must be a multiple of 256; GEMV with silu: act in {0, 1}, residual must not alias out
    assert _status(pkg, "b2_gemm_swiglu", fake, fake, fake, fake, fake, I(8), I(384), I(16), P(None)) == 2
    assert _status(pkg, "b2_gemv_i8_ex", fake, fake, fake, P(None), P(None), fake, I(8), I(16), I(2), P(None)) == 1
    assert _status(pkg, "b2_gemv_i8_ex", fake, fake, fake, P(None), fake, fake, I(8), I(16), I(0), P(None)) == 1
    assert _status(pkg, "b2_decode_qk_rope", fake, fake, fake, fake, P(None), fake, fake, fake, I(8), I(2), F(1e-6),
                   P(None)) == 1
    # int4 path: K % 32 for the unpack, a workspace for the W4A4 GEMM, rotation groups
    assert _status(pkg, "b2_unpack_int4", fake, fake, I(8), I(48), P(None)) == 2
    assert _status(pkg, "b2_gemm_w4a4", fake, fake, fake, fake, P(None), fake, I(4), I(8), I(64), P(None), P(None)) == 1
    assert _status(pkg, "b2_gemm_w4a4", fake, fake, fake, fake, P(None), fake, I(4), I(12), I(64), fake, P(None)) == 2
    assert _status(pkg, "b2_quant_pack_a_i4", fake, I64(512), fake, fake, I(4), I(512), I(64), P(None)) == 2
    # situ: the row stride must hold [hidden | gate]
    assert _status(pkg, "b2_situ_quant_pack_a", fake, I64(256), fake, fake, I(4), I(256), I(0), P(None), P(None)) == 1
    assert _status(pkg, "b2_situ_quant_pack_a", fake, I64(520), fake, fake, I(4), I(260), I(0), P(None), P(None)) == 2
    # bf16 GEMV: K % 8, null table
    assert _status(pkg, "b2_gemv_bf16", fake, fake, fake, I(16), I(12), P(None)) == 2
    assert _status(pkg, "b2_gemv_bf16", fake, P(None), fake, I(16), I(16), P(None)) == 1
    assert _status(pkg, "b2_gemv_bf16", fake, fake, fake, I(0), I(16), P(None)) == 0
    # empty problems succeed without launching
    assert _status(pkg, "b2_gemm_i32", fake, fake, fake, I(0), I(8), I(16), P(None)) == 0
    assert _status(pkg, "b2_quant_pack_a", fake, I64(16), fake, fake, I(0), I(16), I(0), P(None)) == 0


def test_attention_workspace_size(pkg):
    lib = pkg._lib.load()
    assert lib.b2_attention_workspace_bytes(2, 24, 24, 4056, 4056, 0) == 0
    n = lib.b2_attention_workspace_bytes(2, 24, 24, 4056, 4056, 1)
    assert n >= 2 * (2 * 24 * 4056 * 128) + 2 * 2 * 24 * 4056 * 4
    assert n % 1024 == 0


def test_cpu_tensors_are_refused(pkg):
    x = torch.zeros((4, 256), dtype=torch.float16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        pkg.ops.quant_pack_a(x, 256)


def test_attention_hip_refuses_ineligible_inputs(pkg):
    q = torch.zeros((1, 8, 2 * 128), dtype=torch.float16)
    with pytest.raises(NotImplementedError, match="mask"):
        pkg.attention.attention_hip(q, q, q, 2, mask=torch.zeros(1))
    with pytest.raises(NotImplementedError, match="head dim 64"):
        pkg.attention.attention_hip(q, q, q, 4)
    with pytest.raises(NotImplementedError, match="fp16"):
        pkg.attention.attention_hip(q.float(), q.float(), q.float(), 2)
    assert pkg.attention.eligible(q, q, q, 2) is None


def test_int8_linear_refuses_ineligible_inputs(pkg):
    f = pkg.int8_gemm.wrap(None)
    w = torch.zeros((64, 64), dtype=torch.int8)
    with pytest.raises(NotImplementedError, match="x_q"):
        f(torch.zeros((4, 64), dtype=torch.float16), w, 1.0, x_q=torch.zeros(1))
    with pytest.raises(NotImplementedError, match="fp16"):
        f(torch.zeros((4, 64)), w, 1.0)


def test_w4a4_refuses_ineligible_inputs(pkg):
    f = pkg.int8_gemm.wrap_w4a4(None)
    x = torch.zeros((4, 512), dtype=torch.float16)
    qw = torch.zeros((64, 256), dtype=torch.uint8)
    ws = torch.ones(64)
    with pytest.raises(NotImplementedError, match="ConvRot group 128"):
        f(x, qw, ws, None, 128, torch.float16)
    with pytest.raises(NotImplementedError, match="pre-rotated"):
        f(x, qw, ws, None, 256, torch.float16, x_rot=x)
    with pytest.raises(NotImplementedError, match="one per output channel"):
        f(x, qw, torch.ones((64, 2)), None, 256, torch.float16)
    with pytest.raises(NotImplementedError, match="fp16 compute"):
        f(x, qw, ws, None, 256, torch.bfloat16)


def _fake_packs():
    pack = types.ModuleType("fakepack.int8_quant")
    pack.triton_int8_linear = lambda *a, **k: "orig"
    pack.triton_int8_linear_per_row = lambda *a, **k: "orig_row"
    pack._TRITON_AVAILABLE = True

    class Linear:
        def forward(self, x):
            return "forward"

    pack.Int8TensorwiseOps = types.SimpleNamespace(Linear=Linear)
    convrot = types.ModuleType("fakepack.convrot")
    convrot.rotate_activation = lambda x, H, g: ("rotated", x)
    convrot.build_hadamard = lambda n, device=None, dtype=None: None
    return pack, convrot


def test_enable_installs_and_removes_patches(pkg):
    g = pkg.int8_gemm
    pack, convrot = _fake_packs()
    sys.modules["fakepack.int8_quant"], sys.modules["fakepack.convrot"] = pack, convrot
    try:
        g.originals.clear()
        g.enable(True)
        assert pack.triton_int8_linear.__name__ == "int8_linear"
        assert convrot.rotate_activation is g.rotate_activation
        assert g.swiglu_fusable
        # ConvRot hand-off: a fusable 2D fp16 activation is parked, not rotated.
        x = torch.zeros((4, 512), dtype=torch.float16)
        g.fusable = True
        assert g.rotate_activation(x, None, 256) is x and g.pending is x
        g.fusable, g.pending = False, None
        assert g.rotate_activation(x, None, 256)[0] == "rotated"
        g.enable(False)
        assert pack.triton_int8_linear() == "orig" and convrot.rotate_activation(x, None, 256)[0] == "rotated"
        assert not g.swiglu_fusable
    finally:
        del sys.modules["fakepack.int8_quant"], sys.modules["fakepack.convrot"]
        g.originals.clear()
        g.pending = None
        g.fusable = False


def test_situ_hand_off_through_linear_input_act(pkg):
    """int8_gemm.py:152-157: for a fusable situ layer, linear_input_act sets situ_next and calls the linear on the raw
    [hidden | gate] input, whose int8_linear then runs the situ pre-pass; anything else goes to ComfyUI's own
    linear_input_act. enable() installs it into comfy.ops and restores it."""
    g = pkg.int8_gemm
    pack, convrot = _fake_packs()
    comfy = types.ModuleType("comfy")
    comfy_ops = types.ModuleType("comfy.ops")
    comfy_ops.linear_input_act = lambda *a, **k: "core"
    comfy.ops = comfy_ops
    mods = {"fakepack.int8_quant": pack, "fakepack.convrot": convrot, "comfy": comfy, "comfy.ops": comfy_ops}
    saved = {k: sys.modules.get(k) for k in mods}
    sys.modules.update(mods)
    try:
        g.originals.clear()
        g.enable(True)
        assert comfy_ops.linear_input_act is g.linear_input_act
        layer = types.SimpleNamespace(_is_quantized=True, _use_convrot=True, _convrot_groupsize=256, lora_patches=[],
                                      in_features=512)
        seen = []

        def linear(x):
            seen.append(g.situ_next)
            g.situ_next = False
            return "fused"
        x = torch.zeros((3, 1024), dtype=torch.float16)
        fused = type("L", (), {"__call__": lambda self, t: linear(t), **vars(layer)})()
        assert g.linear_input_act(fused, x, "situ") == "fused" and seen == [True]
        assert g.linear_input_act(fused, x, "swiglu") == "core"
        assert g.linear_input_act(fused, x.float(), "situ") == "core"
        assert g.linear_input_act(fused, x, "situ", residual=torch.zeros(1)) == "core"
        g.enable(False)
        assert comfy_ops.linear_input_act() == "core"
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
        g.originals.clear()
        g.situ_next = False


def test_swiglu_interleave_pairs_gate_and_up_blocks(pkg):
    """Row i of the interleaved gate/up weight: block j = i // 256 holds gate rows [128 j, 128 j + 128) then the
    matching up rows [F + 128 j, F + 128 j + 128)."""
    F = 640
    idx = pkg.ops.swiglu_interleave(2 * F).tolist()
    assert sorted(idx) == list(range(2 * F))
    for i, r in enumerate(idx):
        j, o = divmod(i, 256)
        assert r == (128 * j + o if o < 128 else F + 128 * j + o - 128)
    with pytest.raises(RuntimeError):
        pkg.ops.swiglu_interleave(2 * 600)


def test_decode_routing_follows_the_reference(pkg):
    """int8_gemv keeps the reference's routing (int8_gemv.py:49-50,68-69,88-89): prompt encoding, batches and
    non-fp32 inputs go to the module's own forward and never reach the library; patch() installs the linear, MLP,
    logits, generate and KV-cache patches on duck-typed modules."""
    gv = pkg.int8_gemv

    class Linear:
        quant_format = "int8_tensorwise"
        weight_function, bias_function = [], []

        def forward(self, x):
            return "core linear"

    class MLP:
        merged_mlp = False

        def forward(self, x, norm=None):
            return "core mlp"

    class BaseQwen3:
        def logits(self, x):
            return "core logits"

    class Qwen3_4B(BaseQwen3):
        pass

    lin = Linear()
    assert gv.linear_forward(lin, 8, 16, torch.int8, 0, torch.zeros((1, 3, 16))) == "core linear"
    assert gv.linear_forward(lin, 8, 16, torch.int8, 1024, torch.zeros((1, 3, 16))) == "core linear"
    assert gv.linear_forward(lin, 8, 16, torch.int8, 0, torch.zeros((1, 1, 16), dtype=torch.float16)) == "core linear"
    mlp = MLP()
    mlp.gate_proj, mlp.up_proj = Linear(), Linear()
    assert gv.mlp_forward(mlp, torch.int8, torch.zeros((1, 3, 16))) == "core mlp"
    gv.generating = True
    try:
        assert gv.mlp_forward(mlp, torch.int8, torch.zeros((1, 1, 16))) == "core mlp"
    finally:
        gv.generating = False
    qwen = Qwen3_4B()
    embed = types.SimpleNamespace(weight=torch.zeros((32, 16), dtype=torch.bfloat16), weight_function=[], bias_function=[])
    config = types.SimpleNamespace(lm_head=False, head_dim=128, num_attention_heads=32, num_key_value_heads=8)
    qwen.model = types.SimpleNamespace(embed_tokens=embed, config=config, fixed_kv=True)
    assert gv.logits(qwen, torch.zeros((2, 3, 16))) == "core logits"

    lin.weight = types.SimpleNamespace(shape=(8, 16), dtype=torch.int8,
                                       _params=types.SimpleNamespace(scale=torch.ones(8), transposed=False,
                                                                     convrot=False, convrot_groupsize=0))
    mlp.gate_proj.weight = types.SimpleNamespace(dtype=torch.int8)
    patches = {}
    modules = [("layers.0.lin", lin), ("layers.0.mlp", mlp), ("", qwen)]
    clip = types.SimpleNamespace(patcher=types.SimpleNamespace(
        model=types.SimpleNamespace(named_modules=lambda: modules),
        add_object_patch=lambda name, fn: patches.__setitem__(name, fn)))
    gv.patch(clip)
    assert sorted(patches) == [".generate", ".logits", ".model.init_kv_cache", "layers.0.lin.forward", "layers.0.mlp.forward"]
    assert patches["layers.0.mlp.forward"].func is gv.mlp_forward
    assert patches[".logits"].func is gv.logits
