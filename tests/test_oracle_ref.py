"""The oracle restatement against the reference's own kernels, run on the host (oracle/hipref.py).

oracle/hipemu/build.py compiles the reference's int8_gemm.hip, hip_attention.hip, int8_gemv.hip and rms_norm.hip
for the CPU; these tests launch them as the reference's Python does and compare with oracle/*. Integer, byte and
pure IEEE paths must agree bit for bit: the quantizers (half-up after an IEEE divide, half-even for int4), the
ConvRot butterflies, the packed layouts (undone by hipref), the int32 GEMM and its fp16 epilogue with bias and
gated residual, the int4 GEMM, the decode rotation. Paths through exp/exp2/rsqrt are compared with tolerances: the
host's libm and the gfx1030 hardware differ there by an ulp, which moves an int8 value by one on rare elements.
Skipped where the reference sources (environment variable REF_DIR) are not present.
"""
import numpy as np
import pytest

from oracle import attention as oatt
from oracle import decode as odec
from oracle import gemm as ogemm
from oracle import hipref as hr
from oracle import norm as onorm
from oracle import quant as oq
from oracle.hipemu import build as hbuild

F16, F32 = np.float16, np.float32


@pytest.fixture(scope="module", autouse=True)
def reference_lib():
    if hbuild.build() is None or not hr.available():
        pytest.skip("reference kernel sources not present")


def activations(M, K, seed, outliers=True):
    g = np.random.default_rng(seed)
    x = g.standard_normal((M, K)).astype(F32)
    if outliers:
        x[:, g.choice(K, max(1, K // 100), replace=False)] *= 20
    return x.astype(F16)


def edge_rows(K):
    x = np.zeros((8, K), F16)
    x[1, :] = 65504                          # fp16 max: the rotation overflows fp16 to inf
    x[2, ::2] = 6e-8                         # subnormal
    x[3, :8] = [127, 0.5, -0.5, 1.5, -1.5, 2.5, -2.5, -127]  # half-up ties at scale 1
    x[4] = np.linspace(-3, 3, K).astype(F16)
    x[6] = np.linspace(-1, 1, K).astype(F16)
    x[6, 130] = np.nan
    x[7] = np.linspace(-2, 2, K).astype(F16)
    x[7, 5] = -np.inf
    return x


@pytest.mark.parametrize("M,K", [(1, 256), (70, 3072), (513, 512), (5, 16384)])
def test_quant_and_convrot_bit_exact(M, K):
    """quant_row (int8_gemm.hip:29-60) with and without rot_quant's ConvRot (:105-116, :154-247)."""
    x = activations(M, K, M + K)
    for kind, rot in (("plain", 0), ("rotate", 256)):
        q, s = hr.quant(x, kind)
        q_ref, s_ref, _ = oq.prepass(x, rot)
        assert np.array_equal(s, s_ref), kind
        assert np.array_equal(q, q_ref), kind


@pytest.mark.parametrize("K", [256, 1024])
def test_quant_edge_values(K):
    x = edge_rows(K)
    for kind, rot in (("plain", 0), ("rotate", 256)):
        q, s = hr.quant(x, kind)
        q_ref, s_ref, _ = oq.prepass(x, rot)
        assert np.array_equal(s, s_ref) and np.array_equal(q, q_ref), kind


def test_int4_activations_bit_exact():
    """quant_row_i4 (int8_gemm.hip:62-91) after ConvRot: scale max(absmax, 1e-10) / 7, rint, clamp to [-7, 7]."""
    for M, K, seed in ((33, 512, 1), (8, 1024, 2)):
        x = activations(M, K, seed) if seed == 1 else edge_rows(K)
        q, s = hr.quant(x, "i4")
        q_ref, s_ref = oq.quant_rows_i4(oq.rotate_rows(x, 256))
        assert np.array_equal(s, s_ref) and np.array_equal(q, q_ref)


@pytest.mark.parametrize("kind", ["plain", "rotate"])
def test_linear_epilogue_bit_exact(kind):
    """run() (int8_gemm.py:56-80): pack_b + gemm; y = fp16((float)acc * sa * sw (+ bias)) (int8_gemm.hip:382-383)."""
    g = np.random.default_rng(5)
    M, K, N = 600, 512, 192
    x = activations(M, K, 6)
    w = g.integers(-127, 128, (N, K), dtype=np.int8)
    ws = (g.random(N) * 1e-3).astype(F32)
    b = (g.standard_normal(N) * 0.01).astype(F16)
    q, s, _ = oq.prepass(x, 0 if kind == "plain" else 256)
    for bias in (None, b):
        y = hr.linear(x, w, ws, bias, kind=kind)
        assert np.array_equal(y, ogemm.epilogue(ogemm.int_mm(q, w), s, ws, bias))


def test_linear_gated_residual_bit_exact():
    """The block epilogue out = fp16(R + fp16(G[row / L] * y)) (int8_gemm.hip:394-400)."""
    g = np.random.default_rng(7)
    M, K, N, L = 600, 256, 128, 300
    x = activations(M, K, 8)
    w = g.integers(-127, 128, (N, K), dtype=np.int8)
    ws = (g.random(N) * 1e-3).astype(F32)
    R = g.standard_normal((M, N)).astype(F16)
    G = (g.standard_normal((M // L, N)) * 0.5).astype(F16)
    q, s, _ = oq.prepass(x, 0)
    y = hr.linear(x, w, ws, None, res=(R, G, L))
    assert np.array_equal(y, ogemm.epilogue(ogemm.int_mm(q, w), s, ws, None, R=R, G=G, L=L))


def test_raw_weight_gemm_bit_exact():
    """gemm_k6144 reads 6144-byte weight rows in place (int8_gemm.py:70-71, int8_gemm.hip:414)."""
    g = np.random.default_rng(9)
    x = activations(64, 6144, 10)
    w = g.integers(-127, 128, (64, 6144), dtype=np.int8)
    ws = (g.random(64) * 1e-3).astype(F32)
    q, s, _ = oq.prepass(x, 0)
    assert np.array_equal(hr.linear(x, w, ws), ogemm.epilogue(ogemm.int_mm(q, w), s, ws))


def test_w4a4_bit_exact():
    """wrap_w4a4 (int8_gemm.py:90-103): ConvRot + int4 activations, gemm_i4 on the packed weight, per-channel scale."""
    g = np.random.default_rng(11)
    M, K, N = 520, 512, 128
    x = activations(M, K, 12)
    packed = g.integers(0, 256, (N, K // 2), dtype=np.uint8)
    ws = (g.random(N) * 1e-2).astype(F32)
    b = (g.standard_normal(N) * 0.01).astype(F16)
    q4, s4 = oq.quant_rows_i4(oq.rotate_rows(x, 256))
    y = hr.linear(x, packed, ws, b, i4=True)
    assert np.array_equal(y, ogemm.epilogue(ogemm.int_mm(q4, ogemm.unpack_int4(packed)), s4, ws, b))


def _close_int8(q, s, q_ref, s_ref, rate=1e-4):
    # An exp or rsqrt an ulp apart can move an fp16 activation by a step, and an int8 value by one.
    d = np.abs(q.astype(np.int32) - q_ref.astype(np.int32))
    assert d.max() <= 1 and np.mean(d != 0) < rate
    rel = np.abs(s.astype(np.float64) - s_ref) / s_ref
    assert rel.max() < 2e-3


def test_activation_prepasses():
    """SwiGLU, sigmoid gate, situ (int8_gemm.hip:118-137) and the modulated RMSNorm (:139-143, :167-191), each
    followed by ConvRot and quant_row."""
    g = np.random.default_rng(13)
    M, K = 97, 3072
    gate = (g.standard_normal((M, K)) * 2).astype(F16)
    up = g.standard_normal((M, K)).astype(F16)
    for kind, act in (("swiglu", oq.swiglu(gate, up)), ("gate", oq.sigmoid_gate(gate, up))):
        q, s = hr.quant(gate, kind, u=up)
        _close_int8(q, s, *oq.quant_rows(oq.rotate_rows(act, 256)))
    h = (g.standard_normal((M, K)) * 30).astype(F16)
    gt = (g.standard_normal((M, K)) * 3).astype(F16)
    q, s = hr.quant(np.concatenate([h, gt], 1), "situ")
    _close_int8(q, s, *oq.quant_rows(oq.rotate_rows(oq.situ(h, gt), 256)))
    B, L = 2, 50
    x = activations(B * L, K, 14)
    w = (g.standard_normal(K) * 0.02).astype(F32)
    srow = (1 + g.standard_normal((B, K)) * 0.1).astype(F16)
    trow = (g.standard_normal((B, K)) * 0.1).astype(F16)
    q, s = hr.quant(x, "mod", w=w, s=srow, t=trow, L=L, eps=1e-6)
    _close_int8(q, s, *oq.quant_rows(oq.rotate_rows(oq.modulate(x, w, srow, trow, L, 1e-6), 256)))


@pytest.mark.parametrize("int8_qk", [False, True])
def test_attention_semantics(int8_qk):
    """attn / attn_i8 (hip_attention.hip:160-373) against the oracle's restatement of their arithmetic (16-key steps,
    lazy rescale at m + 8, fp16 P, int8 Q/K half-even): the remaining difference is fdot2's and exp2's rounding."""
    g = np.random.default_rng(15)
    q = g.standard_normal((2, 4, 70, 128)).astype(F16)
    k = g.standard_normal((2, 2, 90, 128)).astype(F16)
    v = g.standard_normal((2, 2, 90, 128)).astype(F16)
    out = hr.attention(q, k, v, 128 ** -0.5, int8_qk)
    sem = oatt.attention_semantics(q, k, v, 128 ** -0.5, int8_qk=int8_qk, tile=16)
    assert oatt.rel_l2(out, sem) < 2e-4
    assert oatt.rel_l2(out, oatt.attention_exact(q, k, v, 128 ** -0.5)) < (1e-2 if int8_qk else 2e-3)


def test_decode_kernels():
    """rotate (int8_gemv.hip:32-52) bit for bit; gemv_i8, gemv_bf16 and the split decode attention (:55-195)
    against the float64 oracle."""
    g = np.random.default_rng(17)
    x = g.standard_normal(4096).astype(F32)
    for group in (4, 256, 1024):
        assert np.array_equal(hr.rotate(x, group), odec.rotate(x, group))
    w = g.integers(-127, 128, (48, 1024), dtype=np.int8)
    s = g.random(48).astype(F32)
    b = g.standard_normal(48).astype(F32)
    xx = g.standard_normal(1024).astype(F32)
    assert oatt.rel_l2(hr.gemv_i8(xx, w, s, b), odec.gemv_i8(xx, w, s, b)) < 1e-6
    bits = (g.standard_normal((32, 512)).astype(F32).view(np.uint32) >> 16).astype(np.uint16)
    xb = g.standard_normal(512).astype(F32)
    assert oatt.rel_l2(hr.gemv_bf16(xb, bits), odec.gemv_bf16(xb, bits)) < 1e-6
    q = g.standard_normal((2, 1, 8, 128)).astype(F32)
    k = g.standard_normal((2, 100, 2, 128)).astype(F32)
    v = g.standard_normal((2, 100, 2, 128)).astype(F32)
    assert oatt.rel_l2(hr.attn_decode(q, k, v, [77, 3]), odec.attn_decode(q, k, v, [77, 3], 128 ** -0.5)) < 1e-6


def test_rms_norm_and_rope():
    """norm_row (rms_norm.hip:9-65): the restatement sums squares in another order, so values may move a step."""
    g = np.random.default_rng(19)
    for shape in ((2, 5, 3072), (1, 9, 128), (2, 3, 4, 64)):
        x = (g.standard_normal(shape) * 3).astype(F16)
        w = (g.standard_normal(shape[-1]) * 0.1).astype(F32)
        a, b = hr.rms_norm(x, w, 1e-6), onorm.rms_norm(x, w, 1e-6)
        d = np.abs(a.astype(F32) - b.astype(F32))
        assert np.all(d <= 2 * np.abs(np.spacing(b.astype(F16))).astype(F32)) and np.mean(a != b) < 2e-3
    B, L, H = 2, 40, 4
    x = g.standard_normal((B, L, H * 128)).astype(F16)
    w = (g.standard_normal(128) * 0.1).astype(F32)
    ang = g.random((B, 1, L, 64)).astype(F32) * 6
    f = np.stack([np.stack([np.cos(ang), -np.sin(ang)], -1), np.stack([np.sin(ang), np.cos(ang)], -1)], -2)
    a, b = hr.rms_norm_rope(x, H, w, 1e-6, f.astype(F32)), onorm.rms_norm_rope(x, H, w, 1e-6, f.astype(F32))
    assert np.mean(a != b) < 2e-3 and np.max(np.abs(a.astype(F32) - b.astype(F32))) < 1e-2
