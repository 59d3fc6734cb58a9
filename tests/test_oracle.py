"""Known-answer tests that pin the CPU oracle to the reference kernels' arithmetic (no GPU needed)."""
import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import decode as odec
from oracle import gemm as ogemm
from oracle import norm as onorm
from oracle import quant as oq
from oracle import weights as ow

F16 = np.float16
F32 = np.float32


def test_quant_rounds_half_up_after_ieee_divide():
    # int8_gemm.hip:38,53: scale = max(127/127, 1e-30) = 1; q = floor(x + 0.5): ties go up, also for negatives.
    row = np.array([[127, 0.5, -0.5, 1.5, -1.5, 2.5, -2.5, -127]], dtype=F16)
    q, s = oq.quant_rows(row)
    assert s[0] == 1.0
    assert q.tolist() == [[127, 1, 0, 2, -1, 3, -2, -127]]


def test_quant_nan_never_wins_absmax():
    # int8_gemm.hip:96-100,32-37: mx = fmaxf chain from 0, so a NaN is skipped; fmaxf(NaN, -128) = -128 (:53).
    row = np.array([[np.nan, 2.54, -1.27, 0]], dtype=F16)
    q, s = oq.quant_rows(row)
    assert s[0] == np.float32(np.float16(2.54)) / np.float32(127)
    assert q.tolist() == [[-128, 127, -63, 0]]


def test_quant_zero_row_uses_scale_floor():
    q, s = oq.quant_rows(np.zeros((2, 16), F16))
    assert np.all(s == F32(1e-30)) and not q.any()


def test_quant_scale_is_ieee_quotient():
    row = (np.arange(1, 17, dtype=F32) * F32(0.37)).astype(F16)[None]
    _, s = oq.quant_rows(row)
    assert s[0] == np.float32(np.abs(row.astype(F32)).max()) / np.float32(127)


def _kron_h256():
    h4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)
    h = h4
    for _ in range(3):
        h = np.kron(h, h4)
    return h


def test_convrot_unit_vectors_match_kronecker_rows():
    # The butterfly of int8_gemm.hip:106-116 is the regular H4 applied per base-4 digit: H4^(x)4 / 16.
    H = _kron_h256() / 16.0
    for i in (0, 1, 3, 17, 255):
        e = np.zeros((1, 256), F32)
        e[0, i] = 1
        assert np.array_equal(oq.hadamard256(e)[0].astype(np.float64), H[:, i])


def test_convrot_matches_matrix_within_rounding():
    x = np.random.default_rng(1).standard_normal((4, 512)).astype(F32)
    ref = (x.reshape(4, 2, 256).astype(np.float64) @ _kron_h256().T / 16.0).reshape(4, 512)
    assert np.allclose(oq.hadamard256(x).astype(np.float64), ref, rtol=2e-3, atol=2e-3)


def test_block128_is_orthonormal_sylvester():
    e = np.zeros((1, 128), F32)
    e[0, 0] = 1
    assert np.all(oq.hadamard128(e) == np.float16(1 / np.sqrt(128)))
    e[0, 0], e[0, 1] = 0, 1
    y = oq.hadamard128(e)[0].astype(F32)
    assert np.all(y[0::2] > 0) and np.all(y[1::2] < 0)
    x = np.random.default_rng(2).standard_normal((3, 256)).astype(F32)
    twice = oq.hadamard128(oq.hadamard128(x).astype(F32))
    assert np.allclose(twice.astype(F32), x, atol=2e-2)


def test_weight_rotation_cancels_activation_rotation():
    g = np.random.default_rng(3)
    x = g.standard_normal((5, 256)).astype(F32)
    w = g.standard_normal((7, 256)).astype(F32)
    for rot_w, rot_x in ((ow.sylvester_rotate, oq.hadamard128), (ow.convrot_rotate, oq.hadamard256)):
        y = rot_x(x).astype(np.float64) @ rot_w(w).astype(np.float64).T
        assert np.allclose(y, x.astype(np.float64) @ w.T.astype(np.float64), rtol=1e-2, atol=3e-2)


def test_swiglu_and_gate_round_at_torch_points():
    g = np.random.default_rng(4)
    gate = g.standard_normal((8, 64)).astype(F16)
    up = g.standard_normal((8, 64)).astype(F16)
    t_gate, t_up = torch.from_numpy(gate), torch.from_numpy(up)
    ref = torch.nn.functional.silu(t_gate.float()).half().float().mul(t_up.float()).half().numpy()
    got = oq.swiglu(gate, up)
    assert np.mean(got != ref) < 1e-2  # exp implementations differ by an ulp at most
    ref_g = (t_up.float() * torch.sigmoid(t_gate.float()).half().float()).half().numpy()
    assert np.mean(oq.sigmoid_gate(up, gate) != ref_g) < 1e-2


def test_int4_activations_round_half_even():
    # int8_gemm.hip:71,84: scale = max(mx, 1e-10) / 7; q = clamp(rint(f / scale), -7, 7); NaN -> -7.
    row = np.array([[7, 3.5, 2.5, -2.5, 0.5, -0.5, 1.5, -6.5, np.nan]], dtype=F16)
    q, s = oq.quant_rows_i4(row)
    assert s[0] == 1.0
    assert q.tolist() == [[7, 4, 2, -2, 0, 0, 2, -6, -7]]
    q, s = oq.quant_rows_i4(np.zeros((1, 8), F16))
    assert s[0] == np.float32(np.float32(1e-10) / np.float32(7)) and not q.any()


def test_situ_is_soft_capped_gated_tanh():
    """int8_gemm.hip:118-127: situ(h, g) = 4 tanh(g/4) sigmoid(g) 25 tanh(h/25), tanh and sigmoid via 2^x with the
    odd series below |x| = 0.02; one fp16 rounding. Against float64 math: within one fp16 step; odd in h; bounded by
    100 in magnitude; the series and exponential branches of tanh meet within an fp32 ulp."""
    g = np.random.default_rng(9)
    h = (g.standard_normal(4096) * 60).astype(F16)
    gt = (g.standard_normal(4096) * 4).astype(F16)
    got = oq.situ(h, gt).astype(np.float64)
    h64, g64 = h.astype(np.float64), gt.astype(np.float64)
    exact = 4 * np.tanh(g64 / 4) / (1 + np.exp(-g64)) * 25 * np.tanh(h64 / 25)
    assert np.all(np.abs(got - exact) <= np.abs(np.spacing(exact.astype(F16))).astype(np.float64))
    assert np.array_equal(oq.situ(-h, gt), -oq.situ(h, gt))
    assert np.all(np.abs(got) < 100)
    edge = np.array([np.nextafter(F32(0.02), F32(0)), F32(0.02)], F32)
    assert abs(float(oq.soft_tanh(edge)[0]) - float(oq.soft_tanh(edge)[1])) < 2 * float(np.spacing(F32(0.02)))
    q, s, a = oq.prepass(np.concatenate([h.reshape(16, 256), gt.reshape(16, 256)], axis=1), 256, act="situ")
    assert a.shape == (16, 256) and np.array_equal(a, oq.situ(h.reshape(16, 256), gt.reshape(16, 256)))


def test_modulate_with_identity_modulation_is_rms_norm():
    g = np.random.default_rng(5)
    x = g.standard_normal((6, 256)).astype(F16)
    w = (g.standard_normal(256) * 0.02).astype(F32)
    s = np.ones((2, 256), F16)
    t = np.zeros((2, 256), F16)
    assert np.array_equal(oq.modulate(x, w, s, t, 3, 1e-6), onorm.rms_norm(x, w, 1e-6))


def test_epilogue_known_answers():
    acc = np.array([[100, -7]], np.int32)
    y = ogemm.epilogue(acc, np.array([0.5], F32), np.array([0.25, 2.0], F32), bias=np.array([1, 0], F16))
    assert y.tolist() == [[13.5, -7.0]]
    r = ogemm.epilogue(acc, np.array([0.5], F32), np.array([0.25, 2.0], F32), R=np.array([[1, 1]], F16),
                       G=np.array([[2, 0.5]], F16), L=1)
    assert r.tolist() == [[26.0, -2.5]]


def test_int_mm_exact():
    g = np.random.default_rng(6)
    a = g.integers(-128, 128, (33, 64), dtype=np.int8)
    b = g.integers(-128, 128, (24, 64), dtype=np.int8)
    assert np.array_equal(ogemm.int_mm(a, b), a.astype(np.int64) @ b.astype(np.int64).T)


def test_int4_pack_roundtrip_and_grouped_reference():
    g = np.random.default_rng(7)
    w = (g.standard_normal((16, 256)) * 0.02).astype(F32)
    packed, s16 = ow.quantize_int4_groups(w)
    q = ogemm.unpack_int4(packed)
    assert q.min() >= -8 and q.max() <= 7
    deq = q.reshape(16, 2, 128).astype(F32) * s16.astype(F32)[:, :, None]
    assert np.abs(deq.reshape(16, 256) - w).max() <= np.abs(w).max() / 7 * 0.51 + 1e-6
    a = g.integers(-127, 128, (4, 256), dtype=np.int8)
    sa = np.full(4, 0.01, F32)
    out = ogemm.w4a8_grouped(a, sa, packed, s16)
    ref = (a.astype(np.float64) @ deq.reshape(16, 256).T.astype(np.float64)) * 0.01
    assert np.allclose(out.astype(np.float64), ref, rtol=1e-2, atol=1e-3)


def test_decode_rotate_is_involutive_and_matches_convrot():
    x = np.random.default_rng(8).standard_normal(1024).astype(F32)
    assert np.allclose(odec.rotate(odec.rotate(x, 256), 256), x, atol=1e-5)
    e = np.zeros(256, F32)
    e[5] = 1
    assert np.allclose(odec.rotate(e, 256) * 16, _kron_h256()[:, 5] / 16 * 16)


def test_rope_identity_rotation_keeps_values():
    y = np.random.default_rng(9).standard_normal((1, 2, 3, 128)).astype(F16)
    f = np.zeros((1, 1, 3, 64, 2, 2), F32)
    f[..., 0, 0] = 1
    f[..., 1, 1] = 1
    assert np.array_equal(onorm.rope(y, f), y)


@pytest.mark.parametrize("int8_qk", [False, True])
def test_attention_semantics_close_to_exact(int8_qk):
    g = np.random.default_rng(10)
    q = g.standard_normal((1, 2, 70, 128)).astype(F16)
    k = g.standard_normal((1, 1, 150, 128)).astype(F16)
    v = g.standard_normal((1, 1, 150, 128)).astype(F16)
    ref = oatt.attention_exact(q, k, v, 128 ** -0.5)
    for tile in (16, 128):
        got = oatt.attention_semantics(q, k, v, 128 ** -0.5, int8_qk=int8_qk, tile=tile)
        assert oatt.rel_l2(got, ref) < (1e-2 if int8_qk else 2e-3)


def test_attention_bmm_matches_exact():
    g = np.random.default_rng(11)
    q, k, v = (torch.from_numpy(g.standard_normal((1, 2, 40, 128)).astype(F16)) for _ in range(3))
    out = oatt.attention_bmm(q, k, v)
    assert oatt.rel_l2(out.numpy(), oatt.attention_exact(q.numpy(), k.numpy(), v.numpy(), 128 ** -0.5)) < 3e-3


def test_quant_rows_rint_is_half_even():
    x = np.zeros((1, 128), F16)
    x[0, 0] = 127
    x[0, 1] = 0.5
    x[0, 2] = 1.5
    x[0, 3] = -2.5
    q, s = oatt.quant_rows_rint(x)
    assert s[0] == 1.0 and q[0, :4].tolist() == [127, 0, 2, -2]

