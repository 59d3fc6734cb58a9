"""W4A8 (group-128) GEMM parity on the GPU against the specification oracle (oracle.gemm.w4a8_grouped): int32 per
group, F = fma(acc_g, s_g, F) in fp32, y = F * sa (+ bias) -> fp16. Compared bit for bit, for both kernels: the one
that widens the packed weight in shared memory and the one that reads a widened int8 copy; the configuration-3
linear (M=2809, K=3072, N=8192, block-128 rotated int8 activations) end to end."""
import numpy as np
import pytest
import torch

from oracle import gemm as ogemm
from oracle import quant as oq
from oracle import weights as ow

pytestmark = pytest.mark.gpu

F16 = np.float16
F32 = np.float32


def dev_(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def case(M, N, K, seed):
    g = np.random.default_rng(seed)
    w = (g.standard_normal((N, K)) * 0.02).astype(F32)
    packed, s16 = ow.quantize_int4_groups(w)
    a = g.integers(-127, 128, (M, K), dtype=np.int8)
    sa = (g.random(M) * 0.05 + 1e-3).astype(F32)
    bias = (g.standard_normal(N) * 0.01).astype(F16)
    return a, sa, packed, s16, bias


@pytest.mark.parametrize("wide", [False, True])
@pytest.mark.parametrize("M,N,K", [(1, 8, 128), (100, 136, 256), (257, 512, 1024), (128, 128, 3072), (1000, 264, 640),
                                   (300, 520, 384)])
def test_w4a8_matches_spec(pkg, dev, M, N, K, wide):
    a, sa, packed, s16, bias = case(M, N, K, M + N + K)
    gs = pkg.ops.w4a8_scales(dev_(s16, dev))
    wp = dev_(packed, dev)
    ww = pkg.ops.unpack_int4(wp) if wide else None
    for b in (None, bias):
        got = pkg.ops.gemm_w4a8(dev_(a, dev), dev_(sa, dev), wp, gs, None if b is None else dev_(b, dev), w_wide=ww)
        ref = ogemm.w4a8_grouped(a, sa, packed, s16, bias=b)
        assert np.array_equal(got.cpu().numpy(), ref)
    assert pkg._lib.device_status() == 0


def test_w4a8_extreme_nibbles(pkg, dev):
    M, N, K = 130, 128, 512
    a = np.full((M, K), -128, np.int8)
    packed = np.full((N, K // 2), 0x88, np.uint8)  # every weight -8
    packed[1] = 0x77                                  # every weight 7
    s16 = np.ones((N, K // 128), F16)
    sa = np.ones(M, F32)
    wp, gs = dev_(packed, dev), pkg.ops.w4a8_scales(dev_(s16, dev))
    ref = ogemm.w4a8_grouped(a, sa, packed, s16)
    for ww in (None, pkg.ops.unpack_int4(wp)):
        got = pkg.ops.gemm_w4a8(dev_(a, dev), dev_(sa, dev), wp, gs, w_wide=ww)
        assert np.array_equal(got.cpu().numpy(), ref)


def test_config3_linear(pkg, dev):
    """Configuration 3: X [2809, 3072] ~N(0,1) block-128 rotated, per-token int8; W [8192, 3072] int4 in [-8, 7]
    with fp16 scales per 128 along K (from an N(0, 0.02) weight rotated the same way)."""
    g = np.random.default_rng(3)
    M, K, N = 2809, 3072, 8192
    x = g.standard_normal((M, K)).astype(F16)
    w = (g.standard_normal((N, K)) * 0.02).astype(F32)
    packed, s16 = ow.quantize_int4_groups(ow.sylvester_rotate(w))
    q, s = pkg.ops.quant_pack_a(dev_(x, dev), 128)
    wp, gs = dev_(packed, dev), pkg.ops.w4a8_scales(dev_(s16, dev))
    got = pkg.ops.gemm_w4a8(q, s, wp, gs).cpu().numpy()
    got_wide = pkg.ops.gemm_w4a8(q, s, wp, gs, w_wide=pkg.ops.unpack_int4(wp)).cpu().numpy()
    q_ref, s_ref, _ = oq.prepass(x, 128)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    ref = ogemm.w4a8_grouped(q_ref, s_ref, packed, s16)
    assert np.array_equal(got, ref)
    assert np.array_equal(got_wide, ref)
    exact = x.astype(np.float64) @ w.T.astype(np.float64)
    assert np.linalg.norm(got - exact) / np.linalg.norm(exact) < 0.15  # int4 weight error, for scale


# ---------------------------------------------------------------- per-channel W4A4 (the reference's int4 form)
@pytest.mark.parametrize("rot", [0, 128, 256])
@pytest.mark.parametrize("M,K", [(1, 256), (77, 3072), (300, 1024)])
def test_int4_activations_bit_exact(pkg, dev, rot, M, K):
    """quant_row_i4 (int8_gemm.hip:62-91): scale = max(absmax, 1e-10) / 7, q = clamp(rint(y / scale), -7, 7)."""
    g = np.random.default_rng(M + K + rot)
    x = (g.standard_normal((M, K)) * 2).astype(F16)
    q, s = pkg.ops.quant_pack_a_i4(dev_(x, dev), rot)
    q_ref, s_ref = oq.quant_rows_i4(oq.rotate_rows(x, rot))
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)


def test_int4_activation_edges(pkg, dev):
    """Half-way quotients round to even, a NaN becomes -7, an all-zero row takes the 1e-10 floor, inf rows."""
    K = 256
    x = np.zeros((5, K), F16)
    x[0, :8] = [7, 3.5, 2.5, -2.5, 0.5, -0.5, 1.5, -6.5]   # scale 1: ties to even
    x[1] = np.linspace(-1, 1, K).astype(F16)
    x[1, 9] = np.nan
    x[3] = np.linspace(-3, 3, K).astype(F16)
    x[3, 4] = np.inf
    x[4, 100] = -65504
    for rot in (0, 256):
        q, s = pkg.ops.quant_pack_a_i4(dev_(x, dev), rot)
        q_ref, s_ref = oq.quant_rows_i4(oq.rotate_rows(x, rot))
        assert np.array_equal(s.cpu().numpy(), s_ref), rot
        assert np.array_equal(q.cpu().numpy(), q_ref), rot
    q, _ = pkg.ops.quant_pack_a_i4(dev_(x, dev), 0)
    assert q.cpu().numpy()[0, :8].tolist() == [7, 4, 2, -2, 0, 0, 2, -6]


@pytest.mark.parametrize("N,K", [(8, 32), (264, 3072), (4096, 1024)])
def test_unpack_int4_bit_exact(pkg, dev, N, K):
    packed = np.random.default_rng(N + K).integers(0, 256, (N, K // 2), dtype=np.uint8)
    got = pkg.ops.unpack_int4(dev_(packed, dev)).cpu().numpy()
    assert np.array_equal(got, ogemm.unpack_int4(packed))


@pytest.mark.parametrize("M,N,K", [(1, 8, 256), (130, 264, 1024), (1100, 3072, 3072)])
def test_w4a4_convrot_forward_bit_exact(pkg, dev, M, N, K):
    """convrot_w4a4_forward (int8_gemm.py:90-103): ConvRot-256 + int4-valued activations, packed int4 weights with
    per-channel scales, int32 over all of K, the W8A8 epilogue; against the oracle bit for bit."""
    g = np.random.default_rng(M + N)
    x = g.standard_normal((M, K)).astype(F16)
    packed = g.integers(0, 256, (N, K // 2), dtype=np.uint8)
    ws = (g.random(N) * 1e-2 + 1e-4).astype(F32)
    bias = (g.standard_normal(N) * 0.01).astype(F16)
    fwd = pkg.int8_gemm.wrap_w4a4(None)
    wide = pkg.ops.unpack_int4(dev_(packed, dev))  # the load-time int8 copy (qweight_unpacked)
    for b in (None, bias):
        q_ref, s_ref = oq.quant_rows_i4(oq.rotate_rows(x, 256))
        ref = ogemm.epilogue(ogemm.int_mm(q_ref, ogemm.unpack_int4(packed)), s_ref, ws, b)
        for unpacked in (None, wide):
            got = fwd(dev_(x, dev).view(1, M, K), dev_(packed, dev), dev_(ws, dev), None if b is None else dev_(b, dev),
                      256, torch.float16, qweight_unpacked=unpacked)
            assert got.shape == (1, M, N)
            assert np.array_equal(got.cpu().numpy().reshape(M, N), ref)
    with pytest.raises(NotImplementedError, match="qweight_unpacked"):
        fwd(dev_(x, dev), dev_(packed, dev), dev_(ws, dev), None, 256, torch.float16, qweight_unpacked=wide[:, :-16])
