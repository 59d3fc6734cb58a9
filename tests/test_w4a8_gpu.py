"""W4A8 (group-128) GEMM parity on the GPU against the specification oracle (oracle.gemm.w4a8_grouped): int32 per
group, F = fma(acc_g, s_g, F) in fp32, y = F * sa (+ bias) -> fp16. Compared bit for bit; the configuration-3 linear
(M=2809, K=3072, N=8192, block-128 rotated int8 activations) end to end."""
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


@pytest.mark.parametrize("M,N,K", [(1, 8, 128), (100, 136, 256), (257, 512, 1024), (128, 128, 3072), (1000, 264, 640)])
def test_w4a8_matches_spec(pkg, dev, M, N, K):
    a, sa, packed, s16, bias = case(M, N, K, M + N + K)
    gs = pkg.ops.w4a8_scales(dev_(s16, dev))
    for b in (None, bias):
        got = pkg.ops.gemm_w4a8(dev_(a, dev), dev_(sa, dev), dev_(packed, dev), gs, None if b is None else dev_(b, dev))
        ref = ogemm.w4a8_grouped(a, sa, packed, s16, bias=b)
        assert np.array_equal(got.cpu().numpy(), ref)


def test_w4a8_extreme_nibbles(pkg, dev):
    M, N, K = 130, 128, 512
    a = np.full((M, K), -128, np.int8)
    packed = np.full((N, K // 2), 0x88, np.uint8)  # every weight -8
    packed[1] = 0x77                                  # every weight 7
    s16 = np.ones((N, K // 128), F16)
    sa = np.ones(M, F32)
    got = pkg.ops.gemm_w4a8(dev_(a, dev), dev_(sa, dev), dev_(packed, dev), pkg.ops.w4a8_scales(dev_(s16, dev)))
    ref = ogemm.w4a8_grouped(a, sa, packed, s16)
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
    got = pkg.ops.gemm_w4a8(q, s, dev_(packed, dev), pkg.ops.w4a8_scales(dev_(s16, dev))).cpu().numpy()
    q_ref, s_ref, _ = oq.prepass(x, 128)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    ref = ogemm.w4a8_grouped(q_ref, s_ref, packed, s16)
    assert np.array_equal(got, ref)
    exact = x.astype(np.float64) @ w.T.astype(np.float64)
    assert np.linalg.norm(got - exact) / np.linalg.norm(exact) < 0.15  # int4 weight error, for scale
