"""W8A8 GEMM parity on the GPU: int32 accumulators bit-exact (int_mm), fp16 epilogue bit-exact against the oracle's
IEEE restatement of int8_gemm.hip:371-405, and the full configuration-1 linear end to end."""
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


def rand_i8(shape, seed):
    return np.random.default_rng(seed).integers(-128, 128, shape, dtype=np.int8)


# The last three have at least 74 tiles of 256 x 256 and run on the CTA-pair kernel (ragged in M and N).
SHAPES = [(1, 8, 16), (100, 136, 112), (129, 264, 3072), (1000, 256, 256), (300, 520, 160), (128, 256, 128),
          (257, 1024, 2048), (6642, 256, 3072), (64, 9216, 512), (2048, 2560, 512), (2000, 2600, 384),
          (6642, 9216, 3072)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_int32_accumulators_bit_exact(pkg, dev, M, N, K):
    a, b = rand_i8((M, K), M + K), rand_i8((N, K), N * 3 + K)
    got = pkg.ops.gemm_i32(dev_(a, dev), dev_(b, dev)).cpu().numpy()
    assert np.array_equal(got, ogemm.int_mm(a, b))


def test_int32_extremes(pkg, dev):
    # All -128: the largest accumulator magnitude (K * 16384) stays exact in int32.
    M, N, K = 130, 72, 4096
    a = np.full((M, K), -128, np.int8)
    b = np.full((N, K), -128, np.int8)
    b[1] = 127
    got = pkg.ops.gemm_i32(dev_(a, dev), dev_(b, dev)).cpu().numpy()
    assert np.array_equal(got, ogemm.int_mm(a, b))


@pytest.mark.parametrize("M,N,K", [(77, 264, 384), (1024, 3072, 3072), (513, 128, 8192), (2049, 2568, 512),
                                   (1100, 2600, 384)])
def test_epilogue_bit_exact(pkg, dev, M, N, K):
    g = np.random.default_rng(M)
    a, b = rand_i8((M, K), 1), rand_i8((N, K), 2)
    sa = (g.random(M) * 0.05 + 1e-3).astype(F32)
    sw = (g.random(N) * 1e-3 + 1e-5).astype(F32)
    bias = (g.standard_normal(N) * 0.01).astype(F16)
    acc = ogemm.int_mm(a, b)
    for with_bias in (False, True):
        bb = bias if with_bias else None
        got = pkg.ops.gemm(dev_(a, dev), dev_(sa, dev), dev_(b, dev), dev_(sw, dev), None if bb is None else dev_(bb, dev))
        assert np.array_equal(got.cpu().numpy(), ogemm.epilogue(acc, sa, sw, bb))


@pytest.mark.parametrize("B,L,N,K", [(2, 150, 264, 512), (2, 1100, 2816, 256)])
def test_residual_epilogue_bit_exact(pkg, dev, B, L, N, K):
    M = B * L
    g = np.random.default_rng(5)
    a, b = rand_i8((M, K), 3), rand_i8((N, K), 4)
    sa = (g.random(M) * 0.05).astype(F32)
    sw = (g.random(N) * 1e-3).astype(F32)
    R = g.standard_normal((M, N)).astype(F16)
    G = g.standard_normal((B, N)).astype(F16)
    got = pkg.ops.gemm(dev_(a, dev), dev_(sa, dev), dev_(b, dev), dev_(sw, dev), residual=dev_(R, dev), gate=dev_(G, dev), L=L)
    ref = ogemm.epilogue(ogemm.int_mm(a, b), sa, sw, R=R, G=G, L=L)
    assert np.array_equal(got.cpu().numpy(), ref)
    # No gate: R + y, bit for bit the gate of ones (fp16(1 * y) = y), through the 1-CTA (M = 300) and pair kernels.
    ones = np.ones((1, N), F16)
    got1 = pkg.ops.gemm(dev_(a, dev), dev_(sa, dev), dev_(b, dev), dev_(sw, dev), residual=dev_(R, dev))
    assert np.array_equal(got1.cpu().numpy(), ogemm.epilogue(ogemm.int_mm(a, b), sa, sw, R=R, G=ones, L=M))


@pytest.mark.parametrize("rot", [128, 256])
def test_config1_linear_end_to_end(pkg, dev, rot):
    """Configuration 1: X [1024, 3072] ~N(0,1) with 1% outlier channels x20, W [3072, 3072] ~N(0, 0.02), bias
    ~N(0, 0.01); both rotated along K; per-channel int8 weights (half-even), per-token int8 activations."""
    g = np.random.default_rng(0)
    M, K, N = 1024, 3072, 3072
    x = g.standard_normal((M, K)).astype(F32)
    x[:, g.choice(K, K // 100, replace=False)] *= 20
    x = x.astype(F16)
    w = (g.standard_normal((N, K)) * 0.02).astype(F32)
    bias = (g.standard_normal(N) * 0.01).astype(F16)
    wr = ow.sylvester_rotate(w) if rot == 128 else ow.convrot_rotate(w)
    wq, ws = ow.quantize_per_channel(wr)
    y = pkg.int8_gemm.linear(dev_(x, dev), dev_(wq, dev), dev_(ws, dev), dev_(bias, dev), rotate=True, rot_group=rot)
    q_ref, s_ref, _ = oq.prepass(x, rot)
    ref = ogemm.epilogue(ogemm.int_mm(q_ref, wq), s_ref, ws, bias)
    got = y.cpu().numpy()
    assert np.array_equal(got, ref)
    exact = x.astype(np.float64) @ w.T.astype(np.float64) + bias.astype(np.float64)
    rel = np.linalg.norm(got.astype(np.float64) - exact) / np.linalg.norm(exact)
    assert rel < 3e-2  # W8A8 quantization error with outliers, for scale


@pytest.mark.parametrize("M,F,K", [(300, 1024, 384), (2049, 2048, 512)])
def test_swiglu_epilogue_matches_gemm_then_prepass(pkg, dev, M, F, K):
    """The SwiGLU epilogue (gate/up rows interleaved in blocks of 128) equals the plain GEMM followed by the SwiGLU
    pre-pass's activation bit for bit (F % 1024 == 0: the pre-pass kernel with the same SwiGLU arithmetic), on the
    single-CTA (300 rows) and CTA-pair (2049 rows) kernels."""
    a, b = rand_i8((M, K), 7), rand_i8((2 * F, K), 8)
    g = np.random.default_rng(9)
    sa = (g.random(M) * 0.05 + 1e-3).astype(F32)
    sw = (g.random(2 * F) * 2e-3 + 1e-5).astype(F32)
    A, Bw, SA, SW = dev_(a, dev), dev_(b, dev), dev_(sa, dev), dev_(sw, dev)
    gu = pkg.ops.gemm(A, SA, Bw, SW)
    act = torch.empty((M, F), dtype=torch.float16, device=dev)
    pkg.ops.swiglu_quant_pack_a(gu[:, :F].contiguous(), gu[:, F:].contiguous(), 128, act_out=act)
    perm = pkg.ops.swiglu_interleave(2 * F, dev)
    fused = pkg.ops.gemm_swiglu(A, SA, Bw.index_select(0, perm).contiguous(), SW.index_select(0, perm).contiguous())
    assert torch.equal(fused, act)
