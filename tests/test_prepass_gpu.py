"""Pre-pass parity on the GPU: int8 activations and fp32 scales bit-exact against the oracle (int8_gemm.hip
quant/rotation semantics). Stages with exp/rsqrt are checked to two fp16 steps, then bit-exact downstream of the
kernel's own fp16 activation."""
import numpy as np
import pytest
import torch

from oracle import quant as oq

pytestmark = pytest.mark.gpu

F16 = np.float16


def dev_(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def activations(M, K, seed, outliers=True):
    g = np.random.default_rng(seed)
    x = g.standard_normal((M, K)).astype(np.float32)
    if outliers:
        ch = g.choice(K, max(1, K // 100), replace=False)
        x[:, ch] *= 20
    return x.astype(F16)


SHAPES = [(1, 256), (7, 512), (64, 3072), (130, 1024), (33, 640), (5, 16384), (300, 8192)]


@pytest.mark.parametrize("rot", [0, 128, 256])
@pytest.mark.parametrize("M,K", SHAPES)
def test_quant_bit_exact(pkg, dev, rot, M, K):
    if rot and K % rot:
        pytest.skip("K not a multiple of the rotation group")
    x = activations(M, K, M * 7 + K)
    q, s = pkg.ops.quant_pack_a(dev_(x, dev), rot)
    q_ref, s_ref, _ = oq.prepass(x, rot)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)


@pytest.mark.parametrize("K", [256, 1024])
def test_quant_edge_values(pkg, dev, K):
    x = np.zeros((8, K), F16)
    x[1, :] = 65504                      # fp16 max: the rotation overflows fp16 to inf
    x[2, ::2] = 6e-8                     # subnormal fp16
    x[3, :8] = [127, 0.5, -0.5, 1.5, -1.5, 2.5, -2.5, -127]  # half-up ties with scale 1
    x[4] = np.linspace(-3, 3, K).astype(F16)
    x[5, 17] = -1
    x[6] = np.linspace(-1, 1, K).astype(F16)
    x[6, 130] = np.nan                   # NaN never wins the absmax and quantizes to -128
    x[7] = np.linspace(-2, 2, K).astype(F16)
    x[7, 5] = -np.inf
    for rot in (0, 128, 256):
        q, s = pkg.ops.quant_pack_a(dev_(x, dev), rot)
        q_ref, s_ref, _ = oq.prepass(x, rot)
        assert np.array_equal(s.cpu().numpy(), s_ref), rot
        assert np.array_equal(q.cpu().numpy(), q_ref), rot
    q, _ = pkg.ops.quant_pack_a(dev_(x, dev), 0)
    assert q.cpu().numpy()[3, :8].tolist() == [127, 1, 0, 2, -1, 3, -2, -127]


def test_quant_strided_rows(pkg, dev):
    big = activations(40, 1024, 3)
    x = dev_(big, dev)[:, 256:768]  # row stride 1024, 512 values per row
    q, s = pkg.ops.quant_pack_a(x, 256)
    q_ref, s_ref, _ = oq.prepass(big[:, 256:768], 256)
    assert np.array_equal(q.cpu().numpy(), q_ref) and np.array_equal(s.cpu().numpy(), s_ref)


def test_quant_gathered_segments(pkg, dev):
    # A row gathered from 4 per-rank segments [g, T, 384]: element k at (k // 384) * T * 384 + t * 384 + k % 384.
    g_, T, w = 4, 50, 384
    parts = activations(g_ * T, w, 4).reshape(g_, T, w)
    x = dev_(parts, dev)
    q, s = pkg.ops.quant_pack_a_segments(x, g_ * w, 128, w, T * w, T, w)
    full = parts.transpose(1, 0, 2).reshape(T, g_ * w)
    q_ref, s_ref, _ = oq.prepass(full, 128)
    assert np.array_equal(q.cpu().numpy(), q_ref) and np.array_equal(s.cpu().numpy(), s_ref)


def _check_act(pkg, dev, act16, ref16, q, s, rot, mag=None):
    # exp/rsqrt and the fp32 sum order differ from the oracle by an ulp; after the chained fp16 roundings of the
    # activation that is at most two fp16 steps of the largest intermediate (``mag``, default the result itself:
    # a final "+ t" can cancel most of an intermediate, so steps are measured at |y| + |t| there), on a small
    # fraction of the values.
    a = act16.cpu().numpy()
    diff = np.abs(a.astype(np.float32) - ref16.astype(np.float32))
    mag = np.abs(ref16.astype(np.float32)) if mag is None else mag
    ulp = np.abs(np.spacing(mag.astype(F16))).astype(np.float32)
    assert np.all(diff <= 2 * ulp), f"activation off by {np.max(diff / ulp)} fp16 steps"
    rate = np.mean(a != ref16)
    assert rate < 5e-3, f"{rate:.2e} of the activations differ"
    q_ref, s_ref = oq.quant_rows(oq.rotate_rows(a, rot))
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)


@pytest.mark.parametrize("rot", [0, 128, 256])
def test_swiglu_prepass(pkg, dev, rot):
    M, K = 97, 8192
    g = np.random.default_rng(11)
    gate = (g.standard_normal((M, K)) * 2).astype(F16)
    up = g.standard_normal((M, K)).astype(F16)
    act = torch.empty((M, K), dtype=torch.float16, device=dev)
    q, s = pkg.ops.swiglu_quant_pack_a(dev_(gate, dev), dev_(up, dev), rot, act_out=act)
    _check_act(pkg, dev, act, oq.swiglu(gate, up), q, s, rot)


@pytest.mark.parametrize("rot", [0, 128, 256])
def test_gate_prepass(pkg, dev, rot):
    M, K = 65, 3072
    g = np.random.default_rng(12)
    x = g.standard_normal((M, K)).astype(F16)
    gate = (g.standard_normal((M, K)) * 3).astype(F16)
    act = torch.empty((M, K), dtype=torch.float16, device=dev)
    q, s = pkg.ops.gate_quant_pack_a(dev_(x, dev), dev_(gate, dev), rot, act_out=act)
    _check_act(pkg, dev, act, oq.sigmoid_gate(x, gate), q, s, rot)


@pytest.mark.parametrize("rot", [0, 128, 256])
def test_mod_prepass(pkg, dev, rot):
    B, L, K = 2, 131, 3072
    g = np.random.default_rng(13)
    x = activations(B * L, K, 14)
    w = (g.standard_normal(K) * 0.02).astype(np.float32)
    s_rows = (1 + g.standard_normal((B, K)) * 0.1).astype(F16)
    t_rows = (g.standard_normal((B, K)) * 0.1).astype(F16)
    act = torch.empty((B * L, K), dtype=torch.float16, device=dev)
    q, s = pkg.ops.mod_quant_pack_a(dev_(x, dev), dev_(w, dev), dev_(s_rows, dev), dev_(t_rows, dev), L, 1e-6, rot,
                                    act_out=act)
    ref = oq.modulate(x, w, s_rows, t_rows, L, 1e-6)
    mag = np.abs(ref.astype(np.float32)) + np.abs(np.repeat(t_rows, L, axis=0).astype(np.float32))
    _check_act(pkg, dev, act, ref, q, s, rot, mag=mag)


@pytest.mark.parametrize("rot", [0, 128, 256])
@pytest.mark.parametrize("M,K", [(300, 3072), (33, 640)])
def test_mod_prepass_without_modulation(pkg, dev, rot, M, K):
    """The RMSNorm alone (scale and shift None, as the configuration-4 block uses it): the same int8 and scales, bit
    for bit, and the same activation, as modulation rows of ones and zeros; through the one-row-per-CTA kernel
    (K = 3072 under the block-128 rotation) and the warp-per-row kernel (the other cases)."""
    if rot and K % rot:
        pytest.skip("K not a multiple of the rotation group")
    g = np.random.default_rng(M + K + rot)
    x = (g.standard_normal((M, K)) * 2).astype(F16)
    x[3, :8] = 0  # zero activations: +0 and -0 must quantize alike
    w = (g.standard_normal(K) * 0.1).astype(np.float32)
    ones, zeros = torch.ones((1, K), dtype=torch.float16, device=dev), torch.zeros((1, K), dtype=torch.float16, device=dev)
    act_a = torch.empty((M, K), dtype=torch.float16, device=dev)
    act_b = torch.empty((M, K), dtype=torch.float16, device=dev)
    qa, sa = pkg.ops.mod_quant_pack_a(dev_(x, dev), dev_(w, dev), ones, zeros, M, 1e-6, rot, act_out=act_a)
    qb, sb = pkg.ops.mod_quant_pack_a(dev_(x, dev), dev_(w, dev), None, None, M, 1e-6, rot, act_out=act_b)
    assert torch.equal(qa, qb) and torch.equal(sa, sb)
    assert torch.equal(act_a, act_b)
    with pytest.raises(RuntimeError, match="both given or both None"):
        pkg.ops.mod_quant_pack_a(dev_(x, dev), dev_(w, dev), ones, None, M, 1e-6, rot)


@pytest.mark.parametrize("rot", [0, 128, 256])
@pytest.mark.parametrize("M,K", [(97, 3072), (33, 640)])
def test_situ_prepass(pkg, dev, rot, M, K):
    """situ on [hidden | gate] rows (int8_gemm.hip:118-127): the fp16 activation within two steps of the float32
    restatement (base-2 exponentials differ by an ulp), then int8 bit-exact from the kernel's own activation. Hidden
    values reach the soft cap (|h| up to ~100), gates cross the series branch of tanh (|g / 4| < 0.02)."""
    if rot and K % rot:
        pytest.skip("K not a multiple of the rotation group")
    g = np.random.default_rng(M + K)
    h = (g.standard_normal((M, K)) * 30).astype(F16)
    gt = (g.standard_normal((M, K)) * 3).astype(F16)
    gt[:, :64] = (g.standard_normal((M, 64)) * 0.02).astype(F16)
    x = np.concatenate([h, gt], axis=1)
    act = torch.empty((M, K), dtype=torch.float16, device=dev)
    q, s = pkg.ops.situ_quant_pack_a(dev_(x, dev), rot, act_out=act)
    _check_act(pkg, dev, act, oq.situ(h, gt), q, s, rot)


def test_situ_linear_drop_in(pkg, dev):
    """int8_gemm.linear(situ=True): [hidden | gate] rows -> situ -> ConvRot -> int8 -> GEMM, bit-exact against the
    oracle's pre-pass of the kernel's activation and the epilogue restatement."""
    from oracle import gemm as ogemm

    M, K, N = 130, 1024, 264
    g = np.random.default_rng(21)
    x = np.concatenate([(g.standard_normal((M, K)) * 10).astype(F16), g.standard_normal((M, K)).astype(F16)], axis=1)
    wq = g.integers(-127, 128, (N, K), dtype=np.int8)
    ws = (g.random(N) * 1e-3).astype(np.float32)
    y = pkg.int8_gemm.linear(dev_(x, dev), dev_(wq, dev), dev_(ws, dev), None, situ=True).cpu().numpy()
    act = torch.empty((M, K), dtype=torch.float16, device=dev)
    pkg.ops.situ_quant_pack_a(dev_(x, dev), 256, act_out=act)
    q_ref, s_ref = oq.quant_rows(oq.rotate_rows(act.cpu().numpy(), 256))
    assert np.array_equal(y, ogemm.epilogue(ogemm.int_mm(q_ref, wq), s_ref, ws))
