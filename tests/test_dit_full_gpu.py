"""The configuration-4 DiT stack at its full size, stage by stage against the oracle.

The benchmark times 8 blocks of hidden 3072, 24 heads of 128, MLP 8192 on 2 CFG branches of 3321 tokens. Here that
exact stack runs on the GPU, and each of its 9 stages in every block is checked on sampled rows, fed with the GPU's
own input to that stage (so an error cannot hide behind the previous stage's tolerance):

  norm1 / norm2   RMSNorm + block-128 rotation + int8 (mod pre-pass): the fp16 activation (recomputed by the same
                  kernel on the sampled rows) within two fp16 steps of the oracle; int8 and scales bit-exact from it
  qkv, out_proj,  int32 GEMM + fp16 epilogue (residual for out_proj and down): bit-exact
  down
  attention       2 heads x 121 query rows per branch against all 3321 keys: relative L2 within 1e-3 of the
                  kernel-semantics oracle (fp16 P, lazy warp-uniform rescale), 2e-3 of float64
  out_prepass,    rotation + int8 of the GPU's attention output / SwiGLU activation: bit-exact
  down_prepass
  gate_up         GEMM whose epilogue applies the SwiGLU: within two fp16 steps of the oracle's GEMM + swiglu

Sampled query rows are whole 32-row groups (the attention kernel's rescale unit): the first rows, two inner groups
(one across the image/text boundary at token 2809) and the ragged last group of 25 rows.
"""
import importlib

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import gemm as ogemm
from oracle import quant as oq

pytestmark = pytest.mark.gpu

F16 = np.float16
F32 = np.float32
ROW_GROUPS = [(0, 32), (1376, 1408), (2784, 2816), (3296, 3321)]
HEADS = [0, 23]


def cpu(t):
    return t.detach().cpu().numpy()


def within_two_steps(got, ref, what, rate_max=5e-3):
    diff = np.abs(got.astype(F32) - ref.astype(F32))
    ulp = np.abs(np.spacing(np.abs(ref.astype(F32)).astype(F16))).astype(F32)
    assert np.all(diff <= 2 * ulp), f"{what}: off by {np.max(diff / ulp)} fp16 steps"
    rate = np.mean(got != ref)
    assert rate < rate_max, f"{what}: {rate:.2e} of the values differ"


def test_dit_full_config_stage_parity(pkg, dev):
    dit = importlib.import_module(pkg.__name__ + ".dit")
    ops = pkg.ops
    cfg = dit.DiTConfig()
    assert (cfg.blocks, cfg.hidden, cfg.heads, cfg.mlp, cfg.batch, cfg.tokens) == (8, 3072, 24, 8192, 2, 3321)
    T, D, F, H, hd = cfg.tokens, cfg.hidden, cfg.mlp, cfg.heads, cfg.head_dim
    stack = dit.DiTStack(cfg, dit.shard_plan(1, 0, cfg.batch, cfg.heads), dev, seed=7)
    x = torch.randn((cfg.batch, T, D), generator=torch.Generator().manual_seed(17)).half().to(dev)

    local = np.concatenate([np.arange(a, b) for a, b in ROW_GROUPS])
    rows = np.concatenate([b * T + local for b in range(cfg.batch)])
    rows_d = torch.from_numpy(rows).to(dev)
    n = rows.size
    seen = {}

    def probe(stage, *ts):
        if stage == "qkv":
            qkv = ts[0].view(cfg.batch, T, 3, H, hd)
            seen["qkv"] = cpu(ts[0].index_select(0, rows_d))
            # all keys and values of the sampled heads, [B, T, head, 128]
            seen["kv"] = (cpu(qkv[:, :, 1, HEADS]), cpu(qkv[:, :, 2, HEADS]))
        elif stage == "attention":
            seen["attention"] = cpu(ts[0].reshape(cfg.batch * T, D).index_select(0, rows_d))
        elif stage == "norm1":
            seen["x_in"] = ts[0].index_select(0, rows_d).clone()
            seen["norm1"] = (cpu(ts[1].index_select(0, rows_d)), cpu(ts[2].index_select(0, rows_d)))
        else:
            seen[stage] = tuple(cpu(t.index_select(0, rows_d)) for t in ts)

    stack.probe = probe
    ones_s = torch.ones((n, D), dtype=torch.float16, device=dev)
    zeros_s = torch.zeros((n, D), dtype=torch.float16, device=dev)
    ones_np = np.ones((n, D), F16)

    def check_norm(x_rows, norm_w, q8, sa, what):
        # The mod pre-pass is row-independent: the same kernel on the sampled rows alone gives the same int8 and
        # scales, and exposes its fp16 activation.
        act = torch.empty((n, D), dtype=torch.float16, device=dev)
        q_s, s_s = ops.mod_quant_pack_a(x_rows, norm_w, ones_s, zeros_s, 1, cfg.eps, cfg.rot_group, act_out=act)
        assert np.array_equal(cpu(q_s), q8) and np.array_equal(cpu(s_s), sa), f"{what}: not row-independent"
        a = cpu(act)
        ref = oq.modulate(cpu(x_rows), cpu(norm_w), ones_np, np.zeros((n, D), F16), 1, cfg.eps)
        within_two_steps(a, ref, what)
        q_ref, s_ref = oq.quant_rows(oq.rotate_rows(a, cfg.rot_group))
        assert np.array_equal(s_ref, sa) and np.array_equal(q_ref, q8), f"{what}: int8 from the activation"

    for bi, blk in enumerate(stack.blocks):
        seen.clear()
        stack.block(blk, x)
        torch.cuda.synchronize()
        tag = f"block {bi}"
        x_in = seen["x_in"]
        x_in_np = cpu(x_in)

        q8, sa = seen["norm1"]
        check_norm(x_in, blk.norm1, q8, sa, f"{tag} norm1")
        qkv_ref = ogemm.epilogue(ogemm.int_mm(q8, cpu(blk.w_qkv)), sa, cpu(blk.s_qkv))
        assert np.array_equal(seen["qkv"], qkv_ref), f"{tag} qkv"

        k_all, v_all = seen["kv"]
        att = seen["attention"].reshape(cfg.batch, local.size, H, hd)
        q_rows = seen["qkv"].reshape(cfg.batch, local.size, 3, H, hd)[:, :, 0]
        for hi, h in enumerate(HEADS):
            for b in range(cfg.batch):
                qh = q_rows[b, :, h][None, None]
                kh, vh = k_all[b, :, hi][None, None], v_all[b, :, hi][None, None]
                got = att[b, :, h][None, None]
                sem = oatt.attention_semantics(qh, kh, vh, hd ** -0.5, tile=128)
                assert oatt.rel_l2(got, sem) < 1e-3, f"{tag} attention head {h} branch {b} vs semantics"
                assert oatt.rel_l2(got, oatt.attention_exact(qh, kh, vh, hd ** -0.5)) < 2e-3, f"{tag} head {h}"

        q8, sa = seen["out_prepass"]
        q_ref, s_ref = oq.quant_rows(oq.rotate_rows(seen["attention"], cfg.rot_group))
        assert np.array_equal(s_ref, sa) and np.array_equal(q_ref, q8), f"{tag} out-proj pre-pass"
        xa = seen["out_proj"][0]
        xa_ref = ogemm.epilogue(ogemm.int_mm(q8, cpu(blk.w_o)), sa, cpu(blk.s_o), R=x_in_np, G=ones_np, L=1)
        assert np.array_equal(xa, xa_ref), f"{tag} out-proj + residual"

        q8, sa = seen["norm2"]
        check_norm(torch.from_numpy(xa).to(dev), blk.norm2, q8, sa, f"{tag} norm2")
        inv = np.argsort(cpu(blk.gu_perm))
        gu = ogemm.epilogue(ogemm.int_mm(q8, cpu(blk.w_gu)[inv]), sa, cpu(blk.s_gu)[inv])
        act = seen["gate_up"][0]
        within_two_steps(act, oq.swiglu(gu[:, :F], gu[:, F:]), f"{tag} gate/up + SwiGLU")

        q8, sa = seen["down_prepass"]
        q_ref, s_ref = oq.quant_rows(oq.rotate_rows(act, cfg.rot_group))
        assert np.array_equal(s_ref, sa) and np.array_equal(q_ref, q8), f"{tag} down pre-pass"
        out_ref = ogemm.epilogue(ogemm.int_mm(q8, cpu(blk.w_down)), sa, cpu(blk.s_down), R=xa, G=ones_np, L=1)
        assert np.array_equal(seen["down"][0], out_ref), f"{tag} down + residual"
        assert np.isfinite(seen["down"][0].astype(F32)).all()
    assert pkg._lib.device_status() == 0
