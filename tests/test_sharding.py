"""Multi-rank host logic of the DiT sharding on CPU (gloo, world sizes 2 and 4): the shard plans cover every
(CFG branch, head) pair exactly once, the QKV row selection picks each head's q/k/v rows, and an all-gather of
per-rank attention outputs, read through the pre-pass's segment addressing, reassembles the full [T, H*128] rows.
No CUDA is used; the segment read is emulated with the same index formula the kernel uses."""
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _dit():
    import __graft_entry__

    pkg = __graft_entry__.load_package()
    return importlib.import_module(pkg.__name__ + ".dit")


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plans_cover_branches_and_heads_once(world):
    dit = _dit()
    seen = np.zeros((2, 24), int)
    for r in range(world):
        p = dit.shard_plan(world, r, 2, 24)
        seen[p.batch_lo:p.batch_hi, p.head_lo:p.head_hi] += 1
        assert r in p.group_ranks
        assert all(dit.shard_plan(world, q, 2, 24).head_lo != p.head_lo or q == r for q in p.group_ranks)
    assert (seen == 1).all()


def test_qkv_rows_select_each_heads_projection():
    dit = _dit()
    cfg = dit.DiTConfig(heads=4, hidden=512)
    rows = dit.qkv_rows(cfg, 1, 3).numpy()
    assert rows.tolist() == list(range(128, 384)) + list(range(640, 896)) + list(range(1152, 1408))


def test_bad_splits_are_refused():
    dit = _dit()
    with pytest.raises(ValueError):
        dit.shard_plan(3, 0, 2, 24)
    with pytest.raises(ValueError):
        dit.shard_plan(10, 0, 2, 24)


def segment_read(flat, M, K, seg, seg_stride, ldx):
    """Row m, element k at m*ldx + (k // seg) * seg_stride + k % seg (prepass.cu, b2_quant_pack_a_seg)."""
    m = np.arange(M)[:, None]
    k = np.arange(K)[None, :]
    return flat[m * ldx + (k // seg) * seg_stride + k % seg]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dit = _dit()
        B, H, T, D = 2, 8, 6, 8 * 128
        plan = dit.shard_plan(world, rank, B, H)
        groups = {}
        for r in range(world):
            gr = dit.shard_plan(world, r, B, H).group_ranks
            if gr not in groups:
                groups[gr] = dist.new_group(list(gr)) if len(gr) > 1 else None
        b = plan.batch_hi - plan.batch_lo
        hl = plan.head_hi - plan.head_lo
        # Attention output of this rank's heads, [b, T, hl, 128]; value encodes (batch, token, head, dim).
        bi, ti, hi, di = np.meshgrid(np.arange(plan.batch_lo, plan.batch_hi), np.arange(T),
                                     np.arange(plan.head_lo, plan.head_hi), np.arange(128), indexing="ij")
        att = torch.from_numpy((bi * 1e6 + ti * 1e4 + hi * 1e2 + di % 97).astype(np.float64))
        g = plan.group_size
        if g > 1:
            gathered = torch.empty((g * att.numel(),), dtype=att.dtype)
            dist.all_gather_into_tensor(gathered, att.reshape(-1), group=groups[plan.group_ranks])
            w = hl * 128
            rows = segment_read(gathered.numpy(), b * T, D, w, b * T * w, w)
        else:
            rows = att.numpy().reshape(b * T, D)
        bi, ti, hi, di = np.meshgrid(np.arange(plan.batch_lo, plan.batch_hi), np.arange(T), np.arange(H),
                                     np.arange(128), indexing="ij")
        want = (bi * 1e6 + ti * 1e4 + hi * 1e2 + di % 97).reshape(b * T, D)
        out[rank] = bool(np.array_equal(rows, want))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_gather_reassembles_rows_over_gloo(world):
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    assert dict(out) == {r: True for r in range(world)}
