"""The attention with the head-group gather fused into it (b2_attention_gather, b2_wait_count).

On one GPU the peers' buffers and counters are ordinary device buffers: the kernel's delivery must equal its own
output bit for bit, count one arrival per CTA on every counter, and leave the attention's result unchanged. The
configuration-4 stack sharded over 4 ranks, emulated in lockstep on one GPU with fused gathers (every rank's
attention of a block before any rank waits, so no kernel ever waits for a kernel that has not finished), must equal
the unsharded stack bit for bit. A wait whose count is never reached must return with its error flag set after its
time limit, leaving the GPU usable. With two or more GPUs, two processes exchange over the real peer mappings
(torch symmetric memory) and must match NCCL's all-gather bit for bit.
"""
import importlib
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _qkv(dev, B, H, T, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    return [torch.randn((B, H, T, 128), generator=g, device=dev).half() for _ in range(3)]


def test_gather_delivers_tiles_and_counts(pkg, dev):
    ops = pkg.ops
    B, H, T = 2, 3, 700
    q, k, v = _qkv(dev, B, H, T, 1)
    ref = torch.empty_like(q)
    ops.attention(q, k, v, ref, 128 ** -0.5)
    out = torch.empty_like(q)
    peers = [torch.zeros_like(q) for _ in range(3)]
    cnts = torch.zeros((3, 8), dtype=torch.int64, device=dev)
    ops.attention(q, k, v, out, 128 ** -0.5,
                  gather=([p.data_ptr() for p in peers], [cnts[i].data_ptr() for i in range(3)]))
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    for p in peers:
        assert torch.equal(p, ref)
    n = ops.attention_gather_ctas(B, H, T)
    assert n == ((T + 255) // 256) * B * H
    assert cnts[:, 0].tolist() == [n, n, n]
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.wait_count(cnts[0, :1], n, err)  # already reached: returns at once
    torch.cuda.synchronize()
    assert err.item() == 0 and pkg._lib.device_status() == 0


def test_wait_runs_out_and_reports(pkg, dev):
    """Nothing ever arrives: the wait gives up after 2 ms, sets the flag, and the stream goes on."""
    ops = pkg.ops
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.wait_count(cnt, 1, err, timeout_ns=2_000_000)
    after = torch.ones(4, device=dev) * 2
    torch.cuda.synchronize()
    assert err.item() == 1
    assert after.sum().item() == 8.0


def test_dit_fused_gather_lockstep_equals_unsharded(pkg, dev):
    dit = importlib.import_module(pkg.__name__ + ".dit")
    ops = pkg.ops
    cfg = dit.DiTConfig(hidden=512, heads=4, mlp=1024, blocks=3, tokens=300, batch=2)
    world = 4
    x0 = torch.randn((cfg.batch, cfg.tokens, cfg.hidden), generator=torch.Generator().manual_seed(7)).half().to(dev)
    full = dit.DiTStack(cfg, dit.shard_plan(1, 0, cfg.batch, cfg.heads), dev, seed=9)
    x_full = x0.clone()
    full.forward(x_full)

    plans = [dit.shard_plan(world, r, cfg.batch, cfg.heads) for r in range(world)]
    g, hl = plans[0].group_size, plans[0].head_hi - plans[0].head_lo
    bufs = [torch.zeros((2, g, 1, cfg.tokens, hl * 128), dtype=torch.float16, device=dev) for _ in range(world)]
    cnts = [torch.zeros(8, dtype=torch.int64, device=dev) for _ in range(world)]
    fgs = []
    for r, p in enumerate(plans):
        others = [rr for rr in p.group_ranks if rr != r]
        fgs.append(dit.FusedGather(bufs[r], [bufs[rr].data_ptr() for rr in others], cnts[r],
                                   [cnts[rr].data_ptr() for rr in others],
                                   torch.zeros(1, dtype=torch.int32, device=dev), p.group_index, timeout_ns=200_000_000))
    stacks = [dit.DiTStack(cfg, p, dev, seed=9, fused_gather=fgs[r]) for r, p in enumerate(plans)]
    xs = [x0[p.batch_lo:p.batch_hi].clone() for p in plans]
    nctas = ops.attention_gather_ctas(1, hl, cfg.tokens)
    for bi in range(cfg.blocks):
        par = bi % 2
        for r, st in enumerate(stacks):
            fg = fgs[r]
            seg, off = fg.segment(par)
            out = seg.view(1, cfg.tokens, hl, 128)
            st.attention_part(st.blocks[bi], xs[r], gather=(out, [a + off for a in fg.peer_buf], fg.peer_cnt))
        for r, st in enumerate(stacks):
            fg = fgs[r]
            fg.blocks_done += 1
            ops.wait_count(fg.cnt, fg.blocks_done * (g - 1) * nctas, fg.err, fg.timeout_ns)
            st.mlp_part(st.blocks[bi], xs[r], fg.buf[par], gathered=True)
    torch.cuda.synchronize()
    for r, p in enumerate(plans):
        assert not fgs[r].failed(), f"rank {r} wait ran out"
        assert torch.equal(xs[r], x_full[p.batch_lo:p.batch_hi]), f"rank {r}"
    assert pkg._lib.device_status() == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank, world, port, root, result):
    import datetime
    import sys

    import torch.distributed as dist

    sys.path.insert(0, root)
    import __graft_entry__

    pkg = __graft_entry__.load_package()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60), device_id=dev)
    dit = importlib.import_module(pkg.__name__ + ".dit")
    B, HL, T = 1, 6, 900
    q, k, v = _qkv(dev, B, HL, T, 100 + rank)
    att = torch.empty((B, T, HL, 128), dtype=torch.float16, device=dev)
    pkg.ops.attention(q, k, v, att.transpose(1, 2), 128 ** -0.5)
    ref = torch.empty((world, B, T, HL * 128), dtype=torch.float16, device=dev)
    dist.all_gather_into_tensor(ref.view(-1), att.view(-1))
    fg = dit.FusedGather.create(dist.group.WORLD, rank, world, B, T, HL * 128, dev)
    ok = True
    for it in range(3):  # both parities, and one reuse of the first
        par = it % 2
        seg, off = fg.segment(par)
        pkg.ops.attention(q, k, v, seg.view(B, T, HL, 128).transpose(1, 2), 128 ** -0.5,
                          gather=([a + off for a in fg.peer_buf], fg.peer_cnt))
        fg.blocks_done += 1
        pkg.ops.wait_count(fg.cnt, fg.blocks_done * (world - 1) * pkg.ops.attention_gather_ctas(B, HL, T), fg.err)
        torch.cuda.synchronize()
        ok = ok and not fg.failed() and torch.equal(fg.buf[par].view(world, B, T, HL * 128), ref)
        dist.barrier()
    flag = torch.tensor([int(ok)], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    result[rank] = int(flag.item())
    del fg
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_fused_gather_equals_nccl():
    import torch.multiprocessing as mp

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_two_rank_worker, args=(2, _free_port(), root, result), nprocs=2, join=True, start_method="spawn")
    assert dict(result) == {0: 1, 1: 1}
