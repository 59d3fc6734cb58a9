"""Stack of W8A8 DiT blocks (benchmark configuration 4) on the sm_100a kernels, sharded over GPUs.

Block (per the configuration): x += out_proj(attention(qkv(rotate(RMSNorm(x))))); x += down(SwiGLU(gate_up(
rotate(RMSNorm(x))))), every linear W8A8 with per-channel int8 weights, block-128 Hadamard rotation on both sides,
fp16 attention with 24 heads of 128. On the device one block is 9 launches:
  mod pre-pass (RMSNorm + rotation + int8) -> QKV GEMM -> attention (reads Q/K/V as strided views of the QKV
  output) -> pre-pass -> out-proj GEMM with the residual in its epilogue -> mod pre-pass -> gate|up GEMM (one
  N = 2 x 8192 GEMM whose epilogue applies the SwiGLU and writes the 8192-wide activation: its weight rows are
  interleaved in blocks of 128) -> pre-pass -> down GEMM with the residual. The configuration fuses the SwiGLU into
  the down projection's pre-pass; here it moves one kernel earlier, with the same fp16 arithmetic, which halves the
  activation written to and read back from HBM.
The reference's fused Krea-2 block (int8_gemm.py:189-226) has the same shape with modulation and gates; this is the
configuration's simplified form.

Sharding (one process per GPU): the two CFG branches split first; within a branch, heads split into groups. A GPU
computes the QKV rows and the attention of its heads, the head group's attention outputs are assembled on every GPU
of the group (the out-proj pre-pass reads the gathered [g, T, w] buffer in place through its segment mode), and the
out-projection and MLP run replicated inside the group. That exchange is the only collective. It is either an NCCL
all-gather after the attention, or fused into the attention (FusedGather): each CTA copies its finished output tile
into the group's peers' gathered buffers (symmetric memory) and counts its arrival there, and a stream-ordered
bounded wait on the local counter precedes the out-projection, so the transfer overlaps the attention's compute.
"""
import contextlib
import dataclasses

import torch

from . import ops


@dataclasses.dataclass
class DiTConfig:
    hidden: int = 3072
    heads: int = 24
    head_dim: int = 128
    mlp: int = 8192
    blocks: int = 8
    eps: float = 1e-6
    rot_group: int = 128
    batch: int = 2          # CFG branches
    tokens: int = 3321      # 2809 image + 512 text


@dataclasses.dataclass
class ShardPlan:
    """Which CFG branches and heads a rank computes, and which ranks share its heads' all-gather."""
    world: int
    rank: int
    batch_lo: int
    batch_hi: int
    head_lo: int
    head_hi: int
    group_ranks: tuple

    @property
    def group_size(self):
        return len(self.group_ranks)

    @property
    def group_index(self):
        return self.group_ranks.index(self.rank)


def shard_plan(world, rank, batch, heads):
    """world 1: everything; world <= batch: branches split; world = batch * g: g head groups per branch."""
    if world <= batch:
        if batch % world:
            raise ValueError(f"{batch} CFG branches do not split over {world} GPUs")
        per = batch // world
        return ShardPlan(world, rank, rank * per, (rank + 1) * per, 0, heads, (rank,))
    if world % batch:
        raise ValueError(f"{world} GPUs do not split into {batch} CFG branches")
    groups = world // batch
    if heads % groups:
        raise ValueError(f"{heads} heads do not split into {groups} groups")
    branch, gi = divmod(rank, groups)
    hp = heads // groups
    ranks = tuple(branch * groups + i for i in range(groups))
    return ShardPlan(world, rank, branch, branch + 1, gi * hp, (gi + 1) * hp, ranks)


def qkv_rows(cfg, head_lo, head_hi):
    """Rows of the [3 * heads * 128, hidden] QKV weight that produce q, k and v of heads [head_lo, head_hi)."""
    d = cfg.head_dim
    idx = []
    for part in range(3):
        base = part * cfg.heads * d
        idx.extend(range(base + head_lo * d, base + head_hi * d))
    return torch.tensor(idx, dtype=torch.long)


def hadamard128(device):
    """Normalised Sylvester Hadamard of order 128 (fp32), used to rotate weights along K."""
    h = torch.ones((1, 1), dtype=torch.float64)
    for _ in range(7):
        h = torch.cat((torch.cat((h, h), 1), torch.cat((h, -h), 1)), 0)
    return (h / 128 ** 0.5).to(torch.float32).to(device)


def quantize_weight(w, h128):
    """Rotate rows along K by the block-128 Hadamard, then per-output-channel int8 (absmax / 127, half-even)."""
    N, K = w.shape
    wr = (w.float().reshape(N, K // 128, 128) @ h128.t()).reshape(N, K)
    scale = wr.abs().amax(dim=1) / 127.0
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    q = torch.round(wr / scale[:, None]).clamp_(-127, 127).to(torch.int8)
    return q.contiguous(), scale.float().contiguous()


class DiTBlock:
    def __init__(self, cfg, plan, device, seed):
        gen = torch.Generator(device=device).manual_seed(seed)
        D, F = cfg.hidden, cfg.mlp
        h128 = hadamard128(device)

        def weight(n, k):
            return quantize_weight(torch.randn((n, k), generator=gen, device=device, dtype=torch.float32) * 0.02, h128)

        w_qkv, s_qkv = weight(3 * cfg.heads * cfg.head_dim, D)
        rows = qkv_rows(cfg, plan.head_lo, plan.head_hi).to(device)
        self.w_qkv, self.s_qkv = w_qkv.index_select(0, rows).contiguous(), s_qkv.index_select(0, rows).contiguous()
        self.w_o, self.s_o = weight(D, D)
        # Gate and up rows interleaved in blocks of 128 (gu_perm[i] = natural row of stored row i), so that the
        # gate/up GEMM applies the SwiGLU in its epilogue.
        w_gu, s_gu = weight(2 * F, D)
        self.gu_perm = ops.swiglu_interleave(2 * F, device)
        self.w_gu, self.s_gu = w_gu.index_select(0, self.gu_perm).contiguous(), s_gu.index_select(0, self.gu_perm).contiguous()
        del w_gu, s_gu
        self.w_down, self.s_down = weight(D, F)
        self.norm1 = (torch.randn(D, generator=gen, device=device) * 0.02).float()
        self.norm2 = (torch.randn(D, generator=gen, device=device) * 0.02).float()
        del w_qkv, s_qkv


class FusedGather:
    """Buffers of the fused head-group gather on one rank: ``buf`` [2, g, b, T, w] fp16 (double-buffered by block
    parity), its peers' copies at ``peer_buf`` (device addresses, one per other rank of the group, in group order),
    an int64 arrival counter ``cnt`` and its peers' counters ``peer_cnt``, and an int32 error flag set by a wait
    that runs out. Counters only grow: after n blocks this rank expects n * (g - 1) * (CTAs per launch) arrivals.

    Reuse is safe without further synchronization: a rank writes block i + 2's tiles into a peer's buffer of parity
    i % 2 only after its own wait for block i + 1, i.e. after every peer finished block i + 1's attention, which
    each peer's stream orders after its block-i out-projection pre-pass, the last reader of that buffer."""

    def __init__(self, buf, peer_buf, cnt, peer_cnt, err, index, timeout_ns=2_000_000_000):
        self.buf, self.peer_buf, self.cnt, self.peer_cnt, self.err = buf, list(peer_buf), cnt, list(peer_cnt), err
        self.index, self.timeout_ns = index, timeout_ns
        self.blocks_done = 0
        self.g = buf.shape[1]

    @classmethod
    def create(cls, group, group_index, g, b, T, w, device):
        """Allocates the buffers in torch symmetric memory and exchanges their addresses inside ``group``."""
        import torch.distributed._symmetric_memory as symm_mem

        buf = symm_mem.empty((2, g, b, T, w), dtype=torch.float16, device=device)
        cnt = symm_mem.empty((8,), dtype=torch.int64, device=device)
        cnt.zero_()
        torch.cuda.synchronize(device)
        hb = symm_mem.rendezvous(buf, group.group_name)
        hc = symm_mem.rendezvous(cnt, group.group_name)
        peers = [p for p in range(g) if p != group_index]
        err = torch.zeros((1,), dtype=torch.int32, device=device)
        fg = cls(buf, [hb.buffer_ptrs[p] for p in peers], cnt, [hc.buffer_ptrs[p] for p in peers], err, group_index)
        fg._handles = (hb, hc)  # keep the mappings alive
        return fg

    def segment(self, par):
        """This rank's [b, T, w] segment of the parity-`par` buffer, and its byte offset."""
        seg = self.buf[par, self.index]
        return seg, (par * self.g + self.index) * seg.numel() * seg.element_size()

    def failed(self):
        return bool(self.err.item())


class DiTStack:
    """Runs ``cfg.blocks`` blocks on this rank's share. ``all_gather(out, inp)`` gathers [g * n] from [n] inside the
    rank's head group (torch.distributed.all_gather_into_tensor in production)."""

    def __init__(self, cfg, plan, device, seed=0, all_gather=None, timer=None, fused_gather=None):
        self.cfg, self.plan, self.device = cfg, plan, device
        self.fused = fused_gather
        self.timer = timer or (lambda kind, work=0: contextlib.nullcontext())
        # probe(stage, *tensors), when set, sees each stage's outputs before the next stage overwrites the buffers
        # they live in (parity tests read sampled rows from them); it adds no launches when unset.
        self.probe = None
        self.blocks = [DiTBlock(cfg, plan, device, seed * 1000 + i) for i in range(cfg.blocks)]
        self.all_gather = all_gather
        b = plan.batch_hi - plan.batch_lo
        M, D, F = b * cfg.tokens, cfg.hidden, cfg.mlp
        hl = plan.head_hi - plan.head_lo
        self.hl = hl
        # Buffers are allocated once and reused by every block and step (graph-capturable).
        dev = device
        self.q8 = torch.empty((M * max(D, F),), dtype=torch.int8, device=dev)
        self.sa = torch.empty((M,), dtype=torch.float32, device=dev)
        self.qkv = torch.empty((M, 3 * hl * cfg.head_dim), dtype=torch.float16, device=dev)
        self.att = torch.empty((b, cfg.tokens, hl, cfg.head_dim), dtype=torch.float16, device=dev)
        g = plan.group_size
        self.gathered = torch.empty((g, b, cfg.tokens, hl * cfg.head_dim), dtype=torch.float16, device=dev) if g > 1 else None
        self.act = torch.empty((M, F), dtype=torch.float16, device=dev)
        self.xa = torch.empty((M, D), dtype=torch.float16, device=dev)

    def attention_part(self, blk, x, gather=None):
        """RMSNorm -> QKV of this rank's heads -> attention. x [b, T, D] fp16; returns att [b, T, hl, 128]. With
        ``gather`` = (output [b, T, hl, 128], peer addresses, peer counters) the attention writes there and also
        delivers each tile to the peers (ops.attention's gather)."""
        cfg, hl, t = self.cfg, self.hl, self.timer
        b, T, D = x.shape
        M = b * T
        q8 = self.q8[:M * D].view(M, D)
        with t("prepass"):
            ops.mod_quant_pack_a(x.view(M, D), blk.norm1, None, None, T, cfg.eps, cfg.rot_group, out=(q8, self.sa))
        if self.probe:
            self.probe("norm1", x.view(M, D), q8, self.sa)
        with t("gemm", 2 * M * D * self.qkv.shape[1]):
            ops.gemm(q8, self.sa, blk.w_qkv, blk.s_qkv, out=self.qkv)
        if self.probe:
            self.probe("qkv", self.qkv)
        qkv = self.qkv.view(b, T, 3, hl, cfg.head_dim)
        q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))
        att = self.att if gather is None else gather[0]
        with t("attention", 4 * b * hl * T * T * cfg.head_dim):
            ops.attention(q, k, v, att.transpose(1, 2), cfg.head_dim ** -0.5,
                          gather=None if gather is None else gather[1:])
        if self.probe:
            self.probe("attention", att)
        return att

    def mlp_part(self, blk, x, att, gathered=False):
        """Out-projection (+ residual) and the SwiGLU MLP (+ residual), in place on x. ``att`` is this rank's
        [b, T, hl, 128] attention output, or (gathered=True) the group's [g, b, T, hl * 128] buffer."""
        cfg, t = self.cfg, self.timer
        b, T, D = x.shape
        M, F = b * T, cfg.mlp
        x2 = x.view(M, D)
        q8 = self.q8[:M * D].view(M, D)
        with t("prepass"):
            if not gathered:
                ops.quant_pack_a(att.reshape(M, D), cfg.rot_group, out=(q8, self.sa))
            else:
                w = att.shape[-1]
                ops.quant_pack_a_segments(att, D, cfg.rot_group, w, M * w, M, w, out=(q8, self.sa))
        if self.probe:
            self.probe("out_prepass", q8, self.sa)
        with t("gemm", 2 * M * D * D):
            ops.gemm(q8, self.sa, blk.w_o, blk.s_o, residual=x2, out=self.xa)
        if self.probe:
            self.probe("out_proj", self.xa)
        with t("prepass"):
            ops.mod_quant_pack_a(self.xa, blk.norm2, None, None, T, cfg.eps, cfg.rot_group, out=(q8, self.sa))
        if self.probe:
            self.probe("norm2", q8, self.sa)
        with t("gemm", 2 * M * D * 2 * F):
            ops.gemm_swiglu(q8, self.sa, blk.w_gu, blk.s_gu, out=self.act)
        if self.probe:
            self.probe("gate_up", self.act)
        q8f = self.q8[:M * F].view(M, F)
        with t("prepass"):
            ops.quant_pack_a(self.act, cfg.rot_group, out=(q8f, self.sa))
        if self.probe:
            self.probe("down_prepass", q8f, self.sa)
        with t("gemm", 2 * M * F * D):
            ops.gemm(q8f, self.sa, blk.w_down, blk.s_down, residual=self.xa, out=x2)
        if self.probe:
            self.probe("down", x2)
        return x

    def block(self, blk, x):
        fg = self.fused
        if fg is not None and self.gathered is not None:
            par = fg.blocks_done % 2
            seg, off = fg.segment(par)
            b, T = x.shape[0], x.shape[1]
            out = seg.view(b, T, self.hl, self.cfg.head_dim)
            self.attention_part(blk, x, gather=(out, [p + off for p in fg.peer_buf], fg.peer_cnt))
            fg.blocks_done += 1
            expected = fg.blocks_done * (fg.g - 1) * ops.attention_gather_ctas(b, self.hl, T)
            with self.timer("gather_wait"):
                ops.wait_count(fg.cnt, expected, fg.err, fg.timeout_ns)
            return self.mlp_part(blk, x, fg.buf[par], gathered=True)
        att = self.attention_part(blk, x)
        if self.gathered is not None:
            with self.timer("all_gather"):
                self.all_gather(self.gathered.view(-1), att.view(-1))
            return self.mlp_part(blk, x, self.gathered, gathered=True)
        return self.mlp_part(blk, x, att)

    def forward(self, x):
        """In place on x [b, T, D] fp16 contiguous."""
        for blk in self.blocks:
            self.block(blk, x)
        return x

    launches_per_block = 9

    def flops(self):
        """Algorithmic work of one step on this rank: (int8 ops, fp16 attention flops)."""
        cfg, p = self.cfg, self.plan
        b = p.batch_hi - p.batch_lo
        M, D, F = b * cfg.tokens, cfg.hidden, cfg.mlp
        lin = 2 * M * D * (3 * self.hl * cfg.head_dim + D + 2 * F) + 2 * M * F * D
        att = 4 * b * self.hl * cfg.tokens ** 2 * cfg.head_dim
        return cfg.blocks * lin, cfg.blocks * att
