"""Single-token decode of an int8 decoder-only text encoder (benchmark configuration 5) on the sm_100a kernels.

Architecture (the configuration's): hidden 2560, 36 layers, 32 query / 8 KV heads of 128, SwiGLU MLP 9728, RMSNorm,
per-output-channel int8 linears read by the HBM-streaming GEMV, fp32 activations and fp32 decode attention over a
fixed-capacity KV cache (int8_gemv.py:117-126). Three ways to run a token, all on this library's kernels:
  mode "persistent" (default): the whole token, every layer, in ONE launch (b2_decode_step): one CTA per SM streams
    its rows of every layer's weights through a shared-memory ring while grid barriers separate the stages below.
  mode "layers": 9 launches per layer:
    RMSNorm -> GEMV(q|k|v) -> QK-norm + rope + KV-cache write -> decode attention (split 32 + merge)
    -> GEMV(o) with the residual in its epilogue -> RMSNorm -> GEMV(gate|up) -> GEMV(down) reading silu(gate) * up
    as its input and adding the residual.
  fused = False: `layer_reference`, the same layer with the element-wise work as torch ops (about 25 launches per
    layer), kept as the reference the other two are tested against.
The q/k/v and gate/up weights of a layer are stored concatenated, so each is one GEMV over one x. The whole step is
captured once in a CUDA graph and replayed (the position and the cache length live on the device, as in the
reference, int8_gemv.hip:121-131).
"""
import dataclasses

import torch

from . import ops


@dataclasses.dataclass
class DecoderConfig:
    hidden: int = 2560
    layers: int = 36
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    mlp: int = 9728
    eps: float = 1e-6
    capacity: int = 1024
    rope_theta: float = 1000000.0


def quantize_rows(w):
    """Per-output-channel symmetric int8, scale = absmax / 127, round half even."""
    scale = w.abs().amax(dim=1) / 127.0
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    return torch.round(w / scale[:, None]).clamp_(-127, 127).to(torch.int8).contiguous(), scale.float().contiguous()


class Layer:
    def __init__(self, cfg, device, gen):
        D, H, Hk, d, F = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.mlp

        def weight(n, k):
            return quantize_rows(torch.randn((n, k), generator=gen, device=device) * 0.02)

        self.w_qkv, self.s_qkv = weight((H + 2 * Hk) * d, D)
        self.w_o, self.s_o = weight(D, H * d)
        self.w_gu, self.s_gu = weight(2 * F, D)
        self.w_down, self.s_down = weight(D, F)
        self.norm_in = 1 + torch.randn(D, generator=gen, device=device) * 0.02
        self.norm_post = 1 + torch.randn(D, generator=gen, device=device) * 0.02
        self.q_norm = 1 + torch.randn(d, generator=gen, device=device) * 0.02
        self.k_norm = 1 + torch.randn(d, generator=gen, device=device) * 0.02
        self.k_cache = torch.randn((1, cfg.capacity, Hk, d), generator=gen, device=device)
        self.v_cache = torch.randn((1, cfg.capacity, Hk, d), generator=gen, device=device)


def rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


class TextDecoder:
    def __init__(self, cfg, device, seed=0):
        self.cfg, self.device = cfg, device
        gen = torch.Generator(device=device).manual_seed(seed)
        self.layers = [Layer(cfg, device, gen) for _ in range(cfg.layers)]
        d = cfg.head_dim
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, device=device, dtype=torch.float32) / d))
        self.inv_freq = inv
        self.pos = torch.zeros((1,), dtype=torch.int64, device=device)
        self.lengths = torch.zeros((1,), dtype=torch.int32, device=device)
        self.x = torch.zeros((1, cfg.hidden), dtype=torch.float32, device=device)
        H, Hk = cfg.heads, cfg.kv_heads
        self.partial = torch.empty((H, ops.DECODE_SPLITS, d), dtype=torch.float32, device=device)
        self.stats = torch.empty((H, ops.DECODE_SPLITS, 2), dtype=torch.float32, device=device)
        self.att = torch.empty((1, 1, H, d), dtype=torch.float32, device=device)
        D, F = cfg.hidden, cfg.mlp
        self.h = torch.empty((D,), dtype=torch.float32, device=device)
        self.x2 = torch.empty((D,), dtype=torch.float32, device=device)
        self.xb = torch.empty((D,), dtype=torch.float32, device=device)
        self.qkv = torch.empty(((H + 2 * Hk) * d,), dtype=torch.float32, device=device)
        self.q = torch.empty((H, d), dtype=torch.float32, device=device)
        self.gu = torch.empty((2 * F,), dtype=torch.float32, device=device)
        self.act = torch.empty((F,), dtype=torch.float32, device=device)
        self.sync = torch.zeros((ops.DECODE_STEP_SYNC_WORDS,), dtype=torch.int32, device=device)
        self.err = torch.zeros((1,), dtype=torch.int32, device=device)
        self.table = None
        self.mode = "persistent"
        self.fused = True
        self.graph = None

    def rope(self, t):
        """t [n, 128] rotated at position self.pos (half-split rotary, as Qwen-style models)."""
        ang = self.pos.to(torch.float32)[:, None] * self.inv_freq[None, :]
        cos, sin = torch.cos(ang), torch.sin(ang)
        a, b = t[:, :64], t[:, 64:]
        return torch.cat((a * cos - b * sin, a * sin + b * cos), dim=-1)

    def layer(self, L, x, out):
        """x [D] -> out [D] (distinct buffers) through the fused kernels."""
        cfg = self.cfg
        H, Hk, d = cfg.heads, cfg.kv_heads, cfg.head_dim
        ops.rms_norm_f32(x, L.norm_in, cfg.eps, out=self.h)
        ops.gemv_i8(self.h, L.w_qkv, L.s_qkv, out=self.qkv)
        ops.decode_qk_rope(self.qkv, L.q_norm, L.k_norm, self.inv_freq, self.pos, self.q, L.k_cache, L.v_cache, H, Hk,
                           cfg.eps)
        ops.attn_decode(self.q.view(1, 1, H, d), L.k_cache, L.v_cache, self.lengths, d ** -0.5, out=self.att,
                        partial=self.partial, stats=self.stats)
        ops.gemv_i8_ex(self.att.reshape(-1), L.w_o, L.s_o, residual=x, out=self.x2)
        ops.rms_norm_f32(self.x2, L.norm_post, cfg.eps, out=self.h)
        ops.gemv_i8(self.h, L.w_gu, L.s_gu, out=self.gu)
        return ops.gemv_i8_ex(self.gu, L.w_down, L.s_down, residual=self.x2, silu_mul=True, out=out)

    def layer_reference(self, L, x):
        cfg = self.cfg
        H, Hk, d, F = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.mlp
        h = rms(x, L.norm_in, cfg.eps)
        qkv = ops.gemv_i8(h.reshape(-1), L.w_qkv, L.s_qkv)
        q = rms(qkv[:H * d].view(H, d), L.q_norm, cfg.eps)
        k = rms(qkv[H * d:(H + Hk) * d].view(Hk, d), L.k_norm, cfg.eps)
        v = qkv[(H + Hk) * d:].view(Hk, d)
        q, k = self.rope(q), self.rope(k)
        L.k_cache[0].index_copy_(0, self.pos, k.unsqueeze(0))
        L.v_cache[0].index_copy_(0, self.pos, v.unsqueeze(0))
        ops.attn_decode(q.view(1, 1, H, d), L.k_cache, L.v_cache, self.lengths, d ** -0.5, out=self.att,
                        partial=self.partial, stats=self.stats)
        x = x + ops.gemv_i8(self.att.reshape(-1), L.w_o, L.s_o).view(1, -1)
        h = rms(x, L.norm_post, cfg.eps)
        gu = ops.gemv_i8(h.reshape(-1), L.w_gu, L.s_gu)
        a = torch.nn.functional.silu(gu[:F]) * gu[F:]
        return x + ops.gemv_i8(a, L.w_down, L.s_down).view(1, -1)

    def persistent_step(self):
        """One token through all layers in one launch; self.x is the residual stream in and out."""
        cfg = self.cfg
        if self.table is None:
            self.table = ops.decode_step_table(self.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.mlp, cfg.capacity)
        ops.decode_step(self.table, self.x.view(-1), self.xb, self.qkv, self.att.view(-1), self.act, self.partial,
                        self.stats, self.inv_freq, self.pos, self.lengths, self.sync, self.err, cfg.hidden, cfg.heads,
                        cfg.kv_heads, cfg.mlp, cfg.capacity, cfg.eps)
        return self.x

    def failed(self):
        """Error code the persistent step left (0: none; see b2_decode_step)."""
        return int(self.err.item())

    def step_eager(self):
        if self.fused and self.mode == "persistent":
            return self.persistent_step()
        if not self.fused:
            x = self.x
            for L in self.layers:
                x = self.layer_reference(L, x)
            self.x.copy_(x)
            return self.x
        bufs = (self.x.view(-1), self.xb)
        for i, L in enumerate(self.layers):
            self.layer(L, bufs[i & 1], bufs[(i + 1) & 1])
        if len(self.layers) & 1:
            self.x.view(-1).copy_(self.xb)
        return self.x

    def capture(self):
        """Records one token step in a CUDA graph (warm-up run first, on a side stream as torch requires)."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.step_eager()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step_eager()
        return self.graph

    def set_position(self, pos):
        """Position of the new token (the cache then holds pos + 1 entries)."""
        self.pos.fill_(pos)
        self.lengths.fill_(pos + 1)

    def step(self):
        if self.graph is None:
            self.capture()
        self.graph.replay()
        return self.x

    def bytes_per_token(self):
        """Algorithmic HBM bytes of one step: every int8 weight once, the KV cache of the attended positions, plus
        the fp32 scales."""
        cfg = self.cfg
        w = sum(L.w_qkv.numel() + L.w_o.numel() + L.w_gu.numel() + L.w_down.numel() for L in self.layers)
        s = sum(L.s_qkv.numel() + L.s_o.numel() + L.s_gu.numel() + L.s_down.numel() for L in self.layers) * 4
        kv = cfg.layers * 2 * cfg.capacity * cfg.kv_heads * cfg.head_dim * 4
        return w + s + kv, w

    launches_per_layer = 9  # mode "layers": 2 RMSNorms, 4 GEMVs, q/k rope, decode attention (2 kernels)
    launches_per_token_persistent = 1  # mode "persistent": one kernel (plus the counters' memset node)
