"""Benchmark of the quantized DiT/LLM inner loop on B200 (one JSON line on rank 0).

Workloads:
  gemm    C1  W8A8 rotated linear 1024x3072x3072 (block-128 Hadamard), TOPS
  attn    C2  fused attention B2 H24 S4056 d128, fp16 QK (and attn_i8: int8 QK), TFLOPS
  w4a8    C3  W4A8 linear 2809x3072x8192, group 128, TOPS
  dit     C4  8 DiT blocks, B2 (CFG) x 3321 tokens, hidden 3072, 24 heads, MLP 8192, ms/step (default)
  decode  C5  single-token decode, 36 layers, hidden 2560, 32/8 heads, MLP 9728, ctx 1024, ms/token

``--impl reference`` times the reference's CPU path (the oracle restatement, on all host threads) for the same
workload and metric. Run with torchrun for N > 1 GPUs (one process per GPU).
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
DECODE_MODE, DECODE_LAYERS = "persistent", 36

# DRAM traffic per launch of each workload's roofline kernel: dram__bytes_read.sum + dram__bytes_write.sum from one
# ncu capture of that kernel on a B200 (cold L2).  Output lines still dirty in L2 when a kernel ends are not counted
# as written yet, so a kernel whose output fits in L2 can show less than its algorithmic bytes.
NCU_TRAFFIC = {
    "attn": 149.87e6 + 31.14e6,      # C2 fp16, one launch
    "attn_i8": 101.35e6 + 23.09e6,   # C2 int8 QK, one launch
    "w4a8": 36.48e6 + 6.38e6,        # C3, one launch of gemm_w4a8_wide_kernel
    "w4a4": 33.93e6 + 9.12e6,        # C3 shapes, one launch of the W8A8 pair GEMM on the widened int4 weight
    "prepass": 40.87e6 + 0.46e6,     # C4 QKV pre-pass (MOD), one launch; the 20.4 MB int8 output stays in L2
    "decode": 15.78e6 * 19456 / 6144,  # captured on the 6144-row qkv GEMV; bytes grow with rows (2568 B per row)
    "decode_step": (438.05e6 + 4.04e6) / 4,  # per layer of decode_step_kernel (4-layer decoder, one launch)
    "dit": 113.8e6 + 52.1e6,         # mean over the 32 W8A8 GEMM launches of one DiT step
}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class Clocks:
    """Samples nvidia-smi during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout=3.0):
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < timeout:
            time.sleep(0.05)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl != "reference":
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1 and dist.is_initialized():
        dist.barrier()


def max_over_ranks(x, world):
    if world > 1 and dist.is_initialized():
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()
    return x


def timed(run_step, steps, warmup, world, begin=None, finish=None):
    """W warm-up steps, then K steps between a barrier + synchronize on both sides; CUDA events on the current
    stream. ``begin`` runs right after the start event (a pipelined step restarts there, so that every timed step's
    copies happen after it), ``finish`` right before the end event (it makes the current stream wait for work
    that the steps left on other streams). Returns the total ms over the K steps, max over ranks."""
    for i in range(warmup):
        run_step(i)
    if finish:
        finish()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    if begin:
        begin()
    for i in range(steps):
        run_step(warmup + i)
    if finish:
        finish()
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    return max_over_ranks(start.elapsed_time(end), world)


def kernel_ms(events):
    """Average duration of the dominant kernel from (start, end) event pairs recorded around its launches."""
    torch.cuda.synchronize()
    times = [s.elapsed_time(e) for s, e in events]
    return sum(times) / len(times) if times else None


def pkg():
    import __graft_entry__

    return __graft_entry__.load_package()


# ---------------------------------------------------------------------------------------------------------- workloads
class GemmC1:
    name = "gemm"
    metric = "W8A8 GEMM TOPS (C1: 1024x3072x3072 rotated linear, pre-pass + GEMM)"
    unit = "TOPS"
    higher = True
    M, K, N = 1024, 3072, 3072

    def __init__(self, dev):
        from oracle import weights as ow

        p = pkg()
        self.ops, self.int8_gemm = p.ops, p.int8_gemm
        g = np.random.default_rng(0)
        x = g.standard_normal((self.M, self.K)).astype(np.float32)
        x[:, g.choice(self.K, self.K // 100, replace=False)] *= 20
        self.x_host = torch.from_numpy(x.astype(np.float16)).pin_memory()
        w = (g.standard_normal((self.N, self.K)) * 0.02).astype(np.float32)
        wq, ws = ow.quantize_per_channel(ow.sylvester_rotate(w))
        bias = (g.standard_normal(self.N) * 0.01).astype(np.float16)
        # Rotating sets of inputs and weights, together larger than 2x L2, so each step reads from DRAM.
        per = self.M * self.K * 3 + self.N * self.K + self.M * self.N * 2
        self.sets = max(2, math.ceil(2 * L2_BYTES / per))
        self.xs = [self.x_host.to(dev) for _ in range(self.sets)]
        self.ws = [torch.from_numpy(wq).to(dev) for _ in range(self.sets)]
        self.wscale = torch.from_numpy(ws).to(dev)
        self.bias = torch.from_numpy(bias).to(dev)
        self.qs = [(torch.empty((self.M, self.K), dtype=torch.int8, device=dev),
                    torch.empty((self.M,), dtype=torch.float32, device=dev)) for _ in range(self.sets)]
        self.outs = [torch.empty((self.M, self.N), dtype=torch.float16, device=dev) for _ in range(self.sets)]
        self.y_host = torch.empty((self.M, self.N), dtype=torch.float16).pin_memory()
        self.events = []
        self.launches_per_step = 2
        self.ops_per_step = 2.0 * self.M * self.N * self.K
        # The two launches of a step (pre-pass, GEMM) are captured once per input set as one graph and replayed, as a
        # serving loop would run the linear: a 10-15 us GEMM otherwise waits on the Python and ctypes path that
        # enqueues it, and every graph launch adds a few microseconds. The kernel-timing pass replays the pre-pass and
        # the GEMM as separate graphs so that events can bracket the GEMM alone.
        self.g_pre, self.g_gemm, self.g_linear = [], [], []
        for s in range(self.sets):
            self._pre(s)
            self._gemm(s)
        torch.cuda.synchronize()
        for s in range(self.sets):
            gp, gg, gl = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            with torch.cuda.graph(gp):
                self._pre(s)
            with torch.cuda.graph(gg):
                self._gemm(s)
            with torch.cuda.graph(gl):
                self._pre(s)
                self._gemm(s)
            self.g_pre.append(gp)
            self.g_gemm.append(gg)
            self.g_linear.append(gl)
        torch.cuda.synchronize()

    def _pre(self, s):
        self.ops.quant_pack_a(self.xs[s], 128, out=self.qs[s])

    def _gemm(self, s):
        q = self.qs[s]
        self.ops.gemm(q[0], q[1], self.ws[s], self.wscale, self.bias, out=self.outs[s])

    def step(self, i, record=False):
        s = i % self.sets
        if not record:
            self.g_linear[s].replay()
            return
        self.g_pre[s].replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        self.g_gemm[s].replay()
        e1.record()
        self.events.append((e0, e1))

    def e2e_step(self, i):
        s = i % self.sets
        x = self.x_host.to(self.xs[s].device, non_blocking=True)
        y = self.int8_gemm.linear(x, self.ws[s], self.wscale, self.bias, rotate=True, rot_group=128)
        self.y_host.copy_(y, non_blocking=True)

    h2d_bytes = property(lambda self: self.M * self.K * 2)
    d2h_bytes = property(lambda self: self.M * self.N * 2)

    def value(self, ms, steps, world):
        return self.ops_per_step * steps * world / (ms * 1e-3) / 1e12

    def roofline(self, peaks, kms):
        peak = 2.0 * peaks["bf16_tflops"]
        achieved = self.ops_per_step / (kms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOPS", "frac": achieved / peak,
                "traffic": None, "kernel": "gemm_w8a8_kernel",
                "note": f"int8 peak = 2 x {peaks['source']} bf16 ({peaks['bf16_tflops']} TFLOP/s)"}

    config = {"workload": "C1 W8A8 rotated linear", "M": 1024, "K": 3072, "N": 3072, "rotation": "block-128 Sylvester",
              "l2": "rotating input/weight sets > 2x L2",
              "launch": "pre-pass + GEMM replayed as one CUDA graph per input set; the GEMM alone for the roofline"}

    @staticmethod
    def cpu_baseline(threads):
        from oracle import gemm as ogemm
        from oracle import quant as oq
        from oracle import weights as ow

        torch.set_num_threads(threads)
        g = np.random.default_rng(0)
        M, K, N = GemmC1.M, GemmC1.K, GemmC1.N
        x = g.standard_normal((M, K)).astype(np.float16)
        wq, ws = ow.quantize_per_channel(ow.sylvester_rotate((g.standard_normal((N, K)) * 0.02).astype(np.float32)))
        bias = (g.standard_normal(N) * 0.01).astype(np.float16)

        def run():
            t0 = time.perf_counter()
            q, s, _ = oq.prepass(x, 128)
            ogemm.epilogue(ogemm.int_mm(q, wq), s, ws, bias)
            dt = time.perf_counter() - t0
            return 2.0 * M * N * K / dt / 1e12, dt
        return run, "one full C1 linear per sample (oracle pre-pass + torch._int_mm + epilogue), scale 1"


class AttnC2:
    name = "attn"
    unit = "TFLOPS"
    higher = True
    B, H, S = 2, 24, 4056

    def __init__(self, dev, int8_qk=False):
        p = pkg()
        self.ops, self.attention = p.ops, p.attention
        self.int8_qk = int8_qk
        self.metric = f"attention TFLOPS (C2: B2 H24 S4056 d128, {'int8' if int8_qk else 'fp16'} QK)"
        gen = torch.Generator().manual_seed(2)
        shape = (self.B, self.H, self.S, 128)
        self.host = [torch.randn(shape, generator=gen).half().pin_memory() for _ in range(3)]
        per = 4 * self.B * self.H * self.S * 128 * 2
        self.sets = max(2, math.ceil(2 * L2_BYTES / per))
        self.qkv = [[t.to(dev) for t in self.host] for _ in range(self.sets)]
        self.outs = [torch.empty(shape, dtype=torch.float16, device=dev) for _ in range(self.sets)]
        lib = p._lib.load()
        n = lib.b2_attention_workspace_bytes(self.B, self.H, self.H, self.S, self.S, int(int8_qk))
        self.ws = torch.empty(max(n, 16), dtype=torch.uint8, device=dev)
        self.out_host = torch.empty(shape, dtype=torch.float16).pin_memory()
        self.events = []
        self.launches_per_step = 3 if int8_qk else 1
        self.flops = 4.0 * self.B * self.H * self.S * self.S * 128
        self.config = {"workload": "C2 fused attention", "B": 2, "H": 24, "S": 4056, "d": 128,
                       "qk": "int8" if int8_qk else "fp16", "l2": "rotating q/k/v sets > 2x L2"}

    def step(self, i, record=False):
        s = i % self.sets
        q, k, v = self.qkv[s]
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        self.ops.attention(q, k, v, self.outs[s], 128 ** -0.5, int8_qk=self.int8_qk, workspace=self.ws)
        if record:
            e1.record()
            self.events.append((e0, e1))

    def e2e_step(self, i):
        dev = self.qkv[0][0].device
        q, k, v = (t.to(dev, non_blocking=True) for t in self.host)
        out = self.attention.attention_hip(q, k, v, self.H, skip_reshape=True, skip_output_reshape=True,
                                           int8_qk=self.int8_qk)
        self.out_host.copy_(out, non_blocking=True)

    h2d_bytes = property(lambda self: 3 * self.B * self.H * self.S * 128 * 2)
    d2h_bytes = property(lambda self: self.B * self.H * self.S * 128 * 2)

    def value(self, ms, steps, world):
        return self.flops * steps * world / (ms * 1e-3) / 1e12

    def roofline(self, peaks, kms):
        peak = peaks["bf16_tflops"]
        achieved = self.flops / (kms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": NCU_TRAFFIC["attn_i8" if self.int8_qk else "attn"], "kernel": "attention_kernel",
                "note": f"fp16 peak = {peaks['source']} bf16 dense" + ("; includes the int8 Q/K quantization" if self.int8_qk else "")}

    @staticmethod
    def cpu_baseline(threads, int8_qk=False):
        from oracle import attention as oatt

        torch.set_num_threads(threads)
        B, H, S = AttnC2.B, AttnC2.H, AttnC2.S
        gen = torch.Generator().manual_seed(2)
        q, k, v = (torch.randn((1, 1, S, 128), generator=gen).half() for _ in range(3))

        def run():
            t0 = time.perf_counter()
            oatt.attention_bmm(q, k, v)
            dt = time.perf_counter() - t0
            return 4.0 * S * S * 128 / dt / 1e12, dt
        return run, (f"one (batch, head) slice of C2 per sample through the reference's attention_bmm (fp16 CPU); "
                     f"TFLOPS per slice = TFLOPS of the {B * H}-slice call")


class W4A8C3:
    name = "w4a8"
    metric = "W4A8 GEMM TOPS (C3: 2809x3072x8192, int4 weights, group-128 fp16 scales, pre-pass + GEMM)"
    # The weight is widened to int8 once at load time (the unpacked copy convrot_w4a4_forward's qweight_unpacked
    # carries); the GEMM reads it by TMA. The packed-weight kernel is timed beside it in "components".
    unit = "TOPS"
    higher = True
    M, K, N = 2809, 3072, 8192

    def __init__(self, dev):
        from oracle import weights as ow

        p = pkg()
        self.ops = p.ops
        g = np.random.default_rng(3)
        x = g.standard_normal((self.M, self.K)).astype(np.float16)
        self.x_host = torch.from_numpy(x).pin_memory()
        w = (g.standard_normal((self.N, self.K)) * 0.02).astype(np.float32)
        packed, s16 = ow.quantize_int4_groups(ow.sylvester_rotate(w))
        per = self.M * self.K * 3 + self.N * self.K + self.M * self.N * 2
        self.sets = max(2, math.ceil(2 * L2_BYTES / per))
        self.xs = [self.x_host.to(dev) for _ in range(self.sets)]
        self.ws = [torch.from_numpy(packed).to(dev) for _ in range(self.sets)]
        self.gs = self.ops.w4a8_scales(torch.from_numpy(s16).to(dev))
        self.ww = [self.ops.unpack_int4(w) for w in self.ws]
        self.qs = [(torch.empty((self.M, self.K), dtype=torch.int8, device=dev),
                    torch.empty((self.M,), dtype=torch.float32, device=dev)) for _ in range(self.sets)]
        self.outs = [torch.empty((self.M, self.N), dtype=torch.float16, device=dev) for _ in range(self.sets)]
        self.y_host = torch.empty((self.M, self.N), dtype=torch.float16).pin_memory()
        self.events = []
        self.launches_per_step = 2
        self.ops_per_step = 2.0 * self.M * self.N * self.K
        self.config = {"workload": "C3 W4A8 linear", "M": self.M, "K": self.K, "N": self.N, "group": 128,
                       "rotation": "block-128 Sylvester", "l2": "rotating input/weight sets > 2x L2",
                       "weight": "int4 packed, widened to int8 once at load time (qweight_unpacked)"}

    def step(self, i, record=False):
        s = i % self.sets
        q = self.ops.quant_pack_a(self.xs[s], 128, out=self.qs[s])
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        self.ops.gemm_w4a8(q[0], q[1], self.ws[s], self.gs, out=self.outs[s], w_wide=self.ww[s])
        if record:
            e1.record()
            self.events.append((e0, e1))

    def e2e_step(self, i):
        s = i % self.sets
        x = self.x_host.to(self.xs[s].device, non_blocking=True)
        q = self.ops.quant_pack_a(x, 128)
        y = self.ops.gemm_w4a8(q[0], q[1], self.ws[s], self.gs, w_wide=self.ww[s])
        self.y_host.copy_(y, non_blocking=True)

    h2d_bytes = property(lambda self: self.M * self.K * 2)
    d2h_bytes = property(lambda self: self.M * self.N * 2)

    def value(self, ms, steps, world):
        return self.ops_per_step * steps * world / (ms * 1e-3) / 1e12

    def roofline(self, peaks, kms):
        peak = 2.0 * peaks["bf16_tflops"]
        achieved = self.ops_per_step / (kms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOPS", "frac": achieved / peak,
                "traffic": NCU_TRAFFIC["w4a8"], "kernel": "gemm_w4a8_wide_kernel",
                "note": f"int8 peak = 2 x {peaks['source']} bf16 ({peaks['bf16_tflops']} TFLOP/s)"}

    @staticmethod
    def cpu_baseline(threads):
        from oracle import gemm as ogemm
        from oracle import quant as oq
        from oracle import weights as ow

        torch.set_num_threads(threads)
        g = np.random.default_rng(3)
        M, K, N = 512, W4A8C3.K, W4A8C3.N
        x = g.standard_normal((M, K)).astype(np.float16)
        packed, s16 = ow.quantize_int4_groups((g.standard_normal((N, K)) * 0.02).astype(np.float32))

        def run():
            t0 = time.perf_counter()
            q, s, _ = oq.prepass(x, 128)
            ogemm.w4a8_grouped(q, s, packed, s16)
            dt = time.perf_counter() - t0
            return 2.0 * M * N * K / dt / 1e12, dt
        return run, "512 of the 2809 rows per sample (oracle pre-pass + per-group torch._int_mm + fp32 combine); TOPS of the sample"


class W4A4C3(W4A8C3):
    """The reference's own int4 form on the C3 shapes: ConvRot-256 and int4-valued per-token activations, packed int4
    weights with per-channel scales (int8_gemm.py:90-103); the packed weight is widened into a workspace and the
    W8A8 GEMM accumulates in int32 over all of K."""
    name = "w4a4"
    metric = "W4A4 GEMM TOPS (C3 shapes 2809x3072x8192, int4 weights and activations, per-channel scales, pre-pass + GEMM)"
    # As for W4A8, the int4 weight is widened to int8 once at load time (convrot_w4a4_forward's qweight_unpacked);
    # without that copy the drop-in widens it per call, as the reference re-packs it.

    def __init__(self, dev):
        p = pkg()
        self.ops = p.ops
        g = np.random.default_rng(4)
        x = g.standard_normal((self.M, self.K)).astype(np.float16)
        self.x_host = torch.from_numpy(x).pin_memory()
        packed = g.integers(0, 256, (self.N, self.K // 2), dtype=np.uint8)
        per = self.M * self.K * 3 + self.N * self.K + self.M * self.N * 2
        self.sets = max(2, math.ceil(2 * L2_BYTES / per))
        self.xs = [self.x_host.to(dev) for _ in range(self.sets)]
        self.ws = [torch.from_numpy(packed).to(dev) for _ in range(self.sets)]
        self.wscale = torch.from_numpy((g.random(self.N) * 1e-2 + 1e-4).astype(np.float32)).to(dev)
        self.ww = [self.ops.unpack_int4(w) for w in self.ws]
        self.forward = p.int8_gemm.wrap_w4a4(None)
        self.qs = [(torch.empty((self.M, self.K), dtype=torch.int8, device=dev),
                    torch.empty((self.M,), dtype=torch.float32, device=dev)) for _ in range(self.sets)]
        self.outs = [torch.empty((self.M, self.N), dtype=torch.float16, device=dev) for _ in range(self.sets)]
        self.y_host = torch.empty((self.M, self.N), dtype=torch.float16).pin_memory()
        self.events = []
        self.launches_per_step = 2
        self.ops_per_step = 2.0 * self.M * self.N * self.K
        self.config = {"workload": "C3 shapes, per-channel W4A4", "M": self.M, "K": self.K, "N": self.N,
                       "rotation": "ConvRot 256", "l2": "rotating input/weight sets > 2x L2",
                       "weight": "int4 packed, widened to int8 once at load time (qweight_unpacked)"}

    def step(self, i, record=False):
        s = i % self.sets
        q = self.ops.quant_pack_a_i4(self.xs[s], 256, out=self.qs[s])
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        self.ops.gemm(q[0], q[1], self.ww[s], self.wscale, out=self.outs[s])
        if record:
            e1.record()
            self.events.append((e0, e1))

    def e2e_step(self, i):
        s = i % self.sets
        x = self.x_host.to(self.xs[s].device, non_blocking=True)
        y = self.forward(x, self.ws[s], self.wscale, None, 256, torch.float16, qweight_unpacked=self.ww[s])
        self.y_host.copy_(y, non_blocking=True)

    def roofline(self, peaks, kms):
        r = super().roofline(peaks, kms)
        r.update(traffic=NCU_TRAFFIC["w4a4"], kernel="gemm_w8a8_pair_kernel (on the weight widened at load time)")
        return r

    @staticmethod
    def cpu_baseline(threads):
        from oracle import gemm as ogemm
        from oracle import quant as oq

        torch.set_num_threads(threads)
        g = np.random.default_rng(4)
        M, K, N = 512, W4A4C3.K, W4A4C3.N
        x = g.standard_normal((M, K)).astype(np.float16)
        packed = g.integers(0, 256, (N, K // 2), dtype=np.uint8)
        ws = np.full(N, 1e-3, np.float32)

        def run():
            t0 = time.perf_counter()
            q, s = oq.quant_rows_i4(oq.rotate_rows(x, 256))
            ogemm.epilogue(ogemm.int_mm(q, ogemm.unpack_int4(packed)), s, ws)
            dt = time.perf_counter() - t0
            return 2.0 * M * N * K / dt / 1e12, dt
        return run, "512 of the 2809 rows per sample (oracle ConvRot + int4 quant + torch._int_mm + epilogue); TOPS of the sample"


class GemmQKV(GemmC1):
    """The C4 QKV projection alone (M = 2 x 3321 tokens, N = 9216, K = 3072): the DiT step's GEMM shape."""
    name = "gemm_qkv"
    metric = "W8A8 GEMM TOPS (C4 QKV projection 6642x9216x3072, pre-pass + GEMM)"
    M, K, N = 6642, 3072, 9216
    config = {"workload": "C4 QKV projection", "M": 6642, "K": 3072, "N": 9216, "rotation": "block-128 Sylvester",
              "l2": "rotating input/weight sets > 2x L2"}

    cpu_baseline = None


class PrepassC4:
    """The C4 QKV pre-pass alone: RMSNorm + block-128 rotation + per-token int8 of [6642, 3072] fp16."""
    name = "prepass"
    metric = "pre-pass GB/s (C4: RMSNorm + block-128 Hadamard + int8 of 6642x3072 fp16)"
    unit = "GB/s"
    higher = True
    M, K = 6642, 3072

    def __init__(self, dev):
        p = pkg()
        self.ops = p.ops
        g = torch.Generator().manual_seed(6)
        self.x_host = torch.randn((self.M, self.K), generator=g).half().pin_memory()
        self.bytes = self.M * self.K * 2 + self.M * self.K + self.M * 4 + self.K * 4
        self.sets = max(2, math.ceil(2 * L2_BYTES / self.bytes))
        self.xs = [self.x_host.to(dev) for _ in range(self.sets)]
        self.w = (torch.randn(self.K, generator=g) * 0.02).float().to(dev)
        self.outs = [(torch.empty((self.M, self.K), dtype=torch.int8, device=dev),
                      torch.empty((self.M,), dtype=torch.float32, device=dev)) for _ in range(self.sets)]
        self.q_host = torch.empty((self.M, self.K), dtype=torch.int8).pin_memory()
        self.events = []
        self.launches_per_step = 1
        self.config = {"workload": "C4 QKV pre-pass", "M": self.M, "K": self.K, "rotation": "block-128 Sylvester",
                       "l2": "rotating input sets > 2x L2"}

    def step(self, i, record=False):
        s = i % self.sets
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        self.ops.mod_quant_pack_a(self.xs[s], self.w, None, None, self.M, 1e-6, 128, out=self.outs[s])
        if record:
            e1.record()
            self.events.append((e0, e1))

    def e2e_step(self, i):
        s = i % self.sets
        x = self.x_host.to(self.xs[s].device, non_blocking=True)
        q, _ = self.ops.mod_quant_pack_a(x, self.w, None, None, self.M, 1e-6, 128)
        self.q_host.copy_(q, non_blocking=True)

    h2d_bytes = property(lambda self: self.M * self.K * 2)
    d2h_bytes = property(lambda self: self.M * self.K)

    def value(self, ms, steps, world):
        return self.bytes * steps * world / (ms * 1e-3) / 1e9

    def roofline(self, peaks, kms):
        achieved = self.bytes / (kms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": NCU_TRAFFIC["prepass"], "kernel": "prepass128_kernel<MOD>",
                "note": f"{peaks['source']} HBM copy bandwidth"}

    @staticmethod
    def cpu_baseline(threads):
        from oracle import quant as oq

        g = np.random.default_rng(6)
        M, K = 512, PrepassC4.K
        x = g.standard_normal((M, K)).astype(np.float16)

        def run():
            t0 = time.perf_counter()
            oq.prepass(x, 128, act="mod", w=np.zeros(K, np.float32), s=np.ones((1, K), np.float16),
                       t=np.zeros((1, K), np.float16), L=M)
            dt = time.perf_counter() - t0
            return (M * K * 3 + M * 4) / dt / 1e9, dt
        return run, "512 of 6642 rows per sample through the numpy oracle pre-pass; GB/s of the sample"


class DecodeC5:
    name = "decode"
    metric = "single-token decode ms/token (C5: 36-layer int8 decoder, hidden 2560, 32/8 heads of 128, MLP 9728, KV 1024)"
    unit = "ms/token"
    higher = False

    def __init__(self, dev):
        import importlib

        p = pkg()
        self.ops = p.ops
        decoder = importlib.import_module(p.__name__ + ".decoder")
        self.cfg = cfg = decoder.DecoderConfig(layers=DECODE_LAYERS)
        self.dec = decoder.TextDecoder(cfg, dev, seed=0)
        self.dec.mode = DECODE_MODE
        self.dec.set_position(cfg.capacity - 1)
        g = torch.Generator().manual_seed(5)
        self.x_host = torch.randn((1, cfg.hidden), generator=g).pin_memory()
        self.x0 = self.x_host.to(dev)
        self.out_host = torch.empty_like(self.x_host).pin_memory()
        self.dec.x.copy_(self.x0)
        self.dec.capture()
        self.bytes, self.weight_bytes = self.dec.bytes_per_token()
        self.persistent = DECODE_MODE == "persistent"
        self.launches_per_step = 1 if self.persistent else cfg.layers * decoder.TextDecoder.launches_per_layer
        self.events = []
        self.config = {"workload": "C5 single-token decode", "layers": cfg.layers, "hidden": 2560, "heads": 32,
                       "kv_heads": 8, "mlp": 9728, "kv_len": 1024, "batch": 1,
                       "mode": ("one persistent kernel per token (b2_decode_step), in a CUDA graph with its counter memset"
                                if self.persistent else "9 launches per layer, whole token step in one CUDA graph"),
                       "l2": f"{self.weight_bytes / 1e9:.1f} GB of weights per token, larger than L2"}

    def step(self, i, record=False):
        self.dec.x.copy_(self.x0)
        if record and self.persistent:
            # The whole step is the kernel: time the replay (the 256-byte counter memset node + decode_step_kernel).
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            self.dec.graph.replay()
            e1.record()
            self.events.append((e0, e1))
            return
        if record:
            # GEMV kernel timing: the gate|up weights of every layer in turn (50 MB each, 1.8 GB together).
            L = self.dec.layers[i % len(self.dec.layers)]
            h = torch.randn((self.cfg.hidden,), device=self.x0.device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            self.ops.gemv_i8(h, L.w_gu, L.s_gu)
            e1.record()
            self.events.append((e0, e1))
            self.gemv_bytes = L.w_gu.numel() + L.s_gu.numel() * 4 + h.numel() * 4 + L.w_gu.shape[0] * 4
        self.dec.graph.replay()

    def e2e_step(self, i):
        self.dec.x.copy_(self.x_host, non_blocking=True)
        self.dec.graph.replay()
        self.out_host.copy_(self.dec.x, non_blocking=True)

    h2d_bytes = property(lambda self: self.cfg.hidden * 4)
    d2h_bytes = property(lambda self: self.cfg.hidden * 4)

    def value(self, ms, steps, world):
        return ms / steps

    def roofline(self, peaks, kms):
        if self.dec.failed():
            raise RuntimeError(f"decode_step reported error {self.dec.failed()}")
        if self.persistent:
            achieved = self.bytes / (kms * 1e-3) / 1e9
            return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": achieved / peaks["hbm_gbs"],
                    "traffic": (NCU_TRAFFIC["decode_step"] * self.cfg.layers if NCU_TRAFFIC["decode_step"] else None),
                    "kernel": "decode_step_kernel<4> (the whole token: every layer's weights + the attended KV rows)",
                    "note": (f"{peaks['source']} HBM copy bandwidth; algorithmic bytes {self.bytes / 1e9:.3f} GB per token "
                             f"(int8 weights {self.weight_bytes / 1e9:.3f} GB + fp32 scales + KV cache rows)")}
        achieved = self.gemv_bytes / (kms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": NCU_TRAFFIC["decode"],
                "kernel": "gemv_i8_kernel (gate|up, 19456 x 2560)",
                "note": f"{peaks['source']} HBM copy bandwidth; step bytes {self.bytes / 1e9:.3f} GB per token"}

    @staticmethod
    def cpu_baseline(threads):
        """The reference's non-GEMV path, F.linear(x, w.to(fp32) * scale) (int8_gemv.py:58-59), and an fp32 softmax
        decode attention, for 4 of the 36 layers, scaled to 36."""
        import torch.nn.functional as Fn

        torch.set_num_threads(threads)
        g = torch.Generator().manual_seed(0)
        D, F = 2560, 9728
        shapes = [(6144, D), (D, 4096), (2 * F, D), (D, F)]
        ws = [(torch.randint(-127, 128, s, generator=g, dtype=torch.int8), torch.rand(s[0], generator=g) * 1e-3) for s in shapes]
        kc = torch.randn((1024, 8, 128), generator=g)
        vc = torch.randn((1024, 8, 128), generator=g)
        def run():
            t0 = time.perf_counter()
            for _ in range(4):
                for w, sc in ws:
                    Fn.linear(torch.randn((1, w.shape[1]), generator=g), w.to(torch.float32) * sc[:, None])
                q = torch.randn((32, 128), generator=g)
                s_ = torch.einsum("hd,khd->hk", q, kc.repeat_interleave(4, 1)) * 128 ** -0.5
                torch.softmax(s_, -1) @ vc.repeat_interleave(4, 1).transpose(0, 1)
            dt = time.perf_counter() - t0
            return dt / 4 * 36 * 1e3, dt
        return run, ("4 of 36 layers per sample through the reference's F.linear(x, w.float() * scale) fallback + fp32 "
                     "softmax attention; ms of the sample x 36 / 4")


class LogitsC5:
    """The logits of one decode step: the tied bf16 embedding table of the C5 decoder's family (vocab 151936 x 2560,
    778 MB, larger than L2) against one fp32 hidden state (int8_gemv.py:87-98)."""
    name = "logits"
    metric = "LM-head logits GEMV GB/s (bf16 table 151936 x 2560, one fp32 token)"
    unit = "GB/s"
    higher = True
    N, K = 151936, 2560

    def __init__(self, dev):
        p = pkg()
        self.ops = p.ops
        g = torch.Generator().manual_seed(7)
        self.table = (torch.randn((self.N, self.K), generator=g) * 0.02).to(torch.bfloat16).to(dev)
        self.x_host = torch.randn((self.K,), generator=g).pin_memory()
        self.x = self.x_host.to(dev)
        self.out = torch.empty((self.N,), dtype=torch.float32, device=dev)
        self.out_host = torch.empty((self.N,), dtype=torch.float32).pin_memory()
        self.bytes = self.N * self.K * 2 + self.K * 4 + self.N * 4
        self.events = []
        self.launches_per_step = 1
        self.config = {"workload": "C5 logits (tied bf16 embedding table)", "N": self.N, "K": self.K,
                       "l2": "778 MB table per step, larger than L2"}

    def step(self, i, record=False):
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        self.ops.gemv_bf16(self.x, self.table, out=self.out)
        if record:
            e1.record()
            self.events.append((e0, e1))

    def e2e_step(self, i):
        self.x.copy_(self.x_host, non_blocking=True)
        self.ops.gemv_bf16(self.x, self.table, out=self.out)
        self.out_host.copy_(self.out, non_blocking=True)

    h2d_bytes = property(lambda self: self.K * 4)
    d2h_bytes = property(lambda self: self.N * 4)

    def value(self, ms, steps, world):
        return self.bytes * steps * world / (ms * 1e-3) / 1e9

    def roofline(self, peaks, kms):
        achieved = self.bytes / (kms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": NCU_TRAFFIC.get("logits"), "kernel": "gemv_bf16_kernel",
                "note": f"{peaks['source']} HBM copy bandwidth"}

    @staticmethod
    def cpu_baseline(threads):
        """The transformer's own logits on the host: F.linear(x, table.float()) on a 16384-row slice, scaled."""
        import torch.nn.functional as Fn

        torch.set_num_threads(threads)
        g = torch.Generator().manual_seed(7)
        rows = 16384
        table = (torch.randn((rows, LogitsC5.K), generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn((1, LogitsC5.K), generator=g)

        def run():
            t0 = time.perf_counter()
            Fn.linear(x, table.float())
            dt = time.perf_counter() - t0
            return (rows * LogitsC5.K * 2) / dt / 1e9, dt
        return run, "16384 of 151936 rows per sample, F.linear(x, table.float()); GB/s of the sample"


class KindTimer:
    """Records CUDA events around each launch of a kind ("gemm", "attention", ...) during one instrumented step."""

    def __init__(self):
        self.active = False
        self.records = []

    def __call__(self, kind, work=0):
        timer = self

        class _Ctx:
            def __enter__(self):
                if timer.active:
                    self.e0 = torch.cuda.Event(enable_timing=True)
                    self.e0.record()

            def __exit__(self, *exc):
                if timer.active:
                    e1 = torch.cuda.Event(enable_timing=True)
                    e1.record()
                    timer.records.append((kind, work, self.e0, e1))

        return _Ctx()

    def summary(self):
        torch.cuda.synchronize()
        out = {}
        for kind, work, e0, e1 in self.records:
            d = out.setdefault(kind, {"ms": 0.0, "work": 0.0, "launches": 0})
            d["ms"] += e0.elapsed_time(e1)
            d["work"] += work
            d["launches"] += 1
        return out


class DiTC4:
    name = "dit"
    metric = "DiT-block ms/step (C4: 8 W8A8 DiT blocks, B2 CFG x 3321 tokens, hidden 3072, 24 heads, MLP 8192)"
    unit = "ms/step"
    higher = False

    def __init__(self, dev, world=1, rank=0):
        import importlib

        p = pkg()
        dit = importlib.import_module(p.__name__ + ".dit")
        self.cfg = cfg = dit.DiTConfig()
        self.plan = plan = dit.shard_plan(world, rank, cfg.batch, cfg.heads)
        pg = None
        if world > 1:
            groups = {}
            for r in range(world):
                gr = dit.shard_plan(world, r, cfg.batch, cfg.heads).group_ranks
                if gr not in groups:
                    groups[gr] = dist.new_group(list(gr)) if len(gr) > 1 else None
            pg = groups[plan.group_ranks]
        gather = (lambda out, inp: dist.all_gather_into_tensor(out, inp, group=pg)) if pg is not None else None
        b = plan.batch_hi - plan.batch_lo
        self.fused = None
        if pg is not None and GATHER == "fused":
            # The head-group exchange fused into the attention (peer stores + arrival counters in symmetric memory).
            self.fused = dit.FusedGather.create(pg, plan.group_index, plan.group_size, b, cfg.tokens,
                                                (plan.head_hi - plan.head_lo) * cfg.head_dim, dev)
        self.timer = KindTimer()
        self.stack = dit.DiTStack(cfg, plan, dev, seed=0, all_gather=gather, timer=self.timer, fused_gather=self.fused)
        gen = torch.Generator().manual_seed(4)
        x_all = torch.randn((cfg.batch, cfg.tokens, cfg.hidden), generator=gen).half()
        self.x_host = x_all[plan.batch_lo:plan.batch_hi].contiguous().pin_memory()
        self.x0 = self.x_host.to(dev)
        self.x = torch.empty_like(self.x0)
        self.out_host = torch.empty_like(self.x_host).pin_memory()
        self.world = world
        self.lin_ops, self.att_flops = self.stack.flops()
        self.launches_per_step = cfg.blocks * self.stack.launches_per_block
        self.events = []
        self.components = None
        self.config = {"workload": "C4 DiT block stack", "blocks": 8, "batch": 2, "tokens": 3321, "hidden": 3072,
                       "heads": 24, "mlp": 8192, "weights": "W8A8 per-channel int8, block-128 Hadamard",
                       "l2": "weights 0.9 GB per step, inputs larger than L2",
                       "e2e": "per step: pinned host input -> device and result -> pinned host on a copy stream, the next "
                              "step's input and the previous step's result overlapping this step's compute",
                       "shard": {"branches": [plan.batch_lo, plan.batch_hi], "heads": [plan.head_lo, plan.head_hi],
                                 "group": list(plan.group_ranks)},
                       "head_group_exchange": ("none" if pg is None else
                                               "fused into the attention (peer stores, symmetric memory)"
                                               if self.fused is not None else "NCCL all_gather_into_tensor")}

    def step(self, i, record=False):
        self.x.copy_(self.x0)
        self.timer.active = record
        if record:
            self.timer.records = []
        self.stack.forward(self.x)
        if record:
            self.components = self.timer.summary()
            self.timer.active = False
            g = self.components.get("gemm")
            if g:
                self.events = [(None, None)]
                self.gemm_ms, self.gemm_ops = g["ms"], g["work"]

    def e2e_begin(self):
        if not hasattr(self, "copy_stream"):
            self.copy_stream = torch.cuda.Stream()
            self.xb = [torch.empty_like(self.x0), torch.empty_like(self.x0)]
            self.in_ev = [torch.cuda.Event(), torch.cuda.Event()]
            self.fwd_ev = [torch.cuda.Event(), torch.cuda.Event()]
        self.prefetched = None

    def e2e_step(self, i):
        """One step through the public path with host buffers, pipelined the way a serving loop runs it: the step's
        input arrives from pinned host memory on a copy stream (prefetched during the previous step, or fetched now
        for the first step after e2e_begin), the forward runs in place, and the result goes back to pinned host
        memory on the copy stream while the next step computes. The copy stream fetches the next step's input first,
        then returns this step's output, so both transfers overlap compute and stay ordered with the buffer reuse."""
        if not hasattr(self, "copy_stream"):
            self.e2e_begin()
        main, cs = torch.cuda.current_stream(), self.copy_stream
        cur, nxt = i % 2, (i + 1) % 2
        if self.prefetched != i:
            cs.wait_stream(main)
            with torch.cuda.stream(cs):
                self.xb[cur].copy_(self.x_host, non_blocking=True)
                self.in_ev[cur].record(cs)
        main.wait_event(self.in_ev[cur])
        self.stack.forward(self.xb[cur])
        self.fwd_ev[cur].record(main)
        with torch.cuda.stream(cs):
            self.xb[nxt].copy_(self.x_host, non_blocking=True)  # buffer nxt: its previous output left earlier on cs
            self.in_ev[nxt].record(cs)
            cs.wait_event(self.fwd_ev[cur])
            self.out_host.copy_(self.xb[cur], non_blocking=True)
        self.prefetched = i + 1

    def e2e_finish(self):
        torch.cuda.current_stream().wait_stream(self.copy_stream)

    h2d_bytes = property(lambda self: self.x_host.numel() * 2)
    d2h_bytes = property(lambda self: self.x_host.numel() * 2)

    def value(self, ms, steps, world):
        return ms / steps

    def roofline(self, peaks, kms):
        int8_peak = 2.0 * peaks["bf16_tflops"]
        achieved = self.gemm_ops / (self.gemm_ms * 1e-3) / 1e12
        comp = {}
        for kind, d in (self.components or {}).items():
            c = {"ms": d["ms"], "launches": d["launches"]}
            if kind == "gemm":
                c["TOPS"] = d["work"] / (d["ms"] * 1e-3) / 1e12
            if kind == "attention":
                c["TFLOPS"] = d["work"] / (d["ms"] * 1e-3) / 1e12
                c["frac_of_fp16_peak"] = c["TFLOPS"] / peaks["bf16_tflops"]
            comp[kind] = c
        step_roof_ms = (self.lin_ops / (int8_peak * 1e12) + self.att_flops / (peaks["bf16_tflops"] * 1e12)) * 1e3
        return {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOPS", "frac": achieved / int8_peak,
                "traffic": NCU_TRAFFIC["dit"], "kernel": "gemm_w8a8_kernel (all 32 GEMM launches of a step)",
                "note": f"int8 peak = 2 x {peaks['source']} bf16 ({peaks['bf16_tflops']} TFLOP/s)",
                "components": comp, "step_roofline_ms": step_roof_ms}

    @staticmethod
    def cpu_baseline(threads):
        """One block of the reference's CPU path on a sample (1024 of the 6642 rows through the W8A8 linears, 2 of the
        48 (batch, head) attention slices through attention_bmm), scaled to the 8-block step."""
        from oracle import attention as oatt
        from oracle import gemm as ogemm
        from oracle import quant as oq

        torch.set_num_threads(threads)
        g = np.random.default_rng(0)
        D, F, T, Ms = 3072, 8192, 3321, 1024
        w = {n: g.integers(-127, 128, s, dtype=np.int8) for n, s in
             {"qkv": (3 * D, D), "o": (D, D), "gu": (2 * F, D), "down": (D, F)}.items()}
        ws = {n: np.full(v.shape[0], 1e-3, np.float32) for n, v in w.items()}
        x = g.standard_normal((Ms, D)).astype(np.float16)
        ones, zeros = np.ones((1, D), np.float16), np.zeros((1, D), np.float16)
        nw = np.zeros(D, np.float32)
        gen = torch.Generator().manual_seed(2)
        qa, ka, va = (torch.randn((1, 2, T, 128), generator=gen).half() for _ in range(3))
        lin_scale, att_scale = 2 * T / Ms, 24

        def run():
            t0 = time.perf_counter()
            q, s = oq.quant_rows(oq.rotate_rows(oq.modulate(x, nw, ones, zeros, Ms, 1e-6), 128))
            ogemm.epilogue(ogemm.int_mm(q, w["qkv"]), s, ws["qkv"])
            q, s = oq.quant_rows(oq.rotate_rows(x, 128))
            xa = ogemm.epilogue(ogemm.int_mm(q, w["o"]), s, ws["o"], R=x, G=ones, L=Ms)
            q, s = oq.quant_rows(oq.rotate_rows(oq.modulate(xa, nw, ones, zeros, Ms, 1e-6), 128))
            gu = ogemm.epilogue(ogemm.int_mm(q, w["gu"]), s, ws["gu"])
            q, s = oq.quant_rows(oq.rotate_rows(oq.swiglu(gu[:, :F], gu[:, F:]), 128))
            ogemm.epilogue(ogemm.int_mm(q, w["down"]), s, ws["down"], R=xa, G=ones, L=Ms)
            t_lin = time.perf_counter() - t0
            t1 = time.perf_counter()
            oatt.attention_bmm(qa, ka, va)
            t_att = time.perf_counter() - t1
            return 8 * (t_lin * lin_scale + t_att * att_scale) * 1e3, t_lin + t_att
        return run, (f"per sample, one block: 1024 of 6642 rows through the 4 W8A8 linears (oracle pre-pass + "
                     f"torch._int_mm + epilogue; time x {lin_scale:.2f}) and 2 of 48 (batch, head) attention slices "
                     f"(the reference's attention_bmm, fp16; time x 24), x 8 blocks")


def cpu_measure(baseline, threads, reps, warmup=1):
    """Times a workload's CPU sample `reps` times after `warmup` untimed runs; the value is the median of the
    samples' scaled values. Returns (value, description with the measured seconds)."""
    run, desc = baseline(threads)
    for _ in range(warmup):
        run()
    vals, secs = [], []
    for _ in range(reps):
        v, dt = run()
        vals.append(v)
        secs.append(dt)
    return float(np.median(vals)), (f"{desc}. {reps} timed samples after {warmup} untimed: median {float(np.median(secs)):.3f} s "
                                    f"per sample (min {min(secs):.3f}, max {max(secs):.3f}), median value taken")


GATHER = "fused"  # head-group exchange of the sharded DiT stack: "fused" or "nccl" (--gather)

WORKLOADS = {"gemm": GemmC1, "attn": AttnC2, "attn_i8": lambda dev: AttnC2(dev, int8_qk=True), "dit": DiTC4,
             "w4a8": W4A8C3, "gemm_qkv": GemmQKV, "prepass": PrepassC4, "decode": DecodeC5,
             "logits": LogitsC5, "w4a4": W4A4C3}


def reference_arm(args, world, rank):
    """The reference's CPU path (restated: the oracle port, kind "port") on the host cores: W untimed and K timed
    samples of the workload, each scaled to the metric's unit; the value is the median. The reference's own kernels
    also compile for the host (oracle/_ref), but as an emulation of its GPU threads they are a checker, not the
    reference's CPU path, and are not timed here."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    name = args.workload
    meas = lambda baseline: cpu_measure(baseline, threads, max(args.steps, 3), args.warmup)  # noqa: E731
    if name == "gemm":
        v, sample = meas(GemmC1.cpu_baseline)
        metric, unit, higher, cfg = GemmC1.metric, GemmC1.unit, True, GemmC1.config
    elif name in ("attn", "attn_i8"):
        v, sample = meas(lambda t: AttnC2.cpu_baseline(t, name == "attn_i8"))
        w = AttnC2.__new__(AttnC2)
        metric = f"attention TFLOPS (C2: B2 H24 S4056 d128, {'int8' if name == 'attn_i8' else 'fp16'} QK)"
        unit, higher = "TFLOPS", True
        cfg = {"workload": "C2 fused attention", "B": 2, "H": 24, "S": 4056, "d": 128}
    elif name == "w4a8":
        v, sample = meas(W4A8C3.cpu_baseline)
        metric, unit, higher, cfg = W4A8C3.metric, W4A8C3.unit, True, {"workload": "C3 W4A8 linear", "M": 2809,
                                                                         "K": 3072, "N": 8192, "group": 128}
    elif name == "decode":
        v, sample = meas(DecodeC5.cpu_baseline)
        metric, unit, higher = DecodeC5.metric, DecodeC5.unit, False
        cfg = {"workload": "C5 single-token decode", "layers": 36, "hidden": 2560, "kv_len": 1024}
    elif name == "w4a4":
        v, sample = meas(W4A4C3.cpu_baseline)
        metric, unit, higher = W4A4C3.metric, W4A4C3.unit, True
        cfg = {"workload": "C3 shapes, per-channel W4A4", "M": W4A4C3.M, "K": W4A4C3.K, "N": W4A4C3.N}
    elif name == "logits":
        v, sample = meas(LogitsC5.cpu_baseline)
        metric, unit, higher = LogitsC5.metric, LogitsC5.unit, True
        cfg = {"workload": "C5 logits (tied bf16 embedding table)", "N": LogitsC5.N, "K": LogitsC5.K}
    elif name == "dit":
        v, sample = meas(DiTC4.cpu_baseline)
        metric, unit, higher = DiTC4.metric, DiTC4.unit, False
        cfg = {"workload": "C4 DiT block stack", "blocks": 8, "batch": 2, "tokens": 3321, "hidden": 3072, "heads": 24,
               "mlp": 8192}
    else:
        print(json.dumps({"impl": "reference", "unavailable": f"no CPU reference arm for workload {name}"}))
        return
    line = {"metric": metric, "value": v, "unit": unit, "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": higher, "impl": "reference", "dtype": "int8/fp16", "data": "synthetic", "config": cfg,
            "cpu_baseline": {"value": v, "unit": unit, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}, "vs_baseline": None}
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="dit", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gather", default="fused", choices=["fused", "nccl"],
                    help="head-group exchange of the sharded DiT stack (4 or 8 GPUs)")
    ap.add_argument("--decode-mode", default="persistent", choices=["persistent", "layers"],
                    help="C5: one persistent kernel per token, or 9 launches per layer")
    ap.add_argument("--decode-layers", type=int, default=36, help="C5 layers (36; fewer only for ncu captures)")
    args = ap.parse_args()
    global GATHER, DECODE_MODE, DECODE_LAYERS
    GATHER = args.gather
    DECODE_MODE, DECODE_LAYERS = args.decode_mode, args.decode_layers
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks = load_peaks()
    ctor = WORKLOADS[args.workload]
    wl = ctor(dev, world, rank) if ctor is DiTC4 else ctor(dev)

    # Kernel timing pass (dominant kernel), then the timed whole-job pass, then the end-to-end pass.
    for i in range(args.warmup):
        wl.step(i)
    wl.events = []
    for i in range(args.steps):
        wl.step(i, record=True)
    kms = kernel_ms(wl.events) if not isinstance(wl, DiTC4) else None

    with Clocks(local) as clocks:
        # Pre-roll under the sampler so that the clock record covers the load of the timed region that follows. The
        # step count is agreed over ranks (the largest), so every rank issues the same collectives.
        clocks.wait_first()
        pre = max(1, math.ceil(1000.0 / max(timed(wl.step, 1, 0, world), 1e-3)))
        pre = int(max_over_ranks(float(pre), world))
        for i in range(pre):
            wl.step(i)
        torch.cuda.synchronize()
        ms = timed(wl.step, args.steps, args.warmup, world)
    e2e_ms = timed(wl.e2e_step, args.steps, args.warmup, world, begin=getattr(wl, "e2e_begin", None),
                   finish=getattr(wl, "e2e_finish", None))

    line = {"metric": wl.metric, "value": wl.value(ms, args.steps, world), "unit": wl.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": wl.higher, "scaling": "strong" if isinstance(wl, DiTC4) else "weak",
            "vs_baseline": None, "dtype": "int8/fp16", "data": "synthetic (seeded, BASELINE shapes, random-init weights)",
            "config": dict(wl.config, parallelism=(f"cfg x{min(world, 2)} heads x{max(1, world // 2)}" if isinstance(wl, DiTC4)
                                                   else f"replicas x{world}")),
            "e2e": {"value": wl.value(e2e_ms, args.steps, world), "unit": wl.unit,
                    "h2d_bytes_per_step": wl.h2d_bytes, "d2h_bytes_per_step": wl.d2h_bytes},
            "roofline": wl.roofline(peaks, kms), "kernel_ms": kms, "clocks": clocks.summary(),
            "gpu_launches": wl.launches_per_step * args.steps}
    if rank == 0 and world == 1 and not args.no_cpu_baseline and getattr(type(wl), "cpu_baseline", None):
        v, sample = cpu_measure(type(wl).cpu_baseline, os.cpu_count() or 1, 3)
        line["cpu_baseline"] = {"value": v, "unit": wl.unit, "cores": os.cpu_count(), "kind": "port", "sample": sample}
    fused = getattr(wl, "fused", None)
    if fused is not None:
        torch.cuda.synchronize()
        if fused.failed():
            raise RuntimeError(f"rank {rank}: a head-group gather wait ran out (a peer stopped delivering)")
    if rank == 0:
        print(json.dumps(line))
    if fused is not None:
        wl.stack.fused = wl.fused = None
        del fused
        torch.cuda.synchronize()
        barrier(world)
    if world > 1 and dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
