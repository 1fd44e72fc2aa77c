"""Benchmark of the wavo-b200 attention path (BASELINE.json metric: attention audio-sec/sec).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl wavo|reference]

Workloads (synthetic seeded inputs of their shapes and distributions):
  c1  Parakeet/FastConformer rel-pos MHSA layer, f32 weights, T=138, d 1024, 8 x 128
  c2  Whisper large-v3-turbo encoder self-attention, 32 layers, T=1500, d 1280, 20 x 64 (default)
  c3  GigaAM-v3-shaped RoPE attention, 16 layers, d 768, 16 x 48, 16 segments of U[400,750]
  c4  Whisper-turbo decoder attention, 4 layers, batch 32, 224 greedy steps, cross K/V 32x1500
  c5  Parakeet-0.6B long form: 24 rel-pos layers over 400 segments of U[120,300] frames, Q8_0

A step is one pass of the config's unit of work (c2: one 30 s window through 32 layers; c4: one
whole 224-token decode of the batch; c3/c5: the whole batch of segments), captured once as a CUDA
graph and replayed. Every layer's input is a pre-LayerNorm activation ~N(0,1) and its output is
added into an f32 residual stream (the LayerNorm and FFN around the attention are out of scope).
The default is c5, the long-form config: the largest one that fits one GPU and the one whose
1 -> 8 GPU scaling is the target. The multi-segment configs (c3, c4, c5) shard their segments over
the ranks by longest-processing-time-first (strong scaling, no collective) and gather every
segment's output to one host buffer in segment order inside the end-to-end timed region; c1/c2
run one unit per rank (replicas, weak scaling).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "attention audio-sec/sec"
UNIT = "audio-s/s"


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return {"hbm": d["hbm_gbs"], "tensor": d["bf16_tflops"],
                "tensor_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm": 6650.0, "tensor": 1590.0, "tensor_sustained": 1400.0, "source": "fallback"}


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def normal_f16(rng, shape, std):
    return (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float16)


def q8_0_weights(rng, rows, k):
    """GGUF Q8_0 bytes: blocks of 32 int8 ~U[-127,127] with an f16 scale ~|N(0,0.02)|/127."""
    nb = rows * k // 32
    q = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8)
    d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * 0.02 / 127).astype(np.float16)
    out = np.empty((nb, 34), np.uint8)
    out[:, :2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def bf16_weights(rng, rows, k, std):
    w = (rng.standard_normal((rows, k), dtype=np.float32) * std)
    return (w.view(np.uint32) >> 16).astype(np.uint16).tobytes()  # truncated to bf16


def segment_lengths(seed, n, lo, hi):
    return np.random.default_rng(seed).integers(lo, hi + 1, size=n).tolist()


def shard(lengths, rank, world, cost):
    """The plan (LPT over the ranks, deterministic) and this rank's segments costliest first: the
    order they are packed and launched in."""
    from wavo_b200.runner import ShardPlan
    plan = ShardPlan.for_lengths(lengths, world, cost)
    return plan, plan.launch_order(rank)


# ---------------------------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------------------------

class Workload:
    scaling = "weak"
    dtype = "f16 operands, f32 accumulate"
    bound = "tensor"
    # DRAM bytes (read + write) per launch of an op's kernel from one ncu capture at the bench's
    # shapes (dram__bytes_read.sum + dram__bytes_write.sum), when one was taken.
    TRAFFIC: dict = {}

    def audio_s(self) -> float:  # audio seconds this rank processes per step
        raise NotImplementedError

    def total_audio_s(self, world) -> float:  # whole job per step
        return self.audio_s() * world

    # Segment workloads set these: the plan over the ranks, this rank's segments in packed order,
    # every segment's length in rows of the output, and the output's width.
    plan = None
    order = None
    seg_rows = None
    out_width = None

    def host_gather(self, rank):
        """The node-wide segment-ordered host output of this workload's result, or None."""
        if self.plan is None:
            return None
        from wavo_b200.runner import HostGather
        hg = HostGather(self.plan, self.seg_rows, self.out_width, rank, order=self.order)
        return hg if hg.available else None


class C2(Workload):
    """Whisper large-v3-turbo encoder self-attention, 32 layers, batch 1, T=1500."""
    T, D, H, LAYERS = 1500, 1280, 20, 32
    TRAFFIC = {"attention": 11562240, "gemm_qkv": 13730560, "gemm_out": 14854400}

    def __init__(self, gpu, rank, world, seed=2000):
        import torch
        from wavo_b200 import GGML_F16
        from wavo_b200.blocks import EncoderAttention
        self.gpu = gpu
        T, D = self.T, self.D
        rng = np.random.default_rng(seed + rank)
        self.layers = []
        for _ in range(self.LAYERS):
            bqkv = np.concatenate([rng.standard_normal(D, dtype=np.float32) * 0.02,
                                   np.zeros(D, np.float32),  # no bias on k
                                   rng.standard_normal(D, dtype=np.float32) * 0.02])
            self.layers.append(EncoderAttention(
                gpu, GGML_F16, D, self.H, normal_f16(rng, (3 * D, D), 0.02).tobytes(),
                normal_f16(rng, (D, D), 0.02).tobytes(), bqkv,
                rng.standard_normal(D, dtype=np.float32) * 0.02))
        dev = gpu.torch_device
        self.y_host = torch.from_numpy(rng.standard_normal((T, D), dtype=np.float32)).pin_memory()
        self.x_host = torch.empty((T, D), dtype=torch.float32).pin_memory()
        self.y = self.y_host.to(dev)
        self.y16 = torch.empty((T, D), dtype=torch.float16, device=dev)
        self.x = torch.zeros((T, D), dtype=torch.float32, device=dev)
        self.s = self.layers[0].scratch(T)

    def record(self, p, timer=None):
        tick = timer or (lambda name, fn: fn())
        tick("cast", lambda: self.y16.copy_(self.y))
        for lay in self.layers:
            tick("gemm_qkv", lambda: p.gemm(self.y16, lay.qkv, self.s["qkv"], self.T, "bias"))
            tick("attention", lambda: p.attention(self.s["qkv"], None, None, self.s["o"], self.T,
                                                  self.H, self.D // self.H))
            tick("gemm_out", lambda: p.gemm(self.s["o"], lay.out, self.x, self.T, "residual", 1.0))

    def inputs(self):
        return [(self.y, self.y_host)]

    def outputs(self):
        return [(self.x_host, self.x)]

    def launches(self):
        return 1 + 3 * self.LAYERS

    def work(self):
        T, D = self.T, self.D
        return {"gemm_qkv": 2.0 * T * D * 3 * D, "gemm_out": 2.0 * T * D * D,
                "attention": 4.0 * T * T * D, "cast": 0.0}

    def audio_s(self):
        return 30.0

    def config(self):
        return {"workload": "C2: Whisper large-v3-turbo encoder self-attention, 32 layers, T=1500",
                "global_batch": 1, "seq_len": self.T, "d_model": self.D, "heads": self.H,
                "head_dim": self.D // self.H, "layers": self.LAYERS, "weights": "f16 ~N(0,0.02)",
                "l2": "no flush: the step's weights (419 MB) exceed the 126 MB L2",
                "parallelism": "replicas (independent windows), no collective"}

    @staticmethod
    def cpu_sample(layers=1, seed=1):
        from oracle import oracle as O
        T, D, H = 1500, 1280, 20
        rng = np.random.default_rng(seed)
        y = rng.standard_normal(T * D, dtype=np.float32)
        x = np.zeros(T * D, np.float32)
        lins = [(O.Linear(O.TY_F16, 3 * D, D, normal_f16(rng, (3 * D, D), 0.02).tobytes(),
                          np.zeros(3 * D, np.float32)),
                 O.Linear(O.TY_F16, D, D, normal_f16(rng, (D, D), 0.02).tobytes(),
                          np.zeros(D, np.float32))) for _ in range(layers)]
        t0 = time.perf_counter()
        for lq, lo in lins:
            qkv = lq.gemm(y, T)
            o = O.attention(qkv, 3 * D, np.ascontiguousarray(qkv[2 * D:]), 3 * D, T, H, D)
            lo.gemm(np.ascontiguousarray(o.ravel()), T, x, "residual", 1.0)
        return time.perf_counter() - t0, 30.0 * layers / 32, f"{layers} of 32 layers of a C2 window"


class RelPosWorkload(Workload):
    """Parakeet rel-pos MHSA layers over segments (C1: one layer, one segment of 138, f32
    weights; C5: 24 layers, 400 segments of U[120,300], Q8_0 weights, sharded)."""
    D, H = 1024, 8
    FRAME_S = 0.08

    def __init__(self, gpu, rank, world, lengths, layers, ty_name, seed):
        import torch
        from wavo_b200 import GGML_F32, GGML_Q8_0
        from wavo_b200.blocks import RelPosAttention, Segments, rel_positions
        self.gpu, self.layers_n, self.world = gpu, layers, world
        D = self.D
        self.all_lengths = lengths
        cost = lambda t: 24 * (6 * t * t * D + 10 * t * D * D)  # noqa: E731
        self.plan, mine = shard(lengths, rank, world, cost)
        self.order, self.seg_rows, self.out_width = mine, list(lengths), D
        self.lengths = [lengths[i] for i in mine]
        rng = np.random.default_rng(seed)  # the same weights on every rank
        ty = GGML_Q8_0 if ty_name == "q8_0" else GGML_F32
        self.blocks = []
        for _ in range(layers):
            if ty == GGML_Q8_0:
                wqkv, wpos, wout = (q8_0_weights(rng, 3 * D, D), q8_0_weights(rng, D, D),
                                    q8_0_weights(rng, D, D))
            else:
                wqkv = (rng.standard_normal((3 * D, D), dtype=np.float32) * 0.02).tobytes()
                wpos = (rng.standard_normal((D, D), dtype=np.float32) * 0.02).tobytes()
                wout = (rng.standard_normal((D, D), dtype=np.float32) * 0.02).tobytes()
            u = rng.standard_normal(D, dtype=np.float32) * 0.02
            v = rng.standard_normal(D, dtype=np.float32) * 0.02
            self.blocks.append(RelPosAttention(gpu, ty, D, self.H, wqkv, wpos, wout, u, v))
        dev = gpu.torch_device
        self.segs = Segments(self.lengths, dev)
        rows = self.segs.rows
        self.t_pos = max(lengths)
        self.table = gpu.upload(rel_positions(D, self.t_pos + 15, 2 * self.t_pos + 15))
        drng = np.random.default_rng(seed + 1 + rank)
        self.y_host = torch.from_numpy(drng.standard_normal((rows, D), dtype=np.float32)).pin_memory()
        self.x_host = torch.empty((rows, D), dtype=torch.float32).pin_memory()
        self.y = self.y_host.to(dev)
        self.y16 = torch.empty((rows, D), dtype=torch.float16, device=dev)
        self.x = torch.zeros((rows, D), dtype=torch.float32, device=dev)
        self.s = self.blocks[0].scratch(rows, self.t_pos)

    def record(self, p, timer=None):
        tick = timer or (lambda name, fn: fn())
        rows, D = self.segs.rows, self.D
        tick("cast", lambda: self.y16.copy_(self.y))
        from wavo_b200.gpu import pos_rows
        for b in self.blocks:
            tick("gemm_qkv", lambda: p.gemm(self.y16, b.qkv, self.s["qkv"], rows, "bias"))
            tick("gemm_pos", lambda: p.gemm(self.table, b.pos, self.s["p"], pos_rows(self.t_pos),
                                            "bias"))
            tick("attention", lambda: p.attention_varlen(
                self.s["qkv"], None, self.s["p"], self.s["o"], rows, self.segs.start_t,
                self.segs.len_t, self.segs.max_len, self.H, D // self.H, self.t_pos))
            tick("gemm_out", lambda: p.gemm(self.s["o"], b.out, self.x, rows, "residual", 1.0))

    def inputs(self):
        return [(self.y, self.y_host)]

    def outputs(self):
        return [(self.x_host, self.x)]

    def launches(self):
        return 1 + 4 * self.layers_n

    def work(self):
        D = self.D
        rows = self.segs.rows
        att = sum(6.0 * t * t * D for t in self.lengths)  # AC + BD + PV (the reference's count)
        # The QKV GEMM multiplies 3D columns; its fourth section (q + v) is the epilogue writing q
        # a second time with the other bias (the reference's dual outputs).
        return {"gemm_qkv": 2.0 * rows * D * 3 * D, "gemm_out": 2.0 * rows * D * D,
                "gemm_pos": 2.0 * (2 * self.t_pos + 15) * D * D, "attention": att, "cast": 0.0}

    def audio_s(self):
        return sum(self.lengths) * self.FRAME_S

    def total_audio_s(self, world):
        return sum(self.all_lengths) * self.FRAME_S


class C1(RelPosWorkload):
    scaling = "weak"

    def __init__(self, gpu, rank, world, seed=1000):
        # One unit per rank (replicas): every rank runs the same single segment on its own.
        super().__init__(gpu, 0, 1, [138], 1, "f32", seed)
        self.plan = None

    def total_audio_s(self, world):
        return self.audio_s() * world

    def config(self):
        return {"workload": "C1: Parakeet rel-pos MHSA layer, f32 weights, batch 1, T=138",
                "global_batch": 1, "seq_len": 138, "d_model": 1024, "heads": 8, "head_dim": 128,
                "layers": 1, "weights": "f32 ~N(0,0.02) (rounded to f16 in the GEMM, as the "
                "reference GPU GEMM)", "l2": "small working set: L2-resident (latency-bound)",
                "parallelism": "replicas, no collective"}

    @staticmethod
    def cpu_sample(layers=1, seed=1):
        return RelPosWorkload.cpu(seed, [138], layers, "f32", 1)


def _relpos_cpu(seed, lengths, layers, ty_name, reps):
    from oracle import oracle as O
    D, H = 1024, 8
    rng = np.random.default_rng(seed)
    lins = []
    for _ in range(layers):
        if ty_name == "q8_0":
            ws = [(O.TY_Q8_0, q8_0_weights(rng, r, D)) for r in (3 * D, D, D)]
        else:
            ws = [(O.TY_F32, (rng.standard_normal((r, D), dtype=np.float32) * 0.02).tobytes())
                  for r in (3 * D, D, D)]
        lins.append([O.Linear(ty, r, D, data) for (ty, data), r in zip(ws, (3 * D, D, D))] +
                    [rng.standard_normal(D, dtype=np.float32) * 0.02,
                     rng.standard_normal(D, dtype=np.float32) * 0.02])
    ys = [np.random.default_rng(seed + 7 + i).standard_normal(t * D, dtype=np.float32)
          for i, t in enumerate(lengths)]
    t0 = time.perf_counter()
    for _ in range(reps):
        for y, t in zip(ys, lengths):
            x = np.zeros(t * D, np.float32)
            tab = O.rel_positions(D, t + 15, O.pos_rows(t))
            for lq, lp, lo, u, v in lins:
                qkv = lq.gemm(y, t)
                pos = lp.gemm(np.ascontiguousarray(tab.ravel()), O.pos_rows(t))
                o = O.relative_attention(qkv, pos, u, v, t, H, D)
                lo.gemm(np.ascontiguousarray(o.ravel()), t, x, "residual", 1.0)
    return time.perf_counter() - t0


RelPosWorkload.cpu = staticmethod(
    lambda seed, lengths, layers, ty, reps: (
        _relpos_cpu(seed, lengths, layers, ty, reps),
        reps * sum(lengths) * 0.08 * layers / (24 if ty == "q8_0" else 1),
        f"{reps} x {len(lengths)} segment(s) {lengths[:4]}... through {layers} layer(s)"))


class C5(RelPosWorkload):
    scaling = "strong"
    TRAFFIC = {"attention": 708701440 + 159529728, "gemm_qkv": 180414720 + 644850432}

    def __init__(self, gpu, rank, world, seed=5000):
        super().__init__(gpu, rank, world, segment_lengths(seed, 400, 120, 300), 24, "q8_0", seed)

    def config(self):
        return {"workload": "C5: Parakeet-0.6B long form, 24 rel-pos layers, 400 segments of "
                "U[120,300] frames, Q8_0 weights", "global_batch": 400, "seq_len": "120-300",
                "total_frames": int(sum(self.all_lengths)), "d_model": 1024, "heads": 8,
                "head_dim": 128, "layers": 24, "weights": "GGUF Q8_0 (dequantized to f16 at load)",
                "l2": "inputs larger than L2", "parallelism": f"segments sharded LPT over "
                f"{self.world} GPU(s), no collective"}

    @staticmethod
    def cpu_sample(layers=2, seed=5000):
        # Every 25th of the 400 segments (16, spanning the length distribution) through 2 of the
        # 24 identical layers, scaled to the set by their audio seconds.
        lens = segment_lengths(seed, 400, 120, 300)[::25]
        return RelPosWorkload.cpu(seed, lens, layers, "q8_0", 1)


class C5Block(Workload):
    """Whole Parakeet 0.6B FastConformer blocks (the caller side of the attention path, the
    reference's Block::record, src/conformer.rs:232-265) over C5's 400 segments: 24 blocks of
    d 1024, FFN 4096, 8 heads of 128, conv kernel 9 with the folded batch norm, Q8_0 weights."""
    D, H, F, KERNEL, LAYERS = 1024, 8, 4096, 9, 24
    FRAME_S = 0.08
    scaling = "strong"
    METRIC = "encoder-block audio-sec/sec"

    def __init__(self, gpu, rank, world, seed=5000):
        import torch
        from wavo_b200 import GGML_Q8_0
        from wavo_b200.blocks import ConformerBlock, Segments, rel_positions
        self.gpu, self.world = gpu, world
        D, F = self.D, self.F
        lengths = segment_lengths(seed, 400, 120, 300)
        self.all_lengths = lengths
        cost = lambda t: 24 * (6 * t * t * D + (12 + 8 * F // D) * t * D * D)  # noqa: E731
        self.plan, mine = shard(lengths, rank, world, cost)
        self.order, self.seg_rows, self.out_width = mine, list(lengths), D
        self.lengths = [lengths[i] for i in mine]
        rng = np.random.default_rng(seed)
        self.blocks = []
        for _ in range(self.LAYERS):
            w = {"ff1_1": q8_0_weights(rng, F, D), "ff1_2": q8_0_weights(rng, D, F),
                 "ff2_1": q8_0_weights(rng, F, D), "ff2_2": q8_0_weights(rng, D, F),
                 "qkv": q8_0_weights(rng, 3 * D, D), "pos": q8_0_weights(rng, D, D),
                 "out": q8_0_weights(rng, D, D), "pw1": q8_0_weights(rng, 2 * D, D),
                 "pw2": q8_0_weights(rng, D, D),
                 "u": rng.standard_normal(D, dtype=np.float32) * 0.02,
                 "v": rng.standard_normal(D, dtype=np.float32) * 0.02,
                 "dw": rng.standard_normal((D, self.KERNEL), dtype=np.float32) * 0.2,
                 "dw_b": rng.standard_normal(D, dtype=np.float32) * 0.02}
            norms = {k: (1.0 + rng.standard_normal(D, dtype=np.float32) * 0.1,
                         rng.standard_normal(D, dtype=np.float32) * 0.1)
                     for k in ("ff1", "attn", "conv", "ff2", "out", "conv_norm")}
            self.blocks.append(ConformerBlock(gpu, GGML_Q8_0, D, F, self.H, self.KERNEL, w, norms,
                                              conv_ln=False))
        dev = gpu.torch_device
        self.segs = Segments(self.lengths, dev)
        rows = self.segs.rows
        self.t_pos = max(lengths)
        self.table = gpu.upload(rel_positions(D, self.t_pos + 15, 2 * self.t_pos + 15),
                                torch.float16)
        drng = np.random.default_rng(seed + 1 + rank)
        self.y_host = torch.from_numpy(drng.standard_normal((rows, D), dtype=np.float32)).pin_memory()
        self.x_host = torch.empty((rows, D), dtype=torch.float32).pin_memory()
        self.y = self.y_host.to(dev)
        self.xa = torch.zeros((rows, D), dtype=torch.float32, device=dev)
        self.xb = torch.zeros((rows, D), dtype=torch.float32, device=dev)
        self.s = self.blocks[0].scratch(rows, self.t_pos)

    def record(self, p, timer=None):
        tick = timer or (lambda name, fn: fn())
        tick("cast", lambda: self.xa.copy_(self.y))
        src, dst = self.xa, self.xb
        for b in self.blocks:
            b.record(p, src, dst, self.segs, self.table, self.t_pos, self.s, tick)
            src, dst = dst, src
        self.result = src

    def inputs(self):
        return [(self.y, self.y_host)]

    def outputs(self):
        return [(self.x_host, self.xa if self.LAYERS % 2 == 0 else self.xb)]

    def launches(self):
        return 1 + sum(b.launches() for b in self.blocks)

    def work(self):
        D, F, rows = self.D, self.F, self.segs.rows
        return {"gemm_ff1": 2.0 * rows * D * F, "gemm_ff2": 2.0 * rows * D * F,
                "gemm_qkv": 2.0 * rows * D * 3 * D, "gemm_out": 2.0 * rows * D * D,
                "gemm_pos": 2.0 * (2 * self.t_pos + 15) * D * D,
                "attention": sum(6.0 * t * t * D for t in self.lengths),
                "gemm_pw1": 2.0 * rows * D * 2 * D, "gemm_pw2": 2.0 * rows * D * D,
                "layer_norm": 0.0, "conv_glu": 0.0, "cast": 0.0}

    def audio_s(self):
        return sum(self.lengths) * self.FRAME_S

    def total_audio_s(self, world):
        return sum(self.all_lengths) * self.FRAME_S

    def config(self):
        return {"workload": "C5 blocks: Parakeet-0.6B FastConformer blocks (FFN, rel-pos MHSA, "
                "conv module, norms), 24 blocks, 400 segments of U[120,300] frames, Q8_0 weights",
                "global_batch": 400, "seq_len": "120-300",
                "total_frames": int(sum(self.all_lengths)), "d_model": 1024, "d_ff": 4096,
                "heads": 8, "head_dim": 128, "conv_kernel": 9, "layers": 24,
                "weights": "GGUF Q8_0 (dequantized to f16 at load)", "l2": "inputs larger than L2",
                "parallelism": f"segments sharded LPT over {self.world} GPU(s), no collective"}

    @staticmethod
    def cpu_sample(layers=1, seed=5000):
        # Every 50th of the 400 segments (8, spanning the length distribution) through one block
        # of the CPU oracle (src/cpu/conformer.rs:159-199), scaled to the set by audio seconds.
        from oracle import oracle as O
        D, F, H, K = 1024, 4096, 8, 9
        lens = segment_lengths(seed, 400, 120, 300)[::50]
        rng = np.random.default_rng(seed)
        lin = lambda n, k: O.Linear(O.TY_Q8_0, n, k, q8_0_weights(rng, n, k))  # noqa: E731
        ff = [lin(F, D), lin(D, F), lin(F, D), lin(D, F)]
        lq, lp, lo, l1, l2 = lin(3 * D, D), lin(D, D), lin(D, D), lin(2 * D, D), lin(D, D)
        u, v = (rng.standard_normal(D, dtype=np.float32) * 0.02 for _ in range(2))
        taps = np.ascontiguousarray(rng.standard_normal((K, D), dtype=np.float32) * 0.2)
        dw_b = np.zeros(D, np.float32)
        nw, nb = np.ones(D, np.float32), np.zeros(D, np.float32)
        xs = [rng.standard_normal(t * D, dtype=np.float32) for t in lens]
        t0 = time.perf_counter()
        for x, t in zip(xs, lens):
            for _ in range(layers):
                y = O.layer_norm(x, nw, nb, t, D)
                ff[1].gemm(ff[0].gemm(y, t, epilogue="silu"), t, x, "residual", 0.5)
                y = O.layer_norm(x, nw, nb, t, D)
                pos = lp.gemm(np.ascontiguousarray(O.rel_positions(D, t + 15, O.pos_rows(t)).ravel()),
                              O.pos_rows(t))
                o = O.relative_attention(lq.gemm(y, t), pos, u, v, t, H, D)
                lo.gemm(np.ascontiguousarray(o.ravel()), t, x, "residual", 1.0)
                y = O.layer_norm(x, nw, nb, t, D)
                yc = O.conv_glu(l1.gemm(y, t), taps, dw_b, nw, nb, False, t, D, K)
                l2.gemm(yc, t, x, "residual", 1.0)
                y = O.layer_norm(x, nw, nb, t, D)
                ff[3].gemm(ff[2].gemm(y, t, epilogue="silu"), t, x, "residual", 0.5)
                x = O.layer_norm(x, nw, nb, t, D)
        dt = time.perf_counter() - t0
        audio = sum(lens) * 0.08 * layers / 24
        return dt, audio, f"{len(lens)} of 400 segments through {layers} of 24 blocks"


class C3(Workload):
    """GigaAM-v3-shaped attention with RoPE: 16 layers, d 768, 16 x 48, 16 segments."""
    D, H, LAYERS = 768, 16, 16
    FRAME_S = 0.04
    scaling = "strong"
    # DRAM read + write of one attention launch at 1 GPU (ncu capture of this config).
    TRAFFIC = {"attention": 40322048 + 291584}

    def __init__(self, gpu, rank, world, seed=3000):
        import torch
        from wavo_b200 import GGML_BF16
        from wavo_b200.blocks import RotaryAttention, Segments
        self.gpu, self.world = gpu, world
        D = self.D
        self.all_lengths = segment_lengths(seed, 16, 400, 750)
        cost = lambda t: 16 * (4 * t * t * D + 8 * t * D * D)  # noqa: E731
        self.plan, mine = shard(self.all_lengths, rank, world, cost)
        self.order, self.seg_rows, self.out_width = mine, list(self.all_lengths), D
        self.lengths = [self.all_lengths[i] for i in mine]
        rng = np.random.default_rng(seed)
        self.blocks = [RotaryAttention(gpu, GGML_BF16, D, self.H, bf16_weights(rng, 3 * D, D, 0.02),
                                       bf16_weights(rng, D, D, 0.02), theta=10000.0,
                                       max_frames=750) for _ in range(self.LAYERS)]
        dev = gpu.torch_device
        self.segs = Segments(self.lengths, dev)
        rows = self.segs.rows
        drng = np.random.default_rng(seed + 1 + rank)
        self.y_host = torch.from_numpy(drng.standard_normal((rows, D), dtype=np.float32)).pin_memory()
        self.x_host = torch.empty((rows, D), dtype=torch.float32).pin_memory()
        self.y = self.y_host.to(dev)
        self.y16 = torch.empty((rows, D), dtype=torch.float16, device=dev)
        self.x = torch.zeros((rows, D), dtype=torch.float32, device=dev)
        self.s = self.blocks[0].scratch(rows)

    def record(self, p, timer=None):
        tick = timer or (lambda name, fn: fn())
        rows, D, H = self.segs.rows, self.D, self.H
        tick("cast", lambda: self.y16.copy_(self.y))
        for b in self.blocks:
            tick("gemm_qkv", lambda: p.gemm(self.y16, b.qkv, self.s["qkv"], rows, "bias"))
            # RoPE as its own pass (faster here than the rotation inside the attention kernel,
            # wavo_attention_rope_varlen: 12.5 + 54.3 us against 72.9 us a layer).
            tick("rope", lambda: p.rope_rows(b.table, self.s["qkv"], rows, self.segs.positions,
                                             (H, D // H, D // H), True))
            tick("attention", lambda: p.attention_varlen(
                self.s["qkv"], None, None, self.s["o"], rows, self.segs.start_t, self.segs.len_t,
                self.segs.max_len, H, D // H))
            tick("gemm_out", lambda: p.gemm(self.s["o"], b.out, self.x, rows, "residual", 1.0))

    def inputs(self):
        return [(self.y, self.y_host)]

    def outputs(self):
        return [(self.x_host, self.x)]

    def launches(self):
        return 1 + 4 * self.LAYERS

    def work(self):
        D, rows = self.D, self.segs.rows
        return {"gemm_qkv": 2.0 * rows * D * 3 * D, "gemm_out": 2.0 * rows * D * D,
                "attention": sum(4.0 * t * t * D for t in self.lengths), "rope": 0.0, "cast": 0.0}

    def audio_s(self):
        return sum(self.lengths) * self.FRAME_S

    def total_audio_s(self, world):
        return sum(self.all_lengths) * self.FRAME_S

    def config(self):
        return {"workload": "C3: GigaAM-v3-shaped RoPE attention, 16 layers, 16 segments of "
                "U[400,750] frames (key-padding mask as per-segment lengths)", "global_batch": 16,
                "seq_len": "400-750", "total_frames": int(sum(self.all_lengths)), "d_model": 768,
                "heads": 16, "head_dim": 48, "layers": 16,
                "rope": "base 10000 on Q/K, NEOX",
                "weights": "bf16 ~N(0,0.02) (converted to f16 at load)",
                "parallelism": f"segments sharded LPT over {self.world} GPU(s), no collective"}

    @staticmethod
    def cpu_sample(layers=1, seed=3000):
        from oracle import oracle as O
        D, H = 768, 16
        t = segment_lengths(seed, 16, 400, 750)[0]
        rng = np.random.default_rng(seed)
        lq = O.Linear(O.TY_F32, 3 * D, D, (rng.standard_normal((3 * D, D), dtype=np.float32) *
                                          0.02).tobytes())
        lo = O.Linear(O.TY_F32, D, D, (rng.standard_normal((D, D), dtype=np.float32) * 0.02)
                      .tobytes())
        y = rng.standard_normal(t * D, dtype=np.float32)
        tab = O.rope_table(t, D // H, 10000.0)
        x = np.zeros(t * D, np.float32)
        t0 = time.perf_counter()
        for _ in range(layers):
            qkv = lq.gemm(y, t)
            O.rope(qkv, tab, t, H, D // H, D // H, True)
            o = O.attention(qkv, 3 * D, np.ascontiguousarray(qkv[2 * D:]), 3 * D, t, H, D)
            lo.gemm(np.ascontiguousarray(o.ravel()), t, x, "residual", 1.0)
        return (time.perf_counter() - t0, t * 0.04 * layers / 16,
                f"1 segment of {t} frames through {layers} of 16 layers")


class C4(Workload):
    """Whisper-turbo decoder attention: 4 layers, batch 32, 224 greedy steps over F16 caches."""
    D, H, LAYERS, FRAMES, CONTEXT, STEPS, BATCH = 1280, 20, 4, 1500, 448, 224, 32
    scaling = "strong"
    bound = "hbm"
    TRAFFIC = {"attend_cross": 245957376 + 3753216, "gemv_self_out": 3638016}

    def __init__(self, gpu, rank, world, seed=4000):
        import torch
        from wavo_b200 import GGML_F16
        from wavo_b200.blocks import DecoderAttention
        self.gpu, self.world = gpu, world
        D = self.D
        # Decode streams of equal cost: longest-first over the ranks deals them round-robin.
        self.plan, _ = shard([1] * self.BATCH, rank, world, lambda t: 1)
        self.order = self.plan.mine(rank)
        self.seg_rows, self.out_width = [1] * self.BATCH, D
        self.batch = len(self.order)
        rng = np.random.default_rng(seed)
        self.layers = []
        for _ in range(self.LAYERS):
            w = {"qkv": normal_f16(rng, (3 * D, D), 0.02).tobytes(),
                 "self_out": normal_f16(rng, (D, D), 0.02).tobytes(),
                 "cross_q": normal_f16(rng, (D, D), 0.02).tobytes(),
                 "cross_kv": normal_f16(rng, (2 * D, D), 0.02).tobytes(),
                 "cross_out": normal_f16(rng, (D, D), 0.02).tobytes()}
            b = {"qkv": np.concatenate([rng.standard_normal(D, dtype=np.float32) * 0.02,
                                        np.zeros(D, np.float32),
                                        rng.standard_normal(D, dtype=np.float32) * 0.02]),
                 "cross_kv": np.concatenate([np.zeros(D, np.float32),
                                             rng.standard_normal(D, dtype=np.float32) * 0.02])}
            self.layers.append(DecoderAttention(gpu, GGML_F16, D, self.H, self.CONTEXT,
                                                self.FRAMES, self.batch, w, b))
        dev = gpu.torch_device
        drng = np.random.default_rng(seed + 1 + rank)
        # The one-time cross K/V of the batch: encoder outputs ~N(0,1), projected and packed.
        enc = torch.from_numpy(drng.standard_normal((self.batch, self.FRAMES, D),
                                                    dtype=np.float32)).to(dev)
        p = gpu.pass_()
        t0 = time.perf_counter()
        for lay in self.layers:
            lay.record_cross(p, enc)
        gpu.sync()
        self.cross_setup_s = time.perf_counter() - t0
        del enc
        self.y_host = torch.from_numpy(drng.standard_normal((2, self.batch, D),
                                                            dtype=np.float32)).pin_memory()
        self.x_host = torch.empty((self.batch, D), dtype=torch.float32).pin_memory()
        self.y = self.y_host.to(dev)
        self.x = torch.zeros((self.batch, D), dtype=torch.float32, device=dev)

    def record(self, p, timer=None):
        tick = timer or (lambda name, fn: fn())
        for pos in range(self.STEPS):
            for lay in self.layers:
                if timer is None:
                    lay.record_step(p, self.y[0], self.y[1], self.x, pos)
                else:
                    self._timed_step(p, lay, pos, tick)

    def _timed_step(self, p, lay, pos, tick):
        d, B = self.D, self.batch
        tick("gemv_qkv", lambda: p.gemv_rows(self.y[0], lay.qkv, lay.qkv_buf, B, "bias",
                                             ldc=3 * d))
        tick("pack", lambda: p.pack_batch(lay.qkv_buf, (d, 0), 3 * d, lay.own, d * lay.context, 1,
                                          d, (lay.context, pos), B))
        tick("attend_self", lambda: p.attend_batch(lay.qkv_buf, 3 * d, lay.own, d * lay.context,
                                                   lay.part, lay.att, d, pos + 1, lay.context,
                                                   lay.heads, lay.hd, B))
        tick("gemv_self_out", lambda: p.gemv_rows(lay.att, lay.self_out, self.x, B, "residual",
                                                  1.0, ldc=d))
        tick("gemv_cross_q", lambda: p.gemv_rows(self.y[1], lay.cross_q, lay.q_buf, B, "bias",
                                                 ldc=d))
        tick("attend_cross", lambda: p.attend_batch(lay.q_buf, d, lay.cross, d * lay.frames,
                                                    lay.part, lay.att, d, lay.frames, lay.frames,
                                                    lay.heads, lay.hd, B))
        tick("gemv_cross_out", lambda: p.gemv_rows(lay.att, lay.cross_out, self.x, B, "residual",
                                                   1.0, ldc=d))

    def inputs(self):
        return [(self.y, self.y_host)]

    def outputs(self):
        return [(self.x_host, self.x)]

    def launches(self):
        # per layer and step: 5 projections, pack, 2 attends (the cross one with its combine)
        return self.STEPS * self.LAYERS * (5 + 1 + 1 + 2)

    def work(self):
        d, B, T = self.D, self.batch, self.FRAMES
        # HBM bytes per launch: the caches of the batch (K and V, f16; the self cache averaged
        # over the steps), and for a projection its f16 weights plus the f32 rows in and out.
        proj = lambda n, k: 2.0 * n * k + 4.0 * B * (n + k)  # noqa: E731
        return {"attend_cross": 2.0 * B * T * d * 2,
                "attend_self": 2.0 * B * (self.STEPS + 1) / 2 * d * 2,
                "gemv_qkv": proj(3 * d, d), "gemv_self_out": proj(d, d),
                "gemv_cross_q": proj(d, d), "gemv_cross_out": proj(d, d), "pack": 0.0}

    def audio_s(self):
        return self.batch * 30.0

    def total_audio_s(self, world):
        return self.BATCH * 30.0

    def config(self):
        return {"workload": "C4: Whisper-turbo decoder attention, 4 layers, batch 32, 224 greedy "
                "steps, self + cross attention over F16 caches", "global_batch": self.BATCH,
                "seq_len": f"{self.CONTEXT} context, {self.FRAMES} frames", "d_model": self.D,
                "heads": self.H, "head_dim": self.D // self.H, "layers": self.LAYERS,
                "steps": self.STEPS, "weights": "f16 ~N(0,0.02)",
                "cross_kv_setup_s": round(self.cross_setup_s, 4),
                "l2": "cross K/V caches (983 MB per step) exceed L2",
                "parallelism": f"segments split over {self.world} GPU(s), no collective"}

    @staticmethod
    def cpu_sample(layers=1, seed=4000):
        from oracle import oracle as O
        d, H, T = 1280, 20, 1500
        rng = np.random.default_rng(seed)
        kv = rng.standard_normal(T * 2 * d, dtype=np.float32)
        cache = np.zeros(T * 2 * d, np.float32)
        O.pack_cache(kv, T, d, d // H, cache, T, 0)
        q = rng.standard_normal(d, dtype=np.float32)
        lq = O.Linear(O.TY_F16, d, d, normal_f16(rng, (d, d), 0.02).tobytes())
        steps = 32
        t0 = time.perf_counter()
        for _ in range(steps):
            qq = lq.gemv(q)
            O.attend(qq, cache, T, T, H, d // H)
        dt = time.perf_counter() - t0
        # one cross attend + one projection per (segment, layer, step); scale to the unit
        return dt, 30.0 * steps / (224 * 4), f"{steps} cross-attention steps of one segment"


class C4Full(Workload):
    """The whole Whisper large-v3-turbo decoder for a batch of 32 windows, kept on the device: 224
    greedy steps of embedding, 4 decoder layers (LayerNorms, self attention over the growing F16
    cache, cross attention over the 1500 encoder frames, FFN 5120 with GELU), final LayerNorm,
    logits over the 51 866-token vocabulary through the tied embedding, and the greedy pick with
    the suppression and timestamp rules (src/transformer.rs:254-290, src/whisper/search.rs:35-123);
    tokens never leave the GPU. EOT is in the suppression list so that every window runs all 224
    steps (the config's fixed decode length)."""
    D, H, F, LAYERS, FRAMES, CONTEXT, STEPS, BATCH, VOCAB = 1280, 20, 5120, 4, 1500, 448, 224, 32, 51866
    EOT, NO_TS, BEGIN = 50257, 50364, 50365
    scaling = "strong"
    bound = "hbm"
    METRIC = "decoder audio-sec/sec"

    def __init__(self, gpu, rank, world, seed=4100):
        import torch
        from wavo_b200 import GGML_F16
        from wavo_b200.blocks import WhisperDecoder
        self.gpu, self.world = gpu, world
        D, F = self.D, self.F
        self.plan, _ = shard([1] * self.BATCH, rank, world, lambda t: 1)
        self.order = self.plan.mine(rank)
        self.seg_rows, self.out_width = [1] * self.BATCH, 1
        self.batch = len(self.order)
        rng = np.random.default_rng(seed)
        vec = lambda n: rng.standard_normal(n, dtype=np.float32) * 0.02  # noqa: E731
        norm = lambda: (1.0 + vec(D), vec(D))  # noqa: E731
        layers = []
        for _ in range(self.LAYERS):
            lw = {"qkv": normal_f16(rng, (3 * D, D), 0.02).tobytes(),
                  "self_out": normal_f16(rng, (D, D), 0.02).tobytes(),
                  "cross_q": normal_f16(rng, (D, D), 0.02).tobytes(),
                  "cross_kv": normal_f16(rng, (2 * D, D), 0.02).tobytes(),
                  "cross_out": normal_f16(rng, (D, D), 0.02).tobytes(),
                  "fc1": normal_f16(rng, (F, D), 0.02).tobytes(),
                  "fc2": normal_f16(rng, (D, F), 0.02).tobytes(),
                  "b": {"qkv": np.concatenate([vec(D), np.zeros(D, np.float32), vec(D)]),
                        "self_out": vec(D), "cross_q": vec(D),
                        "cross_kv": np.concatenate([np.zeros(D, np.float32), vec(D)]),
                        "cross_out": vec(D)},
                  "fc1_b": vec(F), "fc2_b": vec(D),
                  "norm_self": norm(), "norm_cross": norm(), "norm_ffn": norm()}
            layers.append(lw)
        w = {"embed": normal_f16(rng, (self.VOCAB, D), 0.02).tobytes(),
             "positions": rng.standard_normal((self.CONTEXT, D), dtype=np.float32) * 0.02,
             "norm": norm(), "layers": layers}
        suppress = sorted(set(int(i) for i in rng.integers(0, self.EOT, 88)) | {self.EOT})
        ids = {"eot": self.EOT, "no_timestamps": self.NO_TS, "begin": self.BEGIN,
               "suppress": suppress, "begin_suppress": [220]}
        self.dec = WhisperDecoder(gpu, GGML_F16, D, self.H, F, self.VOCAB, self.CONTEXT,
                                  self.FRAMES, self.batch, w, ids)
        dev = gpu.torch_device
        drng = np.random.default_rng(seed + 1 + rank)
        enc = torch.from_numpy(drng.standard_normal((self.batch, self.FRAMES, D),
                                                    dtype=np.float32)).to(dev)
        self.dec.record_cross(gpu.pass_(), enc)
        gpu.sync()
        del enc
        # Inputs: each window's last prompt token; result: the generated tokens.
        self.tok_host = torch.full((self.batch,), 50360, dtype=torch.int32).pin_memory()
        self.out_host = torch.empty((self.batch, self.CONTEXT), dtype=torch.int32).pin_memory()

    def record(self, p, timer=None):
        tick = timer or (lambda name, fn: fn())
        tick("reset", lambda: self.dec.hist_len.zero_())
        for pos in range(self.STEPS):
            self.dec.record_step(p, pos, tick)

    def profile_unit(self, p):
        """One greedy step (at position 13, after the steps before it, which are not profiled)."""
        self.dec.hist_len.zero_()
        for pos in range(13):
            self.dec.record_step(p, pos)
        self.gpu.sync()
        import torch
        torch.cuda.profiler.start()
        self.dec.record_step(p, 13)

    def host_gather(self, rank):
        return None  # each rank reads back its own windows' tokens

    def inputs(self):
        return [(self.dec.tokens, self.tok_host)]

    def outputs(self):
        return [(self.out_host, self.dec.history)]

    def launches(self):
        return self.STEPS * self.dec.launches_per_step()

    def work(self):
        # HBM bytes a call of each group reads and writes (f16 weights, f16 caches, f32 rows).
        D, F, B = self.D, self.F, self.batch
        mean_n = (self.STEPS + 1) / 2  # self-attention keys, averaged over the steps
        return {"cross_attention": 2.0 * D * D * 2 + B * self.FRAMES * D * 2 * 2,
                "self_attention": 2.0 * 4 * D * D + B * mean_n * D * 2 * 2,
                "ffn": 2.0 * 2 * D * F, "logits": 2.0 * self.VOCAB * D + 4.0 * B * self.VOCAB,
                "pick": 4.0 * B * self.VOCAB, "layer_norm": 4.0 * 2 * B * D,
                "embed": 2.0 * B * D + 4.0 * B * D, "reset": 0.0}

    def audio_s(self):
        return self.batch * 30.0

    def total_audio_s(self, world):
        return self.BATCH * 30.0

    def config(self):
        return {"workload": "C4 full decoder: Whisper large-v3-turbo decoder (4 layers, d 1280, "
                "FFN 5120, vocabulary 51866), batch 32, 224 greedy steps on the device",
                "global_batch": self.BATCH, "seq_len": self.STEPS, "d_model": self.D,
                "heads": self.H, "layers": self.LAYERS, "frames": self.FRAMES,
                "weights": "f16 ~N(0,0.02)", "l2": "inputs larger than L2 (the cross caches)",
                "eot": "suppressed, so that every window decodes all 224 steps",
                "parallelism": f"windows dealt over {self.world} GPU(s), no collective"}

    @staticmethod
    def cpu_sample(steps=4, seed=4100):
        # One window through `steps` greedy steps of the oracle's CPU decoder (f32 gemv, f16
        # caches) and search, scaled to 32 windows x 224 steps by tokens.
        from oracle import oracle as O
        D, F, H, L, V, frames = 1280, 5120, 20, 4, 51866, 1500
        hd = D // H
        rng = np.random.default_rng(seed)
        lin = lambda n, k: O.Linear(O.TY_F16, n, k, normal_f16(rng, (n, k), 0.02).tobytes())  # noqa: E731
        emb = normal_f16(rng, (V, D), 0.02)
        E = O.Linear(O.TY_F16, V, D, emb.tobytes())
        lay = [{k: lin(*sh) for k, sh in {"qkv": (3 * D, D), "self_out": (D, D),
                                          "cross_q": (D, D), "cross_out": (D, D),
                                          "fc1": (F, D), "fc2": (D, F)}.items()}
               for _ in range(L)]
        one, zero = np.ones(D, np.float32), np.zeros(D, np.float32)
        cross = [rng.standard_normal(frames * 2 * D, dtype=np.float32) for _ in range(L)]
        own = [np.zeros(448 * 2 * D, np.float32) for _ in range(L)]
        pos_t = rng.standard_normal((448, D), dtype=np.float32) * 0.02
        token, gen = 50360, []
        t0 = time.perf_counter()
        for pos in range(steps):
            x = (emb[token].astype(np.float32) + pos_t[pos]).astype(np.float32)
            for l in range(L):
                w = lay[l]
                y = O.layer_norm(x, one, zero, 1, D)
                qkv = w["qkv"].gemv(y)
                O.pack_cache(np.ascontiguousarray(qkv[D:]), 1, D, hd, own[l], 448, pos)
                att = O.attend(np.ascontiguousarray(qkv[:D]), own[l], 448, pos + 1, H, hd)
                w["self_out"].gemv(att, x, "residual", 1.0)
                y = O.layer_norm(x, one, zero, 1, D)
                att = O.attend(w["cross_q"].gemv(y), cross[l], frames, frames, H, hd)
                w["cross_out"].gemv(att, x, "residual", 1.0)
                y = O.layer_norm(x, one, zero, 1, D)
                w["fc2"].gemv(w["fc1"].gemv(y, None, "gelu"), x, "residual", 1.0)
            y = O.layer_norm(x, one, zero, 1, D)
            logits = E.gemv(y)[:V].copy()
            token, _ = O.pick(logits, gen, [50257], [220], 50257, 50364, 50365)
            gen.append(token)
        dt = time.perf_counter() - t0
        audio = 30.0 * steps / 224
        return dt, audio, f"1 window through {steps} of 224 steps"


class C5Mel(Workload):
    """§8 f4: the step before the encoder on the device for C5's audio: 400 segments of U[120, 300]
    encoder frames (1280 samples of 16 kHz pcm an encoder frame), each as the reference runs a
    piece: the log-mel features computed and normalised on their own (wavo_mel_features:
    pre-emphasis, Hann(400), f64 FFT of 512, power, 128 Slaney mel bins, ln, per-bin
    normalisation; src/parakeet/frontend.rs), then Parakeet-0.6B's 8x conv subsampling
    (wavo_subsample_batch over every segment, each segment's rows as its own subsampling:
    256 channels, F16 pointwise and output weights ~N(0, 0.02), d 1024;
    src/parakeet/encoder.rs:103-121). Input: the segments' pcm; output: the encoder's input rows
    [Σ frames][1024]."""
    METRIC = "frontend audio-sec/sec"
    CH, D = 256, 1024
    BOUNDS = {"mel_features": "hbm", "subsample": "tensor"}
    FRAME_S = 0.08
    bound = "hbm"
    dtype = "f64 FFT, f32 mel"

    def __init__(self, gpu, rank, world, seed=5000):
        import torch
        self.gpu, self.world = gpu, world
        lengths = segment_lengths(seed, 400, 120, 300)
        self.all_lengths = lengths
        self.plan, mine = shard(lengths, rank, world, lambda t: t)
        self.order = mine
        self.lengths = [lengths[i] for i in mine]
        self.samples = [t * 8 * 160 for t in self.lengths]
        self.frames = [n // 160 + 1 for n in self.samples]
        self.seg_rows, self.out_width = [t * 8 * 160 // 160 + 1 for t in lengths], 128
        rng = np.random.default_rng(seed + 1 + rank)
        total = sum(self.samples)
        t = np.arange(total) / 16000.0
        pcm = (0.05 * rng.standard_normal(total) + 0.2 * np.sin(2 * np.pi * 440.0 * t)).astype(np.float32)
        dev = gpu.torch_device
        self.pcm_host = torch.from_numpy(pcm).pin_memory()
        self.pcm = self.pcm_host.to(dev)
        rows = sum(self.frames)
        self.mel = torch.zeros(rows, 128, device=dev)
        self.s0 = np.concatenate([[0], np.cumsum(self.samples)[:-1]]).astype(int)
        self.r0 = np.concatenate([[0], np.cumsum(self.frames)[:-1]]).astype(int)
        self.x0 = np.concatenate([[0], np.cumsum(self.lengths)[:-1]]).astype(int)
        wrng = np.random.default_rng(seed)
        ch, d = self.CH, self.D
        self.taps = {k: gpu.upload((wrng.standard_normal((9, ch)) * 0.3).astype(np.float32))
                     for k in ("w0", "w2", "w5")}
        self.taps.update({k: gpu.upload((wrng.standard_normal(ch) * 0.1).astype(np.float32))
                          for k in ("b0", "b2", "b5")})
        from wavo_b200 import GGML_F16
        self.conv3 = gpu.linear(GGML_F16, ch, ch, normal_f16(wrng, (ch, ch), 0.02).tobytes(),
                                wrng.standard_normal(ch).astype(np.float32) * 0.02)
        self.conv6 = gpu.linear(GGML_F16, ch, ch, normal_f16(wrng, (ch, ch), 0.02).tobytes(),
                                wrng.standard_normal(ch).astype(np.float32) * 0.02)
        self.out = gpu.linear(GGML_F16, d, 16 * ch, normal_f16(wrng, (d, 16 * ch), 0.02).tobytes(),
                              wrng.standard_normal(d).astype(np.float32) * 0.02)
        from wavo_b200 import _lib as L
        import ctypes
        fr = (ctypes.c_uint32 * len(self.frames))(*self.frames)
        nbytes = int(L.lib().wavo_subsample_batch_scratch_bytes(fr, len(self.frames), ch))
        self.scratch = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
        self.x = torch.zeros(sum(self.lengths), d, device=dev)
        self.x_host = torch.empty(sum(self.lengths), d).pin_memory()
        self.seg_rows, self.out_width = list(lengths), d

    def mel_features(self, i):
        a, n, r, f = int(self.s0[i]), self.samples[i], int(self.r0[i]), self.frames[i]
        self.gpu.mel_features(self.pcm[a:a + n], self.mel[r:r + f])

    def subsample(self, n):
        """The first n segments' subsampling in one call (their mel rows and output rows are
        contiguous): conv0/conv2, conv3, conv5 segment by segment, conv6 and the output projection
        over all their rows."""
        r, x0 = int(sum(self.frames[:n])), int(sum(self.lengths[:n]))
        self.gpu.subsample_batch(self.mel[:r], self.frames[:n], self.frames[:n], self.taps,
                                 self.conv3, self.conv6, self.out, self.x[:x0], self.scratch)

    def record(self, p, timer=None):
        tick = timer or (lambda name, fn: fn())
        for i in range(len(self.samples)):
            tick("mel_features", lambda i=i: self.mel_features(i))
        tick("subsample", lambda: self.subsample(len(self.samples)))

    def profile_unit(self, p):
        """The first two segments' log-mel and subsampling, for a launch list."""
        import torch
        torch.cuda.profiler.start()
        for i in range(2):
            self.mel_features(i)
        self.subsample(2)

    def inputs(self):
        return [(self.pcm, self.pcm_host)]

    def outputs(self):
        return [(self.x_host, self.x)]

    def launches(self):
        # mel_features: the log-mel (with the normalisation's sums) and the normalisation a
        # segment; subsample: conv0/conv2, the conv3 GEMM and conv5 a segment, then the conv6
        # GEMM, the flatten and the output GEMM once.
        return (2 + 3) * len(self.samples) + 3

    def work(self):
        # Per call. mel_features (a segment, averaged over the segments): HBM bytes (the pcm read
        # once, the features written, read and written again by the normalisation); subsample
        # (every segment at once): flop (the convs' and GEMMs' multiply-adds).
        n = len(self.samples)
        mel = 4.0 * sum(self.samples) + 3 * 2 * 4.0 * 128 * sum(self.frames)
        ch, d = self.CH, self.D
        flop = 0.0
        for f, t in zip(self.frames, self.lengths):
            t1, t2 = (f - 1) // 2 + 1, ((f - 1) // 2) // 2 + 1
            flop += 2 * 9 * 9 * t2 * 32 * ch + 2 * t2 * 32 * ch * ch + 2 * 9 * t * 16 * ch
            flop += 2 * t * 16 * ch * ch + 2 * t * 16 * ch * d
        return {"mel_features": mel / n, "subsample": flop}

    def audio_s(self):
        return sum(self.lengths) * self.FRAME_S

    def total_audio_s(self, world):
        return sum(self.all_lengths) * self.FRAME_S

    def config(self):
        return {"workload": WORKLOAD_NAMES["c5mel"], "segments": len(self.all_lengths),
                "total_mel_frames": int(sum(t * 8 + 1 for t in self.all_lengths)),
                "audio_s": sum(self.all_lengths) * self.FRAME_S, "n_fft": 512, "mels": 128,
                "subsampling": f"8x, {self.CH} channels, d {self.D}, F16 pointwise weights",
                "l2": "inputs larger than L2 (430 MB of pcm)",
                "parallelism": f"segments sharded LPT over {self.world} GPU(s), no collective"}

    @staticmethod
    def cpu_sample(seed=5000):
        # 16 of the 400 segments (every 25th) through the oracle's frontend and subsampling (the
        # reference's Frontend::compute and the CPU encoder's subsampling restated; its GEMMs on the
        # host's threads), scaled by audio seconds.
        from oracle import oracle as O
        lens = segment_lengths(seed, 400, 120, 300)[::25]
        rng = np.random.default_rng(seed)
        pcms = [(0.05 * rng.standard_normal(t * 1280) + 0.2 * np.sin(
            2 * np.pi * 440.0 * np.arange(t * 1280) / 16000.0)).astype(np.float32) for t in lens]
        ch, d = C5Mel.CH, C5Mel.D
        taps = {k: (rng.standard_normal((9, ch)) * 0.3).astype(np.float32) for k in ("w0", "w2", "w5")}
        taps.update({k: (rng.standard_normal(ch) * 0.1).astype(np.float32) for k in ("b0", "b2", "b5")})
        l3 = O.Linear(O.TY_F16, ch, ch, normal_f16(rng, (ch, ch), 0.02).tobytes(), np.zeros(ch, np.float32))
        l6 = O.Linear(O.TY_F16, ch, ch, normal_f16(rng, (ch, ch), 0.02).tobytes(), np.zeros(ch, np.float32))
        lo = O.Linear(O.TY_F16, d, 16 * ch, normal_f16(rng, (d, 16 * ch), 0.02).tobytes(),
                      np.zeros(d, np.float32))
        from concurrent.futures import ThreadPoolExecutor
        t0 = time.perf_counter()
        with ThreadPoolExecutor(os.cpu_count() or 1) as ex:  # ctypes calls release the GIL
            mels = list(ex.map(O.mel_features, pcms))
        for m in mels:
            O.subsample(m, m.shape[0], taps, l3, l6, lo)
        dt = time.perf_counter() - t0
        return dt, sum(lens) * 0.08, ("16 of the 400 segments (every 25th): log-mel a thread a "
                                      "segment, subsampling with multithreaded GEMMs")


class C5Load:
    """§8 f3: C5's projection weights (24 layers of Q8_0 q, k, v, out and linear_pos, d = 1024,
    the C5 distributions: int8 ~U[-127, 127], f16 scales |N(0, 0.02)| / 127) loaded from a GGUF
    file into device-ready layers, as a model load does (src/gpu/mod.rs:758-827): per layer the
    stacked [q; k; v] projection, the output and the position projection through
    wavo_linear_from_gguf, which streams the file's bytes to the device in pinned pieces and builds
    the kernels' forms there. A step loads all 72 layers (133.7 MB of tensor data) from the page
    cache and frees them again."""
    LAYERS, D = 24, 1024
    METRIC = "GGUF weight load GB/s"
    UNIT = "GB/s"
    scaling = "weak"
    _path = None

    @classmethod
    def path(cls) -> str:
        if cls._path is None or not os.path.exists(cls._path):
            import tempfile
            from wavo_b200 import gguf as G
            rng = np.random.default_rng(5000)
            d = cls.D
            tensors = []
            for layer in range(cls.LAYERS):
                for name in ("attn_q", "attn_k", "attn_v", "attn_out", "linear_pos"):
                    nb = d * d // 32
                    blk = np.empty((nb, 34), np.uint8)
                    sc = (np.abs(rng.standard_normal(nb)) * 0.02 / 127).astype(np.float16)
                    blk[:, :2] = sc.view(np.uint8).reshape(nb, 2)
                    blk[:, 2:] = rng.integers(-127, 128, (nb, 32), dtype=np.int8).view(np.uint8)
                    tensors.append((f"blk.{layer}.{name}.weight", [d, d], G.TY_Q8_0, blk.tobytes()))
            fd, p = tempfile.mkstemp(suffix=".gguf")
            os.close(fd)
            G.write_gguf(p, [("general.architecture", G.STR, "parakeet")], tensors)
            import atexit
            atexit.register(lambda: os.path.exists(p) and os.remove(p))
            cls._path = p
        return cls._path

    @classmethod
    def layers(cls):
        for layer in range(cls.LAYERS):
            b = f"blk.{layer}."
            yield [b + "attn_q.weight", b + "attn_k.weight", b + "attn_v.weight"]
            yield [b + "attn_out.weight"]
            yield [b + "linear_pos.weight"]

    @classmethod
    def total_bytes(cls) -> int:
        return cls.LAYERS * 5 * cls.D * cls.D // 32 * 34

    @classmethod
    def config(cls):
        return {"workload": WORKLOAD_NAMES["c5load"], "layers": cls.LAYERS, "d_model": cls.D,
                "weights": "Q8_0, C5's distributions", "tensor_bytes": cls.total_bytes(),
                "source": "a GGUF v3 file in the page cache",
                "parallelism": "each GPU loads its own copy, no collective"}

    @classmethod
    def cpu_sample(cls):
        # The reference loader's host work (src/gpu/mod.rs:793-827 with src/gguf.rs:258-272): the
        # file read in pieces of 8192 Q8_0 blocks (the native reader's pread), each block's scale
        # and 32 values split into the two mapped buffers; here into host arrays (numpy).
        from wavo_b200 import gguf as G
        g = G.Gguf(cls.path())
        piece = 34 << 13
        t0 = time.perf_counter()
        for names in cls.layers():
            total = sum(g.tensor(n)[1] for n in names)
            data = np.empty(total // 34 * 32, np.uint8)
            scales = np.empty(total // 34 * 2, np.uint8)
            blk = 0
            for n in names:
                size = g.tensor(n)[1]
                for off in range(0, size, piece):
                    b = np.frombuffer(g.read(n, off, min(piece, size - off)), np.uint8).reshape(-1, 34)
                    data[blk * 32:(blk + len(b)) * 32] = b[:, 2:].ravel()
                    scales[blk * 2:(blk + len(b)) * 2] = b[:, :2].ravel()
                    blk += len(b)
        dt = time.perf_counter() - t0
        g.close()
        return dt, cls.total_bytes() / 1e9, "all 72 layers' bytes read in pieces and split (numpy)"


def run_load(args):
    """§8 f3 measurement: GGUF -> device-ready layers, GB/s of tensor data (`--config c5load`)."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from wavo_b200 import gguf as G
    from wavo_b200.gpu import Gpu
    W = C5Load
    gpu = Gpu(local)
    path = W.path()
    g = G.Gguf(path)
    stream = torch.cuda.current_stream(local)

    def step():
        # The layers' loads are timed; freeing them afterwards (a device-wide cudaFree each) is not
        # part of loading a model.
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        t0 = time.perf_counter()
        lins = [gpu.linear_from_gguf(g, names) for names in W.layers()]
        gpu.sync()
        e1.record(stream)
        torch.cuda.synchronize()
        t = max(e0.elapsed_time(e1), (time.perf_counter() - t0) * 1e3)
        del lins
        return t

    for _ in range(args.warmup):
        step()
    gpu.sync()
    if world > 1:
        dist.barrier()
    with Clocks(local) as clocks:
        ms = sum(step() for _ in range(args.steps)) / args.steps
    # The bound: a pinned host -> device copy of the same size on this host.
    src = torch.empty(W.total_bytes(), dtype=torch.uint8).pin_memory()
    dst = torch.empty(W.total_bytes(), dtype=torch.uint8, device="cuda")
    best = None
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        dst.copy_(src, non_blocking=True)
        b.record(stream)
        torch.cuda.synchronize()
        t = a.elapsed_time(b)
        best = t if best is None else min(best, t)
    pcie = W.total_bytes() / (best * 1e-3) / 1e9
    from wavo_b200.runner import max_over_ranks
    (ms,) = max_over_ranks([ms], device="cuda")
    if rank == 0:
        gbs = world * W.total_bytes() / (ms * 1e-3) / 1e9
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            W.cpu_sample()
            dt, gb, sample = W.cpu_sample()
            cpu = {"value": gb / dt, "unit": W.UNIT, "cores": 1, "kind": "port", "sample": sample}
        line = {"metric": W.METRIC, "value": gbs, "unit": W.UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": W.scaling, "vs_baseline": None,
                "dtype": "q8_0", "data": "synthetic (seeded, C5's weight distributions)",
                "config": W.config(),
                "e2e": {"value": gbs, "unit": W.UNIT, "h2d_bytes_per_step": W.total_bytes(),
                        "d2h_bytes_per_step": 0,
                        "copies": "the load is the host -> device path itself"},
                "gpu_launches": 72 * args.steps,
                "roofline": {"bound": "pcie", "kernel": "wavo_linear_from_gguf",
                             "achieved": gbs / world, "peak": pcie, "unit": "GB/s",
                             "frac": gbs / world / pcie,
                             "peak_source": "measured pinned host->device copy of the same bytes",
                             "traffic": None},
                "clocks": clocks.summary(), "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    g.close()
    if world > 1:
        dist.destroy_process_group()


WORKLOADS = {"c1": C1, "c2": C2, "c3": C3, "c4": C4, "c4full": C4Full, "c5": C5,
             "c5block": C5Block, "c5load": C5Load, "c5mel": C5Mel}
WORKLOAD_NAMES = {
    "c1": "C1: Parakeet rel-pos MHSA layer, f32 weights, batch 1, T=138",
    "c2": "C2: Whisper large-v3-turbo encoder self-attention, 32 layers, T=1500",
    "c3": "C3: GigaAM-v3-shaped RoPE attention, 16 layers, 16 segments of U[400,750] frames "
          "(key-padding mask as per-segment lengths)",
    "c4": "C4: Whisper-turbo decoder attention, 4 layers, batch 32, 224 greedy steps, self + "
          "cross attention over F16 caches",
    "c5": "C5: Parakeet-0.6B long form, 24 rel-pos layers, 400 segments of U[120,300] frames, "
          "Q8_0 weights",
    "c4full": "C4 full decoder: Whisper large-v3-turbo decoder, batch 32, 224 greedy steps on the "
              "device (LayerNorms, attention, FFN, logits, pick)",
    "c5block": "C5 blocks: Parakeet-0.6B FastConformer blocks (FFN, rel-pos MHSA, conv module, "
               "norms), 24 blocks, 400 segments of U[120,300] frames, Q8_0 weights",
    "c5mel": "C5 frontend: Parakeet's log-mel (f64 FFT of 512, 128 Slaney mel bins, per-segment "
             "normalisation) and 8x conv subsampling (256 channels, d 1024) over C5's 400 "
             "segments of U[120,300] encoder frames of 16 kHz audio",
    "c5load": "C5 weights from GGUF: 24 layers of Q8_0 q/k/v/out/linear_pos (d 1024) loaded from a "
              "GGUF file into device-ready layers",
}


# ---------------------------------------------------------------------------------------------

def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    O.set_threads(os.cpu_count() or 1)
    O.set_vnni(-1)
    W = WORKLOADS[args.config]
    for _ in range(args.warmup):
        W.cpu_sample()
    times, audio, sample = [], 0.0, ""
    for _ in range(args.steps):
        dt, audio, sample = W.cpu_sample()
        times.append(dt)
    t = float(np.mean(times))
    value = audio / t
    unit = getattr(W, "UNIT", UNIT)
    line = {"metric": getattr(W, "METRIC", METRIC), "value": value, "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
            "higher_is_better": True, "scaling": W.scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD_NAMES[args.config],
                       "sample": sample + " per step; value = the sample's audio seconds over "
                                 "its CPU time (the layers and segments are alike, so the rate "
                                 "carries over to the whole workload)"},
            "cpu_baseline": {"value": value, "unit": unit, "cores": O.threads(), "kind": "port",
                             "sample": sample + " per step (CPU oracle restating the "
                             "reference's src/cpu attention path)"},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c5", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="wavo", choices=["wavo", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="for an ncu capture (--profile-from-start off): warm the workload up, then "
                         "run one unit of it (one decoder step, two segments, or one whole step) "
                         "between cudaProfilerStart and cudaProfilerStop, and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.steps is None:
        args.steps = {"c1": 2000, "c2": 200, "c3": 100, "c4": 10, "c5": 30}.get(args.config, 5)
    if args.impl == "reference":
        if args.steps > 20:
            args.steps = 5
        return run_reference(args)
    if args.config == "c5load":
        return run_load(args)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        # NCCL prints its banner to the process's stdout when it builds the communicator; rank 0's
        # one JSON line must stand alone there, so stdout points at stderr meanwhile.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
        finally:
            import ctypes
            ctypes.CDLL(None).fflush(None)  # C stdio buffers out before fd 1 is restored
            os.dup2(saved, 1)
            os.close(saved)
    from wavo_b200.gpu import Gpu

    gpu = Gpu(local)
    gpu.reserve(256 << 20)
    wl = WORKLOADS[args.config](gpu, rank, world)
    stream = torch.cuda.current_stream(local)
    if args.profile:
        for _ in range(2):
            wl.record(gpu.pass_())
        gpu.sync()
        unit = getattr(wl, "profile_unit", None)
        if unit is None:
            torch.cuda.profiler.start()
            wl.record(gpu.pass_())
        else:
            unit(gpu.pass_())  # starts the profiler after its own lead-in
        gpu.sync()
        torch.cuda.profiler.stop()
        return

    for _ in range(2):  # eager warm-up (also configures the kernels before the capture)
        wl.record(gpu.pass_())
    gpu.sync()
    graph = gpu.capture(wl.record)

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident throughput (value) ----
    for _ in range(args.warmup):
        graph.launch()
    gpu.sync()
    barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clocks:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            graph.launch()
        e1.record(stream)
        torch.cuda.synchronize()
    gpu.sync()
    ms = e0.elapsed_time(e1) / args.steps
    barrier()

    # ---- end to end: H2D of the step's inputs (pinned), the step, D2H of its result ----
    # Serial: the copies and the step one after another on the launching stream. Segment
    # workloads read their result back segment by segment into one node-wide host buffer in
    # segment order (every rank over its own host link), and the step ends when every rank's rows
    # are there (each rank's stream drained, then a barrier): the ordered gather to the host.
    hg = wl.host_gather(rank)

    def read_back():
        if hg is not None:
            for _, dev_t in wl.outputs():
                hg.copy_from(dev_t)
        else:
            for host_t, dev_t in wl.outputs():
                host_t.copy_(dev_t, non_blocking=True)

    def e2e_step():
        for dev_t, host_t in wl.inputs():
            dev_t.copy_(host_t, non_blocking=True)
        graph.launch()
        read_back()
        if hg is not None:
            hg.wait(stream)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    f1.record(stream)
    torch.cuda.synchronize()
    gpu.sync()
    ms_e2e_serial = f0.elapsed_time(f1) / args.steps

    # Pipelined, as a serving loop runs it: every step's input still crosses PCIe into pinned
    # staging on the device and every step's result comes back to pinned host memory, but on two
    # copy streams, so that step k+1's upload and step k's read-back overlap step k's kernels.
    # The step's own buffers are filled from / drained to the staging buffers by device copies.
    h2d_s, d2h_s = torch.cuda.Stream(local), torch.cuda.Stream(local)
    in_stage = [(dev_t, host_t, torch.empty_like(dev_t)) for dev_t, host_t in wl.inputs()]
    out_stage = [(host_t, dev_t, torch.empty_like(dev_t)) for host_t, dev_t in wl.outputs()]
    if hg is not None:
        hg.wait(stream)  # the serial loop's last rows are in place before the buffer is reused
    in_free, in_ready = torch.cuda.Event(), torch.cuda.Event()
    out_free, out_ready = torch.cuda.Event(), torch.cuda.Event()

    def pipelined_step():
        with torch.cuda.stream(h2d_s):
            h2d_s.wait_event(in_free)  # the previous step has taken its input from staging
            for _, host_t, st in in_stage:
                st.copy_(host_t, non_blocking=True)
            in_ready.record(h2d_s)
        stream.wait_event(in_ready)
        for dev_t, _, st in in_stage:
            dev_t.copy_(st, non_blocking=True)
        in_free.record(stream)
        graph.launch()
        stream.wait_event(out_free)  # the previous step's result has left staging
        for _, dev_t, st in out_stage:
            st.copy_(dev_t, non_blocking=True)
        out_ready.record(stream)
        with torch.cuda.stream(d2h_s):
            d2h_s.wait_event(out_ready)
            for host_t, _, st in out_stage:
                if hg is not None:
                    hg.copy_from(st)
                else:
                    host_t.copy_(st, non_blocking=True)
            out_free.record(d2h_s)

    for _ in range(args.warmup):
        pipelined_step()
    torch.cuda.synchronize()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    h2d_s.wait_event(f0)
    for _ in range(args.steps):
        pipelined_step()
    stream.wait_event(out_free)  # the last result is in host memory
    if hg is not None:
        hg.wait(stream)  # and every rank's
    f1.record(stream)
    torch.cuda.synchronize()
    gpu.sync()
    ms_e2e = f0.elapsed_time(f1) / args.steps
    h2d = sum(t.numel() * t.element_size() for _, t in wl.inputs())
    d2h = sum(t.numel() * t.element_size() for t, _ in wl.outputs())

    # ---- per-kernel durations for the roofline: each op's launches of one step, alone in a
    # graph (same buffers, weights and order as in the step), replayed back to back and timed with
    # CUDA events on the launching stream; per launch = elapsed / (replays x launches) ----
    counts: dict[str, int] = {}
    wl.record(gpu.pass_(), lambda name, fn: counts.__setitem__(name, counts.get(name, 0) + 1))
    per = {}
    for name in counts:
        g = gpu.capture(lambda p: wl.record(p, lambda n, fn: fn() if n == name else None))
        for _ in range(2):
            g.launch()
        gpu.sync()
        # Replays for about 0.15 s (at least 3), from a first timed replay.
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g.launch()
        b.record(stream)
        torch.cuda.synchronize()
        reps = max(3, int(150.0 / max(a.elapsed_time(b), 1e-3)))
        a.record(stream)
        for _ in range(reps):
            g.launch()
        b.record(stream)
        torch.cuda.synchronize()
        gpu.sync()
        per[name] = a.elapsed_time(b) / (reps * counts[name])
        del g
    totals = {k: per[k] * counts[k] for k in per}
    work = wl.work()
    top = max((k for k in totals if work.get(k, 0) > 0), key=totals.get)
    # The dominant kernel again, replayed for about half a second with the SM clock sampled
    # meanwhile, so that its roofline fraction can be read at the clock it actually ran at (the
    # replays come after the timed steps, when the power cap may hold the clocks down).
    g = gpu.capture(lambda p: wl.record(p, lambda n, fn: fn() if n == top else None))
    g.launch()
    gpu.sync()
    reps = max(3, int(0.5e3 / max(per[top] * counts[top], 1e-3)))
    with Clocks(local) as top_clocks:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            g.launch()
        b.record(stream)
        torch.cuda.synchronize()
    gpu.sync()
    per_top = a.elapsed_time(b) / (reps * counts[top])
    per[top] = per_top
    del g

    from wavo_b200.runner import max_over_ranks
    ms, ms_e2e, ms_e2e_serial = max_over_ranks([ms, ms_e2e, ms_e2e_serial], device="cuda")

    if rank == 0:
        peaks = load_peaks()
        clk = clocks.summary()
        tclk = top_clocks.summary()
        clock_frac = None
        bound = getattr(wl, "BOUNDS", {}).get(top, wl.bound)
        if bound == "hbm":
            achieved = work[top] / (per_top * 1e-3) / 1e9
            peak, unit, src = peaks["hbm"], "GB/s", "HBM copy"
        else:
            achieved = work[top] / (per_top * 1e-3) / 1e12
            # The burst GEMM peak (cuBLAS at free-running clocks) is the denominator. The kernel
            # is timed in a half-second replay loop, under the power cap like the driver's
            # sustained GEMM, so the fraction of the sustained peak is reported beside it (the
            # 100 ms clock samples are too coarse to scale a peak by).
            peak, unit, src = peaks["tensor"], "TFLOP/s", "bf16 burst"
            clock_frac = achieved / peaks["tensor_sustained"]
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            from oracle import oracle as O
            O.set_threads(os.cpu_count() or 1)
            O.set_vnni(-1)
            type(wl).cpu_sample()  # warm
            dt, audio, sample = type(wl).cpu_sample()
            cpu = {"value": audio / dt, "unit": UNIT, "cores": O.threads(), "kind": "port",
                   "sample": sample + " (CPU oracle restating the reference's src/cpu path)"}
        total_audio = wl.total_audio_s(world)
        line = {
            "metric": getattr(wl, "METRIC", METRIC), "value": total_audio / (ms * 1e-3), "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None,
            "dtype": wl.dtype, "data": "synthetic (seeded, BASELINE.json shapes/distributions)",
            "config": wl.config(),
            "e2e": {"value": total_audio / (ms_e2e_serial * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "copies": "serial: each step's H2D, the step, its D2H, one after another",
                    "gather": ("every segment's output rows to their place in one node-wide "
                               "host buffer in segment order (each rank over its own host "
                               "link), every rank's copies done and a barrier, each step")
                              if hg is not None else "none (one unit per rank)",
                    "pipelined_value": total_audio / (ms_e2e * 1e-3),
                    "pipelined": "step k+1's H2D and step k's D2H on two copy streams overlap "
                                 "step k (pinned staging, device copies in and out)"},
            "gpu_launches": wl.launches() * args.steps,
            "roofline": {"bound": bound, "kernel": top, "achieved": achieved, "peak": peak,
                         "unit": unit, "frac": achieved / peak,
                         "frac_of_sustained": clock_frac, "ms_per_launch": per_top,
                         "clocks_while_timed": tclk,
                         "traffic": wl.TRAFFIC.get(top),
                         "peak_source": f"{peaks['source']} {src}"},
            "kernels_ms": per,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del graph
    if hg is not None:
        hg.close()
    gpu.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
