#!/usr/bin/env python
"""Benchmark of the fused-op hot path on B200 (one JSON line on rank 0).

Metric: fwd+bwd tokens/s per fused op at Qwen3-VL shapes, with
the fraction of the HBM / tensor-core roofline, on 1-8 GPUs.  The line's own
workload (``value``) is BASELINE configs[1] — SwiGLU (gate/up [8,2048,6144]
bf16) plus RoPE (q [8,16,2048,128], k [8,8,2048,128] bf16, positions
0..2047, theta 5e6, cos/sin recomputed in-kernel), forward + backward — one
"step" = one fwd+bwd pass of both ops over the 16,384 tokens.  The default run
also measures every other fused op at its BASELINE config, each with its own
roofline, e2e, launch count, peak memory and (N=1) CPU baseline, under
``workloads``: rmsnorm, flce, lora and
c5_step (configs[4], the Qwen3-VL-8B LoRA training step; data-parallel with
the NCCL gradient all-reduce at N > 1).  Under ``flce_vp`` it reports the
FLCE at N GPUs: vocabulary-parallel (lm_head rows sharded, NCCL all-reduce of
the per-token statistics and of the partial dX), strong scaling, with its
speed-up over the single-GPU op timed on the same GPUs in the same run and a
parity check of every rank's shard against the single-GPU result.
``--workload NAME`` runs one workload alone as the line (also ``generate``:
greedy decoding with the static-KV generator; its metric is generated
tokens/s).

  value    device-timed tokens/s, inputs resident in HBM, CUDA events on the
           launching stream, max over ranks (weak scaling: every rank runs
           the full per-GPU workload, no collective on the data path);
  e2e      the same metric through the public autograd API with HOST
           (pinned) buffers: per step H2D of all inputs and D2H of all
           outputs inside the timed region (row-wise ops: the batch rows
           pipelined over H2D / compute / D2H streams);
  roofline the dominant kernel's algorithmic bytes (or FLOPs) per launch over
           its event-timed average duration, against MEASURED_PEAKS.json;
  cpu_baseline  the CPU oracle (a restatement of the reference's torch ops)
           on the host cores over a bounded sample (rank 0, N=1 only).

``--impl reference`` times that CPU implementation alone (the reference arm).

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
       torchrun --nproc-per-node N bench.py --gpus N ...
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")

import torch  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return d, "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(workload: str, kernel: str):
    """DRAM bytes per launch of `kernel` from a committed ncu summary, or None."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d.get(workload, {}).get(kernel)
    except Exception:
        return None


class ClockSampler:
    """Polls NVML (SM clock, throttle reasons) from a thread during the timed region."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        self._thr = None
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            # NVML enumerates physical GPUs; map through CUDA_VISIBLE_DEVICES.
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = device_index
            if vis:
                ids = [v.strip() for v in vis.split(",") if v.strip()]
                if device_index < len(ids) and ids[device_index].isdigit():
                    idx = int(ids[device_index])
            self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *exc):
        if self._thr is not None:
            self._stop.set()
            self._thr.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit]
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": names,
            "samples": len(self.samples),
        }


class KernelTimer:
    """CUDA-event brackets around named launches on the current stream
    (`before`, if given, runs on the stream ahead of each bracket)."""

    def __init__(self, before=None):
        self.marks = []
        self.before = before

    def __call__(self, name, fn, *args):
        if self.before is not None:
            self.before()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        out = fn(*args)
        e.record()
        self.marks.append((name, s, e))
        return out

    def averages_ms(self):
        acc = {}
        for name, s, e in self.marks:
            acc.setdefault(name, []).append(s.elapsed_time(e))
        return {k: sum(v) / len(v) for k, v in acc.items()}


def plain(name, fn, *args):
    return fn(*args)


class CopyPipeline:
    """Host<->device copies overlapped with compute for an end-to-end step.

    The step's token rows are split into chunks; chunk i's inputs go up on an
    H2D stream, its compute runs on a compute stream once they have arrived,
    and its outputs come back on a D2H stream once computed, so the H2D of
    chunk i+1, the compute of chunk i and the D2H of chunk i-1 run together
    (PCIe is full duplex).  Device input buffers are reused across steps: the
    H2D of a chunk waits until the previous step's compute of that chunk has
    finished reading it.  Consecutive steps are not joined, so the next step's
    uploads run while this step's last downloads drain, as behind a
    prefetching data loader; join() makes the caller's stream wait for all
    three streams, so events recorded on it after join() bracket every step
    issued before it.  The host runs at most `depth` steps ahead of the
    device (it waits for the step `depth` back before issuing another), so
    the caching allocator recycles the outputs of finished steps instead of
    growing, and blocking, while the host races ahead.  With `slots` > 1 the
    caller keeps that many sets of device input buffers and uses set
    `self.slot` in a step, so a step's uploads also overlap the previous
    step's compute (one-chunk steps whose inputs are all needed up front)."""

    def __init__(self, device, nchunks, depth=2, slots=1):
        self.nchunks = nchunks
        self.depth = depth
        self.slots = slots
        self.slot = 0
        self.steps = 0
        self.h2d = torch.cuda.Stream(device)
        self.comp = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self.freed = [[None] * nchunks for _ in range(slots)]
        self.issued = []  # completion events of the steps in flight

    def run(self, load, compute, store):
        while len(self.issued) >= self.depth:
            self.issued.pop(0).synchronize()
        self.slot = self.steps % self.slots
        self.steps += 1
        freed = self.freed[self.slot]
        main = torch.cuda.current_stream()
        start = main.record_event()
        for s in (self.h2d, self.comp, self.d2h):
            s.wait_event(start)
        for i in range(self.nchunks):
            with torch.cuda.stream(self.h2d):
                # chunk 0 may also reload buffers every chunk of a step reads
                # (a weight): it waits for the last compute that read this
                # buffer set
                wait = freed[self.nchunks - 1] if i == 0 else freed[i]
                if wait is not None:
                    self.h2d.wait_event(wait)
                load(i)
                arrived = self.h2d.record_event()
            with torch.cuda.stream(self.comp):
                self.comp.wait_event(arrived)
                outs = compute(i)
                done = self.comp.record_event()
                freed[i] = done
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(done)
                for t in store(i, outs):
                    t.record_stream(self.d2h)
        # the D2H stream ends after every compute and copy of this step
        self.issued.append(self.d2h.record_event())

    def join(self):
        main = torch.cuda.current_stream()
        for s in (self.h2d, self.comp, self.d2h):
            main.wait_stream(s)


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

class SwigluRope:
    """SwiGLU + RoPE fwd+bwd, bf16, Qwen3-VL-2B layer shape."""

    name = "swiglu_rope"
    short = "configs[1] SwiGLU [8,2048,6144] + RoPE q[8,16,2048,128] k[8,8,2048,128] bf16"
    bound = "hbm"
    dtype = "bf16"
    e2e_pipelined = True
    B, S, I = 8, 2048, 6144
    HQ, HK, D = 16, 8, 128
    THETA = 5e6
    dominant = "swiglu_backward"

    def __init__(self):
        self.tokens = self.B * self.S
        n = self.tokens * self.I
        rq = self.B * self.HQ * self.S * self.D
        rk = self.B * self.HK * self.S * self.D
        # algorithmic bytes per launch (bf16 = 2 B): every tensor read/written once
        self.bytes = {
            "swiglu_forward": 3 * n * 2,
            "swiglu_backward": 5 * n * 2,
            "rope_forward": 2 * (rq + rk) * 2,
            "rope_backward": 2 * (rq + rk) * 2,
        }
        self.launches_per_step = 4

    def config(self):
        return {
            "workload": "swiglu_rope_bf16 (BASELINE configs[1]): SwiGLU gate/up [8,2048,6144] + "
                        "RoPE q [8,16,2048,128], k [8,8,2048,128], positions 0..2047, "
                        "theta 5e6, cos/sin recomputed in-kernel; fwd+bwd",
            "tokens_per_step": self.tokens,
            "global_batch": self.B,
            "seq_len": self.S,
            "intermediate": self.I,
            "parallelism": "replicas (token rows; no collective)",
            "l2": "inputs larger than L2 (every tensor >= 67 MB; 2.0 GB touched per step)",
        }

    def make_inputs(self, device, seed=1235):
        g = torch.Generator(device=device).manual_seed(seed)
        shp = (self.B, self.S, self.I)
        t = {
            "gate": torch.randn(shp, generator=g, device=device).bfloat16(),
            "up": torch.randn(shp, generator=g, device=device).bfloat16(),
            "dout": torch.randn(shp, generator=g, device=device).bfloat16(),
            "q": torch.randn(self.B, self.HQ, self.S, self.D, generator=g,
                             device=device).bfloat16(),
            "k": torch.randn(self.B, self.HK, self.S, self.D, generator=g,
                             device=device).bfloat16(),
            "dq": torch.randn(self.B, self.HQ, self.S, self.D, generator=g,
                              device=device).bfloat16(),
            "dk": torch.randn(self.B, self.HK, self.S, self.D, generator=g,
                              device=device).bfloat16(),
        }
        t["pos"] = torch.arange(self.S, device=device).expand(self.B, self.S).contiguous()
        from metal_liger_b200.ops.fused_rope import rope_inv_freq

        t["inv_freq"] = rope_inv_freq(self.D, self.THETA, device=device)
        return t

    def step(self, t, timer=plain):
        ops = torch.ops.metal_liger
        timer("swiglu_forward", ops.swiglu_forward, t["gate"], t["up"], "")
        timer("swiglu_backward", ops.swiglu_backward, t["gate"], t["up"], t["dout"], "")
        timer("rope_forward", ops.rope_apply_qk_pos, t["q"], t["k"], t["pos"], t["inv_freq"],
              1.0, 1)
        timer("rope_backward", ops.rope_apply_qk_pos, t["dq"], t["dk"], t["pos"], t["inv_freq"],
              1.0, -1)

    # ---- end to end through the public API with host buffers ----
    def e2e_setup(self, device):
        t = self.make_inputs(device, seed=77)
        host = {k: v.cpu().pin_memory() for k, v in t.items() if k not in ("pos", "inv_freq")}
        dev = {k: torch.empty_like(v) for k, v in t.items() if k not in ("pos", "inv_freq")}
        outs_shapes = {"out": t["gate"], "dgate": t["gate"], "dup": t["up"], "q_rot": t["q"],
                       "k_rot": t["k"], "dq_in": t["q"], "dk_in": t["k"]}
        host_out = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True)
                    for k, v in outs_shapes.items()}
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        d2h = sum(v.numel() * v.element_size() for v in host_out.values())
        return {"host": host, "dev": dev, "host_out": host_out, "pos": t["pos"],
                "inv_freq": t["inv_freq"], "h2d": h2d, "d2h": d2h,
                "pipe": CopyPipeline(device, self.B * self.E2E_SPLIT)}

    # Chunks per batch row in the e2e pipeline.  Every chunk stays contiguous:
    # SwiGLU rows split along the sequence, RoPE rows along the heads (all
    # positions of the batch row in every chunk).  One chunk per batch row
    # (8 per step) keeps the host's enqueue time per step (copies and
    # autograd calls, ~0.5 ms per chunk) well under the ~16 ms the copies
    # take on the host link; 16 and more chunks measured slower.
    E2E_SPLIT = 1

    def _e2e_views(self, i):
        sp = self.E2E_SPLIT
        b, part = divmod(i, sp)
        rows, hq, hk = self.S // sp, self.HQ // sp, self.HK // sp
        sw = (b, slice(part * rows, (part + 1) * rows))
        rq = (b, slice(part * hq, (part + 1) * hq))
        rk = (b, slice(part * hk, (part + 1) * hk))
        return {"gate": sw, "up": sw, "dout": sw, "q": rq, "dq": rq, "k": rk, "dk": rk,
                "out": sw, "dgate": sw, "dup": sw, "q_rot": rq, "dq_in": rq,
                "k_rot": rk, "dk_in": rk}, b

    def e2e_step(self, s):
        from metal_liger_b200.ops.fused_swiglu import fused_swiglu
        from metal_liger_b200.ops.fused_rope import apply_fused_rotary_from_positions

        d, h, ho = s["dev"], s["host"], s["host_out"]

        def load(i):
            v, _ = self._e2e_views(i)
            for k in d:
                d[k][v[k]].copy_(h[k][v[k]], non_blocking=True)

        def compute(i):
            v, b = self._e2e_views(i)
            gate = d["gate"][v["gate"]].unsqueeze(0).detach().requires_grad_(True)
            up = d["up"][v["up"]].unsqueeze(0).detach().requires_grad_(True)
            out = fused_swiglu(gate, up)
            q = d["q"][v["q"]].unsqueeze(0).detach().requires_grad_(True)
            k = d["k"][v["k"]].unsqueeze(0).detach().requires_grad_(True)
            qr, kr = apply_fused_rotary_from_positions(q, k, s["pos"][b:b + 1],
                                                       inv_freq=s["inv_freq"])
            # one backward pass for both ops (one autograd engine call per chunk)
            torch.autograd.backward([out, qr, kr], [d["dout"][v["dout"]].unsqueeze(0),
                                                    d["dq"][v["dq"]].unsqueeze(0),
                                                    d["dk"][v["dk"]].unsqueeze(0)])
            return {"out": out.detach(), "dgate": gate.grad, "dup": up.grad,
                    "q_rot": qr.detach(), "k_rot": kr.detach(), "dq_in": q.grad,
                    "dk_in": k.grad}

        def store(i, outs):
            v, _ = self._e2e_views(i)
            for name, src in outs.items():
                ho[name][v[name]].copy_(src[0], non_blocking=True)
            return outs.values()

        s["pipe"].run(load, compute, store)

    # ---- CPU oracle on a bounded sample ----
    def cpu_inputs(self, tokens, seed=5):
        g = torch.Generator().manual_seed(seed)
        return {
            "gate": torch.randn(tokens, self.I, generator=g).bfloat16(),
            "up": torch.randn(tokens, self.I, generator=g).bfloat16(),
            "dout": torch.randn(tokens, self.I, generator=g).bfloat16(),
            "q": torch.randn(1, self.HQ, tokens, self.D, generator=g).bfloat16(),
            "k": torch.randn(1, self.HK, tokens, self.D, generator=g).bfloat16(),
            "dq": torch.randn(1, self.HQ, tokens, self.D, generator=g).bfloat16(),
            "dk": torch.randn(1, self.HK, tokens, self.D, generator=g).bfloat16(),
            "pos": torch.arange(tokens)[None],
        }

    def cpu_step(self, c):
        from oracle import ops as O

        O.swiglu_forward(c["gate"], c["up"])
        O.swiglu_backward(c["gate"], c["up"], c["dout"])
        cos, sin = O.rope_cos_sin(c["pos"], O.rope_inv_freq(self.D, self.THETA))
        cos, sin = cos[:, None], sin[:, None]
        for x in (c["q"], c["k"]):
            O.rope_apply(x, cos, sin).to(torch.bfloat16)
        for gx in (c["dq"], c["dk"]):
            O.rope_backward(gx, cos, sin).to(torch.bfloat16)


class RmsNorm:
    """RMSNorm fwd+bwd fp32, x [8,1024,2048]."""

    name = "rmsnorm"
    short = "configs[0] RMSNorm fp32 x[8,1024,2048]"
    bound = "hbm"
    dtype = "f32"
    e2e_pipelined = True
    B, S, H = 8, 1024, 2048
    dominant = "rms_norm_backward"

    def __init__(self):
        self.tokens = self.B * self.S
        n = self.tokens * self.H
        self.bytes = {"rms_norm_forward": 2 * n * 4 + self.tokens * 4,
                      "rms_norm_backward": 3 * n * 4 + self.tokens * 4}
        self.launches_per_step = 3  # fwd, bwd, dweight reduce

    def config(self):
        return {"workload": "rmsnorm_f32 (BASELINE configs[0]): x [8,1024,2048], eps 1e-6; "
                            "fwd+bwd (y, dX, dW)",
                "tokens_per_step": self.tokens, "global_batch": self.B, "seq_len": self.S,
                "hidden": self.H, "parallelism": "replicas (token rows; no collective)",
                "l2": "inputs larger than L2 is false (67 MB); L2 flushed before every step "
                      "(256 MB write, then 256 MB read), outside the timed spans"}

    def make_inputs(self, device, seed=1234):
        g = torch.Generator(device=device).manual_seed(seed)
        x = torch.randn(self.B, self.S, self.H, generator=g, device=device)
        w = 1.0 + 0.1 * torch.randn(self.H, generator=g, device=device)
        dy = torch.randn(self.B, self.S, self.H, generator=g, device=device)
        flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
        flush_rd = torch.zeros(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
        return {"x": x, "w": w, "dy": dy, "flush": flush, "flush_rd": flush_rd}

    def prelude(self, t):
        # Evict L2 (126 MB) so the inputs come from HBM: write a 256 MB buffer,
        # then read another 256 MB so the lines left behind are clean and the
        # timed kernels do not pay for the flush's write-back.
        t["flush"].fill_(0.0)
        t["flush_rd"].amax()

    def step(self, t, timer=plain):
        ops = torch.ops.metal_liger
        y, rrms = timer("rms_norm_forward", ops.rms_norm_forward, t["x"], t["w"], 1e-6, "")
        timer("rms_norm_backward", ops.rms_norm_backward, t["x"], t["w"], t["dy"], 1e-6, "",
              rrms)

    def e2e_setup(self, device):
        t = self.make_inputs(device, seed=78)
        host = {k: t[k].cpu().pin_memory() for k in ("x", "w", "dy")}
        dev = {k: torch.empty_like(t[k]) for k in ("x", "w", "dy")}
        host_out = {"y": torch.empty_like(host["x"]).pin_memory(),
                    "dx": torch.empty_like(host["x"]).pin_memory(),
                    "dw": torch.empty_like(host["w"]).pin_memory()}
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        d2h = sum(v.numel() * v.element_size() for v in host_out.values())
        return {"host": host, "dev": dev, "host_out": host_out, "h2d": h2d, "d2h": d2h,
                "pipe": CopyPipeline(device, self.E2E_CHUNKS)}

    # Chunks of batch rows in the e2e pipeline: two keep the host's enqueue
    # time per step (copies and autograd calls, ~0.3 ms per chunk) under the
    # ~2.7 ms the copies take on the host link; consecutive steps overlap.
    E2E_CHUNKS = 2

    def e2e_step(self, s):
        from metal_liger_b200.ops.fused_rms_norm import _FusedRMSNormFunction

        d, h, ho = s["dev"], s["host"], s["host_out"]
        nc = s["pipe"].nchunks
        per = self.B // nc
        # the weight is one leaf for the whole step: its gradient accumulates
        # over the chunks (autograd adds), as over the batch rows of one call
        w = d["w"].detach().requires_grad_(True)

        def load(i):
            sl = slice(i * per, (i + 1) * per)
            if i == 0:
                d["w"].copy_(h["w"], non_blocking=True)
            d["x"][sl].copy_(h["x"][sl], non_blocking=True)
            d["dy"][sl].copy_(h["dy"][sl], non_blocking=True)

        def compute(i):
            sl = slice(i * per, (i + 1) * per)
            x = d["x"][sl].detach().requires_grad_(True)
            y = _FusedRMSNormFunction.apply(x, w, 1e-6)
            y.backward(d["dy"][sl])
            outs = {"y": y.detach(), "dx": x.grad}
            if i == nc - 1:
                outs["dw"] = w.grad
            return outs

        def store(i, outs):
            sl = slice(i * per, (i + 1) * per)
            ho["y"][sl].copy_(outs["y"], non_blocking=True)
            ho["dx"][sl].copy_(outs["dx"], non_blocking=True)
            if "dw" in outs:
                ho["dw"].copy_(outs["dw"], non_blocking=True)
            return outs.values()

        s["pipe"].run(load, compute, store)

    def cpu_inputs(self, tokens, seed=6):
        g = torch.Generator().manual_seed(seed)
        return {"x": torch.randn(tokens, self.H, generator=g),
                "w": 1 + 0.1 * torch.randn(self.H, generator=g),
                "dy": torch.randn(tokens, self.H, generator=g)}

    def cpu_step(self, c):
        from oracle import ops as O

        _, rr = O.rms_norm_forward(c["x"], c["w"], 1e-6)
        O.rms_norm_backward(c["x"], c["w"], rr, c["dy"])


class Flce:
    """chunked fused linear cross-entropy, bf16, N 16384, H 2048, V 151936."""

    name = "flce"
    bound = "tensor"
    dtype = "bf16"
    N, H, V, CHUNK = 16384, 2048, 151936, 8192
    dominant = "flce_forward"

    short = "configs[2] FLCE bf16 h[16384,2048] W[151936,2048] chunk 8192"

    def __init__(self, world=None, rank=None):
        self.tokens = self.N
        self.world = int(os.environ.get("WORLD_SIZE", "1")) if world is None else world
        self.rank = int(os.environ.get("RANK", "0")) if rank is None else rank
        # vocabulary shard of this rank (the whole vocabulary on one GPU)
        base, rem = divmod(self.V, self.world)
        self.v_local = base + (1 if self.rank < rem else 0)
        f = 6.0 * self.N * self.H * self.v_local  # logits, dX and dW GEMMs once each
        self.flops = {"flce_forward": f}
        self.bytes = {}
        if self.world > 1:
            self.scaling = "strong"
            self.per_rank_tokens = False
        # count, (logits GEMM, lse, transform, dX GEMM, dW GEMM, memset) per chunk, loss;
        # backward: two scale-casts
        self.launches_per_step = 1 + 5 * (-(-self.N // self.CHUNK)) + 1 + 2

    def config(self):
        par = ("single GPU" if self.world == 1 else
               f"vocab-parallel over {self.world} GPUs (lm_head rows sharded; per-chunk NCCL "
               f"all-reduce of row max / sum-exp / target logit and of partial dX)")
        base = "BASELINE configs[2]" if self.N == 16384 else "smaller than BASELINE configs[2]"
        return {"workload": f"flce_bf16 ({base}): hidden [{self.N},2048] ~N(0,1), "
                            "lm_head W [151936,2048] ~N(0,0.02), 10% labels = -100, token "
                            f"chunk {self.CHUNK}, mean over non-ignored; loss + dX + dW",
                "tokens_per_step": self.N, "hidden": self.H, "vocab": self.V,
                "vocab_per_rank": self.v_local, "chunk_tokens": self.CHUNK,
                "parallelism": par, "l2": "inputs larger than L2 (W 622 MB)"}

    def make_inputs(self, device, seed=1236):
        from metal_liger_b200.ops.fused_linear_cross_entropy import shard_lm_head

        g = torch.Generator(device=device).manual_seed(seed)
        h = torch.randn(self.N, self.H, generator=g, device=device).bfloat16()
        w = (0.02 * torch.randn(self.V, self.H, generator=g, device=device)).bfloat16()
        lab = torch.randint(0, self.V, (self.N,), generator=g, device=device)
        lab[torch.randperm(self.N, generator=g, device=device)[: self.N // 10]] = -100
        go = torch.ones((), device=device)
        ws, off = shard_lm_head(w, self.rank, self.world)
        ws = ws.contiguous()
        del w
        return {"h": h, "w": ws, "off": off, "lab": lab, "go": go}

    def _vp(self, t):
        from metal_liger_b200.ops.fused_linear_cross_entropy import vocab_parallel_flce

        loss, dx, dw = vocab_parallel_flce(t["h"], t["w"], t["lab"], t["off"],
                                           chunk_size=self.CHUNK)
        return loss, dx.unsqueeze(0), dw

    def step(self, t, timer=plain):
        ops = torch.ops.metal_liger
        if self.world == 1:
            loss, dx, dw = timer("flce_forward", ops.flce_forward, t["h"], t["w"], t["lab"], None,
                                 -100, self.CHUNK, True, True)
        else:
            loss, dx, dw = timer("flce_forward", self._vp, t)
        timer("flce_backward", ops.flce_backward, t["go"], dx, dw, 1, 1)

    e2e_pipelined = True

    def e2e_setup(self, device):
        t = self.make_inputs(device, seed=79)
        host = {k: t[k].cpu().pin_memory() for k in ("h", "w", "lab")}
        # two device input sets: a step's uploads (the whole lm_head among
        # them) run during the previous step's compute, its downloads during
        # the next one's
        dev = [{k: torch.empty_like(t[k]) for k in ("h", "w", "lab")} for _ in range(2)]
        host_out = {"loss": torch.empty((), pin_memory=True),
                    "dh": torch.empty_like(host["h"]).pin_memory(),
                    "dw": torch.empty_like(host["w"]).pin_memory()}
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        d2h = sum(v.numel() * v.element_size() for v in host_out.values())
        return {"host": host, "dev": dev, "host_out": host_out, "h2d": h2d, "d2h": d2h,
                "off": t["off"], "pipe": CopyPipeline(device, 1, slots=2)}

    def e2e_step(self, s):
        from metal_liger_b200.ops.fused_linear_cross_entropy import \
            _FusedLinearCrossEntropyFunction

        h, ho, pipe = s["host"], s["host_out"], s["pipe"]

        def load(i):
            d = s["dev"][pipe.slot]
            for k in d:
                d[k].copy_(h[k], non_blocking=True)

        def compute(i):
            d = s["dev"][pipe.slot]
            hid = d["h"].detach().requires_grad_(True)
            w = d["w"].detach().requires_grad_(True)
            if self.world == 1:
                loss = _FusedLinearCrossEntropyFunction.apply(hid, w, d["lab"], None, -100,
                                                              self.CHUNK)
            else:
                from metal_liger_b200.ops.fused_linear_cross_entropy import \
                    _VocabParallelFLCEFunction
                loss = _VocabParallelFLCEFunction.apply(hid, w, d["lab"], None, s["off"], -100,
                                                        self.CHUNK, None)
            loss.backward()
            return {"loss": loss.detach(), "dh": hid.grad, "dw": w.grad}

        def store(i, outs):
            for name, src in outs.items():
                ho[name].copy_(src, non_blocking=True)
            return outs.values()

        pipe.run(load, compute, store)

    def cpu_inputs(self, tokens, seed=7):
        g = torch.Generator().manual_seed(seed)
        if not hasattr(self, "_cpu_w"):
            self._cpu_w = (0.02 * torch.randn(self.V, self.H, generator=g)).bfloat16()
        h = torch.randn(tokens, self.H, generator=g).bfloat16()
        lab = torch.randint(0, self.V, (tokens,), generator=g)
        lab[: tokens // 10] = -100
        return {"h": h, "w": self._cpu_w, "lab": lab}

    def cpu_step(self, c):
        from oracle import ops as O

        loss, lse, mask = O.flce_forward(c["h"], c["w"], c["lab"], None, -100, 8192)
        O.flce_backward(c["h"], c["w"], c["lab"], lse, mask, 1.0, None, 8192)


class Lora:
    """fused LoRA QKV + MLP fwd+bwd, bf16, X [8,2048,4096], r=16, alpha=32."""

    name = "lora"
    short = "configs[3] LoRA QKV+MLP bf16 X[8,2048,4096] r16"
    bound = "tensor"
    dtype = "bf16"
    e2e_pipelined = True
    T, H, I, R, S = 8 * 2048, 4096, 12288, 16, 2.0
    QO, KVO = 4096, 1024
    dominant = "lora_mlp_backward"

    def __init__(self):
        T, H, I, r = self.T, self.H, self.I, self.R
        self.tokens = T
        qkv_o = self.QO + 2 * self.KVO
        lora_f = lambda i, o: 2 * r * (i + o)  # noqa: E731  x A^T and U B^T
        self.flops = {
            "lora_qkv_forward": T * (2 * H * qkv_o + sum(lora_f(H, o) for o in
                                                         (self.QO, self.KVO, self.KVO))),
            "lora_qkv_backward": T * (2 * H * qkv_o + sum(2 * r * (2 * o + 2 * H) for o in
                                                          (self.QO, self.KVO, self.KVO))),
            "lora_mlp_forward": T * (3 * 2 * H * I + 2 * lora_f(H, I) + lora_f(I, H)),
            "lora_mlp_backward": T * (3 * 2 * H * I + 2 * 2 * r * (2 * I + 2 * H) +
                                      2 * r * (2 * H + 2 * I)),
        }
        self.bytes = {}
        # GEMM + pack launches per op (counted from csrc/lora.cu)
        self.launches_per_step = (4 + 4) + (1 + 3 * 2 + 2 + 2 + 3 * 2 + 3) + \
            (6 + 4 + 1 + 1) + (5 + 6 + 2 + 1 + 1 + 4 + 2 + 4)

    def config(self):
        return {"workload": "lora_bf16 (BASELINE configs[3]): X [8,2048,4096]; Wq [4096,4096], "
                            "Wk/Wv [1024,4096], Wgate/Wup [12288,4096], Wdown [4096,12288] "
                            "~N(0,0.02); r=16, alpha=32; QKV + MLP forward and backward "
                            "(dX, dA, dB of all 6 adapters)",
                "tokens_per_step": self.T, "hidden": self.H, "intermediate": self.I,
                "rank": self.R, "parallelism": "replicas (token rows; no collective)",
                "l2": "inputs larger than L2 (X 128 MB, Wgate/Wup/Wdown 100 MB each)"}

    def _proj(self, g, o, i, device):
        w = (0.02 * torch.randn(o, i, generator=g, device=device)).bfloat16()
        a = (0.01 * torch.randn(self.R, i, generator=g, device=device)).bfloat16()
        b = (0.01 * torch.randn(o, self.R, generator=g, device=device)).bfloat16()
        return w, a, b

    def make_inputs(self, device, seed=1237):
        g = torch.Generator(device=device).manual_seed(seed)
        T, H, I = self.T, self.H, self.I
        t = {"x": torch.randn(T, H, generator=g, device=device).bfloat16()}
        t["q"], t["k"], t["v"] = (self._proj(g, o, H, device) for o in (self.QO, self.KVO,
                                                                          self.KVO))
        t["g"], t["u"] = self._proj(g, I, H, device), self._proj(g, I, H, device)
        t["d"] = self._proj(g, H, I, device)
        for name, o in (("dq", self.QO), ("dk", self.KVO), ("dv", self.KVO), ("dy", H)):
            t[name] = torch.randn(T, o, generator=g, device=device).bfloat16()
        return t

    def step(self, t, timer=plain):
        ops = torch.ops.metal_liger
        s3 = [self.S] * 3
        qkv = (*t["q"], *t["k"], *t["v"])
        Q, K, V, U = timer("lora_qkv_forward", ops.lora_qkv_forward, t["x"], *qkv, s3)
        timer("lora_qkv_backward", ops.lora_qkv_backward, t["x"], U, *qkv, s3, t["dq"], t["dk"],
              t["dv"])
        mlp = (*t["g"], *t["u"], *t["d"])
        out, gate, up, h, u1, u2 = timer("lora_mlp_forward", ops.lora_mlp_forward, t["x"], *mlp,
                                         s3)
        timer("lora_mlp_backward", ops.lora_mlp_backward, t["x"], gate, up, h, u1, u2, *mlp, s3,
              t["dy"])

    def e2e_setup(self, device):
        t = self.make_inputs(device, seed=80)
        names = ("x", "dq", "dk", "dv", "dy")
        host = {k: t[k].cpu().pin_memory() for k in names}
        dev = {k: torch.empty_like(t[k]) for k in names}
        T, H = self.T, self.H
        outs = {"Q": (T, self.QO), "K": (T, self.KVO), "V": (T, self.KVO), "out": (T, H),
                "dx_qkv": (T, H), "dx_mlp": (T, H)}
        host_out = {k: torch.empty(s, dtype=torch.bfloat16, pin_memory=True)
                    for k, s in outs.items()}
        for i, (o, fin) in enumerate(((self.QO, H), (self.KVO, H), (self.KVO, H), (self.I, H),
                                      (self.I, H), (H, self.I))):
            host_out[f"dA{i}"] = torch.empty((self.R, fin), pin_memory=True)
            host_out[f"dB{i}"] = torch.empty((o, self.R), pin_memory=True)
        params = {k: t[k] for k in ("q", "k", "v", "g", "u", "d")}
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        d2h = sum(v.numel() * v.element_size() for v in host_out.values())
        return {"host": host, "dev": dev, "host_out": host_out, "params": params, "h2d": h2d,
                "d2h": d2h, "pipe": CopyPipeline(device, self.E2E_CHUNKS)}

    E2E_CHUNKS = 4  # 4096 token rows per chunk

    def e2e_step(self, s):
        from metal_liger_b200.ops.fused_lora import _LoRA_MLP, _LoRA_QKV

        d, h, ho, P = s["dev"], s["host"], s["host_out"], s["params"]
        nc = s["pipe"].nchunks
        rows = self.T // nc
        # one set of adapter leaves per step: their gradients accumulate over
        # the chunks (autograd adds), as over the token rows of one call
        leaves = {}
        for k in ("q", "k", "v", "g", "u", "d"):
            w, a, b = P[k]
            leaves[k] = (w, a.detach().requires_grad_(True), b.detach().requires_grad_(True),
                         self.S)

        def load(i):
            sl = slice(i * rows, (i + 1) * rows)
            for k in d:
                d[k][sl].copy_(h[k][sl], non_blocking=True)

        def compute(i):
            sl = slice(i * rows, (i + 1) * rows)
            x = d["x"][sl].detach().requires_grad_(True)
            Q, K, V = _LoRA_QKV.apply(x, *leaves["q"], *leaves["k"], *leaves["v"])
            torch.autograd.backward([Q, K, V], [d["dq"][sl], d["dk"][sl], d["dv"][sl]])
            x2 = d["x"][sl].detach().requires_grad_(True)
            out = _LoRA_MLP.apply(x2, *leaves["g"], *leaves["u"], *leaves["d"])
            out.backward(d["dy"][sl])
            outs = {"Q": Q.detach(), "K": K.detach(), "V": V.detach(), "out": out.detach(),
                    "dx_qkv": x.grad, "dx_mlp": x2.grad}
            if i == nc - 1:
                for j, k in enumerate(("q", "k", "v", "g", "u", "d")):
                    outs[f"dA{j}"] = leaves[k][1].grad.float()
                    outs[f"dB{j}"] = leaves[k][2].grad.float()
            return outs

        def store(i, outs):
            sl = slice(i * rows, (i + 1) * rows)
            for name, src in outs.items():
                dst = ho[name] if name.startswith("d") and name[1] in "AB" else ho[name][sl]
                dst.copy_(src, non_blocking=True)
            return outs.values()

        s["pipe"].run(load, compute, store)

    def cpu_inputs(self, tokens, seed=8):
        g = torch.Generator().manual_seed(seed)
        if not hasattr(self, "_cpu_p"):
            self._cpu_p = {k: (*self._proj(g, o, i, "cpu"), self.S) for k, o, i in
                           (("q", self.QO, self.H), ("k", self.KVO, self.H),
                            ("v", self.KVO, self.H), ("g", self.I, self.H), ("u", self.I, self.H),
                            ("d", self.H, self.I))}
        c = {"x": torch.randn(tokens, self.H, generator=g).bfloat16()}
        for name, o in (("dq", self.QO), ("dk", self.KVO), ("dv", self.KVO), ("dy", self.H)):
            c[name] = torch.randn(tokens, o, generator=g).bfloat16()
        return c

    def cpu_step(self, c):
        from oracle import ops as O

        P = self._cpu_p
        O.lora_qkv_forward(c["x"], P["q"], P["k"], P["v"])
        O.lora_qkv_backward(c["x"], P["q"], P["k"], P["v"], c["dq"], c["dk"], c["dv"])
        O.lora_mlp_forward(c["x"], P["g"], P["u"], P["d"])
        O.lora_mlp_backward(c["x"], P["g"], P["u"], P["d"], c["dy"])


class FullStep:
    """one LoRA training step of the Qwen3-VL-8B text decoder.

    transformers' ``Qwen3VLTextModel`` at the 8B text shape (36 layers, hidden
    4096, 32 q / 8 kv heads of 128, SwiGLU 12288, vocab 151936, RMSNorm eps
    1e-6, RoPE theta 5e6), random init, bf16, PEFT-layout LoRA r=16 alpha=32 on
    q/k/v/o/gate/up/down, patched with ``apply_metal_liger_to_qwen3vl`` (all
    fusions on, including the B200 extensions: per-head q/k norm, RoPE inside
    attention, fused o_proj) and the loss from
    ``MetalLigerFusedLinearCrossEntropy`` over the frozen lm_head.  A step is
    forward, backward, the NCCL all-reduce of the LoRA gradients (N > 1) and an
    AdamW step.  One sequence of 4096 random token ids per GPU (8 GPUs = the
    BASELINE's batch 8 x 4096).  Attention is torch SDPA (library kernel).
    """

    name = "c5_step"
    short = "configs[4] Qwen3-VL-8B text LoRA step, 36 layers, seq 4096 per GPU"
    bound = "tensor"
    dtype = "bf16"
    single_bracket = True  # one timed bracket, the whole training step
    L, H, NH, NKV, D, I, V = 36, 4096, 32, 8, 128, 12288, 151936
    R, ALPHA, SEQ, THETA = 16, 32.0, 4096, 5e6
    dominant = "train_step"
    TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")

    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.batch = 1
        self.tokens = self.batch * self.SEQ
        self.flops = {"train_step": self.flops_per_token(self.L) * self.tokens}
        self.bytes = {}
        self.launches_per_step = None  # counted with the profiler

    # algorithmic FLOPs per token (frozen base weights: no dW; causal attention)
    def flops_per_token(self, layers):
        H, I, r = self.H, self.I, self.R
        q, kv = self.NH * self.D, self.NKV * self.D
        dense = 2 * (H * q + 2 * H * kv + q * H + 3 * H * I)        # forward GEMMs
        adapters = [(H, q), (H, kv), (H, kv), (q, H), (H, I), (H, I), (I, H)]
        lora = sum(2 * r * 3 * (fin + fout) for fin, fout in adapters)  # fwd + bwd rank terms
        attn_fwd = 2 * 2 * self.D * self.NH * (self.SEQ // 2)      # QK^T and PV, causal
        layer = 2 * dense + lora + 3 * attn_fwd                     # fwd + bwd (dX only)
        head = 2 * 2 * H * self.V                                   # logits + dX
        return layers * layer + head

    def config(self):
        return {"workload": "c5_full_step (BASELINE configs[4]): Qwen3-VL-8B text decoder LoRA "
                            "training step, transformers Qwen3VLTextModel random init, bf16, "
                            "36 layers, hidden 4096, 32/8 heads x 128, SwiGLU 12288, vocab "
                            "151936, LoRA r=16 alpha=32 on q/k/v/o/gate/up/down, fused FLCE "
                            "loss, AdamW on the adapters",
                "model": "Qwen3-VL-8B (text decoder)", "layers": self.L,
                "global_batch": self.batch * self.world, "seq_len": self.SEQ,
                "tokens_per_step_per_gpu": self.tokens,
                "parallelism": (f"dp{self.world} (token rows; NCCL all-reduce of LoRA grads)"
                                if self.world > 1 else "single GPU"),
                "attention": "torch SDPA (causal)",
                "flops_per_token": self.flops_per_token(self.L),
                "l2": "inputs larger than L2 (16 GB of frozen weights streamed per step)"}

    def _build(self, device, layers, dtype=torch.bfloat16, fused=True, seed=1238):
        import torch.nn as nn
        from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
        from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel

        from metal_liger_b200.lora_adapters import inject_lora, lora_parameters

        cfg = Qwen3VLTextConfig(hidden_size=self.H, intermediate_size=self.I,
                                num_hidden_layers=layers, num_attention_heads=self.NH,
                                num_key_value_heads=self.NKV, head_dim=self.D, vocab_size=self.V,
                                rms_norm_eps=1e-6, max_position_embeddings=self.SEQ,
                                rope_parameters={"rope_type": "default", "rope_theta": self.THETA,
                                                 "mrope_section": [24, 20, 20]})
        cfg._attn_implementation = "sdpa"
        torch.manual_seed(seed)
        holder = nn.Module()
        with torch.device(device):
            holder.model = Qwen3VLTextModel(cfg).to(dtype)
            holder.lm_head = nn.Linear(self.H, self.V, bias=False).to(dtype)
            with torch.no_grad():
                holder.lm_head.weight.normal_(0.0, 0.02)
        inject_lora(holder, r=self.R, alpha=self.ALPHA, targets=self.TARGETS, init_std=0.01)
        if fused:
            from metal_liger_b200 import apply_metal_liger_to_qwen3vl

            apply_metal_liger_to_qwen3vl(holder, fuse_qk_norm=True, fuse_rope_in_attention=True,
                                         fuse_lora_o_proj=True)
            # the patched norms hold new (trainable) Parameters, as in the
            # reference's patcher; LoRA training keeps everything but the
            # adapters frozen
            for n, p in holder.named_parameters():
                if "lora_" not in n:
                    p.requires_grad_(False)
        params = lora_parameters(holder)
        opt = torch.optim.AdamW(params, lr=1e-4, fused=(device != "cpu" and
                                                         torch.device(device).type == "cuda"))
        return holder, params, opt

    def make_inputs(self, device, seed=1239):
        self.model, self.params, self.opt = self._build(device, self.L)
        g = torch.Generator(device=device).manual_seed(seed + self.rank)
        ids = torch.randint(0, self.V, (self.batch, self.SEQ), generator=g, device=device)
        labels = torch.roll(ids, -1, dims=1)
        labels[:, -1] = -100
        return {"ids": ids, "labels": labels}

    def _train_step(self, ids, labels):
        from metal_liger_b200.ops.fused_linear_cross_entropy import \
            MetalLigerFusedLinearCrossEntropy

        m = self.model
        # Text-only positions (0..S-1 in every mrope section) passed as the 3-D
        # [3, B, S] ids the model builds itself; as 3-D ids they skip HF's
        # packed-sequence probe, a device-to-host sync every step.
        pos = self._positions(ids)
        h = m.model(input_ids=ids, position_ids=pos, use_cache=False).last_hidden_state
        loss = MetalLigerFusedLinearCrossEntropy(m.lm_head)(h, labels)
        loss.backward()
        if self.world > 1:
            from metal_liger_b200.data_parallel import all_reduce_gradients

            all_reduce_gradients(self.params)
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return loss.detach()

    def _positions(self, ids):
        key = (ids.shape, ids.device)
        if getattr(self, "_pos_key", None) != key:
            b, s = ids.shape
            self._pos = torch.arange(s, device=ids.device).view(1, 1, s).expand(3, b, s)
            self._pos_key = key
        return self._pos

    def step(self, t, timer=plain):
        timer("train_step", self._train_step, t["ids"], t["labels"])

    def e2e_setup(self, device):
        g = torch.Generator().manual_seed(81 + self.rank)
        ids = torch.randint(0, self.V, (self.batch, self.SEQ), generator=g)
        labels = torch.roll(ids, -1, dims=1)
        labels[:, -1] = -100
        host = {"ids": ids.pin_memory(), "labels": labels.pin_memory()}
        dev = {k: torch.empty_like(v, device=device) for k, v in host.items()}
        host_out = {"loss": torch.empty((), pin_memory=True)}
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        return {"host": host, "dev": dev, "host_out": host_out, "h2d": h2d, "d2h": 4}

    def e2e_step(self, s):
        d, h, ho = s["dev"], s["host"], s["host_out"]
        for k in d:
            d[k].copy_(h[k], non_blocking=True)
        loss = self._train_step(d["ids"], d["labels"])
        ho["loss"].copy_(loss.float(), non_blocking=True)

    # CPU baseline: the same step, unfused (transformers' modules, PEFT-layout
    # adapters, F.cross_entropy) in fp32 with ONE decoder layer; tokens/s are
    # scaled to 36 layers by the FLOP ratio (labelled as extrapolated).
    cpu_extrapolated = True
    cpu_desc = ("the unfused step with ONE decoder layer (transformers modules, PEFT-layout "
                "adapters, F.cross_entropy, fp32)")

    def cpu_inputs(self, tokens, seed=9):
        if not hasattr(self, "_cpu_model"):
            self._cpu_model, self._cpu_params, self._cpu_opt = self._build(
                "cpu", 1, dtype=torch.float32, fused=False)
        g = torch.Generator().manual_seed(seed)
        ids = torch.randint(0, self.V, (1, tokens), generator=g)
        labels = torch.roll(ids, -1, dims=1)
        labels[:, -1] = -100
        return {"ids": ids, "labels": labels}

    def cpu_step(self, c):
        import sys

        import torch.nn.functional as F

        m = self._cpu_model
        # The GPU model's patch rebinds the modeling module's rotary function
        # (shared with this unpatched CPU model): use the original here.
        mod = sys.modules[type(m.model.layers[0].self_attn).__module__]
        orig = getattr(mod, "_metal_liger_original_rope", None)
        fused = mod.apply_rotary_pos_emb
        if orig is not None:
            mod.apply_rotary_pos_emb = orig
        try:
            h = m.model(input_ids=c["ids"], use_cache=False).last_hidden_state
            logits = h @ m.lm_head.weight.t()
            loss = F.cross_entropy(logits.view(-1, self.V), c["labels"].view(-1),
                                   ignore_index=-100)
            loss.backward()
            self._cpu_opt.step()
            self._cpu_opt.zero_grad(set_to_none=True)
        finally:
            mod.apply_rotary_pos_emb = fused

    def cpu_scale(self):
        """Multiply the 1-layer CPU tokens/s by this to extrapolate to 36 layers."""
        return self.flops_per_token(1) / self.flops_per_token(self.L)


class Generate:
    """Greedy decoding with the static-KV generator (the reference's
    generation.py:68-129 path) on the Qwen3-VL-8B text decoder.

    transformers' ``Qwen3VLTextModel`` at the 8B text shape, random init,
    bf16, patched for inference (fused RMSNorm incl. the per-head q/k norms,
    fused SwiGLU, RoPE inside attention), with a bf16 lm_head.  A step is one
    ``MetalLigerGenerator.generate`` call: a 128-token prompt, then 64 new
    tokens for one sequence, greedy.  Decode is HBM-bound on the weights
    (16.4 GB per token); the roofline line is this library's kernel on that
    path, the fused lm_head argmax (one pass over the 1.24 GB lm_head per
    token).  Decoding replays a CUDA graph of one self-advancing decode step
    per token (the generator's default) in which every decoder layer runs as
    five of this library's launches (input norm + q/k/v GEMV; q/k norm,
    RoPE, cache write and attention; o GEMV + residual; post-attention norm
    + gate/up/SwiGLU GEMV; down GEMV + residual); the prefill runs the
    patched modules (cuBLAS projections, SDPA attention)."""

    name = "generate"
    short = "static-KV greedy generate, Qwen3-VL-8B text, prompt 128 + 64 tokens"
    bound = "hbm"
    dtype = "bf16"
    L, H, NH, NKV, D, I, V = 36, 4096, 32, 8, 128, 12288, 151936
    PROMPT, NEW, THETA = 128, 64, 5e6
    dominant = "lm_head_argmax"

    def __init__(self):
        self.batch = 1
        self.tokens = self.batch * self.NEW           # generated tokens per step
        self.bytes = {"lm_head_argmax": self.V * self.H * 2}
        self.launches_per_step = None

    def flops_per_token(self, layers):
        H, I = self.H, self.I
        q, kv = self.NH * self.D, self.NKV * self.D
        return layers * 2 * (H * q + 2 * H * kv + q * H + 3 * H * I) + 2 * H * self.V

    def config(self):
        return {"workload": "generate (static-KV greedy generator): Qwen3-VL-8B text "
                            "decoder, transformers Qwen3VLTextModel random init, bf16, 36 layers, "
                            "hidden 4096, 32/8 heads x 128, SwiGLU 12288, vocab 151936; prompt "
                            f"{self.PROMPT} tokens, {self.NEW} new tokens, batch 1, greedy",
                "model": "Qwen3-VL-8B (text decoder)", "layers": self.L,
                "global_batch": self.batch, "seq_len": self.PROMPT + self.NEW,
                "tokens_per_step": self.tokens, "parallelism": "replicas",
                "metric_note": "value = generated tokens/s including the prefill of each call",
                "l2": "inputs larger than L2 (16.4 GB of weights streamed per token)"}

    def _build(self, device, layers, dtype=torch.bfloat16, fused=True, seed=1240):
        import torch.nn as nn
        from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
        from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel

        cfg = Qwen3VLTextConfig(hidden_size=self.H, intermediate_size=self.I,
                                num_hidden_layers=layers, num_attention_heads=self.NH,
                                num_key_value_heads=self.NKV, head_dim=self.D, vocab_size=self.V,
                                rms_norm_eps=1e-6, max_position_embeddings=4096,
                                rope_parameters={"rope_type": "default", "rope_theta": self.THETA,
                                                 "mrope_section": [24, 20, 20]})
        cfg._attn_implementation = "sdpa"
        torch.manual_seed(seed)
        holder = nn.Module()
        with torch.device(device):
            holder.model = Qwen3VLTextModel(cfg).to(dtype)
            holder.lm_head = nn.Linear(self.H, self.V, bias=False).to(dtype)
            with torch.no_grad():
                holder.lm_head.weight.normal_(0.0, 0.02)
        holder.config = cfg
        if fused:
            from metal_liger_b200 import apply_metal_liger_to_qwen3vl

            apply_metal_liger_to_qwen3vl(holder, fuse_lora=False, fuse_qk_norm=True,
                                         fuse_rope_in_attention=True)
        holder.eval()
        for p in holder.parameters():
            p.requires_grad_(False)
        return holder

    def make_inputs(self, device, seed=1241):
        from metal_liger_b200.generation import MetalLigerGenerator

        self.model = self._build(device, self.L)
        outer = self

        class _Timed(MetalLigerGenerator):
            # The head is timed where it runs eagerly (prefill and the steps
            # before the decode graph is captured); inside the captured step
            # events cannot be timed.
            def _greedy(self, h):
                if torch.cuda.is_current_stream_capturing():
                    return super()._greedy(h)
                return outer._timer("lm_head_argmax", super()._greedy, h)

        self.gen = _Timed(self.model)
        self._timer = plain
        g = torch.Generator(device=device).manual_seed(seed)
        ids = torch.randint(0, self.V, (self.batch, self.PROMPT), generator=g, device=device)
        return {"ids": ids}

    def step(self, t, timer=plain):
        self._timer = timer
        try:
            return self.gen.generate(t["ids"], max_new_tokens=self.NEW)
        finally:
            self._timer = plain

    def e2e_setup(self, device):
        g = torch.Generator().manual_seed(82)
        host = {"ids": torch.randint(0, self.V, (self.batch, self.PROMPT), generator=g)
                .pin_memory()}
        dev = {"ids": torch.empty_like(host["ids"], device=device)}
        host_out = {"out": torch.empty((self.batch, self.PROMPT + self.NEW), dtype=torch.int64,
                                       pin_memory=True)}
        return {"host": host, "dev": dev, "host_out": host_out,
                "h2d": host["ids"].numel() * 8, "d2h": host_out["out"].numel() * 8}

    def e2e_step(self, s):
        from metal_liger_b200.generation import MetalLigerGenerator

        if not hasattr(self, "_plain_gen"):
            self._plain_gen = MetalLigerGenerator(self.model)
        s["dev"]["ids"].copy_(s["host"]["ids"], non_blocking=True)
        out = self._plain_gen.generate(s["dev"]["ids"], max_new_tokens=self.NEW)
        s["host_out"]["out"][:, :out.shape[1]].copy_(out, non_blocking=True)

    def extra_measurements(self, device, steps=3):
        """The reference's decode loop run on the same GPU model for
        comparison: transformers' DynamicCache, [batch, vocab] logits from
        the lm_head, torch.argmax and a torch.cat per token
        (generation.py:88-127), timed with CUDA events."""
        from transformers.cache_utils import DynamicCache

        m = self.model

        @torch.inference_mode()
        def loop(ids):
            cache = DynamicCache()
            h = m.model(input_ids=ids, past_key_values=cache, use_cache=True).last_hidden_state
            nxt = torch.argmax(m.lm_head(h[:, -1:, :])[:, -1, :], dim=-1, keepdim=True)
            out = torch.cat([ids, nxt], dim=-1)
            for _ in range(self.NEW - 1):
                h = m.model(input_ids=nxt, past_key_values=cache, use_cache=True).last_hidden_state
                nxt = torch.argmax(m.lm_head(h[:, -1:, :])[:, -1, :], dim=-1, keepdim=True)
                out = torch.cat([out, nxt], dim=-1)
            return out

        g = torch.Generator(device=device).manual_seed(83)
        ids = torch.randint(0, self.V, (self.batch, self.PROMPT), generator=g, device=device)
        loop(ids)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            ref = loop(ids)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        ours = self.gen.generate(ids, max_new_tokens=self.NEW)

        # The head alone at batch 1 (one decode step's lm_head pass), against
        # the reference's logits GEMM + argmax (torch / cuBLAS).
        h1 = torch.randn(1, self.H, generator=g, device=device).bfloat16()
        w = m.lm_head.weight
        from metal_liger_b200.generation import _logit_code

        def head_ms(fn, reps=50):
            for _ in range(5):
                fn()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(reps)]
            for a, b in ev:
                a.record()
                fn()
                b.record()
            torch.cuda.synchronize()
            return sorted(a.elapsed_time(b) for a, b in ev)[reps // 2]

        fused = head_ms(lambda: torch.ops.metal_liger.lm_head_argmax(h1, w, None,
                                                                     _logit_code(w.dtype)))
        plain_head = head_ms(lambda: torch.argmax(torch.nn.functional.linear(h1, w), dim=-1))
        # Token agreement: equal prefix length, and whether the first
        # difference is a near-tie of the reference's own logits there (the
        # best two within one bf16 ulp), i.e. a rounding-order divergence.
        same = bool(torch.equal(ref, ours))
        agree = int(ref.shape[1])
        near_tie = None
        if not same:
            diff = (ref[0] != ours[0]).nonzero()
            agree = int(diff[0]) if diff.numel() else int(ref.shape[1])
            with torch.inference_mode():
                hh = m.model(input_ids=ref[:, :agree]).last_hidden_state[:, -1]
                top2 = m.lm_head(hh).float()[0].topk(2).values
            gap = float(top2[0] - top2[1])
            ulp = 2.0 ** (int(torch.floor(torch.log2(top2[0].abs()))) - 7)
            near_tie = gap <= ulp

        return {"lm_head_argmax_alone": {
            "batch": 1, "median_us": fused * 1e3,
            "GB/s": self.bytes["lm_head_argmax"] / (fused / 1e3) / 1e9,
            "torch_linear_argmax_us": plain_head * 1e3,
            "what": "one lm_head pass (151936 x 4096 bf16), median of 50 event-timed calls"},
            "reference_loop_on_gpu": {
            "value": self.tokens / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "what": "the reference's decode loop (transformers DynamicCache, full-vocabulary "
                    "logits, argmax, torch.cat) on the same patched model and GPU",
            "same_tokens": same, "generated_tokens_agreeing": agree - self.PROMPT,
            "first_difference_is_bf16_near_tie": near_tie}}

    # CPU baseline: the reference's decode loop (oracle/generation.py: a
    # transformers KV cache, full-vocabulary logits, argmax, torch.cat) in
    # fp32 with ONE decoder layer; tokens/s scaled to 36 layers by the FLOP
    # ratio (labelled as extrapolated).
    cpu_extrapolated = True
    cpu_desc = ("the reference's greedy decode loop (transformers KV cache, full-vocabulary "
                "logits, argmax, torch.cat; oracle/generation.py) with ONE decoder layer, fp32")
    metric = "greedy decode tokens/s (static-KV generator, Qwen3-VL-8B text)"
    e2e_api = ("MetalLigerGenerator.generate from pinned host prompt ids; the generated ids "
               "copied back to pinned host memory every step")

    def cpu_inputs(self, tokens, seed=10):
        if not hasattr(self, "_cpu_model"):
            self._cpu_model = self._build("cpu", 1, dtype=torch.float32, fused=False)
        g = torch.Generator().manual_seed(seed)
        return {"ids": torch.randint(0, self.V, (1, self.PROMPT), generator=g),
                "new": max(1, int(tokens))}

    def cpu_step(self, c):
        import sys

        from oracle import generation as OG

        m = self._cpu_model
        mod = sys.modules[type(m.model.layers[0].self_attn).__module__]
        orig = getattr(mod, "_metal_liger_original_rope", None)
        fused = mod.apply_rotary_pos_emb
        if orig is not None:
            mod.apply_rotary_pos_emb = orig
        try:
            OG.generate(m, c["ids"], max_new_tokens=c["new"])
        finally:
            mod.apply_rotary_pos_emb = fused

    def cpu_scale(self):
        return self.flops_per_token(1) / self.flops_per_token(self.L)


METRIC = "fwd+bwd tokens/s per fused op at Qwen3-VL shapes"

WORKLOADS = {"swiglu_rope": SwigluRope, "rmsnorm": RmsNorm, "flce": Flce, "lora": Lora,
             "c5_step": FullStep, "generate": Generate}


def _register_optional_workloads():
    return


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------

_OUR_KERNEL = None


def count_our_launches(wl, t, table: bool = False) -> int | None:
    """Kernels from this repository's library launched by one step, counted
    with the CUDA profiler (CUPTI) on an extra, untimed step.  With `table`,
    also prints that step's per-kernel device time (all kernels) to stderr."""
    global _OUR_KERNEL
    import re

    if _OUR_KERNEL is None:
        _OUR_KERNEL = re.compile(r"(^|[^A-Za-z0-9_])(ml|gemm|flce|lora)::")
    try:
        from torch.profiler import ProfilerActivity, profile

        prelude = getattr(wl, "prelude", None)
        if prelude:
            prelude(t)
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            wl.step(t)
            torch.cuda.synchronize()
        n = 0
        per = {}
        for ev in prof.events():
            if getattr(ev, "device_type", None) != torch.autograd.DeviceType.CUDA:
                continue
            name = ev.name or ""
            ours = bool(_OUR_KERNEL.search(name))
            n += ours
            c, us = per.get(name, (0, 0.0))
            tr = getattr(ev, "time_range", None)
            per[name] = (c + 1, us + ((tr.end - tr.start) if tr is not None else 0.0))
        if table:
            total = sum(us for _, us in per.values()) or 1.0
            print(f"# one step, per-kernel device time (CUPTI): total {total / 1e3:.2f} ms",
                  file=sys.stderr)
            for name, (c, us) in sorted(per.items(), key=lambda kv: -kv[1][1])[:40]:
                print(f"# {us / 1e3:9.3f} ms {100 * us / total:5.1f}% {c:6d}  {name[:120]}",
                      file=sys.stderr)
        return n
    except Exception:
        return None


def cpu_measure(wl, budget_s: float, max_steps: int | None = None):
    """Time the CPU oracle on a bounded sample: returns (tokens/s, tokens, steps, cores)."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    tokens = 64
    c = wl.cpu_inputs(tokens)
    t0 = time.perf_counter()
    wl.cpu_step(c)
    dt = max(time.perf_counter() - t0, 1e-4)
    per_tok = dt / tokens
    steps = max_steps or 3
    tokens = int(max(16, min(wl.tokens, budget_s / steps / per_tok)))
    c = wl.cpu_inputs(tokens)
    wl.cpu_step(c)  # warm
    t0 = time.perf_counter()
    for _ in range(steps):
        wl.cpu_step(c)
    el = time.perf_counter() - t0
    return tokens * steps / el, tokens, steps, torch.get_num_threads()


def run_reference_arm(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    budget = float(os.environ.get("BENCH_CPU_BUDGET_S", "90"))
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    per_step_budget = budget / max(1, args.steps + args.warmup)
    # calibrate the sample size so the whole run stays within the budget
    c = wl.cpu_inputs(64)
    t0 = time.perf_counter()
    wl.cpu_step(c)
    per_tok = max(time.perf_counter() - t0, 1e-4) / 64
    tokens = int(max(16, min(wl.tokens, per_step_budget / per_tok)))
    c = wl.cpu_inputs(tokens)
    for _ in range(args.warmup):
        wl.cpu_step(c)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        wl.cpu_step(c)
    el = time.perf_counter() - t0
    value = tokens * args.steps / el
    sample = (f"{tokens} of {wl.tokens} tokens per step (same shapes per token), "
              f"torch CPU fp32 oracle restating the reference ops, TORCHDYNAMO_DISABLE=1")
    if getattr(wl, "cpu_extrapolated", False):
        value *= wl.cpu_scale()
        sample = (f"{tokens} tokens per step of {wl.cpu_desc}; "
                  f"tokens/s extrapolated to {wl.L} layers by the FLOP ratio "
                  f"{wl.cpu_scale():.4f}")
    line = {
        "impl": "reference",
        "metric": getattr(wl, "metric", METRIC),
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * wl.tokens / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": wl.dtype,
        "data": "synthetic", "config": wl.config(),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _sig(x, n=5):
    """x rounded to n significant digits (keeps the JSON line short)."""
    if isinstance(x, float) and math.isfinite(x) and x != 0.0:
        return float(f"{x:.{n}g}")
    return x


def _rounded(o, n=5):
    if isinstance(o, dict):
        return {k: _rounded(v, n) for k, v in o.items()}
    if isinstance(o, (list, tuple)):
        return [_rounded(v, n) for v in o]
    return _sig(o, n)


class Ctx:
    """Rank, device, process group and peaks shared by every measurement."""

    def __init__(self, args):
        self.args = args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.device = torch.device("cuda", self.local)
        self.dist = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist_mod

            dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                        device_id=self.device)
            self.dist = dist_mod
        self.peaks, self.peaks_kind = load_peaks()

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def reduce(self, x, op="max"):
        """x reduced over ranks (MAX or MIN) with one NCCL all-reduce."""
        if not self.dist:
            return x
        t = torch.tensor([float(x)], device=self.device, dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX if op == "max" else
                             self.dist.ReduceOp.MIN)
        return t.item()

    def close(self):
        if self.dist:
            self.dist.barrier()
            self.dist.destroy_process_group()


def timed_steps(ctx, wl, t, steps, warmup, spin_us, per_kernel=True):
    """W untimed steps, then the K timed steps: each step bracketed by one
    pair of CUDA events on the launching stream, with nothing between its
    launches.  Before a step's first event the stream gets the workload's
    untimed prelude (the L2 flush) and a short GPU spin, so the host has
    queued the whole step before the GPU reaches it.

    Then, for the per-kernel breakdown, K more steps with a pair of events
    around every launch (events between back-to-back launches add a few
    microseconds of launch gap each, which is why the step value comes from
    the first K); and for HBM-bound workloads each launch once more alone,
    after an L2 flush whose lines are then clean (the kernel's own bandwidth,
    without the write-back of the previous kernel's output).

    Returns (sum of the K step spans in ms, max over ranks; per-kernel
    average ms inside steps; per-kernel average ms alone; clock summary
    sampled during the K timed steps)."""
    prelude = getattr(wl, "prelude", None)
    for _ in range(warmup):
        if prelude:
            prelude(t)
        wl.step(t)
    torch.cuda.synchronize()
    spans = []
    spin_cycles = int(spin_us * 2000)  # ~2 GHz SM clock
    ctx.barrier()
    torch.cuda.synchronize()
    with ClockSampler(ctx.local) as clk:
        for _ in range(steps):
            if prelude:
                prelude(t)
            if spin_cycles:
                torch.cuda._sleep(spin_cycles)
            s_ev = torch.cuda.Event(enable_timing=True)
            e_ev = torch.cuda.Event(enable_timing=True)
            s_ev.record()
            wl.step(t)
            e_ev.record()
            spans.append((s_ev, e_ev))
        torch.cuda.synchronize()
    ctx.barrier()
    elapsed = ctx.reduce(sum(a.elapsed_time(b) for a, b in spans))
    name = getattr(wl, "dominant", "step")
    in_step = {name: elapsed / steps}
    alone = {}
    if per_kernel and not getattr(wl, "single_bracket", False):
        timer = KernelTimer()
        for _ in range(steps):
            if prelude:
                prelude(t)
            if spin_cycles:
                torch.cuda._sleep(spin_cycles)
            wl.step(t, timer)
        torch.cuda.synchronize()
        in_step = timer.averages_ms()
        if wl.bound == "hbm":
            flush = L2Flush(ctx.device)
            timer = KernelTimer(before=flush)
            for _ in range(steps):
                wl.step(t, timer)
            torch.cuda.synchronize()
            alone = timer.averages_ms()
    ctx.barrier()
    return elapsed, in_step, alone, clk.summary()


class L2Flush:
    """Evicts L2 (126 MB) so the next kernel reads from HBM and finds no
    dirty lines to write back: writes a 256 MB buffer, then reads another
    256 MB; a short spin follows so the next launch is queued in time."""

    def __init__(self, device):
        n = 256 * 1024 * 1024 // 4
        self.wr = torch.empty(n, dtype=torch.float32, device=device)
        self.rd = torch.zeros(n, dtype=torch.float32, device=device)

    def __call__(self):
        self.wr.fill_(0.0)
        self.rd.amax()
        torch.cuda._sleep(100000)


def peak_extra_bytes(wl, t):
    """Device memory one step allocates beyond what is resident before it
    (workspaces, temporaries and the step's outputs), from the caching
    allocator's peak counter on an extra, untimed step."""
    prelude = getattr(wl, "prelude", None)
    if prelude:
        prelude(t)
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    wl.step(t)
    torch.cuda.synchronize()
    return int(torch.cuda.max_memory_allocated() - base)


_LINK = {}


def host_link_ceiling(device, nbytes=256 << 20, reps=3):
    """Pinned host<->device copy rates of this GPU's host link, measured once
    per process: H2D alone, D2H alone and both directions at once (GB/s,
    best of `reps`, CUDA events).  The e2e step's copies cannot beat them."""
    if device in _LINK:
        return _LINK[device]
    hs = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    hd = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d1 = torch.empty(nbytes, dtype=torch.uint8, device=device)
    d2 = torch.empty(nbytes, dtype=torch.uint8, device=device)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def best(h2d, d2h):
        t = float("inf")
        for _ in range(reps):
            main = torch.cuda.current_stream(device)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(main)
            for st, on, fn in ((up, h2d, lambda: d1.copy_(hs, non_blocking=True)),
                               (down, d2h, lambda: hd.copy_(d2, non_blocking=True))):
                if on:
                    st.wait_event(a)
                    with torch.cuda.stream(st):
                        fn()
                    main.wait_stream(st)
            b.record(main)
            b.synchronize()
            t = min(t, a.elapsed_time(b))
        return t / 1e3

    _LINK[device] = {"h2d_gbs": nbytes / best(True, False) / 1e9,
                     "d2h_gbs": nbytes / best(False, True) / 1e9,
                     "duplex_gbs": 2 * nbytes / best(True, True) / 1e9}
    del hs, hd, d1, d2
    torch.cuda.empty_cache()
    return _LINK[device]


def link_roofline(link, h2d, d2h, ms_per_step):
    """The e2e step's copy floor on the measured link and the fraction of it
    reached: floor = the slowest of H2D alone, D2H alone and both at once."""
    if h2d + d2h == 0:
        return None
    floor_s = max(h2d / (link["h2d_gbs"] * 1e9), d2h / (link["d2h_gbs"] * 1e9),
                  (h2d + d2h) / (link["duplex_gbs"] * 1e9))
    return {**link, "floor_ms": 1e3 * floor_s, "frac": 1e3 * floor_s / ms_per_step}


def e2e_measure(ctx, wl, steps):
    s = wl.e2e_setup(ctx.device)
    for _ in range(2):
        wl.e2e_step(s)
    torch.cuda.synchronize()
    ctx.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        wl.e2e_step(s)
    if s.get("pipe") is not None:
        s["pipe"].join()
    e1.record()
    torch.cuda.synchronize()
    ms = ctx.reduce(e0.elapsed_time(e1))
    h2d, d2h = s["h2d"], s["d2h"]
    del s
    torch.cuda.empty_cache()
    return ms, h2d, d2h


def roofline(ctx, wl, kernel_ms, burst, alone_ms=None, step_ms=None):
    """The dominant kernel's roofline entry and the per-kernel fractions
    (inside the step, and alone after a clean L2 flush where measured); the
    entry also carries the whole step's algorithmic work over its time."""
    peaks = ctx.peaks
    dom = wl.dominant
    dom_ms = kernel_ms.get(dom)
    if wl.bound == "hbm":
        peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        achieved = wl.bytes[dom] / (dom_ms / 1e3) / 1e9
        unit = "GB/s"
        which = ""
    else:
        # The tensor-bound kernels run inside multi-millisecond steps repeated for
        # the whole timed region, i.e. under the 1 kW power cap: the sustained
        # cuBLAS figure is the matching denominator (--burst selects the other).
        key = "bf16_tflops" if burst else "bf16_tflops_sustained"
        peak = float(peaks.get(key, FALLBACK_PEAKS[key]))
        achieved = wl.flops[dom] / (dom_ms / 1e3) / 1e12
        unit = "TFLOP/s"
        which = ", burst" if burst else ", sustained"
    src = "MEASURED_PEAKS.json" if ctx.peaks_kind == "measured" else "profiling-recipe fallback"
    roof = {"kernel": dom, "bound": wl.bound, "achieved": achieved, "peak": peak,
            "peak_source": f"{ctx.peaks_kind} ({src}{which})", "unit": unit,
            "frac": achieved / peak, "traffic": load_traffic(wl.name, dom)}
    work = wl.bytes if wl.bound == "hbm" else getattr(wl, "flops", {})
    if step_ms and work:
        per_s = sum(work.values()) / (step_ms / 1e3) / (1e9 if wl.bound == "hbm" else 1e12)
        roof["step"] = {"achieved": per_s, "frac": per_s / peak,
                        "what": "all kernels' algorithmic work over the step time"}
    alone_ms = alone_ms or {}
    per_kernel = {}
    for k, ms in kernel_ms.items():
        entry = {"ms": ms}
        if wl.bound == "hbm" and k in wl.bytes:
            gbs = wl.bytes[k] / (ms / 1e3) / 1e9
            entry.update({"GB/s": gbs, "frac": gbs / float(peaks.get("hbm_gbs", 1))})
            if k in alone_ms:
                entry["frac_alone"] = (wl.bytes[k] / (alone_ms[k] / 1e3) / 1e9
                                       / float(peaks.get("hbm_gbs", 1)))
        if getattr(wl, "flops", None) and k in wl.flops:
            tf = wl.flops[k] / (ms / 1e3) / 1e12
            key = "bf16_tflops" if burst else "bf16_tflops_sustained"
            entry.update({"TFLOP/s": tf, "frac": tf / float(peaks.get(key, 1))})
        per_kernel[k] = entry
    return roof, per_kernel


def cpu_baseline(wl, budget_s):
    v, tok, st, cores = cpu_measure(wl, budget_s=budget_s)
    sample = (f"{tok} of {wl.tokens} tokens x {st} steps through the CPU oracle "
              f"(torch fp32 restatement of the reference ops), {cores} threads")
    if getattr(wl, "cpu_extrapolated", False):
        v *= wl.cpu_scale()
        sample = (f"{tok} tokens x {st} steps of {wl.cpu_desc} on {cores} threads; "
                  f"tokens/s extrapolated to {wl.L} layers by the FLOP ratio "
                  f"{wl.cpu_scale():.4f}")
    return {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}


def measure_workload(ctx, wl, steps, warmup, e2e_steps, cpu_budget, table=False, keep=False):
    """Device-timed value, roofline, launch count, peak memory, e2e and (rank 0
    at N=1) the CPU baseline of one workload.  With `keep`, the resident
    inputs are returned in the result under "inputs" instead of freed."""
    args = ctx.args
    t = wl.make_inputs(ctx.device)
    elapsed_ms, kernel_ms, alone_ms, clocks = timed_steps(ctx, wl, t, steps, warmup,
                                                          args.spin_us)
    launches = count_our_launches(wl, t, table=table and ctx.rank == 0)
    if launches is None:
        launches = wl.launches_per_step
    peak = peak_extra_bytes(wl, t)
    extra = None
    if ctx.rank == 0 and hasattr(wl, "extra_measurements"):
        extra = wl.extra_measurements(ctx.device)
    inputs = t if keep else None
    del t
    torch.cuda.empty_cache()
    # weak scaling: every rank processes wl.tokens; strong: the job processes wl.tokens
    job_tokens = wl.tokens * (ctx.world if getattr(wl, "scaling", "weak") == "weak" else 1)
    e2e_steps = max(1, min(steps, e2e_steps))
    e2e_ms, h2d, d2h = e2e_measure(ctx, wl, e2e_steps)
    roof, per_kernel = roofline(ctx, wl, kernel_ms, args.burst, alone_ms, elapsed_ms / steps)
    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu:
        cpu = cpu_baseline(wl, cpu_budget)
    return {
        "value": job_tokens * steps / (elapsed_ms / 1e3),
        "ms_per_step": elapsed_ms / steps,
        "roofline": roof, "per_kernel": per_kernel, "clocks": clocks,
        "gpu_launches": launches * steps if launches is not None else None,
        "peak_extra_bytes": peak,
        "e2e": {"value": job_tokens * e2e_steps / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "link": link_roofline(host_link_ceiling(ctx.device), h2d, d2h,
                                      e2e_ms / e2e_steps)},
        "cpu_baseline": cpu, "extra": extra, "inputs": inputs,
    }


def compact_entry(wl, r, steps):
    """One workload of the default run's `workloads` object."""
    roof = dict(r["roofline"])
    roof.pop("peak_source", None)
    if "step" in roof:
        roof["step"] = {k: v for k, v in roof["step"].items() if k != "what"}
    e = {"config": wl.short, "value": r["value"], "unit": "tokens/s",
         "ms_per_step": r["ms_per_step"], "steps": steps,
         "scaling": getattr(wl, "scaling", "weak"), "roofline": roof,
         "kernel_frac": {k: v.get("frac") for k, v in r["per_kernel"].items()},
         **({"kernel_frac_alone": {k: v["frac_alone"] for k, v in r["per_kernel"].items()
                                   if "frac_alone" in v}}
            if any("frac_alone" in v for v in r["per_kernel"].values()) else {}),
         "e2e": {**{k: r["e2e"][k] for k in ("value", "h2d_bytes_per_step", "d2h_bytes_per_step")},
                 **({"link_frac": r["e2e"]["link"]["frac"]} if r["e2e"].get("link") else {})},
         "gpu_launches": r["gpu_launches"], "peak_extra_bytes": r["peak_extra_bytes"],
         "clocks": {"sm_mhz": r["clocks"].get("sm_mhz"), "reasons": r["clocks"].get("reasons")}}
    if r["cpu_baseline"]:
        c = r["cpu_baseline"]
        e["cpu_baseline"] = {"value": c["value"], "cores": c["cores"], "kind": c["kind"],
                             "sample": c["sample"]}
    return e


def _frob(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp(min=1e-30)).item()


def _bf16_close(a, b):
    """Element-wise bf16 contract with the absolute term scaled to the
    tensor's largest magnitude (the FLCE gradients carry a 1/n_valid factor,
    so a fixed 1e-2 would pass anything): |a - b| <= 2e-2 |b| + 1e-2 max|b|."""
    a, b = a.float(), b.float()
    bad = (a - b).abs() > 2e-2 * b.abs() + 1e-2 * b.abs().max()
    return int(bad.sum().item())


def measure_flce_vp_p2p(ctx, args):
    """flce_vp again with VP_DX_EXCHANGE = "p2p" (no collective in the step);
    the compact fields, or the error every rank recorded."""
    import metal_liger_b200.ops.fused_linear_cross_entropy as flce_ops

    previous = flce_ops.VP_DX_EXCHANGE
    flce_ops.VP_DX_EXCHANGE = "p2p"
    try:
        fl = Flce()
        vp = measure_workload(ctx, fl, args.steps, args.warmup, 1, 0.0, keep=True)
        r = measure_flce_vp(ctx, args.steps, args.warmup, vp)
        del fl, vp
        from metal_liger_b200 import _C

        err = int(_C.load().ml_device_error(None))
        out = {k: r[k] for k in ("tokens_per_s", "ms_per_step", "one_gpu_ms_per_step",
                                 "speedup_vs_1", "parity", "worst_errors", "timeline_rank0")}
        out["device_error"] = err
    except Exception as exc:  # every rank runs the same steps; report, do not abort the line
        out = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    finally:
        flce_ops.VP_DX_EXCHANGE = previous
        torch.cuda.empty_cache()
    ctx.barrier()
    return out


def measure_flce_vp(ctx, steps, warmup, vp):
    """The vocabulary-parallel FLCE at N ranks (already timed in `vp`, with
    its inputs kept) against the single-GPU FLCE on the same seeded inputs:
    every rank times the single-GPU op on its own GPU (no collectives) for the
    speed-up, and checks its own vocabulary shard of the parallel result
    against the single-GPU result (loss, dX, dW rows, exact ignore count)."""
    from metal_liger_b200 import _C

    ops = torch.ops.metal_liger
    t = vp["inputs"]
    single = Flce(world=1, rank=0)
    full = single.make_inputs(ctx.device)  # the same seeded tensors, whole vocabulary
    ms1, _, _, _ = timed_steps(ctx, single, full, steps, warmup, ctx.args.spin_us,
                               per_kernel=False)

    # parity: one step of each on the same inputs
    vpw = Flce()
    loss_v, dx_v, dw_v = vpw._vp(t)
    gh_v, gw_v = ops.flce_backward(t["go"], dx_v, dw_v, 1, 1)
    loss_1, dx_1, dw_1 = ops.flce_forward(full["h"], full["w"], full["lab"], None, -100,
                                          single.CHUNK, True, True)
    gh_1, gw_1 = ops.flce_backward(full["go"], dx_1, dw_1, 1, 1)
    off, vl = t["off"], t["w"].shape[0]
    rows_1 = gw_1[off:off + vl]
    cnt = torch.empty(2, dtype=torch.float32, device=ctx.device)
    _C.call("ml_flce_count_valid", t["lab"].data_ptr(), t["lab"].numel(), -100,
            cnt.data_ptr(), _C.stream_of(t["lab"]))
    torch.cuda.synchronize()
    n_valid = int((t["lab"] != -100).sum().item())
    errs = {
        "loss_rel": abs(loss_v.item() - loss_1.item()) / max(abs(loss_1.item()), 1e-30),
        "dx_frob": _frob(gh_v, gh_1), "dw_frob": _frob(gw_v, rows_1),
        "dx_bad": _bf16_close(gh_v, gh_1), "dw_bad": _bf16_close(gw_v, rows_1),
    }
    ok = (errs["loss_rel"] <= 1e-4 and errs["dx_frob"] <= 1e-2 and errs["dw_frob"] <= 1e-2
          and errs["dx_bad"] == 0 and errs["dw_bad"] == 0 and int(cnt[0].item()) == n_valid)
    all_ok = ctx.reduce(1.0 if ok else 0.0, "min") == 1.0
    worst = {k: ctx.reduce(v) for k, v in errs.items()}
    del full, dx_1, dw_1, gh_1, gw_1, rows_1, gh_v, gw_v, dx_v, dw_v
    torch.cuda.empty_cache()

    # where the step's time goes: one profiled step (CUPTI) on every rank
    timeline = vp_timeline(vpw, t)
    tok = single.tokens
    import metal_liger_b200.ops.fused_linear_cross_entropy as flce_ops

    out = {"n_gpus": ctx.world, "scaling": "strong", "tokens_per_step": tok,
           "dx_exchange": (flce_ops.VP_DX_EXCHANGE if ctx.world > 1 else None),
           "tokens_per_s": tok * steps / (vp["ms_per_step"] * steps / 1e3),
           "ms_per_step": vp["ms_per_step"], "one_gpu_ms_per_step": ms1 / steps,
           "speedup_vs_1": (ms1 / steps) / vp["ms_per_step"],
           "parity": all_ok,
           "parity_vs": "single-GPU FLCE on the same seeded inputs, every rank's shard: loss "
                        "1e-4 rel, dX/dW |d| <= 2e-2|ref| + 1e-2 max|ref| and 1e-2 Frobenius, "
                        "ignore count exact",
           "worst_errors": worst, "n_valid": n_valid, "timeline_rank0": timeline,
           "roofline": {k: vp["roofline"][k] for k in ("kernel", "achieved", "peak", "unit",
                                                       "frac")},
           "clocks": {"sm_mhz": vp["clocks"].get("sm_mhz"),
                      "reasons": vp["clocks"].get("reasons")}}
    return out


def vp_timeline(wl, t):
    """Device time of one vocabulary-parallel step split into NCCL kernels and
    this library's kernels (CUPTI), with the step's event-timed span."""
    try:
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            wl.step(t)
            e.record()
            torch.cuda.synchronize()
        nccl = ours = other = 0.0
        for ev in prof.events():
            if getattr(ev, "device_type", None) != torch.autograd.DeviceType.CUDA:
                continue
            tr = getattr(ev, "time_range", None)
            us = (tr.end - tr.start) if tr is not None else 0.0
            name = ev.name or ""
            if "nccl" in name.lower():
                nccl += us
            elif _OUR_KERNEL is not None and _OUR_KERNEL.search(name):
                ours += us
            else:
                other += us
        return {"span_ms": s.elapsed_time(e), "nccl_kernel_ms": nccl / 1e3,
                "library_kernel_ms": ours / 1e3, "other_kernel_ms": other / 1e3}
    except Exception as exc:  # the timeline is diagnostic only
        return {"error": str(exc)[:120]}


SUITE_N1 = ("rmsnorm", "flce", "lora", "c5_step")
SUITE_NN = ("rmsnorm", "lora", "c5_step")  # flce runs as flce_vp at N > 1


def run_gpu_arm(args, wl):
    if not torch.cuda.is_available():
        print(json.dumps({"error": "no CUDA device"}), flush=True)
        return 1
    ctx = Ctx(args)
    import metal_liger_b200  # noqa: F401  (registers ops, loads the library on first call)
    from metal_liger_b200 import _C

    _C.load()
    suite = args.workload is None and not args.headline_only
    r = measure_workload(ctx, wl, args.steps, args.warmup, args.e2e_steps, args.cpu_budget,
                         table=args.kernel_table)

    workloads, flce_vp = {}, None
    chosen = None if args.suite is None else {x for x in args.suite.split(",") if x}
    if suite:
        for name in (SUITE_N1 if ctx.world == 1 else SUITE_NN):
            if chosen is not None and name not in chosen:
                continue
            sub = WORKLOADS[name]()
            res = measure_workload(ctx, sub, args.steps, args.warmup, args.e2e_steps,
                                   args.cpu_budget_sub)
            workloads[name] = compact_entry(sub, res, args.steps)
            if ctx.world == 1 and name == "flce":
                flce_vp = {"n_gpus": 1, "scaling": "strong", "tokens_per_step": sub.tokens,
                           "tokens_per_s": res["value"], "ms_per_step": res["ms_per_step"],
                           "one_gpu_ms_per_step": res["ms_per_step"], "speedup_vs_1": 1.0,
                           "parity": None,
                           "parity_vs": "one GPU holds the whole vocabulary: no shards"}
            del sub, res
            torch.cuda.empty_cache()
        if ctx.world > 1 and (chosen is None or "flce" in chosen):
            fl = Flce()
            vp = measure_workload(ctx, fl, args.steps, args.warmup, args.e2e_steps, 0.0,
                                  keep=True)
            flce_vp = measure_flce_vp(ctx, args.steps, args.warmup, vp)
            del fl, vp
            torch.cuda.empty_cache()
            if args.vp_dx_exchange is None:
                # the same measurement with the collective-free exchange (peer
                # memory from the dX GEMM's epilogue) beside the NCCL one
                flce_vp["p2p"] = measure_flce_vp_p2p(ctx, args)

    if ctx.rank == 0:
        line = {
            "metric": getattr(wl, "metric", METRIC),
            "value": r["value"],
            "unit": "tokens/s",
            "n_gpus": ctx.world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": r["ms_per_step"],
            "higher_is_better": True,
            "scaling": getattr(wl, "scaling", "weak"),
            "vs_baseline": None,
            "dtype": wl.dtype,
            "data": "synthetic (seeded normal inputs of the BASELINE shapes)",
            "config": {**wl.config(),
                       "timed_region": "sum of K per-step CUDA-event spans on the launching "
                                       "stream (no events between a step's launches), max "
                                       "over ranks; L2 flush and a "
                                       f"{args.spin_us:g} us GPU spin before each step, "
                                       "outside the spans; per_kernel from K more steps with "
                                       "events around every launch, frac_alone from each "
                                       "launch alone after a clean L2 flush"},
            "roofline": r["roofline"],
            "per_kernel": {k: {kk: vv for kk, vv in v.items() if kk in ("ms", "frac",
                                                                         "frac_alone")}
                           for k, v in r["per_kernel"].items()},
            "cpu_baseline": r["cpu_baseline"],
            "e2e": {**r["e2e"],
                    "api": getattr(wl, "e2e_api", "public autograd Functions, pinned host "
                                   "buffers, H2D of inputs + D2H of all outputs every step"
                                   + (", copies overlapped with compute on 3 streams "
                                      "(H2D / compute / D2H; consecutive steps overlap, the "
                                      "host at most 2 steps ahead)"
                                      if getattr(wl, "e2e_pipelined", False) else ""))},
            "gpu_launches": r["gpu_launches"],
            "peak_extra_bytes": r["peak_extra_bytes"],
            "clocks": r["clocks"],
        }
        if r["extra"]:
            line.update(r["extra"])
        if workloads:
            line["workloads"] = workloads
        if flce_vp is not None:
            line["flce_vp"] = flce_vp
        print(json.dumps(_rounded(line)), flush=True)
    ctx.close()
    return 0


def main(argv=None):
    _register_optional_workloads()
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=None,
                    help="run this workload alone as the line (default: swiglu_rope as the "
                         "line plus every other op under 'workloads' and 'flce_vp')")
    ap.add_argument("--headline-only", action="store_true",
                    help="default workload without the other ops")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--kernel-table", action="store_true",
                    help="print one extra step's per-kernel device times (CUPTI) to stderr")
    ap.add_argument("--spin-us", type=float, default=200.0,
                    help="untimed GPU spin before each timed step (host run-ahead); 0 = off")
    ap.add_argument("--cpu-budget", type=float, default=15.0,
                    help="seconds of CPU-oracle work for the line's cpu_baseline")
    ap.add_argument("--cpu-budget-sub", type=float, default=6.0,
                    help="seconds of CPU-oracle work for each entry of 'workloads'")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline measurements")
    ap.add_argument("--burst", action="store_true",
                    help="use the burst (not sustained) bf16 peak for tensor-bound rooflines")
    ap.add_argument("--lora-swiglu-fusion", type=int, choices=[0, 1], default=None,
                    help="LoRA MLP: SwiGLU inside the GEMMs (1, the library default) or as "
                         "separate elementwise passes (0)")
    ap.add_argument("--lora-tokens", type=int, default=None,
                    help="token rows of the lora workload (default: BASELINE's 16,384); a "
                         "smaller case for profiler captures")
    ap.add_argument("--suite", default=None,
                    help="comma-separated subset of the default run's extra workloads "
                         "(rmsnorm,flce,lora,c5_step; flce is flce_vp at N > 1)")
    ap.add_argument("--vp-dx-exchange", choices=["nccl", "p2p"], default=None,
                    help="vocabulary-parallel FLCE (N > 1): sum the partial dX with NCCL "
                         "(default) or through peer memory from the dX GEMM's epilogue")
    ap.add_argument("--e2e-split", type=int, default=None,
                    help="e2e pipeline chunks per batch row of the swiglu_rope workload "
                         "(default 1)")
    ap.add_argument("--flce-tokens", type=int, default=None,
                    help="token rows of the flce workload (default: BASELINE's 16,384); a "
                         "smaller case for profiler captures")
    ap.add_argument("--flce-chunk", type=int, default=None,
                    help="FLCE token-chunk length (default: BASELINE's 8192; smaller chunks "
                         "bound the exponentials buffer, chunk x vocab bf16)")
    args = ap.parse_args(argv)
    if args.flce_chunk:
        Flce.CHUNK = int(args.flce_chunk)
    if args.lora_tokens:
        Lora.T = int(args.lora_tokens)
    if args.flce_tokens:
        Flce.N = int(args.flce_tokens)
    if args.vp_dx_exchange:
        import metal_liger_b200.ops.fused_linear_cross_entropy as flce_ops

        flce_ops.VP_DX_EXCHANGE = args.vp_dx_exchange
    if args.e2e_split:
        if SwigluRope.HK % args.e2e_split or args.e2e_split < 1:
            ap.error(f"--e2e-split must divide the {SwigluRope.HK} k heads")
        SwigluRope.E2E_SPLIT = int(args.e2e_split)
    if args.lora_swiglu_fusion is not None and args.impl != "reference":
        from metal_liger_b200 import _C

        _C.call("ml_lora_set_mlp_swiglu_fusion", int(args.lora_swiglu_fusion), None)
    if args.warmup < 3:
        args.warmup = 3  # timing rule: at least 3 warm-up steps
    wl = WORKLOADS[args.workload or "swiglu_rope"]()
    if args.impl == "reference":
        return run_reference_arm(args, wl)
    return run_gpu_arm(args, wl)


if __name__ == "__main__":
    sys.exit(main())
