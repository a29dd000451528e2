#!/usr/bin/env python
"""Grad-grad attention step benchmark (forward + first-order backward with
create_graph + double backward) on B200.

Default workload (the metric's T=16k multi-GPU case):
b=8 h=32 T=16384 d=128 bf16 causal, inputs, dO and probes iid N(0,1)*0.5,
the b*h = 256 heads split into contiguous equal shards over the N ranks (no
collective on the data path; NCCL only for the barrier and the max-over-ranks
timing). One step, per rank:

    o = triton_attention(q, k, v, causal=True)                       # forward
    dq, dk, dv = autograd.grad(o, (q, k, v), dO, create_graph=True)  # backward
    gq, gk, gv = autograd.grad((dq, dk, dv), (q, k, v), (u_q, u_k, u_v))  # double backward

Reported (one JSON line from rank 0):
  value     whole-job algorithmic TFLOP/s (28*T^2*d per head, x (T+1)/(2T) causal)
            with inputs resident in HBM, device-timed with CUDA events, max over ranks;
  e2e       the same step through the same public API with pinned host inputs
            copied in and the second-order results copied out inside the timed region;
  roofline  the dominant kernel's algorithmic TFLOP/s against the measured bf16 peak;
  cpu_baseline  the reference's math path (oracle port, fp32, host cores) on a bounded sample.

Workloads whose inputs are smaller than twice the L2 size (config 3, config 2)
are timed with an L2 flush between steps, outside the per-step events.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c4|c3|c3s|c3nc|c2|...]
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path
from typing import Optional

import torch

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "grad-grad attention step ms & TFLOP/s (fwd+bwd+2nd-bwd), T=16k, 1/2/4/8 B200"
CONFIGS = {
    "c4": dict(b=8, h=32, t=16384, d=128, dtype="bf16", causal=True, scale_in=0.5,
               workload="BASELINE config 4: grad-grad b=8 h=32 T=16384 d=128 bf16 causal, b*h sharded over GPUs"),
    "c3": dict(b=1, h=1, t=16384, d=64, dtype="fp16", causal=True, scale_in=1.0,
               workload="BASELINE config 3 (largest T): grad-grad b=1 h=1 T=16384 d=64 fp16 causal"),
    "c3nc": dict(b=1, h=1, t=16384, d=64, dtype="fp16", causal=False, scale_in=1.0,
                 workload="BASELINE config 3 (largest T): grad-grad b=1 h=1 T=16384 d=64 fp16 non-causal"),
    # config 3 in the loss form of the reference's own sweep (tests/bench_gradgrad_sweep.py:56-61):
    # loss = mean(O), grads with create_graph, s = sum of mean(g^2), grad-grads of s
    "c3s": dict(b=1, h=1, t=16384, d=64, dtype="fp16", causal=True, scale_in=1.0, step="sweep",
                workload="BASELINE config 3 (largest T), the reference sweep's loss form: loss = mean(O), "
                         "s = sum mean(g^2), b=1 h=1 T=16384 d=64 fp16 causal"),
    "c3snc": dict(b=1, h=1, t=16384, d=64, dtype="fp16", causal=False, scale_in=1.0, step="sweep",
                  workload="BASELINE config 3 (largest T), the reference sweep's loss form: loss = mean(O), "
                           "s = sum mean(g^2), b=1 h=1 T=16384 d=64 fp16 non-causal"),
    "c4x8": dict(b=1, h=8, t=16384, d=128, dtype="bf16", causal=True, scale_in=0.5,
                 workload="8-head slice of BASELINE config 4 (profiling size): T=16384 d=128 bf16 causal"),
    "c2": dict(b=2, h=4, t=2048, d=128, dtype="fp16", causal=False, scale_in=0.5,
               workload="BASELINE config 2 shape: grad-grad b=2 h=4 T=2048 d=128 fp16 non-causal"),
    # P-streaming first-order backward (the reference's save_p_triton_full data flow):
    # forward writing P, then dv / rowsum / dq+dk from P; HBM-bound on P.
    "c2p": dict(b=2, h=4, t=2048, d=128, dtype="fp16", causal=False, scale_in=0.5, step="from_p", flush=True,
                workload="BASELINE config 2: fwd (P written) + first-order backward from P "
                         "(dv/rowsum/dq+dk from P) b=2 h=4 T=2048 d=128 fp16 non-causal"),
    "c2pc": dict(b=2, h=4, t=2048, d=128, dtype="fp16", causal=True, scale_in=0.5, step="from_p", flush=True,
                 workload="BASELINE config 2: fwd (P written) + first-order backward from P "
                          "(dv/rowsum/dq+dk from P) b=2 h=4 T=2048 d=128 fp16 causal"),
    # forward only (the reference's tests/bench.py: triton_attention forward at config 2's shape)
    "c2f": dict(b=2, h=4, t=2048, d=128, dtype="fp16", causal=False, scale_in=0.5, step="fwd", flush=True,
                workload="forward only, BASELINE config 2 shape: b=2 h=4 T=2048 d=128 fp16 non-causal"),
    "c2fc": dict(b=2, h=4, t=2048, d=128, dtype="fp16", causal=True, scale_in=0.5, step="fwd", flush=True,
                 workload="forward only, BASELINE config 2 shape: b=2 h=4 T=2048 d=128 fp16 causal"),
    "c4f": dict(b=8, h=32, t=16384, d=128, dtype="bf16", causal=True, scale_in=0.5, step="fwd",
                workload="forward only, BASELINE config 4 shape: b=8 h=32 T=16384 d=128 bf16 causal"),
    # the TTT-E2E meta step (one inner SGD step with create_graph, outer loss backward)
    "c5": dict(b=1, h=12, t=8192, d=64, dtype="bf16", causal=True, scale_in=1.0, step="meta",
               model=dict(n_layers=12, d_model=768, n_heads=12, d_ff=3072, vocab_size=32000, max_seq_len=8192,
                          window_size=None),
               workload="BASELINE config 5: TTT-E2E meta step, 12 layers d_model=768 12 heads d_ff=3072 vocab 32000, "
                        "bf16, b=1 T=8192, inner_steps=1 inner_lr=0.01 on the first 6144 tokens, outer loss on the "
                        "last 2048, all parameters updated, attention on the kernels"),
    # the forward-only streaming path of the reference's latency demo (scripts/demo_infer.py:11-27,
    # :70-100): its model, seq 8192 in chunks of 512 new tokens, each call over the last 512 tokens
    "c5s": dict(b=1, h=8, t=8192, d=64, dtype="bf16", causal=True, scale_in=1.0, step="stream",
                window=512, chunk=512,
                model=dict(n_layers=8, d_model=512, n_heads=8, d_ff=2048, vocab_size=4096, max_seq_len=10240,
                           window_size=512, dropout=0.0),
                workload="streaming inference of the reference's latency demo: 8 layers d_model=512 8 heads "
                         "d_ff=2048 vocab 4096 window 512, bf16 (the demo's fp32 model cast: the kernels take "
                         "16-bit), 8192 tokens in chunks of 512, each forward over the last 512 tokens"),
    # BASELINE config 3 as the reference's own sweep runs it (tests/bench_gradgrad_sweep.py:76):
    # T in {512 ... 16384} x causal / non-causal, mode save_p_triton_full; one JSON line with a row per case
    "c3sweep": dict(b=1, h=1, t=16384, d=64, dtype="fp16", causal=True, scale_in=1.0, step="c3sweep",
                    ts=(512, 1024, 2048, 4096, 8192, 16384),
                    workload="BASELINE config 3: grad-grad sweep b=1 h=1 d=64 fp16, T in {512..16384}, causal and "
                             "non-causal, mode save_p_triton_full"),
    # BASELINE config 2 as defined: forward + first-order backward in the modes save_p and
    # save_p_triton_full, causal and non-causal, 50 iterations (tests/bench_gradgrad.py:54, tests/bench.py:30-38)
    "c2modes": dict(b=2, h=4, t=2048, d=128, dtype="fp16", causal=False, scale_in=0.5, step="c2modes",
                    modes=("save_p", "save_p_triton_full"), iters=50,
                    workload="BASELINE config 2: fwd+bwd b=2 h=4 T=2048 d=128 fp16, modes save_p and "
                             "save_p_triton_full, causal and non-causal, 50 iterations"),
    "c8p": dict(b=1, h=8, t=8192, d=128, dtype="fp16", causal=False, scale_in=0.5, step="from_p",
                workload="fwd (P written) + first-order backward from P, b=1 h=8 T=8192 d=128 fp16 "
                         "non-causal (P = 1 GiB, larger than L2)"),
}
# Algorithmic flops per head, in units of T^2 d, that each kernel kind contributes
# (each of the 14 distinct products of the grad-grad step is assigned to the
# kernel that first computes it; recomputed products count nowhere).
ALGO_UNITS = {"fwd": 4, "delta": 0, "bwd_kv": 6, "bwd_q": 2, "bwd2_stats": 6, "bwd2_q": 4, "bwd2_kv": 6,
              "from_p": 0}
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def causal_factor(t: int, causal: bool) -> float:
    return (t + 1) / (2 * t) if causal else 1.0


def step_flops(cfg: dict, heads: int) -> float:
    """Algorithmic flops of one step: 28 T^2 d per head for the grad-grad step,
    12 T^2 d for forward + first-order backward (the from-P and config-2 steps)."""
    units = {"from_p": 12.0, "fwd": 4.0, "fwdbwd": 12.0}.get(cfg.get("step"), 28.0)
    return units * cfg["t"] ** 2 * cfg["d"] * heads * causal_factor(cfg["t"], cfg["causal"])


def from_p_bytes(cfg: dict, heads: int) -> float:
    """Algorithmic HBM bytes of the four from-P launches of one step: P read by each
    of them (the causal ones only its lower triangle), each [t, d] 16-bit operand
    read or written once per launch, and the fp32 rowsum rows."""
    t, d = cfg["t"], cfg["d"]
    cf = causal_factor(t, cfg["causal"])
    p_reads = 2.0 * t * t * (1.0 + 3.0 * cf)
    td = 2.0 * t * d * (3 + 3 + 5 + 5)   # dv: dO, dV; rowsum: V, dO; dk: V, dO, Q, dK; dq: dO, V, K, dQ
    rows = 4.0 * t * 3
    return heads * (p_reads + td + rows)


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(config_name: str) -> dict:
    """Per-kernel DRAM bytes per launch from a committed ncu capture, if any."""
    p = ROOT / "profiles" / "dram_traffic.json"
    if not p.exists():
        return {}
    try:
        return json.loads(p.read_text()).get(config_name, {})
    except Exception:
        return {}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            gid = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", gid, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        # nvidia-smi's start-up (NVML initialization) can stall CUDA API calls of this
        # process for milliseconds: let it settle before a timed region begins
        time.sleep(0.5)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- the step
def make_inputs(cfg: dict, heads: range, device: torch.device, seed: int = 1234) -> dict:
    """Inputs of the given global heads; a head's values do not depend on the sharding."""
    from testtimeideas_b200.sharding import head_inputs
    dtype = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
    return head_inputs(heads, cfg["t"], cfg["d"], dtype, device, seed=seed, scale_in=cfg["scale_in"])


def math_path_step(kind: str):
    """The reference's math formulation on the GPU (torch matmul / masked_fill /
    softmax, triton_attention.py:18-25) in the same dtype, differentiated by
    autograd as the reference's recompute path does (:416-420): the baseline the
    north-star speed-up is quoted against. Materializes [t, t] tensors."""
    from testtimeideas_b200.attention import attention_math

    def step(x: dict, causal: bool):
        scale = 1.0 / math.sqrt(x["q"].shape[-1])
        if kind == "fwd":
            with torch.no_grad():
                return (attention_math(x["q"], x["k"], x["v"], causal, scale),)
        q, k, v = (x[n].detach().requires_grad_(True) for n in ("q", "k", "v"))
        o = attention_math(q, k, v, causal, scale)
        if kind == "fwdbwd":
            return torch.autograd.grad(o, (q, k, v), x["do"])
        if kind == "sweep":
            grads = torch.autograd.grad(o.float().mean(), (q, k, v), create_graph=True)
            return torch.autograd.grad(sum(g.float().pow(2).mean() for g in grads), (q, k, v))
        dq, dk, dv = torch.autograd.grad(o, (q, k, v), x["do"], create_graph=True)
        return torch.autograd.grad((dq, dk, dv), (q, k, v), (x["uq"], x["uk"], x["uv"]))
    return step


def time_math_path(cfg: dict, x: dict, kind: str, steps: int, device,
                   flush: Optional[torch.Tensor] = None) -> Optional[dict]:
    """CUDA-event time of the math path on the same inputs, when its [t, t]
    intermediates fit comfortably (about 12 of them per head in flight); with
    `flush`, L2 is flushed between steps outside the per-step events, as for ours."""
    heads = x["q"].shape[0] * x["q"].shape[1]
    if kind not in ("gradgrad", "fwd", "sweep", "fwdbwd") or heads * cfg["t"] ** 2 * 2 * 12 > 48 * 2 ** 30:
        return None
    step = math_path_step(kind)
    try:
        for _ in range(2):
            step(x, cfg["causal"])
        torch.cuda.synchronize(device)
        evs = []
        for _ in range(steps):
            if flush is not None:
                flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            step(x, cfg["causal"])
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize(device)
    except torch.cuda.OutOfMemoryError:
        return {"unavailable": "out of memory"}
    finally:
        torch.cuda.empty_cache()
    return {"ms_per_step": sum(a.elapsed_time(b) for a, b in evs) / steps,
            "what": "the reference's math formulation (torch matmul/softmax, autograd) on this GPU, same inputs"}


def fwd_step(x: dict, causal: bool):
    """Forward only, through the public API without a graph (inference)."""
    from ttt_kernels import triton_attention
    with torch.no_grad():
        return (triton_attention(x["q"], x["k"], x["v"], causal=causal),)


def from_p_step(x: dict, causal: bool):
    """Forward writing P, then the first-order backward from P through the
    reference-compatible backward_stubs helpers (the data flow of the reference's
    save_p_triton_full backward, triton_attention.py:354-362)."""
    from testtimeideas_b200 import _lib
    from ttt_kernels import backward_stubs as bs
    q, k, v, do = x["q"], x["k"], x["v"], x["do"]
    scale = 1.0 / math.sqrt(q.shape[-1])
    _, _, p = _lib.attn_fwd(q, k, v, causal, scale, save_p=True)
    dv = bs.triton_attn_bwd_dv_from_p(p, do)
    rs = bs.triton_attn_rowsum_from_p(p, do, v, causal=causal)
    dq, dk = bs.triton_attn_bwd_dqdk_from_p(q, k, v, do, p, rs, causal=causal, scale=scale)
    return dq, dk, dv


def sweep_step(x: dict, causal: bool):
    """One step in the loss form of the reference's sweep (tests/bench_gradgrad_sweep.py:56-61):
    loss = mean(O); grads with create_graph; s = sum over q, k, v of mean(g^2); grad-grads of s.
    The upstream gradient of O is a constant and the probes are 2 g / numel."""
    from ttt_kernels import triton_attention
    q, k, v = (x[n].detach().requires_grad_(True) for n in ("q", "k", "v"))
    o = triton_attention(q, k, v, causal=causal)
    grads = torch.autograd.grad(o.float().mean(), (q, k, v), create_graph=True)
    return torch.autograd.grad(sum(g.float().pow(2).mean() for g in grads), (q, k, v))


def gradgrad_step(x: dict, causal: bool, mode: str = "recompute"):
    """One step through the public, reference-compatible API."""
    from ttt_kernels import triton_attention
    q, k, v = (x[n].detach().requires_grad_(True) for n in ("q", "k", "v"))
    o = triton_attention(q, k, v, causal=causal, bwd_mode=mode)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), x["do"], create_graph=True)
    return torch.autograd.grad((dq, dk, dv), (q, k, v), (x["uq"], x["uk"], x["uv"]))


def fwd_bwd_step(mode: str):
    """Forward + first-order backward (no graph kept) through the public API in
    bwd_mode `mode`: the step BASELINE config 2 times per mode."""
    def step(x: dict, causal: bool):
        from ttt_kernels import triton_attention
        q, k, v = (x[n].detach().requires_grad_(True) for n in ("q", "k", "v"))
        o = triton_attention(q, k, v, causal=causal, bwd_mode=mode)
        return torch.autograd.grad(o, (q, k, v), x["do"])
    return step


# ---------------------------------------------------------------- timing helpers
def timed_ms(step, x: dict, causal: bool, steps: int, flush: Optional[torch.Tensor] = None) -> float:
    """Total CUDA-event milliseconds of `steps` steps on the current stream. With
    `flush`, a 512 MiB write before each step flushes L2, outside that step's events."""
    if flush is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            step(x, causal)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)
    evs = []
    for _ in range(steps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step(x, causal)
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs)


def profiled_kernels(step, x: dict, causal: bool, steps: int, flush: Optional[torch.Tensor] = None) -> dict:
    """{kernel kind: (launches, total ms)} over `steps` steps with the library's profiling
    hook on (each launch bracketed by CUDA events on its stream)."""
    from testtimeideas_b200 import _lib
    torch.cuda.synchronize()
    _lib.profile_collect()
    _lib.profile_enable(True)
    for _ in range(steps):
        if flush is not None:
            flush.fill_(1)
        step(x, causal)
    torch.cuda.synchronize()
    _lib.profile_enable(False)
    return {k: v for k, v in _lib.profile_collect().items() if v[0] > 0}


def soak(step, x: dict, causal: bool, seconds: float, flush: Optional[torch.Tensor] = None) -> dict:
    """Untimed steps, one at a time, until `seconds` have passed: the GPU reaches the
    clocks of sustained load (the power cap) before the timed region starts, so timed
    regions of any length (a 4 s region at one GPU, a 0.6 s one at eight) see the
    same clock state."""
    t0 = time.perf_counter()
    n = 0
    held = None  # the previous step's outputs, alive while the next step runs (as in the timed loop)
    while time.perf_counter() - t0 < seconds:
        if flush is not None:
            flush.fill_(1)
        held = step(x, causal)
        torch.cuda.synchronize()
        n += 1
    del held
    return {"steps": n, "seconds": round(time.perf_counter() - t0, 2)}


def fused_bwd_summary(kernel_ms: dict, cfg: dict, heads: int, peak: float) -> dict:
    """The first-order backward (delta + dK/dV + dQ passes) per step: its algorithmic
    8 T^2 d per head over its kernels' time, against the sustained tensor peak."""
    ms = sum(kernel_ms.get(k, 0.0) for k in ("delta", "bwd_kv", "bwd_q"))
    flops = 8.0 * cfg["t"] ** 2 * cfg["d"] * heads * causal_factor(cfg["t"], cfg["causal"])
    tflops = flops / (ms * 1e-3) / 1e12 if ms > 0 else None
    return {"ms_per_step": ms, "algorithmic_tflops": tflops, "frac_of_sustained_peak": tflops / peak if tflops else None,
            "kernels": ["delta", "bwd_kv", "bwd_q"], "target_frac": 0.5}


# ---------------------------------------------------------------- CPU baseline (oracle port)
def cpu_baseline(cfg: dict, t_sample: int, reps: int = 1, warm: bool = True) -> dict:
    """The reference's math path (_attention_math + autograd twice, fp32) on this
    host's cores for one head at T=t_sample; returns TFLOP/s of that sample."""
    from oracle import attention_oracle as orc
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sample = dict(cfg, t=t_sample)
    inp = orc.seeded_inputs(1, 1, t_sample, cfg["d"], seed=99, scale_in=cfg["scale_in"])
    names = ("q", "k", "v", "do", "uq", "uk", "uv")
    if warm:
        orc.math_gradgrad(*(inp[n] for n in names), causal=cfg["causal"], dtype=torch.float32)
    t0 = time.perf_counter()
    for _ in range(reps):
        orc.math_gradgrad(*(inp[n] for n in names), causal=cfg["causal"], dtype=torch.float32)
    dt = (time.perf_counter() - t0) / reps
    return {"value": step_flops(sample, 1) / dt / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port", "ms_per_sample": dt * 1e3,
            "sample": f"one head of the workload at T={t_sample} (d={cfg['d']}, causal={cfg['causal']}), fp32 "
                      f"math path (_attention_math + autograd twice), {reps} timed rep(s) after 1 warm-up, "
                      f"os.cpu_count()={os.cpu_count()}"}


def run_reference(args, cfg: dict) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_baseline(cfg, args.cpu_t, reps=1, warm=False)
    runs = [cpu_baseline(cfg, args.cpu_t, reps=1, warm=False) for _ in range(args.steps)]
    base = runs[len(runs) // 2]
    value = statistics.median(r["value"] for r in runs)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.median(r["ms_per_sample"] for r in runs),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": {"workload": cfg["workload"], "sample_t": args.cpu_t},
            "cpu_baseline": dict(base, value=value, sample=base["sample"] + f"; median of {args.steps} samples"),
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm
def verify_sharded(cfg: dict, results, total_heads: int, device: torch.device) -> Optional[dict]:
    """Gather every rank's grad-grads to rank 0 and compare them with rank 0 running
    all heads alone (same kernels, same per-head inputs): the sharded job must give
    bit-identical results. Returns the summary on rank 0, None elsewhere."""
    from testtimeideas_b200.sharding import gather_heads
    full = [gather_heads(r, total_heads) for r in results]
    if full[0] is None:
        return None
    ref = step_fn(cfg)(make_inputs(cfg, range(total_heads), device), cfg["causal"])
    diffs = [float((a.float() - b.float()).abs().max()) for a, b in zip(full, ref)]
    return {"heads": total_heads, "max_abs_diff": max(diffs),
            "bit_identical": all(torch.equal(a, b) for a, b in zip(full, ref)),
            "against": "rank 0 running every head alone"}


def step_fn(cfg: dict):
    return {"from_p": from_p_step, "fwd": fwd_step, "sweep": sweep_step}.get(cfg.get("step"), gradgrad_step)


STEP_INPUTS = {"gradgrad": ("q", "k", "v", "do", "uq", "uk", "uv"), "from_p": ("q", "k", "v", "do"),
               "fwd": ("q", "k", "v"), "sweep": ("q", "k", "v")}
# L2 of one B200; workloads whose inputs are smaller than twice this are timed with
# an L2 flush between steps
L2_BYTES = 126 << 20


def run_meta(args, cfg: dict) -> None:
    """Config 5: one TTT-E2E meta step per timed step (meta_step + outer backward) on one GPU.
    value = tokens per second; the attention kernels' share comes from the profiling hook."""
    from testtimeideas_b200 import _lib, ttt_model
    if int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("the meta-step workload runs on one GPU")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    mcfg = ttt_model.ModelConfig(**cfg["model"])
    torch.manual_seed(0)
    model = ttt_model.TTTModel(mcfg).to(device, torch.bfloat16)
    t, ctx = cfg["t"], 3 * cfg["t"] // 4
    g = torch.Generator(device=device).manual_seed(1)
    ids = torch.randint(0, mcfg.vocab_size, (1, t), generator=g, device=device)
    tgt = torch.randint(0, mcfg.vocab_size, (1, t), generator=g, device=device)
    inner_mask = torch.zeros(1, t, device=device)
    inner_mask[:, :ctx] = 1.0
    outer_mask = 1.0 - inner_mask

    def step(a, b_, im, om):
        model.zero_grad(set_to_none=True)
        inner, outer = ttt_model.meta_step(model, a, b_, im, om, inner_lr=0.01, inner_steps=1)
        outer.backward()
        return outer.detach()

    for _ in range(args.warmup):
        step(ids, tgt, inner_mask, outer_mask)
    _lib.check_device_errors(device)
    clocks = ClockSampler(0)
    torch.cuda.synchronize(device)
    _lib.profile_collect()
    _lib.profile_enable(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step(ids, tgt, inner_mask, outer_mask)
    e1.record()
    torch.cuda.synchronize(device)
    _lib.profile_enable(False)
    prof = _lib.profile_collect()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    # end to end: token ids and masks from pinned host memory, the outer loss back
    host = [x.cpu().pin_memory() for x in (ids, tgt, inner_mask, outer_mask)]
    dev = [torch.empty_like(x) for x in (ids, tgt, inner_mask, outer_mask)]
    loss_host = torch.empty((), dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize(device)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        for d_, h_ in zip(dev, host):
            d_.copy_(h_, non_blocking=True)
        loss_host.copy_(step(*dev), non_blocking=True)
    f1.record()
    torch.cuda.synchronize(device)
    e2e_ms = f0.elapsed_time(f1) / args.steps
    kern = {k: v for k, v in prof.items() if v[0] > 0}
    attn_ms = sum(v[1] for v in kern.values()) / args.steps
    line = {"metric": "TTT-E2E meta step tokens/s (config 5)", "value": t / (ms * 1e-3), "unit": "tokens/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform token ids)",
            "config": {"workload": cfg["workload"], "t": t, "l2": "activations far larger than L2"},
            "e2e": {"value": t / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": sum(x.numel() * x.element_size() for x in host),
                    "d2h_bytes_per_step": loss_host.element_size()},
            "attention_ms_per_step": attn_ms, "attention_share": attn_ms / ms,
            "kernel_ms_per_step": {k: v[1] / args.steps for k, v in kern.items()},
            "gpu_launches": sum(v[0] for v in kern.values()), "clocks": clk, "roofline": None, "cpu_baseline": None}
    print(json.dumps(line), flush=True)


def run_stream(args, cfg: dict) -> None:
    """Streaming inference (no graph): one timed step = the whole sequence streamed in
    chunks (ttt_model.stream_logits); value = tokens per second."""
    from testtimeideas_b200 import _lib, ttt_model
    if int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("the streaming workload runs on one GPU")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    mcfg = ttt_model.ModelConfig(**cfg["model"])
    torch.manual_seed(0)
    model = ttt_model.TTTModel(mcfg).to(device, torch.bfloat16).eval()
    t, window, chunk = cfg["t"], cfg["window"], cfg["chunk"]
    g = torch.Generator(device=device).manual_seed(1)
    tokens = torch.randint(0, mcfg.vocab_size, (1, t), generator=g, device=device)

    def step(tok):
        return ttt_model.stream_logits(model, tok, window, chunk)[-1]

    clocks = ClockSampler(0)
    for _ in range(args.warmup):
        step(tokens)
    _lib.check_device_errors(device)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step(tokens)
    e1.record()
    torch.cuda.synchronize(device)
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    _lib.profile_collect()
    _lib.profile_enable(True)
    for _ in range(args.steps):
        step(tokens)
    torch.cuda.synchronize(device)
    _lib.profile_enable(False)
    prof = _lib.profile_collect()
    # end to end: token ids from pinned host memory, the last chunk's logits back to the host
    host = tokens.cpu().pin_memory()
    dev = torch.empty_like(tokens)
    last = step(tokens)
    out_host = torch.empty(last.shape, dtype=last.dtype).pin_memory()
    torch.cuda.synchronize(device)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        dev.copy_(host, non_blocking=True)
        out_host.copy_(step(dev), non_blocking=True)
    f1.record()
    torch.cuda.synchronize(device)
    e2e_ms = f0.elapsed_time(f1) / args.steps
    kern = {k: v for k, v in prof.items() if v[0] > 0}
    attn_ms = sum(v[1] for v in kern.values()) / args.steps
    line = {"metric": "TTT-E2E streaming inference tokens/s (forward-only path)", "value": t / (ms * 1e-3),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform token ids)",
            "config": {"workload": cfg["workload"], "t": t, "window": window, "chunk": chunk,
                       "l2": "weights and activations of 16 forward calls per step (not flushed)"},
            "e2e": {"value": t / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": host.numel() * host.element_size(),
                    "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
            "attention_ms_per_step": attn_ms, "attention_share": attn_ms / ms,
            "kernel_ms_per_step": {k: v[1] / args.steps for k, v in kern.items()},
            "gpu_launches": sum(v[0] for v in kern.values()), "clocks": clk, "roofline": None, "cpu_baseline": None}
    print(json.dumps(line), flush=True)


def north_star(device: torch.device, peaks: dict, peak_src: str, steps: int = 20) -> dict:
    """BASELINE config 3 at its largest T, the north_star's target configuration: b=h=1
    T=16384 d=64 fp16 causal on one GPU, in the reference sweep's mode
    (save_p_triton_full). Ours (CUDA events, L2 flushed between steps); the reference's
    math formulation (torch matmul/softmax, autograd twice) on the same GPU and inputs
    with the speed-up over it (target >= 2x); and the first-order backward's
    algorithmic fraction of the sustained tensor peak (target >= 0.5)."""
    cfg = CONFIGS["c3"]
    x = make_inputs(cfg, range(1), device)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=device)
    step = lambda x_, c_: gradgrad_step(x_, c_, "save_p_triton_full")  # noqa: E731
    for _ in range(5):
        flush.fill_(1)
        step(x, True)
    ms = timed_ms(step, x, True, steps, flush) / steps
    prof = profiled_kernels(step, x, True, steps, flush)
    kernel_ms = {k: v[1] / steps for k, v in prof.items()}
    sustained = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    math_path = time_math_path(cfg, x, "gradgrad", 10, device, flush)
    out = {"workload": "BASELINE config 3 at T=16384: grad-grad b=1 h=1 d=64 fp16 causal, mode save_p_triton_full, "
                       "one GPU, L2 flushed between steps",
           "ms_per_step": ms, "algorithmic_tflops": step_flops(cfg, 1) / (ms * 1e-3) / 1e12, "steps": steps,
           "kernel_ms_per_step": kernel_ms,
           "fused_bwd": dict(fused_bwd_summary(kernel_ms, cfg, 1, sustained),
                             peak=sustained, peak_source=f"{peak_src} bf16_tflops_sustained"),
           "math_path_gpu": math_path, "target_speedup_vs_math_path": 2.0}
    if math_path and "ms_per_step" in math_path:
        out["speedup_vs_math_path"] = math_path["ms_per_step"] / ms
    return out


def run_sweep(args, cfg: dict) -> None:
    """Config 3 over the reference sweep's sequence lengths (tests/bench_gradgrad_sweep.py:76),
    causal and non-causal, mode save_p_triton_full, one GPU: per case ours and the math path on
    the same GPU, each in the probe form (28 T^2 d) and in the sweep's loss form (mean(O),
    sum mean(g^2)); L2 flushed between steps. Prints one JSON line with a row per case."""
    if int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("the sweep runs on one GPU")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peaks, peak_src = load_peaks()
    sustained = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=device)
    steps = max(args.steps, 10)
    rows = []
    clocks = ClockSampler(0)
    probe = lambda x_, c_: gradgrad_step(x_, c_, "save_p_triton_full")  # noqa: E731
    for causal in (False, True):
        for t in cfg["ts"]:
            c = dict(cfg, t=t, causal=causal, step=None)
            x = make_inputs(c, range(1), device)
            row = {"t": t, "causal": causal}
            for form, fn in (("probe", probe), ("loss", sweep_step)):
                for _ in range(args.warmup):
                    flush.fill_(1)
                    fn(x, causal)
                ms = timed_ms(fn, x, causal, steps, flush) / steps
                row[f"{form}_ms"] = ms
                mp = time_math_path(c, x, "gradgrad" if form == "probe" else "sweep", min(steps, 10), device, flush)
                if mp and "ms_per_step" in mp:
                    row[f"{form}_math_path_ms"] = mp["ms_per_step"]
                    row[f"{form}_speedup_vs_math_path"] = mp["ms_per_step"] / ms
            row["algorithmic_tflops"] = step_flops(c, 1) / (row["probe_ms"] * 1e-3) / 1e12
            row["frac_of_sustained_peak"] = row["algorithmic_tflops"] / sustained
            rows.append(row)
    clk = clocks.stop()
    big = [r for r in rows if r["t"] == max(cfg["ts"]) and r["causal"]][0]
    line = {"metric": METRIC, "value": big["algorithmic_tflops"], "unit": "TFLOP/s", "n_gpus": 1,
            "steps": steps, "warmup": args.warmup, "ms_per_step": big["probe_ms"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic",
            "config": {"workload": cfg["workload"], "value_row": "T=16384 causal, probe form",
                       "l2": "L2 flushed (512 MiB write) between timed steps"},
            "peak": sustained, "peak_source": f"{peak_src} bf16_tflops_sustained", "rows": rows, "clocks": clk}
    print(json.dumps(line), flush=True)


def run_c2modes(args, cfg: dict) -> None:
    """Config 2 as BASELINE defines it: forward + first-order backward through the public API
    in the modes save_p and save_p_triton_full, causal and non-causal, 50 timed iterations
    each (tests/bench_gradgrad.py:54 modes; the shape of tests/bench.py:30-38), with the math
    path on the same GPU; L2 flushed between steps. One JSON line with a row per case."""
    if int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("config 2 runs on one GPU")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=device)
    iters = cfg["iters"]
    heads = cfg["b"] * cfg["h"]
    rows = []
    clocks = ClockSampler(0)
    for causal in (False, True):
        c = dict(cfg, causal=causal, step="fwdbwd")
        x = {n: v.reshape(cfg["b"], cfg["h"], cfg["t"], cfg["d"])
             for n, v in make_inputs(c, range(heads), device).items() if n in ("q", "k", "v", "do")}
        mp = time_math_path(c, x, "fwdbwd", iters, device, flush)
        for mode in cfg["modes"]:
            step = fwd_bwd_step(mode)
            for _ in range(max(args.warmup, 10)):
                flush.fill_(1)
                step(x, causal)
            ms = timed_ms(step, x, causal, iters, flush) / iters
            prof = profiled_kernels(step, x, causal, iters, flush)
            row = {"mode": mode, "causal": causal, "ms": ms,
                   "algorithmic_tflops": step_flops(c, heads) / (ms * 1e-3) / 1e12,
                   "kernel_ms_per_step": {k: v[1] / iters for k, v in prof.items()}}
            if mp and "ms_per_step" in mp:
                row["math_path_ms"] = mp["ms_per_step"]
                row["speedup_vs_math_path"] = mp["ms_per_step"] / ms
            rows.append(row)
    clk = clocks.stop()
    first = rows[0]
    line = {"metric": "fwd+bwd attention step ms & TFLOP/s (BASELINE config 2)", "value": first["algorithmic_tflops"],
            "unit": "TFLOP/s", "n_gpus": 1, "steps": iters, "warmup": max(args.warmup, 10),
            "ms_per_step": first["ms"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": cfg["dtype"], "data": "synthetic",
            "config": {"workload": cfg["workload"], "value_row": "save_p non-causal",
                       "l2": "L2 flushed (512 MiB write) between timed steps"},
            "rows": rows, "clocks": clk}
    print(json.dumps(line), flush=True)


def run_ours(args, cfg: dict) -> None:
    from testtimeideas_b200 import _lib
    from testtimeideas_b200.sharding import head_range, max_over_ranks as _max_over_ranks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    total_heads = cfg["b"] * cfg["h"]
    if total_heads % world:
        raise SystemExit(f"{total_heads} heads do not split over {world} GPUs")
    mine = head_range(total_heads, world, rank)
    heads = len(mine)
    _lib.load_library()

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        return _max_over_ranks(x, device=device)

    step = step_fn(cfg)
    kind = cfg.get("step", "gradgrad")
    x = {n: t for n, t in make_inputs(cfg, mine, device).items() if n in STEP_INPUTS[kind]}
    # Workloads whose inputs are not well above L2 get an L2 flush (a 512 MiB write)
    # between timed steps, outside the per-step events; the others are larger than L2.
    # The flush buffer exists before the warm-up steps, so that they leave the
    # allocator's pool as the timed steps need it (no device allocation inside them).
    in_bytes = sum(t.numel() * t.element_size() for t in x.values())
    need_flush = cfg.get("flush") or in_bytes < 2 * L2_BYTES
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=device) if need_flush else None
    # The clock sampler starts (and settles) before the warm-up steps, which then
    # bring the GPU back to speed after that pause.
    clocks = ClockSampler(local)
    # Warm-up and soak steps hold the previous step's outputs until the next step
    # returns, as the timed loop does (it keeps them for --verify): the allocator's
    # pool then already holds the blocks the timed steps need, and no device
    # allocation lands inside the timed region.
    last = None
    for _ in range(args.warmup):
        if flush is not None:
            flush.fill_(1)
        last = step(x, cfg["causal"])
    _lib.check_device_errors(device)
    # then untimed steps until the clocks settle under sustained load, so that every N's
    # timed region (4 s at one GPU, under a second at eight) starts in the same state
    soaked = soak(step, x, cfg["causal"], args.soak_s, flush) if args.soak_s > 0 else {"steps": 0, "seconds": 0.0}

    # ---- device-timed region: inputs resident in HBM. Timed without the profiling
    # hook (with it on, the library keeps every launch on one stream so that each
    # launch's events time that kernel alone); the per-kernel breakdown below comes
    # from a second, profiled pass of the same steps.
    barrier()
    torch.cuda.synchronize(device)
    if flush is None:
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            last = step(x, cfg["causal"])
        stop.record()
        torch.cuda.synchronize(device)
        dev_ms = start.elapsed_time(stop)
    else:
        evs = []
        for _ in range(args.steps):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            last = step(x, cfg["causal"])
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize(device)
        dev_ms = sum(a.elapsed_time(b) for a, b in evs)
    barrier()
    clk = clocks.stop()
    _lib.profile_collect()
    _lib.profile_enable(True)
    for _ in range(args.steps):
        if flush is not None:
            flush.fill_(1)
        step(x, cfg["causal"])
    torch.cuda.synchronize(device)
    _lib.profile_enable(False)
    prof = _lib.profile_collect()
    _lib.check_device_errors(device)
    ms = max_over_ranks(dev_ms)
    ms_per_step = ms / args.steps
    value = step_flops(cfg, total_heads) / (ms_per_step * 1e-3) / 1e12

    # ---- end to end: pinned host inputs -> device -> step -> results back to pinned host
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    host_in = {n: torch.empty_like(t, device="cpu").pin_memory() for n, t in x.items()}
    for n, t in x.items():
        host_in[n].copy_(t)
    host_out = [torch.empty_like(x["q"], device="cpu").pin_memory() for _ in range(1 if kind == "fwd" else 3)]
    dev_in = {n: torch.empty_like(t) for n, t in x.items()}
    h2d = sum(t.numel() * t.element_size() for t in host_in.values())
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    # With 16 or more heads per GPU the step runs over chunks of heads (the heads are
    # independent), so that one chunk's host-to-device copy, another's compute and a
    # third's device-to-host copy overlap on three streams; every step still copies
    # all of its inputs in and all of its results out.
    nchunk = min(8, heads) if heads >= 8 else 1
    bounds = [round(i * heads / nchunk) for i in range(nchunk + 1)]
    comp = torch.cuda.current_stream(device)
    copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    done = [None] * nchunk  # compute of each chunk's previous step (its input buffers are reused)
    for _ in range(e2e_steps):
        for c in range(nchunk):
            sl = slice(bounds[c], bounds[c + 1])
            with torch.cuda.stream(copy_in):
                if done[c] is not None:
                    copy_in.wait_event(done[c])
                for n in dev_in:
                    dev_in[n][:, sl].copy_(host_in[n][:, sl], non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(copy_in)
            comp.wait_event(landed)
            gg = step({n: t[:, sl] for n, t in dev_in.items()}, cfg["causal"])
            done[c] = torch.cuda.Event()
            done[c].record(comp)
            copy_out.wait_event(done[c])
            with torch.cuda.stream(copy_out):
                for dst, src in zip(host_out, gg):
                    dst[:, sl].copy_(src, non_blocking=True)
                    src.record_stream(copy_out)
    comp.wait_stream(copy_out)
    e1.record()
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
    e2e_value = step_flops(cfg, total_heads) / (e2e_ms * 1e-3) / 1e12
    # The ceiling the copies alone set: the same pinned copies, in and out on their two
    # streams, with no compute, on every rank at once (the ranks share the host).
    out_dev = [torch.empty_like(x["q"]) for _ in host_out]
    barrier()
    torch.cuda.synchronize(device)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record()
    for _ in range(e2e_steps):
        with torch.cuda.stream(copy_in):
            copy_in.wait_event(c0)
            for n in dev_in:
                dev_in[n].copy_(host_in[n], non_blocking=True)
        with torch.cuda.stream(copy_out):
            copy_out.wait_event(c0)
            for dst, src in zip(host_out, out_dev):
                dst.copy_(src, non_blocking=True)
    comp.wait_stream(copy_in)
    comp.wait_stream(copy_out)
    c1.record()
    torch.cuda.synchronize(device)
    barrier()
    copy_ms = max_over_ranks(c0.elapsed_time(c1)) / e2e_steps
    del out_dev

    # ---- roofline of the dominant kernel (per-launch CUDA-event time inside the timed region)
    peaks, peak_src = load_peaks()
    kern = {k: v for k, v in prof.items() if v[0] > 0}
    dom = max(kern, key=lambda k: kern[k][1])
    launches, dom_ms = kern[dom]
    per_launch_ms = dom_ms / launches
    traffic = load_traffic(args.config).get(dom)
    if dom == "from_p":
        # HBM-bound: algorithmic bytes of the from-P launches over their time
        dom_bytes = from_p_bytes(cfg, heads) / launches * args.steps
        achieved = dom_bytes / (per_launch_ms * 1e-3) / 1e9
        peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        roofline = {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "traffic": traffic,
                    "peak_source": f"{peak_src} hbm_gbs (copy bandwidth)",
                    "algorithmic_bytes_per_launch": dom_bytes, "ms_per_launch": per_launch_ms}
    else:
        dom_flops = ALGO_UNITS[dom] * cfg["t"] ** 2 * cfg["d"] * heads * causal_factor(cfg["t"], cfg["causal"])
        achieved = dom_flops / (per_launch_ms * 1e-3) / 1e12
        peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        roofline = {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "traffic": traffic,
                    "peak_source": f"{peak_src} bf16_tflops_sustained (kernel timed inside a long step)",
                    "algorithmic_flops_per_launch": dom_flops, "ms_per_launch": per_launch_ms}

    gpu_launches = sum(v[0] for v in prof.values())
    kernel_ms = {k: v[1] / args.steps for k, v in kern.items()}

    verify = None
    if args.verify:
        barrier()
        verify = verify_sharded(cfg, last, total_heads, device)
        barrier()
    del last

    math_path = None
    if world == 1 and not args.no_math_path:
        math_path = time_math_path(cfg, x, kind, args.steps, device, flush)
        if math_path and "ms_per_step" in math_path:
            math_path["ours_speedup"] = math_path["ms_per_step"] / ms_per_step

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, args.cpu_t, reps=1)

    ns = None
    if world == 1 and args.config == "c4" and not args.no_north_star:
        ns = north_star(device, peaks, peak_src)

    if rank == 0:
        dtype = cfg["dtype"]
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": dtype, "data": "synthetic",
            "config": {"workload": cfg["workload"], "b": cfg["b"], "h": cfg["h"], "t": cfg["t"], "d": cfg["d"],
                       "causal": cfg["causal"], "global_heads": total_heads, "heads_per_gpu": heads,
                       "parallelism": f"bh-shard x{world}",
                       "l2": ("L2 flushed (512 MiB write) between timed steps (inputs %.1f MiB per GPU)" % (
                                  in_bytes / 2 ** 20) if flush is not None else
                              "inputs larger than L2 (%d tensors of %.2f GiB per GPU%s)" % (
                                  len(x), x["q"].numel() * x["q"].element_size() / 2 ** 30,
                                  ", plus P" if kind == "from_p" else ""))},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "ms_per_step": e2e_ms, "steps": e2e_steps,
                    "head_chunks": nchunk,
                    "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                    "copy_only_ms_per_step": copy_ms,
                    "copy_only_gbs_per_gpu": (h2d + d2h) / (copy_ms * 1e-3) / 1e9,
                    "ceiling_ms_per_step": max(ms_per_step, copy_ms)},
            "soak": soaked,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clk,
            "gpu_launches": gpu_launches,
            "kernel_ms_per_step": kernel_ms,
        }
        if kind == "gradgrad":
            sustained = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
            line["fused_bwd"] = dict(fused_bwd_summary(kernel_ms, cfg, heads, sustained), per="rank 0, per GPU")
        if ns is not None:
            line["north_star"] = ns
        if verify is not None:
            line["verify"] = verify
        if math_path is not None:
            line["math_path_gpu"] = math_path
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c4")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-t", type=int, default=4096, help="T of the one-head CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-math-path", action="store_true",
                    help="skip timing the reference's math formulation on the GPU beside the kernels")
    ap.add_argument("--no-north-star", action="store_true",
                    help="skip the config-3 north-star measurement appended to the default (config 4) line")
    ap.add_argument("--soak-s", type=float, default=4.0,
                    help="seconds of untimed steps after the warm-up, so that the timed region starts with the "
                         "clocks of sustained load")
    ap.add_argument("--verify", action="store_true",
                    help="gather the last step's grad-grads to rank 0 and check them against rank 0 running "
                         "every head alone (untimed)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        run_reference(args, cfg)
    elif cfg.get("step") == "meta":
        run_meta(args, cfg)
    elif cfg.get("step") == "stream":
        run_stream(args, cfg)
    elif cfg.get("step") == "c3sweep":
        run_sweep(args, cfg)
    elif cfg.get("step") == "c2modes":
        run_c2modes(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
