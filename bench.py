"""Headline benchmark: the 96-request continuous-batching serving trace on B200.

Workload (synthetic, seeded; no dataset): Qwen2-0.5B architecture (24 layers, hidden
896, 14/2 heads, intermediate 4864, vocab 151936) with seeded random bf16 weights; 96
requests arriving at t=0, prompts uniform in [32, 256] tokens, output lengths lognormal
(median 75, sigma 0.8) clipped to [1, 256] and generated in full (no EOS); packed KV
cache with max_len 512; 32 slots. One bench step = one complete run of the trace through
`Engine.step`; the timed unit is the WINDOW of engine steps 50..109 of that run (60
scheduler iterations, decode-dominated, with the admissions that fall inside it), the
same window the reference arm times, so both arms report the same quantity.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl qweninfer_b200|reference]

Printed JSON (rank 0, one line):
  value   output tokens produced in the window / device time of the window's forwards
          (CUDA events on the launching stream; max over ranks, tokens summed).
  e2e     the same tokens / time of the window's Engine.step calls through the public
          API (CUDA events around them): host bookkeeping, per-step H2D of (ids,
          positions, rows) from pinned memory and D2H of the argmax words included.
  roofline  the kernel with the largest share of a decode step of the window (each launch
          of that step timed alone with CUDA events, `kernels` lists them all): algorithmic
          bytes per launch (weights streamed, KV read or appended, embedding rows) / launch
          time vs the measured HBM copy peak; step_roofline: the same for the whole step.
  serve3072  the scaled serving trace (3072 requests, rid % N over N replicas, 128 slots
          and max_len 4096 per GPU): whole-job tok/s = all output tokens / slowest rank.
  full_trace, batch1, prefill, serve64_padded  the other benchmark configurations on the
          same model (N = 1 only): the whole 96-request trace, batch-1 decode at contexts
          16/256/1024, prefill time to first token, 64 slots with autotuned padding.
  cpu_baseline  the numpy oracle (the reference's algorithm restated) on the host cores
          over a bounded sample of the same window.

Under torchrun (N > 1) every rank runs its own replica of the trace on its own GPU
(weak scaling, no collective on the data path).
"""

from __future__ import annotations

import argparse
import copy
from collections import deque
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

MAX_LEN = 512
WINDOW = (50, 110)                  # engine steps timed in both arms
WEIGHT_BYTES = 988_065_536          # bf16 layer weights + norms + biases + tied head
KV_BYTES_PER_TOKEN = 12_288         # 2 (K,V) * 24 layers * 2 heads * 64 * 2 B
EMBED_ROW_BYTES = 1_792
METRIC = "decode tok/s on 96-req continuous-batch workload"
LAYER_PARAMS = 357_897_216          # weights of the 24 blocks
HEAD_PARAMS = 136_134_656           # tied head (vocab x hidden)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="qweninfer_b200", choices=["qweninfer_b200", "reference"])
    ap.add_argument("--slots", type=int, default=32)
    ap.add_argument("--no-extras", action="store_true", help="skip the other configurations (N = 1 extras)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-window-steps", type=int, default=10,
                    help="engine steps of the window the in-process cpu_baseline times")
    ap.add_argument("--only", choices=["decode", "batch1", "prefill", "serve64", "serve3072"], default=None,
                    help="one measurement alone (profiling cases): graph-replayed decode steps at --batch, "
                         "config-1 batch-1 decode, config-2 prefill, config-3 64 padded slots")
    ap.add_argument("--batch", type=int, default=22, help="decode batch of --only decode")
    ap.add_argument("--context", type=int, default=200, help="decode positions of --only decode")
    ap.add_argument("--max-len", type=int, default=512, help="cache slots per row of --only decode")
    ap.add_argument("--lengths", default="64,256,512,1024", help="prompt lengths of --only prefill")
    return ap.parse_args()


def peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d.get("bf16_tflops"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def step_bytes(pos: list[int]) -> int:
    """Algorithmic HBM bytes of one decode step over rows at positions `pos`."""
    B = len(pos)
    return WEIGHT_BYTES + sum(p + 1 for p in pos) * KV_BYTES_PER_TOKEN + B * KV_BYTES_PER_TOKEN + B * EMBED_ROW_BYTES


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples (200 ms) of this rank's GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.rows: list[list[str]] = []
        self.proc = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------- our arm

def load_model(device: torch.device):
    from qweninfer_b200 import synthetic
    from qweninfer_b200.models.qwen2 import Qwen2
    ckpt = synthetic.checkpoint_dir(synthetic.full_config(), seed=0, dtype=torch.bfloat16)
    return Qwen2.from_pretrained(ckpt, dtype=torch.bfloat16, device=device)


class TimedRunner:
    """Wraps an engine's runner: CUDA-event device time of every forward (prefill and
    decode separately), per-decode-step algorithmic bytes; `active` gates the tally."""

    def __init__(self, runner) -> None:
        self.r = runner
        self.active = False
        self.reset()
        self.ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        self._prefill, self._prefill_many, self._decode = runner.prefill, runner.prefill_many, runner.decode
        runner.prefill, runner.prefill_many, runner.decode = self.prefill, self.prefill_many, self.decode

    def reset(self) -> None:
        self.prefill_ms = self.decode_ms = 0.0
        self.decode_bytes = 0
        self.decode_rows: list[int] = []
        self.decode_inputs: list[tuple] = []
        self.prefill_tokens = 0

    def _timed(self, fn, *a):
        self.ev[0].record()
        out = fn(*a)
        self.ev[1].record()
        self.ev[1].synchronize()
        return out, self.ev[0].elapsed_time(self.ev[1])

    def prefill(self, row, prompt):
        tok, ms = self._timed(self._prefill, row, prompt)
        if self.active:
            self.prefill_ms += ms
            self.prefill_tokens += len(prompt)
        return tok

    def prefill_many(self, rows, prompts):
        toks, ms = self._timed(self._prefill_many, rows, prompts)
        if self.active:
            self.prefill_ms += ms
            self.prefill_tokens += sum(len(p) for p in prompts)
        return toks

    def decode(self, toks, pos, row_start=0):
        out, ms = self._timed(self._decode, toks, pos, row_start)
        if self.active:
            self.decode_ms += ms
            self.decode_bytes += step_bytes(list(pos))
            self.decode_rows.append(len(toks))
            self.decode_inputs.append((list(toks), list(pos), row_start))
        return out


def run_trace(eng, timed: TimedRunner, workload, window=WINDOW) -> dict:
    """One full run of the trace through Engine.step; device and end-to-end time of the
    window of engine steps [window[0], window[1]) and of the whole trace."""
    from qweninfer_b200.engine.engine import Request
    reqs = [Request(r.rid, r.prompt, r.max_new_tokens) for r in workload]
    for r in reqs:
        eng.submit(r)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    timed.reset()  # this run's forwards only
    launches0 = eng.runner.launches
    h2d0, d2h0 = eng.runner.h2d_bytes, eng.runner.d2h_bytes
    out: dict = {}
    step = 0
    torch.cuda.synchronize()
    ev[0].record()
    full_dev = 0.0
    while eng.waiting or eng.active:
        if step == window[0]:
            full_dev += timed.prefill_ms + timed.decode_ms
            timed.reset()
            toks0 = sum(len(r.output) for r in reqs)
            l0, hb0, db0 = eng.runner.launches, eng.runner.h2d_bytes, eng.runner.d2h_bytes
            ev[2].record()
        eng.step()
        step += 1
        if step == window[1]:
            ev[3].record()
            ev[3].synchronize()
            out["window"] = {"tokens": sum(len(r.output) for r in reqs) - toks0,
                             "dev_ms": timed.prefill_ms + timed.decode_ms, "e2e_ms": ev[2].elapsed_time(ev[3]),
                             "decode_ms": timed.decode_ms, "decode_bytes": timed.decode_bytes,
                             "decode_steps": len(timed.decode_rows), "prefill_ms": timed.prefill_ms,
                             "prefill_tokens": timed.prefill_tokens,
                             "mean_batch": float(np.mean(timed.decode_rows)) if timed.decode_rows else 0.0,
                             "launches": eng.runner.launches - l0, "h2d": eng.runner.h2d_bytes - hb0,
                             "d2h": eng.runner.d2h_bytes - db0,
                             "mid_decode": timed.decode_inputs[len(timed.decode_inputs) // 2]
                             if timed.decode_inputs else None}
            full_dev += timed.prefill_ms + timed.decode_ms
            timed.reset()
    ev[1].record()
    ev[1].synchronize()
    full_dev += timed.prefill_ms + timed.decode_ms
    done = sorted(reqs, key=lambda r: r.rid)
    toks = sum(len(r.output) for r in done)
    out["full"] = {"tokens": toks, "dev_ms": full_dev, "e2e_ms": ev[0].elapsed_time(ev[1]), "steps": step,
                   "ttft_mean_s": statistics.mean(r.first_token - r.arrival for r in done),
                   "latency_mean_s": statistics.mean(r.finished - r.arrival for r in done),
                   "launches": eng.runner.launches - launches0,
                   "h2d": eng.runner.h2d_bytes - h2d0, "d2h": eng.runner.d2h_bytes - d2h0}
    return out


def main_line(args, world, eng, runs, W, F, dev_ms, e2e_ms, tokens, clock_info, pk) -> dict:
    """Rank 0's JSON line of the serving window."""
    K = args.steps
    launch_s = W["decode_ms"] / 1e3 / max(1, W["decode_steps"])
    algo = W["decode_bytes"] / max(1, W["decode_steps"])
    gbs = algo / launch_s / 1e9
    res = {
        "metric": METRIC,
        "value": tokens / (dev_ms / 1e3),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": dev_ms / K,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random weights of the Qwen2-0.5B architecture; seeded synthetic requests)",
        "config": {"workload": f"serve96 window: engine steps {WINDOW[0]}-{WINDOW[1] - 1} of the 96-request trace "
                               f"(prompts U[32,256], outputs lognormal(75,0.8)<=256, seed 4), {args.slots} slots, "
                               f"max_len {MAX_LEN}, one replica per GPU",
                   "model": "Qwen2-0.5B architecture, random bf16 weights", "slots": args.slots,
                   "max_len": MAX_LEN, "window": list(WINDOW), "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2: every decode step streams 988 MB of weights"},
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": W["h2d"] // K,
                "d2h_bytes_per_step": W["d2h"] // K, "ms_per_step": e2e_ms / K},
        "gpu_launches": W["launches"],
        "window": {"output_tokens_per_step": W["tokens"] // K, "decode_steps_per_step": W["decode_steps"] // K,
                   "mean_decode_batch": W["mean_batch"] / K, "decode_ms_per_decode_step": launch_s * 1e3,
                   "prefill_ms_per_step": W["prefill_ms"] / K, "prefill_tokens_per_step": W["prefill_tokens"] // K},
        "step_roofline": {"what": "the whole decode step (embedding, 24 layers, head + argmax; one CUDA graph "
                                  "of the launches below), over the window's decode steps", "bound": "hbm",
                          "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gbs / pk["hbm_gbs"],
                          "algorithmic_bytes_per_step": algo, "us_per_step": launch_s * 1e6,
                          "bytes": "988,065,536 weights + sum(len+1)*12,288 KV read + B*12,288 KV write + "
                                   "B*1,792 embed, per decode step"},
        "full_trace": {"value": F["tokens"] / (F["dev_ms"] / 1e3), "e2e": F["tokens"] / (F["e2e_ms"] / 1e3),
                       "unit": "tok/s", "output_tokens": F["tokens"] // K, "engine_steps": runs[0]["full"]["steps"],
                       "ttft_mean_s": statistics.mean(r["full"]["ttft_mean_s"] for r in runs),
                       "latency_mean_s": statistics.mean(r["full"]["latency_mean_s"] for r in runs),
                       "gpu_launches_per_trace": F["launches"] // K},
        "clocks": clock_info,
    }
    mid = runs[-1]["window"]["mid_decode"]
    if mid is not None:
        kt = kernel_table(eng.runner, mid, pk)
        name, top = max(kt["by_kernel"].items(), key=lambda e: e[1]["share"])
        n = top["launches_per_step"]
        res["roofline"] = {"kernel": name, "bound": "hbm", "achieved": top["achieved_gbs"],
                           "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": top["frac"], "peak_source": pk["source"],
                           "traffic": None, "algorithmic_bytes_per_launch": top["bytes_per_step"] / n,
                           "us_per_launch": top["us_per_step"] / n, "launches_per_step": n, "share": top["share"],
                           "measured_at": f"decode batch {kt['batch']}, mean position {kt['mean_position']:.0f} "
                                          "(the window's middle decode step), each launch timed alone; the "
                                          "kernel with the largest share of the step, all its launches"}
        res["kernels"] = kt
    return res


def our_arm(args, rank: int, world: int, device: torch.device) -> dict | None:
    from qweninfer_b200 import synthetic
    from qweninfer_b200.engine.engine import Engine

    model = load_model(device)
    workload = synthetic.serving96()
    eng = Engine(model, max_slots=args.slots, max_len=MAX_LEN)
    timed = TimedRunner(eng.runner)
    timed.active = True
    for _ in range(args.warmup):
        run_trace(eng, timed, workload)
    eng.runner.check()

    clocks = ClockSampler(device.index or 0)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.start()
    runs = [run_trace(eng, timed, workload) for _ in range(args.steps)]
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    eng.runner.check()
    W = {k: sum(r["window"][k] for r in runs) for k in runs[0]["window"] if k != "mid_decode"}
    F = {k: sum(r["full"][k] for r in runs) for k in ("tokens", "dev_ms", "e2e_ms", "launches", "h2d", "d2h")}
    dev_ms, e2e_ms, tokens = W["dev_ms"], W["e2e_ms"], float(W["tokens"])
    if world > 1:
        t = torch.tensor([dev_ms, e2e_ms, tokens], device=device, dtype=torch.float64)
        mx, sm = t.clone(), t.clone()
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(sm, op=torch.distributed.ReduceOp.SUM)
        dev_ms, e2e_ms, tokens = float(mx[0]), float(mx[1]), float(sm[2])
        torch.distributed.barrier()
    pk = peaks()
    res = main_line(args, world, eng, runs, W, F, dev_ms, e2e_ms, tokens, clock_info, pk) if rank == 0 else None
    if not args.no_extras:
        s4 = serve3072(model, rank, world, device, pk)
        if res is not None:
            res["serve3072"] = s4
    if world == 1 and not args.no_extras:
        res["batch1"] = batch1_latency(model, pk)
        res["prefill"] = prefill_ttft(model, pk)
        res["serve64_padded"] = serve64(model)
    return res


# Algorithmic HBM bytes of one launch of each kind at decode batch B (positions pos): the
# weights it must stream, the KV bytes it must read or append, the embedding rows. The
# activations between launches stay in L2 and are not counted.
KERNEL_NAMES = {"embed": "embed_kernel", "qkv": "tc_proj_kernel<qkv_rope>", "attention": "attention_kernel",
                "o_proj": "tc_proj_kernel<residual>", "gate_up": "tc_proj_kernel<swiglu>",
                "down": "tc_proj_kernel<residual>", "head": "tc_proj_kernel<logits>"}


def kernel_bytes(pos: list[int]) -> dict:
    B = len(pos)
    kv_row = 2 * 2 * 64 * 2  # K and V, 2 KV heads x 64 dims, bf16: per cached token and layer
    return {"embed": B * EMBED_ROW_BYTES, "qkv": 1152 * 896 * 2 + 1152 * 4 + B * kv_row,
            "attention": sum(p + 1 for p in pos) * kv_row, "o_proj": 896 * 896 * 2,
            "gate_up": 9728 * 896 * 2, "down": 896 * 4864 * 2, "head": 151936 * 896 * 2}


def kernel_table(runner, decode_input, pk: dict, reps: int = 5) -> dict:
    """Every launch of one decode step timed alone with CUDA events (`launch_times`), at a
    decode step of the timed window (its batch and positions): per kind launches per step,
    microseconds per launch, algorithmic bytes, achieved GB/s and fraction of the measured
    copy peak, and share of the step's summed launch time."""
    toks, pos, row_start = decode_input
    runner.launch_times(toks, pos, row_start)
    acc: dict[str, list[float]] = {}
    for _ in range(reps):
        for k, us in runner.launch_times(toks, pos, row_start):
            acc.setdefault(k, []).append(us)
    runner.check()
    algo = kernel_bytes(pos)
    total = sum(sum(v) for v in acc.values())
    table = {}
    for k, v in acc.items():
        mean = sum(v) / len(v)
        gbs = algo[k] / (mean * 1e-6) / 1e9
        table[k] = {"kernel": KERNEL_NAMES[k], "launches_per_step": len(v) // reps, "us_per_launch": mean,
                    "algorithmic_bytes_per_launch": algo[k], "achieved_gbs": gbs, "frac": gbs / pk["hbm_gbs"],
                    "share": sum(v) / total}
    # per kernel (template): o_proj and down are both tc_proj_kernel<residual>
    per: dict[str, dict] = {}
    for k, e in table.items():
        a = per.setdefault(e["kernel"], {"launches_per_step": 0, "us_per_step": 0.0, "bytes_per_step": 0})
        a["launches_per_step"] += e["launches_per_step"]
        a["us_per_step"] += e["us_per_launch"] * e["launches_per_step"]
        a["bytes_per_step"] += e["algorithmic_bytes_per_launch"] * e["launches_per_step"]
    for a in per.values():
        a["achieved_gbs"] = a["bytes_per_step"] / (a["us_per_step"] * 1e-6) / 1e9
        a["frac"] = a["achieved_gbs"] / pk["hbm_gbs"]
        a["share"] = a["us_per_step"] / (total / reps)
    return {"batch": len(toks), "mean_position": float(np.mean(pos)), "sum_us_per_step": total / reps,
            "kernels": table, "by_kernel": per}


def decode_steps(model, B: int, steps: int, warmup: int, context: int = 200, max_len: int = 512) -> dict:
    """Graph-replayed decode steps of B rows at positions ~context (row b at context + 7 b
    mod 1024, so a batch spans contexts context .. context + 1023) in a cache of max_len
    slots per row: the profiling case."""
    from qweninfer_b200.engine.kv_cache import KVCache
    from qweninfer_b200.engine.runner import DecodeRunner
    cache = KVCache(model.cfg, B, max_len, dtype=torch.bfloat16, device=model.device)
    r = DecodeRunner(model, cache, max_batch=B)
    toks = [1] * B
    base = [context + (7 * b) % 1024 for b in range(B)] if context > 200 else [context] * B
    if max(base) + warmup + steps >= max_len:
        raise ValueError("contexts past the cache")
    for i in range(warmup):
        r.decode(toks, [p + i for p in base])
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        r.decode(toks, [p + warmup + i for p in base])
    b.record()
    b.synchronize()
    r.check()
    ms = a.elapsed_time(b) / steps
    byts = step_bytes([p + warmup + steps // 2 for p in base])
    return {"batch": B, "steps": steps, "context": context, "max_len": max_len, "ms_per_step": ms,
            "hbm_gbs": byts / (ms / 1e3) / 1e9}


def batch1_latency(model, pk: dict) -> dict:
    """Config 1: batch-1 decode at contexts 16/256/1024 (seed-2 prompts, prefill then 128
    greedy tokens), ms/token (CUDA events over the decode steps) and HBM fraction."""
    from qweninfer_b200 import synthetic
    from qweninfer_b200.engine.kv_cache import KVCache
    from qweninfer_b200.engine.runner import DecodeRunner
    out = {}
    for C_, prompt in synthetic.decode_latency_prompts().items():
        cache = KVCache(model.cfg, 1, C_ + 130, dtype=torch.bfloat16, device=model.device)
        r = DecodeRunner(model, cache, max_batch=1)
        tok = r.prefill(0, prompt)
        for i in range(3):
            tok = int(r.decode([tok], [C_ + i])[0])
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 125
        a.record()
        for i in range(n):
            tok = int(r.decode([tok], [C_ + 3 + i])[0])
        b.record()
        b.synchronize()
        r.check()
        ms = a.elapsed_time(b) / n
        byts = step_bytes([C_ + 3 + n // 2])
        gbs = byts / (ms / 1e3) / 1e9
        out[str(C_)] = {"ms_per_token": ms, "hbm_gbs": gbs, "frac": gbs / pk["hbm_gbs"]}
        del r, cache
    return out


def prefill_ttft(model, pk: dict, lengths=(64, 256, 512, 1024)) -> dict:
    """Config 2: batch-1 causal prefill of seed-3 prompts of 64/256/512/1024 tokens writing
    the cache and emitting the first greedy token; TTFT (CUDA events, median of 5 after a
    warm-up) and the achieved dense rate: 2 * (block params * P + head params) plus the
    causal attention products 2 * 2 * layers * heads * head_dim * P(P+1)/2."""
    from qweninfer_b200 import synthetic
    from qweninfer_b200.engine.kv_cache import KVCache
    from qweninfer_b200.engine.runner import DecodeRunner
    out = {}
    for P, prompt in synthetic.prefill_prompts().items():
        if P not in lengths:
            continue
        cache = KVCache(model.cfg, 1, P, dtype=torch.bfloat16, device=model.device)
        r = DecodeRunner(model, cache, max_batch=1)
        r.prefill(0, prompt)
        ts = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            r.prefill(0, prompt)
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        r.check()
        ms = statistics.median(ts)
        flops = 2 * (LAYER_PARAMS * P + HEAD_PARAMS) + 4 * 24 * 14 * 64 * P * (P + 1) / 2
        tflops = flops / (ms / 1e3) / 1e12
        out[str(P)] = {"ttft_ms": ms, "tflops": tflops, "frac_of_bf16_peak": tflops / pk["bf16_tflops"]
                       if pk.get("bf16_tflops") else None}
        del r, cache
    return out


def serve64(model) -> dict:
    """Config 3, second arm: 64 slots with autotuned padding (autotune_padding on this
    GPU, then the full 96-request trace)."""
    from qweninfer_b200 import synthetic
    from qweninfer_b200.engine.engine import Engine, autotune_padding
    pad_to, ms = autotune_padding(model, 64)
    eng = Engine(model, max_slots=64, max_len=MAX_LEN, pad_to=pad_to)
    timed = TimedRunner(eng.runner)
    timed.active = True
    run_trace(eng, timed, synthetic.serving96())
    r = run_trace(eng, timed, synthetic.serving96())["full"]
    eng.runner.check()
    return {"value": r["tokens"] / (r["dev_ms"] / 1e3), "e2e": r["tokens"] / (r["e2e_ms"] / 1e3), "unit": "tok/s",
            "ttft_mean_s": r["ttft_mean_s"], "latency_mean_s": r["latency_mean_s"],
            "pad_sizes": sorted(set(pad_to[1:])), "autotune_ms": {str(k): v for k, v in ms.items()}}


def serve3072(model, rank: int, world: int, device: torch.device, pk: dict) -> dict | None:
    """Config 4: the scaled serving trace (3072 requests at t=0, prompts U[128,2048],
    outputs lognormal(200,0.9) <= 1024, seed 5) over `world` replicas, one per GPU, each
    with 128 slots and max_len 4096, dispatched rid % world through ReplicaGroup (results
    published to the process group's store). Whole-box tok/s = all output tokens / the
    slowest rank's time (CUDA events around its serve, host scheduling included; the
    device-only figure sums each rank's forward times). Per-GPU HBM fraction: algorithmic
    bytes of the decode steps / their device time, over all ranks. Total work is fixed, so
    this is strong scaling."""
    from qweninfer_b200 import synthetic
    from qweninfer_b200.engine.engine import Engine, Request
    from qweninfer_b200.engine.replicas import ReplicaGroup
    slots, max_len = 128, 4096
    reqs = [Request(r.rid, r.prompt, r.max_new_tokens)
            for r in synthetic.serving_requests(3072, 128, 2048, 200.0, 0.9, 1024, seed=5)]
    eng = Engine(model, max_slots=slots, max_len=max_len)
    # warm-up outside the timed region: every decode batch size's graph, the prefill workspace
    for B in range(1, slots + 1):
        eng.runner.decode([0] * B, [0] * B)
    eng.runner.prefill_many([0, 1], [[0] * 2048, [0] * 2048])
    timed = TimedRunner(eng.runner)
    timed.active = True
    if world > 1:
        store = torch.distributed.distributed_c10d._get_default_store()
    else:
        store = torch.distributed.HashStore()
    group = ReplicaGroup(lambda: eng, rank, world, store, prefix="serve3072", timeout_s=300.0)
    mine = [r for r in reqs if r.rid % world == rank]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev[0].record()
    group.serve(reqs, collect=False)
    ev[1].record()
    ev[1].synchronize()
    eng.runner.check()
    wall_ms = ev[0].elapsed_time(ev[1])
    done = group.results(mine)
    t = torch.tensor([wall_ms, timed.prefill_ms + timed.decode_ms, sum(len(r.output) for r in done),
                      timed.decode_bytes, timed.decode_ms, timed.prefill_ms, timed.prefill_tokens,
                      len(timed.decode_rows), sum(timed.decode_rows),
                      statistics.mean(r.first_token - r.arrival for r in done) if done else 0.0],
                     dtype=torch.float64, device=device)
    if world > 1:
        mx, sm = t.clone(), t.clone()
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(sm, op=torch.distributed.ReduceOp.SUM)
        torch.distributed.barrier()
    else:
        mx = sm = t
    if rank != 0:
        return None
    tokens = float(sm[2])
    gbs = float(sm[3]) / (float(sm[4]) / 1e3) / 1e9  # bytes and device time summed over the ranks
    return {"workload": "serve3072: 3072 requests (prompts U[128,2048], outputs lognormal(200,0.9)<=1024, seed 5), "
                        f"rid % {world} over {world} replica(s), {slots} slots and max_len {max_len} per GPU",
            "value": tokens / (float(mx[0]) / 1e3), "unit": "tok/s", "scaling": "strong",
            "device_value": tokens / (float(mx[1]) / 1e3), "output_tokens": int(tokens),
            "max_rank_ms": float(mx[0]), "max_rank_device_ms": float(mx[1]),
            "decode_hbm_gbs_per_gpu": gbs, "decode_frac_per_gpu": gbs / pk["hbm_gbs"],
            "decode_ms_total": float(sm[4]), "prefill_ms_total": float(sm[5]),
            "prefill_tokens": int(sm[6]), "decode_steps": int(sm[7]),
            "mean_decode_batch": float(sm[8]) / max(1.0, float(sm[7])),
            "ttft_mean_s": float(sm[9]) / world}


# ------------------------------------------------------------- CPU arms

def cpu_threads() -> int:
    """Use every host thread for numpy (torchrun sets OMP_NUM_THREADS=1 per rank)."""
    from threadpoolctl import threadpool_limits
    n = os.cpu_count() or 1
    threadpool_limits(limits=n)
    return n


def oracle_window(slice_steps: int, samples: int, warmup: int, slices: int = 1) -> dict:
    """The numpy oracle (the reference's fp32 algorithm) on the host cores over the timed
    window of the serving trace (32 slots), in slices of `slice_steps` engine steps: slice
    j starts at engine step WINDOW[0] + j * slice_steps, a state reached by the scheduler's
    bookkeeping alone (no arithmetic; the cache stays zero, which changes no operation
    count). Sample i runs slice i % slices with full arithmetic from its start state; with
    slices * slice_steps = the window's length, samples cycle through the whole window.
    Returns output tokens per second over all samples (after `warmup` untimed steps)."""
    from oracle import OracleModel, OracleRequest, bf16_round
    from oracle.engine_ref import OracleEngine, StubModel
    from qweninfer_b200 import synthetic
    threads = cpu_threads()
    cfg = synthetic.full_config()
    state = {k: bf16_round(v.numpy()) for k, v in synthetic.synthetic_state(cfg, 0).items()}
    oracle = OracleModel(state, vars(cfg))
    del state
    eng = OracleEngine(oracle, max_slots=32, max_len=MAX_LEN)
    reqs = [OracleRequest(r.rid, r.prompt, r.max_new_tokens) for r in synthetic.serving96()]
    for r in reqs:
        eng.submit(r)
    eng.model = StubModel(cfg.vocab_size)
    for _ in range(WINDOW[0]):
        eng.step()
    # the scheduler's queues at the start of every slice (the cache is all zero there)
    starts = []
    for _ in range(slices):
        starts.append(copy.deepcopy((list(eng.waiting), list(eng.active))))
        for _ in range(slice_steps):
            if eng.waiting or eng.active:
                eng.step()
    eng.model = oracle

    def restore(j: int) -> list:
        eng.cache.k[...] = 0.0
        eng.cache.v[...] = 0.0
        w, a = copy.deepcopy(starts[j])
        eng.waiting, eng.active = deque(w), a
        return w + a

    for _ in range(warmup):
        restore(0)
        eng.step()
    per = []
    for i in range(samples):
        live = restore(i % slices)
        t0 = sum(len(r.output) for r in live)
        s0 = time.perf_counter()
        for _ in range(slice_steps):
            if not (eng.waiting or eng.active):
                break
            eng.step()
        dt = time.perf_counter() - s0
        per.append((sum(len(r.output) for r in live) - t0, dt))
    toks = sum(t for t, _ in per)
    secs = sum(d for _, d in per)
    last = WINDOW[0] + slices * slice_steps - 1
    return {"value": toks / secs, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"engine steps {WINDOW[0]}-{last} of the 96-request trace (32 slots) in {slices} slice(s) "
                      f"of {slice_steps} steps, {samples} sample(s) cycling through them, through the numpy "
                      f"oracle (fp32, {threads} host threads), {toks / samples:.0f} output tokens and "
                      f"{secs / samples:.1f} s per sample; slice starts reached by bookkeeping alone"}


def reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    # one step = a 10-engine-step slice of the window; the steps cycle through its 6 slices
    r = oracle_window(10, max(1, args.steps), args.warmup, slices=(WINDOW[1] - WINDOW[0]) // 10)
    line = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"serve96 window: engine steps {WINDOW[0]}-{WINDOW[1] - 1} of the 96-request "
                                   f"trace (prompts U[32,256], outputs lognormal(75,0.8)<=256, seed 4), "
                                   f"{args.slots} slots, max_len {MAX_LEN}, one replica per GPU",
                       "model": "Qwen2-0.5B architecture, random bf16 weights", "slots": args.slots,
                       "max_len": MAX_LEN, "window": list(WINDOW), "parallelism": f"replicas x{world}",
                       "l2": "inputs larger than L2: every decode step streams 988 MB of weights"},
            "cpu_baseline": r,
            "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.only == "serve3072":  # every rank serves its share
        if world > 1:
            torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
        try:
            r = serve3072(load_model(device), rank, world, device, peaks())
            if rank == 0:
                print(json.dumps(r), flush=True)
        finally:
            if world > 1:
                torch.distributed.destroy_process_group()
        return
    if args.only is not None:
        model = load_model(device)
        pk = peaks()
        r = {"decode": lambda: decode_steps(model, args.batch, args.steps, args.warmup, args.context, args.max_len),
             "batch1": lambda: batch1_latency(model, pk),
             "prefill": lambda: prefill_ttft(model, pk, tuple(int(x) for x in args.lengths.split(","))),
             "serve64": lambda: serve64(model)}[args.only]()
        print(json.dumps(r), flush=True)
        return
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    try:
        res = our_arm(args, rank, world, device)
        if rank == 0 and res is not None:
            if world == 1 and not args.no_cpu_baseline:
                try:
                    res["cpu_baseline"] = oracle_window(args.cpu_window_steps, 1, 0)
                except Exception as e:  # the baseline must not hide the GPU result
                    res["cpu_baseline"] = {"error": repr(e)}
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
