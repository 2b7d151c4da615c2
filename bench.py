"""Headline benchmark: the 96-request continuous-batching serving trace on B200.

Workload (synthetic, seeded; no dataset): Qwen2-0.5B architecture (24 layers, hidden
896, 14/2 heads, intermediate 4864, vocab 151936) with seeded random bf16 weights; 96
requests arriving at t=0, prompts uniform in [32, 256] tokens, output lengths lognormal
(median 75, sigma 0.8) clipped to [1, 256] and generated in full (no EOS); packed KV
cache with max_len 512; 32 slots. One bench step = one complete run of the trace
through `Engine.run` (the prefills of each step's admissions, batched into forwards of
up to 512 tokens, + every batched decode step + row moves).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl qweninfer_b200|reference]

Printed JSON (rank 0, one line):
  value  output tokens / device time of the trace's forwards (prefill + decode graph
         replays, CUDA events on the launching stream); host scheduling excluded.
  e2e    output tokens / time of Engine.run through the public API, CUDA events around
         the whole run: host bookkeeping, per-step H2D of (ids, positions, rows) from
         pinned memory and D2H of the argmax words included.
  roofline  the gate/up+SwiGLU tensor-core projection (tc_proj_kernel<swiglu>, the
         largest per-layer weight stream) at the trace's mean decode batch, timed alone
         over the 24 layers' distinct weights (418 MB > L2), achieved HBM GB/s vs the
         measured copy peak; traffic = DRAM bytes per launch from an ncu capture
         (profiles/tc_proj_swiglu_decode.md).
  cpu_baseline  the numpy oracle (the reference's algorithm restated) on the host cores
         over a bounded sample of the same workload.

Under torchrun (N > 1) every rank runs its own replica of the trace on its own GPU
(weak scaling, no collective on the data path); value = all ranks' tokens / max over
ranks of the device time.
"""

from __future__ import annotations

import argparse
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
WEIGHT_BYTES = 988_065_536          # bf16 layer weights + norms + biases + tied head
KV_BYTES_PER_TOKEN = 12_288         # 2 (K,V) * 24 layers * 2 heads * 64 * 2 B
# DRAM bytes (read + write) per launch of tc_proj_kernel<swiglu> by token tile, from one
# ncu capture of the same launch (profiles/tc_proj_swiglu_decode.md: token tile 32, the
# batch-22 case; 16 from an earlier capture of the same kernel); None until captured.
TRAFFIC: dict[int, int | None] = {16: 17_615_616, 32: 17_612_288}
EMBED_ROW_BYTES = 1_792


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="qweninfer_b200", choices=["qweninfer_b200", "reference"])
    ap.add_argument("--slots", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-seconds", type=float, default=15.0)
    ap.add_argument("--only", choices=["roofline", "decode"], default=None,
                    help="roofline: only the timed gate/up projection loop; decode: only graph-replayed "
                         "decode steps at --batch (the profiling cases)")
    ap.add_argument("--batch", type=int, default=22, help="decode batch of --only roofline")
    return ap.parse_args()


def peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


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
    """Wraps an engine's runner: CUDA-event device time of every forward, per-decode-step
    algorithmic bytes, kernel launch count."""

    def __init__(self, runner) -> None:
        self.r = runner
        self.device_ms = 0.0
        self.decode_ms = 0.0
        self.decode_bytes = 0
        self.decode_rows = []
        self.ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        self._prefill, self._prefill_many, self._decode = runner.prefill, runner.prefill_many, runner.decode
        runner.prefill, runner.prefill_many, runner.decode = self.prefill, self.prefill_many, self.decode

    def prefill(self, row, prompt):
        self.ev[0].record()
        tok = self._prefill(row, prompt)
        self.ev[1].record()
        self.ev[1].synchronize()
        self.device_ms += self.ev[0].elapsed_time(self.ev[1])
        return tok

    def prefill_many(self, rows, prompts):
        self.ev[0].record()
        toks = self._prefill_many(rows, prompts)
        self.ev[1].record()
        self.ev[1].synchronize()
        self.device_ms += self.ev[0].elapsed_time(self.ev[1])
        return toks

    def decode(self, toks, pos, row_start=0):
        self.ev[0].record()
        out = self._decode(toks, pos, row_start)
        self.ev[1].record()
        self.ev[1].synchronize()
        ms = self.ev[0].elapsed_time(self.ev[1])
        self.device_ms += ms
        self.decode_ms += ms
        B = len(toks)
        self.decode_bytes += (WEIGHT_BYTES + sum(p + 1 for p in pos) * KV_BYTES_PER_TOKEN
                              + B * KV_BYTES_PER_TOKEN + B * EMBED_ROW_BYTES)
        self.decode_rows.append(B)
        return out


def our_arm(args, rank: int, world: int, device: torch.device) -> dict | None:
    from qweninfer_b200 import synthetic
    from qweninfer_b200.engine.engine import Engine, Request

    model = load_model(device)
    workload = synthetic.serving96()
    eng = Engine(model, max_slots=args.slots, max_len=MAX_LEN)
    timed = TimedRunner(eng.runner)
    moves = [0]
    orig_move = eng.cache.move_row

    def move_row(src, dst, length):
        moves[0] += 1
        orig_move(src, dst, length)

    eng.cache.move_row = move_row

    def one_trace():
        reqs = [Request(r.rid, r.prompt, r.max_new_tokens) for r in workload]
        done = eng.run(reqs)
        return done

    for _ in range(args.warmup):
        one_trace()
    eng.runner.check()

    # timed region
    tokens = 0
    timed.device_ms = timed.decode_ms = 0.0
    timed.decode_bytes = 0
    timed.decode_rows = []
    launches0, h2d0, d2h0, moves0 = eng.runner.launches, eng.runner.h2d_bytes, eng.runner.d2h_bytes, moves[0]
    ttft, lat = [], []
    clocks = ClockSampler(device.index or 0)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.start()
    start.record()
    for _ in range(args.steps):
        done = one_trace()
        tokens += sum(len(r.output) for r in done)
        ttft += [r.first_token - r.arrival for r in done]
        lat += [r.finished - r.arrival for r in done]
    stop.record()
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    e2e_ms = start.elapsed_time(stop)
    dev_ms = timed.device_ms
    if world > 1:
        t = torch.tensor([dev_ms, e2e_ms, float(tokens)], device=device, dtype=torch.float64)
        mx = t.clone()
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        sm = t.clone()
        torch.distributed.all_reduce(sm, op=torch.distributed.ReduceOp.SUM)
        dev_ms, e2e_ms, tokens_all = float(mx[0]), float(mx[1]), float(sm[2])
        torch.distributed.barrier()
    else:
        tokens_all = float(tokens)
    eng.runner.check()
    if rank != 0:
        return None

    K = args.steps
    launches = (eng.runner.launches - launches0) + (moves[0] - moves0)
    res = {
        "metric": "decode tok/s on 96-req continuous-batch workload",
        "value": tokens_all / (dev_ms / 1e3),
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
        "config": {"workload": f"serve96: 96 requests, prompts U[32,256], outputs lognormal(75,0.8)<=256, "
                               f"{args.slots} slots, max_len {MAX_LEN}, one replica per GPU",
                   "model": "Qwen2-0.5B architecture, random bf16 weights",
                   "slots": args.slots, "max_len": MAX_LEN, "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2: every decode step streams 988 MB of weights"},
        "e2e": {"value": tokens_all / (e2e_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": (eng.runner.h2d_bytes - h2d0) // K,
                "d2h_bytes_per_step": (eng.runner.d2h_bytes - d2h0) // K,
                "ms_per_step": e2e_ms / K},
        "gpu_launches": launches,
        "serving": {"output_tokens_per_trace": tokens // K, "ttft_mean_s": statistics.mean(ttft),
                    "latency_mean_s": statistics.mean(lat),
                    "decode_steps_per_trace": len(timed.decode_rows) // K,
                    "mean_decode_batch": float(np.mean(timed.decode_rows)),
                    "decode_ms_per_step": timed.decode_ms / max(1, len(timed.decode_rows)),
                    "prefill_ms_total_per_trace": (timed.device_ms - timed.decode_ms) / K},
        "clocks": clock_info,
    }
    pk = peaks()
    step_gbs = timed.decode_bytes / (timed.decode_ms / 1e3) / 1e9
    res["decode_step_roofline"] = {"bound": "hbm", "achieved": step_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                                   "frac": step_gbs / pk["hbm_gbs"], "peak_source": pk["source"],
                                   "bytes": "988,065,536 weights + sum(len+1)*12,288 KV read + B*12,288 KV "
                                            "write + B*1,792 embed, per decode step"}
    res["roofline"] = kernel_roofline(model, int(round(np.mean(timed.decode_rows))), pk)
    res["batch1"] = batch1_latency(model)
    return res


def kernel_roofline(model, M: int, pk: dict) -> dict:
    """The forward's gate/up + SwiGLU projection (tc_proj_kernel<swiglu>, the launch
    qi_forward issues for it, through qi_tc_gate_up_swiglu) at decode batch M, cycling
    through the 24 layers' distinct weights (418 MB > L2), CUDA events on its stream."""
    import ctypes as C
    from qweninfer_b200 import _lib
    from qweninfer_b200.models.qwen2 import gate_up_tile
    dev = model.device
    NT = gate_up_tile(M)
    Mp = -(-M // NT) * NT
    L = _lib.lib()
    s = _lib.stream_ptr(dev)
    x = torch.randn(M, 896, device=dev)
    nw = model.layers[0].post_attention_layernorm.weight.float().contiguous()
    act = torch.zeros(Mp * 896 * 2, dtype=torch.int16, device=dev)
    ss = torch.zeros(7 * Mp, device=dev)
    _lib.check(L.qi_act_tiles(x.data_ptr(), nw.data_ptr(), M, 896, NT, act.data_ptr(), ss.data_ptr(), Mp, s),
               "act_tiles")
    out = torch.zeros(Mp * 4864 * 2, dtype=torch.int16, device=dev)
    scratch = torch.empty(148 * 2 * 128 * NT, device=dev)
    counters = torch.zeros(1024, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = [blk.mlp.w_gate_up_tiled.data_ptr() for blk in model.layers]

    def launch_all():
        for w in ws:
            _lib.check(L.qi_tc_gate_up_swiglu(w, act.data_ptr(), M, NT, ss.data_ptr(), Mp, C.c_float(1e-6),
                                              out.data_ptr(), scratch.data_ptr(), scratch.numel(),
                                              counters.data_ptr(), counters.numel(), 0, err.data_ptr(), s),
                       "tc_gate_up_swiglu")

    for _ in range(3):
        launch_all()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    a.record()
    for _ in range(reps):
        launch_all()
    b.record()
    b.synchronize()
    if int(err.item()) != 0:
        raise RuntimeError("gate/up kernel reported an error")
    per_launch_s = a.elapsed_time(b) / 1e3 / (reps * len(ws))
    # algorithmic bytes: weights once, activation tiles in (hi/lo bf16), the 7 partial sums
    # of squares, SwiGLU activation tiles out (hi/lo bf16), for the M live tokens
    algo = 9728 * 896 * 2 + M * 896 * 4 + 7 * M * 4 + M * 4864 * 4
    gbs = algo / per_launch_s / 1e9
    return {"kernel": "tc_proj_kernel<swiglu>: RMSNorm-folded gate/up projection + SwiGLU (tcgen05, bulk-copy "
                      "ring, the forward's stream-K partition), the forward's largest weight stream", "bound": "hbm",
            "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gbs / pk["hbm_gbs"],
            "peak_source": pk["source"], "traffic": TRAFFIC.get(NT), "batch": M, "token_tile": NT,
            "us_per_launch": per_launch_s * 1e6, "algorithmic_bytes_per_launch": algo}


def decode_steps(model, B: int, steps: int, warmup: int) -> dict:
    """Graph-replayed decode steps of B rows at positions ~200 (the profiling case)."""
    from qweninfer_b200.engine.kv_cache import KVCache
    from qweninfer_b200.engine.runner import DecodeRunner
    cache = KVCache(model.cfg, B, 512, dtype=torch.bfloat16, device=model.device)
    r = DecodeRunner(model, cache, max_batch=B)
    toks = [1] * B
    for i in range(warmup):
        r.decode(toks, [200 + i] * B)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        r.decode(toks, [200 + warmup + i] * B)
    b.record()
    b.synchronize()
    r.check()
    return {"batch": B, "steps": steps, "ms_per_step": a.elapsed_time(b) / steps}


def batch1_latency(model) -> dict:
    """Batch-1 decode ms/token at contexts 16/256/1024 (128 tokens each, CUDA events)."""
    from qweninfer_b200 import synthetic
    from qweninfer_b200.engine.kv_cache import KVCache
    from qweninfer_b200.engine.runner import DecodeRunner
    out = {}
    prompts = synthetic.decode_latency_prompts()
    for C_, prompt in prompts.items():
        cache = KVCache(model.cfg, 1, C_ + 130, dtype=torch.bfloat16, device=model.device)
        r = DecodeRunner(model, cache, max_batch=1)
        tok = r.prefill(0, prompt)
        for i in range(3):
            tok = int(r.decode([tok], [C_ + i])[0])
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        n = 125
        for i in range(n):
            tok = int(r.decode([tok], [C_ + 3 + i])[0])
        b.record()
        b.synchronize()
        ms = a.elapsed_time(b) / n
        byts = WEIGHT_BYTES + (C_ + 64) * KV_BYTES_PER_TOKEN
        out[str(C_)] = {"ms_per_token": ms, "hbm_gbs": byts / (ms / 1e3) / 1e9}
        del r, cache
    return out


# ------------------------------------------------------------- CPU arms

def cpu_sample(seconds: float) -> dict:
    """The numpy oracle (the reference's fp32 algorithm) on this host's cores: the serving
    trace (32 slots) run from its start until `seconds` of work, as tok/s."""
    from oracle import OracleModel, OracleRequest, bf16_round
    from oracle.engine_ref import OracleEngine
    from qweninfer_b200 import synthetic
    cfg = synthetic.full_config()
    state = {k: bf16_round(v.numpy()) for k, v in synthetic.synthetic_state(cfg, 0).items()}
    oracle = OracleModel(state, vars(cfg))
    del state
    eng = OracleEngine(oracle, max_slots=32, max_len=MAX_LEN)
    reqs = [OracleRequest(r.rid, r.prompt, r.max_new_tokens) for r in synthetic.serving96()]
    for r in reqs:
        eng.submit(r)
    t0 = time.perf_counter()
    steps = 0
    while (eng.waiting or eng.active) and time.perf_counter() - t0 < seconds:
        eng.step()
        steps += 1
    dt = time.perf_counter() - t0
    toks = sum(len(r.output) for r in reqs)
    return {"value": toks / dt, "unit": "tok/s", "cores": os.cpu_count() or 1,
            "kind": "port", "sample": f"first {steps} engine steps of the 96-request trace (32 slots) "
                                       f"through the numpy oracle (fp32, all host threads), {dt:.1f} s, "
                                       f"{toks} output tokens"}


def reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    per = []
    for i in range(args.warmup + args.steps):
        r = cpu_sample(args.cpu_sample_seconds / 3)
        if i >= args.warmup:
            per.append(r)
    v = statistics.mean(p["value"] for p in per)
    line = {"impl": "reference", "metric": "decode tok/s on 96-req continuous-batch workload", "value": v,
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "serve96, 32 slots, max_len 512 (bounded sample)"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": per[0]["cores"], "kind": "port",
                             "sample": per[0]["sample"]},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
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
    if args.only == "roofline":
        print(json.dumps(kernel_roofline(load_model(device), args.batch, peaks())), flush=True)
        return
    if args.only == "decode":
        print(json.dumps(decode_steps(load_model(device), args.batch, args.steps, args.warmup)), flush=True)
        return
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    try:
        res = our_arm(args, rank, world, device)
        if rank == 0 and res is not None:
            if world == 1 and not args.no_cpu_baseline:
                try:
                    res["cpu_baseline"] = cpu_sample(args.cpu_sample_seconds)
                except Exception as e:  # the baseline must not hide the GPU result
                    res["cpu_baseline"] = {"error": repr(e)}
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
