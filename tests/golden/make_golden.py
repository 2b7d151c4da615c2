"""Generate the golden fixtures in this directory by running the REFERENCE package.

Run once, on a machine that has the reference checked out (read-only); point
$QI_REFERENCE at its project root:

    QI_REFERENCE=<path to the QwenInfer checkout> python tests/golden/make_golden.py

The fixtures pin the numpy oracle (`oracle/`) to the reference's own behaviour:

* config0_{fp32,bf16w,refbf16}.npz — the CPU reference run: 24-layer Qwen2-0.5B with
  seeded random weights (qweninfer_b200.synthetic, seed 0), a 64-token prompt (torch
  generator seed 1), prefill then 32 greedy tokens through the reference `generate`.
  fp32 = fp32 weights; bf16w = bf16-rounded weights on the fp32 path (the parity
  oracle for the bf16 CUDA path); refbf16 = the reference's own bf16 path, kept to
  show how far it strays from fp32. Each holds the greedy tokens, per-forward logits
  at a strided vocabulary subset, top-8 logits, whole-vector statistics, per-layer
  hidden states at two prompt positions and rows of the RoPE tables.
* engine_small.json — the reference `Engine` on the real model (bf16w weights):
  6 requests through 2 slots, a padded run, a static run and a capped-prefill run,
  with every scheduler action recorded, plus each request generated alone.
* sched_traces.json — the reference `Engine` driven by a stub model (bookkeeping
  only) over the 96-request serving workload (32 slots; 64 slots padded) and the
  rank-0-of-8 slice of the 3072-request workload (128 slots, max_len 4096): full
  trace for the 96-request runs, sha256 of the canonical trace for the large one.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if not os.environ.get("QI_REFERENCE"):
    sys.exit("set QI_REFERENCE to the QwenInfer project root (the reference checkout)")
REF = Path(os.environ["QI_REFERENCE"])
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REF))

from qweninfer.engine.engine import Engine, Request  # noqa: E402  (reference)
from qweninfer.engine.generate import generate  # noqa: E402  (reference)
from qweninfer.models.config import Qwen2Config as RefConfig  # noqa: E402
from qweninfer.models.qwen2 import Qwen2  # noqa: E402  (reference)

from qweninfer_b200 import synthetic  # noqa: E402
from oracle.engine_ref import pad_table, stub_token  # noqa: E402

V = 151936
LOGIT_STRIDE = 149
HIDDEN_POS = [0, 63]
ROPE_ROWS = [0, 1, 2, 63, 64, 100, 1000, 4095]


def canon_hash(trace) -> str:
    return hashlib.sha256(json.dumps(trace, separators=(",", ":")).encode()).hexdigest()


def load_ref(ckpt: Path, dtype) -> Qwen2:
    return Qwen2.from_pretrained(ckpt, dtype=dtype, device="cpu")


def config0(model: Qwen2, prompt: list[int], out_path: Path) -> None:
    step_logits: list[torch.Tensor] = []
    hidden: list[torch.Tensor] = []

    def logit_hook(_m, _i, out):
        step_logits.append(out[0, -1].detach().float().clone())

    def block_hook(_m, _i, out):
        if len(step_logits) == 0:  # prefill only
            hidden.append(out[0, HIDDEN_POS].detach().float().clone())

    h1 = model.register_forward_hook(logit_hook)
    hb = [b.register_forward_hook(block_hook) for b in model.layers]
    ids = torch.tensor([prompt])
    t0 = time.perf_counter()
    toks = generate(model, ids, 32)
    dt = time.perf_counter() - t0
    h1.remove()
    for h in hb:
        h.remove()
    L = torch.stack(step_logits).numpy()                     # (33, V)
    top_i = np.argsort(-L, axis=1, kind="stable")[:, :8]
    top_v = np.take_along_axis(L, top_i, axis=1)
    L64 = L.astype(np.float64)
    stats = np.stack([L64.sum(1), (L64 ** 2).sum(1), L64.max(1), L64.argmax(1)], 1)
    cos = model.rope_cos[ROPE_ROWS].float().numpy()
    sin = model.rope_sin[ROPE_ROWS].float().numpy()
    np.savez_compressed(
        out_path, prompt=np.array(prompt), tokens=np.array(toks),
        logit_idx=np.arange(0, V, LOGIT_STRIDE), logits_sub=L[:, ::LOGIT_STRIDE].copy(),
        top_idx=top_i, top_val=top_v, stats=stats,
        hidden=torch.stack(hidden).numpy(), hidden_pos=np.array(HIDDEN_POS),
        rope_rows=np.array(ROPE_ROWS), rope_cos=cos, rope_sin=sin, seconds=np.array(dt))
    print(f"{out_path.name}: tokens {toks[:8]}... ({dt:.1f}s)", flush=True)


class Recorder(torch.nn.Module):
    """Wraps a model (real or stub) and records every scheduler action of an Engine."""

    def __init__(self, inner, rid_of_prompt: dict) -> None:
        super().__init__()
        self.inner = inner
        self.cfg = inner.cfg
        self.norm = inner.norm
        self.rid_of_prompt = rid_of_prompt
        self.engine = None
        self.rec = None

    @property
    def dtype(self):
        return self.inner.dtype

    def forward(self, ids, positions=None, cache=None, last_only=False):
        out = self.inner(ids, positions=positions, cache=cache, last_only=last_only)
        if last_only:  # admission prefill, B = 1 (engine.py:127-129)
            tok = int(out[0, -1].argmax())
            rid = self.rid_of_prompt[tuple(ids[0].tolist())]
            self.rec["admit"].append([rid, cache.row_start, ids.shape[1], tok])
        else:  # batched decode (engine.py:152-155)
            act = self.engine.active
            rows = []
            for i in range(ids.shape[0]):
                rid = act[i].rid if i < len(act) else -1
                rows.append([rid, i, int(ids[i, 0]), int(positions[i, 0])])
            self.rec["decode"] = [ids.shape[0], rows]
        return out


class StubRef(torch.nn.Module):
    """Bookkeeping-only model for the reference Engine: argmax = stub_token(...)."""

    def __init__(self, vocab: int = 1000) -> None:
        super().__init__()
        self.vocab = vocab
        self.cfg = RefConfig(vocab, 1, 1, 1, 1, 1, 8192, 1e-6, 1e6, True)
        self.norm = torch.nn.Module()
        self.norm.weight = torch.nn.Parameter(torch.ones(1))

    @property
    def dtype(self):
        return torch.float32

    def forward(self, ids, positions=None, cache=None, last_only=False):
        B, S = ids.shape
        if positions is None:
            positions = torch.arange(S).expand(B, S)
        elif positions.dim() == 1:
            positions = positions.expand(B, S)
        out = torch.zeros(B, 1 if last_only else S, self.vocab)
        for b in range(B):
            out[b, -1, stub_token(int(ids[b, -1]), int(positions[b, -1]), self.vocab)] = 1.0
        return out


def run_engine(model, reqs: list[Request], **kw):
    rid_of_prompt = {tuple(r.prompt): r.rid for r in reqs}
    rec_model = Recorder(model, rid_of_prompt)
    eng = Engine(rec_model, **kw)
    rec_model.engine = eng
    trace = []
    orig_move = eng.cache.move_row

    def move_row(src, dst, length):
        rec_model.rec["move"].append([src, dst, length])
        orig_move(src, dst, length)

    eng.cache.move_row = move_row
    for r in reqs:
        eng.submit(r)
    finished = []
    with torch.inference_mode():
        while eng.waiting or eng.active:
            rec_model.rec = {"admit": [], "decode": None, "move": [], "done": []}
            done = eng.step()
            rec_model.rec["done"] = [r.rid for r in done]
            trace.append(rec_model.rec)
            finished += done
    finished.sort(key=lambda r: r.rid)
    return {str(r.rid): r.output for r in finished}, trace


def engine_small(model: Qwen2, out_path: Path) -> None:
    rng = np.random.default_rng(11)
    plens = [4, 9, 3, 7, 6, 5]
    olens = [5, 12, 3, 9, 7, 4]
    prompts = [rng.integers(0, V, p).tolist() for p in plens]

    def reqs():
        return [Request(i, list(p), n) for i, (p, n) in enumerate(zip(prompts, olens))]

    alone = {}
    with torch.inference_mode():
        for i, (p, n) in enumerate(zip(prompts, olens)):
            alone[str(i)] = generate(model, torch.tensor([p]), n)
    runs = {}
    for name, kw in [("slots2", dict(max_slots=2, max_len=64)),
                     ("slots4_pad", dict(max_slots=4, max_len=64, pad_to=[0, 4, 4, 4, 4])),
                     ("slots3_static", dict(max_slots=3, max_len=64, static=True)),
                     ("slots3_cap1", dict(max_slots=3, max_len=64, max_prefills_per_step=1))]:
        outs, trace = run_engine(model, reqs(), **kw)
        runs[name] = {"kwargs": kw, "outputs": outs, "trace": trace}
        print(f"engine {name}: {len(trace)} steps", flush=True)
    out_path.write_text(json.dumps({"prompts": prompts, "max_new_tokens": olens,
                                    "alone": alone, "runs": runs}, separators=(",", ":")))


def sched_traces(out_path: Path) -> None:
    res = {}

    def as_ref(reqs):
        return [Request(r.rid, r.prompt, r.max_new_tokens) for r in reqs]

    w96 = synthetic.serving96()
    for name, kw, full in [
        ("serve96_slots32", dict(max_slots=32, max_len=512), True),
        ("serve96_slots64_pad", dict(max_slots=64, max_len=512, pad_to=pad_table(64)), True),
        ("serve96_slots32_cap4", dict(max_slots=32, max_len=512, max_prefills_per_step=4), False),
        ("serve96_slots16_static", dict(max_slots=16, max_len=512, static=True), False),
    ]:
        outs, trace = run_engine(StubRef(), as_ref(w96), **kw)
        dec = [t["decode"] for t in trace if t["decode"]]
        res[name] = {"kwargs": kw, "sha256": canon_hash(trace), "steps": len(trace),
                     "decode_steps": len(dec),
                     "mean_rows": float(np.mean([len([x for x in d[1] if x[0] >= 0]) for d in dec])),
                     "moves": sum(len(t["move"]) for t in trace),
                     "outputs_sha256": canon_hash(outs)}
        if full:
            res[name]["trace"] = trace
        print(f"sched {name}: {res[name]['decode_steps']} decode steps, "
              f"mean B {res[name]['mean_rows']:.1f}, {res[name]['moves']} moves", flush=True)
    w3k = synthetic.serving3072(rank=0, world=8)
    kw = dict(max_slots=128, max_len=4096)
    outs, trace = run_engine(StubRef(), as_ref(w3k), **kw)
    dec = [t["decode"] for t in trace if t["decode"]]
    res["serve3072_rank0of8_slots128"] = {
        "kwargs": kw, "sha256": canon_hash(trace), "steps": len(trace), "decode_steps": len(dec),
        "mean_rows": float(np.mean([len([x for x in d[1] if x[0] >= 0]) for d in dec])),
        "moves": sum(len(t["move"]) for t in trace), "outputs_sha256": canon_hash(outs)}
    print(f"sched serve3072 slice: {len(dec)} decode steps", flush=True)
    out_path.write_text(json.dumps(res, separators=(",", ":")))


def main() -> None:
    torch.set_num_threads(os.cpu_count() or 8)
    cfg = synthetic.full_config()
    prompt = synthetic.config0_prompt()
    with tempfile.TemporaryDirectory() as td:
        td = Path(td)
        synthetic.write_checkpoint(td / "fp32", cfg, seed=0, dtype=torch.float32)
        synthetic.write_checkpoint(td / "bf16", cfg, seed=0, dtype=torch.bfloat16)
        m = load_ref(td / "fp32", torch.float32)
        config0(m, prompt, HERE / "config0_fp32.npz")
        del m
        m = load_ref(td / "bf16", torch.float32)   # bf16-rounded weights, fp32 path
        config0(m, prompt, HERE / "config0_bf16w.npz")
        engine_small(m, HERE / "engine_small.json")
        del m
        m = load_ref(td / "bf16", torch.bfloat16)  # the reference's own bf16 path
        config0(m, prompt, HERE / "config0_refbf16.npz")
        del m
    sched_traces(HERE / "sched_traces.json")


if __name__ == "__main__":
    main()
