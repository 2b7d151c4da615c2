"""Seeded synthetic checkpoints and request workloads.

There is no real Qwen2.5-0.5B checkpoint or dataset on the machines this package is
measured on, so every run uses seeded random weights of the real architecture and
seeded synthetic requests:

* Weights: a dedicated `torch.Generator` seeded with `seed` draws every parameter in
  the reference module's registration order (qweninfer/models/qwen2.py:304-318,
  221-231, 131-147, 104-111): Linear/Embedding weights and the Q/K/V biases are
  N(0, 0.02); RMSNorm weights are 1.0 and draw nothing. The result is written as an
  HF-named safetensors checkpoint (`model.` prefix, tied embeddings, no lm_head) plus
  `config.json`, so both this package and the reference load it through their own
  `from_pretrained`.
* Requests: numpy `default_rng(seed)`, consumed as prompt lengths, then output
  lengths, then each request's token ids.
"""

from __future__ import annotations

import hashlib
import os
import tempfile
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from qweninfer_b200.models.config import Qwen2Config, qwen2_0p5b

INIT_STD = 0.02


def param_specs(cfg: Qwen2Config) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) of every parameter in the reference's registration order."""
    d, i_sz = cfg.hidden_size, cfg.intermediate_size
    hd, h, hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    specs: list[tuple[str, tuple[int, ...]]] = [("embed_tokens.weight", (cfg.vocab_size, d))]
    for li in range(cfg.num_hidden_layers):
        p = f"layers.{li}."
        specs += [
            (p + "input_layernorm.weight", (d,)),
            (p + "self_attn.q_proj.weight", (h * hd, d)),
            (p + "self_attn.q_proj.bias", (h * hd,)),
            (p + "self_attn.k_proj.weight", (hkv * hd, d)),
            (p + "self_attn.k_proj.bias", (hkv * hd,)),
            (p + "self_attn.v_proj.weight", (hkv * hd, d)),
            (p + "self_attn.v_proj.bias", (hkv * hd,)),
            (p + "self_attn.o_proj.weight", (d, h * hd)),
            (p + "post_attention_layernorm.weight", (d,)),
            (p + "mlp.gate_proj.weight", (i_sz, d)),
            (p + "mlp.up_proj.weight", (i_sz, d)),
            (p + "mlp.down_proj.weight", (d, i_sz)),
        ]
    specs.append(("norm.weight", (d,)))
    return specs


def synthetic_state(cfg: Qwen2Config, seed: int = 0) -> dict[str, torch.Tensor]:
    """fp32 parameters, keyed without the `model.` prefix."""
    g = torch.Generator().manual_seed(seed)
    out: dict[str, torch.Tensor] = {}
    for name, shape in param_specs(cfg):
        if name.endswith("norm.weight"):
            out[name] = torch.ones(shape, dtype=torch.float32)
        else:
            out[name] = torch.empty(shape, dtype=torch.float32).normal_(0.0, INIT_STD, generator=g)
    return out


def write_checkpoint(path: str | Path, cfg: Qwen2Config, seed: int = 0,
                     dtype: torch.dtype = torch.bfloat16) -> Path:
    """Write `config.json` + `model.safetensors` (HF key names) under `path`."""
    from safetensors.torch import save_file

    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    state = synthetic_state(cfg, seed)
    tensors = {"model." + k: v.to(dtype).contiguous() for k, v in state.items()}
    del state
    save_file(tensors, str(path / "model.safetensors"))
    cfg.to_json(path / "config.json")
    (path / "DONE").write_text("ok\n")
    return path


def checkpoint_dir(cfg: Qwen2Config, seed: int = 0, dtype: torch.dtype = torch.bfloat16) -> Path:
    """A cached synthetic checkpoint for (cfg, seed, dtype), written on first use.

    The cache root is `$QI_SYNTH_DIR` if set, else `<tmp>/qweninfer_b200_synth`.
    """
    root = Path(os.environ.get("QI_SYNTH_DIR", Path(tempfile.gettempdir()) / "qweninfer_b200_synth"))
    tag = hashlib.sha1(repr((sorted(vars(cfg).items()), seed, str(dtype))).encode()).hexdigest()[:12]
    dname = str(dtype).split(".")[-1]
    path = root / f"L{cfg.num_hidden_layers}_V{cfg.vocab_size}_{dname}_s{seed}_{tag}"
    if not (path / "DONE").exists():
        tmp = Path(tempfile.mkdtemp(prefix=path.name + ".", dir=root if root.exists() else None))
        write_checkpoint(tmp, cfg, seed, dtype)
        root.mkdir(parents=True, exist_ok=True)
        try:
            tmp.rename(path)
        except OSError:
            pass  # another process finished first; its copy is identical
    return path


# ------------------------------------------------------------------ workloads

@dataclass
class SyntheticRequest:
    rid: int
    prompt: list[int]
    max_new_tokens: int


def config0_prompt(vocab_size: int = 151936, length: int = 64) -> list[int]:
    """The CPU reference run's prompt: torch uniform ids, generator seed 1."""
    g = torch.Generator().manual_seed(1)
    return torch.randint(0, vocab_size, (1, length), generator=g)[0].tolist()


def decode_latency_prompts(contexts=(16, 256, 1024), seed: int = 2,
                           vocab_size: int = 151936) -> dict[int, list[int]]:
    """Batch-1 decode latency prompts: one uniform prompt per context length."""
    rng = np.random.default_rng(seed)
    return {c: rng.integers(0, vocab_size, c).tolist() for c in contexts}


def prefill_prompts(lengths=(64, 256, 512, 1024), seed: int = 3,
                    vocab_size: int = 151936) -> dict[int, list[int]]:
    """Time-to-first-token prompts."""
    rng = np.random.default_rng(seed)
    return {p: rng.integers(0, vocab_size, p).tolist() for p in lengths}


def serving_requests(n: int, p_lo: int, p_hi: int, out_median: float, out_sigma: float,
                     out_cap: int, seed: int, vocab_size: int = 151936) -> list[SyntheticRequest]:
    """Requests with uniform prompt lengths in [p_lo, p_hi] and lognormal output lengths
    (rounded, clipped to [1, out_cap]); rng draws lengths first, then ids per request."""
    rng = np.random.default_rng(seed)
    plens = rng.integers(p_lo, p_hi + 1, n)
    olens = np.clip(np.rint(rng.lognormal(np.log(out_median), out_sigma, n)), 1, out_cap).astype(int)
    return [SyntheticRequest(i, rng.integers(0, vocab_size, int(p)).tolist(), int(o))
            for i, (p, o) in enumerate(zip(plens, olens))]


def serving96() -> list[SyntheticRequest]:
    """96 requests, prompts 32..256, outputs lognormal(median 75, sigma 0.8) <= 256, seed 4."""
    return serving_requests(96, 32, 256, 75.0, 0.8, 256, seed=4)


def serving3072(rank: int = 0, world: int = 1) -> list[SyntheticRequest]:
    """3072 requests, prompts 128..2048, outputs lognormal(200, 0.9) <= 1024, seed 5;
    rank `rank` of `world` replicas keeps the requests with rid % world == rank."""
    reqs = serving_requests(3072, 128, 2048, 200.0, 0.9, 1024, seed=5)
    return [r for r in reqs if r.rid % world == rank]


def full_config() -> Qwen2Config:
    return qwen2_0p5b()
