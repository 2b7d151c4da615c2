"""numpy float32 restatement of the reference's Qwen2 forward, KV cache and `generate`.

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`). Every function cites the
reference line it restates (paths relative to the reference project root). The
arithmetic is the reference's fp32 path (`residual_fp32=True`, fp32 weights); to
model a bf16 checkpoint, pass weights already rounded to bf16 (`bf16_round`), which
is exactly what the reference's `from_pretrained(dtype=torch.float32)` sees when it
loads a bf16 checkpoint.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

F32 = np.float32


# ------------------------------------------------------------------ helpers

def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); return float32."""
    u = np.ascontiguousarray(a, dtype=F32).view(np.uint32)
    r = (u + (((u >> 16) & 1) + np.uint32(0x7FFF))) & np.uint32(0xFFFF0000)
    return r.astype(np.uint32).view(F32)


def load_safetensors_fp32(path: str | Path) -> dict[str, np.ndarray]:
    """Read a safetensors file into float32 arrays, keys without the `model.` prefix.

    Mirrors qweninfer/models/qwen2.py:325-327 (load, strip prefix, cast). Written by
    hand because numpy has no bfloat16 dtype.
    """
    path = Path(path)
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
        blob = f.read()
    out: dict[str, np.ndarray] = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        s, e = info["data_offsets"]
        raw = blob[s:e]
        shape = tuple(info["shape"])
        dt = info["dtype"]
        if dt == "F32":
            arr = np.frombuffer(raw, dtype=F32).reshape(shape).copy()
        elif dt == "BF16":
            arr = (np.frombuffer(raw, dtype=np.uint16).astype(np.uint32) << 16).view(F32).reshape(shape)
        elif dt == "F16":
            arr = np.frombuffer(raw, dtype=np.float16).astype(F32).reshape(shape)
        else:
            raise ValueError(f"unsupported safetensors dtype {dt} for {name}")
        out[name.removeprefix("model.")] = arr
    return out


# ---------------------------------------------------------------- components

def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """RMSNorm.forward, qwen2.py:44-48: x * rsqrt(mean(x^2) + eps) * w, in fp32."""
    sq = np.mean(np.square(x, dtype=F32), axis=-1, keepdims=True, dtype=F32)
    rms_inv = (F32(1.0) / np.sqrt(sq + F32(eps))).astype(F32)
    return (x * rms_inv * w).astype(F32)


def build_rope_cache(head_dim: int, max_seq_len: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """build_rope_cache, qwen2.py:53-73: fp32 cos/sin tables (max_seq_len, head_dim),
    angle(p, i) = p * theta^(-2i/head_dim), duplicated across the two halves."""
    exps = np.arange(0, head_dim, 2, dtype=F32) / F32(head_dim)
    inv_freq = (F32(1.0) / np.power(F32(theta), exps, dtype=F32)).astype(F32)
    pos = np.arange(max_seq_len, dtype=F32)
    angles = np.outer(pos, inv_freq).astype(F32)
    emb = np.concatenate([angles, angles], axis=-1)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)


def rotate_half(x: np.ndarray) -> np.ndarray:
    """_rotate_half, qwen2.py:76-83: (x1, x2) -> (-x2, x1) over the two halves."""
    half = x.shape[-1] // 2
    return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)


def apply_rope(q, k, cos, sin, positions):
    """apply_rope, qwen2.py:86-99; q (B,H,S,hd), k (B,Hkv,S,hd), positions (S,) or (B,S)."""
    c = np.expand_dims(cos[positions], -3)
    s = np.expand_dims(sin[positions], -3)
    return (q * c + rotate_half(q) * s).astype(F32), (k * c + rotate_half(k) * s).astype(F32)


# --------------------------------------------------------------------- cache

class OracleCache:
    """KVCache, qweninfer/engine/kv_cache.py:24-76, in float32 numpy.

    k, v: (layers, max_batch, kv_heads, max_len, head_dim). Slot j of a row holds the
    token at absolute position j; `row_start` and `window` are set by the caller.
    `kv_bf16=True` stores k/v rounded to bfloat16, as the reference's cache does when
    the model dtype is bf16 (KVCache(dtype=model.dtype), engine.py:89-90).
    """

    def __init__(self, cfg: dict, max_batch: int, max_len: int, kv_bf16: bool = False) -> None:
        self.kv_bf16 = kv_bf16
        shape = (cfg["num_hidden_layers"], max_batch, cfg["num_key_value_heads"], max_len,
                 cfg["hidden_size"] // cfg["num_attention_heads"])
        self.k = np.zeros(shape, dtype=F32)
        self.v = np.zeros(shape, dtype=F32)
        self.max_batch, self.max_len = max_batch, max_len
        self.window = 0
        self.row_start = 0

    def update(self, layer: int, k: np.ndarray, v: np.ndarray, positions: np.ndarray):
        """kv_cache.py:48-63: scatter (B,Hkv,S,hd) at `positions` (B,S), return the
        (B,Hkv,window,hd) history of the same rows."""
        b = k.shape[0]
        if self.kv_bf16:
            k, v = bf16_round(k), bf16_round(v)
        rows = (self.row_start + np.arange(b))[:, None]
        self.k[layer, rows, :, positions] = k.transpose(0, 2, 1, 3)
        self.v[layer, rows, :, positions] = v.transpose(0, 2, 1, 3)
        r = slice(self.row_start, self.row_start + b)
        return self.k[layer, r, :, : self.window], self.v[layer, r, :, : self.window]

    def move_row(self, src: int, dst: int, length: int) -> None:
        """kv_cache.py:65-73: copy positions [0, length) of row src to row dst, all layers."""
        self.k[:, dst, :, :length] = self.k[:, src, :, :length]
        self.v[:, dst, :, :length] = self.v[:, src, :, :length]

    def memory_bytes(self) -> int:
        return 2 * self.k.size * 2  # as a bf16 cache would hold it


# --------------------------------------------------------------------- model

class OracleModel:
    """Qwen2 forward, qwen2.py:243-292, with the fused layout of qwen2.py:294-308.

    `state` holds float32 arrays keyed like the checkpoint without `model.`
    (`embed_tokens.weight`, `layers.{i}.self_attn.q_proj.weight`, ...).
    """

    def __init__(self, state: dict[str, np.ndarray], cfg: dict, max_seq_len: int = 4096) -> None:
        self.cfg = dict(cfg)
        self.L = cfg["num_hidden_layers"]
        self.H = cfg["num_attention_heads"]
        self.Hkv = cfg["num_key_value_heads"]
        self.d = cfg["hidden_size"]
        self.hd = self.d // self.H
        self.R = self.H // self.Hkv
        self.eps = cfg["rms_norm_eps"]
        self.scale = F32(1.0 / np.sqrt(self.hd))
        self.embed = np.ascontiguousarray(state["embed_tokens.weight"], dtype=F32)  # (V, d)
        self.layers = []
        for i in range(self.L):
            p = f"layers.{i}."
            g = lambda n: np.asarray(state[p + n], dtype=F32)  # noqa: E731
            # Attention.fuse / MLP.fuse, qwen2.py:207-216 and 119-126 (transposed to (in, out)).
            w_qkv = np.concatenate([g("self_attn.q_proj.weight"), g("self_attn.k_proj.weight"),
                                    g("self_attn.v_proj.weight")], 0).T.copy()
            b_qkv = np.concatenate([g("self_attn.q_proj.bias"), g("self_attn.k_proj.bias"),
                                    g("self_attn.v_proj.bias")], 0)
            w_gu = np.concatenate([g("mlp.gate_proj.weight"), g("mlp.up_proj.weight")], 0).T.copy()
            self.layers.append(dict(
                ln1=g("input_layernorm.weight"), ln2=g("post_attention_layernorm.weight"),
                w_qkv=w_qkv, b_qkv=b_qkv, w_o=g("self_attn.o_proj.weight").T.copy(),
                w_gate_up=w_gu, w_down=g("mlp.down_proj.weight").T.copy()))
        self.norm = np.asarray(state["norm.weight"], dtype=F32)
        self.cos, self.sin = build_rope_cache(self.hd, max_seq_len, cfg["rope_theta"])

    # Attention.forward, qwen2.py:149-205
    def attention(self, li: int, x: np.ndarray, positions: np.ndarray, cache) -> np.ndarray:
        lw = self.layers[li]
        B, S, _ = x.shape
        H, Hkv, hd, R = self.H, self.Hkv, self.hd, self.R
        qkv = (x @ lw["w_qkv"] + lw["b_qkv"]).astype(F32)
        q, k, v = np.split(qkv, [H * hd, H * hd + Hkv * hd], axis=-1)
        q = q.reshape(B, S, H, hd).transpose(0, 2, 1, 3)
        k = k.reshape(B, S, Hkv, hd).transpose(0, 2, 1, 3)
        v = v.reshape(B, S, Hkv, hd).transpose(0, 2, 1, 3)
        q, k = apply_rope(q, k, self.cos, self.sin, positions)
        if cache is not None:
            k, v = cache.update(li, k, v, positions)
        T = k.shape[-2]
        qf = np.ascontiguousarray(q).reshape(B, Hkv, R * S, hd)
        scores = (qf @ k.transpose(0, 1, 3, 2)) * self.scale               # (B,Hkv,R*S,T)
        visible = np.arange(T).reshape(1, 1, T) <= positions[..., None]      # (B,S,T)
        scores = scores.reshape(B, Hkv, R, S, T)
        scores = np.where(visible[:, None, None], scores, -np.inf).astype(F32)
        scores = scores - scores.max(-1, keepdims=True)
        e = np.exp(scores, dtype=F32)
        probs = (e / e.sum(-1, keepdims=True, dtype=F32)).astype(F32)
        out = probs.reshape(B, Hkv, R * S, T) @ v                            # (B,Hkv,R*S,hd)
        out = out.reshape(B, H, S, hd).transpose(0, 2, 1, 3).reshape(B, S, H * hd)
        return (out @ lw["w_o"]).astype(F32)

    # MLP.forward, qwen2.py:113-117
    def mlp(self, li: int, x: np.ndarray) -> np.ndarray:
        lw = self.layers[li]
        gu = (x @ lw["w_gate_up"]).astype(F32)
        gate, up = np.split(gu, 2, axis=-1)
        silu = gate / (F32(1.0) + np.exp(-gate, dtype=F32))
        return ((silu * up).astype(F32) @ lw["w_down"]).astype(F32)

    # Qwen2.forward, qwen2.py:263-292 (residual stream in fp32)
    def forward(self, input_ids, positions=None, cache=None, last_only: bool = False,
                hidden: list | None = None) -> np.ndarray:
        ids = np.asarray(input_ids, dtype=np.int64)
        B, S = ids.shape
        if positions is None:
            positions = np.broadcast_to(np.arange(S), (B, S))
        else:
            positions = np.asarray(positions, dtype=np.int64)
            if positions.ndim == 1:
                positions = np.broadcast_to(positions, (B, S))
        x = self.embed[ids].astype(F32)                                      # (B,S,d)
        if hidden is not None:
            hidden.append(x.copy())
        for li in range(self.L):
            lw = self.layers[li]
            x = x + self.attention(li, rmsnorm(x, lw["ln1"], self.eps), positions, cache)
            x = x + self.mlp(li, rmsnorm(x, lw["ln2"], self.eps))
            if hidden is not None:
                hidden.append(x.copy())
        x = rmsnorm(x, self.norm, self.eps)
        if last_only:
            x = x[:, -1:]
        return (x @ self.embed.T).astype(F32)

    __call__ = forward


# ------------------------------------------------------------------ generate

def oracle_generate(model: OracleModel, prompt: list[int], max_new_tokens: int,
                    eos_ids: set[int] | None = None, cache: OracleCache | None = None,
                    on_token=None, step_logits: list | None = None,
                    kv_bf16: bool = False) -> list[int]:
    """generate, qweninfer/engine/generate.py:18-51 (greedy, one token per forward).

    `step_logits`, if given, receives the last-position logits of every forward
    (prefill first), for parity checks. `kv_bf16` selects a bf16-storing cache when
    none is given.
    """
    P = len(prompt)
    if cache is None:
        cache = OracleCache(model.cfg, 1, P + max_new_tokens, kv_bf16=kv_bf16)
    cache.window = P
    logits = model.forward(np.array([prompt]), positions=np.arange(P), cache=cache, last_only=True)
    if step_logits is not None:
        step_logits.append(logits[0, -1].copy())
    nxt = int(np.argmax(logits[0, -1]))
    out: list[int] = []
    for step in range(max_new_tokens):
        tok = nxt
        if eos_ids and tok in eos_ids:
            break
        out.append(tok)
        if on_token is not None:
            on_token(tok)
        pos = P + step
        cache.window = pos + 1
        logits = model.forward(np.array([[tok]]), positions=np.array([[pos]]), cache=cache)
        if step_logits is not None:
            step_logits.append(logits[0, -1].copy())
        nxt = int(np.argmax(logits[0, -1]))
    return out
