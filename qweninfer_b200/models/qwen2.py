"""Qwen2 (Qwen2.5-0.5B) on B200: QwenInfer's model API over the libqi.so kernels.

Same public surface as qweninfer/models/qwen2.py — `RMSNorm`, `build_rope_cache`,
`apply_rope`, `MLP`, `Attention`, `Block`, `Qwen2` with `from_pretrained`, `fuse` and
`forward(input_ids, positions=None, cache=None, last_only=False)` — so code written
against QwenInfer runs unchanged. The arithmetic runs in hand-written sm_100a kernels:

* `Qwen2.forward` is ONE native call (`qi_forward`): embedding, 24 blocks of
  {RMSNorm+QKV+bias+RoPE+KV-append, ragged attention, o_proj+residual,
  RMSNorm+gate/up+SwiGLU, down+residual}, final norm, tied head and argmax.
* Weights are bf16, activations and the residual stream fp32 (the reference's
  `residual_fp32=True` path keeps only the stream in fp32; here every activation stays
  fp32 because decode is bound by weight bytes, not activation math).
* `fuse()` repacks once, on the host, into the kernels' tiled layout (128x64 blocks of
  8x8 core matrices), with Q/K/V rows reordered so RoPE pairs are adjacent and gate/up
  rows interleaved so SwiGLU pairs are adjacent. The tied embedding keeps its (vocab,
  hidden) orientation: row gathers for lookup and K-major tiles for the head.

There is no CPU path: the modules raise on CPU tensors, and a missing libqi.so raises.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import torch
import torch.nn as nn

from qweninfer_b200 import _lib
from qweninfer_b200.models.config import Qwen2Config, check_supported

HIDDEN = 896
HEAD_DIM = 64
INTER = 4864


# ------------------------------------------------------------------ packing

def tile_weight(w: torch.Tensor) -> torch.Tensor:
    """Row-major (N, K) -> flat tiled layout of qi_tile_offset (N % 128 == 0, K % 64 == 0):
    (row tile, k block, 8-row group, 8-col chunk, row, col)."""
    n, k = w.shape
    if n % 128 or k % 64:
        raise ValueError(f"cannot tile a ({n}, {k}) matrix: need N % 128 == 0 and K % 64 == 0")
    t = w.reshape(n // 128, 16, 8, k // 64, 8, 8).permute(0, 3, 1, 4, 2, 5)
    return t.contiguous().reshape(-1)


def untile_weight(t: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """Inverse of `tile_weight`."""
    return t.reshape(n // 128, k // 64, 16, 8, 8, 8).permute(0, 2, 4, 1, 3, 5).reshape(n, k)


def rope_pair_order(n_heads: int, head_dim: int = HEAD_DIM) -> torch.Tensor:
    """Row order that puts RoPE partners (d, d + head_dim/2) of every head side by side."""
    half = head_dim // 2
    per_head = torch.stack([torch.arange(half), torch.arange(half) + half], 1).reshape(head_dim)
    return (torch.arange(n_heads)[:, None] * head_dim + per_head[None]).reshape(-1)


def _as_bf16(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.bfloat16)


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise _lib.QiError(f"{what}: qweninfer_b200 computes on CUDA (sm_100) tensors only, got {t.device}")


# ---------------------------------------------------------------- components

class RMSNorm(nn.Module):
    """qwen2.py:39-48: x * rsqrt(mean(x^2) + eps) * w, statistics in fp32 (kernel qi_rmsnorm)."""

    def __init__(self, hidden_dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _require_cuda(x, "RMSNorm")
        if x.shape[-1] != HIDDEN:
            raise ValueError(f"RMSNorm kernel is compiled for hidden size {HIDDEN}")
        _lib.ensure_device(x.device)
        out_dtype = torch.promote_types(x.dtype, self.weight.dtype)
        xf = x.reshape(-1, HIDDEN).float().contiguous()
        w = self.weight.detach().float().contiguous()
        out = torch.empty_like(xf)
        _lib.check(_lib.lib().qi_rmsnorm(xf.data_ptr(), w.data_ptr(), C.c_float(self.eps), xf.shape[0],
                                         out.data_ptr(), _lib.stream_ptr(x.device)), "qi_rmsnorm")
        return out.reshape(x.shape).to(out_dtype)


def build_rope_cache(head_dim: int, max_seq_len: int, theta: float,
                     device: torch.device | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """qwen2.py:53-73: fp32 cos/sin tables (max_seq_len, head_dim); plane i turns by
    position * theta^(-2i/head_dim), duplicated across the two halves. Computed exactly
    as the reference does so the kernels see the same table values."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
    pos = torch.arange(max_seq_len, device=device).float()
    angles = torch.outer(pos, inv_freq)
    emb = torch.cat([angles, angles], dim=-1)
    return emb.cos(), emb.sin()


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    """qwen2.py:76-83: for the half-split pairs (x[i], x[i + half]) return
    (-x[i + half], x[i]). A tensor helper of the API: the kernels rotate inside the QKV
    epilogue (and qi_rope) and never call it."""
    half = x.shape[-1] // 2
    return torch.cat([-x[..., half:], x[..., :half]], dim=-1)


def apply_rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
               positions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """qwen2.py:86-99: rotate q (B,H,S,hd) and k (B,Hkv,S,hd) by their positions ((S,) or
    (B,S)), half-split convention (kernel qi_rope, fp32 arithmetic)."""
    _require_cuda(q, "apply_rope")
    B, H, S, hd = q.shape
    Hk = k.shape[1]
    if hd != HEAD_DIM or k.shape[-1] != HEAD_DIM:
        raise ValueError(f"RoPE kernel is compiled for head_dim {HEAD_DIM}")
    _lib.ensure_device(q.device)
    pos = positions.to(q.device)
    pos = pos.expand(B, S) if pos.dim() == 1 else pos
    if int(pos.max()) >= cos.shape[0] or int(pos.min()) < 0:
        raise IndexError("position outside the RoPE table")
    pos32 = pos.to(torch.int32).contiguous()
    qf = q.float().contiguous().clone()
    kf = k.float().contiguous().clone()
    cf = cos.float().contiguous().to(q.device)
    sf = sin.float().contiguous().to(q.device)
    _lib.check(_lib.lib().qi_rope(qf.data_ptr(), H, kf.data_ptr(), Hk, B, S, pos32.data_ptr(),
                                  cf.data_ptr(), sf.data_ptr(), _lib.stream_ptr(q.device)), "qi_rope")
    return qf.to(q.dtype), kf.to(k.dtype)


class MLP(nn.Module):
    """qwen2.py:104-126: SwiGLU, down(silu(gate(x)) * up(x)); kernels qi_gate_up_swiglu
    (no norm) and qi_down_residual (into zeros)."""

    def __init__(self, cfg: Qwen2Config) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.up_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.down_proj = nn.Linear(cfg.intermediate_size, cfg.hidden_size, bias=False)

    @torch.no_grad()
    def fuse(self) -> None:
        """MLP.fuse (qwen2.py:119-126), repacked for the kernels: gate/up interleaved row
        by row into one tiled (2I, d) matrix, down tiled as (d, I)."""
        gu = torch.stack([_as_bf16(self.gate_proj.weight), _as_bf16(self.up_proj.weight)], 1)
        self.register_buffer("w_gate_up_tiled", tile_weight(gu.reshape(-1, gu.shape[-1])))
        self.register_buffer("w_down_tiled", tile_weight(_as_bf16(self.down_proj.weight)))
        del self.gate_proj, self.up_proj, self.down_proj

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _require_cuda(x, "MLP")
        if not hasattr(self, "w_gate_up_tiled"):
            self.fuse()
        _lib.ensure_device(x.device)
        xf = x.reshape(-1, HIDDEN).float().contiguous()
        M = xf.shape[0]
        h = torch.empty(M, INTER, dtype=torch.float32, device=x.device)
        out = torch.zeros(M, HIDDEN, dtype=torch.float32, device=x.device)
        err = torch.zeros(1, dtype=torch.int32, device=x.device)
        s = _lib.stream_ptr(x.device)
        L = _lib.lib()
        _lib.check(L.qi_gate_up_swiglu(xf.data_ptr(), None, C.c_float(0.0), self.w_gate_up_tiled.data_ptr(), M,
                                       h.data_ptr(), err.data_ptr(), s), "qi_gate_up_swiglu")
        _lib.check(L.qi_down_residual(h.data_ptr(), self.w_down_tiled.data_ptr(), M, out.data_ptr(),
                                      err.data_ptr(), s), "qi_down_residual")
        return out.reshape(x.shape).to(x.dtype)


class Attention(nn.Module):
    """qwen2.py:131-216: fused QKV (+bias), RoPE, cache append, GQA attention over each
    query's live keys, o_proj. Standalone use runs the same kernels as the model."""

    def __init__(self, cfg: Qwen2Config, layer_idx: int) -> None:
        super().__init__()
        self.layer_idx = layer_idx
        self.n_heads = cfg.num_attention_heads
        self.n_kv_heads = cfg.num_key_value_heads
        self.head_dim = cfg.head_dim
        self.n_rep = self.n_heads // self.n_kv_heads
        d = cfg.hidden_size
        self.q_proj = nn.Linear(d, self.n_heads * self.head_dim, bias=True)
        self.k_proj = nn.Linear(d, self.n_kv_heads * self.head_dim, bias=True)
        self.v_proj = nn.Linear(d, self.n_kv_heads * self.head_dim, bias=True)
        self.o_proj = nn.Linear(self.n_heads * self.head_dim, d, bias=False)

    @torch.no_grad()
    def fuse(self) -> None:
        """Attention.fuse (qwen2.py:207-216), repacked: q/k/v rows in RoPE-pair order,
        tiled (1152, 896) bf16; bias in the same order (fp32 of the bf16 values); o_proj
        tiled (896, 896)."""
        w = torch.cat([_as_bf16(self.q_proj.weight), _as_bf16(self.k_proj.weight),
                       _as_bf16(self.v_proj.weight)], 0)
        b = torch.cat([_as_bf16(self.q_proj.bias), _as_bf16(self.k_proj.bias),
                       _as_bf16(self.v_proj.bias)], 0)
        order = rope_pair_order(self.n_heads + 2 * self.n_kv_heads, self.head_dim)
        self.register_buffer("w_qkv_tiled", tile_weight(w[order]))
        self.register_buffer("b_qkv_f32", b[order].float().contiguous())
        self.register_buffer("w_o_tiled", tile_weight(_as_bf16(self.o_proj.weight)))
        del self.q_proj, self.k_proj, self.v_proj, self.o_proj

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, positions: torch.Tensor,
                cache=None) -> torch.Tensor:
        _require_cuda(x, "Attention")
        if not hasattr(self, "w_qkv_tiled"):
            self.fuse()
        from qweninfer_b200.engine.kv_cache import KVCache, _single_layer_view
        B, S, _ = x.shape
        dev = x.device
        _lib.ensure_device(dev)
        pos = positions.to(dev)
        pos = pos.expand(B, S) if pos.dim() == 1 else pos
        if cache is None:
            kl = torch.zeros(B, 2, S, HEAD_DIM, dtype=torch.bfloat16, device=dev)
            vl = torch.zeros_like(kl)
            row_start, max_len = 0, S
        else:
            kl, vl = _single_layer_view(cache, self.layer_idx)
            row_start, max_len = cache.row_start, cache.max_len
        if positions.device.type == "cpu" and (int(positions.max()) >= max_len or
                                               int(positions.max()) >= cos.shape[0]):
            raise IndexError("position beyond the cache or RoPE table")
        M = B * S
        pos32 = pos.reshape(M).to(torch.int32).contiguous()
        rows32 = (row_start + torch.arange(B, device=dev, dtype=torch.int32)).repeat_interleave(S)
        xf = x.reshape(M, HIDDEN).float().contiguous()
        q = torch.empty(M, HIDDEN, dtype=torch.float32, device=dev)
        attn = torch.empty_like(q)
        out = torch.zeros_like(q)
        # split scratch, kept per (tokens, cache length) so repeated calls allocate nothing
        key = (M, max_len, dev)
        ws = self._scratch.get(key) if hasattr(self, "_scratch") else None
        if ws is None:
            if not hasattr(self, "_scratch"):
                self._scratch = {}
            ws = self._scratch[key] = _AttnScratch(M, max_len, dev)
        err = ws.err
        s = _lib.stream_ptr(dev)
        L = _lib.lib()
        cf = cos.float().contiguous().to(dev)
        sf = sin.float().contiguous().to(dev)
        _lib.check(L.qi_qkv_rope_append(xf.data_ptr(), None, C.c_float(0.0), self.w_qkv_tiled.data_ptr(),
                                        self.b_qkv_f32.data_ptr(), cf.data_ptr(), sf.data_ptr(), pos32.data_ptr(),
                                        rows32.data_ptr(), M, kl.data_ptr(), vl.data_ptr(), max_len, q.data_ptr(),
                                        err.data_ptr(), s), "qi_qkv_rope_append")
        _lib.check(L.qi_attention(q.data_ptr(), kl.data_ptr(), vl.data_ptr(), pos32.data_ptr(), rows32.data_ptr(),
                                  M, max_len, ws.split_keys, ws.max_splits, attn.data_ptr(), ws.part.data_ptr(),
                                  ws.counters.data_ptr(), err.data_ptr(), s), "qi_attention")
        _lib.check(L.qi_o_proj_residual(attn.data_ptr(), self.w_o_tiled.data_ptr(), M, out.data_ptr(),
                                        err.data_ptr(), s), "qi_o_proj_residual")
        return out.reshape(B, S, HIDDEN).to(x.dtype)


class Block(nn.Module):
    """qwen2.py:221-240: pre-norm residual block."""

    def __init__(self, cfg: Qwen2Config, layer_idx: int) -> None:
        super().__init__()
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.self_attn = Attention(cfg, layer_idx)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.mlp = MLP(cfg)

    def forward(self, x, cos, sin, positions, cache=None) -> torch.Tensor:
        w = self.post_attention_layernorm.weight.dtype
        x = x + self.self_attn(self.input_layernorm(x).to(w), cos, sin, positions, cache).to(x.dtype)
        x = x + self.mlp(self.post_attention_layernorm(x).to(w)).to(x.dtype)
        return x


# ------------------------------------------------------------- scratch space

def _split_plan(max_tokens: int, max_len: int) -> tuple[int, int]:
    """Key-split size and count for attention over `max_len` cache slots. A split costs a
    merge (max-rescaled sums, in a thread-block cluster for 2-8 splits) and buys CTAs; with
    the tensor-core tile loop (~0.2 us per 128 keys) the merge dominates short rows.
    Measured on graph-replayed decode steps (ms, B = decode batch):
    max_len <= 1024 — one split: B 32 / 128 at contexts ~300, max_len 512: 0.989 / 1.626
    against 1.012 / 1.808 with 256-key splits (B 1: equal); max_len 4096 — 512 keys (8
    splits) up to B 32: B 32 at contexts ~1000 1.142 (256: 1.168, 1024: 1.185), B 1 at
    ~3000 0.954 (256: 1.075); 2048 keys beyond: B 64 at ~2000 1.608 (512: 1.792), B 128
    2.519 (1024: 2.500, 256: 3.028). Prefill-sized M (the per-token kernel serves the
    prompts below the block kernel's threshold): one split up to 4096 slots (a 512-token
    prompt at a 4096-slot cache 3.84 -> 2.95 ms against 1024-key splits, which made 4-CTA
    clusters of mostly empty splits)."""
    if max_tokens > 128:
        split = min(-(-max_len // 128) * 128, 4096)
    elif max_len <= 1024:
        split = -(-max_len // 128) * 128
    else:
        split = 512 if max_tokens <= 32 else 2048
    import os
    if os.environ.get("QI_ATTN_SPLIT"):  # tuning experiments: keys per split for every M
        split = max(128, int(os.environ["QI_ATTN_SPLIT"]) // 128 * 128)
    split = max(split, -(-max_len // (128 * 128)) * 128)  # at most 128 splits (the merge's capacity)
    return split, max(1, -(-max_len // split))


class _AttnScratch:
    """Attention split partials, arrival counters and the error word for M queries."""

    def __init__(self, M: int, max_len: int, device: torch.device) -> None:
        self.split_keys, self.max_splits = _split_plan(M, max_len)
        n = M * 2 * self.max_splits * 7 * 66 if self.max_splits > 1 else 1
        self.part = torch.empty(n, dtype=torch.float32, device=device)
        self.counters = torch.zeros(M * 2, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)


def token_tile(M: int) -> int:
    """Token tile of the forward's tensor-core projections for M tokens (the rule of
    token_tile in csrc/api.cu): 8 up to 8 tokens, 16 up to 96, 32 up to 384, 64 beyond.
    Non-decreasing in M, so buffers sized for max_tokens cover every smaller forward."""
    return 8 if M <= 8 else 16 if M <= 96 else 32 if M <= 384 else 64


def gate_up_tile(M: int) -> int:
    """Token tile of the forward's gate/up projection for M tokens (token_tiles in
    csrc/api.cu): 8 up to 8 tokens, 32 up to 32, 64 up to 384, 128 beyond."""
    return 8 if M <= 8 else 32 if M <= 32 else 64 if M <= 384 else 128


def use_tensor_cores() -> bool:
    """tcgen05 projections (default) or the CUDA-core GEMV path (QI_TENSOR_CORES=0)."""
    import os
    return os.environ.get("QI_TENSOR_CORES", "1") != "0"


class Workspace:
    """Activation buffers and scratch of `qi_forward` for up to `max_tokens` tokens of a
    cache with `max_len` slots per row. The library never allocates; this does, once."""

    def __init__(self, max_tokens: int, max_len: int, device: torch.device, vocab: int = 151936) -> None:
        f32 = dict(dtype=torch.float32, device=device)
        self.max_tokens, self.max_len = max_tokens, max_len
        self.x = torch.empty(max_tokens, HIDDEN, **f32)
        self.q = torch.empty(max_tokens, HIDDEN, **f32)
        self.attn = torch.empty(max_tokens, HIDDEN, **f32)
        self.h = torch.empty(max_tokens, INTER, **f32)
        small = min(max_tokens, 128)
        s_small, n_small = _split_plan(small, max_len)
        s_big, n_big = _split_plan(max(max_tokens, 129), max_len)
        parts = max(small * n_small, max_tokens * n_big) * 2 * 7 * 66
        self.attn_part = torch.empty(parts, **f32)
        self.attn_counters = torch.zeros(max_tokens * 2, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        # tensor-core path: activation tiles (hi/lo bf16), sums of squares, stream-K scratch,
        # padded to whole 128-token tiles so that any projection's token tile (a power of
        # two up to 128, tiles chosen per projection) and the decode step's fit
        nt = 128
        pad = -(-max_tokens // nt) * nt
        bf = dict(dtype=torch.bfloat16, device=device)
        self.act_x = torch.zeros(pad * HIDDEN * 2, **bf)
        self.act_attn = torch.zeros(pad * HIDDEN * 2, **bf)
        self.act_h = torch.zeros(pad * INTER * 2, **bf)
        self.ss = torch.zeros(7 * pad, **f32)
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        self.tc_scratch = torch.empty(sms * 2 * 128 * nt, **f32)
        n_counters = max(76 * -(-pad // 8), -(-vocab // 128), 64)  # any token tile down to 8
        self.tc_counters = torch.zeros(n_counters, dtype=torch.int32, device=device)
        self.struct = _lib.QiWorkspace(
            self.x.data_ptr(), self.q.data_ptr(), self.attn.data_ptr(), self.h.data_ptr(),
            self.attn_part.data_ptr(), self.attn_counters.data_ptr(), max_tokens, 1, 128, self.err.data_ptr(),
            int(use_tensor_cores()), self.act_x.data_ptr(), self.act_attn.data_ptr(), self.act_h.data_ptr(),
            self.ss.data_ptr(), pad, self.tc_scratch.data_ptr(), self.tc_scratch.numel(),
            self.tc_counters.data_ptr(), n_counters, 0)

    def plan(self, M: int, query_run: int = 0) -> "Workspace":
        """Attention splits for M query tokens; `query_run`: the longest prompt among them
        (its tokens consecutive and in one cache row), 0 if unknown — it picks the prefill
        attention kernel; 1 declares a decode step (one token per row, the rows' earlier
        keys already cached), whose attention starts its copies early."""
        self.struct.split_keys, self.struct.max_splits = _split_plan(M, self.max_len)
        self.struct.query_run = query_run
        return self

    def check(self) -> None:
        """Raise if a kernel recorded a timed-out wait (synchronises)."""
        e = int(self.err.item())
        if e:
            raise _lib.QiError(f"device error word = {e} (a bounded wait gave up)")


# --------------------------------------------------------------------- model

class Qwen2(nn.Module):
    """qwen2.py:243-337. Construct, load (`from_pretrained`), `fuse()`, move to an sm_100
    device, then call. `forward` returns logits (B, S or 1, vocab) in the model dtype
    (or `logits_dtype`)."""

    def __init__(self, cfg: Qwen2Config, max_seq_len: int = 4096, residual_fp32: bool = False) -> None:
        super().__init__()
        check_supported(cfg)
        self.cfg = cfg
        self.max_seq_len = max_seq_len
        self.residual_fp32 = residual_fp32
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(Block(cfg, i) for i in range(cfg.num_hidden_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        cos, sin = build_rope_cache(cfg.head_dim, max_seq_len, cfg.rope_theta)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)
        self._native = None
        self._workspaces: dict[tuple, Workspace] = {}

    @property
    def dtype(self) -> torch.dtype:
        return self.norm.weight.dtype

    @property
    def device(self) -> torch.device:
        return self.norm.weight.device

    @torch.no_grad()
    def fuse(self) -> None:
        """Qwen2.fuse (qwen2.py:294-308): repack every layer once, on the host, before the
        move to the GPU. The tied embedding is stored once, tiled (vocab, hidden)."""
        for layer in self.layers:
            layer.self_attn.fuse()
            layer.mlp.fuse()
        self.register_buffer("embed_tiled", tile_weight(_as_bf16(self.embed_tokens.weight)))
        del self.embed_tokens
        self._native = None

    def _apply(self, fn, recurse=True):
        self._native = None
        self._workspaces = {}
        return super()._apply(fn, recurse)

    # ------------------------------------------------------------- native

    def native(self) -> _lib.QiModel:
        """The qi_model descriptor of this model's device tensors (built once per move)."""
        if not hasattr(self, "embed_tiled"):
            raise _lib.QiError("call fuse() before running the model (from_pretrained does)")
        if self._native is None:
            dev = self.device
            _require_cuda(self.embed_tiled, "Qwen2")
            keep = []

            def f32(t):
                t = t.detach().float().contiguous()
                keep.append(t)
                return t.data_ptr()

            layers = (_lib.QiLayer * len(self.layers))()
            for i, blk in enumerate(self.layers):
                a, m = blk.self_attn, blk.mlp
                layers[i] = _lib.QiLayer(f32(blk.input_layernorm.weight), a.w_qkv_tiled.data_ptr(),
                                         a.b_qkv_f32.data_ptr(), a.w_o_tiled.data_ptr(),
                                         f32(blk.post_attention_layernorm.weight),
                                         m.w_gate_up_tiled.data_ptr(), m.w_down_tiled.data_ptr())
            cos = self.rope_cos.float().contiguous()
            sin = self.rope_sin.float().contiguous()
            keep += [cos, sin]
            st = _lib.QiModel(len(self.layers), self.cfg.vocab_size, cos.shape[0],
                              float(self.cfg.rms_norm_eps), self.embed_tiled.data_ptr(),
                              f32(self.norm.weight), cos.data_ptr(), sin.data_ptr(),
                              C.cast(layers, C.POINTER(_lib.QiLayer)))
            self._native = (st, layers, keep, dev)
        return self._native[0]

    def workspace(self, max_tokens: int, max_len: int) -> Workspace:
        key = (max_tokens, max_len)
        ws = self._workspaces.get(key)
        if ws is None:
            ws = Workspace(max_tokens, max_len, self.device, self.cfg.vocab_size)
            self._workspaces[key] = ws
        return ws

    # ------------------------------------------------------------ forward

    def _inputs(self, input_ids, positions, cache):
        """Build the int32 (ids, positions, rows) of B*S tokens. Inputs given on the host are
        checked there; inputs already on the device are not read back (no host
        synchronisation, as in the reference's forward): the kernels check every position
        and cache row and clamp token ids, and record QI_ERR_INDEX in the workspace error
        word (`check()`) instead of touching memory outside the cache."""
        from qweninfer_b200.engine.kv_cache import KVCache, PagedKVCache
        dev = self.device
        _lib.ensure_device(dev)
        B, S = input_ids.shape
        if positions is None:
            positions = torch.arange(S).expand(B, S)
        elif positions.dim() == 1:
            positions = positions.expand(B, S)
        if cache is None:
            cache = KVCache(self.cfg, B, S, dtype=torch.bfloat16, device=dev)
        if cache.row_start < 0 or cache.row_start + B > cache.max_batch:
            raise IndexError(f"rows [{cache.row_start}, {cache.row_start + B}) outside the cache")
        M = B * S
        if positions.device.type == "cpu":
            lo, hi = int(positions.min()), int(positions.max())
            if lo < 0 or hi >= cache.max_len or hi >= self.rope_cos.shape[0]:
                raise IndexError(f"positions [{lo}, {hi}] outside cache ({cache.max_len}) or RoPE table")
        if input_ids.device.type == "cpu":
            if int(input_ids.min()) < 0 or int(input_ids.max()) >= self.cfg.vocab_size:
                raise IndexError("token id outside the vocabulary")
        if isinstance(cache, PagedKVCache):
            # a paged cache maps the pages of the positions this forward writes and reads
            if positions.device.type != "cpu":
                raise ValueError("a paged KV cache needs the positions on the host")
            last = positions.reshape(B, S).max(dim=1).values
            for b in range(B):
                cache.reserve(cache.row_start + b, int(last[b]) + 1)
            cache.sync()
        ids32 = input_ids.reshape(M).to(device=dev, dtype=torch.int32, non_blocking=True).contiguous()
        pos32 = positions.reshape(M).to(device=dev, dtype=torch.int32, non_blocking=True).contiguous()
        rows32 = (cache.row_start + torch.arange(B, device=dev, dtype=torch.int32)).repeat_interleave(S)
        return cache, M, ids32, pos32, rows32

    def check(self) -> None:
        """Raise if a kernel of this model's forwards recorded an error (an index outside
        the cache or vocabulary, or a timed-out wait); synchronises."""
        for ws in self._workspaces.values():
            ws.check()

    @torch.inference_mode()
    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor | None = None, cache=None,
                last_only: bool = False, logits_dtype: torch.dtype | None = None) -> torch.Tensor:
        dev = self.device
        B, S = input_ids.shape
        cache, M, ids32, pos32, rows32 = self._inputs(input_ids, positions, cache)
        # head tokens: every token, or the last of each sequence (b*S + S-1)
        n_head, head_lo, head_stride = (B, S - 1, S) if last_only else (M, 0, 1)
        want = logits_dtype or getattr(self, "logits_dtype", None) or self.dtype
        # the kernels write fp32 or bf16 logits; a float16 request is converted from fp32
        ldt = torch.bfloat16 if want == torch.bfloat16 else torch.float32
        logits = torch.empty(n_head, self.cfg.vocab_size, dtype=ldt, device=dev)
        slots = torch.zeros(M, dtype=torch.int64, device=dev)
        ws = self.workspace(max(M, 1), cache.max_len).plan(M, S)
        _lib.check(_lib.lib().qi_forward(
            C.byref(self.native()), C.byref(cache.native()), C.byref(ws.struct), ids32.data_ptr(),
            pos32.data_ptr(), rows32.data_ptr(), M, head_lo, head_stride, n_head, logits.data_ptr(),
            int(ldt == torch.bfloat16), self.cfg.vocab_size, slots.data_ptr(), _lib.stream_ptr(dev)),
            "qi_forward")
        self.last_argmax = self.decode_argmax(slots[:n_head])
        return logits.view(B, 1 if last_only else S, self.cfg.vocab_size).to(want)

    @torch.inference_mode()
    def residual_stream(self, input_ids: torch.Tensor, n_layers: int, positions: torch.Tensor | None = None,
                        cache=None) -> torch.Tensor:
        """fp32 residual stream (B, S, hidden) after the first `n_layers` blocks (no head):
        the per-layer diagnostic of test_parity.py:195-261."""
        if not 0 <= n_layers <= self.cfg.num_hidden_layers:
            raise ValueError(f"n_layers must be in 0..{self.cfg.num_hidden_layers}")
        B, S = input_ids.shape
        cache, M, ids32, pos32, rows32 = self._inputs(input_ids, positions, cache)
        ws = self.workspace(max(M, 1), cache.max_len).plan(M, S)
        full = self.native()
        part = _lib.QiModel(n_layers, full.vocab, full.max_seq, full.eps, full.embed, full.norm,
                            full.rope_cos, full.rope_sin, full.layers)
        if n_layers == 0:
            part.num_layers = 1  # qi_forward needs >= 1 layer; embed-only is read before it
            _lib.check(_lib.lib().qi_embed(self.embed_tiled.data_ptr(), full.vocab, ids32.data_ptr(), M,
                                           ws.x.data_ptr(), None, None, _lib.stream_ptr(self.device)),
                       "qi_embed")
            return ws.x[:M].clone().view(B, S, HIDDEN)
        _lib.check(_lib.lib().qi_forward(
            C.byref(part), C.byref(cache.native()), C.byref(ws.struct), ids32.data_ptr(), pos32.data_ptr(),
            rows32.data_ptr(), M, 0, 1, 0, None, 0, 0, None, _lib.stream_ptr(self.device)), "qi_forward")
        return ws.x[:M].clone().view(B, S, HIDDEN)

    @staticmethod
    def decode_argmax(slots: torch.Tensor) -> torch.Tensor:
        """Token ids from packed argmax slots (index = 0xffffffff - low 32 bits)."""
        return 0xFFFFFFFF - (slots & 0xFFFFFFFF)

    # ------------------------------------------------------------- loading

    @classmethod
    def from_pretrained(cls, path: str | Path, dtype: torch.dtype = torch.float16,
                        device: str | torch.device = "cuda", max_seq_len: int = 4096,
                        fuse: bool = True, residual_fp32: bool = True,
                        load_on_device: bool = True) -> "Qwen2":
        """qwen2.py:310-337: meta-device construction, safetensors load (strict), RoPE
        tables rebuilt in fp32, `fuse()`, on `device`.

        With `load_on_device` (the default for a CUDA `device`) the safetensors tensors are
        read straight into device memory and the repack into the kernels' tiled layout
        (`fuse`) runs there as device copies: the host never holds a repacked weight, and
        the only host work is the file read. Otherwise the repack runs on the host before
        one move to `device` (the reference's order). Both give identical buffers.

        The kernels compute with bfloat16 weights and fp32 activations, whatever `dtype`
        asks for (the reference's default is float16). A float16 or float32 request loads
        the checkpoint in that dtype and rounds the weights to bfloat16 once (8 mantissa
        bits instead of float16's 11: the weight rounding the parity bar is measured
        against); `dtype` then only sets the dtype of the returned logits."""
        from safetensors.torch import load_file

        if dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise ValueError(f"dtype must be bfloat16, float16 or float32; got {dtype}")
        path = Path(path)
        device = torch.device(device)
        on_dev = load_on_device and device.type == "cuda"
        if on_dev and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        cfg = Qwen2Config.from_json(path / "config.json")
        with torch.device("meta"):
            model = cls(cfg, max_seq_len, residual_fp32)
        state = load_file(path / "model.safetensors", device=str(device) if on_dev else "cpu")
        state = {k.removeprefix("model."): t.to(dtype).to(torch.bfloat16) for k, t in state.items()}
        model.load_state_dict(state, strict=True, assign=True)
        del state
        model.rope_cos, model.rope_sin = build_rope_cache(cfg.head_dim, max_seq_len, cfg.rope_theta)
        model.logits_dtype = dtype
        if on_dev:
            model.rope_cos, model.rope_sin = model.rope_cos.to(device), model.rope_sin.to(device)
        if fuse:
            model.fuse()
        return model.to(device).eval()
