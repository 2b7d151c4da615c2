"""The one-time repack (`fuse`) on the host: tiled layout, RoPE-pair row order, gate/up
interleave. No GPU needed; the packed buffers must decode back to the checkpoint."""

from __future__ import annotations

import torch

from qweninfer_b200.models.config import qwen2_0p5b
from qweninfer_b200.models.qwen2 import Qwen2, rope_pair_order, tile_weight, untile_weight


def test_tile_roundtrip():
    w = torch.randn(384, 320)
    assert torch.equal(untile_weight(tile_weight(w), 384, 320), w)


def test_tile_core_matrix_is_contiguous():
    w = torch.arange(128 * 64).reshape(128, 64)
    t = tile_weight(w)
    # first 128 bytes (64 bf16) = rows 0..7, columns 0..7
    assert torch.equal(t[:64].reshape(8, 8), w[:8, :8])
    # next core matrix along K starts 64 elements later
    assert torch.equal(t[64:128].reshape(8, 8), w[:8, 8:16])
    # next 8-row group starts after the 8 core matrices of a 64-column block
    assert torch.equal(t[512:576].reshape(8, 8), w[8:16, :8])


def test_rope_pair_order():
    o = rope_pair_order(2, 64)
    assert o[:6].tolist() == [0, 32, 1, 33, 2, 34]
    assert o[64:66].tolist() == [64, 96]
    assert sorted(o.tolist()) == list(range(128))


def test_fuse_decodes_back_to_checkpoint():
    cfg = qwen2_0p5b(num_hidden_layers=1, vocab_size=256)
    torch.manual_seed(0)
    m = Qwen2(cfg)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0, 0.02)
    attn, mlp = m.layers[0].self_attn, m.layers[0].mlp
    wq, wk, wv = attn.q_proj.weight.clone(), attn.k_proj.weight.clone(), attn.v_proj.weight.clone()
    bq = attn.q_proj.bias.clone()
    wg, wu, wd = mlp.gate_proj.weight.clone(), mlp.up_proj.weight.clone(), mlp.down_proj.weight.clone()
    emb = m.embed_tokens.weight.clone()
    m.fuse()
    bf = lambda t: t.to(torch.bfloat16)  # noqa: E731
    qkv = untile_weight(attn.w_qkv_tiled, 1152, 896)
    inv = torch.argsort(rope_pair_order(18))
    assert torch.equal(qkv[inv], torch.cat([bf(wq), bf(wk), bf(wv)]))
    assert torch.equal(attn.b_qkv_f32[inv][:896], bf(bq).float())
    gu = untile_weight(mlp.w_gate_up_tiled, 9728, 896)
    assert torch.equal(gu[0::2], bf(wg)) and torch.equal(gu[1::2], bf(wu))
    assert torch.equal(untile_weight(mlp.w_down_tiled, 896, 4864), bf(wd))
    assert torch.equal(untile_weight(m.embed_tiled, 256, 896), bf(emb))
    assert not hasattr(m, "embed_tokens") and not hasattr(attn, "q_proj")
