"""Seeded synthetic weights generated on the device, and their host copies.

No checkpoint exists for the benchmark configurations, so weights are random:
N(0, 0.02) rounded to bf16 for every matrix and bias, 1.0 for the RMSNorm
gains, one counter-hash stream per tensor (dllm_fill_normal_bf16). The host copy
(`read_back`) is the exact bf16 bits the kernels read, so a CPU check can run
the same model.
"""
from __future__ import annotations

import numpy as np

WEIGHT_STD = 0.02

LAYER_SUFFIXES = ("input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
                  "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                  "self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias", "mlp.gate_proj.weight",
                  "mlp.up_proj.weight", "mlp.down_proj.weight")


def layer_sizes(cfg) -> dict:
    D, QD, KD, I = (cfg.hidden_size, cfg.num_q_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim,
                    cfg.intermediate_size)
    n = (D, D, QD * D, KD * D, KD * D, D * QD, QD, KD, KD, I * D, I * D, D * I)
    return dict(zip(LAYER_SUFFIXES, n))


def device_weights(ctx, stage, cfg, start: int, end: int, embed: bool, head: bool, seed: int = 0) -> dict:
    """Create and fill the tensors of layers [start, end) (and the embedding /
    final norm / LM head when asked) on the device and hand them to `stage.W`.
    Returns the leader buffers by role ("embed", "norm", "lm_head")."""
    sizes = layer_sizes(cfg)
    for L in range(start, end):
        for i, (suf, n) in enumerate(sizes.items()):
            name = f"model.layers.{L}.{suf}"
            b = ctx.createBf16(n, name)
            if "layernorm" in suf:
                ctx.fillConstBf16(b, 1.0)
            else:  # one stream per (layer, tensor): a layer gets the same values in any stage split
                ctx.fillNormalBf16(b, seed * 100003 + L * 97 + i, WEIGHT_STD)
            stage.W[name] = b
    V, D = cfg.vocab_size, cfg.hidden_size
    bufs = {}
    if embed or (head and cfg.tie_word_embeddings):
        bufs["embed"] = ctx.createBf16(V * D, "model.embed_tokens.weight")
        ctx.fillNormalBf16(bufs["embed"], seed * 100003 + 90001, WEIGHT_STD)
        stage.W["model.embed_tokens.weight"] = bufs["embed"]
    if head:
        bufs["norm"] = ctx.createBf16(D, "model.norm.weight")
        ctx.fillConstBf16(bufs["norm"], 1.0)
        stage.W["model.norm.weight"] = bufs["norm"]
        if not cfg.tie_word_embeddings:
            bufs["lm_head"] = ctx.createBf16(V * D, "lm_head.weight")
            ctx.fillNormalBf16(bufs["lm_head"], seed * 100003 + 90002, WEIGHT_STD)
            stage.W["lm_head.weight"] = bufs["lm_head"]
    return bufs


def read_back(ctx, stage) -> dict:
    """Host copies (uint16 bf16 bits) of every tensor the stage holds, by HF name."""
    out = {}
    for name, buf in stage.W.items():
        out[name] = np.asarray(ctx.readBf16(buf), dtype=np.uint16)
    return out
