"""Seeded synthetic inputs for parity tests and the CPU baseline — TEST INFRASTRUCTURE.

Weights: N(0, std) float32 draws rounded to bf16 (round to nearest even). Each
tensor is cut into blocks of 2^22 elements and block b of the t-th tensor (in
the tensor order of tensorsForLayers, weights.js:167-182, then embed_tokens,
norm and, for untied models, lm_head) draws from its own numpy PCG64 stream
seeded with SeedSequence([seed, t, b]); blocks are independent, so a thread
pool fills them and the result does not depend on the thread count. Norm
weights are exactly 1.0. Biases are N(0, std).
Named configurations follow the dims of the Qwen2.5 family.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from ref_forward import Config, f32_to_bf16_bits

CONFIGS = {
    # Qwen2.5-0.5B
    "0.5b": Config(vocab_size=151936, hidden_size=896, num_layers=24, num_q_heads=14, num_kv_heads=2, head_dim=64,
                   intermediate_size=4864, tie_word_embeddings=True),
    # Qwen2.5-1.5B (constants.js:10-23)
    "1.5b": Config(vocab_size=151936, hidden_size=1536, num_layers=28, num_q_heads=12, num_kv_heads=2, head_dim=128,
                   intermediate_size=8960, tie_word_embeddings=True),
    # Qwen2.5-7B
    "7b": Config(vocab_size=152064, hidden_size=3584, num_layers=28, num_q_heads=28, num_kv_heads=4, head_dim=128,
                 intermediate_size=18944, tie_word_embeddings=False),
    # Qwen2.5-32B
    "32b": Config(vocab_size=152064, hidden_size=5120, num_layers=64, num_q_heads=40, num_kv_heads=8, head_dim=128,
                  intermediate_size=27648, tie_word_embeddings=False),
}


BLOCK = 1 << 22


def tiny_config(**kw) -> Config:
    """A small Qwen2-shaped model that runs through every code path quickly."""
    base = dict(vocab_size=4096, hidden_size=256, num_layers=2, num_q_heads=4, num_kv_heads=2, head_dim=64,
                intermediate_size=512, tie_word_embeddings=True, eos_token_id=4000, max_pos=512)
    base.update(kw)
    return Config(**base)


def synthetic_weights(cfg: Config, seed: int = 0, std: float = 0.02, qkv_bias: bool = True,
                      layers: range | None = None, head: bool = True) -> dict[str, np.ndarray]:
    D, NQ, KVH, HD, I, V = (cfg.hidden_size, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim,
                            cfg.intermediate_size, cfg.vocab_size)
    pool = ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1))
    counter = [0]

    def normal(n: int) -> np.ndarray:
        t = counter[0]
        counter[0] += 1
        out = np.empty(n, np.uint16)

        def fill(b: int):
            lo, hi = b * BLOCK, min(n, (b + 1) * BLOCK)
            rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, t, b])))
            x = rng.standard_normal(size=hi - lo, dtype=np.float32)
            x *= np.float32(std)
            out[lo:hi] = f32_to_bf16_bits(x)

        list(pool.map(fill, range((n + BLOCK - 1) // BLOCK)))
        return out

    ones = f32_to_bf16_bits(np.ones(D, np.float32))
    W: dict[str, np.ndarray] = {}
    for L in (range(cfg.num_layers) if layers is None else layers):
        p = f"model.layers.{L}."
        W[p + "input_layernorm.weight"] = ones
        W[p + "post_attention_layernorm.weight"] = ones
        W[p + "self_attn.q_proj.weight"] = normal(NQ * HD * D)
        W[p + "self_attn.k_proj.weight"] = normal(KVH * HD * D)
        W[p + "self_attn.v_proj.weight"] = normal(KVH * HD * D)
        W[p + "self_attn.o_proj.weight"] = normal(D * NQ * HD)
        if qkv_bias:
            W[p + "self_attn.q_proj.bias"] = normal(NQ * HD)
            W[p + "self_attn.k_proj.bias"] = normal(KVH * HD)
            W[p + "self_attn.v_proj.bias"] = normal(KVH * HD)
        W[p + "mlp.gate_proj.weight"] = normal(I * D)
        W[p + "mlp.up_proj.weight"] = normal(I * D)
        W[p + "mlp.down_proj.weight"] = normal(D * I)
    if head:
        W["model.embed_tokens.weight"] = normal(V * D)
        W["model.norm.weight"] = ones
        if not cfg.tie_word_embeddings:
            W["lm_head.weight"] = normal(V * D)
    pool.shutdown()
    return W


def prompt_tokens(cfg: Config, n: int = 16, seed: int = 0) -> list[int]:
    """n prompt ids uniform in [0, vocab) from PCG64(seed) (a stream separate from the weights)."""
    rng = np.random.Generator(np.random.PCG64([seed, 1]))
    return [int(t) for t in rng.integers(0, cfg.vocab_size, size=n)]
