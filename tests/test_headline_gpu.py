"""Parity of the instantiations the benchmark runs, against the oracle.

The decode benchmark runs stage_kernel<bf16 KV, head_dim 128, 1 row> with the
split-K MLP, the bf16 paged attention (G = NQ/KVH query heads per KV head, up
to 64 splits per head and their cooperative merge), the embedding gather and
the final norm + LM head + argmax, replayed as a CUDA graph (the device decode
loop of pipeline.js:262-267). These tests run exactly that path at the real
model widths, with fewer layers so the oracle finishes in seconds:

* Qwen2.5-7B dims (28/4 heads, G = 7, MLP 18944, untied 152064-row LM head),
  2 layers, 2048 prefilled bf16 KV slots, 6 greedy steps;
* Qwen2.5-1.5B dims (12/2 heads, G = 6, tied 151936-row head), 2 layers,
  8192 prefilled slots, 4 steps;
* Qwen2.5-32B dims (40/8 heads, G = 5, MLP 27648: split-K column slices of up
  to 192 columns, one warp per row group), 2 layers, 4096 prefilled slots,
  3 steps.

Weights are generated on the device and read back bit-exact; the prefilled KV
is read back from the device cache, so the oracle (oracle/ref_forward.cpp in
its bf16-KV mode: appended K/V rounded to bf16, kernels.js:86-132 and
pipeline.js:48-87,141-174 otherwise in fp32) starts from the same state. The
bar is BASELINE's: logits within rtol 2e-2 / atol 2e-2 and identical greedy
tokens. The per-step top-2 logit margin is printed so a near-tie is visible.

The attention phase alone is checked against the oracle's attention on the
q and the cache contents the kernel used, for 1k-32k slots at 7B dims and 32k
at 32B dims (G = 5)."""
import importlib
import os

import numpy as np
import pytest

import ref_forward as ref
from helpers import RefModel, assert_close, ref_lib, top2_margin

pytestmark = pytest.mark.gpu

CASES = {
    "7b": dict(preset="qwen2.5-7b", layers=2, kv_len=2048, steps=6),
    "1.5b": dict(preset="qwen2.5-1.5b", layers=2, kv_len=8192, steps=4),
    "32b": dict(preset="qwen2.5-32b", layers=2, kv_len=4096, steps=3),
}


def _oracle_cfg(cfg) -> ref.Config:
    return ref.Config(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, num_layers=cfg.num_layers,
                      num_q_heads=cfg.num_q_heads, num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                      intermediate_size=cfg.intermediate_size, rope_theta=cfg.rope_theta,
                      rms_norm_eps=cfg.rms_norm_eps, tie_word_embeddings=cfg.tie_word_embeddings,
                      eos_token_id=cfg.eos_token_id, max_pos=cfg.max_pos)


def _threads(lib):
    lib.ref_set_threads(os.cpu_count() or 1)  # results do not depend on the thread count
    return lib


@pytest.mark.parametrize("case", list(CASES))
def test_benched_decode_matches_oracle(dllm, case):
    syn = importlib.import_module("distributed-llm1_b200.synthetic")
    c = CASES[case]
    cfg = dllm.PRESETS[c["preset"]].with_(num_layers=c["layers"], kv_dtype="bf16",
                                          max_pos=c["kv_len"] + c["steps"] + 8)
    ctx = dllm.initKernels(0, cfg)
    ld = dllm.LeaderPipeline(ctx, (0, cfg.num_layers))
    bufs = syn.device_weights(ctx, ld.stage, cfg, 0, cfg.num_layers, embed=True, head=True, seed=7)
    ld.stage.fill_kv_random(0, c["kv_len"], seed=3)
    ctx.synchronize(120000)
    W = syn.read_back(ctx, ld.stage)
    rm = RefModel(_threads(ref_lib()), _oracle_cfg(cfg), W, kv_bf16=True)
    for L in range(cfg.num_layers):
        rm.set_kv(L, 0, 0, ld.stage.kv[L].k.read(0, c["kv_len"]))
        rm.set_kv(L, 1, 0, ld.stage.kv[L].v.read(0, c["kv_len"]))
    rm.T0 = c["kv_len"]
    ld.set_keep_logits(c["steps"])
    first = 4321
    got = ld.decode(first, c["steps"])  # the benchmark's graph-replayed decode loop
    tok, want, margins, worst = first, [], [], 0.0
    for i in range(c["steps"]):
        nxt, lg = rm.decode_step(tok)
        dev = ld.read_logits(i)
        assert_close(dev, lg, rtol=2e-2, atol=2e-2, what=f"{case} step {i} logits")
        worst = max(worst, float(np.max(np.abs(dev.astype(np.float64) - lg))))
        margins.append(top2_margin(lg))
        want.append(nxt)
        tok = nxt
    print(f"{case}: tokens {got}; max |logit diff| {worst:.3e}; top-2 margins {[round(m, 4) for m in margins]}")
    assert got == want, f"{case}: device tokens {got} != oracle {want} (top-2 margins {margins})"
    assert ld.stage.T0 == c["kv_len"] + c["steps"]
    del bufs
    rm.close()
    ld.close()
    ctx.close()


@pytest.mark.parametrize("preset,T,kv", [("qwen2.5-7b", 1024, "bf16"), ("qwen2.5-7b", 4096, "bf16"),
                                         ("qwen2.5-7b", 16384, "bf16"), ("qwen2.5-7b", 32768, "bf16"),
                                         ("qwen2.5-32b", 32768, "bf16"), ("qwen2.5-1.5b", 8192, "bf16"),
                                         ("qwen2.5-7b", 16384, "f32"), ("qwen2.5-32b", 5000, "f32")])
def test_paged_attention_matches_oracle(dllm, preset, T, kv):
    """One decode row at position T over T prefilled slots plus its own: the
    attention output of the stage kernel equals the oracle's attention
    (kernels.js:86-132) on the same q and the same cache contents. Stages whose
    attention items average more than 256 slots (max_pos * KV heads / SMs: here
    7B from 16k, 32B from 5k) stage K/V through the multi-round ring (rounds of
    64 slots at G = 7, 96 at G = 5; up to 4 rounds in flight for bf16, 2 for
    f32), the others one round at a time."""
    import ctypes as C
    syn = importlib.import_module("distributed-llm1_b200.synthetic")
    cfg = dllm.PRESETS[preset].with_(num_layers=1, kv_dtype=kv, max_pos=T + 64)
    ctx = dllm.initKernels(0, cfg)
    st = dllm.Stage(ctx, 0, 1)
    syn.device_weights(ctx, st, cfg, 0, 1, embed=False, head=False, seed=T)
    st.fill_kv_random(0, T, seed=T + 1)
    h = np.random.default_rng(T).standard_normal(cfg.hidden_size).astype(np.float32)
    st.forward(h, 1, T)
    q = st.read_workspace("q", 1).reshape(-1)
    att = st.read_workspace("att", 1).reshape(-1)
    K = st.kv[0].k.read(0, T + 1)
    V = st.kv[0].v.read(0, T + 1)
    out = np.zeros_like(att)
    F = C.POINTER(C.c_float)
    ref_lib().ref_attention(q.ctypes.data_as(F), K.ctypes.data_as(F), V.ctypes.data_as(F), out.ctypes.data_as(F),
                            T, 1, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim)
    assert_close(att, out, rtol=1e-3, atol=1e-4, what=f"{preset} {kv} attention T={T}")
    st.close()
    ctx.close()
