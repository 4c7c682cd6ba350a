"""Wide passes against the oracle: prefill chunks and micro-batches of more rows
than the persistent stage kernel takes (its limit is 8), which run their
projections as tcgen05 GEMMs (Stage.forward / generate's prefill of
pipeline.js:48-78,255-261 and the multi-sequence decode of a micro-batch).

* generate() with a prompt long enough for the wide prefill, at Qwen2.5-7B dims
  (2 layers, bf16 KV, untied head) and Qwen2.5-0.5B dims (3 layers, fp32 KV,
  head_dim 64): emitted tokens equal the oracle's generate and the kept logits
  agree within the north_star bar (rtol/atol 2e-2);
* a micro-batch of 16 sequences with different KV lengths decoded in one wide
  pass (embedding, layers, LM head, argmax per row): each row's hidden state and
  greedy token equal the oracle's single-sequence decode step, and the same rows
  through 8-row stage-kernel passes agree with the wide pass."""
import importlib
import os

import numpy as np
import pytest

import ref_forward as ref
from helpers import RefModel, assert_close, ref_lib, top2_margin

pytestmark = pytest.mark.gpu


def _oracle_cfg(cfg) -> ref.Config:
    return ref.Config(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, num_layers=cfg.num_layers,
                      num_q_heads=cfg.num_q_heads, num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                      intermediate_size=cfg.intermediate_size, rope_theta=cfg.rope_theta,
                      rms_norm_eps=cfg.rms_norm_eps, tie_word_embeddings=cfg.tie_word_embeddings,
                      eos_token_id=cfg.eos_token_id, max_pos=cfg.max_pos)


def _lib():
    lib = ref_lib()
    lib.ref_set_threads(os.cpu_count() or 1)
    return lib


@pytest.mark.parametrize("preset,layers,kv,prompt_len", [("qwen2.5-7b", 2, "bf16", 48),
                                                         ("qwen2.5-0.5b", 3, "f32", 20)])
def test_wide_prefill_generate_matches_oracle(dllm, preset, layers, kv, prompt_len):
    syn = importlib.import_module("distributed-llm1_b200.synthetic")
    steps = 5
    cfg = dllm.PRESETS[preset].with_(num_layers=layers, kv_dtype=kv, max_pos=prompt_len + steps + 8)
    ctx = dllm.initKernels(0, cfg)
    ld = dllm.LeaderPipeline(ctx, (0, layers))
    syn.device_weights(ctx, ld.stage, cfg, 0, layers, embed=True, head=True, seed=11)
    ctx.synchronize(120000)
    W = syn.read_back(ctx, ld.stage)
    prompt = [int(t) for t in np.random.default_rng(prompt_len).integers(0, cfg.vocab_size, prompt_len)]
    ld.set_keep_logits(steps)
    got = []
    ld.onToken = got.append
    ld.generate(prompt, steps)
    rm = RefModel(_lib(), _oracle_cfg(cfg), W, kv_bf16=(kv == "bf16"))
    want, logits = rm.generate(prompt, steps, keep_logits=True)
    for i in range(len(want)):
        assert_close(ld.read_logits(i), logits[i], rtol=2e-2, atol=2e-2, what=f"{preset} step {i} logits")
    margins = [round(top2_margin(lg), 4) for lg in logits]
    assert got == want, f"device {got} != oracle {want} (top-2 margins {margins})"
    rm.close()
    ld.close()
    ctx.close()


def test_wide_microbatch_16_sequences_matches_oracle(dllm):
    """16 sequences in one decode pass (row i = sequence i at its own T0)."""
    import torch
    syn = importlib.import_module("distributed-llm1_b200.synthetic")
    B, layers = 16, 2
    lens = [64 + 13 * i for i in range(B)]
    cfg = dllm.PRESETS["qwen2.5-7b"].with_(num_layers=layers, kv_dtype="bf16", max_seqs=B, max_pos=max(lens) + 8)
    ctx = dllm.initKernels(0, cfg)
    st = dllm.Stage(ctx, 0, layers)
    syn.device_weights(ctx, st, cfg, 0, layers, embed=True, head=True, seed=5)
    for s, n in enumerate(lens):
        st.fill_kv_random(s, n, seed=100 + s)
    ctx.synchronize(120000)
    W = syn.read_back(ctx, st)
    kvs = {s: [(st.kv[L].k.read(0, lens[s], seq=s), st.kv[L].v.read(0, lens[s], seq=s)) for L in range(layers)]
           for s in range(B)}
    toks_in = torch.tensor([(977 * s + 31) % cfg.vocab_size for s in range(B)], dtype=torch.int32, device="cuda")
    outs = {}
    for mode in ("wide", "stage"):
        if mode == "stage":
            ctx.set_tensor_core_rows(0)  # the same rows as 8-row stage-kernel passes
            for s, n in enumerate(lens):  # rewind: the wide pass appended one slot per sequence
                st.set_t0(s, n)
        h = torch.zeros(B, cfg.hidden_size, dtype=torch.float32, device="cuda")
        tout = torch.zeros(B, dtype=torch.int32, device="cuda")
        st.forward_rows(h.data_ptr(), list(range(B)), toks_in.data_ptr(), tout.data_ptr())
        torch.cuda.synchronize()
        ctx.synchronize()
        outs[mode] = (h.cpu().numpy(), tout.cpu().numpy())
        assert [st.t0_of(s) for s in range(B)] == [n + 1 for n in lens]
    ctx.set_tensor_core_rows(8)
    lib = _lib()
    ocfg = _oracle_cfg(cfg)
    for s in range(B):
        rm = RefModel(lib, ocfg, W, kv_bf16=True)
        for L in range(layers):
            rm.set_kv(L, 0, 0, kvs[s][L][0])
            rm.set_kv(L, 1, 0, kvs[s][L][1])
        rm.T0 = lens[s]
        tok = int(toks_in[s].item())
        e = np.zeros(cfg.hidden_size, np.float32)
        import ctypes as C
        t = np.array([tok], np.int32)
        lib.ref_embed(rm.h, t.ctypes.data_as(C.POINTER(C.c_int)), 1, e.ctypes.data_as(C.POINTER(C.c_float)))
        hrow = rm.forward(e, 1, lens[s])
        lg = np.zeros(cfg.vocab_size, np.float32)
        want_tok = lib.ref_sample_last(rm.h, hrow.ctypes.data_as(C.POINTER(C.c_float)),
                                       lg.ctypes.data_as(C.POINTER(C.c_float)))
        scale = float(np.max(np.abs(hrow)))
        assert_close(outs["wide"][0][s], hrow, rtol=2e-2, atol=2e-3 * scale, what=f"seq {s} hidden (wide)")
        assert int(outs["wide"][1][s]) == want_tok, f"seq {s}: wide token {outs['wide'][1][s]} != oracle {want_tok} " \
                                                    f"(top-2 margin {top2_margin(lg):.4f})"
        rm.close()
    np.testing.assert_array_equal(outs["wide"][1], outs["stage"][1])
    assert_close(outs["wide"][0], outs["stage"][0], rtol=1e-3, atol=1e-3 * float(np.max(np.abs(outs["stage"][0]))),
                 what="wide vs stage-kernel passes")
    st.close()
    ctx.close()
