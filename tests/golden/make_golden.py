"""Generates tests/golden/tiny_decode.npz: greedy decode of the tiny Qwen2-shaped
config with an untied LM head (synthetic bf16 weights, seed 0), as golden
vectors for the parity tests. (With tied embeddings and small random weights the
greedy stream just repeats the last prompt token.)

Two independent producers are recorded for the same weights and prompt:
  * the oracle (oracle/ref_forward.py, the numpy restatement of the reference's
    shaders and pipeline.js): emitted tokens and per-step logits;
  * transformers' Qwen2ForCausalLM (fp32, eager attention): the logits of the
    same teacher-forced steps, an implementation independent of this repo.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import ref_forward as ref  # noqa: E402
import synth  # noqa: E402

SEED, STEPS, PROMPT_LEN = 0, 8, 5


def hf_step_logits(cfg, W, seq):
    """Logits of every position of `seq` from transformers' Qwen2 (fp32)."""
    import torch
    import transformers as tr
    hf_cfg = tr.Qwen2Config(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                            intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_layers,
                            num_attention_heads=cfg.num_q_heads, num_key_value_heads=cfg.num_kv_heads,
                            head_dim=cfg.head_dim, rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta,
                            tie_word_embeddings=cfg.tie_word_embeddings, max_position_embeddings=cfg.max_pos,
                            attn_implementation="eager")
    model = tr.Qwen2ForCausalLM(hf_cfg).float().eval()
    shapes = {k: v.shape for k, v in model.state_dict().items()}
    sd = {k: torch.from_numpy(ref.bf16_bits_to_f32(v).copy()).reshape(shapes[k]) for k, v in W.items() if k in shapes}
    if cfg.tie_word_embeddings:
        sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    missing, _ = model.load_state_dict(sd, strict=False)
    assert not [m for m in missing if "rotary" not in m], missing
    with torch.no_grad():
        return model(torch.tensor([seq])).logits[0].numpy()


def golden_config():
    return synth.tiny_config(tie_word_embeddings=False)


def main():
    cfg = golden_config()
    W = synth.synthetic_weights(cfg, seed=SEED)
    prompt = synth.prompt_tokens(cfg, PROMPT_LEN, seed=SEED)
    o = ref.OracleLeader(cfg, ref.Weights(W))
    toks, logits = o.generate(prompt, STEPS, keep_logits=True)
    # transformers on the same token stream: step i predicts from prompt + toks[:i]
    hf = hf_step_logits(cfg, W, list(prompt) + list(toks[:-1]))
    hf_logits = hf[PROMPT_LEN - 1:PROMPT_LEN - 1 + len(toks)]
    out = os.path.join(ROOT, "tests", "golden", "tiny_decode.npz")
    np.savez_compressed(out, seed=SEED, steps=STEPS, prompt=np.array(prompt, np.int64),
                        tokens=np.array(toks, np.int64), logits=np.stack(logits).astype(np.float32),
                        hf_logits=hf_logits.astype(np.float32),
                        q0_checksum=int(np.sum(W["model.layers.0.self_attn.q_proj.weight"].astype(np.uint64))))
    print(out, "tokens", toks, "max |oracle - transformers|", float(np.abs(np.stack(logits) - hf_logits).max()))


if __name__ == "__main__":
    main()
