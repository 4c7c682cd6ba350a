"""CPU checks of the oracle and the host-side logic (no GPU).

The reference cannot be executed here (JavaScript + WebGPU, no runtime), so the
oracle is pinned as far as possible by:
  * known answers that follow from the reference's code alone (bf16 decode of
    weights.js, Math.round semantics of assignLayers, RoPE at position 0,
    single-slot attention, first-max argmax),
  * agreement of two independent restatements (numpy vs the C++ loop-order
    restatement of the WGSL shaders),
  * an independent implementation of the same model (transformers' Qwen2),
  * the committed golden fixtures (tests/golden, made by tests/golden/make_golden.py).
"""
import ctypes as C
import os

import numpy as np
import pytest

import ref_forward as ref
import synth
from helpers import ROOT, RefModel, assert_close, mulberry32, ref_lib

F = C.POINTER(C.c_float)
U16 = C.POINTER(C.c_uint16)


# ---- weights.js known answers --------------------------------------------------------------
def test_bf16_bits_decode():
    bits = np.array([0x3F80, 0xBF80, 0x4000, 0x0000, 0x8000, 0x7F80, 0xFF80, 0x3F81, 0x0001], np.uint32)
    want = np.array([1.0, -1.0, 2.0, 0.0, -0.0, np.inf, -np.inf, 1.0078125, 9.183549615799121e-41], np.float32)
    np.testing.assert_array_equal(ref.bf16_bits_to_f32(bits), want)
    # the JS side keeps one u32 per element; the upper half is discarded by << 16
    np.testing.assert_array_equal(ref.bf16_bits_to_f32(np.array([0xABCD3F80], np.uint32)), [1.0])


def test_bf16_round_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, np.inf, np.nan, 1.0 + 2 ** -8 + 2 ** -20], np.float32)
    got = ref.f32_to_bf16_bits(x)
    assert got[0] == 0x3F80
    assert got[1] == 0x3F80  # halfway, even stays
    assert got[2] == 0x3F82  # halfway, odd rounds up
    assert got[3] == 0xC020
    assert got[5] == 0x7F80 and got[6] == 0x7FC0
    assert got[7] == 0x3F81  # above halfway rounds up


def test_bf16_bytes_to_bits_and_package_helpers(dllm):
    raw = np.array([0x3F80, 0x4049, 0xC2F7], "<u2").tobytes()
    np.testing.assert_array_equal(dllm.bf16BytesToF32Bits(raw), [0x3F80, 0x4049, 0xC2F7])
    np.testing.assert_array_equal(dllm.bf16BitsToF32(np.array([0x3F80, 0x4049, 0xC2F7]), 1, 2),
                                  ref.bf16_bits_to_f32(np.array([0x4049, 0xC2F7])))
    assert dllm.reinterpretBits(0x3F800000) == 1.0


def test_tensors_for_layers(dllm):
    names = dllm.tensorsForLayers(2, 4, True)
    assert len(names) == 2 * 12 + 2
    assert names[0] == "model.layers.2.input_layernorm.weight"
    assert names[-2:] == ["model.embed_tokens.weight", "model.norm.weight"]
    assert [n.split(".", 3)[3] for n in names[:12]] == list(ref.LAYER_SUFFIXES)


# ---- assignLayers (pipeline.js:6-23) -----------------------------------------------------
CASES = [
    # 8 equal GPU peers over 28 layers: seven shares of round(3.5) = 4, the last stage empty
    ([{"id": i, "profile": {"memGB": 8, "gpu": True}} for i in range(8)], 28,
     [(0, 4), (4, 8), (8, 12), (12, 16), (16, 20), (20, 24), (24, 28), (28, 28)]),
    # defaults: memGB 4, no gpu -> cap 2 each; 3 peers over 28 -> round(9.33)=9, 9, rest 10
    ([{"id": "a"}, {"id": "b", "profile": {}}, {"id": "c", "profile": None}], 28, [(0, 9), (9, 18), (18, 28)]),
    # a weak peer still gets max(1, ...) layers
    ([{"id": 1, "profile": {"memGB": 64, "gpu": True}}, {"id": 2, "profile": {"memGB": 1}}], 28, [(0, 28), (28, 28)]),
    # Math.round half-up: 2 equal peers over 5 layers -> round(2.5) = 3 (Python round gives 2)
    ([{"id": 1}, {"id": 2}], 5, [(0, 3), (3, 5)]),
    ([{"id": 0, "profile": {"memGB": 16, "gpu": True}}], 24, [(0, 24)]),
]


@pytest.mark.parametrize("peers,L,want", CASES)
def test_assign_layers(dllm, peers, L, want):
    got = [(r["start"], r["end"]) for r in dllm.assignLayers(peers, L)]
    assert got == want
    assert [(r["start"], r["end"]) for r in ref.assign_layers(peers, L)] == want
    assert [r["id"] for r in dllm.assignLayers(peers, L)] == [p["id"] for p in peers]


def test_plan_stages_balanced(dllm):
    cfg = dllm.PRESETS["qwen2.5-7b"]
    for n in (1, 2, 4, 8):
        r = dllm.plan_stages(cfg, n)
        assert len(r) == n and r[0][0] == 0 and r[-1][1] == cfg.num_layers
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        cost = [(e - s) * cfg.layer_weight_bytes() + (cfg.head_weight_bytes() if i == n - 1 else 0)
                for i, (s, e) in enumerate(r)]
        total = cfg.num_layers * cfg.layer_weight_bytes() + cfg.head_weight_bytes()
        assert max(cost) <= total / n + cfg.layer_weight_bytes()


# ---- frames (rtc.js:7-22) --------------------------------------------------------------------
def test_frame_round_trip(dllm):
    f32 = np.arange(7, dtype=np.float32) / 3
    b = dllm.frames.pack(dllm.FRAME["HIDDEN_REQ"], 5, 17, f32)
    assert len(b) == 16 + 28
    assert np.frombuffer(b[:16], "<i4").tolist() == [1, 5, 17, 7]
    fr = dllm.frames.unpack(b)
    assert (fr["msgType"], fr["seqId"], fr["posStart"]) == (1, 5, 17)
    np.testing.assert_array_equal(fr["f32"], f32)
    with pytest.raises(ValueError):
        dllm.frames.unpack(b[:-1])
    with pytest.raises(ValueError):
        dllm.frames.unpack(b"\0" * 8)


# ---- shader known answers -------------------------------------------------------------------
def test_rope_identity_at_position_zero():
    x = np.random.default_rng(0).standard_normal(3 * 128, dtype=np.float32)
    np.testing.assert_array_equal(ref.rope(x, 1, 3, 128, 0).reshape(-1), x)


def test_rope_freq_formula():
    fr = ref.rope_freqs(128, 1e6)
    assert fr[0] == 1.0
    assert abs(float(fr[1]) - 1e6 ** (-2 / 128)) < 1e-7
    assert abs(float(fr[63]) - 1e6 ** (-126 / 128)) / float(fr[63]) < 1e-6


def test_attention_single_slot_is_v():
    """With T0 = 0 and n = 1 the softmax has one term: the output is V (test.js:161-167)."""
    rng = np.random.default_rng(1)
    q = rng.standard_normal(12 * 128, dtype=np.float32)
    kc = rng.standard_normal((4, 256), dtype=np.float32)
    vc = rng.standard_normal((4, 256), dtype=np.float32)
    out = ref.attention(q, kc, vc, 0, 1, 12, 2, 128).reshape(12, 128)
    for h in range(12):
        np.testing.assert_array_equal(out[h], vc[0, (h // 6) * 128:(h // 6 + 1) * 128])


def test_argmax_first_max():
    v = np.array([0, 3, 1, 3, np.nan, -np.inf], np.float32)
    assert ref.argmax_first(v) == 1
    assert ref.argmax_first(np.full(5, np.nan, np.float32)) == 0
    assert ref.argmax_first(np.full(5, -np.inf, np.float32)) == 0


def test_mulberry32_matches_js():
    """test.js:8-10; values computed from the JS definition by hand-checked 32-bit steps."""
    r = mulberry32(42)
    first = [r() for _ in range(3)]
    assert all(0 <= x < 1 for x in first)
    r2 = mulberry32(42)
    assert [r2() for _ in range(3)] == first
    assert abs(first[0] - 0.6011037519201636) < 1e-15


# ---- numpy oracle vs C++ loop-order restatement -------------------------------------------
@pytest.fixture(scope="module")
def clib():
    lib = ref_lib()
    lib.ref_set_threads(4)
    return lib


def test_ops_numpy_vs_cpp(clib):
    rng = np.random.default_rng(2)
    n, din, dout = 3, 896, 1152
    x = rng.standard_normal(n * din, dtype=np.float32)
    w = ref.f32_to_bf16_bits(rng.standard_normal(din * dout, dtype=np.float32) * 0.02)
    out = np.empty(n * dout, np.float32)
    clib.ref_matmul(x.ctypes.data_as(F), w.ctypes.data_as(U16), out.ctypes.data_as(F), n, din, dout)
    assert_close(out, ref.matmul(x, w, n, din, dout).reshape(-1), rtol=1e-4, atol=1e-5, what="matmul")
    g = ref.f32_to_bf16_bits(rng.standard_normal(din, dtype=np.float32))
    clib.ref_rmsnorm(x.ctypes.data_as(F), g.ctypes.data_as(U16), out.ctypes.data_as(F), n, din, 1e-6)
    assert_close(out[:n * din], ref.rmsnorm(x, g, n, din).reshape(-1), rtol=1e-5, atol=1e-6, what="rmsnorm")
    fr = np.empty(64, np.float32)
    clib.ref_rope_freqs(128, 1e6, fr.ctypes.data_as(F))
    np.testing.assert_array_equal(fr, ref.rope_freqs(128, 1e6))
    xr = rng.standard_normal(2 * 4 * 128, dtype=np.float32)
    a = xr.copy()
    clib.ref_rope(a.ctypes.data_as(F), 2, 4, 128, 4095, fr.ctypes.data_as(F))
    assert_close(a, ref.rope(xr, 2, 4, 128, 4095).reshape(-1), rtol=1e-6, atol=1e-6, what="rope")
    q = rng.standard_normal(3 * 14 * 64, dtype=np.float32)
    kc = rng.standard_normal((64, 128), dtype=np.float32)
    vc = rng.standard_normal((64, 128), dtype=np.float32)
    o = np.empty(3 * 14 * 64, np.float32)
    clib.ref_attention(q.ctypes.data_as(F), kc.ctypes.data_as(F), vc.ctypes.data_as(F), o.ctypes.data_as(F), 40, 3,
                       14, 2, 64)
    assert_close(o, ref.attention(q, kc, vc, 40, 3, 14, 2, 64).reshape(-1), rtol=1e-5, atol=1e-6, what="attention")
    s = np.empty(1000, np.float32)
    aa, bb = rng.standard_normal(1000, dtype=np.float32) * 5, rng.standard_normal(1000, dtype=np.float32)
    clib.ref_silu_mul(aa.ctypes.data_as(F), bb.ctypes.data_as(F), s.ctypes.data_as(F), 1000)
    np.testing.assert_array_equal(s, ref.silu_mul(aa, bb))


@pytest.mark.parametrize("kv_bf16", [False, True])
def test_generate_numpy_vs_cpp(clib, kv_bf16):
    cfg = synth.tiny_config()
    W = synth.synthetic_weights(cfg, seed=3)
    prompt = synth.prompt_tokens(cfg, 7, seed=3)
    o = ref.OracleLeader(cfg, ref.Weights(W), kv_dtype="bf16" if kv_bf16 else "f32")
    t_np, l_np = o.generate(prompt, 12, keep_logits=True)
    m = RefModel(clib, cfg, W, kv_bf16=kv_bf16)
    t_c, l_c = m.generate(prompt, 12, keep_logits=True)
    assert t_np == t_c
    for a, b in zip(l_np, l_c):
        assert_close(a, b, rtol=1e-3, atol=1e-4, what="logits numpy vs C++")


def test_thread_count_does_not_change_results(clib):
    cfg = synth.tiny_config()
    W = synth.synthetic_weights(cfg, seed=4)
    prompt = [1, 2, 3]
    outs = []
    for th in (1, 5):
        clib.ref_set_threads(th)
        outs.append(RefModel(clib, cfg, W).generate(prompt, 6, keep_logits=True))
    clib.ref_set_threads(4)
    assert outs[0][0] == outs[1][0]
    np.testing.assert_array_equal(outs[0][1], outs[1][1])


# ---- independent implementation: transformers Qwen2 ------------------------------------------
def test_oracle_vs_transformers_qwen2():
    torch = pytest.importorskip("torch")
    tr = pytest.importorskip("transformers")
    cfg = synth.tiny_config(num_layers=2, vocab_size=512, eos_token_id=511)
    W = synth.synthetic_weights(cfg, seed=5)
    hf_cfg = tr.Qwen2Config(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                            intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_layers,
                            num_attention_heads=cfg.num_q_heads, num_key_value_heads=cfg.num_kv_heads,
                            head_dim=cfg.head_dim, rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta,
                            tie_word_embeddings=True, max_position_embeddings=cfg.max_pos,
                            attn_implementation="eager")
    model = tr.Qwen2ForCausalLM(hf_cfg).float().eval()
    sd = {}
    for name, bits in W.items():
        sd[name] = torch.from_numpy(ref.bf16_bits_to_f32(bits).copy())
    shapes = {k: v.shape for k, v in model.state_dict().items()}
    sd = {k: v.reshape(shapes[k]) for k, v in sd.items() if k in shapes}
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not [m for m in missing if "rotary" not in m], missing
    prompt = synth.prompt_tokens(cfg, 9, seed=5)
    with torch.no_grad():
        hf_logits = model(torch.tensor([prompt])).logits[0, -1].numpy()
    o = ref.OracleLeader(cfg, ref.Weights(W))
    row = o.forward(o.embed_tokens(prompt), len(prompt), 0)
    _, logits = o.sample_last(row)
    assert_close(logits, hf_logits, rtol=1e-3, atol=2e-4, what="oracle vs transformers Qwen2")


# ---- golden fixtures ----------------------------------------------------------------------------
GOLDEN = os.path.join(ROOT, "tests", "golden", "tiny_decode.npz")


def golden():
    """The committed fixture and its config (tests/golden/make_golden.py)."""
    if not os.path.exists(GOLDEN):
        pytest.skip("golden fixture not generated")
    return np.load(GOLDEN), synth.tiny_config(tie_word_embeddings=False)


def test_golden_fixture():
    """The oracle reproduces the committed greedy decode (tokens and logits)."""
    g, cfg = golden()
    W = synth.synthetic_weights(cfg, seed=int(g["seed"]))
    # weights fingerprint: the generator is deterministic
    assert int(np.sum(W["model.layers.0.self_attn.q_proj.weight"].astype(np.uint64))) == int(g["q0_checksum"])
    o = ref.OracleLeader(cfg, ref.Weights(W))
    toks, logits = o.generate([int(t) for t in g["prompt"]], int(g["steps"]), keep_logits=True)
    assert toks == [int(t) for t in g["tokens"]]
    assert_close(np.stack(logits), g["logits"], rtol=1e-5, atol=1e-6, what="golden logits")


def test_golden_fixture_agrees_with_transformers():
    """The fixture's logits match transformers' Qwen2ForCausalLM (an independent
    implementation) on the same teacher-forced token stream."""
    g, _ = golden()
    assert_close(g["logits"], g["hf_logits"], rtol=1e-3, atol=1e-4, what="oracle vs transformers (golden)")
    assert [int(t) for t in g["tokens"]] == [int(np.argmax(r)) for r in g["hf_logits"]]
