"""Stage parity (pipeline.js:26-88): the fused persistent stage kernel against the
oracle's Stage.forward, KV slot indexing, paged layout, overflow, micro-batches.

These tests hold the persistent kernel to fp32-tight tolerances, so their
contexts keep every pass on it (tensor-core rows off): an 8+ row prefill would
otherwise take the tensor-core pass, whose hi/lo products move a projection by
~1e-6 relative, which can flip the bf16 rounding of an appended K/V element and
shift a bf16-KV output by ~1e-4. The tensor-core pass has its own oracle tests
(test_wide_gpu.py) at the north_star bar."""
import numpy as np
import pytest

import ref_forward as ref
from helpers import assert_close, get_weights, load_stage_weights, model_config, oracle_cfg

pytestmark = pytest.mark.gpu


def make_stage(dllm, cfg, W, start, end, kv_dtype="f32", max_seqs=1, page=64):
    ctx = dllm.initKernels(0, model_config(dllm, cfg, kv_dtype, max_seqs, page))
    ctx.set_tensor_core_rows(0)
    st = dllm.Stage(ctx, start, end)
    load_stage_weights(ctx, st, W, start, end)
    return ctx, st


@pytest.mark.parametrize("kv_dtype", ["f32", "bf16"])
def test_stage_forward_tiny(dllm, weights_cache, kv_dtype):
    cfg = oracle_cfg("tiny")
    W = get_weights(weights_cache, "tiny", cfg)
    ctx, st = make_stage(dllm, cfg, W, 0, cfg.num_layers, kv_dtype)
    o = ref.OracleStage(cfg, ref.Weights(W), 0, cfg.num_layers, kv_dtype)
    rng = np.random.default_rng(0)
    # prefill 11 rows at posStart 0, then decode rows at arbitrary positions
    for n, pos in ((11, 0), (1, 11), (1, 12), (3, 40), (1, 17)):
        h = (rng.standard_normal(n * cfg.hidden_size, dtype=np.float32) * 0.05)
        got = ctx.readF32(st.forward(h, n, pos), n * cfg.hidden_size)
        want = o.forward(h, n, pos).reshape(-1)
        assert_close(got, want, rtol=2e-4, atol=2e-5, what=f"stage n={n} pos={pos} {kv_dtype}")
        assert st.T0 == o.T0
    # every KV slot written so far matches the oracle cache
    for L in range(cfg.num_layers):
        for which, key in ((st.kv[L].k, "k"), (st.kv[L].v, "v")):
            assert_close(which.read(0, st.T0), o.kv[L][key][:o.T0], rtol=1e-3 if kv_dtype == "bf16" else 2e-4,
                         atol=1e-4, what=f"kv[{L}].{key}")


def test_layer0_reference_case(dllm, weights_cache):
    """test.js TEST 5: one layer, n=1, posStart=17, T0=0, mulberry32(42) input (1.5B dims)."""
    from helpers import mulberry_array
    import synth
    cfg = oracle_cfg("1.5b", num_layers=1)
    key = ("1.5b-layer0",)
    if key not in weights_cache:
        weights_cache[key] = synth.synthetic_weights(cfg, seed=0, head=False)
    W = weights_cache[key]
    ctx, st = make_stage(dllm, cfg, W, 0, 1)
    x = mulberry_array(42, 1536, 0.2, -0.1)
    got = ctx.readF32(st.forward(x, 1, 17), 1536)
    want = ref.OracleStage(cfg, ref.Weights(W), 0, 1).forward(x, 1, 17).reshape(-1)
    assert_close(got, want, rtol=1e-4, atol=1e-5, what="layer0 n=1 pos=17")


def test_stage_multilayer_05b(dllm, weights_cache):
    cfg = oracle_cfg("0.5b", max_pos=256)
    W = get_weights(weights_cache, "0.5b", cfg)
    ctx, st = make_stage(dllm, cfg, W, 3, 9)
    o = ref.OracleStage(cfg, ref.Weights(W), 3, 9)
    rng = np.random.default_rng(1)
    for n, pos in ((9, 0), (1, 9), (1, 10)):
        h = rng.standard_normal(n * cfg.hidden_size, dtype=np.float32) * 0.05
        got = ctx.readF32(st.forward(h, n, pos), n * cfg.hidden_size)
        assert_close(got, o.forward(h, n, pos).reshape(-1), rtol=5e-4, atol=5e-5, what=f"0.5b layers 3..9 n={n}")


@pytest.mark.parametrize("kv_dtype", ["f32", "bf16"])
def test_kv_slot_indexing_paged(dllm, weights_cache, kv_dtype):
    """appendKv rows land in slots T0..T0+n-1 (pipeline.js:80-87) through a
    permuted page table; read back bit-exact (bf16: exactly the RNE rounding)."""
    cfg = oracle_cfg("tiny", max_pos=256)
    W = get_weights(weights_cache, "tiny", cfg)
    ctx, st = make_stage(dllm, cfg, W, 0, cfg.num_layers, kv_dtype, max_seqs=2, page=32)
    pps = st.pages_per_seq()
    perm = np.random.default_rng(3).permutation(2 * pps).astype(np.int32)
    st.set_page_table(0, perm[:pps])
    st.set_page_table(1, perm[pps:])
    row = cfg.num_kv_heads * cfg.head_dim
    rng = np.random.default_rng(4)
    expect = np.zeros((cfg.max_pos, row), np.float32)
    for T0, n in ((0, 5), (5, 40), (45, 1), (100, 60)):
        st.T0 = T0
        kk = rng.standard_normal(n * row, dtype=np.float32)
        vv = rng.standard_normal(n * row, dtype=np.float32)
        kb, vb = ctx.createF32(kk.size), ctx.createF32(vv.size)
        ctx.writeF32(kb, kk)
        ctx.writeF32(vb, vv)
        st.appendKv(1, kb, vb, n)
        assert st.T0 == T0  # appendKv itself does not advance T0
        want = kk.reshape(n, row) if kv_dtype == "f32" else ref.bf16_round(kk).reshape(n, row)
        expect[T0:T0 + n] = want
        np.testing.assert_array_equal(st.kv[1].k.read(T0, n), want)
    np.testing.assert_array_equal(st.kv[1].k.read(0, 160), expect[:160])


def test_kv_overflow_raises(dllm, weights_cache):
    cfg = oracle_cfg("tiny", max_pos=64)
    W = get_weights(weights_cache, "tiny", cfg)
    ctx, st = make_stage(dllm, cfg, W, 0, cfg.num_layers)
    h = np.zeros(60 * cfg.hidden_size, np.float32)
    st.forward(h, 60, 0)
    with pytest.raises(dllm.KvOverflowError):
        st.forward(h[:5 * cfg.hidden_size], 5, 60)
    assert st.T0 == 60
    st.reset()
    assert st.T0 == 0


def test_missing_weight_raises(dllm, weights_cache):
    cfg = oracle_cfg("tiny")
    W = {k: v for k, v in get_weights(weights_cache, "tiny", cfg).items() if "layers.1.mlp.up_proj" not in k}
    ctx, st = make_stage(dllm, cfg, W, 0, cfg.num_layers)
    with pytest.raises(dllm.DllmError, match="up_proj"):
        st.forward(np.zeros(cfg.hidden_size, np.float32), 1, 0)


@pytest.mark.parametrize("kv_dtype", ["f32", "bf16"])
def test_microbatch_rows(dllm, weights_cache, kv_dtype):
    """forward_rows: 3 sequences at different T0 in one pass == each sequence alone."""
    import torch
    cfg = oracle_cfg("tiny")
    W = get_weights(weights_cache, "tiny", cfg)
    ctx, st = make_stage(dllm, cfg, W, 0, cfg.num_layers, kv_dtype, max_seqs=4)
    oracles = {s: ref.OracleStage(cfg, ref.Weights(W), 0, cfg.num_layers, kv_dtype) for s in (0, 1, 3)}
    rng = np.random.default_rng(5)
    D = cfg.hidden_size
    # give each sequence a different history through forward_rows with m=1
    hist = {0: 4, 1: 9, 3: 1}
    for s, steps in hist.items():
        for _ in range(steps):
            x = rng.standard_normal(D, dtype=np.float32) * 0.05
            t = torch.from_numpy(x).cuda()
            st.forward_rows(t.data_ptr(), [s])
            ctx.synchronize()
            want = oracles[s].forward(x, 1, oracles[s].T0).reshape(-1)
            assert_close(t.cpu().numpy(), want, rtol=2e-4, atol=2e-5, what=f"seq {s} single")
    for _ in range(3):
        xs = rng.standard_normal((3, D), dtype=np.float32) * 0.05
        t = torch.from_numpy(xs.copy()).cuda()
        st.forward_rows(t.data_ptr(), [3, 0, 1])
        ctx.synchronize()
        got = t.cpu().numpy()
        for i, s in enumerate((3, 0, 1)):
            want = oracles[s].forward(xs[i], 1, oracles[s].T0).reshape(-1)
            assert_close(got[i], want, rtol=2e-4, atol=2e-5, what=f"micro-batch row {i} seq {s}")
    for s in (0, 1, 3):
        assert st.t0_of(s) == oracles[s].T0
