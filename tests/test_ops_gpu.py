"""Op-level parity: each ctx op (one sm_100a kernel per reference shader) against
the oracle, on the reference self-test's shapes and inputs (test.js:41-196:
mulberry32 seeds 42/7/11+n/99, 1.5B dims) with synthetic weights in place of the
HF checkpoint, plus the isolated kernel sweep shapes. Tolerances are fp32
reduction-order bounds, tighter than test.js's (1e-2 / 1e-3 / 1e-1)."""
import numpy as np
import pytest

import ref_forward as ref
from helpers import assert_close, mulberry_array, oracle_cfg, model_config

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(1234)


def bf16_normal(n, std=0.02, seed=0):
    r = np.random.default_rng(seed)
    return ref.f32_to_bf16_bits(r.standard_normal(n, dtype=np.float32) * np.float32(std))


@pytest.fixture(scope="module")
def ctx15(dllm):
    """Context with the reference's 1.5B dims (kernels.js:173)."""
    cfg = oracle_cfg("1.5b")
    ctx = dllm.initKernels(0, model_config(dllm, cfg))
    yield ctx
    ctx.close()


@pytest.fixture(scope="module")
def ctx7(dllm):
    cfg = oracle_cfg("7b", max_pos=32768 + 64)
    ctx = dllm.initKernels(0, model_config(dllm, cfg, kv_dtype="f32"))
    yield ctx
    ctx.close()


def run_matmul(ctx, x, wbits, n, din, dout):
    xb = ctx.createF32(n * din)
    ctx.writeF32(xb, x)
    wb = ctx.loadWeightBf16(wbits)
    return ctx.readF32(ctx.matmul(xb, wb, n, din, dout), n * dout)


# ---- test.js TEST 1 / TEST 2 -----------------------------------------------------------
def test_matmul_n1_q_proj(ctx15):
    x = mulberry_array(42, 1536, 0.2, -0.1)
    w = bf16_normal(1536 * 1536, seed=1)
    got = run_matmul(ctx15, x, w, 1, 1536, 1536)
    want = ref.matmul(x, w, 1, 1536, 1536).reshape(-1)
    assert_close(got, want, rtol=1e-4, atol=2e-6, what="matmul n=1")


def test_matmul_n30_prefill(ctx15):
    n = 30
    x = mulberry_array(7, n * 1536, 0.2, -0.1)
    w = bf16_normal(1536 * 1536, seed=2)
    got = run_matmul(ctx15, x, w, n, 1536, 1536)
    want = ref.matmul(x, w, n, 1536, 1536).reshape(-1)
    assert_close(got, want, rtol=1e-4, atol=2e-6, what="matmul n=30")


@pytest.mark.parametrize("din,dout", [(896, 1152), (1536, 8960), (3584, 18944), (18944, 3584), (8, 3), (24, 4099)])
@pytest.mark.parametrize("n", [1, 3, 8])
def test_matmul_sweep(ctx15, din, dout, n):
    """Kernel-sweep shapes (N(0,1) activations, N(0,0.02) bf16 weights) and ragged edges."""
    x = RNG.standard_normal(n * din, dtype=np.float32)
    w = bf16_normal(din * dout, seed=din + dout)
    got = run_matmul(ctx15, x, w, n, din, dout)
    want = ref.matmul(x, w, n, din, dout).reshape(-1)
    scale = np.sqrt(din) * 0.02
    assert_close(got, want, rtol=1e-4, atol=1e-5 * scale, what=f"matmul {n}x{din}->{dout}")


def test_matmul_lm_head_shape(ctx15):
    din, dout = 3584, 152064
    x = RNG.standard_normal(din, dtype=np.float32)
    w = bf16_normal(din * dout, seed=7)
    got = run_matmul(ctx15, x, w, 1, din, dout)
    want = ref.matmul(x, w, 1, din, dout).reshape(-1)
    assert_close(got, want, rtol=1e-4, atol=2e-5, what="matmul lm head")


def test_matmul_rejects_bad_sizes(ctx15, dllm):
    xb = ctx15.createF32(16)
    wb = ctx15.loadWeightBf16(np.zeros(16 * 4, np.uint16))
    with pytest.raises(dllm.DllmError):
        ctx15.matmul(xb, wb, 1, 12, 4)  # din not a multiple of 8
    with pytest.raises(dllm.DllmError):
        ctx15.matmul(xb, wb, 2, 16, 4)  # x too small


# ---- test.js TEST 3 ----------------------------------------------------------------------
@pytest.mark.parametrize("n", [1, 30])
def test_rmsnorm(ctx15, n):
    x = mulberry_array(11 + n, n * 1536, 0.3, -0.15)
    g = bf16_normal(1536, std=0.5, seed=3)
    xb = ctx15.createF32(n * 1536)
    ctx15.writeF32(xb, x)
    gb = ctx15.loadWeightBf16(g)
    got = ctx15.readF32(ctx15.rmsnorm(xb, gb, n), n * 1536)
    want = ref.rmsnorm(x, g, n, 1536).reshape(-1)
    assert_close(got, want, rtol=2e-6, atol=1e-6, what=f"rmsnorm n={n}")


# ---- RoPE --------------------------------------------------------------------------------
@pytest.mark.parametrize("pos0,n", [(0, 1), (17, 1), (5, 7), (8191, 2), (32767, 1)])
def test_rope(ctx15, pos0, n):
    for heads, fn in ((12, "ropeQ"), (2, "ropeK")):
        x = RNG.standard_normal(n * heads * 128, dtype=np.float32)
        xb = ctx15.createF32(x.size)
        ctx15.writeF32(xb, x)
        getattr(ctx15, fn)(xb, pos0, n)
        got = ctx15.readF32(xb, x.size)
        want = ref.rope(x, n, heads, 128, pos0, 1e6).reshape(-1)
        # angles are bit-identical (same fp32 freq table and product); only sin/cos differ by ulps
        assert_close(got, want, rtol=1e-5, atol=1e-5, what=f"{fn} pos0={pos0}")


def test_rope_pos0_identity(ctx15):
    x = RNG.standard_normal(12 * 128, dtype=np.float32)
    xb = ctx15.createF32(x.size)
    ctx15.writeF32(xb, x)
    ctx15.ropeQ(xb, 0, 1)
    np.testing.assert_array_equal(ctx15.readF32(xb, x.size), x)


# ---- test.js TEST 4 ----------------------------------------------------------------------
def reference_test4_inputs():
    """q, K, V exactly as test.js:90-97 draws them (mulberry32(99))."""
    r = __import__("helpers").mulberry32(99)
    q = np.array([r() * 2 - 1 for _ in range(12 * 128)], np.float32)
    kc = np.zeros((4096, 2 * 128), np.float32)
    vc = np.zeros((4096, 2 * 128), np.float32)
    for p in range(4):
        for hv in range(2):
            for e in range(128):
                kc[p, hv * 128 + e] = r() * 2 - 1
                vc[p, hv * 128 + e] = r() * 2 - 1
    return q, kc, vc


@pytest.mark.parametrize("T0", [3, 0, 1, 5, 20])
def test_attention_reference_cases(ctx15, T0):
    q, kc, vc = reference_test4_inputs()
    qb, kb, vb = ctx15.createF32(q.size), ctx15.createF32(kc.size), ctx15.createF32(vc.size)
    ctx15.writeF32(qb, q)
    ctx15.writeF32(kb, kc)
    ctx15.writeF32(vb, vc)
    got = ctx15.readF32(ctx15.attention(qb, kb, vb, T0, 1), 12 * 128)
    want = ref.attention(q, kc, vc, T0, 1, 12, 2, 128).reshape(-1)
    assert_close(got, want, rtol=1e-5, atol=1e-6, what=f"attention T0={T0}")


@pytest.mark.parametrize("T", [1024, 4096, 16384, 32768])
def test_attention_sweep_7b(ctx7, T):
    """GQA decode attention, head_dim 128, 28 Q / 4 KV heads, KV length T."""
    nq, kvh, hd = 28, 4, 128
    q = RNG.standard_normal(nq * hd, dtype=np.float32)
    kc = np.zeros((32768 + 64, kvh * hd), np.float32)
    vc = np.zeros_like(kc)
    kc[:T] = RNG.standard_normal((T, kvh * hd), dtype=np.float32)
    vc[:T] = RNG.standard_normal((T, kvh * hd), dtype=np.float32)
    qb, kb, vb = ctx7.createF32(q.size), ctx7.createF32(kc.size), ctx7.createF32(vc.size)
    ctx7.writeF32(qb, q)
    ctx7.writeF32(kb, kc)
    ctx7.writeF32(vb, vc)
    got = ctx7.readF32(ctx7.attention(qb, kb, vb, T - 1, 1), nq * hd)
    want = ref.attention(q, kc, vc, T - 1, 1, nq, kvh, hd).reshape(-1)
    assert_close(got, want, rtol=1e-4, atol=2e-5, what=f"attention T={T}")


def test_attention_causal_rows(ctx15):
    """n > 1: row t attends to slots [0, T0 + t] (kernels.js:121)."""
    n, T0 = 6, 37
    q = RNG.standard_normal(n * 12 * 128, dtype=np.float32)
    kc = RNG.standard_normal((4096, 256), dtype=np.float32)
    vc = RNG.standard_normal((4096, 256), dtype=np.float32)
    qb, kb, vb = ctx15.createF32(q.size), ctx15.createF32(kc.size), ctx15.createF32(vc.size)
    ctx15.writeF32(qb, q)
    ctx15.writeF32(kb, kc)
    ctx15.writeF32(vb, vc)
    got = ctx15.readF32(ctx15.attention(qb, kb, vb, T0, n), q.size)
    want = ref.attention(q, kc, vc, T0, n, 12, 2, 128).reshape(-1)
    assert_close(got, want, rtol=1e-5, atol=2e-6, what="attention causal rows")


# ---- SILUMUL / ADD / ADDBIAS ----------------------------------------------------------------
def test_elementwise(ctx15):
    n = 8960 * 3 + 5
    a = RNG.standard_normal(n, dtype=np.float32) * 4
    b = RNG.standard_normal(n, dtype=np.float32)
    ab, bb = ctx15.createF32(n), ctx15.createF32(n)
    ctx15.writeF32(ab, a)
    ctx15.writeF32(bb, b)
    assert_close(ctx15.readF32(ctx15.siluMul(ab, bb, n), n), ref.silu_mul(a, b), rtol=2e-6, atol=1e-7, what="silu")
    np.testing.assert_array_equal(ctx15.readF32(ctx15.add(ab, bb, n), n), ref.add(a, b))
    dout = 256
    rows = 7
    bias = bf16_normal(dout, seed=9)
    biasb = ctx15.loadWeightBf16(bias)
    got = ctx15.readF32(ctx15.addBias(ab, biasb, rows, dout), rows * dout)
    np.testing.assert_array_equal(got, ref.add_bias(a[:rows * dout], bias, rows, dout))


# ---- greedy argmax -------------------------------------------------------------------------
def test_argmax_ties_and_nan(ctx15):
    n = 151936
    v = RNG.standard_normal(n, dtype=np.float32)
    top = np.float32(v.max() + 1)
    v[[5000, 90000, 151935]] = top  # ties: lowest index wins (pipeline.js:162 strict '>')
    v[77] = np.nan                  # NaN never wins
    b = ctx15.createF32(n)
    ctx15.writeF32(b, v)
    assert ctx15.argmax(b, n) == 5000 == ref.argmax_first(v)
    v2 = np.full(n, -np.inf, np.float32)
    ctx15.writeF32(b, v2)
    assert ctx15.argmax(b, n) == 0 == ref.argmax_first(v2)
    v3 = np.full(n, np.nan, np.float32)
    ctx15.writeF32(b, v3)
    assert ctx15.argmax(b, n) == 0 == ref.argmax_first(v3)


# ---- buffers ---------------------------------------------------------------------------------
def test_buffers_and_weight_bits(ctx15, dllm):
    with pytest.raises(dllm.DllmError):
        ctx15.createF32(0)  # kernels.js:189
    with pytest.raises(dllm.DllmError):
        ctx15.loadWeightBits(np.zeros(0, np.uint32))  # kernels.js:182
    bits = np.array([0x3F80, 0xBF80, 0x0001, 0x7F80, 0x12345678], np.uint32)  # upper half ignored
    wb = ctx15.loadWeightBits(bits)
    np.testing.assert_array_equal(ctx15.readBf16(wb), (bits & 0xFFFF).astype(np.uint16))
    f = ctx15.createF32(1000)
    x = RNG.standard_normal(1000, dtype=np.float32)
    ctx15.writeF32(f, x)
    np.testing.assert_array_equal(ctx15.readF32(f, 1000), x)
    with pytest.raises(dllm.DllmError):
        ctx15.readF32(f, 1001)


def test_device_fill_matches_distribution(ctx15):
    b = ctx15.createBf16(1 << 20)
    ctx15.fillNormalBf16(b, seed=5, std=0.02)
    v = ref.bf16_bits_to_f32(ctx15.readBf16(b))
    assert abs(float(v.mean())) < 1e-3 and abs(float(v.std()) - 0.02) < 5e-4
