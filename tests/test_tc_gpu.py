"""The tcgen05 tensor-core matmul (MATMUL, kernels.js:26-44, for n > 1 rows) against
the oracle's matmul (oracle/ref_forward.cpp: fp32, k ascending in steps of 4).

Rows are the sequences of a wide micro-batch or the tokens of a prefill chunk:
n in {16, 30, 64, 128, 200} at the kernel-sweep shapes [K, N] = [896, 1152],
[1536, 8960], [3584, 18944], [18944, 3584] and the LM head [3584, 152064]
(fewer rows there, so the oracle finishes in seconds). The activations are
fp32 as in the reference; the kernel feeds them to the bf16 tensor cores as a
hi + lo pair, so the tolerance here (1e-3 of the output scale) is far tighter
than what a plain bf16 cast of the activations would meet (~5e-3 at K = 18944),
and tighter than the north_star bar (2e-2). The CUDA-core matvec is checked
against the same rows for agreement between the two paths."""
import ctypes as C
import os

import numpy as np
import pytest

from helpers import assert_close, ref_lib

pytestmark = pytest.mark.gpu

SHAPES = [(896, 1152), (1536, 8960), (3584, 18944), (18944, 3584)]


@pytest.fixture(scope="module")
def ctx7(dllm):
    cfg = dllm.PRESETS["qwen2.5-7b"].with_(num_layers=1)
    ctx = dllm.initKernels(0, cfg)
    yield ctx
    ctx.close()


def _oracle(x, wbits, n, K, N):
    lib = ref_lib()
    lib.ref_set_threads(os.cpu_count() or 1)
    out = np.zeros(n * N, np.float32)
    F, U16 = C.POINTER(C.c_float), C.POINTER(C.c_uint16)
    lib.ref_matmul(x.ctypes.data_as(F), wbits.ctypes.data_as(U16), out.ctypes.data_as(F), n, K, N)
    return out


def _case(ctx, n, K, N, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n * K, dtype=np.float32)
    w = ctx.createBf16(K * N, "w")
    ctx.fillNormalBf16(w, seed, 0.02)
    wbits = ctx.readBf16(w)
    xb = ctx.createF32(x.size)
    ctx.writeF32(xb, x)
    return x, w, wbits, xb


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("n", [16, 30, 64])
def test_tc_matmul_sweep_shapes(ctx7, K, N, n):
    x, w, wbits, xb = _case(ctx7, n, K, N, seed=K + N + n)
    got = ctx7.readF32(ctx7.matmul(xb, w, n, K, N), n * N)
    want = _oracle(x, wbits, n, K, N)
    scale = float(np.max(np.abs(want)))
    assert_close(got, want, rtol=1e-3, atol=1e-3 * scale, what=f"tc matmul n={n} [{K},{N}]")


@pytest.mark.parametrize("n", [16, 24])
def test_tc_matmul_lm_head(ctx7, n):
    K, N = 3584, 152064
    x, w, wbits, xb = _case(ctx7, n, K, N, seed=n)
    got = ctx7.readF32(ctx7.matmul(xb, w, n, K, N), n * N)
    want = _oracle(x, wbits, n, K, N)
    scale = float(np.max(np.abs(want)))
    assert_close(got, want, rtol=1e-3, atol=1e-3 * scale, what=f"tc LM head n={n}")
    # greedy tokens per row agree with the oracle's first-max scan
    assert [int(np.argmax(r)) for r in got.reshape(n, N)] == [int(np.argmax(r)) for r in want.reshape(n, N)]


@pytest.mark.parametrize("n", [128, 200])
def test_tc_matmul_many_rows(ctx7, n):
    """128 rows fill one launch (256 MMA columns); 200 rows take two launches."""
    K, N = 1536, 1152
    x, w, wbits, xb = _case(ctx7, n, K, N, seed=n)
    got = ctx7.readF32(ctx7.matmul(xb, w, n, K, N), n * N)
    want = _oracle(x, wbits, n, K, N)
    scale = float(np.max(np.abs(want)))
    assert_close(got, want, rtol=1e-3, atol=1e-3 * scale, what=f"tc matmul n={n}")


def test_tc_and_cuda_core_paths_agree(ctx7):
    K, N, n = 3584, 4096, 16
    x, w, wbits, xb = _case(ctx7, n, K, N, seed=5)
    tc = ctx7.readF32(ctx7.matmul(xb, w, n, K, N), n * N)
    ctx7.set_tensor_core_rows(0)
    try:
        cc = ctx7.readF32(ctx7.matmul(xb, w, n, K, N), n * N)
    finally:
        ctx7.set_tensor_core_rows(8)
    scale = float(np.max(np.abs(cc)))
    assert_close(tc, cc, rtol=1e-3, atol=1e-4 * scale, what="tensor-core vs CUDA-core matmul")


def test_tc_rows_setting_validated(ctx7, dllm):
    with pytest.raises(dllm.DllmError):
        ctx7.set_tensor_core_rows(1)
    with pytest.raises(dllm.DllmError):
        ctx7.set_tensor_core_rows(129)
