"""dllm_attention_noalloc: the op-level attention for callers that must not
allocate device memory (a host that owns the HBM budget through its own pool,
or a latency-critical loop that cannot afford cudaMalloc/cudaFree). The caller
passes device pointers; the entry point's scratch is a static device array.

Checked through the C ABI against the allocating entry point (dllm_attention)
and against the oracle's attention (kernels.js:86-132 restated in C++), on
calls in a row whose shapes differ so that stale scratch contents (ticket
counters, partials) would show, and with the device error word read back after
every call. The shapes reach every path of the entry point: one row, a few rows,
64 rows (the row limit, several work items per CTA and their split waits), head
dims 128 and 64. This file is collected last."""
import ctypes as C

import numpy as np
import pytest

from helpers import assert_close, model_config, oracle_cfg, ref_lib

pytestmark = pytest.mark.gpu

MAX_POS = 4096


def _noalloc(lib, q, kt, vt, t0, n, nq, kvh, hd):
    import torch
    out = torch.full((n * nq * hd,), float("nan"), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream()
    rc = lib.dllm_attention_noalloc(q.data_ptr(), kt.data_ptr(), vt.data_ptr(), out.data_ptr(), t0, n, nq, kvh, hd,
                                    MAX_POS, C.c_void_p(st.cuda_stream))
    assert rc == 0
    code = C.c_int32(-1)
    assert lib.dllm_attention_noalloc_status(C.c_void_p(st.cuda_stream), 15000, C.byref(code)) == 0
    assert code.value == 0  # no device-side error reported
    return out.cpu().numpy()


@pytest.mark.parametrize("model", ["1.5b", "0.5b"])  # head_dim 128 (12/2 heads), 64 (14/2 heads)
def test_no_alloc_attention_matches_allocating_entry_point(dllm, model):
    import torch
    lib = dllm.load_library()
    oc = oracle_cfg(model)
    NQ, KVH, HD = oc.num_q_heads, oc.num_kv_heads, oc.head_dim
    ctx = dllm.initKernels(0, model_config(dllm, oc))
    rlib = ref_lib()
    rng = np.random.default_rng(11)
    kc = rng.standard_normal((MAX_POS, KVH * HD), dtype=np.float32)
    vc = rng.standard_normal((MAX_POS, KVH * HD), dtype=np.float32)
    kb, vb = ctx.createF32(kc.size), ctx.createF32(vc.size)
    ctx.writeF32(kb, kc)
    ctx.writeF32(vb, vc)
    kt = torch.from_numpy(kc).cuda()
    vt = torch.from_numpy(vc).cuda()
    F = C.POINTER(C.c_float)
    # two calls in a row of each shape: the second sees the first's scratch contents
    for t0, n in ((1500, 5), (1500, 5), (37, 1), (3000, 64), (3000, 64), (0, 1)):
        q = rng.standard_normal(n * NQ * HD, dtype=np.float32)
        qb = ctx.createF32(q.size)
        ctx.writeF32(qb, q)
        want = ctx.readF32(ctx.attention(qb, kb, vb, t0, n), n * NQ * HD)
        got = _noalloc(lib, torch.from_numpy(q).cuda(), kt, vt, t0, n, NQ, KVH, HD)
        assert_close(got, want, rtol=1e-5, atol=1e-6, what=f"noalloc vs dllm_attention t0={t0} n={n}")
        ref = np.zeros(n * NQ * HD, np.float32)
        rlib.ref_attention(q.ctypes.data_as(F), kc.ctypes.data_as(F), vc.ctypes.data_as(F), ref.ctypes.data_as(F),
                           t0, n, NQ, KVH, HD)
        assert_close(got, ref, rtol=1e-4, atol=1e-5, what=f"noalloc vs oracle t0={t0} n={n}")
    ctx.close()


def test_no_alloc_attention_rejects_out_of_limit(dllm):
    import torch
    lib = dllm.load_library()
    NQ, KVH, HD = 12, 2, 128
    buf = torch.zeros(128 * NQ * HD, dtype=torch.float32, device="cuda")
    p = buf.data_ptr()
    # 65 rows exceed the static scratch's row limit
    assert lib.dllm_attention_noalloc(p, p, p, p, 0, 65, NQ, KVH, HD, 128, None) == dllm._lib.DLLM_ERANGE
    # bad shapes are rejected before any launch
    assert lib.dllm_attention_noalloc(p, p, p, p, 0, 1, NQ, KVH, 96, 128, None) == dllm._lib.DLLM_EINVAL
    assert lib.dllm_attention_noalloc(p, p, p, p, 127, 2, NQ, KVH, HD, 128, None) == dllm._lib.DLLM_EINVAL
    assert lib.dllm_attention_noalloc(None, p, p, p, 0, 1, NQ, KVH, HD, 128, None) == dllm._lib.DLLM_EINVAL
