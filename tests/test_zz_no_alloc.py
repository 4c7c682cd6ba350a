"""dllm_attention_noalloc: the op-level attention for callers that must not
allocate device memory (a host that owns the HBM budget through its own pool,
or a latency-critical loop that cannot afford cudaMalloc/cudaFree). The caller
passes device pointers; the entry point's scratch is a static device array.

Checked through the C ABI against the allocating entry point (dllm_attention)
on two calls in a row, the second with a different shape so that stale scratch
contents (ticket counters, partials) would show. This file is collected last."""
import ctypes as C

import numpy as np
import pytest

from helpers import assert_close, model_config, oracle_cfg

pytestmark = pytest.mark.gpu

NQ, KVH, HD, MAX_POS = 12, 2, 128, 4096


def test_no_alloc_attention_matches_allocating_entry_point(dllm):
    import torch
    lib = dllm.load_library()
    ctx = dllm.initKernels(0, model_config(dllm, oracle_cfg("1.5b")))
    rng = np.random.default_rng(11)
    kc = rng.standard_normal((MAX_POS, KVH * HD), dtype=np.float32)
    vc = rng.standard_normal((MAX_POS, KVH * HD), dtype=np.float32)
    kb, vb = ctx.createF32(kc.size), ctx.createF32(vc.size)
    ctx.writeF32(kb, kc)
    ctx.writeF32(vb, vc)
    kt = torch.from_numpy(kc).cuda()
    vt = torch.from_numpy(vc).cuda()
    for t0, n in ((1500, 5), (37, 1)):
        q = rng.standard_normal(n * NQ * HD, dtype=np.float32)
        qb = ctx.createF32(q.size)
        ctx.writeF32(qb, q)
        want = ctx.readF32(ctx.attention(qb, kb, vb, t0, n), n * NQ * HD)
        qt = torch.from_numpy(q).cuda()
        out = torch.full((n * NQ * HD,), float("nan"), dtype=torch.float32, device="cuda")
        st = torch.cuda.current_stream()
        rc = lib.dllm_attention_noalloc(qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), out.data_ptr(), t0, n, NQ, KVH,
                                        HD, MAX_POS, C.c_void_p(st.cuda_stream))
        assert rc == 0
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), want, rtol=1e-5, atol=1e-6, what=f"noalloc attention t0={t0} n={n}")
    ctx.close()


def test_no_alloc_attention_rejects_out_of_limit(dllm):
    import torch
    lib = dllm.load_library()
    buf = torch.zeros(128 * NQ * HD, dtype=torch.float32, device="cuda")
    p = buf.data_ptr()
    # 65 rows exceed the static scratch's row limit
    assert lib.dllm_attention_noalloc(p, p, p, p, 0, 65, NQ, KVH, HD, 128, None) == dllm._lib.DLLM_ERANGE
    # bad shapes are rejected before any launch
    assert lib.dllm_attention_noalloc(p, p, p, p, 0, 1, NQ, KVH, 96, 128, None) == dllm._lib.DLLM_EINVAL
    assert lib.dllm_attention_noalloc(p, p, p, p, 127, 2, NQ, KVH, HD, 128, None) == dllm._lib.DLLM_EINVAL
    assert lib.dllm_attention_noalloc(None, p, p, p, 0, 1, NQ, KVH, HD, 128, None) == dllm._lib.DLLM_EINVAL
