"""The C-ABI library loads on a machine without a GPU, exports every entry point
include/dllm.h declares, and refuses to run without an sm_100 device."""
import ctypes as C
import os
import re
import subprocess

import pytest

from helpers import ROOT


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "dllm.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dllm_[a-z0-9_]+)\s*\(", src)))


def test_header_symbols_exported(dllm):
    lib = dllm.load_library()
    names = declared_symbols()
    assert len(names) >= 50
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", dllm.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\b(dllm_[a-z0-9_]+)\b", out))
    assert set(names) == exported, (set(names) ^ exported)


def test_ctypes_signatures_cover_header(dllm):
    from importlib import import_module
    sig = import_module("distributed-llm1_b200._lib").SIGNATURES
    assert set(declared_symbols()) == set(sig)


def test_library_built_for_sm100a(dllm):
    out = subprocess.run(["cuobjdump", "--list-elf", dllm.LIB_PATH], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout


def test_config_defaults_match_reference(dllm):
    lib = dllm.load_library()
    cfg = dllm._lib.dllm_config()
    lib.dllm_config_default(C.byref(cfg))
    # constants.js:10-23
    assert (cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim,
            cfg.intermediate_size, cfg.eos_token_id, cfg.max_pos) == (151936, 1536, 28, 12, 2, 128, 8960, 151645, 4096)
    assert abs(cfg.rope_theta - 1e6) < 1 and abs(cfg.rms_norm_eps - 1e-6) < 1e-12 and cfg.tie_word_embeddings == 1
    c2 = dllm.CFG.to_c()
    assert bytes(c2) == bytes(cfg)


def test_status_strings(dllm):
    lib = dllm.load_library()
    assert lib.dllm_status_string(0) == b"ok"
    assert lib.dllm_status_string(3) == b"KV cache overflow"


def test_init_fails_loudly_without_sm100(dllm):
    """No CPU fallback: without a B200 the context cannot be created."""
    try:
        import torch
        if torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] >= 10:
            pytest.skip("an sm_100 GPU is present")
    except ImportError:
        pass
    with pytest.raises(dllm.DllmError):
        dllm.initKernels(0)


def test_bad_config_rejected(dllm):
    lib = dllm.load_library()
    h = C.c_void_p()
    bad = dllm.CFG.with_(head_dim=96).to_c()
    assert lib.dllm_init_kernels(0, C.byref(bad), C.byref(h)) != 0
    assert not h.value
