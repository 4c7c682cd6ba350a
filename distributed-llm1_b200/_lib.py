"""ctypes binding of libdllm.so (include/dllm.h).

The library is loaded from this package directory (built in-tree by
csrc/Makefile). There is no fallback: if the shared object is missing or a
call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdllm.so")

DLLM_OK, DLLM_EINVAL, DLLM_ENOMEM, DLLM_ERANGE, DLLM_ETIMEOUT, DLLM_ECUDA, DLLM_ENOTFOUND, DLLM_EDEVICE = range(8)
DLLM_KV_F32, DLLM_KV_BF16 = 0, 1


class DllmError(RuntimeError):
    """A non-zero status from libdllm (the JS shim would `throw new Error(msg)`)."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"{msg} [{_status_name(status)}]")
        self.status = status


class KvOverflowError(DllmError, IndexError):
    pass


def _status_name(s: int) -> str:
    return {0: "ok", 1: "EINVAL", 2: "ENOMEM", 3: "ERANGE", 4: "ETIMEOUT", 5: "ECUDA", 6: "ENOTFOUND",
            7: "EDEVICE"}.get(s, str(s))


class dllm_config(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int32), ("hidden_size", C.c_int32), ("num_layers", C.c_int32),
        ("num_q_heads", C.c_int32), ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32),
        ("intermediate_size", C.c_int32), ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float),
        ("tie_word_embeddings", C.c_int32), ("eos_token_id", C.c_int32), ("max_pos", C.c_int32),
        ("kv_dtype", C.c_int32), ("kv_page_size", C.c_int32), ("max_seqs", C.c_int32),
    ]


P = C.c_void_p
I32P = C.POINTER(C.c_int32)
F32P = C.POINTER(C.c_float)
U16P = C.POINTER(C.c_uint16)
U32P = C.POINTER(C.c_uint32)
PP = C.POINTER(C.c_void_p)

# name: (restype, argtypes)
SIGNATURES = {
    "dllm_version": (C.c_char_p, []),
    "dllm_status_string": (C.c_char_p, [C.c_int]),
    "dllm_config_default": (None, [C.POINTER(dllm_config)]),
    "dllm_init_kernels": (C.c_int, [C.c_int, C.POINTER(dllm_config), PP]),
    "dllm_ctx_destroy": (None, [P]),
    "dllm_last_error": (C.c_char_p, [P]),
    "dllm_ctx_get_config": (C.c_int, [P, C.POINTER(dllm_config)]),
    "dllm_ctx_set_stream": (C.c_int, [P, P]),
    "dllm_ctx_synchronize": (C.c_int, [P, C.c_int]),
    "dllm_ctx_launch_count": (C.c_uint64, [P]),
    "dllm_ctx_set_tensor_core_rows": (C.c_int, [P, C.c_int]),
    "dllm_load_weight_bits": (C.c_int, [P, U32P, C.c_size_t, C.c_char_p, PP]),
    "dllm_load_weight_bf16": (C.c_int, [P, U16P, C.c_size_t, C.c_char_p, PP]),
    "dllm_create_f32": (C.c_int, [P, C.c_size_t, C.c_char_p, PP]),
    "dllm_create_bf16": (C.c_int, [P, C.c_size_t, C.c_char_p, PP]),
    "dllm_write_f32": (C.c_int, [P, P, F32P, C.c_size_t]),
    "dllm_read_f32": (C.c_int, [P, P, F32P, C.c_size_t, C.c_char_p]),
    "dllm_read_bf16": (C.c_int, [P, P, U16P, C.c_size_t]),
    "dllm_buf_free": (None, [P]),
    "dllm_buf_bytes": (C.c_size_t, [P]),
    "dllm_buf_device_ptr": (P, [P]),
    "dllm_fill_normal_bf16": (C.c_int, [P, P, C.c_uint64, C.c_float]),
    "dllm_fill_const_bf16": (C.c_int, [P, P, C.c_float]),
    "dllm_matmul": (C.c_int, [P, P, P, C.c_int, C.c_int, C.c_int, PP]),
    "dllm_rmsnorm": (C.c_int, [P, P, P, C.c_int, PP]),
    "dllm_rope_q": (C.c_int, [P, P, C.c_int, C.c_int]),
    "dllm_rope_k": (C.c_int, [P, P, C.c_int, C.c_int]),
    "dllm_attention": (C.c_int, [P, P, P, P, C.c_int, C.c_int, PP]),
    "dllm_silu_mul": (C.c_int, [P, P, P, C.c_int, PP]),
    "dllm_add": (C.c_int, [P, P, P, C.c_int, PP]),
    "dllm_add_bias": (C.c_int, [P, P, P, C.c_int, C.c_int, PP]),
    "dllm_argmax": (C.c_int, [P, P, C.c_int, I32P]),
    "dllm_stage_create": (C.c_int, [P, C.c_int, C.c_int, PP]),
    "dllm_stage_destroy": (None, [P]),
    "dllm_stage_set_weight": (C.c_int, [P, C.c_char_p, P]),
    "dllm_stage_reset": (C.c_int, [P]),
    "dllm_stage_get_t0": (C.c_int, [P, C.c_int]),
    "dllm_stage_set_t0": (C.c_int, [P, C.c_int, C.c_int]),
    "dllm_stage_forward": (C.c_int, [P, F32P, C.c_int, C.c_int, PP]),
    "dllm_stage_forward_rows": (C.c_int, [P, P, C.c_int, I32P, P, P]),
    "dllm_stage_append_kv": (C.c_int, [P, C.c_int, P, P, C.c_int]),
    "dllm_stage_read_kv": (C.c_int, [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, F32P]),
    "dllm_stage_fill_kv_random": (C.c_int, [P, C.c_int, C.c_int, C.c_uint64]),
    "dllm_stage_set_page_table": (C.c_int, [P, C.c_int, I32P, C.c_int]),
    "dllm_stage_pages_per_seq": (C.c_int, [P]),
    "dllm_stage_read_workspace": (C.c_int, [P, C.c_int, C.c_int, F32P]),
    "dllm_stage_set_trace": (C.c_int, [P, C.c_int]),
    "dllm_stage_read_trace": (C.c_int, [P, C.POINTER(C.c_uint64), C.c_int]),
    "dllm_leader_create": (C.c_int, [P, C.c_int, C.c_int, PP]),
    "dllm_leader_destroy": (None, [P]),
    "dllm_leader_stage": (P, [P]),
    "dllm_leader_set_weights": (C.c_int, [P, P, P, P]),
    "dllm_leader_embed_tokens": (C.c_int, [P, I32P, C.c_int, F32P]),
    "dllm_leader_sample_last": (C.c_int, [P, F32P, I32P, F32P]),
    "dllm_leader_forward": (C.c_int, [P, F32P, C.c_int, C.c_int, F32P]),
    "dllm_leader_generate": (C.c_int, [P, I32P, C.c_int, C.c_int, I32P, I32P]),
    "dllm_leader_decode": (C.c_int, [P, C.c_int32, C.c_int, I32P]),
    "dllm_leader_decode_enqueue": (C.c_int, [P, C.c_int32, C.c_int]),
    "dllm_leader_read_tokens": (C.c_int, [P, I32P, C.c_int]),
    "dllm_leader_set_keep_logits": (C.c_int, [P, C.c_int]),
    "dllm_leader_last_logits": (C.c_int, [P, F32P]),
    "dllm_leader_read_logits": (C.c_int, [P, C.c_int, F32P]),
    "dllm_pipeline_create": (C.c_int, [P, C.c_int, C.c_int, C.c_int, C.c_int, PP]),
    "dllm_pipeline_destroy": (None, [P]),
    "dllm_pipeline_handle": (C.c_int, [P, C.POINTER(C.c_uint8)]),
    "dllm_pipeline_connect": (C.c_int, [P, C.POINTER(C.c_uint8)]),
    "dllm_pipeline_set_tokens": (C.c_int, [P, I32P, C.c_int]),
    "dllm_pipeline_run": (C.c_int, [P, C.c_int]),
    "dllm_pipeline_read_tokens": (C.c_int, [P, I32P, C.c_int]),
    "dllm_pipeline_synchronize": (C.c_int, [P, C.c_int]),
    "dllm_pipeline_set_host_tokens": (C.c_int, [P, C.c_int]),
    "dllm_pipeline_run_micro": (C.c_int, [P, C.c_int, I32P, I32P]),
    "dllm_attention_noalloc": (C.c_int, [P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P]),
    "dllm_attention_noalloc_status": (C.c_int, [P, C.c_int, I32P]),
}

_lib = None


def load() -> C.CDLL:
    """Load libdllm.so once and declare every signature. Raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libdllm.so not built at {LIB_PATH}: run `make -C csrc` (the CUDA path has no fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, ctx_handle=None, what: str = ""):
    if status == DLLM_OK:
        return
    lib = load()
    msg = lib.dllm_last_error(ctx_handle).decode() if ctx_handle else lib.dllm_status_string(status).decode()
    if what:
        msg = f"{what}: {msg}"
    if status == DLLM_ERANGE:
        raise KvOverflowError(status, msg)
    raise DllmError(status, msg)


def ptr(a, ctype):
    """ctypes pointer to a contiguous numpy array (None passes NULL)."""
    if a is None:
        return None
    return a.ctypes.data_as(C.POINTER(ctype))
