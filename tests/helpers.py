"""Shared test helpers: seeded inputs, oracle <-> device model setup."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

import ref_forward as ref
import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def mulberry32(seed: int):
    """The test PRNG of the reference (test.js:8-10), 32-bit exact."""
    s = [seed & 0xFFFFFFFF]

    def imul(a, b):
        return ((a & 0xFFFFFFFF) * (b & 0xFFFFFFFF)) & 0xFFFFFFFF

    def rnd():
        s[0] = (s[0] + 0x6D2B79F5) & 0xFFFFFFFF
        z = s[0]
        t = imul(z ^ (z >> 15), 1 | z)
        t = ((t + imul(t ^ (t >> 7), 61 | t)) & 0xFFFFFFFF) ^ t
        return ((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296.0

    return rnd


def mulberry_array(seed: int, n: int, scale: float, shift: float) -> np.ndarray:
    r = mulberry32(seed)
    return np.array([r() * scale + shift for _ in range(n)], dtype=np.float32)


def oracle_cfg(name: str, **kw) -> ref.Config:
    from dataclasses import replace
    base = synth.tiny_config() if name == "tiny" else synth.CONFIGS[name]
    return replace(base, **kw)


def get_weights(cache: dict, name: str, cfg: ref.Config, seed: int = 0) -> dict:
    key = (name, cfg.num_layers, cfg.hidden_size, seed)
    if key not in cache:
        cache[key] = synth.synthetic_weights(cfg, seed=seed)
    return cache[key]


def model_config(dllm, cfg: ref.Config, kv_dtype: str = "f32", max_seqs: int = 1, page: int = 64):
    return dllm.ModelConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, num_layers=cfg.num_layers,
                            num_q_heads=cfg.num_q_heads, num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                            intermediate_size=cfg.intermediate_size, rope_theta=cfg.rope_theta,
                            rms_norm_eps=cfg.rms_norm_eps, tie_word_embeddings=cfg.tie_word_embeddings,
                            eos_token_id=cfg.eos_token_id, max_pos=cfg.max_pos, kv_dtype=kv_dtype,
                            kv_page_size=page, max_seqs=max_seqs)


def load_stage_weights(ctx, stage, W: dict, start: int, end: int):
    for name, bits in W.items():
        if name.startswith("model.layers."):
            L = int(name.split(".")[2])
            if start <= L < end:
                stage.W[name] = ctx.loadWeightBf16(bits, name)


def build_leader(dllm, cfg: ref.Config, W: dict, kv_dtype: str = "f32", device: int = 0, max_seqs: int = 1):
    ctx = dllm.initKernels(device, model_config(dllm, cfg, kv_dtype, max_seqs))
    ld = dllm.LeaderPipeline(ctx, (0, cfg.num_layers))
    load_stage_weights(ctx, ld.stage, W, 0, cfg.num_layers)
    ld.loadLeaderWeights(W["model.embed_tokens.weight"], W["model.norm.weight"], W.get("lm_head.weight"))
    return ctx, ld


def max_rel_err(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(1e-30, np.max(np.abs(b))))


def assert_close(got, want, rtol: float, atol: float, what: str = ""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    if bad.any():
        i = int(np.argmax(err - (atol + rtol * np.abs(want))))
        raise AssertionError(f"{what}: {int(bad.sum())}/{bad.size} outside rtol={rtol} atol={atol}; "
                             f"worst idx {i}: got {got.flat[i]!r} want {want.flat[i]!r} (max abs err {err.max():.3e})")


def top2_margin(logits) -> float:
    v = np.sort(np.asarray(logits, np.float64))
    return float(v[-1] - v[-2])


def ref_lib():
    """ctypes handle of the C++ oracle (oracle/_build/libref_forward.so), built on demand."""
    path = os.path.join(ROOT, "oracle", "_build", "libref_forward.so")
    if not os.path.exists(path):
        import subprocess
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True, capture_output=True)
    lib = C.CDLL(path)
    F, U16, I = C.POINTER(C.c_float), C.POINTER(C.c_uint16), C.POINTER(C.c_int)
    lib.ref_matmul.argtypes = [F, U16, F, C.c_int, C.c_int, C.c_int]
    lib.ref_rmsnorm.argtypes = [F, U16, F, C.c_int, C.c_int, C.c_float]
    lib.ref_rope_freqs.argtypes = [C.c_int, C.c_float, F]
    lib.ref_rope.argtypes = [F, C.c_int, C.c_int, C.c_int, C.c_int, F]
    lib.ref_attention.argtypes = [F, F, F, F, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
    lib.ref_silu_mul.argtypes = [F, F, F, C.c_int]
    lib.ref_set_threads.argtypes = [C.c_int]
    lib.ref_model_create.restype = C.c_void_p
    lib.ref_model_create.argtypes = [I, C.c_float, C.c_float, C.POINTER(C.c_void_p), C.c_void_p, C.c_void_p,
                                     C.c_void_p]
    lib.ref_model_destroy.argtypes = [C.c_void_p]
    lib.ref_stage_forward.argtypes = [C.c_void_p, F, C.c_int, C.c_int]
    lib.ref_sample_last.argtypes = [C.c_void_p, F, F]
    lib.ref_generate.argtypes = [C.c_void_p, I, C.c_int, C.c_int, C.c_int, I, F]
    lib.ref_model_fill_kv.argtypes = [C.c_void_p, C.c_int, C.c_uint64]
    lib.ref_model_set_kv.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, F]
    lib.ref_model_set_t0.argtypes = [C.c_void_p, C.c_int]
    lib.ref_model_t0.argtypes = [C.c_void_p]
    lib.ref_embed.argtypes = [C.c_void_p, I, C.c_int, F]
    lib.ref_fill_normal_bf16.argtypes = [U16, C.c_size_t, C.c_uint64, C.c_float]
    return lib


class RefModel:
    """C++ oracle model over numpy-owned bf16 weights (kept alive here)."""

    def __init__(self, lib, cfg: ref.Config, W: dict, start: int = 0, end: int | None = None, kv_bf16: bool = False,
                 head: bool = True):
        end = cfg.num_layers if end is None else end
        self.lib, self.cfg, self.keep = lib, cfg, []
        ptrs = (C.c_void_p * (12 * (end - start)))()
        for li, L in enumerate(range(start, end)):
            for i, suf in enumerate(ref.LAYER_SUFFIXES):
                a = W.get(f"model.layers.{L}.{suf}")
                if a is not None:
                    a = np.ascontiguousarray(a, np.uint16)
                    self.keep.append(a)
                    ptrs[li * 12 + i] = a.ctypes.data
        self.keep.append(ptrs)

        def hp(name):
            a = W.get(name) if head else None
            if a is None:
                return None
            a = np.ascontiguousarray(a, np.uint16)
            self.keep.append(a)
            return a.ctypes.data

        dims = (C.c_int * 10)(cfg.hidden_size, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim,
                              cfg.intermediate_size, cfg.vocab_size, start, end, cfg.max_pos, int(kv_bf16))
        self.keep.append(dims)
        self.h = lib.ref_model_create(dims, cfg.rms_norm_eps, cfg.rope_theta, ptrs, hp("model.embed_tokens.weight"),
                                      hp("model.norm.weight"), hp("lm_head.weight"))

    def forward(self, hidden, n, pos_start):
        h = np.ascontiguousarray(hidden, np.float32).reshape(-1).copy()
        assert self.lib.ref_stage_forward(self.h, h.ctypes.data_as(C.POINTER(C.c_float)), n, pos_start) == 0
        return h

    def set_kv(self, layer: int, which: int, slot0: int, rows):
        a = np.ascontiguousarray(rows, np.float32)
        assert self.lib.ref_model_set_kv(self.h, layer, which, slot0, a.shape[0],
                                         a.ctypes.data_as(C.POINTER(C.c_float))) == 0

    @property
    def T0(self) -> int:
        return int(self.lib.ref_model_t0(self.h))

    @T0.setter
    def T0(self, v: int):
        self.lib.ref_model_set_t0(self.h, int(v))

    def decode_step(self, token: int):
        """One greedy step at position == slot == T0 (the decode branch of
        pipeline.js:262-267): embed, layers, final norm + LM head; returns
        (next token, logits)."""
        t = np.array([token], np.int32)
        h = np.zeros(self.cfg.hidden_size, np.float32)
        self.lib.ref_embed(self.h, t.ctypes.data_as(C.POINTER(C.c_int)), 1, h.ctypes.data_as(C.POINTER(C.c_float)))
        h = self.forward(h, 1, self.T0)
        lg = np.zeros(self.cfg.vocab_size, np.float32)
        tok = self.lib.ref_sample_last(self.h, h.ctypes.data_as(C.POINTER(C.c_float)),
                                       lg.ctypes.data_as(C.POINTER(C.c_float)))
        return int(tok), lg

    def generate(self, tokens, max_new, keep_logits=False):
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(max_new, np.int32)
        lg = np.zeros((max_new, self.cfg.vocab_size), np.float32) if keep_logits else None
        n = self.lib.ref_generate(self.h, t.ctypes.data_as(C.POINTER(C.c_int)), t.size, max_new,
                                  self.cfg.eos_token_id, out.ctypes.data_as(C.POINTER(C.c_int)),
                                  lg.ctypes.data_as(C.POINTER(C.c_float)) if lg is not None else None)
        assert n >= 0
        return [int(x) for x in out[:n]], (lg[:n] if lg is not None else None)

    def close(self):
        if self.h:
            self.lib.ref_model_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()
