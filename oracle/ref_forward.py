"""Oracle for the Qwen2.5 decode path — TEST INFRASTRUCTURE ONLY.

A CPU restatement, in numpy fp32, of the reference's decode path:
  * the WGSL shaders of kernels.js (MATMUL :26-44, RMSNORM :46-63, ROPE :66-83,
    ATTENTION :86-132, SILUMUL :134-145, ADDBIAS :148-159, ADD :161-171),
  * the orchestration of pipeline.js (Stage.forward :48-78, appendKv :80-87,
    sampleLast :141-174, generate :255-281, assignLayers :6-23),
  * the bf16 weight helpers of weights.js (:144-164).
Model dims are parameters (the reference hard-codes Qwen2.5-1.5B).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this module, and only as the checker; the product path never calls it.

Parity status: UNPINNED. The reference is JavaScript + WebGPU. Neither machine
has a JS engine (node/deno/bun/qjs absent) or a WebGPU adapter, its weights and
tokenizer come from the network, and its only known-answer tests (test.js:41-196)
need the real HF checkpoint, which is absent. No reference output exists to pin
this restatement to. It is cross-checked against an independent implementation
(transformers' Qwen2ForCausalLM, tests/test_oracle.py) and against the C
restatement in ref_forward.cpp (reference loop order).

Numerics: fp32 everywhere as in the shaders; transcendentals (exp2, cos, sin,
exp, sqrt) are evaluated in float64 and rounded to fp32 where the reference uses
them on fp32 values, which is the correctly rounded answer the WGSL builtins
approximate. The optional bf16 KV mode rounds appended K/V rows to bf16 (round
to nearest even), the storage rounding of the B200 build's bf16 cache; the
reference itself stores fp32.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

F32 = np.float32


# ---- weights.js:144-164 ------------------------------------------------------------
def bf16_bytes_to_f32_bits(b: bytes | np.ndarray) -> np.ndarray:
    """bf16 bytes -> Uint32Array of raw bf16 bits, one per element (weights.js:144-150)."""
    a = np.frombuffer(bytes(b), dtype="<u2") if not isinstance(b, np.ndarray) else b.view("<u2")
    return a.astype(np.uint32)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """u32/u16 raw bf16 bits -> float32 via bits << 16 (weights.js:153-164)."""
    b = np.asarray(bits).astype(np.uint32) & np.uint32(0xFFFF)
    return (b << np.uint32(16)).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even; NaN -> quiet NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    # finite values cannot overflow: u <= 0xFF7FFFFF, + 0x8000 < 2^32
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ---- shaders (kernels.js) ----------------------------------------------------------------
def matmul(x: np.ndarray, w: np.ndarray, n: int, din: int, dout: int) -> np.ndarray:
    """MATMUL (kernels.js:26-44): out[t,j] = sum_k X[t,k] * bf16(W[j,k]), fp32."""
    W = w if w.dtype == np.float32 else bf16_bits_to_f32(w)
    X = np.asarray(x, dtype=F32).reshape(n, din)
    return (X @ W.reshape(dout, din).T).astype(F32)


def rmsnorm(x: np.ndarray, g: np.ndarray, n: int, d: int, eps: float = 1e-6) -> np.ndarray:
    """RMSNORM (kernels.js:46-63): x * (1 / sqrt(sum(x^2)/d + eps)) * g."""
    X = np.asarray(x, dtype=F32).reshape(n, d)
    G = g if g.dtype == np.float32 else bf16_bits_to_f32(g)
    ss = np.sum((X * X).astype(F32), axis=1, dtype=F32)
    scale = (F32(1.0) / np.sqrt(ss / F32(d) + F32(eps))).astype(F32)
    return ((X * scale[:, None]).astype(F32) * G[None, :]).astype(F32)


def rope_freqs(hd: int, theta: float) -> np.ndarray:
    """freq[half] = exp2(-2*half/hd * log2(theta)) with fp32 steps (kernels.js:77)."""
    half = np.arange(hd // 2, dtype=F32)
    e = ((F32(-2.0) * half) / F32(hd)).astype(F32) * F32(math.log2(theta))
    return np.exp2(e.astype(np.float64)).astype(F32)


def rope(x: np.ndarray, n: int, heads: int, hd: int, pos0: int, theta: float = 1e6) -> np.ndarray:
    """ROPE (kernels.js:66-83): rotate-half pairs (i, i + hd/2); ang = f32(pos) * freq."""
    X = np.asarray(x, dtype=F32).reshape(n, heads, hd).copy()
    fr = rope_freqs(hd, theta)
    pos = (pos0 + np.arange(n)).astype(F32)
    ang = (pos[:, None] * fr[None, :]).astype(F32)
    c = np.cos(ang.astype(np.float64)).astype(F32)[:, None, :]
    s = np.sin(ang.astype(np.float64)).astype(F32)[:, None, :]
    h = hd // 2
    x1 = X[:, :, :h].copy()
    x2 = X[:, :, h:].copy()
    X[:, :, :h] = (x1 * c).astype(F32) - (x2 * s).astype(F32)
    X[:, :, h:] = (x1 * s).astype(F32) + (x2 * c).astype(F32)
    return X.reshape(n, heads * hd)


def attention(q, kcache, vcache, T0: int, n: int, nq: int, kvh: int, hd: int) -> np.ndarray:
    """ATTENTION (kernels.js:86-132): causal GQA; row t attends slots [0, T0+t];
    kv head = h / (nq/kvh); scores (q.k) * f32(1/sqrt(hd)); softmax; weights . V."""
    Q = np.asarray(q, dtype=F32).reshape(n, nq, hd)
    KC = np.asarray(kcache, dtype=F32).reshape(-1, kvh, hd)
    VC = np.asarray(vcache, dtype=F32).reshape(-1, kvh, hd)
    scale = F32(1.0 / math.sqrt(hd))
    grp = nq // kvh
    out = np.zeros((n, nq, hd), dtype=F32)
    for t in range(n):
        tend = T0 + t + 1
        for g in range(kvh):
            K = KC[:tend, g, :]
            V = VC[:tend, g, :]
            qs = Q[t, g * grp:(g + 1) * grp, :]
            s = ((qs @ K.T).astype(F32) * scale).astype(F32)  # [grp, tend]
            m = s.max(axis=1, keepdims=True)
            e = np.exp((s - m).astype(np.float64)).astype(F32)
            w = (e / e.sum(axis=1, dtype=F32, keepdims=True)).astype(F32)
            out[t, g * grp:(g + 1) * grp, :] = (w @ V).astype(F32)
    return out.reshape(n, nq * hd)


def silu_mul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """SILUMUL (kernels.js:134-145): a / (1 + exp(-a)) * b."""
    A = np.asarray(a, dtype=F32)
    e = np.exp((-A).astype(np.float64)).astype(F32)
    return ((A / (F32(1.0) + e)).astype(F32) * np.asarray(b, dtype=F32)).astype(F32)


def add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """ADD (kernels.js:161-171)."""
    return (np.asarray(a, dtype=F32) + np.asarray(b, dtype=F32)).astype(F32)


def add_bias(a: np.ndarray, bias: np.ndarray, n: int, dout: int) -> np.ndarray:
    """ADDBIAS (kernels.js:148-159): A[i] + bf16(B[i % dout])."""
    B = bias if bias.dtype == np.float32 else bf16_bits_to_f32(bias)
    return (np.asarray(a, dtype=F32).reshape(n, dout) + B[None, :]).astype(F32).reshape(-1)


def argmax_first(logits: np.ndarray) -> int:
    """Host scan of sampleLast (pipeline.js:152-169): strict '>' from bestV = -inf
    in index order, so the lowest index wins ties and NaN never wins."""
    v = np.asarray(logits, dtype=F32)
    v = np.where(np.isnan(v), F32(-np.inf), v)
    return int(np.argmax(v))


# ---- assignLayers (pipeline.js:6-23) ----------------------------------------------------
def js_round(x: float) -> int:
    """Math.round: halves round toward +inf."""
    return int(math.floor(x + 0.5))


def assign_layers(peers: list[dict], num_layers: int) -> list[dict]:
    caps = []
    for p in peers:
        prof = p.get("profile") or {}
        mem = prof.get("memGB")
        mem = 4 if mem is None else mem
        caps.append({"id": p["id"], "cap": mem * (1.5 if prof.get("gpu") else 0.5)})
    total = 0.0
    for c in caps:
        total = total + c["cap"]
    assigned = 0
    out = []
    for i, c in enumerate(caps):
        share = num_layers - assigned if i == len(caps) - 1 else max(1, js_round((c["cap"] / total) * num_layers))
        rng = (assigned, min(num_layers, assigned + share))
        assigned = rng[1]
        out.append({"id": c["id"], "start": rng[0], "end": rng[1]})
    return out


# ---- model ----------------------------------------------------------------------------
@dataclass
class Config:
    vocab_size: int = 151936
    hidden_size: int = 1536
    num_layers: int = 28
    num_q_heads: int = 12
    num_kv_heads: int = 2
    head_dim: int = 128
    intermediate_size: int = 8960
    rope_theta: float = 1e6
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = True
    eos_token_id: int = 151645
    max_pos: int = 4096


LAYER_SUFFIXES = (
    "input_layernorm.weight", "post_attention_layernorm.weight",
    "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
    "self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias",
    "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight",
)


class Weights:
    """Name -> bf16 bits (uint16) with a cache of the fp32 decode."""

    def __init__(self, bits: dict[str, np.ndarray]):
        self.bits = bits
        self._f32: dict[str, np.ndarray] = {}

    def has(self, name: str) -> bool:
        return name in self.bits

    def f32(self, name: str) -> np.ndarray:
        a = self._f32.get(name)
        if a is None:
            a = bf16_bits_to_f32(self.bits[name])
            self._f32[name] = a
        return a


@dataclass
class OracleStage:
    """Stage (pipeline.js:26-88): layers [start, end) with fp32 KV [maxPos, KVH*HD]."""
    cfg: Config
    W: Weights
    start: int
    end: int
    kv_dtype: str = "f32"
    T0: int = 0
    kv: dict = field(default_factory=dict)

    def __post_init__(self):
        self.reset()

    def reset(self):
        row = self.cfg.num_kv_heads * self.cfg.head_dim
        for L in range(self.start, self.end):
            if L not in self.kv:
                self.kv[L] = {"k": np.zeros((self.cfg.max_pos, row), F32), "v": np.zeros((self.cfg.max_pos, row), F32)}
        self.T0 = 0

    def append_kv(self, L: int, kk: np.ndarray, vv: np.ndarray, n: int):
        row = self.cfg.num_kv_heads * self.cfg.head_dim
        if self.T0 + n > self.cfg.max_pos:
            raise IndexError("KV cache overflow")
        kk = np.asarray(kk, F32).reshape(n, row)
        vv = np.asarray(vv, F32).reshape(n, row)
        if self.kv_dtype == "bf16":
            kk, vv = bf16_round(kk), bf16_round(vv)
        self.kv[L]["k"][self.T0:self.T0 + n] = kk
        self.kv[L]["v"][self.T0:self.T0 + n] = vv

    def forward(self, hidden: np.ndarray, n: int, pos_start: int) -> np.ndarray:
        c, W = self.cfg, self.W
        D, NQ, KVH, HD, I = c.hidden_size, c.num_q_heads, c.num_kv_heads, c.head_dim, c.intermediate_size
        h = np.asarray(hidden, F32).reshape(n, D).copy()
        for L in range(self.start, self.end):
            p = f"model.layers.{L}."
            x = rmsnorm(h, W.f32(p + "input_layernorm.weight"), n, D, c.rms_norm_eps)
            q = matmul(x, W.f32(p + "self_attn.q_proj.weight"), n, D, NQ * HD)
            kk = matmul(x, W.f32(p + "self_attn.k_proj.weight"), n, D, KVH * HD)
            vv = matmul(x, W.f32(p + "self_attn.v_proj.weight"), n, D, KVH * HD)
            if W.has(p + "self_attn.q_proj.bias"):
                q = add_bias(q, W.f32(p + "self_attn.q_proj.bias"), n, NQ * HD).reshape(n, -1)
            if W.has(p + "self_attn.k_proj.bias"):
                kk = add_bias(kk, W.f32(p + "self_attn.k_proj.bias"), n, KVH * HD).reshape(n, -1)
            if W.has(p + "self_attn.v_proj.bias"):
                vv = add_bias(vv, W.f32(p + "self_attn.v_proj.bias"), n, KVH * HD).reshape(n, -1)
            q = rope(q, n, NQ, HD, pos_start, c.rope_theta)
            kk = rope(kk, n, KVH, HD, pos_start, c.rope_theta)
            self.append_kv(L, kk, vv, n)
            att = attention(q, self.kv[L]["k"], self.kv[L]["v"], self.T0, n, NQ, KVH, HD)
            o = matmul(att, W.f32(p + "self_attn.o_proj.weight"), n, NQ * HD, D)
            h1 = add(h, o)
            x2 = rmsnorm(h1, W.f32(p + "post_attention_layernorm.weight"), n, D, c.rms_norm_eps)
            g = matmul(x2, W.f32(p + "mlp.gate_proj.weight"), n, D, I)
            u = matmul(x2, W.f32(p + "mlp.up_proj.weight"), n, D, I)
            m = silu_mul(g, u)
            d = matmul(m, W.f32(p + "mlp.down_proj.weight"), n, I, D)
            h = add(h1, d)
        self.T0 += n
        return h


class OracleLeader:
    """LeaderPipeline (pipeline.js:91-282), single node: embed, own stage, sample."""

    CHUNK_ROWS = 8192  # pipeline.js:103

    def __init__(self, cfg: Config, W: Weights, kv_dtype: str = "f32"):
        self.cfg, self.W = cfg, W
        self.stage = OracleStage(cfg, W, 0, cfg.num_layers, kv_dtype)

    def lm_head_name(self) -> str:
        if self.W.has("lm_head.weight"):
            return "lm_head.weight"
        return "model.embed_tokens.weight"

    def embed_tokens(self, tokens) -> np.ndarray:
        E = self.W.bits["model.embed_tokens.weight"].reshape(self.cfg.vocab_size, self.cfg.hidden_size)
        return bf16_bits_to_f32(E[np.asarray(tokens, dtype=np.int64)])

    def logits(self, hidden_row: np.ndarray) -> np.ndarray:
        c = self.cfg
        D = c.hidden_size
        nrm = rmsnorm(np.asarray(hidden_row, F32)[:D], self.W.f32("model.norm.weight"), 1, D, c.rms_norm_eps)
        E = self.W.f32(self.lm_head_name()).reshape(c.vocab_size, D)
        out = np.empty(c.vocab_size, F32)
        for r0 in range(0, c.vocab_size, self.CHUNK_ROWS):
            r1 = min(c.vocab_size, r0 + self.CHUNK_ROWS)
            out[r0:r1] = (E[r0:r1] @ nrm[0]).astype(F32)
        return out

    def sample_last(self, hidden_row: np.ndarray) -> tuple[int, np.ndarray]:
        lg = self.logits(hidden_row)
        return argmax_first(lg), lg

    def forward(self, hidden: np.ndarray, n: int, pos_start: int) -> np.ndarray:
        h = self.stage.forward(hidden, n, pos_start)
        return h[n - 1]

    def teacher_forced(self, tokens, continuation) -> list[np.ndarray]:
        """Logits of every step of generate() when the emitted tokens are forced to
        `continuation` (step i feeds continuation[i-1]): compares a run whose
        greedy choices differ only at near-ties on identical inputs."""
        logs = []
        row = self.forward(self.embed_tokens(tokens), len(tokens), 0)
        logs.append(self.logits(row))
        for i in range(1, len(continuation)):
            row = self.forward(self.embed_tokens([continuation[i - 1]]), 1, len(tokens) + i - 1)
            logs.append(self.logits(row))
        return logs

    def generate(self, tokens, max_new: int, keep_logits: bool = False):
        """pipeline.js:255-281. Returns (emitted tokens, per-step logits or None)."""
        out, logs = [], []
        row = self.forward(self.embed_tokens(tokens), len(tokens), 0)
        nxt, lg = self.sample_last(row)
        out.append(nxt)
        if keep_logits:
            logs.append(lg)
        for i in range(1, max_new):
            if nxt == self.cfg.eos_token_id:
                break
            row = self.forward(self.embed_tokens([nxt]), 1, len(tokens) + i - 1)
            nxt, lg = self.sample_last(row)
            out.append(nxt)
            if keep_logits:
                logs.append(lg)
        return out, (logs if keep_logits else None)
