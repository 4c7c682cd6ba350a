"""Stage forward logic, leader decoder and layer split (pipeline.js) on the B200 path.

`Stage` (pipeline.js:26-88) and `LeaderPipeline` (pipeline.js:91-282) keep the
reference's names and semantics; their compute runs in libdllm.so (one
persistent sm_100a kernel per pass). The hop between stages keeps the frame
protocol of pipeline.js:226-253 / script.js:163-172 behind a transport callable,
so a stage can live in another context or another process; the multi-GPU
runner (multigpu.py) replaces the frame hop with NCCL send/recv.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import _lib, frames
from .constants import FRAME
from .kernels import GpuBuffer, KernelContext


# ---- assignLayers (pipeline.js:6-23) ---------------------------------------------------
def _js_round(x: float) -> int:
    """Math.round: halves toward +inf (Python's round() is banker's)."""
    return int(math.floor(x + 0.5))


def assignLayers(peers: list[dict], num_layers: int | None = None) -> list[dict]:
    """Split layers across peers by capacity memGB * (gpu ? 1.5 : 0.5), memGB
    defaulting to 4; each share max(1, round(cap/total * L)); the last peer takes
    the remainder (which can be empty, e.g. 8 equal peers over 28 layers)."""
    from .constants import CFG
    L = CFG.num_layers if num_layers is None else num_layers
    caps = []
    for p in peers:
        prof = p.get("profile") or {}
        mem = prof.get("memGB")
        caps.append({"id": p["id"], "cap": (4 if mem is None else mem) * (1.5 if prof.get("gpu") else 0.5)})
    total = 0.0
    for c in caps:
        total += c["cap"]
    assigned, out = 0, []
    for i, c in enumerate(caps):
        share = L - assigned if i == len(caps) - 1 else max(1, _js_round((c["cap"] / total) * L))
        rng = (assigned, min(L, assigned + share))
        assigned = rng[1]
        out.append({"id": c["id"], "start": rng[0], "end": rng[1]})
    return out


assign_layers = assignLayers


def plan_stages(cfg, n_stages: int) -> list[tuple[int, int]]:
    """Contiguous layer ranges for n_stages GPUs minimising the largest per-stage
    weight bytes, with the LM head on the last stage (embedding on the first is
    one row per token and costs nothing). Used by the multi-GPU runner; the
    reference-compatible split is assignLayers."""
    L = cfg.num_layers
    lw, hw = cfg.layer_weight_bytes(), cfg.head_weight_bytes()
    best = None
    # binary search on the bottleneck: largest cost per stage
    lo, hi = 0, L * lw + hw
    while lo < hi:
        mid = (lo + hi) // 2
        if _fits(L, lw, hw, n_stages, mid):
            hi = mid
        else:
            lo = mid + 1
    cap = lo
    # greedy fill from the back so the head stage gets fewer layers
    ranges, end, cost_cap = [], L, cap
    for s in range(n_stages - 1, -1, -1):
        budget = cost_cap - (hw if s == n_stages - 1 else 0)
        k = max(0, budget // lw) if budget >= 0 else 0
        k = min(k, end - 0)
        if s == 0:
            k = end
        ranges.append((end - k, end))
        end -= k
    ranges.reverse()
    best = ranges
    return best


def _fits(L: int, lw: int, hw: int, S: int, cap: int) -> bool:
    left = L
    for s in range(S - 1, -1, -1):
        budget = cap - (hw if s == S - 1 else 0)
        if budget < 0:
            return False
        left -= min(left, budget // lw)
    return left == 0


# ---- Stage (pipeline.js:26-88) -----------------------------------------------------------
class _StageWeights(dict):
    """stage.W: assigning a buffer hands the stage a reference (pipeline.js:31)."""

    def __init__(self, stage: "Stage"):
        super().__init__()
        self._stage = stage

    def __setitem__(self, name: str, buf: GpuBuffer):
        st = self._stage
        st.k._check(st.lib.dllm_stage_set_weight(st.handle, name.encode(), st.k._h(buf)), f"W[{name}]")
        super().__setitem__(name, buf)


class _KvTensor:
    def __init__(self, stage: "Stage", layer: int, which: int):
        self.stage, self.layer, self.which = stage, layer, which

    def read(self, slot_start: int = 0, n_slots: int | None = None, seq: int = 0) -> np.ndarray:
        """Slots in the reference layout [n, KVH*HD] fp32 (pipeline.js:38-43)."""
        st = self.stage
        n = st.T0 - slot_start if n_slots is None else n_slots
        row = st.k.KVH * st.k.HD
        out = np.empty((max(n, 0), row), np.float32)
        if n <= 0:
            return out
        st.k._check(st.lib.dllm_stage_read_kv(st.handle, self.layer, self.which, seq, slot_start, n,
                                              _lib.ptr(out, C.c_float)), "read_kv")
        return out


class _KvLayer:
    def __init__(self, stage, layer):
        self.k = _KvTensor(stage, layer, 0)
        self.v = _KvTensor(stage, layer, 1)


class Stage:
    """Runs a contiguous block of decoder layers, resumable with its own KV cache."""

    def __init__(self, kctx: KernelContext, start: int, end: int, _handle: int | None = None):
        self.k = kctx
        self.lib = kctx.lib
        self.start, self.end = start, end
        self._owned = _handle is None
        if _handle is None:
            h = C.c_void_p()
            kctx._check(self.lib.dllm_stage_create(kctx.handle, start, end, C.byref(h)), "Stage")
            _handle = h.value
        self.handle = _handle
        self.W = _StageWeights(self)
        self.kv = {L: _KvLayer(self, L) for L in range(start, end)}

    @property
    def T0(self) -> int:
        return self.t0_of(0)

    @T0.setter
    def T0(self, v: int):
        self.k._check(self.lib.dllm_stage_set_t0(self.handle, 0, int(v)), "T0")

    def t0_of(self, seq: int) -> int:
        return int(self.lib.dllm_stage_get_t0(self.handle, seq))

    def set_t0(self, seq: int, v: int):
        self.k._check(self.lib.dllm_stage_set_t0(self.handle, seq, int(v)), "set_t0")

    def reset(self):
        self.k._check(self.lib.dllm_stage_reset(self.handle), "reset")

    def forward(self, hiddenF32, n: int, posStart: int) -> GpuBuffer:
        a = np.ascontiguousarray(hiddenF32, dtype=np.float32).reshape(-1)
        if a.size < n * self.k.D:
            raise _lib.DllmError(_lib.DLLM_EINVAL, f"forward: {a.size} floats for n={n}")
        out = C.c_void_p()
        self.k._check(self.lib.dllm_stage_forward(self.handle, _lib.ptr(a, C.c_float), n, posStart, C.byref(out)),
                      "Stage.forward")
        return GpuBuffer(self.k, out.value, n * self.k.D, "f32", "stage_out")

    def appendKv(self, L: int, kkBuf: GpuBuffer, vvBuf: GpuBuffer, n: int):
        self.k._check(self.lib.dllm_stage_append_kv(self.handle, L, self.k._h(kkBuf), self.k._h(vvBuf), n), "appendKv")

    def forward_rows(self, h_dev_ptr: int, seq_ids, tokens_in_ptr: int | None = None,
                     tokens_out_ptr: int | None = None):
        """Decode pass of one micro-batch on device rows (see dllm_stage_forward_rows)."""
        ids = np.ascontiguousarray(seq_ids, dtype=np.int32)
        self.k._check(self.lib.dllm_stage_forward_rows(self.handle, h_dev_ptr, ids.size, _lib.ptr(ids, C.c_int32),
                                                       tokens_in_ptr or None, tokens_out_ptr or None),
                      "forward_rows")

    def fill_kv_random(self, seq: int, n_slots: int, seed: int = 0):
        self.k._check(self.lib.dllm_stage_fill_kv_random(self.handle, seq, n_slots, seed), "fill_kv_random")

    def set_trace(self, cap: int):
        """Stamp the GPU global timer at kernel start and after every grid barrier."""
        self.k._check(self.lib.dllm_stage_set_trace(self.handle, cap), "set_trace")

    def read_trace(self, cap: int) -> np.ndarray:
        out = np.zeros(cap, np.uint64)
        self.k._check(self.lib.dllm_stage_read_trace(self.handle, out.ctypes.data_as(C.POINTER(C.c_uint64)), cap),
                      "read_trace")
        return out

    def read_workspace(self, which: str, rows: int = 1) -> np.ndarray:
        """Latest pass's q (after bias + RoPE), attention output or SiLU(gate)*up
        of the stage's last layer, [rows, width] fp32 (test hook)."""
        idx = {"q": 0, "att": 1, "mid": 2}[which]
        width = self.k.cfg.intermediate_size if which == "mid" else self.k.NQ * self.k.HD
        out = np.empty((rows, width), np.float32)
        self.k._check(self.lib.dllm_stage_read_workspace(self.handle, idx, rows, _lib.ptr(out, C.c_float)),
                      "read_workspace")
        return out

    def pages_per_seq(self) -> int:
        return int(self.lib.dllm_stage_pages_per_seq(self.handle))

    def set_page_table(self, seq: int, pages):
        p = np.ascontiguousarray(pages, dtype=np.int32)
        self.k._check(self.lib.dllm_stage_set_page_table(self.handle, seq, _lib.ptr(p, C.c_int32), p.size),
                      "set_page_table")

    def close(self):
        if self._owned and getattr(self, "handle", None):
            self.lib.dllm_stage_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def handle_stage_frame(stage: Stage, data: bytes) -> bytes:
    """Stage side of a hop (script.js:163-172): run the frame's rows, reply RESP
    with all rows (HIDDEN_REQ) or only the last row (FINAL_REQ), posStart = T0."""
    frame = frames.unpack(data)
    D = stage.k.D
    n = frame["f32"].size // D
    h = stage.forward(frame["f32"], n, frame["posStart"])
    out = stage.k.readF32(h, n * D)
    if frame["msgType"] == FRAME["FINAL_REQ"]:
        out = out[(n - 1) * D:n * D]
    return frames.pack(FRAME["RESP"], frame["seqId"], stage.T0, out)


class LocalTransport:
    """Synchronous hop transport to stages held in this process (any device)."""

    def __init__(self, stages_by_id: dict):
        self.stages = stages_by_id

    def __call__(self, peer_id, data: bytes) -> bytes:
        return handle_stage_frame(self.stages[peer_id], data)


# ---- LeaderPipeline (pipeline.js:91-282) -----------------------------------------------------
class LeaderPipeline:
    CHUNK_ROWS = 8192  # pipeline.js:103 (the device LM head needs no chunking)

    def __init__(self, kctx: KernelContext, myRange, stages: list[dict] | None = None, opts: dict | None = None):
        opts = opts or {}
        self.k = kctx
        self.lib = kctx.lib
        self.myId = opts.get("myId", 0)
        h = C.c_void_p()
        kctx._check(self.lib.dllm_leader_create(kctx.handle, myRange[0], myRange[1], C.byref(h)), "LeaderPipeline")
        self.handle = h.value
        self.stage = Stage(kctx, myRange[0], myRange[1], _handle=self.lib.dllm_leader_stage(self.handle))
        self.stages = stages or [{"id": self.myId, "start": myRange[0], "end": myRange[1]}]
        self.stagesTail = [s for s in self.stages if s["id"] != self.myId]
        self.singleNode = len(self.stagesTail) == 0 and myRange[1] >= kctx.cfg.num_layers
        self.transport = opts.get("transport")  # callable(peerId, bytes) -> bytes
        self.onToken = opts.get("onToken") or (lambda t: None)
        self.seq = 1
        self._leader_bufs = []
        self.last_logits = None

    # loadLeaderWeights(embedBits, normBits) (pipeline.js:109-119); lm_head for untied models
    def loadLeaderWeights(self, embedBits, normBits, lmHeadBits=None):
        def up(a, name):
            if a is None:
                return None
            a = np.asarray(a)
            return self.k.loadWeightBf16(a, name) if a.dtype == np.uint16 else self.k.loadWeightBits(a, name)
        self.setLeaderWeights(up(embedBits, "model.embed_tokens.weight"), up(normBits, "model.norm.weight"),
                              up(lmHeadBits, "lm_head.weight"))

    def setLeaderWeights(self, embedBuf=None, normBuf=None, lmHeadBuf=None):
        h = lambda b: self.k._h(b) if b is not None else None
        self.k._check(self.lib.dllm_leader_set_weights(self.handle, h(embedBuf), h(normBuf), h(lmHeadBuf)),
                      "loadLeaderWeights")
        self._leader_bufs += [b for b in (embedBuf, normBuf, lmHeadBuf) if b is not None]

    def embedTokens(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(t.size * self.k.D, np.float32)
        self.k._check(self.lib.dllm_leader_embed_tokens(self.handle, _lib.ptr(t, C.c_int32), t.size,
                                                        _lib.ptr(out, C.c_float)), "embedTokens")
        return out

    def lastTokRow(self, f32, n):
        return np.asarray(f32, np.float32)[(n - 1) * self.k.D:n * self.k.D]

    def sampleLast(self, hiddenF32, return_logits: bool = False):
        row = np.ascontiguousarray(hiddenF32, dtype=np.float32).reshape(-1)[:self.k.D]
        tok = C.c_int32()
        lg = np.empty(self.k.cfg.vocab_size, np.float32) if return_logits else None
        self.k._check(self.lib.dllm_leader_sample_last(self.handle, _lib.ptr(row, C.c_float), C.byref(tok),
                                                       _lib.ptr(lg, C.c_float)), "sampleLast")
        self.last_logits = lg
        return (int(tok.value), lg) if return_logits else int(tok.value)

    def hop(self, peerId, hiddenF32, n: int, posStart: int, isFinal: bool) -> dict:
        """pipeline.js:226-243, synchronous: frame out through the transport, RESP back."""
        if self.transport is None:
            raise RuntimeError(f"hop to {peerId}: no transport configured")
        seq = self.seq
        self.seq += 1
        data = frames.pack(FRAME["FINAL_REQ"] if isFinal else FRAME["HIDDEN_REQ"], seq, posStart, hiddenF32)
        resp = frames.unpack(self.transport(peerId, data))
        if resp["seqId"] != seq or resp["msgType"] != FRAME["RESP"]:
            raise RuntimeError(f"hop to {peerId}: unexpected reply {resp['msgType']}/{resp['seqId']}")
        return resp

    def forward(self, hiddenF32, n: int, posStart: int) -> np.ndarray:
        """pipeline.js:187-224: own layers, then each remote stage; returns the last row."""
        D = self.k.D
        if self.stage.end > self.stage.start:
            h = self.stage.forward(hiddenF32, n, posStart)
            cur = self.k.readF32(h, n * D)
            if not self.stagesTail:
                return self.lastTokRow(cur, n)
            cur_n = n
        else:
            cur = self.lastTokRow(hiddenF32, n)
            if not self.stagesTail:
                return cur
            cur_n = 1
        for i, s in enumerate(self.stagesTail):
            is_last = i == len(self.stagesTail) - 1
            resp = self.hop(s["id"], cur, cur_n, posStart, is_last)
            if is_last:
                return resp["f32"]  # FINAL_REQ reply is just the last row
            cur = resp["f32"] if cur_n > 1 else resp["f32"][:D]
        return cur

    def generate(self, tokens, maxNew: int) -> int:
        """pipeline.js:255-281: prefill, greedy decode, EOS break; onToken per token."""
        toks = [int(t) for t in tokens]
        if self.singleNode:
            t = np.ascontiguousarray(toks, dtype=np.int32)
            cap = max(1, int(maxNew))
            out = np.empty(cap, np.int32)
            n_out = C.c_int()
            self.k._check(self.lib.dllm_leader_generate(self.handle, _lib.ptr(t, C.c_int32), t.size, cap,
                                                        _lib.ptr(out, C.c_int32), C.byref(n_out)), "generate")
            emitted = [int(x) for x in out[:n_out.value]]
            for tok in emitted:
                self.onToken(tok)
            return emitted[-1]
        row = self.forward(self.embedTokens(toks), len(toks), 0)
        nxt = self.sampleLast(row)
        self.onToken(nxt)
        for i in range(1, maxNew):
            if nxt == self.k.cfg.eos_token_id:
                break
            row = self.forward(self.embedTokens([nxt]), 1, len(toks) + i - 1)
            nxt = self.sampleLast(row)
            self.onToken(nxt)
        return nxt

    def decode(self, first_token: int, steps: int) -> list[int]:
        """Device-resident greedy decode of `steps` tokens at the current T0 (no EOS
        break, no per-token host round trip); single node only."""
        out = np.empty(steps, np.int32)
        self.k._check(self.lib.dllm_leader_decode(self.handle, int(first_token), steps, _lib.ptr(out, C.c_int32)),
                      "decode")
        return [int(x) for x in out]

    def decode_enqueue(self, first_token: int, steps: int):
        """Enqueue `steps` graph replays on the ctx stream without waiting."""
        self.k._check(self.lib.dllm_leader_decode_enqueue(self.handle, int(first_token), steps), "decode_enqueue")

    def read_tokens(self, steps: int) -> list[int]:
        out = np.empty(steps, np.int32)
        self.k._check(self.lib.dllm_leader_read_tokens(self.handle, _lib.ptr(out, C.c_int32), steps), "read_tokens")
        return [int(x) for x in out]

    def set_keep_logits(self, steps: int):
        self.k._check(self.lib.dllm_leader_set_keep_logits(self.handle, steps), "set_keep_logits")

    def read_logits(self, index: int) -> np.ndarray:
        out = np.empty(self.k.cfg.vocab_size, np.float32)
        self.k._check(self.lib.dllm_leader_read_logits(self.handle, index, _lib.ptr(out, C.c_float)), "read_logits")
        return out

    def close(self):
        if getattr(self, "handle", None):
            self.stage.handle = None
            self.lib.dllm_leader_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
