"""bf16 weight layout and tensor naming (weights.js:143-182), plus local
safetensors ingestion.

The reference keeps each bf16 element as one u32 of raw bits on the JS side and
on the GPU (4 bytes per weight). Here the JS-side helpers keep that layout for
drop-in callers, while the device stores 2-byte bf16 (`loadWeightBits` packs).
`load_safetensors_slice` reads the tensors of a layer range straight from a
local .safetensors file (header = 8-byte little-endian length + JSON, the format
fetchTensorMap parses over HTTP, weights.js:25-40).
"""
from __future__ import annotations

import json
import mmap
import os

import numpy as np


def bf16BytesToF32Bits(b) -> np.ndarray:
    """bf16 bytes -> u32 array of raw bf16 bits, one per element (weights.js:144-150)."""
    a = np.frombuffer(b if isinstance(b, (bytes, bytearray, memoryview)) else bytes(b), dtype="<u2")
    return a.astype(np.uint32)


def bf16BitsToF32(u32, offset: int = 0, length: int | None = None) -> np.ndarray:
    """u32 of raw bf16 bits -> float32 via bits << 16 (weights.js:153-157)."""
    a = np.asarray(u32)
    length = a.size - offset if length is None else length
    bits = a.reshape(-1)[offset:offset + length].astype(np.uint32) & np.uint32(0xFFFF)
    return (bits << np.uint32(16)).view(np.float32)


def reinterpretBits(bits: int) -> float:
    """u32 bit pattern -> float32 value (weights.js:159-162)."""
    return float(np.array([bits & 0xFFFFFFFF], dtype=np.uint32).view(np.float32)[0])


def tensorsForLayers(start: int, end: int, isLeader: bool) -> list[str]:
    """HF tensor names needed by a stage owning layers [start, end) (weights.js:167-182)."""
    names = []
    for i in range(start, end):
        b = f"model.layers.{i}."
        names += [
            f"{b}input_layernorm.weight", f"{b}post_attention_layernorm.weight",
            f"{b}self_attn.q_proj.weight", f"{b}self_attn.k_proj.weight",
            f"{b}self_attn.v_proj.weight", f"{b}self_attn.o_proj.weight",
            f"{b}self_attn.q_proj.bias", f"{b}self_attn.k_proj.bias",
            f"{b}self_attn.v_proj.bias",
            f"{b}mlp.gate_proj.weight", f"{b}mlp.up_proj.weight", f"{b}mlp.down_proj.weight",
        ]
    if isLeader:
        names += ["model.embed_tokens.weight", "model.norm.weight"]
    return names


bf16_bytes_to_f32_bits = bf16BytesToF32Bits
bf16_bits_to_f32 = bf16BitsToF32
tensors_for_layers = tensorsForLayers


# ---- local safetensors ----------------------------------------------------------------
def read_tensor_map(path: str) -> dict:
    """Parse the safetensors header: name -> {dtype, shape, data_offsets} with
    offsets made absolute (weights.js:25-40 does the same over HTTP Range)."""
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(n).decode("utf-8"))
    header.pop("__metadata__", None)
    start = 8 + n
    for t in header.values():
        t["data_offsets"] = [t["data_offsets"][0] + start, t["data_offsets"][1] + start]
    return header


def read_tensors(path: str, names, tensor_map: dict | None = None) -> dict[str, np.ndarray]:
    """Raw bf16 tensors (uint16) for the names present in the file (fetchTensors,
    weights.js:46-123, without the network and cache)."""
    tm = tensor_map or read_tensor_map(path)
    out = {}
    with open(path, "rb") as f, mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as mm:
        for n in names:
            t = tm.get(n)
            if t is None:
                continue
            if t["dtype"] != "BF16":
                raise ValueError(f"tensor {n}: dtype {t['dtype']}, expected BF16")
            a, b = t["data_offsets"]
            if b > len(mm) or b < a:
                raise ValueError(f"tensor {n}: byte range {a}..{b} outside the file")
            out[n] = np.frombuffer(mm[a:b], dtype="<u2").copy()
    return out


def write_safetensors(path: str, tensors: dict[str, np.ndarray], shapes: dict[str, tuple] | None = None):
    """Write bf16 (uint16) tensors as a safetensors file (test fixtures, synthetic checkpoints)."""
    header, off, blobs = {}, 0, []
    for n, a in tensors.items():
        a = np.ascontiguousarray(a, dtype="<u2")
        shape = list(shapes[n]) if shapes and n in shapes else [int(a.size)]
        header[n] = {"dtype": "BF16", "shape": shape, "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
        blobs.append(a)
    hb = json.dumps(header).encode("utf-8")
    hb += b" " * ((8 - len(hb) % 8) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(len(hb).to_bytes(8, "little"))
        f.write(hb)
        for a in blobs:
            f.write(a.tobytes())
    os.replace(tmp, path)


# ---- checkpoint slices straight to the device ----------------------------------------------
def checkpoint_files(path: str) -> list[str]:
    """The safetensors files of a checkpoint: `path` itself, the shards named by a
    Hugging Face `model.safetensors.index.json` (given directly or inside the
    directory `path`), or every `*.safetensors` file of the directory."""
    if os.path.isdir(path):
        idx = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(idx):
            path = idx
        else:
            files = sorted(os.path.join(path, f) for f in os.listdir(path) if f.endswith(".safetensors"))
            if not files:
                raise FileNotFoundError(f"no .safetensors files in {path}")
            return files
    if path.endswith(".json"):
        with open(path) as f:
            wm = json.load(f)["weight_map"]
        base = os.path.dirname(path)
        return sorted({os.path.join(base, v) for v in wm.values()})
    return [path]


def load_checkpoint(kctx, path: str, start: int, end: int, stage=None, leader=None) -> list[str]:
    """Upload the tensors a stage owning layers [start, end) needs (tensorsForLayers,
    weights.js:167-182), one tensor at a time from the memory-mapped file to the
    device, so the host holds one tensor at most. `stage` receives the layer
    tensors (`stage.W[name]`); `leader` (a LeaderPipeline) the embedding, final
    norm and, for untied models, `lm_head.weight`. Returns the names uploaded.
    Only the q/k/v projection biases (absent in bias-free models) and
    `lm_head.weight` (absent when the embeddings are tied) may be missing; any
    other missing tensor raises KeyError, and every tensor's element count is
    checked against the context's model config before it is uploaded (a
    truncated or mis-sharded checkpoint fails here, not in a later kernel)."""
    cfg = kctx.cfg
    D, QD, KD, I, V = (cfg.hidden_size, cfg.num_q_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim,
                       cfg.intermediate_size, cfg.vocab_size)
    sizes = {"input_layernorm.weight": D, "post_attention_layernorm.weight": D,
             "self_attn.q_proj.weight": QD * D, "self_attn.k_proj.weight": KD * D,
             "self_attn.v_proj.weight": KD * D, "self_attn.o_proj.weight": D * QD,
             "self_attn.q_proj.bias": QD, "self_attn.k_proj.bias": KD, "self_attn.v_proj.bias": KD,
             "mlp.gate_proj.weight": I * D, "mlp.up_proj.weight": I * D, "mlp.down_proj.weight": D * I,
             "model.embed_tokens.weight": V * D, "model.norm.weight": D, "lm_head.weight": V * D}

    def expected(name: str) -> int:
        key = name.split(".", 3)[3] if name.startswith("model.layers.") else name
        return sizes[key]

    def optional(name: str) -> bool:
        return name.endswith("_proj.bias") or name == "lm_head.weight"

    where = {}
    maps = {}
    for f in checkpoint_files(path):
        maps[f] = read_tensor_map(f)
        for n in maps[f]:
            where.setdefault(n, f)
    done = []

    def one(name):
        f = where.get(name)
        if f is None:
            if optional(name):
                return None
            raise KeyError(f"checkpoint {path} has no tensor {name}")
        bits = read_tensors(f, [name], maps[f])[name]
        if bits.size != expected(name):
            raise ValueError(f"{name}: {bits.size} elements in the checkpoint, the model config needs "
                             f"{expected(name)}")
        buf = kctx.loadWeightBf16(bits, name)
        done.append(name)
        return buf

    if stage is not None:
        for name in tensorsForLayers(start, end, False):
            buf = one(name)
            if buf is not None:
                stage.W[name] = buf
    if leader is not None:
        embed, norm, head = one("model.embed_tokens.weight"), one("model.norm.weight"), one("lm_head.weight")
        leader.setLeaderWeights(embed, norm, head)
    return done
