"""Model configuration and frame codes (constants.js:3-23), parameterised.

CFG mirrors the reference's Qwen2.5-1.5B object; ModelConfig carries the same
fields for any Qwen2.5-family size plus the KV-cache layout of this build.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, replace

from . import _lib

# constants.js:3-7
FRAME = {"HIDDEN_REQ": 1, "FINAL_REQ": 2, "RESP": 3}


@dataclass(frozen=True)
class ModelConfig:
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
    kv_dtype: str = "f32"  # "f32" (the reference's precision) or "bf16"
    kv_page_size: int = 64
    max_seqs: int = 1

    # JS-style aliases (CFG.hiddenSize ...)
    @property
    def vocabSize(self): return self.vocab_size
    @property
    def hiddenSize(self): return self.hidden_size
    @property
    def numLayers(self): return self.num_layers
    @property
    def numQHeads(self): return self.num_q_heads
    @property
    def numKVHeads(self): return self.num_kv_heads
    @property
    def headDim(self): return self.head_dim
    @property
    def intermediateSize(self): return self.intermediate_size
    @property
    def ropeTheta(self): return self.rope_theta
    @property
    def rmsNormEps(self): return self.rms_norm_eps
    @property
    def tieWordEmbeddings(self): return self.tie_word_embeddings
    @property
    def eosTokenId(self): return self.eos_token_id
    @property
    def maxPos(self): return self.max_pos

    def with_(self, **kw) -> "ModelConfig":
        return replace(self, **kw)

    def to_c(self) -> _lib.dllm_config:
        c = _lib.dllm_config()
        c.vocab_size = self.vocab_size
        c.hidden_size = self.hidden_size
        c.num_layers = self.num_layers
        c.num_q_heads = self.num_q_heads
        c.num_kv_heads = self.num_kv_heads
        c.head_dim = self.head_dim
        c.intermediate_size = self.intermediate_size
        c.rope_theta = self.rope_theta
        c.rms_norm_eps = self.rms_norm_eps
        c.tie_word_embeddings = int(self.tie_word_embeddings)
        c.eos_token_id = self.eos_token_id
        c.max_pos = self.max_pos
        c.kv_dtype = _lib.DLLM_KV_BF16 if self.kv_dtype == "bf16" else _lib.DLLM_KV_F32
        c.kv_page_size = self.kv_page_size
        c.max_seqs = self.max_seqs
        return c

    def asdict(self) -> dict:
        return asdict(self)

    # byte accounting (bf16 weights) used by the bench's roofline
    def layer_weight_bytes(self) -> int:
        D, QD, KD, I = (self.hidden_size, self.num_q_heads * self.head_dim, self.num_kv_heads * self.head_dim,
                        self.intermediate_size)
        mats = QD * D + 2 * KD * D + D * QD + 3 * I * D
        vecs = 2 * D + QD + 2 * KD  # norms + biases
        return 2 * (mats + vecs)

    def head_weight_bytes(self) -> int:
        return 2 * (self.vocab_size * self.hidden_size + self.hidden_size)

    def kv_bytes_per_pos(self) -> int:
        es = 2 if self.kv_dtype == "bf16" else 4
        return 2 * self.num_layers * self.num_kv_heads * self.head_dim * es


# constants.js:10-23 (Qwen2.5-1.5B-Instruct)
CFG = ModelConfig()

PRESETS = {
    "qwen2.5-0.5b": ModelConfig(vocab_size=151936, hidden_size=896, num_layers=24, num_q_heads=14, num_kv_heads=2,
                                head_dim=64, intermediate_size=4864, tie_word_embeddings=True),
    "qwen2.5-1.5b": CFG,
    "qwen2.5-7b": ModelConfig(vocab_size=152064, hidden_size=3584, num_layers=28, num_q_heads=28, num_kv_heads=4,
                              head_dim=128, intermediate_size=18944, tie_word_embeddings=False),
    "qwen2.5-32b": ModelConfig(vocab_size=152064, hidden_size=5120, num_layers=64, num_q_heads=40, num_kv_heads=8,
                               head_dim=128, intermediate_size=27648, tie_word_embeddings=False),
}
