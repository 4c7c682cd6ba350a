"""Checkpoint slices (weights.js:25-123, 167-182): a stage's layer range read from
safetensors files (single file, directory, or a sharded checkpoint with its
index) and uploaded tensor by tensor."""
import json
import os

import numpy as np
import pytest

import synth
from helpers import get_weights, load_stage_weights, model_config, oracle_cfg


def write_sharded(dirpath, W):
    """Two shards + model.safetensors.index.json, the layout of HF checkpoints."""
    from importlib import import_module
    wts = import_module("distributed-llm1_b200.weights")
    names = sorted(W)
    shards = {"model-00001-of-00002.safetensors": names[::2], "model-00002-of-00002.safetensors": names[1::2]}
    wm = {}
    for fname, ns in shards.items():
        wts.write_safetensors(os.path.join(dirpath, fname), {n: W[n] for n in ns})
        wm.update({n: fname for n in ns})
    with open(os.path.join(dirpath, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wm}, f)


class FakeCtx:
    """Records uploads instead of calling the library (CPU test)."""
    def __init__(self, cfg):
        self.cfg = cfg
        self.up = {}

    def loadWeightBf16(self, bits, name):
        self.up[name] = np.array(bits, copy=True)
        return name


class FakeStage:
    def __init__(self):
        self.W = {}


class FakeLeader:
    def setLeaderWeights(self, e, n, h):
        self.bufs = (e, n, h)


def test_checkpoint_slice_roundtrip(tmp_path, dllm, weights_cache):
    cfg = oracle_cfg("tiny", tie_word_embeddings=False)
    W = synth.synthetic_weights(cfg, seed=3)
    write_sharded(str(tmp_path), W)
    files = dllm.weights.checkpoint_files(str(tmp_path))
    assert [os.path.basename(f) for f in files] == ["model-00001-of-00002.safetensors",
                                                    "model-00002-of-00002.safetensors"]
    ctx, st, ld = FakeCtx(cfg), FakeStage(), FakeLeader()
    done = dllm.load_checkpoint(ctx, str(tmp_path), 1, 2, stage=st, leader=ld)
    want = dllm.tensorsForLayers(1, 2, False)
    assert sorted(st.W) == sorted(want)
    assert ld.bufs == ("model.embed_tokens.weight", "model.norm.weight", "lm_head.weight")
    assert set(done) == set(want) | {"model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"}
    for n in done:  # bit-exact, and nothing of layer 0 was read
        np.testing.assert_array_equal(ctx.up[n], W[n])
    assert not any(n.startswith("model.layers.0.") for n in ctx.up)


def test_checkpoint_single_file_and_missing_biases(tmp_path, dllm):
    cfg = oracle_cfg("tiny")
    W = {k: v for k, v in synth.synthetic_weights(cfg, seed=4).items() if not k.endswith("_proj.bias")}
    path = str(tmp_path / "model.safetensors")
    dllm.weights.write_safetensors(path, W)
    assert dllm.weights.checkpoint_files(path) == [path]
    ctx, st = FakeCtx(cfg), FakeStage()
    dllm.load_checkpoint(ctx, path, 0, cfg.num_layers, stage=st)
    assert not any(n.endswith("_proj.bias") for n in st.W)  # bias-free checkpoints load without them
    assert len(st.W) == 9 * cfg.num_layers


def test_checkpoint_missing_required_tensor_raises(tmp_path, dllm):
    """Only the projection biases and an untied LM head may be absent: a checkpoint
    without a required weight fails at load time with the tensor's name."""
    cfg = oracle_cfg("tiny")
    W = synth.synthetic_weights(cfg, seed=5)
    del W["model.layers.1.mlp.down_proj.weight"]
    path = str(tmp_path / "model.safetensors")
    dllm.weights.write_safetensors(path, W)
    with pytest.raises(KeyError, match="model.layers.1.mlp.down_proj.weight"):
        dllm.load_checkpoint(FakeCtx(cfg), path, 0, cfg.num_layers, stage=FakeStage())
    W2 = synth.synthetic_weights(cfg, seed=5)
    del W2["model.norm.weight"]
    dllm.weights.write_safetensors(path, W2)
    with pytest.raises(KeyError, match="model.norm.weight"):
        dllm.load_checkpoint(FakeCtx(cfg), path, 0, 1, stage=FakeStage(), leader=FakeLeader())


def test_checkpoint_wrong_size_raises(tmp_path, dllm):
    """A tensor whose element count disagrees with the model config (a truncated
    or mis-sharded file) is rejected before upload."""
    cfg = oracle_cfg("tiny")
    W = synth.synthetic_weights(cfg, seed=6)
    W["model.layers.0.self_attn.k_proj.weight"] = W["model.layers.0.self_attn.k_proj.weight"][:-8]
    path = str(tmp_path / "model.safetensors")
    dllm.weights.write_safetensors(path, W)
    ctx = FakeCtx(cfg)
    with pytest.raises(ValueError, match="k_proj.weight"):
        dllm.load_checkpoint(ctx, path, 0, cfg.num_layers, stage=FakeStage())
    assert "model.layers.0.self_attn.k_proj.weight" not in ctx.up


@pytest.mark.gpu
def test_stage_from_checkpoint_matches_memory(tmp_path, dllm, weights_cache):
    """A Stage loaded from a sharded checkpoint computes bit-identically to one
    loaded from the same tensors in memory."""
    cfg = oracle_cfg("tiny")
    W = get_weights(weights_cache, "tiny", cfg)
    write_sharded(str(tmp_path), W)
    h = (np.random.default_rng(1).standard_normal(3 * cfg.hidden_size, dtype=np.float32) * 0.05)
    outs = []
    for from_file in (False, True):
        ctx = dllm.initKernels(0, model_config(dllm, cfg, "f32"))
        st = dllm.Stage(ctx, 0, cfg.num_layers)
        if from_file:
            dllm.load_checkpoint(ctx, str(tmp_path), 0, cfg.num_layers, stage=st)
        else:
            load_stage_weights(ctx, st, W, 0, cfg.num_layers)
        outs.append(ctx.readF32(st.forward(h, 3, 0), 3 * cfg.hidden_size))
        st.close()
        ctx.close()
    np.testing.assert_array_equal(outs[0], outs[1])
