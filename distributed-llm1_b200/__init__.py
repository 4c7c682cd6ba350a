"""B200-native decode path for Qwen2.5-style decoders (drop-in for the WebGPU
path of kernels.js / pipeline.js / weights.js).

    import importlib; dllm = importlib.import_module("distributed-llm1_b200")
    ctx = dllm.initKernels(0, dllm.PRESETS["qwen2.5-7b"])

The compute is libdllm.so (hand-written sm_100a kernels, include/dllm.h); this
package is the host-side mirror of the reference's JavaScript interface.
"""
from . import _lib, constants, frames, net, tokenizer, weights
from .constants import CFG, FRAME, PRESETS, ModelConfig
from .kernels import GpuBuffer, KernelContext, initKernels, init_kernels
from .pipeline import LeaderPipeline, LocalTransport, Stage, assignLayers, assign_layers, handle_stage_frame, plan_stages
from .weights import bf16BitsToF32, bf16BytesToF32Bits, load_checkpoint, reinterpretBits, tensorsForLayers
from ._lib import DllmError, KvOverflowError
from .net import FrameServer, TcpTransport, serve_stage
from .tokenizer import Qwen2Tokenizer, chat_template

LIB_PATH = _lib.LIB_PATH


def load_library():
    """Load libdllm.so (raises ImportError when it has not been built)."""
    return _lib.load()
