"""Kernel context: the `ctx` object of kernels.js on the B200 path.

`initKernels(device)` (kernels.js:5) returns a context whose methods keep the
reference's names, argument order and error behaviour (kernels.js:179-301):
buffer helpers `loadWeightBits / createF32 / writeF32 / readF32` and one op
launcher per shader `matmul / rmsnorm / ropeQ / ropeK / attention / siluMul /
add / addBias`. Each op allocates and returns a new device buffer, as the
reference does; every op runs a hand-written sm_100a kernel from libdllm.so.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .constants import CFG, ModelConfig


class GpuBuffer:
    """A device buffer (the GPUBuffer of the reference). Freed with the object."""

    __slots__ = ("ctx", "handle", "n", "dtype", "label", "__weakref__")

    def __init__(self, ctx: "KernelContext", handle: int, n: int, dtype: str, label: str = ""):
        self.ctx, self.handle, self.n, self.dtype, self.label = ctx, handle, n, dtype, label

    @property
    def size(self) -> int:
        """Bytes on the device (GPUBuffer.size)."""
        return int(self.ctx.lib.dllm_buf_bytes(self.handle))

    @property
    def device_ptr(self) -> int:
        return int(self.ctx.lib.dllm_buf_device_ptr(self.handle) or 0)

    def destroy(self):
        if self.handle:
            self.ctx.lib.dllm_buf_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class KernelContext:
    def __init__(self, device: int = 0, cfg: ModelConfig | None = None):
        self.lib = _lib.load()
        self.cfg = cfg or CFG
        self.device = device
        h = C.c_void_p()
        c = self.cfg.to_c()
        st = self.lib.dllm_init_kernels(device, C.byref(c), C.byref(h))
        if st != _lib.DLLM_OK:
            raise _lib.DllmError(st, f"initKernels(device={device}) failed: "
                                     f"{self.lib.dllm_status_string(st).decode()} (is this an sm_100 GPU?)")
        self.handle = h.value
        # kernels.js:173 dims, exposed on ctx like the reference
        self.D = self.cfg.hidden_size
        self.KVH = self.cfg.num_kv_heads
        self.NQ = self.cfg.num_q_heads
        self.HD = self.cfg.head_dim

    # ---- plumbing
    def _check(self, st: int, what: str = ""):
        _lib.check(st, self.handle, what)

    def _out(self, fn, *args, n: int, label: str) -> GpuBuffer:
        out = C.c_void_p()
        self._check(fn(self.handle, *args, C.byref(out)), label)
        return GpuBuffer(self, out.value, n, "f32", label)

    @staticmethod
    def _h(buf: GpuBuffer):
        if not isinstance(buf, GpuBuffer) or not buf.handle:
            raise ValueError("expected a live GpuBuffer")
        return buf.handle

    def close(self):
        if getattr(self, "handle", None):
            self.lib.dllm_ctx_destroy(self.handle)
            self.handle = None

    def set_stream(self, cuda_stream: int | None):
        """Enqueue on a caller-owned cudaStream_t (e.g. torch.cuda.Stream().cuda_stream); 0 / None
        (the legacy default stream's handle) selects the ctx's own stream."""
        self._check(self.lib.dllm_ctx_set_stream(self.handle, cuda_stream or None), "set_stream")

    def set_tensor_core_rows(self, min_rows: int):
        """Passes of >= min_rows rows use the tcgen05 GEMM (0: never); default 8."""
        self._check(self.lib.dllm_ctx_set_tensor_core_rows(self.handle, int(min_rows)), "set_tensor_core_rows")

    def synchronize(self, timeout_ms: int = 15000):
        self._check(self.lib.dllm_ctx_synchronize(self.handle, timeout_ms), "synchronize")

    @property
    def launch_count(self) -> int:
        return int(self.lib.dllm_ctx_launch_count(self.handle))

    # ---- buffers (kernels.js:181-211)
    def loadWeightBits(self, u32arr, label: str | None = None) -> GpuBuffer:
        a = np.ascontiguousarray(u32arr, dtype=np.uint32) if u32arr is not None else None
        if a is None or a.size == 0:
            raise _lib.DllmError(_lib.DLLM_EINVAL, "loadWeightBits: empty weights")  # kernels.js:182
        out = C.c_void_p()
        self._check(self.lib.dllm_load_weight_bits(self.handle, _lib.ptr(a, C.c_uint32), a.size,
                                                   (label or "weights").encode(), C.byref(out)), "loadWeightBits")
        return GpuBuffer(self, out.value, a.size, "bf16", label or "weights")

    def loadWeightBf16(self, u16arr, label: str | None = None) -> GpuBuffer:
        a = np.ascontiguousarray(u16arr, dtype=np.uint16) if u16arr is not None else None
        if a is None or a.size == 0:
            raise _lib.DllmError(_lib.DLLM_EINVAL, "loadWeightBits: empty weights")
        out = C.c_void_p()
        self._check(self.lib.dllm_load_weight_bf16(self.handle, _lib.ptr(a, C.c_uint16), a.size,
                                                   (label or "weights").encode(), C.byref(out)), "loadWeightBf16")
        return GpuBuffer(self, out.value, a.size, "bf16", label or "weights")

    def createBf16(self, n: int, label: str = "") -> GpuBuffer:
        out = C.c_void_p()
        self._check(self.lib.dllm_create_bf16(self.handle, int(n), label.encode(), C.byref(out)), "createBf16")
        return GpuBuffer(self, out.value, int(n), "bf16", label)

    def fillNormalBf16(self, buf: GpuBuffer, seed: int, std: float):
        self._check(self.lib.dllm_fill_normal_bf16(self.handle, self._h(buf), seed, std), "fillNormalBf16")

    def fillConstBf16(self, buf: GpuBuffer, value: float):
        self._check(self.lib.dllm_fill_const_bf16(self.handle, self._h(buf), value), "fillConstBf16")

    def readBf16(self, buf: GpuBuffer, n: int | None = None) -> np.ndarray:
        n = buf.n if n is None else n
        out = np.empty(n, np.uint16)
        self._check(self.lib.dllm_read_bf16(self.handle, self._h(buf), _lib.ptr(out, C.c_uint16), n), "readBf16")
        return out

    def createF32(self, numFloats: int, label: str = "") -> GpuBuffer:
        if not numFloats or numFloats <= 0:
            raise _lib.DllmError(_lib.DLLM_EINVAL, f"createF32: invalid size {numFloats}")  # kernels.js:189
        out = C.c_void_p()
        self._check(self.lib.dllm_create_f32(self.handle, int(numFloats), label.encode(), C.byref(out)), "createF32")
        return GpuBuffer(self, out.value, int(numFloats), "f32", label)

    def writeF32(self, buf: GpuBuffer, f32):
        a = np.ascontiguousarray(f32, dtype=np.float32).reshape(-1)
        self._check(self.lib.dllm_write_f32(self.handle, self._h(buf), _lib.ptr(a, C.c_float), a.size), "writeF32")

    def readF32(self, buf: GpuBuffer, numFloats: int, label: str = "") -> np.ndarray:
        if not numFloats or numFloats <= 0:
            raise _lib.DllmError(_lib.DLLM_EINVAL, f"readF32: invalid size {numFloats}")  # kernels.js:196
        out = np.empty(int(numFloats), np.float32)
        self._check(self.lib.dllm_read_f32(self.handle, self._h(buf), _lib.ptr(out, C.c_float), out.size,
                                           label.encode()), "readF32")
        return out

    # ---- ops (kernels.js:222-301)
    def matmul(self, xBuf, wBuf, n, din, dout) -> GpuBuffer:
        return self._out(self.lib.dllm_matmul, self._h(xBuf), self._h(wBuf), n, din, dout, n=n * dout,
                         label=f"mm_out_{n}x{dout}")

    def rmsnorm(self, xBuf, gBuf, n) -> GpuBuffer:
        return self._out(self.lib.dllm_rmsnorm, self._h(xBuf), self._h(gBuf), n, n=n * self.D, label=f"rms_out_{n}")

    def ropeQ(self, xBuf, posStart, n) -> GpuBuffer:
        self._check(self.lib.dllm_rope_q(self.handle, self._h(xBuf), posStart, n), "ropeQ")
        return xBuf

    def ropeK(self, xBuf, posStart, n) -> GpuBuffer:
        self._check(self.lib.dllm_rope_k(self.handle, self._h(xBuf), posStart, n), "ropeK")
        return xBuf

    def attention(self, qBuf, kCacheBuf, vCacheBuf, T0, n) -> GpuBuffer:
        return self._out(self.lib.dllm_attention, self._h(qBuf), self._h(kCacheBuf), self._h(vCacheBuf), T0, n,
                         n=n * self.NQ * self.HD, label=f"attn_out_{n}")

    def siluMul(self, aBuf, bBuf, total) -> GpuBuffer:
        return self._out(self.lib.dllm_silu_mul, self._h(aBuf), self._h(bBuf), total, n=total,
                         label=f"silu_out_{total}")

    def add(self, aBuf, bBuf, numFloats) -> GpuBuffer:
        return self._out(self.lib.dllm_add, self._h(aBuf), self._h(bBuf), numFloats, n=numFloats,
                         label=f"add_out_{numFloats}")

    def addBias(self, aBuf, biasBuf, n, dout) -> GpuBuffer:
        return self._out(self.lib.dllm_add_bias, self._h(aBuf), self._h(biasBuf), n, dout, n=n * dout,
                         label=f"bias_out_{n * dout}")

    def argmax(self, logitsBuf, n) -> int:
        """Greedy pick over device logits: the strict '>' scan of pipeline.js:159-162."""
        idx = C.c_int32()
        self._check(self.lib.dllm_argmax(self.handle, self._h(logitsBuf), n, C.byref(idx)), "argmax")
        return int(idx.value)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def initKernels(device: int = 0, cfg: ModelConfig | None = None) -> KernelContext:
    """kernels.js:5. `device` is a CUDA ordinal (the reference takes a GPUDevice)."""
    return KernelContext(device, cfg)


init_kernels = initKernels
