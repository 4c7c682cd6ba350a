#!/usr/bin/env python
"""Decode throughput of the Qwen2.5 decode token loop on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line (rank 0). A "step" is one greedy decode token of every sequence
in flight. Workload (Qwen2.5-7B architecture, random-init bf16 weights, 2048-slot
synthetic N(0,1) bf16 KV prefill per sequence):
  * N=1: batch 1 through the whole model on one GPU; one persistent stage-kernel
    launch per token, replayed as a CUDA graph with the token kept on device.
  * N>1: contiguous layer stages, one per GPU (plan_stages), N micro-batches
    of --micro sequences in flight; the hidden-row hop is fused into the stage
    kernel (16-byte stores into the next GPU's receive buffer over NVLink and a
    released flag; dllm_pipeline_* through multigpu.NvlinkRing). Per-GPU work
    per step is fixed: weak scaling.
`value` is tokens/s of the whole job timed with CUDA events on the launching
stream (max over ranks); `e2e` is the same metric through the public generate
call with the token copied host->device and back every step. Weights (15 GB)
and KV exceed L2 (126 MB), so no L2 flush is needed between steps.

`--impl reference` times the reference's CPU path: the reference is JavaScript +
WebGPU with no runtime on this machine, so its loops are timed through the C++
restatement (oracle/ref_forward.cpp, reference loop order) on all host cores,
every step one full token (all layers, final norm, LM head), timed, not
extrapolated.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s (bf16) at 1/2/4/8 B200; % of HBM roofline per token"
UNIT = "tokens/s"
KV_LEN = 2048
WEIGHT_STD = 0.02


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    p.add_argument("--steps", type=int, default=128)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--model", default="qwen2.5-7b")
    p.add_argument("--kv-len", type=int, default=KV_LEN)
    p.add_argument("--micro", type=int, default=1,
                   help="sequences per micro-batch (N>1), or sequences decoded together (N=1)")
    p.add_argument("--n-micro", type=int, default=0,
                   help="N>1: micro-batches in flight (default: one per stage)")
    p.add_argument("--tc-rows", type=int, default=None,
                   help="passes of at least this many rows use the tensor-core pass (0: never; default: the library's)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-steps", type=int, default=3, help="tokens in the CPU baseline sample")
    p.add_argument("--kernel-sweep", nargs="?", const="all", default=None,
                   choices=["all", "matvec", "gemm", "attention", "norm"],
                   help="isolated kernel sweep (matvec / tensor-core GEMM shapes, attention lengths, RMSNorm and "
                        "RoPE at hidden 3584): one JSON line per case instead of the decode benchmark")
    p.add_argument("--phase-trace", action="store_true",
                   help="per-phase time of the persistent stage kernel (global-timer stamps of CTA 0 after every "
                        "grid barrier) with each phase's algorithmic bytes and fraction of the measured HBM peak: "
                        "one JSON line instead of the decode benchmark")
    p.add_argument("--layers", type=int, default=0,
                   help="profiling case only: run the first N layers + LM head (a few GB on the device); "
                        "the line is marked and is not the benchmark")
    return p.parse_args()


def measured_peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# DRAM traffic of the stage kernel per token, as a multiple of its algorithmic
# bytes: dram__bytes_read.sum + dram__bytes_write.sum of one ncu capture of the
# 7B decode launch (2 layers + LM head, 2048-slot bf16 KV) over that launch's
# weight + KV + embedding bytes. Re-measure with the profiling command when the
# kernel changes.
STAGE_TRAFFIC_RATIO = 1.0028


def traffic_bytes(algorithmic: float, model: str) -> float | None:
    """ncu-measured DRAM bytes per launch, scaled from the profiled 7B capture."""
    return algorithmic * STAGE_TRAFFIC_RATIO if model == "qwen2.5-7b" else None


# ---- clocks --------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU through NVML while active."""

    def __init__(self, index: int, period_s: float = 0.02):
        self.index, self.period, self.samples, self.reasons = index, period_s, [], set()
        self._stop = threading.Event()
        self._t = None
        self.max_mhz = None
        self.ok = False

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.ok = True
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception:
            self.ok = False
        return self

    def _run(self):
        nv = self.nv
        names = {
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, bit in names.items():
                    if r & bit:
                        self.reasons.add(k)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=1)

    def summary(self) -> dict:
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---- model setup on the device ------------------------------------------------------
def device_weights(ctx, stage, cfg, start: int, end: int, embed: bool, head: bool, seed: int = 0):
    """Synthetic bf16 weights generated on the device: N(0, 0.02), norms 1.0."""
    syn = importlib.import_module("distributed-llm1_b200.synthetic")
    return syn.device_weights(ctx, stage, cfg, start, end, embed, head, seed)


def token_bytes(cfg, layers: int, head: bool, embed: bool, kv_positions: float) -> float:
    """Algorithmic HBM bytes of one token through `layers` layers: bf16 weights
    read once, plus K and V of every attended slot, plus the embedding row."""
    b = layers * cfg.layer_weight_bytes()
    if head:
        b += cfg.head_weight_bytes()
    if embed:
        b += 2 * cfg.hidden_size
    es = 2 if cfg.kv_dtype == "bf16" else 4
    b += layers * 2 * cfg.num_kv_heads * cfg.head_dim * es * kv_positions
    return b


# ---- CPU baseline (oracle C++ restatement) ----------------------------------------------
def _cpu_model(cfg, layers: int, kv_len: int, max_steps: int):
    """The oracle's C++ restatement with synthetic weights for `layers` layers +
    final norm + LM head, KV prefilled with `kv_len` slots."""
    import ctypes as C
    import subprocess

    import numpy as np
    so = os.path.join(ROOT, "oracle", "_build", "libref_forward.so")
    if not os.path.exists(so):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True, capture_output=True)
    lib = C.CDLL(so)
    cores = os.cpu_count() or 1
    lib.ref_set_threads.argtypes = [C.c_int]
    lib.ref_set_threads(cores)
    lib.ref_fill_normal_bf16.argtypes = [C.c_void_p, C.c_size_t, C.c_uint64, C.c_float]
    lib.ref_model_create.restype = C.c_void_p
    lib.ref_model_create.argtypes = [C.c_void_p, C.c_float, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    lib.ref_stage_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int]
    lib.ref_sample_last.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
    lib.ref_model_fill_kv.argtypes = [C.c_void_p, C.c_int, C.c_uint64]
    lib.ref_model_destroy.argtypes = [C.c_void_p]
    D, QD, KD, I, V = (cfg.hidden_size, cfg.num_q_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim,
                       cfg.intermediate_size, cfg.vocab_size)
    sizes = [D, D, QD * D, KD * D, KD * D, D * QD, QD, KD, KD, I * D, I * D, D * I]
    keep, ptrs = [], (C.c_void_p * (12 * layers))()
    for L in range(layers):
        for i, n in enumerate(sizes):
            a = np.empty(n, np.uint16)
            if i < 2:
                a[:] = 0x3F80  # norms = 1.0
            else:
                lib.ref_fill_normal_bf16(a.ctypes.data, n, 1000 + L * 12 + i, WEIGHT_STD)
            keep.append(a)
            ptrs[L * 12 + i] = a.ctypes.data
    norm = np.full(D, 0x3F80, np.uint16)
    head = np.empty(V * D, np.uint16)
    lib.ref_fill_normal_bf16(head.ctypes.data, head.size, 77, WEIGHT_STD)
    keep += [ptrs, norm, head]
    kv_bf16 = 1 if getattr(cfg, "kv_dtype", "bf16") == "bf16" else 0
    dims = (C.c_int * 10)(D, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim, I, V, 0, layers,
                          kv_len + max_steps + 2, kv_bf16)
    keep.append(dims)
    m = lib.ref_model_create(dims, cfg.rms_norm_eps, cfg.rope_theta, ptrs, head.ctypes.data, norm.ctypes.data,
                             head.ctypes.data)
    lib.ref_model_fill_kv(m, kv_len, 5)
    return lib, m, keep, cores


def cpu_token_times(cfg, warmup: int, steps: int, kv_len: int):
    """Per-token seconds of the reference loops through the whole model (every
    layer, final norm, LM head) on all host cores, one decode token per step."""
    import numpy as np
    lib, m, keep, cores = _cpu_model(cfg, cfg.num_layers, kv_len, warmup + steps)
    h = np.random.default_rng(0).standard_normal(cfg.hidden_size).astype(np.float32) * np.float32(0.05)
    times = []
    for s in range(warmup + steps):
        x = h.copy()
        t0 = time.perf_counter()
        lib.ref_stage_forward(m, x.ctypes.data, 1, kv_len + s)
        lib.ref_sample_last(m, x.ctypes.data, None)
        t1 = time.perf_counter()
        if s >= warmup:
            times.append(t1 - t0)
    lib.ref_model_destroy(m)
    del keep
    return times, cores


def cpu_baseline(cfg, steps: int, kv_len: int) -> dict:
    times, cores = cpu_token_times(cfg, 1, steps, kv_len)
    per_token = sum(times) / len(times)
    return {"value": 1.0 / per_token, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": (f"{steps} decode tokens (+1 warm-up) through all {cfg.num_layers} layers + final norm + "
                       f"LM head at {kv_len}-slot KV on {cores} host threads; oracle/ref_forward.cpp "
                       f"(reference loop order, fp32 arithmetic, bf16 weights and KV)")}


def run_reference(args):
    """The reference's CPU path through its C++ restatement (no package code)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import synth
    key = {"qwen2.5-0.5b": "0.5b", "qwen2.5-1.5b": "1.5b", "qwen2.5-7b": "7b", "qwen2.5-32b": "32b"}[args.model]
    cfg = synth.CONFIGS[key]
    cfg.kv_dtype = "bf16"
    times, cores = cpu_token_times(cfg, args.warmup, args.steps, args.kv_len)
    v = len(times) / sum(times)
    res = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": workload_config(args, cfg),
           "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                            "sample": (f"each step: one decode token through all {cfg.num_layers} layers + final "
                                       f"norm + LM head at {args.kv_len}-slot KV (timed, not extrapolated); "
                                       f"oracle/ref_forward.cpp")},
           "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "the reference is JavaScript + WebGPU with no JS engine or WebGPU adapter on this machine; "
                   "its loops are timed through the C++ restatement"}
    return res


def workload_config(args, cfg) -> dict:
    if getattr(args, "layers", 0):
        return {"workload": f"PROFILING CASE, not the benchmark: {args.model} dims, first {args.layers} layers + "
                            f"LM head, {args.kv_len}-slot synthetic bf16 KV, batch 1", "layers": args.layers}
    return {"workload": f"{args.model} greedy decode, {args.kv_len}-slot synthetic bf16 KV per sequence, "
                        f"{'batch 1 on one GPU' if args.gpus == 1 else f'{args.gpus}-stage pipeline, {args.n_micro or args.gpus} micro-batches of {args.micro}'}",
            "batch": 1 if args.gpus == 1 else (args.n_micro or args.gpus) * args.micro, "kv_len": args.kv_len,
            "parallelism": f"pp{args.gpus}", "kv_dtype": getattr(cfg, "kv_dtype", "bf16"), "weights": "bf16",
            "l2_policy": "inputs larger than L2 (weights 15 GB per token)"}


# ---- our arm, one GPU ---------------------------------------------------------------------
def run_single(args):
    import torch
    dllm = importlib.import_module("distributed-llm1_b200")
    cfg = dllm.PRESETS[args.model].with_(kv_dtype="bf16",
                                         max_pos=args.kv_len + 2 * (args.warmup + args.steps) + 64)
    if args.layers:
        cfg = cfg.with_(num_layers=args.layers)
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    ctx = dllm.initKernels(0, cfg)
    ctx.set_stream(stream.cuda_stream)
    ld = dllm.LeaderPipeline(ctx, (0, cfg.num_layers))
    bufs = device_weights(ctx, ld.stage, cfg, 0, cfg.num_layers, embed=True, head=True)
    ld.stage.fill_kv_random(0, args.kv_len, seed=1)
    ctx.synchronize(120000)
    first = 1234
    # warmup (graph capture happens on the first call)
    ld.decode_enqueue(first, args.warmup)
    toks = ld.read_tokens(args.warmup)
    t_start = ld.stage.T0
    launches0 = ctx.launch_count
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        torch.cuda.synchronize()
        ev0.record(stream)
        ld.decode_enqueue(toks[-1], args.steps)
        ev1.record(stream)
        ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    out = ld.read_tokens(args.steps)
    launches = ctx.launch_count - launches0
    tps = args.steps / (ms / 1000.0)
    avg_pos = t_start + (args.steps - 1) / 2.0 + 1
    bytes_tok = token_bytes(cfg, cfg.num_layers, head=True, embed=True, kv_positions=avg_pos)
    peak, peak_kind = measured_peaks()
    achieved = bytes_tok / (ms / 1000.0 / args.steps) / 1e9
    traffic = traffic_bytes(bytes_tok, args.model)
    # e2e: public generate call, token in from / out to host every step
    e2e_steps = args.steps
    gen_out = []
    ld.onToken = gen_out.append
    ld.generate([out[-1]], 2)  # warm the e2e graph
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ld.generate([out[-1]], e2e_steps)
    e2e_s = time.perf_counter() - t0
    e2e_tps = len(gen_out[2:]) / e2e_s if len(gen_out) > 2 else None
    res = {"metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "bf16", "data": "synthetic: random-init N(0,0.02) bf16 weights (device hash), N(0,1) bf16 KV",
           "config": workload_config(args, cfg),
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                        "traffic": traffic, "peak_kind": peak_kind, "algorithmic_bytes_per_launch": bytes_tok,
                        "kernel": "stage_kernel (one persistent launch per token)"},
           "e2e": {"value": e2e_tps, "unit": UNIT, "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                   "api": "LeaderPipeline.generate -> dllm_leader_generate"},
           "gpu_launches": launches, "clocks": clk.summary()}
    if not args.no_cpu_baseline:
        try:
            res["cpu_baseline"] = cpu_baseline(cfg, args.cpu_steps, args.kv_len)
        except Exception as e:  # reported, never silently replaced
            res["cpu_baseline"] = {"value": None, "error": repr(e)}
    del bufs
    ld.close()
    ctx.close()
    return res


# ---- our arm, one GPU, several sequences per step ---------------------------------------
def run_single_micro(args):
    """`--micro m` on one GPU: m sequences decoded together, one pass of m rows per
    step (Stage.forward_rows with the embedding and LM head fused in): up to 8
    rows through the persistent stage kernel, 16+ rows through the wide pass whose
    projections run on the tensor cores (tcgen05). Tokens stay on the device and
    feed the next step; value = tokens of all sequences per second."""
    import torch
    dllm = importlib.import_module("distributed-llm1_b200")
    m = args.micro
    cfg = dllm.PRESETS[args.model].with_(kv_dtype="bf16", max_seqs=m,
                                         max_pos=args.kv_len + args.warmup + args.steps + 16)
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx = dllm.initKernels(0, cfg)
    ctx.set_stream(stream.cuda_stream)
    if args.tc_rows is not None:
        ctx.set_tensor_core_rows(args.tc_rows)
    st = dllm.Stage(ctx, 0, cfg.num_layers)
    bufs = device_weights(ctx, st, cfg, 0, cfg.num_layers, embed=True, head=True)
    for q in range(m):
        st.fill_kv_random(q, args.kv_len, seed=1 + q)
    ctx.synchronize(120000)
    h = torch.zeros(m, cfg.hidden_size, dtype=torch.float32, device="cuda")
    tok = (torch.arange(m, dtype=torch.int32, device="cuda") * 7919 + 1000) % cfg.vocab_size
    seqs = list(range(m))

    def step():
        st.forward_rows(h.data_ptr(), seqs, tok.data_ptr(), tok.data_ptr())

    for _ in range(args.warmup):
        step()
    ctx.synchronize(120000)
    launches0 = ctx.launch_count
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        ev1.synchronize()
    ctx.synchronize(120000)
    ms = ev0.elapsed_time(ev1)
    tps = args.steps * m / (ms / 1000.0)
    avg_pos = args.kv_len + args.warmup + (args.steps - 1) / 2.0 + 1
    one = token_bytes(cfg, cfg.num_layers, head=True, embed=True, kv_positions=avg_pos)
    kv_one = cfg.num_layers * 2 * cfg.num_kv_heads * cfg.head_dim * 2 * avg_pos
    step_bytes = one + (m - 1) * (kv_one + 2 * cfg.hidden_size)  # weights once, KV and embedding row per sequence
    peak, peak_kind = measured_peaks()
    achieved = step_bytes / (ms / 1000.0 / args.steps) / 1e9
    tc = 8 if args.tc_rows is None else args.tc_rows
    wide = tc > 0 and m >= tc
    res = {"metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "bf16", "data": "synthetic: random-init N(0,0.02) bf16 weights (device hash), N(0,1) bf16 KV",
           "config": {"workload": f"{args.model} greedy decode of {m} sequences per step on one GPU, "
                                  f"{args.kv_len}-slot synthetic bf16 KV each", "batch": m, "kv_len": args.kv_len,
                      "parallelism": "pp1", "kv_dtype": "bf16", "weights": "bf16",
                      "path": "wide pass: tcgen05 projections, one kernel per op" if wide else
                              "persistent stage kernel, one launch per step",
                      "tensor_core_rows": args.tc_rows},
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                        "traffic": None, "peak_kind": peak_kind, "algorithmic_bytes_per_launch": step_bytes},
           "gpu_launches": ctx.launch_count - launches0, "clocks": clk.summary()}
    del bufs
    st.close()
    ctx.close()
    return res


# ---- isolated kernel sweep ------------------------------------------------------------------
SWEEP_SHAPES = [(896, 1152), (1536, 8960), (3584, 18944), (18944, 3584), (3584, 152064)]
SWEEP_ATTN = [1024, 4096, 16384, 32768]


def run_kernel_sweep(args):
    """CUDA-event time per launch of each kernel in isolation, with an L2 flush
    (a 512 MB write) before every timed launch, and its fraction of the measured
    HBM copy peak: matvec (one row; the stage kernel's matvec phase as an op) and
    the tcgen05 GEMM (16 and 64 rows) at the sweep shapes, decode attention over
    1k-32k slots (28 Q / 4 KV heads, head_dim 128; the reference's fp32 cache
    layout), and RMSNorm + RoPE of one row at hidden 3584."""
    import numpy as np
    import torch
    dllm = importlib.import_module("distributed-llm1_b200")
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()  # not the legacy default stream: its NULL handle means "the ctx's own stream"
    torch.cuda.set_stream(stream)  # the L2 flush, the ops and the events all run on it
    peak, peak_kind = measured_peaks()
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    lines = []

    def timed(fn, iters=20, warm=3):
        for _ in range(warm):
            fn()
        ts = []
        for _ in range(iters):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e-3)
        return float(np.median(ts))

    def emit(kernel, shape, sec, nbytes, flops=None, launches=1):
        d = {"sweep": kernel, "shape": shape, "us": sec * 1e6, "bytes": nbytes, "gbs": nbytes / sec / 1e9,
             "hbm_frac": nbytes / sec / 1e9 / peak, "peak_gbs": peak, "peak_kind": peak_kind,
             "kernel_launches": launches}
        if flops:
            d["tflops"] = flops / sec / 1e12
        print(json.dumps(d), flush=True)
        lines.append(d)

    cfg = dllm.PRESETS["qwen2.5-7b"].with_(num_layers=1, kv_dtype="f32", max_pos=max(SWEEP_ATTN) + 8)
    ctx = dllm.initKernels(0, cfg)
    ctx.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(0)
    which = args.kernel_sweep
    rows = {"all": (1, 16, 64), "matvec": (1,), "gemm": (16, 64)}.get(which, ())
    for K, N in (SWEEP_SHAPES if rows else []):
        w = ctx.createBf16(K * N, "w")
        ctx.fillNormalBf16(w, K + N, WEIGHT_STD)
        for n in rows:
            x = ctx.createF32(n * K, "x")
            ctx.writeF32(x, rng.standard_normal(n * K).astype(np.float32))
            # the output buffer is dropped at once and comes back from the ctx's buffer cache
            sec = timed(lambda: ctx.matmul(x, w, n, K, N))
            nbytes = 2 * K * N + 4 * n * (K + N)
            emit("matvec (CUDA cores)" if n == 1 else "GEMM (tcgen05, hi+lo bf16 activations)",
                 f"n={n} [K={K},N={N}]", sec, nbytes, flops=2.0 * n * K * N, launches=1 if n == 1 else 2)
        del w
    QD, KD = cfg.num_q_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim
    kc = ctx.createF32(cfg.max_pos * KD, "k")
    vc = ctx.createF32(cfg.max_pos * KD, "v")
    ctx.writeF32(kc, rng.standard_normal(cfg.max_pos * KD).astype(np.float32))
    ctx.writeF32(vc, rng.standard_normal(cfg.max_pos * KD).astype(np.float32))
    q = ctx.createF32(QD, "q")
    ctx.writeF32(q, rng.standard_normal(QD).astype(np.float32))
    for T in (SWEEP_ATTN if which in ("all", "attention") else []):
        sec = timed(lambda: ctx.attention(q, kc, vc, T - 1, 1))
        emit("decode attention (fp32 cache, reference layout)", f"T={T} 28/4 heads hd=128", sec,
             2 * T * KD * 4 + 2 * QD * 4)
    if which not in ("all", "norm"):
        ctx.close()
        return lines
    D = cfg.hidden_size
    h = ctx.createF32(D, "h")
    ctx.writeF32(h, rng.standard_normal(D).astype(np.float32))
    g = ctx.createBf16(D, "g")
    ctx.fillConstBf16(g, 1.0)
    sec = timed(lambda: ctx.rmsnorm(h, g, 1))
    emit("rmsnorm", "1 row, hidden 3584", sec, D * 4 * 2 + D * 2)
    sec = timed(lambda: ctx.ropeQ(q, 2048, 1))
    emit("rope (q, 28 heads)", "1 row, theta 1e6", sec, QD * 4 * 2)
    ctx.close()
    return lines


# ---- per-phase trace of the stage kernel ------------------------------------------------------
PHASES = ["qkv", "attention", "o_proj", "mlp"]


def run_phase_trace(args, tokens: int = 5):
    """Decode `tokens` single tokens with the stage kernel's global-timer trace on
    (CTA 0 stamps kernel start and every grid barrier) and report the median time
    of each phase per layer (layers after the first), the phases' algorithmic HBM
    bytes (bf16 weights; bf16 K and V of the attended slots) and their fraction of
    the measured HBM copy peak. With one row and the split-K MLP a layer has four
    phases: QKV (RMSNorm, q|k|v, bias, RoPE, KV append), attention, o_proj +
    residual, MLP (RMSNorm, gate|up, SiLU, split-K down_proj into the fixed-point
    sums)."""
    import numpy as np
    dllm = importlib.import_module("distributed-llm1_b200")
    syn = importlib.import_module("distributed-llm1_b200.synthetic")
    cfg = dllm.PRESETS[args.model].with_(kv_dtype="bf16", max_pos=args.kv_len + 64 + tokens + 8)
    if args.layers:
        cfg = cfg.with_(num_layers=args.layers)
    ctx = dllm.initKernels(0, cfg)
    ld = dllm.LeaderPipeline(ctx, (0, cfg.num_layers))
    bufs = syn.device_weights(ctx, ld.stage, cfg, 0, cfg.num_layers, True, True, 0)
    ld.stage.fill_kv_random(0, args.kv_len, seed=1)
    ctx.synchronize(120000)
    ld.decode_enqueue(1234, 8)
    toks = ld.read_tokens(8)
    cap = 8 * cfg.num_layers + 16
    ld.stage.set_trace(cap)
    runs = []
    for _ in range(tokens):
        ld.decode_enqueue(toks[-1], 1)
        toks = ld.read_tokens(1)
        t = ld.stage.read_trace(cap).astype(np.int64)
        runs.append(np.diff(t[:int(np.count_nonzero(t))]) / 1000.0)
    d = np.median(np.stack(runs), axis=0)
    L, k = cfg.num_layers, len(PHASES)
    assert len(d) >= 1 + k * L, f"unexpected trace length {len(d)} for {L} layers"
    per_layer = d[1:1 + k * L].reshape(L, k)
    body = per_layer[1:] if L > 1 else per_layer
    D, I, QD, KD = cfg.hidden_size, cfg.intermediate_size, cfg.num_q_heads * cfg.head_dim, \
        cfg.num_kv_heads * cfg.head_dim
    T = args.kv_len + 8 + (tokens + 1) / 2
    nbytes = {"qkv": 2 * D * (QD + 2 * KD), "attention": 2 * 2 * KD * T, "o_proj": 2 * QD * D,
              "mlp": 2 * 3 * D * I}
    peak, peak_kind = measured_peaks()
    phases = {}
    for i, name in enumerate(PHASES):
        us = float(np.mean(body[:, i]))
        phases[name] = {"us": us, "bytes": nbytes[name], "gbs": nbytes[name] / us / 1e3,
                        "hbm_frac": nbytes[name] / us / 1e3 / peak}
    tail = [float(x) for x in d[1 + k * L:]]
    res = {"phase_trace": args.model, "kv_len": args.kv_len, "layers": L, "tokens": tokens,
           "token_us": float(np.median([r.sum() for r in runs])), "layer_us": float(np.mean(body.sum(1))),
           "phases": phases, "tail_us": tail, "tail": "fold of the last layer's sums, then final norm + LM head + argmax",
           "peak_gbs": peak, "peak_kind": peak_kind}
    del bufs
    ld.close()
    ctx.close()
    return res


def main():
    args = parse_args()
    if args.kernel_sweep:
        run_kernel_sweep(args)
        return
    if args.phase_trace:
        print(json.dumps(run_phase_trace(args)), flush=True)
        return
    if args.impl == "reference":
        res = run_reference(args)
    elif args.gpus <= 1 and args.micro > 1:
        res = run_single_micro(args)
    elif args.gpus <= 1:
        res = run_single(args)
    else:
        from importlib import import_module
        mg = import_module("distributed-llm1_b200.multigpu")
        res = mg.bench_pipeline(args, sys.modules[__name__])
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
