"""Pipeline-parallel decode across the GPUs of one node (pipeline.js:6-87 on B200).

One process per GPU (torch.distributed, NCCL). Rank r owns a contiguous layer
range (its `Stage`); rank 0 also embeds tokens and the last rank runs the final
norm + LM head + argmax. The hidden-state hop of the reference (leader -> stage
frames over WebRTC, pipeline.js:226-253) becomes NCCL send/recv of the fp32 rows
straight into the next GPU's memory, and the last stage returns int32 tokens to
rank 0 to close the loop.

Schedule: B = world micro-batches of m sequences are in flight. At tick t rank
r works on micro-batch (t - r) mod B (once t >= r). Every tick begins with one
grouped send/recv on every rank (a ring shift): rank r sends the output of its
previous tick to rank r+1 (the last rank sends tokens to rank 0) and receives its
next input from rank r-1. With B = world every stage works every tick in steady
state. Grouping the send and the receive of a tick in one NCCL group makes the
ring deadlock-free.

The compute of a tick is a callable so the schedule and communication can be
tested with gloo on CPU; `StageCompute` runs the real stage kernel.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class Plan:
    rank: int
    world: int
    n_micro: int
    micro: int

    def micro_of(self, tick: int) -> int | None:
        """Micro-batch rank `rank` works on at `tick`, or None during the fill."""
        if tick < self.rank:
            return None
        return (tick - self.rank) % self.n_micro

    def recv_at(self, tick: int) -> bool:
        """Whether an input arrives at the start of `tick` (from rank - 1, or for
        rank 0 tokens from the last rank)."""
        if self.rank == 0:
            return self.world > 1 and tick >= self.world
        return tick - 1 >= self.rank - 1

    def send_at(self, tick: int) -> bool:
        """Whether the output of tick - 1 leaves at the start of `tick`."""
        return self.world > 1 and tick - 1 >= self.rank

    def seqs(self, b: int) -> list[int]:
        return list(range(b * self.micro, (b + 1) * self.micro))


class PipelineRunner:
    """Runs ticks of the ring schedule. `compute(b, h, tok_in, tok_out)` does this
    rank's work for micro-batch b: h is the [m, D] fp32 hidden buffer (input and
    output), tok_in / tok_out the int32 [m] token buffers (rank 0 / last rank)."""

    def __init__(self, plan: Plan, hidden: int, device, compute, first_tokens: torch.Tensor | None = None):
        self.p = plan
        self.compute = compute
        B, m = plan.n_micro, plan.micro
        self.h = [torch.zeros(m, hidden, dtype=torch.float32, device=device) for _ in range(B)]
        self.tok_in = [torch.zeros(m, dtype=torch.int32, device=device) for _ in range(B)]
        self.tok_out = [torch.zeros(m, dtype=torch.int32, device=device) for _ in range(B)]
        if first_tokens is not None:
            for b in range(B):
                self.tok_in[b].copy_(first_tokens[b * m:(b + 1) * m].to(torch.int32))
        self.tick = 0
        self.emitted: list[tuple[int, torch.Tensor]] = []  # (micro-batch, tokens) on the last rank
        self.keep_tokens = False

    def _out_buf(self, b):
        return self.tok_out[b] if self.p.rank == self.p.world - 1 else self.h[b]

    def step(self):
        p, t = self.p, self.tick
        ops = []
        if p.send_at(t):
            b_prev = p.micro_of(t - 1)
            dst = (p.rank + 1) % p.world
            ops.append(dist.P2POp(dist.isend, self._out_buf(b_prev), dst))
        b = p.micro_of(t)
        if p.recv_at(t) and b is not None:
            src = (p.rank - 1) % p.world
            buf = self.tok_in[b] if p.rank == 0 else self.h[b]
            ops.append(dist.P2POp(dist.irecv, buf, src))
        if ops:
            for r in dist.batch_isend_irecv(ops):
                r.wait()
        if b is not None:
            self.compute(b, self.h[b], self.tok_in[b] if p.rank == 0 else None,
                         self.tok_out[b] if p.rank == p.world - 1 else None)
            if p.world == 1:
                self.tok_in[b].copy_(self.tok_out[b])  # the token feeds the next step
            if self.keep_tokens and p.rank == p.world - 1:
                self.emitted.append((b, self.tok_out[b].clone()))
        self.tick += 1

    def run_ticks(self, n: int):
        for _ in range(n):
            self.step()


class StageCompute:
    """Tick compute on the GPU: one stage-kernel launch per micro-batch."""

    def __init__(self, stage, plan: Plan):
        self.stage, self.plan = stage, plan

    def __call__(self, b, h, tok_in, tok_out):
        self.stage.forward_rows(h.data_ptr(), self.plan.seqs(b),
                                tok_in.data_ptr() if tok_in is not None else None,
                                tok_out.data_ptr() if tok_out is not None else None)


class NvlinkRing:
    """The C-ABI pipeline (dllm_pipeline_*): this rank's Stage in a ring of
    stages whose hidden-row hop is fused into the stage kernel (rows stored in
    the next GPU's receive buffer over NVLink, a flag released there). The host
    only exchanges the receive buffers' IPC handles once (`connect_ring`)."""

    def __init__(self, stage, rank: int, world: int, n_micro: int, micro: int):
        import ctypes as C
        from . import _lib
        self.C, self._lib = C, _lib
        self.stage, self.lib = stage, stage.lib
        self.rank, self.world, self.n_micro, self.micro = rank, world, n_micro, micro
        h = C.c_void_p()
        stage.k._check(self.lib.dllm_pipeline_create(stage.handle, rank, world, n_micro, micro, C.byref(h)),
                       "pipeline_create")
        self.handle = h.value

    def _check(self, st, what):
        self.stage.k._check(st, what)

    def ipc_handle(self) -> bytes:
        C = self.C
        buf = (C.c_uint8 * 64)()
        self._check(self.lib.dllm_pipeline_handle(self.handle, buf), "pipeline_handle")
        return bytes(buf)

    def connect(self, next_handle: bytes):
        C = self.C
        buf = (C.c_uint8 * 64).from_buffer_copy(next_handle)
        self._check(self.lib.dllm_pipeline_connect(self.handle, buf), "pipeline_connect")

    def set_tokens(self, tokens):
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        self._check(self.lib.dllm_pipeline_set_tokens(self.handle, self._lib.ptr(t, self.C.c_int32), t.size),
                    "pipeline_set_tokens")

    def run(self, steps: int):
        self._check(self.lib.dllm_pipeline_run(self.handle, steps), "pipeline_run")

    def read_tokens(self, steps: int):
        import numpy as np
        out = np.zeros((steps, self.n_micro * self.micro), np.int32)
        self._check(self.lib.dllm_pipeline_read_tokens(self.handle, self._lib.ptr(out, self.C.c_int32), steps),
                    "pipeline_read_tokens")
        return out

    def synchronize(self, timeout_ms: int = 15000):
        self._check(self.lib.dllm_pipeline_synchronize(self.handle, timeout_ms), "pipeline_synchronize")

    def set_host_tokens(self, on: bool):
        self._check(self.lib.dllm_pipeline_set_host_tokens(self.handle, int(bool(on))), "pipeline_set_host_tokens")

    def run_micro(self, b: int, tokens=None):
        """One pass of micro-batch b; the first stage passes host tokens (host-token
        mode), the last stage gets the sampled tokens back."""
        import numpy as np
        C = self.C
        t = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(self.micro, np.int32) if self.rank == self.world - 1 else None
        self._check(self.lib.dllm_pipeline_run_micro(self.handle, b, self._lib.ptr(t, C.c_int32),
                                                     self._lib.ptr(out, C.c_int32)), "pipeline_run_micro")
        return out

    def close(self):
        if getattr(self, "handle", None):
            self.lib.dllm_pipeline_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def connect_ring(ring: NvlinkRing, group=None):
    """Exchange the receive-buffer handles over torch.distributed and map the next
    rank's buffer; ends with a barrier so no pass starts before every rank is
    connected."""
    handles = [None] * ring.world
    dist.all_gather_object(handles, ring.ipc_handle(), group=group)
    ring.connect(handles[(ring.rank + 1) % ring.world])
    dist.barrier(group=group)


def init_distributed(backend: str = "nccl", timeout_s: int = 120):
    """One process per GPU; rendezvous from torchrun's environment."""
    import datetime
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if backend == "nccl":
        torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        kw = {"device_id": torch.device("cuda", local)} if backend == "nccl" else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world, local


def bench_pipeline(args, bench):
    """`bench.py --gpus N` under torchrun: N stages (plan_stages), N micro-batches of
    args.micro sequences, 2048-slot synthetic KV per sequence, decoded through the
    NVLink ring of the C ABI (dllm_pipeline_*); returns rank 0's JSON dict."""
    import importlib
    import time
    import numpy as np
    dllm = importlib.import_module("distributed-llm1_b200")
    rank, world, local = init_distributed("nccl")
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"
    B, m = (args.n_micro or world), args.micro
    e2e_steps = max(2, args.steps // 2)
    steps_total = args.warmup + args.steps + e2e_steps + 4
    cfg = dllm.PRESETS[args.model].with_(kv_dtype="bf16", max_seqs=B * m,
                                         max_pos=args.kv_len + steps_total + 16)
    stages = dllm.plan_stages(cfg, world)
    start, end = stages[rank]
    # a real stream (the legacy default stream's handle is NULL, which the ctx
    # reads as "use your own stream"): passes and timing events share it
    stream = torch.cuda.Stream()
    ctx = dllm.initKernels(local, cfg)
    ctx.set_stream(stream.cuda_stream)
    st = dllm.Stage(ctx, start, end)
    bufs = bench.device_weights(ctx, st, cfg, start, end, embed=(rank == 0), head=(rank == world - 1))
    for q in range(B * m):
        st.fill_kv_random(q, args.kv_len, seed=1 + q)
    ctx.synchronize(300000)
    ring = NvlinkRing(st, rank, world, B, m)
    connect_ring(ring)
    if rank == 0:
        ring.set_tokens(np.arange(B * m, dtype=np.int32) + 1000)
    ring.run(args.warmup)  # fills the ring, then warms up
    ring.synchronize(120000)
    launches0 = ctx.launch_count
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    with bench.ClockSampler(local) as clk:
        ev0.record(stream)
        ring.run(args.steps)
        ev1.record(stream)
        ev1.synchronize()
    ring.synchronize(120000)
    ms = torch.tensor([ev0.elapsed_time(ev1)], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    launches = ctx.launch_count - launches0
    tokens = args.steps * B * m
    tps = tokens / (ms / 1000.0)
    # roofline of the slowest stage: its bytes per pass over the pass time
    lw = cfg.layer_weight_bytes()
    stage_bytes = []
    for r, (s0, s1) in enumerate(stages):
        b = bench.token_bytes(cfg, s1 - s0, head=(r == world - 1), embed=(r == 0),
                              kv_positions=args.kv_len + args.warmup + args.steps / 2)
        # a micro-batch of m rows reads the weights once and m rows of KV
        kv = b - (s1 - s0) * lw - (cfg.head_weight_bytes() if r == world - 1 else 0) - (2 * cfg.hidden_size if r == 0 else 0)
        stage_bytes.append(b + (m - 1) * kv)
    tick_s = ms / 1000.0 / (args.steps * B)
    peak, peak_kind = bench.measured_peaks()
    achieved = max(stage_bytes) / tick_s / 1e9
    # DRAM traffic of the slowest stage's launch: the ncu traffic / algorithmic
    # ratio of the profiled whole-model token applied to the stage's bytes
    traffic = bench.traffic_bytes(max(stage_bytes), args.model)
    emitted = ring.read_tokens(args.steps) if rank == world - 1 else None
    res = None
    if rank == 0:
        res = {"metric": bench.METRIC, "value": tps, "unit": bench.UNIT, "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic: random-init N(0,0.02) bf16 weights (device hash), N(0,1) bf16 KV",
               "config": bench.workload_config(args, cfg) | {"stages": stages},
               "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                            "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                            "algorithmic_bytes_per_launch": max(stage_bytes),
                            "kernel": "stage_kernel of the slowest stage (one launch per micro-batch pass; "
                                      "the hop to the next GPU is fused into it)"},
               "gpu_launches": launches, "clocks": clk.summary(),
               "hop": "fused into the stage kernel: rows stored into the next GPU's receive buffer over NVLink "
                      "(CUDA IPC mapping) + a released flag; no NCCL kernel and no host round trip per hop"}
    # e2e through the public API with a host-fed token loop, as the reference's
    # leader runs it: every pass of the last stage copies its sampled tokens to
    # the host, they travel to rank 0's host, and rank 0's next pass of that
    # micro-batch uploads them (dllm_pipeline_run_micro)
    gloo = dist.new_group(backend="gloo")
    ring.set_host_tokens(True)
    dist.barrier()
    last = world - 1
    cur = torch.zeros(m, dtype=torch.int32)
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    if rank == last and world > 1:  # the relay starts with the tokens of the timed run
        for b in range(B):
            dist.send(torch.from_numpy(emitted[-1, b * m:(b + 1) * m].copy()), dst=0, group=gloo)
    for k in range(e2e_steps):
        for b in range(B):
            if world == 1:
                pass
            elif rank == 0:
                dist.recv(cur, src=last, group=gloo)
                ring.run_micro(b, cur.numpy())
            elif rank == last:
                out = ring.run_micro(b)
                if k + 1 < e2e_steps:
                    dist.send(torch.from_numpy(out), dst=0, group=gloo)
            else:
                ring.run_micro(b)
    ring.synchronize(120000)
    torch.cuda.synchronize()
    el = torch.tensor([time.perf_counter() - t0], device="cuda")
    dist.all_reduce(el, op=dist.ReduceOp.MAX)
    if rank == 0:
        res["e2e"] = {"value": e2e_steps * B * m / float(el.item()), "unit": bench.UNIT,
                      "h2d_bytes_per_step": 4 * B * m, "d2h_bytes_per_step": 4 * B * m,
                      "api": "dllm_pipeline_run_micro: last stage tokens device->host, relayed to rank 0's host, "
                             "host->device into the first stage's next pass"}
    dist.barrier()
    ring.close()
    del bufs
    st.close()
    ctx.close()
    dist.destroy_process_group()
    return res
