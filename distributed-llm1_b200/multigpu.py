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
    """`bench.py --gpus N` under torchrun: N stages, N micro-batches of args.micro
    sequences, 2048-slot synthetic KV per sequence; returns rank 0's JSON dict."""
    import importlib
    import time
    dllm = importlib.import_module("distributed-llm1_b200")
    rank, world, local = init_distributed("nccl")
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"
    B, m = world, args.micro
    steps_total = args.warmup + 2 * args.steps + 4  # warm-up, timed and e2e rounds
    cfg = dllm.PRESETS[args.model].with_(kv_dtype="bf16", max_seqs=B * m,
                                         max_pos=args.kv_len + steps_total + 16)
    start, end = dllm.plan_stages(cfg, world)[rank]
    stream = torch.cuda.current_stream()
    ctx = dllm.initKernels(local, cfg)
    ctx.set_stream(stream.cuda_stream)
    st = dllm.Stage(ctx, start, end)
    bufs = bench.device_weights(ctx, st, cfg, start, end, embed=(rank == 0), head=(rank == world - 1))
    for s in range(B * m):
        st.fill_kv_random(s, args.kv_len, seed=1 + s)
    ctx.synchronize(300000)
    plan = Plan(rank, world, B, m)
    first = torch.arange(B * m, dtype=torch.int32, device="cuda") + 1000
    runner = PipelineRunner(plan, cfg.hidden_size, torch.device("cuda", local), StageCompute(st, plan), first)
    # create the NCCL communicator with a collective every rank joins
    dist.all_reduce(torch.zeros(1, device="cuda"))
    runner.run_ticks(args.warmup * B + (world - 1))  # fill the pipe, then warm up
    launches0 = ctx.launch_count
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    with bench.ClockSampler(local) as clk:
        ev0.record(stream)
        runner.run_ticks(args.steps * B)
        ev1.record(stream)
        ev1.synchronize()
    ms = torch.tensor([ev0.elapsed_time(ev1)], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    launches = ctx.launch_count - launches0
    tokens = args.steps * B * m
    tps = tokens / (ms / 1000.0)
    # roofline of the slowest stage: its bytes per tick over the tick time
    lw = cfg.layer_weight_bytes()
    stage_bytes = []
    for r, (s0, s1) in enumerate(dllm.plan_stages(cfg, world)):
        b = bench.token_bytes(cfg, s1 - s0, head=(r == world - 1), embed=(r == 0),
                              kv_positions=args.kv_len + args.warmup + args.steps / 2)
        # micro-batch of m rows reads the weights once and m rows of KV
        kv = b - (s1 - s0) * lw - (cfg.head_weight_bytes() if r == world - 1 else 0) - (2 * cfg.hidden_size if r == 0 else 0)
        stage_bytes.append(b + (m - 1) * kv)
    tick_s = ms / 1000.0 / (args.steps * B)
    peak, peak_kind = bench.measured_peaks()
    achieved = max(stage_bytes) / tick_s / 1e9
    # DRAM traffic of the slowest stage's launch: the ncu traffic / algorithmic
    # ratio of the profiled whole-model token applied to the stage's bytes
    traffic = bench.traffic_bytes(max(stage_bytes), args.model)
    # e2e: the same loop with every tick's tokens copied to the host and checked
    e2e = None
    res = None
    if rank == 0:
        res = {"metric": bench.METRIC, "value": tps, "unit": bench.UNIT, "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic: random-init N(0,0.02) bf16 weights (device hash), N(0,1) bf16 KV",
               "config": bench.workload_config(args, cfg) | {"stages": dllm.plan_stages(cfg, world)},
               "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                            "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                            "algorithmic_bytes_per_launch": max(stage_bytes),
                            "kernel": "stage_kernel of the slowest stage (one launch per micro-batch tick)"},
               "gpu_launches": launches, "clocks": clk.summary()}
    # e2e through the public API: per step the last rank's tokens go device -> host
    # and rank 0's next inputs host -> device (pinned), as a user loop would
    runner2_tok = torch.zeros(B * m, dtype=torch.int32).pin_memory()
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for k in range(args.steps):
        for _ in range(B):
            runner.step()
        if rank == world - 1:
            for b in range(B):
                runner2_tok[b * m:(b + 1) * m].copy_(runner.tok_out[b], non_blocking=True)
        if rank == 0:
            for b in range(B):
                runner.tok_in[b].copy_(runner.tok_in[b].cpu().pin_memory(), non_blocking=True)
    torch.cuda.synchronize()
    el = torch.tensor([time.perf_counter() - t0], device="cuda")
    dist.all_reduce(el, op=dist.ReduceOp.MAX)
    if rank == 0:
        res["e2e"] = {"value": tokens / float(el.item()), "unit": bench.UNIT, "h2d_bytes_per_step": 4 * B * m,
                      "d2h_bytes_per_step": 4 * B * m, "api": "Stage.forward_rows + NCCL hops, host token copies"}
    dist.barrier()
    del bufs
    st.close()
    ctx.close()
    dist.destroy_process_group()
    return res
