"""The multi-GPU ring schedule (multigpu.py) on CPU: world sizes 1-3 with the
gloo backend and a stand-in stage compute. Every micro-batch's token stream
must equal a serial run of the same stage chain, whatever the world size."""
import importlib
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

D = 8
VOCAB = 997


def stage_fn(rank, world, h, tok_in, tok_out):
    """Deterministic stand-in for stage `rank` of `world`."""
    if rank == 0:
        h.copy_(tok_in.float()[:, None] * 0.25 + torch.arange(D, dtype=torch.float32)[None, :])
    h.mul_(1.01).add_(rank + 1)
    if rank == world - 1:
        tok_out.copy_((h.sum(dim=1) * 13).long().remainder(VOCAB).to(torch.int32))


def serial(world, n_micro, micro, first, steps):
    out = {b: [] for b in range(n_micro)}
    for b in range(n_micro):
        tok = first[b * micro:(b + 1) * micro].clone()
        for _ in range(steps):
            h = torch.zeros(micro, D)
            nxt = torch.zeros(micro, dtype=torch.int32)
            for r in range(world):
                stage_fn(r, world, h, tok, nxt)
            out[b].append(nxt.clone())
            tok = nxt
    return out


def worker(rank, world, port, path, n_micro, micro, rounds):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    mg = importlib.import_module("distributed-llm1_b200.multigpu")
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world)
    plan = mg.Plan(rank, world, n_micro, micro)
    first = torch.arange(n_micro * micro, dtype=torch.int32) * 3 + 1
    runner = mg.PipelineRunner(plan, D, "cpu", lambda b, h, ti, to: stage_fn(rank, world, h, ti, to), first)
    runner.keep_tokens = True
    runner.run_ticks(rounds * n_micro + world - 1)
    if rank == world - 1:
        torch.save(runner.emitted, path)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,micro", [(1, 2), (2, 1), (3, 2)])
def test_ring_schedule_matches_serial(world, micro):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if root not in sys.path:
        sys.path.insert(0, root)
    n_micro, rounds = world, 4
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "tokens.pt")
        if world == 1:
            worker(0, 1, 0, path, n_micro, micro, rounds)
        else:
            mp.start_processes(worker, args=(world, free_port(), path, n_micro, micro, rounds), nprocs=world,
                               start_method="spawn", join=True)
        emitted = torch.load(path)
    first = torch.arange(n_micro * micro, dtype=torch.int32) * 3 + 1
    want = serial(world, n_micro, micro, first, rounds)
    got = {b: [] for b in range(n_micro)}
    for b, toks in emitted:
        got[b].append(toks)
    for b in range(n_micro):
        assert len(got[b]) == rounds
        for k in range(rounds):
            assert torch.equal(got[b][k], want[b][k]), (b, k, got[b][k], want[b][k])


def test_plan_fill_and_steady_state():
    mg = importlib.import_module("distributed-llm1_b200.multigpu")
    for world in (2, 4, 8):
        for r in range(world):
            p = mg.Plan(r, world, world, 1)
            assert p.micro_of(r - 1) is None and p.micro_of(r) == 0
            # every tick after the fill, every rank is busy on a distinct micro-batch
        t = 3 * world
        assert sorted(mg.Plan(r, world, world, 1).micro_of(t) for r in range(world)) == list(range(world))
        # the receiving rank expects exactly what the sending rank sends
        for r in range(world):
            nxt = (r + 1) % world
            for tick in range(4 * world):
                assert mg.Plan(r, world, world, 1).send_at(tick) == mg.Plan(nxt, world, world, 1).recv_at(tick)


def failing_worker(rank, world, port, path):
    """Rank 1's stage fails at tick 3 and the rank leaves; rank 0 records how its
    own run ended and how long that took."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    mg = importlib.import_module("distributed-llm1_b200.multigpu")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    plan = mg.Plan(rank, world, world, 1)
    first = torch.arange(world, dtype=torch.int32) + 1
    runner = None

    def compute(b, h, ti, to):
        if rank == 1 and runner.tick >= 3:
            raise RuntimeError("stage 1 failed")
        stage_fn(rank, world, h, ti, to)

    runner = mg.PipelineRunner(plan, D, "cpu", compute, first)
    t0 = time.time()
    try:
        runner.run_ticks(40)
        outcome = "completed"
    except Exception as e:  # the failure, or the peer's disappearance
        outcome = type(e).__name__
    if rank == 0:
        with open(path, "w") as f:
            f.write(f"{outcome} {time.time() - t0:.2f} {runner.tick}")
    os._exit(0)  # the peer is gone: no collective teardown


def test_stage_failure_surfaces_on_other_ranks():
    """A rank whose stage raises leaves between ticks; the other rank's next
    exchange ends with an error within the process-group timeout instead of
    hanging (failure detection on the host, no GPU involved)."""
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if root not in sys.path:
        sys.path.insert(0, root)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "outcome.txt")
        mp.start_processes(failing_worker, args=(2, free_port(), path), nprocs=2, start_method="spawn", join=True)
        outcome, secs, tick = open(path).read().split()
    assert outcome != "completed"
    assert float(secs) < 30.0
    assert 3 <= int(tick) < 40
