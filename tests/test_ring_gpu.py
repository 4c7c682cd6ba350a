"""The multi-GPU pipeline behind the C ABI (dllm_pipeline_*, pipeline.js:6-87,
91-282): 2 stages on 2 GPUs, the hidden-row hop fused into the stage kernel over
NVLink. Every sequence's greedy tokens equal the one-GPU decode of the same
sequences and the oracle's decode (oracle/ref_forward.cpp), for the device
token ring and for the host-fed token loop (tokens relayed through the hosts, as
the reference's leader does). Needs 2 GPUs; runs tests/ring_worker.py under
torch.distributed.run."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_two_gpu_ring_matches_single_gpu_and_oracle(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "ring.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", os.path.join(HERE, "ring_worker.py"), str(out)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    steps = len(res["ring"])
    ring = [row for row in res["ring"]] + res["host"]
    assert ring == res["single"], f"ring {ring} != single GPU {res['single']}"
    assert ring == res["oracle"], f"ring {ring} != oracle {res['oracle']}"
    assert steps == 6 and len(res["host"]) == 3
