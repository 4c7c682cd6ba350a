"""Worker of tests/test_ring_gpu.py, run as one process per GPU under
torch.distributed.run: a 2-stage NVLink ring (dllm_pipeline_*) decodes 4
sequences in 2 micro-batches; rank 0 then decodes the same sequences on one GPU
(one Stage with every layer) and with the oracle, and writes all three token
streams to the JSON file given as the first argument."""
import importlib
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, HERE, os.path.join(ROOT, "oracle")):
    sys.path.insert(0, p)

STEPS, HOST_STEPS = 6, 3
LENS = [20, 29, 38, 47]
FIRST = [11, 22, 33, 44]
SPLIT = [(0, 2), (2, 4)]


def main(out_path):
    dllm = importlib.import_module("distributed-llm1_b200")
    mg = importlib.import_module("distributed-llm1_b200.multigpu")
    syn = importlib.import_module("distributed-llm1_b200.synthetic")
    rank, world, local = mg.init_distributed("nccl", timeout_s=120)
    assert world == 2
    cfg = dllm.PRESETS["qwen2.5-0.5b"].with_(num_layers=4, kv_dtype="bf16", max_seqs=4, max_pos=96)
    s0, s1 = SPLIT[rank]
    ctx = dllm.initKernels(local, cfg)
    st = dllm.Stage(ctx, s0, s1)
    syn.device_weights(ctx, st, cfg, s0, s1, embed=(rank == 0), head=(rank == world - 1), seed=3)
    for q, n in enumerate(LENS):
        st.fill_kv_random(q, n, seed=7)
    ctx.synchronize(60000)
    ring = mg.NvlinkRing(st, rank, world, 2, 2)
    mg.connect_ring(ring)
    if rank == 0:
        ring.set_tokens(FIRST)
    ring.run(STEPS)
    ring.synchronize(60000)
    ring_tokens = ring.read_tokens(STEPS).tolist() if rank == world - 1 else None
    # host-token loop (dllm_pipeline_run_micro): tokens relayed through the hosts
    gloo = dist.new_group(backend="gloo")
    ring.set_host_tokens(True)
    dist.barrier()
    host_tokens = []
    cur = torch.zeros(2, dtype=torch.int32)
    if rank == 1:
        for b in range(2):
            dist.send(torch.tensor(ring_tokens[-1][2 * b:2 * b + 2], dtype=torch.int32), dst=0, group=gloo)
    for k in range(HOST_STEPS):
        row = []
        for b in range(2):
            if rank == 0:
                dist.recv(cur, src=1, group=gloo)
                ring.run_micro(b, cur.numpy())
            else:
                out = ring.run_micro(b)
                row += out.tolist()
                if k + 1 < HOST_STEPS:
                    dist.send(torch.from_numpy(out), dst=0, group=gloo)
        host_tokens.append(row)
    ring.synchronize(60000)
    got = [None, None]
    dist.all_gather_object(got, {"ring": ring_tokens, "host": host_tokens})
    ring.close()
    st.close()
    ctx.close()
    dist.barrier()
    if rank == 0:
        res = {"ring": got[1]["ring"], "host": got[1]["host"]}
        res.update(single_gpu_and_oracle(dllm, syn, cfg))
        with open(out_path, "w") as f:
            json.dump(res, f)
    dist.destroy_process_group()


def single_gpu_and_oracle(dllm, syn, cfg):
    """The same 4 sequences on one GPU (all layers, forward_rows per micro-batch)
    and through the oracle's decode step (oracle/ref_forward.cpp, bf16 KV)."""
    import ref_forward as ref
    from helpers import RefModel, ref_lib
    ctx = dllm.initKernels(0, cfg)
    st = dllm.Stage(ctx, 0, cfg.num_layers)
    syn.device_weights(ctx, st, cfg, 0, cfg.num_layers, embed=True, head=True, seed=3)
    for q, n in enumerate(LENS):
        st.fill_kv_random(q, n, seed=7)
    ctx.synchronize(60000)
    W = syn.read_back(ctx, st)
    kv = {q: [(st.kv[L].k.read(0, n, seq=q), st.kv[L].v.read(0, n, seq=q)) for L in range(cfg.num_layers)]
          for q, n in enumerate(LENS)}
    h = torch.zeros(2, cfg.hidden_size, dtype=torch.float32, device="cuda")
    tin = torch.tensor(FIRST, dtype=torch.int32, device="cuda")
    tout = torch.zeros(4, dtype=torch.int32, device="cuda")
    single = []
    for k in range(STEPS + HOST_STEPS):
        for b in range(2):
            st.forward_rows(h.data_ptr(), [2 * b, 2 * b + 1], tin[2 * b:].data_ptr(), tout[2 * b:].data_ptr())
        torch.cuda.synchronize()
        ctx.synchronize()
        single.append(tout.cpu().tolist())
        tin.copy_(tout)
    st.close()
    ctx.close()
    lib = ref_lib()
    lib.ref_set_threads(os.cpu_count() or 1)
    ocfg = ref.Config(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, num_layers=cfg.num_layers,
                      num_q_heads=cfg.num_q_heads, num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                      intermediate_size=cfg.intermediate_size, tie_word_embeddings=cfg.tie_word_embeddings,
                      max_pos=cfg.max_pos)
    oracle = []
    for q, n in enumerate(LENS):
        rm = RefModel(lib, ocfg, W, kv_bf16=True)
        for L in range(cfg.num_layers):
            rm.set_kv(L, 0, 0, kv[q][L][0])
            rm.set_kv(L, 1, 0, kv[q][L][1])
        rm.T0 = n
        tok, seq = FIRST[q], []
        for _ in range(STEPS + HOST_STEPS):
            tok, _lg = rm.decode_step(tok)
            seq.append(tok)
        oracle.append(seq)
        rm.close()
    return {"single": single, "oracle": [[oracle[q][k] for q in range(4)] for k in range(STEPS + HOST_STEPS)]}


if __name__ == "__main__":
    main(sys.argv[1])
