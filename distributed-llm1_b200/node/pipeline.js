// pipeline.js — drop-in for the reference's pipeline.js on the B200 path: the
// same exports (assignLayers, Stage, LeaderPipeline) and call shapes
// (pipeline.js:6-282), with every stage pass, the embedding, the LM head and the
// single-node token loop running in libdllm.so (dllm_napi addon). It sits in the
// reference's directory next to constants.js, rtc.js and weights.js, and takes a
// ctx from this directory's kernels.js. Remote stages keep the reference's frame
// protocol: the leader sends HIDDEN_REQ / FINAL_REQ frames with opts.sendFrame
// and onFrame resolves them (script.js:163-172 answers with handleStageFrame).
import { CFG, FRAME } from "./constants.js";
import { pack, unpack } from "./rtc.js";

const HOP_TIMEOUT_MS = 15000;

// Layer split by capacity (pipeline.js:6-23): share = max(1, round(cap/total*L)),
// cap = (memGB ?? 4) * (gpu ? 1.5 : 0.5), the last peer takes the remainder.
export function assignLayers(peers, numLayers = CFG.numLayers) {
  const caps = peers.map((p) => ({ id: p.id, cap: (p.profile?.memGB ?? 4) * (p.profile?.gpu ? 1.5 : 0.5) }));
  let total = 0;
  for (const c of caps) total += c.cap;
  const out = [];
  let next = 0;
  caps.forEach((c, i) => {
    const share = i === caps.length - 1 ? numLayers - next : Math.max(1, Math.round((c.cap / total) * numLayers));
    const end = Math.min(numLayers, next + share);
    out.push({ id: c.id, start: next, end });
    next = end;
  });
  return out;
}

// A contiguous block of decoder layers with its own (paged) KV cache.
export class Stage {
  constructor(kctx, start, end, handle) {
    const addon = kctx.addon;
    this.k = kctx;
    this.start = start;
    this.end = end;
    this.h = handle ?? addon.stageCreate(kctx.device, start, end);
    const h = this.h;
    // stage.W[name] = buf hands the buffer to the library (pipeline.js:31)
    this.W = new Proxy({}, {
      set(target, name, buf) {
        addon.stageSetWeight(h, String(name), buf);
        target[name] = buf;
        return true;
      },
    });
  }

  get T0() { return this.k.addon.stageGetT0(this.h, 0); }
  set T0(v) { this.k.addon.stageSetT0(this.h, 0, v); }

  reset() { this.k.addon.stageReset(this.h); }

  // Stage.forward(hiddenF32, n, posStart) -> buffer of n rows (T0 += n)
  forward(hiddenF32, n, posStart) { return this.k.addon.stageForward(this.h, hiddenF32, n, posStart); }

  appendKv(L, kkBuf, vvBuf, n) { this.k.addon.stageAppendKv(this.h, L, kkBuf, vvBuf, n); }
}

// The stage side of a hop (script.js:163-172): run the frame's rows, reply RESP
// with every row (HIDDEN_REQ) or the last one (FINAL_REQ), posStart = T0.
export async function handleStageFrame(stage, data) {
  const frame = unpack(data);
  const D = stage.k.D;
  const n = Math.floor(frame.f32.length / D);
  const buf = stage.forward(frame.f32, n, frame.posStart);
  const f32 = await stage.k.readF32(buf, n * D);
  const out = frame.msgType === FRAME.FINAL_REQ ? f32.subarray((n - 1) * D, n * D) : f32;
  return pack(FRAME.RESP, frame.seqId, stage.T0, out);
}

export class LeaderPipeline {
  constructor(kctx, myRange, stages, opts = {}) {
    const addon = kctx.addon;
    this.k = kctx;
    this.myId = opts.myId;
    this.ld = addon.leaderCreate(kctx.device, myRange[0], myRange[1]);
    this.stage = new Stage(kctx, myRange[0], myRange[1], addon.leaderStage(this.ld));
    this.stage.leader = this; // the leader owns its stage: keep it alive with the stage
    this.stages = stages ?? [{ id: this.myId, start: myRange[0], end: myRange[1] }];
    this.stagesTail = this.stages.filter((s) => s.id !== this.myId);
    this.singleNode = this.stagesTail.length === 0 && myRange[1] >= kctx.cfg.numLayers;
    this.sendFrame = opts.sendFrame;
    this.onToken = opts.onToken ?? (() => {});
    this.pending = new Map();
    this.seq = 1;
  }

  // loadLeaderWeights(embedBits, normBits[, lmHeadBits]) (pipeline.js:109-119);
  // untied models (7B, 32B) pass lm_head.weight as the third argument.
  loadLeaderWeights(embedBits, normBits, lmHeadBits) {
    const k = this.k;
    const e = k.loadWeightBits(embedBits, "model.embed_tokens.weight");
    const n = k.loadWeightBits(normBits, "model.norm.weight");
    const h = lmHeadBits ? k.loadWeightBits(lmHeadBits, "lm_head.weight") : null;
    k.addon.leaderSetWeights(this.ld, e, n, h);
  }

  embedTokens(tokens) { return this.k.addon.leaderEmbedTokens(this.ld, Int32Array.from(tokens)); }

  async sampleLast(hidden) { return this.k.addon.leaderSampleLast(this.ld, hidden); }

  // forward(hidden, n, posStart) -> last row (pipeline.js:187-224)
  async forward(hidden, n, posStart) {
    if (this.stagesTail.length === 0) return this.k.addon.leaderForward(this.ld, hidden, n, posStart);
    const D = this.k.D;
    let h = await this.k.readF32(this.stage.forward(hidden, n, posStart), n * D);
    for (let i = 0; i < this.stagesTail.length; i++) {
      const last = i === this.stagesTail.length - 1;
      h = await this.hop(this.stagesTail[i].id, last ? FRAME.FINAL_REQ : FRAME.HIDDEN_REQ, h, posStart);
    }
    return h.length === D ? h : h.subarray((n - 1) * D, n * D);
  }

  hop(peerId, msgType, f32, posStart) {
    const seqId = this.seq++;
    return new Promise((resolve, reject) => {
      const timer = setTimeout(() => {
        this.pending.delete(seqId);
        reject(new Error(`hop timeout (peer ${peerId}, seq ${seqId})`));
      }, HOP_TIMEOUT_MS);
      this.pending.set(seqId, { resolve, reject, timer });
      this.sendFrame(peerId, pack(msgType, seqId, posStart, f32));
    });
  }

  onFrame(data) {
    const frame = unpack(data);
    const p = this.pending.get(frame.seqId);
    if (!p || frame.msgType !== FRAME.RESP) return;
    clearTimeout(p.timer);
    this.pending.delete(frame.seqId);
    p.resolve(frame.f32);
  }

  // generate(tokens, maxNew) (pipeline.js:255-281): prefill, greedy decode, EOS break.
  async generate(tokens, maxNew) {
    if (this.singleNode) {
      const out = this.k.addon.leaderGenerate(this.ld, Int32Array.from(tokens), maxNew);
      for (const t of out) this.onToken(t);
      return out.length;
    }
    const len = tokens.length;
    let row = await this.forward(this.embedTokens(tokens), len, 0);
    let next = await this.sampleLast(row);
    let count = 1;
    this.onToken(next);
    for (let i = 1; i < maxNew && next !== this.k.cfg.eosTokenId; i++) {
      row = await this.forward(this.embedTokens([next]), 1, len + i - 1);
      next = await this.sampleLast(row);
      this.onToken(next);
      count++;
    }
    return count;
  }
}

// Multi-GPU ring of one node (dllm_pipeline_*): each process owns one Stage; the
// hop between GPUs is fused into the stage kernel over NVLink. `exchange(handle)`
// must return every rank's 64-byte handle (Uint8Array) in rank order, over the
// host's own channel (the reference's signaling channel plays this role).
export class GpuRing {
  constructor(stage, rank, world, nMicro, micro) {
    this.addon = stage.k.addon;
    this.rank = rank;
    this.world = world;
    this.seqs = nMicro * micro;
    this.h = this.addon.pipelineCreate(stage.h, rank, world, nMicro, micro);
    this.stage = stage;
  }

  async connect(exchange) {
    const all = await exchange(this.addon.pipelineHandle(this.h));
    this.addon.pipelineConnect(this.h, all[(this.rank + 1) % this.world]);
  }

  setTokens(tokens) { this.addon.pipelineSetTokens(this.h, Int32Array.from(tokens)); }

  run(steps) { this.addon.pipelineRun(this.h, steps); }

  // last rank: tokens of the latest run, [steps][nMicro * micro] flattened
  readTokens(steps) { return this.addon.pipelineReadTokens(this.h, steps, this.seqs); }
}
