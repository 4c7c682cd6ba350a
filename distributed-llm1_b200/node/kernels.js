// kernels.js — drop-in for the reference's kernels.js on the B200 path: the same
// `initKernels(device)` export and ctx surface (kernels.js:5,179-303), backed by
// libdllm.so through the dllm_napi addon. `device` is a CUDA ordinal (a WebGPU
// device object is accepted and means GPU 0). Buffers are opaque handles the
// garbage collector releases; readF32 is async like the reference's and throws
// on its bounded wait, as the reference's 15 s timeout does.
import { createRequire } from "node:module";

const require = createRequire(import.meta.url);
const addon = require("./build/Release/dllm_napi.node");

export const KV_F32 = 0;
export const KV_BF16 = 1;

// cfg: optional overrides of constants.js CFG (vocabSize, hiddenSize, numLayers,
// numQHeads, numKVHeads, headDim, intermediateSize, ropeTheta, rmsNormEps,
// tieWordEmbeddings, eosTokenId, maxPos) plus kvDtype, kvPageSize, maxSeqs.
export async function initKernels(device, cfg) {
  const ordinal = typeof device === "number" ? device : 0;
  const h = addon.initKernels(ordinal, cfg ?? {});
  const c = addon.getConfig(h);
  const ctx = {
    device: h,
    D: c.hiddenSize,
    KVH: c.numKVHeads,
    NQ: c.numQHeads,
    HD: c.headDim,
    cfg: c,
    addon,
  };
  ctx.loadWeightBits = (u32arr, label) => addon.loadWeightBits(h, u32arr, label ?? "weights");
  ctx.loadWeightBf16 = (u16arr, label) => addon.loadWeightBf16(h, u16arr, label ?? "weights");
  ctx.createF32 = (numFloats, label) => addon.createF32(h, numFloats, label ?? "");
  ctx.writeF32 = (buf, f32) => addon.writeF32(h, buf, f32);
  ctx.readF32 = async (buf, numFloats, label = "") => addon.readF32(h, buf, numFloats, label);
  ctx.matmul = (xBuf, wBuf, n, din, dout) => addon.matmul(h, xBuf, wBuf, n, din, dout);
  ctx.rmsnorm = (xBuf, gBuf, n) => addon.rmsnorm(h, xBuf, gBuf, n);
  ctx.ropeQ = (xBuf, posStart, n) => addon.ropeQ(h, xBuf, posStart, n);
  ctx.ropeK = (xBuf, posStart, n) => addon.ropeK(h, xBuf, posStart, n);
  ctx.attention = (qBuf, kCacheBuf, vCacheBuf, T0, n) => addon.attention(h, qBuf, kCacheBuf, vCacheBuf, T0, n);
  ctx.siluMul = (aBuf, bBuf, total) => addon.siluMul(h, aBuf, bBuf, total);
  ctx.add = (aBuf, bBuf, numFloats) => addon.add(h, aBuf, bBuf, numFloats);
  ctx.addBias = (aBuf, biasBuf, n, dout) => addon.addBias(h, aBuf, biasBuf, n, dout);
  ctx.destroy = () => addon.ctxDestroy(h);
  return ctx;
}
