/*
 * dllm.h — C ABI of libdllm.so, the B200 (sm_100a) decode path for Qwen2.5-style
 * decoders.
 *
 * The entry points mirror the JavaScript surface that the reference's decode loop
 * sits behind, so a host binding (N-API, ctypes, cgo ...) can swap the WebGPU path
 * for this library one call at a time:
 *   - kernels.js  `initKernels(device)` -> ctx with buffer helpers and op launchers
 *   - pipeline.js `Stage` (layer range + KV cache) and `LeaderPipeline`
 *   - weights.js  bf16 weight layout (raw bits, one element per u32 on the JS side)
 * Every function cites the reference interface it replaces as file:line.
 *
 * Conventions
 *   - Every call returns a status (DLLM_OK == 0); on error `dllm_last_error(ctx)`
 *     holds a one-line message. The JS shim turns a non-zero status into
 *     `throw new Error(msg)`, as the reference throws (kernels.js:182,189,196,244).
 *   - One host thread per ctx; calls are not re-entrant. Work is enqueued on the
 *     ctx's CUDA stream; only calls that hand data back to the host synchronise,
 *     and those waits are bounded (DLLM_ETIMEOUT), mirroring readF32's 15 s limit
 *     (kernels.js:201-207).
 *   - Buffers are reference counted. The caller owns every dllm_buf it receives
 *     and releases it with dllm_buf_free; a stage that is given a weight buffer
 *     keeps its own reference (JS keeps the GPUBuffer alive the same way).
 *   - Activations are fp32 and weights bf16, as in the reference. The KV cache is
 *     fp32 (the reference's precision) or bf16 (half the bytes), chosen per ctx.
 */
#ifndef DLLM_H
#define DLLM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------- */
enum {
  DLLM_OK = 0,
  DLLM_EINVAL = 1,    /* bad argument: the reference throws "invalid size" (kernels.js:182,189,196,244) */
  DLLM_ENOMEM = 2,    /* device allocation failed */
  DLLM_ERANGE = 3,    /* KV cache overflow: T0 + n > max_pos (pipeline.js:38-43 sizes the cache) */
  DLLM_ETIMEOUT = 4,  /* bounded wait expired (readF32 15 s, kernels.js:201-207) */
  DLLM_ECUDA = 5,     /* CUDA runtime error */
  DLLM_ENOTFOUND = 6, /* missing weight tensor name (Stage.W lookup, pipeline.js:55-73) */
  DLLM_EDEVICE = 7    /* a kernel reported an error status (device-side bounds check) */
};

enum { DLLM_KV_F32 = 0, DLLM_KV_BF16 = 1 };

/* Model and cache configuration. Replaces the hard-coded CFG object of
 * constants.js:10-23 and the dims baked into the shaders (kernels.js:173). */
typedef struct dllm_config {
  int32_t vocab_size;          /* CFG.vocabSize */
  int32_t hidden_size;         /* CFG.hiddenSize (D) */
  int32_t num_layers;          /* CFG.numLayers */
  int32_t num_q_heads;         /* CFG.numQHeads (NQ) */
  int32_t num_kv_heads;        /* CFG.numKVHeads (KVH) */
  int32_t head_dim;            /* CFG.headDim (HD): 64 or 128 */
  int32_t intermediate_size;   /* CFG.intermediateSize */
  float rope_theta;            /* CFG.ropeTheta */
  float rms_norm_eps;          /* CFG.rmsNormEps */
  int32_t tie_word_embeddings; /* CFG.tieWordEmbeddings: LM head = embed_tokens */
  int32_t eos_token_id;        /* CFG.eosTokenId */
  int32_t max_pos;             /* CFG.maxPos: KV slots per sequence */
  int32_t kv_dtype;            /* DLLM_KV_F32 (reference precision) or DLLM_KV_BF16 */
  int32_t kv_page_size;        /* KV slots per page, power of two (paged cache) */
  int32_t max_seqs;            /* sequences one stage holds KV for (micro-batching) */
} dllm_config;

typedef struct dllm_ctx dllm_ctx;
typedef struct dllm_buf dllm_buf;
typedef struct dllm_stage dllm_stage;
typedef struct dllm_leader dllm_leader;

/* ---- library / context ----------------------------------------------------- */
const char* dllm_version(void);
const char* dllm_status_string(int status);
/* Fills the Qwen2.5-1.5B defaults of constants.js:10-23 (max_pos 4096, fp32 KV). */
void dllm_config_default(dllm_config* cfg);

/* initKernels(device) -> ctx (kernels.js:5,179). `device` is a CUDA ordinal. */
int dllm_init_kernels(int device, const dllm_config* cfg, dllm_ctx** out);
void dllm_ctx_destroy(dllm_ctx* ctx);
const char* dllm_last_error(const dllm_ctx* ctx);
int dllm_ctx_get_config(const dllm_ctx* ctx, dllm_config* out);
/* Enqueue on a caller-owned cudaStream_t (NULL restores the ctx's own stream). */
int dllm_ctx_set_stream(dllm_ctx* ctx, void* cuda_stream);
/* Bounded wait for all work on the ctx stream (timeout_ms <= 0: 15000 ms). */
int dllm_ctx_synchronize(dllm_ctx* ctx, int timeout_ms);
/* Number of kernels this ctx has launched (host counter, for launch accounting). */
uint64_t dllm_ctx_launch_count(const dllm_ctx* ctx);
/* Passes of at least `min_rows` rows (MATMUL with n > 1, kernels.js:26-44; prefill
 * chunks and wide micro-batches of Stage.forward, pipeline.js:48-78) run their
 * projections as tcgen05 tensor-core GEMMs; fewer rows use the CUDA-core matvec.
 * Default 8 (at 7B, 8 rows take 14.4 ms through the persistent kernel and ~7 ms
 * through the tensor-core pass); 0 keeps every pass on the matvec; otherwise 2..128. */
int dllm_ctx_set_tensor_core_rows(dllm_ctx* ctx, int min_rows);

/* ---- buffers (kernels.js:181-211) ----------------------------------------- */
/* ctx.loadWeightBits(u32arr, label) (kernels.js:181-186): one u32 per bf16
 * element holding the raw bits in its low half (weights.js:144-150). Stored on
 * the device as 2-byte bf16. Throws on empty input like the reference. */
int dllm_load_weight_bits(dllm_ctx* ctx, const uint32_t* bits, size_t n, const char* label, dllm_buf** out);
/* Same, from packed 2-byte bf16 (the safetensors byte layout). */
int dllm_load_weight_bf16(dllm_ctx* ctx, const uint16_t* bf16, size_t n, const char* label, dllm_buf** out);
/* ctx.createF32(numFloats, label) (kernels.js:188-191). Zero-filled. */
int dllm_create_f32(dllm_ctx* ctx, size_t n, const char* label, dllm_buf** out);
/* ctx.writeF32(buf, f32) (kernels.js:193). */
int dllm_write_f32(dllm_ctx* ctx, dllm_buf* buf, const float* src, size_t n);
/* ctx.readF32(buf, numFloats, label) (kernels.js:195-211): bounded blocking read. */
int dllm_read_f32(dllm_ctx* ctx, const dllm_buf* buf, float* dst, size_t n, const char* label);
/* Raw bf16 read-back of a weight buffer (test hook for the weight layout). */
int dllm_read_bf16(dllm_ctx* ctx, const dllm_buf* buf, uint16_t* dst, size_t n);
void dllm_buf_free(dllm_buf* buf);
size_t dllm_buf_bytes(const dllm_buf* buf);
void* dllm_buf_device_ptr(const dllm_buf* buf);
/* Synthetic weights generated on the device: N(0, std) rounded to bf16, from a
 * counter-based hash of (seed, element). Not on the decode path. */
int dllm_fill_normal_bf16(dllm_ctx* ctx, dllm_buf* buf, uint64_t seed, float std);
int dllm_fill_const_bf16(dllm_ctx* ctx, dllm_buf* buf, float value);
int dllm_create_bf16(dllm_ctx* ctx, size_t n, const char* label, dllm_buf** out);

/* ---- ops: one launcher per shader (kernels.js:222-301) --------------------- */
/* ctx.matmul(x, w, n, din, dout) (kernels.js:222-231): out[t,j] = sum_k x[t,k]*W[j,k]. */
int dllm_matmul(dllm_ctx* ctx, const dllm_buf* x, const dllm_buf* w, int n, int din, int dout, dllm_buf** out);
/* ctx.rmsnorm(x, g, n) (kernels.js:233-241): rows of hidden_size. */
int dllm_rmsnorm(dllm_ctx* ctx, const dllm_buf* x, const dllm_buf* g, int n, dllm_buf** out);
/* ctx.ropeQ / ctx.ropeK (kernels.js:243-254): in place, rotate-half pairs. */
int dllm_rope_q(dllm_ctx* ctx, dllm_buf* x, int pos_start, int n);
int dllm_rope_k(dllm_ctx* ctx, dllm_buf* x, int pos_start, int n);
/* ctx.attention(q, kCache, vCache, T0, n) (kernels.js:256-268): causal GQA over
 * fp32 caches laid out [max_pos, KVH*HD] as Stage.kv holds them (pipeline.js:38-43). */
int dllm_attention(dllm_ctx* ctx, const dllm_buf* q, const dllm_buf* kcache, const dllm_buf* vcache, int t0, int n,
                   dllm_buf** out);
/* ctx.siluMul(a, b, total) (kernels.js:270-279). */
int dllm_silu_mul(dllm_ctx* ctx, const dllm_buf* a, const dllm_buf* b, int total, dllm_buf** out);
/* ctx.add(a, b, n) (kernels.js:281-289); bounds-checked, unlike the shader. */
int dllm_add(dllm_ctx* ctx, const dllm_buf* a, const dllm_buf* b, int n, dllm_buf** out);
/* ctx.addBias(a, bias, n, dout) (kernels.js:291-301). */
int dllm_add_bias(dllm_ctx* ctx, const dllm_buf* a, const dllm_buf* bias, int n, int dout, dllm_buf** out);
/* Greedy argmax over n fp32 logits with the host scan's rule (pipeline.js:159-162):
 * strict '>' in index order, so the lowest index wins ties; NaN never wins. */
int dllm_argmax(dllm_ctx* ctx, const dllm_buf* logits, int n, int32_t* index_out);

/* ---- Stage: contiguous layer range + KV cache (pipeline.js:26-88) ---------- */
int dllm_stage_create(dllm_ctx* ctx, int start, int end, dllm_stage** out);  /* new Stage(k, start, end) */
void dllm_stage_destroy(dllm_stage* st);
/* stage.W[name] = buf (pipeline.js:31). HF tensor names (weights.js:167-182). */
int dllm_stage_set_weight(dllm_stage* st, const char* name, dllm_buf* buf);
/* Stage.reset() (pipeline.js:37-46): T0 = 0 for every sequence. */
int dllm_stage_reset(dllm_stage* st);
/* Stage.T0 for sequence `seq` (pipeline.js:33). */
int dllm_stage_get_t0(const dllm_stage* st, int seq);
int dllm_stage_set_t0(dllm_stage* st, int seq, int t0);
/* Stage.forward(hiddenF32, n, posStart) (pipeline.js:48-78) on sequence 0:
 * uploads n rows, runs the layers, T0 += n, returns the new hidden buffer. */
int dllm_stage_forward(dllm_stage* st, const float* hidden, int n, int pos_start, dllm_buf** out);
/* Device-resident decode pass of one micro-batch (the stage side of a hop,
 * script.js:163-172, with the hidden rows already in device memory): row i of
 * `h_dev` ([m, D] fp32, 1 <= m <= 8) belongs to sequence seq_ids[i] (host
 * array, distinct) at position == slot == that sequence's T0; h is updated in
 * place and every listed sequence's T0 advances by one. Optional device arrays:
 * tokens_in_dev[m] first replaces h with the token embeddings (embedTokens,
 * pipeline.js:121-128; needs model.embed_tokens.weight); tokens_out_dev[m]
 * receives the greedy tokens of final norm + LM head (sampleLast,
 * pipeline.js:141-174; needs model.norm.weight and a LM head). */
int dllm_stage_forward_rows(dllm_stage* st, float* h_dev, int m, const int32_t* seq_ids, const int32_t* tokens_in_dev,
                            int32_t* tokens_out_dev);
/* Stage.appendKv(L, kk, vv, n) (pipeline.js:80-87): rows -> slots T0..T0+n-1. */
int dllm_stage_append_kv(dllm_stage* st, int layer, const dllm_buf* kk, const dllm_buf* vv, int n);
/* Reads KV slots back in the reference layout [n_slots, KVH*HD] fp32
 * (which: 0 = k, 1 = v). Test hook for slot indexing. */
int dllm_stage_read_kv(dllm_stage* st, int layer, int which, int seq, int slot_start, int n_slots, float* dst);
/* Synthetic prefilled KV: slots [0, n_slots) of `seq` in every layer get N(0,1)
 * values from a counter-based hash; T0 = position = n_slots. */
int dllm_stage_fill_kv_random(dllm_stage* st, int seq, int n_slots, uint64_t seed);
/* Replace the logical->physical page map of one sequence (pages must be
 * distinct and < max_seqs * pages_per_seq). Test hook for the paged layout. */
int dllm_stage_set_page_table(dllm_stage* st, int seq, const int32_t* pages, int n_pages);
int dllm_stage_pages_per_seq(const dllm_stage* st);
/* Reads the latest pass's per-row workspace of the stage's last layer: which 0 =
 * q after bias and RoPE [rows, NQ*HD] (the input of ctx.attention,
 * pipeline.js:62-65), 1 = attention output [rows, NQ*HD] (pipeline.js:65),
 * 2 = SiLU(gate)*up [rows, I] (pipeline.js:72). Test hook for op-level checks of
 * the fused phases (the reference creates one buffer per op, kernels.js:222-301). */
int dllm_stage_read_workspace(dllm_stage* st, int which, int rows, float* dst);
/* Tracing (the reference logs performance.now() deltas, pipeline.js:144,158,172):
 * with cap > 0 every stage-kernel launch stamps the GPU global timer (ns) at
 * its start and after each grid barrier into a device buffer of `cap` entries
 * (0 turns it off). Per decode pass: start, [embed], then 5 per layer (after
 * QKV, attention, O, gate/up, down), then [head]. Reads the latest launch's. */
int dllm_stage_set_trace(dllm_stage* st, int cap);
int dllm_stage_read_trace(dllm_stage* st, uint64_t* out, int cap);

/* ---- LeaderPipeline (pipeline.js:91-282), local stage only ------------------ */
/* new LeaderPipeline(k, [start,end), ...) (pipeline.js:92-107). */
int dllm_leader_create(dllm_ctx* ctx, int start, int end, dllm_leader** out);
void dllm_leader_destroy(dllm_leader* ld);
/* The leader's own Stage (pipeline.js:95), borrowed. */
dllm_stage* dllm_leader_stage(dllm_leader* ld);
/* loadLeaderWeights(embedBits, normBits) (pipeline.js:109-119) plus the untied
 * `lm_head.weight` used by 7B/32B (NULL when tied). Buffers are referenced. */
int dllm_leader_set_weights(dllm_leader* ld, dllm_buf* embed, dllm_buf* norm, dllm_buf* lm_head);
/* embedTokens(tokens) (pipeline.js:121-128): host f32 [n, D]. */
int dllm_leader_embed_tokens(dllm_leader* ld, const int32_t* tokens, int n, float* out);
/* sampleLast(hidden) (pipeline.js:141-174): final RMSNorm, LM head, greedy
 * argmax (lowest index wins ties). `logits_out` (host, vocab floats) may be NULL. */
int dllm_leader_sample_last(dllm_leader* ld, const float* hidden_row, int32_t* token, float* logits_out);
/* forward(hidden, n, posStart) (pipeline.js:187-224) through the local stage;
 * writes the last row (D floats) to `last_row`. */
int dllm_leader_forward(dllm_leader* ld, const float* hidden, int n, int pos_start, float* last_row);
/* generate(tokens, maxNew) (pipeline.js:255-281): prefill, then greedy decode
 * with the EOS break; one CUDA-graph replay per token with the token read back
 * to the host every step. Emitted ids go to `out` (capacity max_new). */
int dllm_leader_generate(dllm_leader* ld, const int32_t* tokens, int n_tokens, int max_new, int32_t* out, int* n_out);
/* Device-resident decode: `steps` greedy tokens after `first_token` at the
 * current T0 (position == slot == T0), no EOS break and no per-step host round
 * trip (one CUDA-graph replay per token). Same token loop as generate's decode
 * branch (pipeline.js:262-267). */
int dllm_leader_decode(dllm_leader* ld, int32_t first_token, int steps, int32_t* out);
/* The same, split: enqueue the replays on the ctx stream without waiting, then
 * read the emitted tokens (bounded wait). */
int dllm_leader_decode_enqueue(dllm_leader* ld, int32_t first_token, int steps);
int dllm_leader_read_tokens(dllm_leader* ld, int32_t* out, int steps);
/* Keep the logits of the first `keep` steps of each generate/decode call in
 * device memory (0 = off, the default). */
int dllm_leader_set_keep_logits(dllm_leader* ld, int keep);
/* Logits of the most recent sampleLast, or of the last kept generate/decode step. */
int dllm_leader_last_logits(dllm_leader* ld, float* out);
/* Logits of kept step `index` (0 = the prefill's sample) of the latest call. */
int dllm_leader_read_logits(dllm_leader* ld, int index, float* out);

/* ---- multi-GPU pipeline (pipeline.js:6-87 layer-range stages, :91-282 leader loop) ----
 * One process (or thread) per GPU holds one Stage of a contiguous layer range
 * (assignLayers, pipeline.js:6-23); rank 0's stage also embeds tokens, the last
 * rank's stage holds the final norm and LM head. n_micro micro-batches of
 * `micro` sequences (sequence ids b*micro .. (b+1)*micro-1 of every stage's KV
 * cache) circulate the ring rank 0 -> 1 -> ... -> last -> 0, so with n_micro >=
 * world every GPU works on some micro-batch at once. The hidden-row hop of the
 * reference (frames over WebRTC, pipeline.js:226-253) is fused into the stage
 * kernel: a pass ends by storing its rows (the last stage: its greedy tokens) in
 * the next GPU's receive buffer over NVLink and releasing a flag there; the next
 * pass starts with a bounded wait on its flag. No host round trip per hop.
 * Set-up: every rank creates its pipeline, publishes dllm_pipeline_handle
 * (a CUDA IPC handle of its receive buffer) over the host's own channel, and
 * connects to the handle of rank (rank + 1) % world. Before the first run all
 * ranks should be connected (a host barrier), since a pass waits for its input
 * at most a few seconds. */
typedef struct dllm_pipeline dllm_pipeline;
#define DLLM_PIPELINE_HANDLE_BYTES 64
/* micro <= 8; n_micro * micro <= the stage's max_seqs. Row i of micro-batch b is
 * sequence b*micro + i at its current T0 (position == slot == T0). */
int dllm_pipeline_create(dllm_stage* st, int rank, int world, int n_micro, int micro, dllm_pipeline** out);
void dllm_pipeline_destroy(dllm_pipeline* pl);
/* This rank's receive buffer as DLLM_PIPELINE_HANDLE_BYTES opaque bytes. */
int dllm_pipeline_handle(const dllm_pipeline* pl, uint8_t* handle_out);
/* Map the receive buffer of rank (rank + 1) % world (its dllm_pipeline_handle). */
int dllm_pipeline_connect(dllm_pipeline* pl, const uint8_t* next_rank_handle);
/* Rank 0: the first token of every sequence (n_micro * micro, in sequence order). */
int dllm_pipeline_set_tokens(dllm_pipeline* pl, const int32_t* tokens, int n);
/* Enqueue `steps` greedy decode steps of every micro-batch (steps * n_micro
 * passes on this rank, in ring order) on the stage ctx's stream; no host wait. */
int dllm_pipeline_run(dllm_pipeline* pl, int steps);
/* Last rank: the tokens sampled by the latest run, [steps][n_micro * micro]
 * (bounded wait; a pass whose input never arrived reports DLLM_ETIMEOUT). */
int dllm_pipeline_read_tokens(dllm_pipeline* pl, int32_t* out, int steps);
/* Bounded wait for this rank's enqueued passes, then its device error flag. */
int dllm_pipeline_synchronize(dllm_pipeline* pl, int timeout_ms);
/* Host-fed token loop (the reference's leader: sampled tokens come back to the
 * host, pipeline.js:262-267): with `on`, the last stage keeps its tokens and the
 * first stage takes each micro-batch's tokens from dllm_pipeline_run_micro. All
 * ranks switch together, between passes. */
int dllm_pipeline_set_host_tokens(dllm_pipeline* pl, int on);
/* One pass of micro-batch b on this rank. First stage (host-token mode):
 * `tokens` (host, micro ids) are copied in first. Last stage: the sampled tokens
 * are copied to `tokens_out` (host) with a bounded wait. Others: enqueued only. */
int dllm_pipeline_run_micro(dllm_pipeline* pl, int b, const int32_t* tokens, int32_t* tokens_out);

/* ---- attention that allocates nothing ---------------------------------------
 * No counterpart in the reference. For callers that must not allocate device
 * memory: a host that owns the whole HBM budget through its own pool and forbids
 * allocations after start-up, or a latency-critical loop that cannot afford
 * cudaMalloc/cudaFree (which may synchronise the device). Same math as
 * dllm_attention (kernels.js:86-132 semantics; caches [max_pos, KVH*HD] fp32,
 * row t attends slots [0, t0+t]), but the caller passes every buffer as a device
 * pointer and the split partials, ticket counters, row descriptors and error word
 * live in a 4 MiB static device array that every GPU loading this library holds
 * until the process exits. No ctx is needed; work is enqueued on `cuda_stream`
 * (NULL: the legacy default stream) and the call does not wait for it.
 * Each call, with the caller's device current, resolves the array's device address
 * and sets the kernel's shared-memory limit (cheap, allocation-free, nothing cached,
 * so a device reset between calls is harmless). Calls share the array: calls that
 * overlap on the GPU (other streams, other threads) race. Limits: 1 <= n <= 64 rows
 * (DLLM_ERANGE beyond), head_dim 64 or 128, at most 8 query heads per KV head
 * (DLLM_EINVAL otherwise).
 * The return value covers the arguments and the launch only. Errors the kernels
 * find on the device (a split-merge wait that ran out, a row outside the cache)
 * are read with dllm_attention_noalloc_status after the call and before the next
 * one (the next call clears them). */
int dllm_attention_noalloc(const float* q, const float* kcache, const float* vcache, float* out, int t0, int n,
                           int num_q_heads, int num_kv_heads, int head_dim, int max_pos, void* cuda_stream);
/* Waits (bounded by timeout_ms, <= 0: 15000) for `cuda_stream`, then reads the
 * device error word of the latest dllm_attention_noalloc on the current device.
 * Returns DLLM_OK when the kernels reported nothing, DLLM_ETIMEOUT when a split
 * merge gave up waiting (or the stream wait itself timed out), DLLM_ERANGE when a
 * row fell outside the cache, DLLM_EDEVICE for other device codes; the raw device
 * code goes to *device_error (may be NULL). Allocates nothing. No counterpart in
 * the reference (readF32's bounded wait, kernels.js:201-207, is the model). */
int dllm_attention_noalloc_status(void* cuda_stream, int timeout_ms, int* device_error);

#ifdef __cplusplus
}
#endif
#endif /* DLLM_H */
