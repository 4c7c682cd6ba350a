// api.cu — the C ABI of libdllm.so (include/dllm.h).
//
// Host runtime of the decode path: context and device buffers (kernels.js:179-211),
// the op launchers of the ctx object (kernels.js:222-301), the Stage layer-range
// runner with its paged KV cache (pipeline.js:26-88) and the LeaderPipeline
// decode loop (pipeline.js:91-282). The decode step is one persistent kernel
// launch per pass (stage.cu); generate() replays it as a CUDA graph per token.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <thread>
#include <vector>

#include "dllm.h"
#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "ops.cuh"
#include "stage.cuh"

using dllm::KvLayout;
using dllm::LayerW;
using dllm::RowDesc;
using dllm::StageParams;

namespace {

constexpr int kDefaultTimeoutMs = 15000;  // readF32's limit (kernels.js:201-207)
constexpr int kMaxSplitsAlloc = dllm::kAttnMaxSplits;  // attention splits per (row, kv head)
#ifndef DLLM_PREFETCH_BYTES
#define DLLM_PREFETCH_BYTES (96 * 1024)
#endif
constexpr int kPrefetchBytes = DLLM_PREFETCH_BYTES;  // per-CTA L2 prefetch budget between phases

}  // namespace

struct dllm_buf {
  dllm_ctx* ctx = nullptr;
  int device = 0;  // kept so the buffer can be freed after its ctx is destroyed
  void* ptr = nullptr;
  size_t bytes = 0;
  size_t n = 0;    // elements
  int dtype = 0;   // 0 fp32, 1 bf16
  int refs = 1;
  std::string label;
};

struct dllm_ctx {
  int refs = 1;  // the caller's reference + one per live buffer, stage and leader
  int device = 0;
  dllm_config cfg{};
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  cudaEvent_t sync_event = nullptr;
  std::string err;
  uint64_t launches = 0;
  int sms = 0;
  float* freq = nullptr;           // RoPE inverse frequencies [HD/2]
  float scale = 0.f;               // f32(1/sqrt(HD))
  int* err_dev = nullptr;          // device error flag
  int* err_host = nullptr;         // pinned mirror
  // op-level attention scratch
  dllm::AttnScratch attn{};
  size_t attn_rows_cap = 0;
  RowDesc* attn_rows = nullptr;
  unsigned long long* best = nullptr;  // argmax op
  unsigned long long* best_host = nullptr;
  // tensor-core matmul: passes of >= tc_min_rows rows (0: never) and its scratch
  int tc_min_rows = dllm::kTcMinRows;
  void* tc_scratch = nullptr;
  size_t tc_scratch_bytes = 0;
  // freed buffers kept for reuse, by size in bytes
  std::multimap<size_t, void*> buf_cache;
  size_t buf_cache_bytes = 0;
};

struct dllm_stage {
  dllm_ctx* ctx = nullptr;
  int start = 0, end = 0, nl = 0;
  std::map<std::string, dllm_buf*> W;
  bool dirty = true;
  std::vector<LayerW> lw;
  LayerW* lw_dev = nullptr;
  const __nv_bfloat16* embed = nullptr;
  const __nv_bfloat16* norm = nullptr;
  const __nv_bfloat16* lm_head = nullptr;
  // paged KV cache
  int page = 64, log2_page = 6, pages_per_seq = 0, max_seqs = 1, max_slots = 0;
  size_t layer_elems = 0;
  void* kpool = nullptr;
  void* vpool = nullptr;
  int* page_table = nullptr;
  std::vector<int> T0;
  // workspaces for passes of <= 8 rows
  float *h = nullptr, *q = nullptr, *att = nullptr, *mid = nullptr;
  float *part_o = nullptr, *part_ml = nullptr;
  unsigned int* arrive = nullptr;
  float* h2 = nullptr;     // split-K MLP: the folded hidden row [D] o_proj adds to
  RowDesc* rows = nullptr;
  unsigned int* bar = nullptr;  // [count, epoch, -, -] then the split-K MLP's fixed-point sums [D] (i64)
  unsigned long long* best = nullptr;
  int32_t* tok = nullptr;       // [8]
  // API forwards with many rows
  size_t hbuf_rows = 0;
  float* hbuf = nullptr;
  size_t tokbuf_cap = 0;
  int32_t* tokbuf = nullptr;
  // wide passes (> 8 rows, or >= the ctx's tensor-core rows): per-row workspaces
  // for up to wide_cap rows; projections on the tensor cores, one launch per op
  int wide_cap = 0, wide_splits = 1;
  float *wq = nullptr, *wk = nullptr, *wv = nullptr, *watt = nullptr, *wg = nullptr, *wu = nullptr;
  float *wpart_o = nullptr, *wpart_ml = nullptr;
  unsigned int* warrive = nullptr;
  RowDesc* wrows = nullptr;
  float* wlogits = nullptr;  // [wide_cap][V], allocated when a wide pass samples tokens
  unsigned long long* wbest = nullptr;
  // tracing: %globaltimer at kernel start and after every grid barrier (last launch)
  unsigned long long* trace = nullptr;
  int trace_cap = 0;
  int version = 0;  // bumped when weights or tracing change (captured graphs rebuild)
};

struct dllm_leader {
  dllm_ctx* ctx = nullptr;
  dllm_stage* st = nullptr;
  int32_t* tok_dev = nullptr;      // [8]
  int32_t* pin_in = nullptr;       // pinned [8]
  int32_t* pin_out = nullptr;      // pinned [8]
  RowDesc* dec_rows = nullptr;     // [8]
  int* step_count = nullptr;
  int32_t* hist = nullptr;
  int hist_cap = 0;
  float* logits_ring = nullptr;
  int logits_cap = 0;
  float* last_logits = nullptr;    // [V]
  int last_index = -1;             // ring index of the latest logits, -1 none
  bool last_in_ring = false;
  cudaGraphExec_t g_e2e = nullptr;
  cudaGraphExec_t g_dev = nullptr;
  int graph_version = -1;          // stage version the graphs were captured for
  int pending_steps = 0;           // steps of the latest decode_enqueue
};

// ---------------------------------------------------------------------------------
namespace {

int set_err(dllm_ctx* c, int code, const char* fmt, ...) {
  if (c) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    c->err = buf;
  }
  return code;
}

#define CK(ctx, expr)                                                                            \
  do {                                                                                           \
    cudaError_t e_ = (expr);                                                                     \
    if (e_ != cudaSuccess) return set_err((ctx), DLLM_ECUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

void ctx_free(dllm_ctx* c);
void ctx_retain(dllm_ctx* c) { c->refs += 1; }
void ctx_release(dllm_ctx* c) {
  if (c && --c->refs == 0) ctx_free(c);
}

int use_device(dllm_ctx* c) {
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return set_err(c, DLLM_ECUDA, "cudaSetDevice(%d): %s", c->device, cudaGetErrorString(e));
  return DLLM_OK;
}

template <typename T>
int dev_alloc(dllm_ctx* c, T** p, size_t count, const char* what) {
  *p = nullptr;
  if (count == 0) count = 1;
  cudaError_t e = cudaMalloc((void**)p, count * sizeof(T));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_err(c, DLLM_ENOMEM, "cudaMalloc(%s, %zu bytes): %s", what, count * sizeof(T), cudaGetErrorString(e));
  }
  e = cudaMemsetAsync(*p, 0, count * sizeof(T), c->stream);
  if (e != cudaSuccess) return set_err(c, DLLM_ECUDA, "cudaMemsetAsync(%s): %s", what, cudaGetErrorString(e));
  return DLLM_OK;
}

void dev_free(void* p) {
  if (p) cudaFree(p);
}

// Bounded wait for the ctx stream, then the device error flag. Mirrors the
// 15 s timeout race of readF32 (kernels.js:201-207).
int sync_check(dllm_ctx* c, int timeout_ms) {
  if (timeout_ms <= 0) timeout_ms = kDefaultTimeoutMs;
  CK(c, cudaMemcpyAsync(c->err_host, c->err_dev, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
  CK(c, cudaEventRecord(c->sync_event, c->stream));
  const auto t0 = std::chrono::steady_clock::now();
  int spins = 0;
  for (;;) {
    const cudaError_t e = cudaEventQuery(c->sync_event);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return set_err(c, DLLM_ECUDA, "stream wait: %s", cudaGetErrorString(e));
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (ms > timeout_ms) return set_err(c, DLLM_ETIMEOUT, "device wait timed out after %d ms", timeout_ms);
    if (++spins > 20000) std::this_thread::sleep_for(std::chrono::microseconds(50));
    else std::this_thread::yield();
  }
  const int code = *c->err_host;
  if (code != 0) {
    cudaMemsetAsync(c->err_dev, 0, sizeof(int), c->stream);
    cudaStreamSynchronize(c->stream);
    if (code == dllm::kErrKvRange) return set_err(c, DLLM_ERANGE, "KV slot out of range (T0 + n > max_pos)");
    if (code == dllm::kErrBarrier) return set_err(c, DLLM_ETIMEOUT, "device grid barrier timed out");
    if (code == dllm::kErrToken) return set_err(c, DLLM_EINVAL, "token id out of vocabulary range");
    if (code == dllm::kErrPeerWait)
      return set_err(c, DLLM_ETIMEOUT, "pipeline hop: the previous stage's rows did not arrive in time");
    if (code == dllm::kErrTcWait) return set_err(c, DLLM_ETIMEOUT, "tensor-core matmul: a pipeline wait timed out");
    return set_err(c, DLLM_EDEVICE, "device error code %d", code);
  }
  return DLLM_OK;
}

bool valid_buf(const dllm_ctx* c, const dllm_buf* b) { return b && b->ctx == c && b->ptr; }

int check_f32(dllm_ctx* c, const dllm_buf* b, size_t need, const char* what) {
  if (!valid_buf(c, b)) return set_err(c, DLLM_EINVAL, "%s: null or foreign buffer", what);
  if (b->dtype != 0) return set_err(c, DLLM_EINVAL, "%s: expected an f32 buffer", what);
  if (b->n < need) return set_err(c, DLLM_EINVAL, "%s: buffer holds %zu floats, need %zu", what, b->n, need);
  return DLLM_OK;
}
int check_bf16(dllm_ctx* c, const dllm_buf* b, size_t need, const char* what) {
  if (!valid_buf(c, b)) return set_err(c, DLLM_EINVAL, "%s: null or foreign buffer", what);
  if (b->dtype != 1) return set_err(c, DLLM_EINVAL, "%s: expected a bf16 weight buffer", what);
  if (b->n < need) return set_err(c, DLLM_EINVAL, "%s: buffer holds %zu elements, need %zu", what, b->n, need);
  return DLLM_OK;
}

// Buffers of a ctx come from, and return to, a per-ctx cache of freed device
// blocks keyed by size: the op outputs of a forward (one per op, as the reference
// creates them, kernels.js:222-301) then cost no cudaMalloc/cudaFree (which can
// synchronise the device) after the first pass. Reuse is safe because every op
// of a ctx runs on its one stream, in order.
constexpr size_t kBufCacheBytes = (size_t)4 << 30;

void* cache_take(dllm_ctx* c, size_t bytes) {
  auto it = c->buf_cache.find(bytes);
  if (it == c->buf_cache.end()) return nullptr;
  void* p = it->second;
  c->buf_cache.erase(it);
  c->buf_cache_bytes -= bytes;
  return p;
}

// zero: fill with zeros (createF32 semantics); op outputs that the kernel fully
// overwrites skip it.
int new_buf(dllm_ctx* c, size_t n, int dtype, const char* label, dllm_buf** out, bool zero = true) {
  auto* b = new dllm_buf();
  b->ctx = c;
  b->device = c->device;
  b->n = n;
  b->dtype = dtype;
  b->bytes = n * (dtype == 0 ? 4 : 2);
  b->label = label ? label : "";
  b->ptr = cache_take(c, b->bytes);
  if (!b->ptr) {
    cudaError_t e = cudaMalloc(&b->ptr, b->bytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      delete b;
      return set_err(c, DLLM_ENOMEM, "cudaMalloc(%zu bytes, %s): %s", n * (dtype == 0 ? 4 : 2), label ? label : "",
                     cudaGetErrorString(e));
    }
  }
  if (zero) {
    cudaError_t e = cudaMemsetAsync(b->ptr, 0, b->bytes, c->stream);
    if (e != cudaSuccess) {
      cudaFree(b->ptr);
      delete b;
      return set_err(c, DLLM_ECUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    }
  }
  ctx_retain(c);
  *out = b;
  return DLLM_OK;
}

int ilog2(int v) {
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}

bool valid_config(const dllm_config& f, std::string* why) {
  char b[256];
  auto bad = [&](const char* m) {
    *why = m;
    return false;
  };
  if (f.hidden_size <= 0 || f.hidden_size % 8) return bad("hidden_size must be a positive multiple of 8");
  if (f.num_layers < 0) return bad("num_layers must be >= 0");
  if (f.head_dim != 64 && f.head_dim != 128) return bad("head_dim must be 64 or 128");
  if (f.num_q_heads <= 0 || f.num_kv_heads <= 0 || f.num_q_heads % f.num_kv_heads)
    return bad("num_q_heads must be a positive multiple of num_kv_heads");
  if (f.num_q_heads / f.num_kv_heads > dllm::kGMax) return bad("at most 8 query heads per kv head");
  if (f.intermediate_size <= 0 || f.intermediate_size % 8) return bad("intermediate_size must be a positive multiple of 8");
  if (f.vocab_size <= 0) return bad("vocab_size must be positive");
  if (f.max_pos <= 0) return bad("max_pos must be positive");
  if (f.kv_dtype != DLLM_KV_F32 && f.kv_dtype != DLLM_KV_BF16) return bad("kv_dtype must be DLLM_KV_F32 or DLLM_KV_BF16");
  if (f.kv_page_size < 32 || (f.kv_page_size & (f.kv_page_size - 1))) return bad("kv_page_size must be a power of two >= 32");
  if (f.max_seqs <= 0) return bad("max_seqs must be positive");
  if (!(f.rms_norm_eps > 0.f) || !(f.rope_theta > 0.f)) return bad("rms_norm_eps and rope_theta must be positive");
  snprintf(b, sizeof(b), "ok");
  *why = b;
  return true;
}

// ---- stage internals ------------------------------------------------------------------
const char* kLayerSuffix[] = {"input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
                              "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                              "self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias",
                              "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"};

dllm_buf* find_w(dllm_stage* s, const std::string& name) {
  auto it = s->W.find(name);
  return it == s->W.end() ? nullptr : it->second;
}

KvLayout stage_kv(const dllm_stage* s) {
  const dllm_config& f = s->ctx->cfg;
  KvLayout kv{};
  kv.k = kv.v = nullptr;
  kv.page_table = s->page_table;
  kv.log2_page = s->log2_page;
  kv.max_pages = s->pages_per_seq;
  kv.head_stride = s->page * f.head_dim;
  kv.row_stride = f.head_dim;
  kv.page_stride = (long long)f.num_kv_heads * s->page * f.head_dim;
  kv.max_slots = f.max_pos;
  kv.num_seqs = s->max_seqs;
  return kv;
}

size_t kv_esize(const dllm_ctx* c) { return c->cfg.kv_dtype == DLLM_KV_F32 ? 4 : 2; }

void* layer_pool(const dllm_stage* s, void* pool, int layer_global) {
  return (char*)pool + (size_t)(layer_global - s->start) * s->layer_elems * kv_esize(s->ctx);
}

// Resolve HF tensor names (weights.js:167-182) into per-layer device pointers.
int resolve(dllm_stage* s) {
  if (!s->dirty) return DLLM_OK;
  dllm_ctx* c = s->ctx;
  const dllm_config& f = c->cfg;
  const size_t D = f.hidden_size, QD = (size_t)f.num_q_heads * f.head_dim, KD = (size_t)f.num_kv_heads * f.head_dim,
               I = f.intermediate_size;
  const size_t need[12] = {D, D, QD * D, KD * D, KD * D, D * QD, QD, KD, KD, I * D, I * D, D * I};
  s->lw.assign(s->nl, LayerW{});
  for (int L = s->start; L < s->end; ++L) {
    const __nv_bfloat16* p[12];
    for (int i = 0; i < 12; ++i) {
      const std::string name = "model.layers." + std::to_string(L) + "." + kLayerSuffix[i];
      dllm_buf* b = find_w(s, name);
      const bool optional = (i >= 6 && i <= 8);
      if (!b) {
        if (optional) {
          p[i] = nullptr;
          continue;
        }
        return set_err(c, DLLM_ENOTFOUND, "missing weight %s", name.c_str());
      }
      int rc = check_bf16(c, b, need[i], name.c_str());
      if (rc) return rc;
      p[i] = (const __nv_bfloat16*)b->ptr;
    }
    LayerW& w = s->lw[L - s->start];
    w.ln1 = p[0];
    w.ln2 = p[1];
    w.wq = p[2];
    w.wk = p[3];
    w.wv = p[4];
    w.wo = p[5];
    w.bq = p[6];
    w.bk = p[7];
    w.bv = p[8];
    w.wg = p[9];
    w.wu = p[10];
    w.wd = p[11];
    w.kc = layer_pool(s, s->kpool, L);
    w.vc = layer_pool(s, s->vpool, L);
  }
  if (s->nl > 0) {
    if (!s->lw_dev) {
      int rc = dev_alloc(c, &s->lw_dev, (size_t)s->nl, "layer table");
      if (rc) return rc;
    }
    CK(c, cudaMemcpyAsync(s->lw_dev, s->lw.data(), sizeof(LayerW) * s->nl, cudaMemcpyHostToDevice, c->stream));
  }
  // optional leader weights
  dllm_buf* e = find_w(s, "model.embed_tokens.weight");
  dllm_buf* n = find_w(s, "model.norm.weight");
  dllm_buf* h = find_w(s, "lm_head.weight");
  s->embed = s->norm = s->lm_head = nullptr;
  if (e) {
    int rc = check_bf16(c, e, (size_t)f.vocab_size * D, "model.embed_tokens.weight");
    if (rc) return rc;
    s->embed = (const __nv_bfloat16*)e->ptr;
  }
  if (n) {
    int rc = check_bf16(c, n, D, "model.norm.weight");
    if (rc) return rc;
    s->norm = (const __nv_bfloat16*)n->ptr;
  }
  if (h) {
    int rc = check_bf16(c, h, (size_t)f.vocab_size * D, "lm_head.weight");
    if (rc) return rc;
    s->lm_head = (const __nv_bfloat16*)h->ptr;
  } else if (f.tie_word_embeddings && s->embed) {
    s->lm_head = s->embed;  // tied LM head = embed_tokens (pipeline.js:113-118)
  }
  s->dirty = false;
  return DLLM_OK;
}

int ensure_hbuf(dllm_stage* s, size_t rows) {
  if (rows <= s->hbuf_rows) return DLLM_OK;
  dllm_ctx* c = s->ctx;
  CK(c, cudaStreamSynchronize(c->stream));
  dev_free(s->hbuf);
  s->hbuf = nullptr;
  s->hbuf_rows = 0;
  int rc = dev_alloc(c, &s->hbuf, rows * (size_t)c->cfg.hidden_size, "hidden rows");
  if (rc) return rc;
  s->hbuf_rows = rows;
  return DLLM_OK;
}

int ensure_tokbuf(dllm_stage* s, size_t n) {
  if (n <= s->tokbuf_cap) return DLLM_OK;
  dllm_ctx* c = s->ctx;
  CK(c, cudaStreamSynchronize(c->stream));
  dev_free(s->tokbuf);
  s->tokbuf = nullptr;
  s->tokbuf_cap = 0;
  int rc = dev_alloc(c, &s->tokbuf, n, "token ids");
  if (rc) return rc;
  s->tokbuf_cap = n;
  return DLLM_OK;
}

StageParams base_params(dllm_stage* s) {
  dllm_ctx* c = s->ctx;
  const dllm_config& f = c->cfg;
  StageParams P{};
  P.D = f.hidden_size;
  P.NQ = f.num_q_heads;
  P.KVH = f.num_kv_heads;
  P.HD = f.head_dim;
  P.I = f.intermediate_size;
  P.V = f.vocab_size;
  P.log2_half = ilog2(f.head_dim / 2);
  P.eps = f.rms_norm_eps;
  P.scale = c->scale;
  P.n_layers = s->nl;
  P.layers = s->lw_dev;
  P.freq = c->freq;
  P.rows = s->rows;
  P.h = s->h;
  P.q = s->q;
  P.att = s->att;
  P.mid = s->mid;
  P.part_o = s->part_o;
  P.part_ml = s->part_ml;
  P.arrive = s->arrive;
  P.h2 = s->h2;
  P.acc = reinterpret_cast<long long*>(s->bar + 4);
  P.kv = stage_kv(s);
  P.embed = s->embed;
  P.final_norm = s->norm;
  P.best = s->best;
  P.tokens_out = s->tok;
  P.bar_count = s->bar;
  P.bar_epoch = s->bar + 1;
  P.err = c->err_dev;
  P.pref_bytes = kPrefetchBytes;
  P.trace = s->trace;
  P.trace_cap = s->trace_cap;
  P.attn_kv_floats = (long long)f.max_pos * f.num_kv_heads > (long long)dllm::kAttnRingSlots * c->sms
                         ? dllm::kAttnKvLongFloats : 0;
  P.xs_floats = dllm::kStageXsFloats;
  P.part_floats = dllm::kStagePartFloats;
  return P;
}

// Grow the ctx's tensor-core scratch to `bytes` (synchronises the stream first).
int ensure_tc_scratch(dllm_ctx* c, size_t bytes) {
  if (bytes <= c->tc_scratch_bytes) return DLLM_OK;
  CK(c, cudaStreamSynchronize(c->stream));
  dev_free(c->tc_scratch);
  c->tc_scratch = nullptr;
  c->tc_scratch_bytes = 0;
  char* p = nullptr;
  if (int rc = dev_alloc(c, &p, bytes, "tensor-core scratch")) return rc;
  c->tc_scratch = p;
  c->tc_scratch_bytes = bytes;
  return DLLM_OK;
}

// y[t] (=|+=) rmsnorm?(x[t]) . W^T for n rows on the tensor cores, in launches of
// up to kTcMaxRows rows (MATMUL, kernels.js:26-44, for n > 1).
int tc_rows(dllm_ctx* c, const float* x, int n, int K, const __nv_bfloat16* w, int N, float* y, int accumulate,
            const __nv_bfloat16* norm_w) {
  for (int r0 = 0; r0 < n; r0 += dllm::kTcMaxRows) {
    const int m = std::min(dllm::kTcMaxRows, n - r0);
    const size_t need = dllm::tc_matmul_scratch_bytes(m, K, N, c->sms);
    if (int rc = ensure_tc_scratch(c, need)) return rc;
    cudaError_t e = dllm::tc_matmul(x + (size_t)r0 * K, m, K, w, N, y + (size_t)r0 * N, accumulate, norm_w,
                                    c->cfg.rms_norm_eps, c->tc_scratch, c->tc_scratch_bytes, c->err_dev, c->sms,
                                    c->stream);
    if (e != cudaSuccess) return set_err(c, DLLM_ECUDA, "tensor-core matmul: %s", cudaGetErrorString(e));
    c->launches += 2;
  }
  return DLLM_OK;
}

// Several projections of the same rows (q|k|v, gate|up) in one tensor-core launch
// per chunk of kTcMaxRows rows, behind one RMSNorm + hi/lo split.
int tc_rows_multi(dllm_ctx* c, const float* x, int n, int K, const dllm::TcTarget* t, int nt,
                  const __nv_bfloat16* norm_w) {
  int Ns[3];
  for (int i = 0; i < nt; ++i) Ns[i] = t[i].N;
  for (int r0 = 0; r0 < n; r0 += dllm::kTcMaxRows) {
    const int m = std::min(dllm::kTcMaxRows, n - r0);
    const size_t need = dllm::tc_matmul_multi_scratch_bytes(m, K, Ns, nt, c->sms);
    if (int rc = ensure_tc_scratch(c, need)) return rc;
    dllm::TcTarget tt[3];
    for (int i = 0; i < nt; ++i) tt[i] = dllm::TcTarget{t[i].w, t[i].N, t[i].y + (size_t)r0 * t[i].N, t[i].accumulate};
    cudaError_t e = dllm::tc_matmul_multi(x + (size_t)r0 * K, m, K, tt, nt, norm_w, c->cfg.rms_norm_eps,
                                          c->tc_scratch, c->tc_scratch_bytes, c->err_dev, c->sms, c->stream);
    if (e != cudaSuccess) return set_err(c, DLLM_ECUDA, "tensor-core matmul: %s", cudaGetErrorString(e));
    c->launches += 2;
  }
  return DLLM_OK;
}

int launch(dllm_stage* s, StageParams& P) {
  dllm_ctx* c = s->ctx;
  int ms = c->sms / (P.m_rows * P.KVH);
  if (ms < 1) ms = 1;
  if (ms > kMaxSplitsAlloc) ms = kMaxSplitsAlloc;
  P.max_splits = ms;
  cudaError_t e = dllm::launch_stage(P, c->cfg.kv_dtype, c->sms, c->stream);
  if (e != cudaSuccess) return set_err(c, DLLM_ECUDA, "stage kernel launch: %s", cudaGetErrorString(e));
  c->launches += 1;
  return DLLM_OK;
}

// Whether a pass of n rows takes the wide path (tensor-core projections).
bool use_wide(const dllm_stage* s, int n) {
  const int t = s->ctx->tc_min_rows;
  return t > 0 && n >= t;
}

// Per-row workspaces of wide passes for up to `rows` rows (chunks of kTcMaxRows).
int ensure_wide(dllm_stage* s, int rows, bool logits) {
  dllm_ctx* c = s->ctx;
  const dllm_config& f = c->cfg;
  const int cap = std::min(rows, dllm::kTcMaxRows);
  if (cap > s->wide_cap) {
    CK(c, cudaStreamSynchronize(c->stream));
    for (float** p : {&s->wq, &s->wk, &s->wv, &s->watt, &s->wg, &s->wu, &s->wpart_o, &s->wpart_ml, &s->wlogits}) {
      dev_free(*p);
      *p = nullptr;
    }
    dev_free(s->warrive);
    dev_free(s->wrows);
    dev_free(s->wbest);
    s->warrive = nullptr;
    s->wrows = nullptr;
    s->wbest = nullptr;
    s->wide_cap = 0;
    const size_t R = cap, QD = (size_t)f.num_q_heads * f.head_dim, KD = (size_t)f.num_kv_heads * f.head_dim;
    s->wide_splits = std::max(1, std::min(kMaxSplitsAlloc, c->sms / (dllm::kMaxRows * f.num_kv_heads)));
    const size_t ms = s->wide_splits;
    int rc = dev_alloc(c, &s->wq, R * QD, "wide q");
    if (!rc) rc = dev_alloc(c, &s->wk, R * KD, "wide k");
    if (!rc) rc = dev_alloc(c, &s->wv, R * KD, "wide v");
    if (!rc) rc = dev_alloc(c, &s->watt, R * QD, "wide attention");
    if (!rc) rc = dev_alloc(c, &s->wg, R * f.intermediate_size, "wide gate");
    if (!rc) rc = dev_alloc(c, &s->wu, R * f.intermediate_size, "wide up");
    if (!rc) rc = dev_alloc(c, &s->wpart_o, R * f.num_q_heads * ms * f.head_dim, "wide attention partials");
    if (!rc) rc = dev_alloc(c, &s->wpart_ml, R * f.num_q_heads * ms * 2, "wide attention partials");
    if (!rc) rc = dev_alloc(c, &s->warrive, 2 * R * f.num_kv_heads, "wide attention tickets");
    if (!rc) rc = dev_alloc(c, &s->wrows, R, "wide rows");
    if (!rc) rc = dev_alloc(c, &s->wbest, R, "wide argmax keys");
    if (rc) return rc;
    s->wide_cap = cap;
  }
  if (logits && !s->wlogits) {
    if (int rc = dev_alloc(c, &s->wlogits, (size_t)s->wide_cap * f.vocab_size, "wide logits")) return rc;
  }
  return DLLM_OK;
}

// A wide pass of n rows (rd[t] = {seq, pos, slot}) over the stage's layers, one
// kernel per op: RMSNorm + q|k|v projections on the tensor cores, bias + RoPE +
// appendKv, attention over the paged cache, o_proj + residual, RMSNorm + gate|up,
// SiLU(gate)*up, down_proj + residual (the op order of pipeline.js:52-75). With
// tokens_in the rows start as token embeddings (pipeline.js:121-128); with
// tokens_out each row ends with final norm + LM head + greedy argmax
// (pipeline.js:141-174).
int run_wide(dllm_stage* s, float* h, int n, const RowDesc* rd, const int32_t* tokens_in, int32_t* tokens_out) {
  dllm_ctx* c = s->ctx;
  const dllm_config& f = c->cfg;
  const int D = f.hidden_size, QD = f.num_q_heads * f.head_dim, KD = f.num_kv_heads * f.head_dim,
            I = f.intermediate_size;
  if (int rc = ensure_wide(s, n, tokens_out != nullptr)) return rc;
  const KvLayout kv = stage_kv(s);
  for (int r0 = 0; r0 < n; r0 += s->wide_cap) {
    const int m = std::min(s->wide_cap, n - r0);
    float* hh = h + (size_t)r0 * D;
    CK(c, cudaMemcpyAsync(s->wrows, rd + r0, sizeof(RowDesc) * m, cudaMemcpyHostToDevice, c->stream));
    if (tokens_in) {
      CK(c, dllm::op_embed(s->embed, tokens_in + r0, hh, m, D, f.vocab_size, c->err_dev, c->stream));
      c->launches += 1;
    }
    for (int l = 0; l < s->nl; ++l) {
      const LayerW& L = s->lw[l];
      const dllm::TcTarget qkv[3] = {{L.wq, QD, s->wq, 0}, {L.wk, KD, s->wk, 0}, {L.wv, KD, s->wv, 0}};
      if (int rc = tc_rows_multi(c, hh, m, D, qkv, 3, L.ln1)) return rc;
      CK(c, dllm::op_qkv_post(s->wq, s->wk, s->wv, L.bq, L.bk, L.bv, m, f.num_q_heads, f.num_kv_heads, f.head_dim,
                              c->freq, s->wrows, kv, L.kc, L.vc, f.kv_dtype, c->err_dev, c->stream));
      const dllm::AttnArgs A{s->wq, s->watt, L.kc, L.vc, kv, s->wrows, m, f.num_q_heads, f.num_kv_heads, c->scale,
                             s->wide_splits, s->wpart_o, s->wpart_ml, s->warrive, c->err_dev};
      CK(c, dllm::op_attention_paged(A, f.kv_dtype, f.head_dim, c->sms, c->stream));
      if (int rc = tc_rows(c, s->watt, m, QD, L.wo, D, hh, 1, nullptr)) return rc;
      const dllm::TcTarget gu[2] = {{L.wg, I, s->wg, 0}, {L.wu, I, s->wu, 0}};
      if (int rc = tc_rows_multi(c, hh, m, D, gu, 2, L.ln2)) return rc;
      CK(c, dllm::op_silu_mul(s->wg, s->wu, s->wg, m * I, c->stream));
      if (int rc = tc_rows(c, s->wg, m, I, L.wd, D, hh, 1, nullptr)) return rc;
      c->launches += 3;
    }
    if (tokens_out) {
      if (int rc = tc_rows(c, hh, m, D, s->lm_head, f.vocab_size, s->wlogits, 0, s->norm)) return rc;
      CK(c, dllm::op_argmax_rows(s->wlogits, m, f.vocab_size, s->wbest, tokens_out + r0, c->stream));
      c->launches += 2;
    }
  }
  return DLLM_OK;
}

// Run n rows through the stage: rows t = {seq, pos0 + t, T0 + t}. A wide pass on
// the tensor cores when n reaches the ctx's tensor-core rows, else passes of <= 8
// rows of the persistent stage kernel.
int run_rows(dllm_stage* s, float* hrows, int n, int seq, int pos0, const int32_t* tokens_dev) {
  dllm_ctx* c = s->ctx;
  if (use_wide(s, n)) {
    std::vector<RowDesc> rd(n);
    for (int t = 0; t < n; ++t) rd[t] = RowDesc{seq, pos0 + t, s->T0[seq] + t, 0};
    return run_wide(s, hrows, n, rd.data(), tokens_dev, nullptr);
  }
  for (int r0 = 0; r0 < n; r0 += dllm::kMaxRows) {
    const int m = std::min(dllm::kMaxRows, n - r0);
    RowDesc rd[dllm::kMaxRows];
    for (int t = 0; t < m; ++t) rd[t] = RowDesc{seq, pos0 + r0 + t, s->T0[seq] + r0 + t, 0};
    CK(c, cudaMemcpyAsync(s->rows, rd, sizeof(RowDesc) * m, cudaMemcpyHostToDevice, c->stream));
    StageParams P = base_params(s);
    P.m_rows = m;
    P.h = hrows + (size_t)r0 * c->cfg.hidden_size;
    P.tokens_in = tokens_dev ? tokens_dev + r0 : nullptr;
    P.lm_head = nullptr;
    int rc = launch(s, P);
    if (rc) return rc;
  }
  return DLLM_OK;
}

// Final norm + LM head + argmax of one row (sampleLast, pipeline.js:141-174).
int run_head(dllm_stage* s, float* hrow, int32_t* tok_out, float* logits, int logits_cap, int* step_count,
             int32_t* hist, int hist_cap) {
  StageParams P = base_params(s);
  P.n_layers = 0;
  P.m_rows = 1;
  P.h = hrow;
  P.lm_head = s->lm_head;
  P.tokens_out = tok_out;
  P.logits = logits;
  P.logits_cap = logits_cap;
  P.step_count = step_count;
  P.history = hist;
  P.hist_cap = hist_cap;
  return launch(s, P);
}

int need_head(dllm_stage* s) {
  if (!s->norm) return set_err(s->ctx, DLLM_ENOTFOUND, "missing weight model.norm.weight");
  if (!s->lm_head)
    return set_err(s->ctx, DLLM_ENOTFOUND, "missing weight lm_head.weight (and embeddings are not tied)");
  return DLLM_OK;
}

void rope_table(const dllm_config& f, std::vector<float>* out) {
  // freq = exp2(-2*half/HD * log2(theta)) with f32 rounding at each step (kernels.js:77)
  const int halfn = f.head_dim / 2;
  out->resize(halfn);
  const float l2t = (float)std::log2((double)f.rope_theta);
  for (int h = 0; h < halfn; ++h) {
    const float a = -2.0f * (float)h;
    const float b = a / (float)f.head_dim;
    const float e = b * l2t;
    (*out)[h] = (float)std::exp2((double)e);
  }
}

}  // namespace

namespace {
void ctx_free(dllm_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  dev_free(c->freq);
  dev_free(c->err_dev);
  dev_free(c->best);
  dev_free(c->attn.part_o);
  dev_free(c->attn.part_ml);
  dev_free(c->attn.arrive);
  dev_free(c->attn_rows);
  dev_free(c->tc_scratch);
  for (auto& kv : c->buf_cache) cudaFree(kv.second);
  c->buf_cache.clear();
  if (c->err_host) cudaFreeHost(c->err_host);
  if (c->best_host) cudaFreeHost(c->best_host);
  if (c->sync_event) cudaEventDestroy(c->sync_event);
  if (c->own_stream) cudaStreamDestroy(c->own_stream);
  delete c;
}
}  // namespace

// =====================================================================================
extern "C" {

const char* dllm_version(void) { return "dllm-b200 0.1 (sm_100a)"; }

const char* dllm_status_string(int s) {
  switch (s) {
    case DLLM_OK: return "ok";
    case DLLM_EINVAL: return "invalid argument";
    case DLLM_ENOMEM: return "out of device memory";
    case DLLM_ERANGE: return "KV cache overflow";
    case DLLM_ETIMEOUT: return "timeout";
    case DLLM_ECUDA: return "CUDA error";
    case DLLM_ENOTFOUND: return "weight not found";
    case DLLM_EDEVICE: return "device error";
    default: return "unknown status";
  }
}

void dllm_config_default(dllm_config* f) {
  if (!f) return;
  memset(f, 0, sizeof(*f));
  f->vocab_size = 151936;
  f->hidden_size = 1536;
  f->num_layers = 28;
  f->num_q_heads = 12;
  f->num_kv_heads = 2;
  f->head_dim = 128;
  f->intermediate_size = 8960;
  f->rope_theta = 1000000.0f;
  f->rms_norm_eps = 1e-6f;
  f->tie_word_embeddings = 1;
  f->eos_token_id = 151645;
  f->max_pos = 4096;
  f->kv_dtype = DLLM_KV_F32;
  f->kv_page_size = 64;
  f->max_seqs = 1;
}

int dllm_init_kernels(int device, const dllm_config* cfg, dllm_ctx** out) {
  if (!out) return DLLM_EINVAL;
  *out = nullptr;
  dllm_config f;
  if (cfg) f = *cfg;
  else dllm_config_default(&f);
  std::string why;
  if (!valid_config(f, &why)) return DLLM_EINVAL;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) {
    cudaGetLastError();
    return DLLM_ECUDA;
  }
  if (device < 0 || device >= ndev) return DLLM_EINVAL;
  auto* c = new dllm_ctx();
  c->device = device;
  c->cfg = f;
  auto fail = [&](int code) {
    dllm_ctx_destroy(c);
    return code;
  };
  if (use_device(c)) return fail(DLLM_ECUDA);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return fail(DLLM_ECUDA);
  if (prop.major < 10) return fail(DLLM_EDEVICE);  // built for sm_100a only
  c->sms = prop.multiProcessorCount;
  if (dllm::configure_stage_kernels() != cudaSuccess || dllm::configure_op_kernels() != cudaSuccess) {
    cudaGetLastError();
    return fail(DLLM_ECUDA);
  }
  if (cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess) return fail(DLLM_ECUDA);
  c->stream = c->own_stream;
  if (cudaEventCreateWithFlags(&c->sync_event, cudaEventDisableTiming) != cudaSuccess) return fail(DLLM_ECUDA);
  if (cudaMallocHost(&c->err_host, sizeof(int)) != cudaSuccess) return fail(DLLM_ENOMEM);
  *c->err_host = 0;
  if (cudaMallocHost(&c->best_host, sizeof(unsigned long long)) != cudaSuccess) return fail(DLLM_ENOMEM);
  if (dev_alloc(c, &c->err_dev, 1, "error flag")) return fail(DLLM_ENOMEM);
  if (dev_alloc(c, &c->best, 1, "argmax")) return fail(DLLM_ENOMEM);
  std::vector<float> fr;
  rope_table(f, &fr);
  if (dev_alloc(c, &c->freq, fr.size(), "rope table")) return fail(DLLM_ENOMEM);
  if (cudaMemcpyAsync(c->freq, fr.data(), fr.size() * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
    return fail(DLLM_ECUDA);
  c->scale = (float)(1.0 / std::sqrt((double)f.head_dim));
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return fail(DLLM_ECUDA);
  *out = c;
  return DLLM_OK;
}

void dllm_ctx_destroy(dllm_ctx* c) { ctx_release(c); }



const char* dllm_last_error(const dllm_ctx* c) { return c ? c->err.c_str() : "null context"; }

int dllm_ctx_get_config(const dllm_ctx* c, dllm_config* out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = c->cfg;
  return DLLM_OK;
}

int dllm_ctx_set_stream(dllm_ctx* c, void* s) {
  if (!c) return DLLM_EINVAL;
  c->stream = s ? (cudaStream_t)s : c->own_stream;
  return DLLM_OK;
}

int dllm_ctx_synchronize(dllm_ctx* c, int timeout_ms) {
  if (!c) return DLLM_EINVAL;
  if (int rc = use_device(c)) return rc;
  return sync_check(c, timeout_ms);
}

uint64_t dllm_ctx_launch_count(const dllm_ctx* c) { return c ? c->launches : 0; }

int dllm_ctx_set_tensor_core_rows(dllm_ctx* c, int min_rows) {
  if (!c) return DLLM_EINVAL;
  if (min_rows != 0 && (min_rows < 2 || min_rows > dllm::kTcMaxRows))
    return set_err(c, DLLM_EINVAL, "tensor_core_rows: %d outside 0 or [2, %d]", min_rows, dllm::kTcMaxRows);
  if (min_rows != 0 && !dllm::tc_available())
    return set_err(c, DLLM_ECUDA, "tensor_core_rows: the driver has no tensor-map encoder");
  c->tc_min_rows = min_rows;
  return DLLM_OK;
}

// ---- buffers -----------------------------------------------------------------------------
int dllm_load_weight_bits(dllm_ctx* c, const uint32_t* bits, size_t n, const char* label, dllm_buf** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  if (!bits || n == 0) return set_err(c, DLLM_EINVAL, "loadWeightBits: empty weights");  // kernels.js:182
  if (int rc = use_device(c)) return rc;
  // keep the low 16 bits of every u32 (the shader reads bits << 16, kernels.js:20)
  std::vector<uint16_t> packed(n);
  for (size_t i = 0; i < n; ++i) packed[i] = (uint16_t)(bits[i] & 0xffffu);
  return dllm_load_weight_bf16(c, packed.data(), n, label, out);
}

int dllm_load_weight_bf16(dllm_ctx* c, const uint16_t* bf16, size_t n, const char* label, dllm_buf** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  if (!bf16 || n == 0) return set_err(c, DLLM_EINVAL, "loadWeightBits: empty weights");
  if (int rc = use_device(c)) return rc;
  dllm_buf* b = nullptr;
  if (int rc = new_buf(c, n, 1, label ? label : "weights", &b)) return rc;
  cudaError_t e = cudaMemcpyAsync(b->ptr, bf16, n * 2, cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) {
    dllm_buf_free(b);
    return set_err(c, DLLM_ECUDA, "weight upload: %s", cudaGetErrorString(e));
  }
  *out = b;
  return DLLM_OK;
}

int dllm_create_f32(dllm_ctx* c, size_t n, const char* label, dllm_buf** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  if (n == 0) return set_err(c, DLLM_EINVAL, "createF32: invalid size %zu", n);  // kernels.js:189
  if (int rc = use_device(c)) return rc;
  return new_buf(c, n, 0, label, out);
}

int dllm_create_bf16(dllm_ctx* c, size_t n, const char* label, dllm_buf** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  if (n == 0) return set_err(c, DLLM_EINVAL, "create_bf16: invalid size %zu", n);
  if (int rc = use_device(c)) return rc;
  return new_buf(c, n, 1, label, out);
}

int dllm_write_f32(dllm_ctx* c, dllm_buf* b, const float* src, size_t n) {
  if (!c) return DLLM_EINVAL;
  if (int rc = check_f32(c, b, n, "writeF32")) return rc;
  if (!src && n) return set_err(c, DLLM_EINVAL, "writeF32: null source");
  if (int rc = use_device(c)) return rc;
  CK(c, cudaMemcpyAsync(b->ptr, src, n * 4, cudaMemcpyHostToDevice, c->stream));
  return DLLM_OK;
}

int dllm_read_f32(dllm_ctx* c, const dllm_buf* b, float* dst, size_t n, const char* label) {
  if (!c) return DLLM_EINVAL;
  if (n == 0) return set_err(c, DLLM_EINVAL, "readF32: invalid size 0");  // kernels.js:196
  if (int rc = check_f32(c, b, n, "readF32")) return rc;
  if (!dst) return set_err(c, DLLM_EINVAL, "readF32: null destination");
  if (int rc = use_device(c)) return rc;
  CK(c, cudaMemcpyAsync(dst, b->ptr, n * 4, cudaMemcpyDeviceToHost, c->stream));
  int rc = sync_check(c, kDefaultTimeoutMs);
  if (rc == DLLM_ETIMEOUT)
    return set_err(c, rc, "readF32 timeout (%s, %zu floats)", label ? label : "", n);
  return rc;
}

int dllm_read_bf16(dllm_ctx* c, const dllm_buf* b, uint16_t* dst, size_t n) {
  if (!c) return DLLM_EINVAL;
  if (int rc = check_bf16(c, b, n, "read_bf16")) return rc;
  if (!dst) return set_err(c, DLLM_EINVAL, "read_bf16: null destination");
  if (int rc = use_device(c)) return rc;
  CK(c, cudaMemcpyAsync(dst, b->ptr, n * 2, cudaMemcpyDeviceToHost, c->stream));
  return sync_check(c, kDefaultTimeoutMs);
}

void dllm_buf_free(dllm_buf* b) {
  if (!b) return;
  if (--b->refs > 0) return;
  dllm_ctx* c = b->ctx;
  if (b->ptr) {
    if (c && c->buf_cache_bytes + b->bytes <= kBufCacheBytes) {
      c->buf_cache.emplace(b->bytes, b->ptr);  // reused by the next buffer of this size
      c->buf_cache_bytes += b->bytes;
    } else {
      cudaSetDevice(b->device);
      cudaFree(b->ptr);
    }
  }
  delete b;
  ctx_release(c);
}

size_t dllm_buf_bytes(const dllm_buf* b) { return b ? b->bytes : 0; }
void* dllm_buf_device_ptr(const dllm_buf* b) { return b ? b->ptr : nullptr; }

int dllm_fill_normal_bf16(dllm_ctx* c, dllm_buf* b, uint64_t seed, float std) {
  if (!c) return DLLM_EINVAL;
  if (int rc = check_bf16(c, b, 1, "fill_normal_bf16")) return rc;
  if (int rc = use_device(c)) return rc;
  CK(c, dllm::op_fill_normal_bf16((__nv_bfloat16*)b->ptr, b->n, seed, std, c->stream));
  c->launches += 1;
  return DLLM_OK;
}

int dllm_fill_const_bf16(dllm_ctx* c, dllm_buf* b, float v) {
  if (!c) return DLLM_EINVAL;
  if (int rc = check_bf16(c, b, 1, "fill_const_bf16")) return rc;
  if (int rc = use_device(c)) return rc;
  CK(c, dllm::op_fill_const_bf16((__nv_bfloat16*)b->ptr, b->n, v, c->stream));
  c->launches += 1;
  return DLLM_OK;
}

// ---- ops (kernels.js:222-301) ----------------------------------------------------------------
int dllm_matmul(dllm_ctx* c, const dllm_buf* x, const dllm_buf* w, int n, int din, int dout, dllm_buf** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  if (n <= 0 || din <= 0 || dout <= 0) return set_err(c, DLLM_EINVAL, "matmul: invalid n=%d din=%d dout=%d", n, din, dout);
  if (din % 8) return set_err(c, DLLM_EINVAL, "matmul: din=%d must be a multiple of 8", din);
  if (int rc = check_f32(c, x, (size_t)n * din, "matmul x")) return rc;
  if (int rc = check_bf16(c, w, (size_t)din * dout, "matmul w")) return rc;
  if (int rc = use_device(c)) return rc;
  dllm_buf* o = nullptr;
  if (int rc = new_buf(c, (size_t)n * dout, 0, "mm_out", &o, false)) return rc;
  if (c->tc_min_rows > 0 && n >= c->tc_min_rows) {
    // a real GEMM: the tcgen05 path
    if (int rc = tc_rows(c, (const float*)x->ptr, n, din, (const __nv_bfloat16*)w->ptr, dout, (float*)o->ptr, 0,
                         nullptr)) {
      dllm_buf_free(o);
      return rc;
    }
    *out = o;
    return DLLM_OK;
  }
  cudaError_t e = dllm::op_matmul((const float*)x->ptr, (const __nv_bfloat16*)w->ptr, (float*)o->ptr, n, din, dout,
                                  c->sms, c->stream);
  if (e != cudaSuccess) {
    dllm_buf_free(o);
    return set_err(c, DLLM_ECUDA, "matmul launch: %s", cudaGetErrorString(e));
  }
  c->launches += 1;
  *out = o;
  return DLLM_OK;
}

int dllm_rmsnorm(dllm_ctx* c, const dllm_buf* x, const dllm_buf* g, int n, dllm_buf** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  const int D = c->cfg.hidden_size;
  if (n <= 0) return set_err(c, DLLM_EINVAL, "rmsnorm: invalid n=%d", n);
  if (int rc = check_f32(c, x, (size_t)n * D, "rmsnorm x")) return rc;
  if (int rc = check_bf16(c, g, (size_t)D, "rmsnorm g")) return rc;
  if (int rc = use_device(c)) return rc;
  dllm_buf* o = nullptr;
  if (int rc = new_buf(c, (size_t)n * D, 0, "rms_out", &o, false)) return rc;
  cudaError_t e = dllm::op_rmsnorm((const float*)x->ptr, (const __nv_bfloat16*)g->ptr, (float*)o->ptr, n, D,
                                   c->cfg.rms_norm_eps, c->stream);
  if (e != cudaSuccess) {
    dllm_buf_free(o);
    return set_err(c, DLLM_ECUDA, "rmsnorm launch: %s", cudaGetErrorString(e));
  }
  c->launches += 1;
  *out = o;
  return DLLM_OK;
}

static int rope_common(dllm_ctx* c, dllm_buf* x, int pos_start, int n, int heads, const char* what) {
  if (!c) return DLLM_EINVAL;
  if (n <= 0) return set_err(c, DLLM_EINVAL, "rope: invalid n=%d", n);  // kernels.js:244
  if (pos_start < 0) return set_err(c, DLLM_EINVAL, "rope: invalid posStart=%d", pos_start);
  const int HD = c->cfg.head_dim;
  if (int rc = check_f32(c, x, (size_t)n * heads * HD, what)) return rc;
  if (int rc = use_device(c)) return rc;
  CK(c, dllm::op_rope((float*)x->ptr, n, heads, HD, pos_start, c->freq, c->stream));
  c->launches += 1;
  return DLLM_OK;
}

int dllm_rope_q(dllm_ctx* c, dllm_buf* x, int pos_start, int n) {
  return rope_common(c, x, pos_start, n, c ? c->cfg.num_q_heads : 0, "ropeQ x");
}
int dllm_rope_k(dllm_ctx* c, dllm_buf* x, int pos_start, int n) {
  return rope_common(c, x, pos_start, n, c ? c->cfg.num_kv_heads : 0, "ropeK x");
}

int dllm_attention(dllm_ctx* c, const dllm_buf* q, const dllm_buf* kcache, const dllm_buf* vcache, int t0, int n,
                   dllm_buf** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  const dllm_config& f = c->cfg;
  const int QD = f.num_q_heads * f.head_dim, KD = f.num_kv_heads * f.head_dim;
  if (n <= 0 || t0 < 0) return set_err(c, DLLM_EINVAL, "attention: invalid T0=%d n=%d", t0, n);
  if (int rc = check_f32(c, q, (size_t)n * QD, "attention q")) return rc;
  const size_t slots = (size_t)t0 + n;
  if (int rc = check_f32(c, kcache, slots * KD, "attention kCache")) return rc;
  if (int rc = check_f32(c, vcache, slots * KD, "attention vCache")) return rc;
  const int max_pos = (int)std::min(kcache->n, vcache->n) / KD;
  if (int rc = use_device(c)) return rc;
  // scratch: partials for up to n rows
  if ((size_t)n > c->attn_rows_cap) {
    CK(c, cudaStreamSynchronize(c->stream));
    dev_free(c->attn.part_o);
    dev_free(c->attn.part_ml);
    dev_free(c->attn.arrive);
    dev_free(c->attn_rows);
    c->attn = dllm::AttnScratch{};
    c->attn_rows = nullptr;
    c->attn_rows_cap = 0;
    const size_t cap = std::max<size_t>(n, 8);
    if (int rc = dev_alloc(c, &c->attn.part_o, cap * f.num_q_heads * kMaxSplitsAlloc * f.head_dim, "attn partials"))
      return rc;
    if (int rc = dev_alloc(c, &c->attn.part_ml, cap * f.num_q_heads * kMaxSplitsAlloc * 2, "attn partials"))
      return rc;
    if (int rc = dev_alloc(c, &c->attn.arrive, 2 * cap * f.num_kv_heads, "attn tickets")) return rc;
    if (int rc = dev_alloc(c, &c->attn_rows, cap, "attn rows")) return rc;
    c->attn_rows_cap = cap;
  }
  std::vector<RowDesc> rd(n);
  for (int t = 0; t < n; ++t) rd[t] = RowDesc{0, t0 + t, t0 + t, 0};  // Tend = T0 + t + 1 (kernels.js:121)
  CK(c, cudaMemcpyAsync(c->attn_rows, rd.data(), sizeof(RowDesc) * n, cudaMemcpyHostToDevice, c->stream));
  int ms = c->sms / (std::max(1, std::min(n, 8)) * f.num_kv_heads);
  c->attn.max_splits = std::max(1, std::min(ms, kMaxSplitsAlloc));
  dllm_buf* o = nullptr;
  if (int rc = new_buf(c, (size_t)n * QD, 0, "attn_out", &o, false)) return rc;
  cudaError_t e = dllm::op_attention((const float*)q->ptr, (const float*)kcache->ptr, (const float*)vcache->ptr,
                                     (float*)o->ptr, c->attn_rows, n, f.num_q_heads, f.num_kv_heads, f.head_dim,
                                     max_pos, c->scale, c->attn, c->err_dev, c->sms, c->stream);
  if (e != cudaSuccess) {
    dllm_buf_free(o);
    return set_err(c, DLLM_ECUDA, "attention launch: %s", cudaGetErrorString(e));
  }
  c->launches += 1;
  *out = o;
  return DLLM_OK;
}

int dllm_silu_mul(dllm_ctx* c, const dllm_buf* a, const dllm_buf* b, int total, dllm_buf** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  if (total <= 0) return set_err(c, DLLM_EINVAL, "siluMul: invalid total=%d", total);
  if (int rc = check_f32(c, a, total, "siluMul a")) return rc;
  if (int rc = check_f32(c, b, total, "siluMul b")) return rc;
  if (int rc = use_device(c)) return rc;
  dllm_buf* o = nullptr;
  if (int rc = new_buf(c, total, 0, "silu_out", &o, false)) return rc;
  CK(c, dllm::op_silu_mul((const float*)a->ptr, (const float*)b->ptr, (float*)o->ptr, total, c->stream));
  c->launches += 1;
  *out = o;
  return DLLM_OK;
}

int dllm_add(dllm_ctx* c, const dllm_buf* a, const dllm_buf* b, int n, dllm_buf** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  if (n <= 0) return set_err(c, DLLM_EINVAL, "add: invalid n=%d", n);
  if (int rc = check_f32(c, a, n, "add a")) return rc;
  if (int rc = check_f32(c, b, n, "add b")) return rc;
  if (int rc = use_device(c)) return rc;
  dllm_buf* o = nullptr;
  if (int rc = new_buf(c, n, 0, "add_out", &o, false)) return rc;
  CK(c, dllm::op_add((const float*)a->ptr, (const float*)b->ptr, (float*)o->ptr, n, c->stream));
  c->launches += 1;
  *out = o;
  return DLLM_OK;
}

int dllm_add_bias(dllm_ctx* c, const dllm_buf* a, const dllm_buf* bias, int n, int dout, dllm_buf** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  if (n <= 0 || dout <= 0) return set_err(c, DLLM_EINVAL, "addBias: invalid n=%d dout=%d", n, dout);
  const long long total = (long long)n * dout;
  if (total > 0x7fffffff) return set_err(c, DLLM_EINVAL, "addBias: too large");
  if (int rc = check_f32(c, a, (size_t)total, "addBias a")) return rc;
  if (int rc = check_bf16(c, bias, dout, "addBias bias")) return rc;
  if (int rc = use_device(c)) return rc;
  dllm_buf* o = nullptr;
  if (int rc = new_buf(c, (size_t)total, 0, "bias_out", &o, false)) return rc;
  CK(c, dllm::op_add_bias((const float*)a->ptr, (const __nv_bfloat16*)bias->ptr, (float*)o->ptr, (int)total, dout,
                          c->stream));
  c->launches += 1;
  *out = o;
  return DLLM_OK;
}

int dllm_argmax(dllm_ctx* c, const dllm_buf* logits, int n, int32_t* index_out) {
  if (!c || !index_out) return DLLM_EINVAL;
  if (n <= 0) return set_err(c, DLLM_EINVAL, "argmax: invalid n=%d", n);
  if (int rc = check_f32(c, logits, n, "argmax logits")) return rc;
  if (int rc = use_device(c)) return rc;
  CK(c, cudaMemsetAsync(c->best, 0, sizeof(unsigned long long), c->stream));
  CK(c, dllm::op_argmax((const float*)logits->ptr, n, c->best, c->stream));
  c->launches += 1;
  CK(c, cudaMemcpyAsync(c->best_host, c->best, sizeof(unsigned long long), cudaMemcpyDeviceToHost, c->stream));
  if (int rc = sync_check(c, kDefaultTimeoutMs)) return rc;
  const unsigned long long k = *c->best_host;
  // all-NaN / all -inf input: index 0, like the reference's initial best = 0
  *index_out = k == 0 ? 0 : (int32_t)(~(uint32_t)(k & 0xffffffffull));
  return DLLM_OK;
}

// ---- Stage (pipeline.js:26-88) -------------------------------------------------------------
void dllm_stage_destroy(dllm_stage* s);

int dllm_stage_create(dllm_ctx* c, int start, int end, dllm_stage** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  const dllm_config& f = c->cfg;
  if (start < 0 || end < start || end > f.num_layers)
    return set_err(c, DLLM_EINVAL, "Stage: invalid layer range [%d,%d) of %d", start, end, f.num_layers);
  if (int rc = use_device(c)) return rc;
  auto* s = new dllm_stage();
  s->ctx = c;
  ctx_retain(c);
  s->start = start;
  s->end = end;
  s->nl = end - start;
  s->page = f.kv_page_size;
  s->log2_page = ilog2(f.kv_page_size);
  s->pages_per_seq = (f.max_pos + s->page - 1) / s->page;
  s->max_seqs = f.max_seqs;
  s->max_slots = f.max_pos;
  s->layer_elems = (size_t)s->max_seqs * s->pages_per_seq * f.num_kv_heads * s->page * f.head_dim;
  s->T0.assign(s->max_seqs, 0);
  const size_t D = f.hidden_size, QD = (size_t)f.num_q_heads * f.head_dim;
  const size_t R = dllm::kMaxRows;
  int rc = DLLM_OK;
  auto alloc_pool = [&](void** p) {
    const size_t bytes = std::max<size_t>(1, s->layer_elems * s->nl) * kv_esize(c);
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return set_err(c, DLLM_ENOMEM, "KV cache (%zu bytes): %s", bytes, cudaGetErrorString(e));
    }
    e = cudaMemsetAsync(*p, 0, bytes, c->stream);
    return e == cudaSuccess ? DLLM_OK : set_err(c, DLLM_ECUDA, "KV memset: %s", cudaGetErrorString(e));
  };
  if (!rc) rc = alloc_pool(&s->kpool);
  if (!rc) rc = alloc_pool(&s->vpool);
  if (!rc) rc = dev_alloc(c, &s->page_table, (size_t)s->max_seqs * s->pages_per_seq, "page table");
  if (!rc) {
    std::vector<int> pt((size_t)s->max_seqs * s->pages_per_seq);
    for (size_t i = 0; i < pt.size(); ++i) pt[i] = (int)i;  // sequence-major identity map
    cudaError_t e = cudaMemcpyAsync(s->page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) rc = set_err(c, DLLM_ECUDA, "page table upload: %s", cudaGetErrorString(e));
  }
  if (!rc) rc = dev_alloc(c, &s->h, R * D, "h");
  if (!rc) rc = dev_alloc(c, &s->q, R * QD, "q");
  if (!rc) rc = dev_alloc(c, &s->att, R * QD, "attn");
  if (!rc) rc = dev_alloc(c, &s->mid, R * f.intermediate_size, "mlp");
  if (!rc) rc = dev_alloc(c, &s->part_o, R * f.num_q_heads * kMaxSplitsAlloc * f.head_dim, "attn partials");
  if (!rc) rc = dev_alloc(c, &s->part_ml, R * f.num_q_heads * kMaxSplitsAlloc * 2, "attn partials");
  if (!rc) rc = dev_alloc(c, &s->arrive, 2 * R * f.num_kv_heads, "attn tickets");  // arrivals, finishes
  if (!rc) rc = dev_alloc(c, &s->h2, D, "folded hidden row");
  if (!rc) rc = dev_alloc(c, &s->rows, R, "rows");
  if (!rc) rc = dev_alloc(c, &s->bar, 4 + 2 * D, "barrier + mlp sums");
  if (!rc) rc = dev_alloc(c, &s->best, R, "argmax keys");
  if (!rc) rc = dev_alloc(c, &s->tok, R, "tokens");
  if (!rc) {
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) rc = set_err(c, DLLM_ECUDA, "stage init: %s", cudaGetErrorString(e));
  }
  if (rc) {
    dllm_stage_destroy(s);
    return rc;
  }
  *out = s;
  return DLLM_OK;
}

void dllm_stage_destroy(dllm_stage* s) {
  if (!s) return;
  dllm_ctx* c = s->ctx;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  for (auto& kv : s->W) dllm_buf_free(kv.second);
  dev_free(s->lw_dev);
  dev_free(s->kpool);
  dev_free(s->vpool);
  dev_free(s->page_table);
  dev_free(s->h);
  dev_free(s->q);
  dev_free(s->att);
  dev_free(s->mid);
  dev_free(s->part_o);
  dev_free(s->part_ml);
  dev_free(s->arrive);
  dev_free(s->h2);
  dev_free(s->rows);
  dev_free(s->bar);
  dev_free(s->best);
  dev_free(s->tok);
  dev_free(s->hbuf);
  dev_free(s->tokbuf);
  dev_free(s->trace);
  for (float* p : {s->wq, s->wk, s->wv, s->watt, s->wg, s->wu, s->wpart_o, s->wpart_ml, s->wlogits}) dev_free(p);
  dev_free(s->warrive);
  dev_free(s->wrows);
  dev_free(s->wbest);
  delete s;
  ctx_release(c);
}

int dllm_stage_set_weight(dllm_stage* s, const char* name, dllm_buf* b) {
  if (!s || !name) return DLLM_EINVAL;
  dllm_ctx* c = s->ctx;
  if (!valid_buf(c, b)) return set_err(c, DLLM_EINVAL, "stage.W[%s]: null or foreign buffer", name);
  b->refs += 1;
  auto it = s->W.find(name);
  if (it != s->W.end()) dllm_buf_free(it->second);
  s->W[name] = b;
  s->dirty = true;
  s->version += 1;
  return DLLM_OK;
}

int dllm_stage_reset(dllm_stage* s) {
  if (!s) return DLLM_EINVAL;
  for (auto& t : s->T0) t = 0;
  return DLLM_OK;
}

int dllm_stage_get_t0(const dllm_stage* s, int seq) {
  if (!s || seq < 0 || seq >= s->max_seqs) return -1;
  return s->T0[seq];
}

int dllm_stage_set_t0(dllm_stage* s, int seq, int t0) {
  if (!s) return DLLM_EINVAL;
  if (seq < 0 || seq >= s->max_seqs) return set_err(s->ctx, DLLM_EINVAL, "set_t0: invalid seq %d", seq);
  if (t0 < 0 || t0 > s->max_slots) return set_err(s->ctx, DLLM_ERANGE, "set_t0: T0=%d outside [0,%d]", t0, s->max_slots);
  s->T0[seq] = t0;
  return DLLM_OK;
}

int dllm_stage_forward(dllm_stage* s, const float* hidden, int n, int pos_start, dllm_buf** out) {
  if (!s || !out) return DLLM_EINVAL;
  *out = nullptr;
  dllm_ctx* c = s->ctx;
  if (!hidden || n <= 0) return set_err(c, DLLM_EINVAL, "Stage.forward: invalid n=%d", n);
  if (pos_start < 0) return set_err(c, DLLM_EINVAL, "Stage.forward: invalid posStart=%d", pos_start);
  if ((long long)s->T0[0] + n > s->max_slots)
    return set_err(c, DLLM_ERANGE, "KV cache overflow: T0=%d + n=%d > maxPos=%d", s->T0[0], n, s->max_slots);
  if (int rc = use_device(c)) return rc;
  if (int rc = resolve(s)) return rc;
  const size_t D = c->cfg.hidden_size;
  if (int rc = ensure_hbuf(s, n)) return rc;
  CK(c, cudaMemcpyAsync(s->hbuf, hidden, (size_t)n * D * 4, cudaMemcpyHostToDevice, c->stream));
  if (s->nl > 0) {
    if (int rc = run_rows(s, s->hbuf, n, 0, pos_start, nullptr)) return rc;
  }
  s->T0[0] += n;  // pipeline.js:76
  dllm_buf* o = nullptr;
  if (int rc = new_buf(c, (size_t)n * D, 0, "stage_out", &o, false)) return rc;
  CK(c, cudaMemcpyAsync(o->ptr, s->hbuf, (size_t)n * D * 4, cudaMemcpyDeviceToDevice, c->stream));
  *out = o;
  return DLLM_OK;
}

int dllm_stage_forward_rows(dllm_stage* s, float* h_dev, int m, const int32_t* seq_ids, const int32_t* tokens_in_dev,
                            int32_t* tokens_out_dev) {
  if (!s) return DLLM_EINVAL;
  dllm_ctx* c = s->ctx;
  if (!h_dev || !seq_ids || m <= 0 || m > dllm::kTcMaxRows)
    return set_err(c, DLLM_EINVAL, "forward_rows: need 1..%d rows", dllm::kTcMaxRows);
  std::vector<RowDesc> rd(m);
  for (int i = 0; i < m; ++i) {
    const int q = seq_ids[i];
    if (q < 0 || q >= s->max_seqs) return set_err(c, DLLM_EINVAL, "forward_rows: invalid seq %d", q);
    for (int j = 0; j < i; ++j)
      if (seq_ids[j] == q) return set_err(c, DLLM_EINVAL, "forward_rows: seq %d listed twice", q);
    if (s->T0[q] + 1 > s->max_slots)
      return set_err(c, DLLM_ERANGE, "KV cache overflow: seq %d T0=%d maxPos=%d", q, s->T0[q], s->max_slots);
    rd[i] = RowDesc{q, s->T0[q], s->T0[q], 0};
  }
  if (int rc = use_device(c)) return rc;
  if (int rc = resolve(s)) return rc;
  if (tokens_in_dev && !s->embed) return set_err(c, DLLM_ENOTFOUND, "missing weight model.embed_tokens.weight");
  if (tokens_out_dev)
    if (int rc = need_head(s)) return rc;
  if (s->nl > 0 || tokens_in_dev || tokens_out_dev) {
    if (use_wide(s, m)) {
      if (int rc = run_wide(s, h_dev, m, rd.data(), tokens_in_dev, tokens_out_dev)) return rc;
    } else {
      // passes of <= 8 rows of the stage kernel (rows of distinct sequences are independent)
      const size_t D = c->cfg.hidden_size;
      for (int r0 = 0; r0 < m; r0 += dllm::kMaxRows) {
        const int mm = std::min(dllm::kMaxRows, m - r0);
        CK(c, cudaMemcpyAsync(s->rows, rd.data() + r0, sizeof(RowDesc) * mm, cudaMemcpyHostToDevice, c->stream));
        StageParams P = base_params(s);
        P.m_rows = mm;
        P.h = h_dev + (size_t)r0 * D;
        P.tokens_in = tokens_in_dev ? tokens_in_dev + r0 : nullptr;
        P.lm_head = tokens_out_dev ? s->lm_head : nullptr;
        P.tokens_out = tokens_out_dev ? tokens_out_dev + r0 : nullptr;
        if (int rc = launch(s, P)) return rc;
      }
    }
  }
  for (int i = 0; i < m; ++i) s->T0[seq_ids[i]] += 1;
  return DLLM_OK;
}

int dllm_stage_append_kv(dllm_stage* s, int layer, const dllm_buf* kk, const dllm_buf* vv, int n) {
  if (!s) return DLLM_EINVAL;
  dllm_ctx* c = s->ctx;
  const dllm_config& f = c->cfg;
  const size_t KD = (size_t)f.num_kv_heads * f.head_dim;
  if (layer < s->start || layer >= s->end) return set_err(c, DLLM_EINVAL, "appendKv: layer %d not in stage", layer);
  if (n <= 0) return set_err(c, DLLM_EINVAL, "appendKv: invalid n=%d", n);
  if (int rc = check_f32(c, kk, n * KD, "appendKv kk")) return rc;
  if (int rc = check_f32(c, vv, n * KD, "appendKv vv")) return rc;
  if (s->T0[0] + n > s->max_slots) return set_err(c, DLLM_ERANGE, "appendKv: T0=%d + n=%d > maxPos", s->T0[0], n);
  if (int rc = use_device(c)) return rc;
  const KvLayout kv = stage_kv(s);
  // rows -> slots T0..T0+n-1 (pipeline.js:80-87: byte offset T0 * rowBytes); T0 unchanged
  CK(c, dllm::op_kv_write(kv, layer_pool(s, s->kpool, layer), f.kv_dtype, 0, s->T0[0], n, f.num_kv_heads, f.head_dim,
                          (const float*)kk->ptr, c->stream));
  CK(c, dllm::op_kv_write(kv, layer_pool(s, s->vpool, layer), f.kv_dtype, 0, s->T0[0], n, f.num_kv_heads, f.head_dim,
                          (const float*)vv->ptr, c->stream));
  c->launches += 2;
  return DLLM_OK;
}

int dllm_stage_read_kv(dllm_stage* s, int layer, int which, int seq, int slot_start, int n_slots, float* dst) {
  if (!s) return DLLM_EINVAL;
  dllm_ctx* c = s->ctx;
  const dllm_config& f = c->cfg;
  if (layer < s->start || layer >= s->end) return set_err(c, DLLM_EINVAL, "read_kv: layer %d not in stage", layer);
  if (which != 0 && which != 1) return set_err(c, DLLM_EINVAL, "read_kv: which must be 0 (k) or 1 (v)");
  if (seq < 0 || seq >= s->max_seqs) return set_err(c, DLLM_EINVAL, "read_kv: invalid seq %d", seq);
  if (!dst || n_slots <= 0 || slot_start < 0 || slot_start + n_slots > s->max_slots)
    return set_err(c, DLLM_ERANGE, "read_kv: slots [%d,%d) outside [0,%d)", slot_start, slot_start + n_slots,
                   s->max_slots);
  if (int rc = use_device(c)) return rc;
  const size_t KD = (size_t)f.num_kv_heads * f.head_dim;
  float* tmp = nullptr;
  if (int rc = dev_alloc(c, &tmp, (size_t)n_slots * KD, "kv read")) return rc;
  const KvLayout kv = stage_kv(s);
  cudaError_t e = dllm::op_kv_read(kv, layer_pool(s, which ? s->vpool : s->kpool, layer), f.kv_dtype, seq, slot_start,
                                   n_slots, f.num_kv_heads, f.head_dim, tmp, c->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dst, tmp, (size_t)n_slots * KD * 4, cudaMemcpyDeviceToHost, c->stream);
  int rc = e == cudaSuccess ? sync_check(c, kDefaultTimeoutMs) : set_err(c, DLLM_ECUDA, "read_kv: %s", cudaGetErrorString(e));
  cudaFree(tmp);
  return rc;
}

int dllm_stage_fill_kv_random(dllm_stage* s, int seq, int n_slots, uint64_t seed) {
  if (!s) return DLLM_EINVAL;
  dllm_ctx* c = s->ctx;
  const dllm_config& f = c->cfg;
  if (seq < 0 || seq >= s->max_seqs) return set_err(c, DLLM_EINVAL, "fill_kv_random: invalid seq %d", seq);
  if (n_slots < 0 || n_slots > s->max_slots)
    return set_err(c, DLLM_ERANGE, "fill_kv_random: %d slots > maxPos %d", n_slots, s->max_slots);
  if (int rc = use_device(c)) return rc;
  const KvLayout kv = stage_kv(s);
  for (int L = s->start; L < s->end && n_slots > 0; ++L) {
    CK(c, dllm::op_kv_fill_random(kv, layer_pool(s, s->kpool, L), layer_pool(s, s->vpool, L), f.kv_dtype, seq, n_slots,
                                  f.num_kv_heads, f.head_dim, seed * 1000003ull + (uint64_t)L * 7919ull + (uint64_t)seq,
                                  c->stream));
    c->launches += 1;
  }
  s->T0[seq] = n_slots;
  return DLLM_OK;
}

int dllm_stage_set_page_table(dllm_stage* s, int seq, const int32_t* pages, int n_pages) {
  if (!s) return DLLM_EINVAL;
  dllm_ctx* c = s->ctx;
  if (seq < 0 || seq >= s->max_seqs) return set_err(c, DLLM_EINVAL, "set_page_table: invalid seq %d", seq);
  if (!pages || n_pages != s->pages_per_seq)
    return set_err(c, DLLM_EINVAL, "set_page_table: need exactly %d pages", s->pages_per_seq);
  const int total = s->max_seqs * s->pages_per_seq;
  std::vector<char> seen(total, 0);
  for (int i = 0; i < n_pages; ++i) {
    if (pages[i] < 0 || pages[i] >= total || seen[pages[i]])
      return set_err(c, DLLM_EINVAL, "set_page_table: page %d invalid or repeated", pages[i]);
    seen[pages[i]] = 1;
  }
  if (int rc = use_device(c)) return rc;
  CK(c, cudaMemcpyAsync(s->page_table + (size_t)seq * s->pages_per_seq, pages, (size_t)n_pages * 4,
                        cudaMemcpyHostToDevice, c->stream));
  CK(c, cudaStreamSynchronize(c->stream));
  return DLLM_OK;
}

int dllm_stage_pages_per_seq(const dllm_stage* s) { return s ? s->pages_per_seq : -1; }

int dllm_stage_read_workspace(dllm_stage* s, int which, int rows, float* dst) {
  if (!s) return DLLM_EINVAL;
  dllm_ctx* c = s->ctx;
  const dllm_config& f = c->cfg;
  if (!dst || rows < 1 || rows > dllm::kMaxRows)
    return set_err(c, DLLM_EINVAL, "read_workspace: need 1..%d rows", dllm::kMaxRows);
  const float* src = nullptr;
  size_t width = 0;
  switch (which) {
    case 0: src = s->q; width = (size_t)f.num_q_heads * f.head_dim; break;
    case 1: src = s->att; width = (size_t)f.num_q_heads * f.head_dim; break;
    case 2: src = s->mid; width = (size_t)f.intermediate_size; break;
    default: return set_err(c, DLLM_EINVAL, "read_workspace: which must be 0 (q), 1 (attention) or 2 (mlp)");
  }
  if (int rc = use_device(c)) return rc;
  CK(c, cudaMemcpyAsync(dst, src, (size_t)rows * width * 4, cudaMemcpyDeviceToHost, c->stream));
  return sync_check(c, kDefaultTimeoutMs);
}

int dllm_stage_set_trace(dllm_stage* s, int cap) {
  if (!s) return DLLM_EINVAL;
  dllm_ctx* c = s->ctx;
  if (cap < 0) return set_err(c, DLLM_EINVAL, "set_trace: negative capacity");
  if (int rc = use_device(c)) return rc;
  CK(c, cudaStreamSynchronize(c->stream));
  dev_free(s->trace);
  s->trace = nullptr;
  s->trace_cap = 0;
  if (cap > 0) {
    if (int rc = dev_alloc(c, &s->trace, (size_t)cap, "trace")) return rc;
    s->trace_cap = cap;
  }
  s->version += 1;
  return DLLM_OK;
}

int dllm_stage_read_trace(dllm_stage* s, uint64_t* out, int cap) {
  if (!s || !out) return DLLM_EINVAL;
  dllm_ctx* c = s->ctx;
  if (cap <= 0 || cap > s->trace_cap) return set_err(c, DLLM_EINVAL, "read_trace: %d of %d entries", cap, s->trace_cap);
  if (int rc = use_device(c)) return rc;
  CK(c, cudaMemcpyAsync(out, s->trace, (size_t)cap * 8, cudaMemcpyDeviceToHost, c->stream));
  return sync_check(c, kDefaultTimeoutMs);
}

// ---- LeaderPipeline (pipeline.js:91-282) --------------------------------------------------
void dllm_leader_destroy(dllm_leader* ld);

int dllm_leader_create(dllm_ctx* c, int start, int end, dllm_leader** out) {
  if (!c || !out) return DLLM_EINVAL;
  *out = nullptr;
  auto* ld = new dllm_leader();
  ld->ctx = c;
  ctx_retain(c);
  int rc = dllm_stage_create(c, start, end, &ld->st);
  if (!rc) rc = use_device(c);
  if (!rc) rc = dev_alloc(c, &ld->tok_dev, dllm::kMaxRows, "tokens");
  if (!rc) rc = dev_alloc(c, &ld->dec_rows, dllm::kMaxRows, "decode rows");
  if (!rc) rc = dev_alloc(c, &ld->step_count, 1, "step counter");
  if (!rc) {
    ld->hist_cap = c->cfg.max_pos + 1;
    rc = dev_alloc(c, &ld->hist, (size_t)ld->hist_cap, "token history");
  }
  if (!rc) rc = dev_alloc(c, &ld->last_logits, (size_t)c->cfg.vocab_size, "logits");
  if (!rc && cudaMallocHost(&ld->pin_in, sizeof(int32_t) * dllm::kMaxRows) != cudaSuccess)
    rc = set_err(c, DLLM_ENOMEM, "pinned token buffer");
  if (!rc && cudaMallocHost(&ld->pin_out, sizeof(int32_t) * dllm::kMaxRows) != cudaSuccess)
    rc = set_err(c, DLLM_ENOMEM, "pinned token buffer");
  if (!rc && cudaStreamSynchronize(c->stream) != cudaSuccess) rc = set_err(c, DLLM_ECUDA, "leader init");
  if (rc) {
    dllm_leader_destroy(ld);
    return rc;
  }
  *out = ld;
  return DLLM_OK;
}

static void drop_graphs(dllm_leader* ld) {
  if (ld->g_e2e) cudaGraphExecDestroy(ld->g_e2e);
  if (ld->g_dev) cudaGraphExecDestroy(ld->g_dev);
  ld->g_e2e = ld->g_dev = nullptr;
}

void dllm_leader_destroy(dllm_leader* ld) {
  if (!ld) return;
  cudaSetDevice(ld->ctx->device);
  drop_graphs(ld);
  if (ld->st) dllm_stage_destroy(ld->st);
  dev_free(ld->tok_dev);
  dev_free(ld->dec_rows);
  dev_free(ld->step_count);
  dev_free(ld->hist);
  dev_free(ld->last_logits);
  dev_free(ld->logits_ring);
  if (ld->pin_in) cudaFreeHost(ld->pin_in);
  if (ld->pin_out) cudaFreeHost(ld->pin_out);
  dllm_ctx* c = ld->ctx;
  delete ld;
  ctx_release(c);
}

dllm_stage* dllm_leader_stage(dllm_leader* ld) { return ld ? ld->st : nullptr; }

int dllm_leader_set_weights(dllm_leader* ld, dllm_buf* embed, dllm_buf* norm, dllm_buf* lm_head) {
  if (!ld) return DLLM_EINVAL;
  if (embed)
    if (int rc = dllm_stage_set_weight(ld->st, "model.embed_tokens.weight", embed)) return rc;
  if (norm)
    if (int rc = dllm_stage_set_weight(ld->st, "model.norm.weight", norm)) return rc;
  if (lm_head)
    if (int rc = dllm_stage_set_weight(ld->st, "lm_head.weight", lm_head)) return rc;
  drop_graphs(ld);
  return DLLM_OK;
}

int dllm_leader_embed_tokens(dllm_leader* ld, const int32_t* tokens, int n, float* out) {
  if (!ld) return DLLM_EINVAL;
  dllm_stage* s = ld->st;
  dllm_ctx* c = ld->ctx;
  if (!tokens || !out || n <= 0) return set_err(c, DLLM_EINVAL, "embedTokens: invalid n=%d", n);
  if (int rc = use_device(c)) return rc;
  if (int rc = resolve(s)) return rc;
  if (!s->embed) return set_err(c, DLLM_ENOTFOUND, "missing weight model.embed_tokens.weight");
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= c->cfg.vocab_size)
      return set_err(c, DLLM_EINVAL, "embedTokens: token %d out of range", tokens[i]);
  if (int rc = ensure_hbuf(s, n)) return rc;
  if (int rc = ensure_tokbuf(s, n)) return rc;
  const int D = c->cfg.hidden_size;
  CK(c, cudaMemcpyAsync(s->tokbuf, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream));
  CK(c, dllm::op_embed(s->embed, s->tokbuf, s->hbuf, n, D, c->cfg.vocab_size, c->err_dev, c->stream));
  c->launches += 1;
  CK(c, cudaMemcpyAsync(out, s->hbuf, (size_t)n * D * 4, cudaMemcpyDeviceToHost, c->stream));
  return sync_check(c, kDefaultTimeoutMs);
}

int dllm_leader_sample_last(dllm_leader* ld, const float* hidden_row, int32_t* token, float* logits_out) {
  if (!ld) return DLLM_EINVAL;
  dllm_stage* s = ld->st;
  dllm_ctx* c = ld->ctx;
  if (!hidden_row || !token) return set_err(c, DLLM_EINVAL, "sampleLast: null argument");
  if (int rc = use_device(c)) return rc;
  if (int rc = resolve(s)) return rc;
  if (int rc = need_head(s)) return rc;
  const int D = c->cfg.hidden_size;
  CK(c, cudaMemcpyAsync(s->h, hidden_row, (size_t)D * 4, cudaMemcpyHostToDevice, c->stream));
  if (int rc = run_head(s, s->h, ld->tok_dev, ld->last_logits, 1, nullptr, nullptr, 0)) return rc;
  ld->last_in_ring = false;
  ld->last_index = 0;
  CK(c, cudaMemcpyAsync(ld->pin_out, ld->tok_dev, 4, cudaMemcpyDeviceToHost, c->stream));
  if (logits_out)
    CK(c, cudaMemcpyAsync(logits_out, ld->last_logits, (size_t)c->cfg.vocab_size * 4, cudaMemcpyDeviceToHost,
                          c->stream));
  if (int rc = sync_check(c, kDefaultTimeoutMs)) return rc;
  *token = ld->pin_out[0];
  return DLLM_OK;
}

int dllm_leader_forward(dllm_leader* ld, const float* hidden, int n, int pos_start, float* last_row) {
  if (!ld) return DLLM_EINVAL;
  dllm_ctx* c = ld->ctx;
  if (!last_row) return set_err(c, DLLM_EINVAL, "forward: null output");
  dllm_buf* h = nullptr;
  if (int rc = dllm_stage_forward(ld->st, hidden, n, pos_start, &h)) return rc;
  const size_t D = c->cfg.hidden_size;
  cudaError_t e = cudaMemcpyAsync(last_row, (const float*)h->ptr + (size_t)(n - 1) * D, D * 4, cudaMemcpyDeviceToHost,
                                  c->stream);
  int rc = e == cudaSuccess ? sync_check(c, kDefaultTimeoutMs) : set_err(c, DLLM_ECUDA, "forward readback");
  dllm_buf_free(h);
  return rc;
}

int dllm_leader_set_keep_logits(dllm_leader* ld, int keep) {
  if (!ld) return DLLM_EINVAL;
  dllm_ctx* c = ld->ctx;
  if (keep < 0) return set_err(c, DLLM_EINVAL, "keep_logits: negative capacity");
  if (int rc = use_device(c)) return rc;
  CK(c, cudaStreamSynchronize(c->stream));
  dev_free(ld->logits_ring);
  ld->logits_ring = nullptr;
  ld->logits_cap = 0;
  if (keep > 0) {
    if (int rc = dev_alloc(c, &ld->logits_ring, (size_t)keep * c->cfg.vocab_size, "logits ring")) return rc;
    ld->logits_cap = keep;
  }
  ld->last_index = -1;
  drop_graphs(ld);
  return DLLM_OK;
}

// Capture one decode step (embed -> layers -> head, rows advanced on device) as a
// CUDA graph; the e2e variant also copies the token in from and out to pinned
// host memory (the per-token round trip of pipeline.js:262-266).
static int build_graph(dllm_leader* ld, bool e2e, cudaGraphExec_t* out) {
  dllm_ctx* c = ld->ctx;
  dllm_stage* s = ld->st;
  StageParams P = base_params(s);
  P.m_rows = 1;
  P.rows = ld->dec_rows;
  P.tokens_in = ld->tok_dev;
  P.tokens_out = ld->tok_dev;
  P.lm_head = s->lm_head;
  P.step_count = ld->step_count;
  P.history = ld->hist;
  P.hist_cap = ld->hist_cap;
  P.logits = ld->logits_ring;
  P.logits_cap = ld->logits_cap;
  P.advance_rows = 1;
  cudaGraph_t g = nullptr;
  CK(c, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  if (e2e) cudaMemcpyAsync(ld->tok_dev, ld->pin_in, 4, cudaMemcpyHostToDevice, c->stream);
  int ms = c->sms / P.KVH;
  P.max_splits = std::max(1, std::min(ms, kMaxSplitsAlloc));
  cudaError_t le = dllm::launch_stage(P, c->cfg.kv_dtype, c->sms, c->stream);
  if (e2e) cudaMemcpyAsync(ld->pin_out, ld->tok_dev, 4, cudaMemcpyDeviceToHost, c->stream);
  cudaError_t ee = cudaStreamEndCapture(c->stream, &g);
  if (le != cudaSuccess || ee != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return set_err(c, DLLM_ECUDA, "decode graph capture: %s / %s", cudaGetErrorString(le), cudaGetErrorString(ee));
  }
  cudaError_t ie = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return set_err(c, DLLM_ECUDA, "decode graph instantiate: %s", cudaGetErrorString(ie));
  return DLLM_OK;
}

int dllm_leader_generate(dllm_leader* ld, const int32_t* tokens, int n_tokens, int max_new, int32_t* out, int* n_out) {
  if (!ld) return DLLM_EINVAL;
  dllm_ctx* c = ld->ctx;
  dllm_stage* s = ld->st;
  const dllm_config& f = c->cfg;
  if (n_out) *n_out = 0;
  if (!tokens || n_tokens <= 0 || !out || !n_out || max_new < 1)
    return set_err(c, DLLM_EINVAL, "generate: need tokens, max_new >= 1 and output buffers");
  for (int i = 0; i < n_tokens; ++i)
    if (tokens[i] < 0 || tokens[i] >= f.vocab_size) return set_err(c, DLLM_EINVAL, "generate: token %d out of range", tokens[i]);
  if (s->start != 0 || s->end != f.num_layers)
    return set_err(c, DLLM_EINVAL, "generate: the leader's stage must own every layer (single node)");
  if ((long long)s->T0[0] + n_tokens + (max_new - 1) > s->max_slots)
    return set_err(c, DLLM_ERANGE, "generate: T0=%d + %d prompt + %d new > maxPos=%d", s->T0[0], n_tokens, max_new - 1,
                   s->max_slots);
  if (int rc = use_device(c)) return rc;
  if (int rc = resolve(s)) return rc;
  if (!s->embed) return set_err(c, DLLM_ENOTFOUND, "missing weight model.embed_tokens.weight");
  if (int rc = need_head(s)) return rc;
  if (ld->graph_version != s->version) drop_graphs(ld);
  if (!ld->g_e2e)
    if (int rc = build_graph(ld, true, &ld->g_e2e)) return rc;
  ld->graph_version = s->version;
  const int D = f.hidden_size;
  // ---- prefill: forward(embedTokens(tokens), len, 0) then sampleLast (pipeline.js:259-261)
  if (int rc = ensure_hbuf(s, n_tokens)) return rc;
  if (int rc = ensure_tokbuf(s, n_tokens)) return rc;
  CK(c, cudaMemsetAsync(ld->step_count, 0, sizeof(int), c->stream));
  CK(c, cudaMemcpyAsync(s->tokbuf, tokens, (size_t)n_tokens * 4, cudaMemcpyHostToDevice, c->stream));
  if (s->nl > 0) {
    if (int rc = run_rows(s, s->hbuf, n_tokens, 0, 0, s->tokbuf)) return rc;
  }
  s->T0[0] += n_tokens;
  if (int rc = run_head(s, s->hbuf + (size_t)(n_tokens - 1) * D, ld->tok_dev, ld->logits_ring, ld->logits_cap,
                        ld->step_count, ld->hist, ld->hist_cap))
    return rc;
  CK(c, cudaMemcpyAsync(ld->pin_out, ld->tok_dev, 4, cudaMemcpyDeviceToHost, c->stream));
  if (int rc = sync_check(c, kDefaultTimeoutMs)) return rc;
  int next = ld->pin_out[0];
  int count = 0;
  out[count++] = next;
  // ---- decode loop (pipeline.js:262-267): position of step i is len + i - 1
  RowDesc rd{0, n_tokens, s->T0[0], 0};
  CK(c, cudaMemcpyAsync(ld->dec_rows, &rd, sizeof(rd), cudaMemcpyHostToDevice, c->stream));
  for (int i = 1; i < max_new; ++i) {
    if (next == f.eos_token_id) break;
    ld->pin_in[0] = next;
    CK(c, cudaGraphLaunch(ld->g_e2e, c->stream));
    c->launches += 1;
    if (int rc = sync_check(c, kDefaultTimeoutMs)) return rc;
    s->T0[0] += 1;
    next = ld->pin_out[0];
    out[count++] = next;
  }
  ld->last_in_ring = ld->logits_cap > 0;
  ld->last_index = ld->logits_cap > 0 ? std::min(count, ld->logits_cap) - 1 : -1;
  *n_out = count;
  return DLLM_OK;
}

int dllm_leader_decode_enqueue(dllm_leader* ld, int32_t first_token, int steps) {
  if (!ld) return DLLM_EINVAL;
  dllm_ctx* c = ld->ctx;
  dllm_stage* s = ld->st;
  const dllm_config& f = c->cfg;
  if (steps <= 0) return set_err(c, DLLM_EINVAL, "decode: invalid steps=%d", steps);
  if (first_token < 0 || first_token >= f.vocab_size) return set_err(c, DLLM_EINVAL, "decode: token out of range");
  if (s->start != 0 || s->end != f.num_layers)
    return set_err(c, DLLM_EINVAL, "decode: the leader's stage must own every layer (single node)");
  if ((long long)s->T0[0] + steps > s->max_slots || steps > ld->hist_cap)
    return set_err(c, DLLM_ERANGE, "decode: T0=%d + %d steps > maxPos=%d", s->T0[0], steps, s->max_slots);
  if (int rc = use_device(c)) return rc;
  if (int rc = resolve(s)) return rc;
  if (!s->embed) return set_err(c, DLLM_ENOTFOUND, "missing weight model.embed_tokens.weight");
  if (int rc = need_head(s)) return rc;
  if (ld->graph_version != s->version) drop_graphs(ld);
  if (!ld->g_dev)
    if (int rc = build_graph(ld, false, &ld->g_dev)) return rc;
  ld->graph_version = s->version;
  RowDesc rd{0, s->T0[0], s->T0[0], 0};
  CK(c, cudaMemcpyAsync(ld->dec_rows, &rd, sizeof(rd), cudaMemcpyHostToDevice, c->stream));
  CK(c, cudaMemcpyAsync(ld->tok_dev, &first_token, 4, cudaMemcpyHostToDevice, c->stream));
  CK(c, cudaMemsetAsync(ld->step_count, 0, sizeof(int), c->stream));
  for (int i = 0; i < steps; ++i) {
    CK(c, cudaGraphLaunch(ld->g_dev, c->stream));
    c->launches += 1;
  }
  s->T0[0] += steps;
  ld->pending_steps = steps;
  ld->last_in_ring = ld->logits_cap > 0;
  ld->last_index = ld->logits_cap > 0 ? std::min(steps, ld->logits_cap) - 1 : -1;
  return DLLM_OK;
}

int dllm_leader_read_tokens(dllm_leader* ld, int32_t* out, int steps) {
  if (!ld) return DLLM_EINVAL;
  dllm_ctx* c = ld->ctx;
  if (!out || steps <= 0 || steps > ld->pending_steps)
    return set_err(c, DLLM_EINVAL, "read_tokens: %d steps requested, %d decoded", steps, ld->pending_steps);
  if (int rc = use_device(c)) return rc;
  CK(c, cudaMemcpyAsync(out, ld->hist, (size_t)steps * 4, cudaMemcpyDeviceToHost, c->stream));
  return sync_check(c, std::max(kDefaultTimeoutMs, ld->pending_steps * 100));
}

int dllm_leader_decode(dllm_leader* ld, int32_t first_token, int steps, int32_t* out) {
  if (!ld) return DLLM_EINVAL;
  if (!out) return set_err(ld->ctx, DLLM_EINVAL, "decode: null output");
  if (int rc = dllm_leader_decode_enqueue(ld, first_token, steps)) return rc;
  return dllm_leader_read_tokens(ld, out, steps);
}

int dllm_leader_last_logits(dllm_leader* ld, float* out) {
  if (!ld || !out) return DLLM_EINVAL;
  dllm_ctx* c = ld->ctx;
  if (ld->last_index < 0) return set_err(c, DLLM_EINVAL, "no logits kept (enable keep_logits or call sampleLast)");
  if (int rc = use_device(c)) return rc;
  const float* src = ld->last_in_ring ? ld->logits_ring + (size_t)ld->last_index * c->cfg.vocab_size : ld->last_logits;
  CK(c, cudaMemcpyAsync(out, src, (size_t)c->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, c->stream));
  return sync_check(c, kDefaultTimeoutMs);
}

int dllm_leader_read_logits(dllm_leader* ld, int index, float* out) {
  if (!ld || !out) return DLLM_EINVAL;
  dllm_ctx* c = ld->ctx;
  if (index < 0 || index >= ld->logits_cap)
    return set_err(c, DLLM_EINVAL, "read_logits: index %d outside the kept %d steps", index, ld->logits_cap);
  if (int rc = use_device(c)) return rc;
  CK(c, cudaMemcpyAsync(out, ld->logits_ring + (size_t)index * c->cfg.vocab_size, (size_t)c->cfg.vocab_size * 4,
                        cudaMemcpyDeviceToHost, c->stream));
  return sync_check(c, kDefaultTimeoutMs);
}

// ---- multi-GPU pipeline: the layer-range stages of pipeline.js on one node ----------------
// One process (or thread) per GPU, each holding one Stage. Micro-batch b = the
// sequences [b * micro, (b + 1) * micro) circulates the ring rank 0 -> 1 -> ... ->
// W-1 -> 0: the first stage embeds its tokens, every stage runs its layers, the
// last stage samples the next tokens, which go back to the first stage. The hop
// (pipeline.js:226-253; WebRTC frames in the reference) is fused into the stage
// kernel: the pass ends by storing its output rows (or tokens) into the next
// GPU's receive buffer over NVLink and releasing a per-micro-batch flag there;
// the next stage's pass starts by waiting (bounded) on that flag. Receive
// buffers are shared once through CUDA IPC handles the host exchanges. Flow
// control comes from the ring itself: a stage writes micro-batch b again only
// after b has gone around the ring, i.e. after the next stage finished with it.
struct dllm_pipeline {
  dllm_stage* st = nullptr;
  dllm_ctx* ctx = nullptr;
  int rank = 0, world = 1, n_micro = 1, micro = 1;
  // receive buffer of this rank (one allocation, exported): h [B][m][D] f32,
  // tokens [B][m] i32, flags [B] u32
  char* rx = nullptr;
  size_t rx_bytes = 0, off_tok = 0, off_flag = 0;
  char* peer_rx = nullptr;  // the next rank's receive buffer (IPC mapping), or rx itself for one rank
  float* h0 = nullptr;      // first stage: [B][m][D] work rows
  int32_t* tok_out = nullptr;  // last stage: [B][m] sampled tokens
  RowDesc* rows = nullptr;  // [B][m] device row descriptors, advanced on the device
  int32_t* hist = nullptr;  // last stage: [hist_cap][B * m] tokens of the latest run
  int hist_cap = 0, hist_steps = 0;
  std::vector<unsigned int> passes;  // passes run per micro-batch
  bool connected = false;
  bool host_tokens = false;  // the first stage takes tokens from the host, not from the last stage
};

namespace {
float* rx_h(const dllm_pipeline* pl, char* base, int b) {
  return reinterpret_cast<float*>(base) + (size_t)b * pl->micro * pl->ctx->cfg.hidden_size;
}
int32_t* rx_tok(const dllm_pipeline* pl, char* base, int b) {
  return reinterpret_cast<int32_t*>(base + pl->off_tok) + (size_t)b * pl->micro;
}
unsigned int* rx_flag(const dllm_pipeline* pl, char* base, int b) {
  return reinterpret_cast<unsigned int*>(base + pl->off_flag) + b;
}
}  // namespace

void dllm_pipeline_destroy(dllm_pipeline* pl) {
  if (!pl) return;
  dllm_ctx* c = pl->ctx;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  if (pl->peer_rx && pl->peer_rx != pl->rx) cudaIpcCloseMemHandle(pl->peer_rx);
  dev_free(pl->rx);
  dev_free(pl->h0);
  dev_free(pl->tok_out);
  dev_free(pl->rows);
  dev_free(pl->hist);
  delete pl;
  ctx_release(c);
}

int dllm_pipeline_create(dllm_stage* s, int rank, int world, int n_micro, int micro, dllm_pipeline** out) {
  if (!s || !out) return DLLM_EINVAL;
  *out = nullptr;
  dllm_ctx* c = s->ctx;
  const dllm_config& f = c->cfg;
  if (world < 1 || rank < 0 || rank >= world) return set_err(c, DLLM_EINVAL, "pipeline: rank %d of %d", rank, world);
  if (n_micro < 1 || micro < 1 || micro > dllm::kMaxRows)
    return set_err(c, DLLM_EINVAL, "pipeline: need n_micro >= 1 and 1..%d sequences per micro-batch", dllm::kMaxRows);
  if ((long long)n_micro * micro > s->max_seqs)
    return set_err(c, DLLM_EINVAL, "pipeline: %d x %d sequences > the stage's max_seqs %d", n_micro, micro,
                   s->max_seqs);
  if (int rc = use_device(c)) return rc;
  if (int rc = resolve(s)) return rc;
  if (rank == 0 && !s->embed) return set_err(c, DLLM_ENOTFOUND, "pipeline: the first stage needs model.embed_tokens.weight");
  if (rank == world - 1)
    if (int rc = need_head(s)) return rc;
  auto* pl = new dllm_pipeline();
  pl->st = s;
  pl->ctx = c;
  ctx_retain(c);
  pl->rank = rank;
  pl->world = world;
  pl->n_micro = n_micro;
  pl->micro = micro;
  pl->passes.assign(n_micro, 0u);
  const size_t D = f.hidden_size, B = n_micro, m = micro;
  pl->off_tok = (B * m * D * 4 + 255) / 256 * 256;
  pl->off_flag = pl->off_tok + (B * m * 4 + 255) / 256 * 256;
  pl->rx_bytes = pl->off_flag + 256;
  int rc = dev_alloc(c, &pl->rx, pl->rx_bytes, "pipeline receive buffer");
  if (!rc && rank == 0) rc = dev_alloc(c, &pl->h0, B * m * D, "pipeline rows");
  if (!rc && rank == world - 1) rc = dev_alloc(c, &pl->tok_out, B * m, "pipeline tokens");
  if (!rc) rc = dev_alloc(c, &pl->rows, B * m, "pipeline rows");
  if (!rc) {
    std::vector<RowDesc> rd(B * m);
    for (size_t i = 0; i < B * m; ++i) rd[i] = RowDesc{(int)i, s->T0[i], s->T0[i], 0};
    cudaError_t e = cudaMemcpyAsync(pl->rows, rd.data(), rd.size() * sizeof(RowDesc), cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) rc = set_err(c, DLLM_ECUDA, "pipeline init: %s", cudaGetErrorString(e));
  }
  if (rc) {
    dllm_pipeline_destroy(pl);
    return rc;
  }
  if (world == 1) {
    pl->peer_rx = pl->rx;
    pl->connected = true;
  }
  *out = pl;
  return DLLM_OK;
}

int dllm_pipeline_handle(const dllm_pipeline* pl, uint8_t* out) {
  if (!pl || !out) return DLLM_EINVAL;
  dllm_ctx* c = pl->ctx;
  if (int rc = use_device(c)) return rc;
  cudaIpcMemHandle_t h;
  CK(c, cudaIpcGetMemHandle(&h, pl->rx));
  static_assert(sizeof(cudaIpcMemHandle_t) == DLLM_PIPELINE_HANDLE_BYTES, "IPC handle size");
  std::memcpy(out, &h, sizeof(h));
  return DLLM_OK;
}

int dllm_pipeline_connect(dllm_pipeline* pl, const uint8_t* next_handle) {
  if (!pl) return DLLM_EINVAL;
  dllm_ctx* c = pl->ctx;
  if (pl->world == 1) return DLLM_OK;
  if (!next_handle) return set_err(c, DLLM_EINVAL, "pipeline_connect: null handle");
  if (pl->connected) return set_err(c, DLLM_EINVAL, "pipeline_connect: already connected");
  if (int rc = use_device(c)) return rc;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, next_handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_err(c, DLLM_ECUDA, "pipeline_connect: %s", cudaGetErrorString(e));
  }
  pl->peer_rx = static_cast<char*>(p);
  pl->connected = true;
  return DLLM_OK;
}

int dllm_pipeline_set_tokens(dllm_pipeline* pl, const int32_t* tokens, int n) {
  if (!pl) return DLLM_EINVAL;
  dllm_ctx* c = pl->ctx;
  if (pl->rank != 0) return set_err(c, DLLM_EINVAL, "pipeline_set_tokens: only the first stage takes tokens");
  if (!tokens || n != pl->n_micro * pl->micro)
    return set_err(c, DLLM_EINVAL, "pipeline_set_tokens: need %d tokens", pl->n_micro * pl->micro);
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= c->cfg.vocab_size)
      return set_err(c, DLLM_EINVAL, "pipeline_set_tokens: token %d out of range", tokens[i]);
  if (int rc = use_device(c)) return rc;
  CK(c, cudaMemcpyAsync(rx_tok(pl, pl->rx, 0), tokens, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream));
  return sync_check(c, kDefaultTimeoutMs);
}

namespace {
// One pass of micro-batch b on this rank (enqueued). `hist_row`: where the last
// stage keeps the sampled tokens (device), or null.
int pipeline_pass(dllm_pipeline* pl, int b, int32_t* hist_row) {
  dllm_ctx* c = pl->ctx;
  dllm_stage* s = pl->st;
  const int m = pl->micro, D = c->cfg.hidden_size;
  const bool first = pl->rank == 0, last = pl->rank == pl->world - 1;
  for (int i = 0; i < m; ++i)
    if (s->T0[b * m + i] + 1 > s->max_slots)
      return set_err(c, DLLM_ERANGE, "KV cache overflow: seq %d T0=%d maxPos=%d", b * m + i, s->T0[b * m + i],
                     s->max_slots);
  const unsigned int k = pl->passes[b];  // passes of b so far on this rank
  StageParams P = base_params(s);
  P.m_rows = m;
  P.rows = pl->rows + (size_t)b * m;
  P.advance_rows = 1;
  if (first) {
    P.h = pl->h0 + (size_t)b * m * D;
    P.tokens_in = rx_tok(pl, pl->rx, b);
    if (k > 0 && pl->world > 1 && !pl->host_tokens) {  // the previous round's tokens, from the last stage
      P.in_flag = rx_flag(pl, pl->rx, b);
      P.in_expect = k;
    }
  } else {
    P.h = rx_h(pl, pl->rx, b);
    P.in_flag = rx_flag(pl, pl->rx, b);
    P.in_expect = k + 1;
  }
  if (last) {
    P.lm_head = s->lm_head;
    P.tokens_out = pl->world == 1 ? rx_tok(pl, pl->rx, b) : pl->tok_out + (size_t)b * m;
    if (pl->world > 1 && !pl->host_tokens) {
      P.out_tok = rx_tok(pl, pl->peer_rx, b);
      P.out_flag = rx_flag(pl, pl->peer_rx, b);
      P.out_value = k + 1;
    }
  } else {
    P.lm_head = nullptr;
    P.out_h = rx_h(pl, pl->peer_rx, b);
    P.out_flag = rx_flag(pl, pl->peer_rx, b);
    P.out_value = k + 1;
  }
  if (int rc = launch(s, P)) return rc;
  if (last && hist_row)
    CK(c, cudaMemcpyAsync(hist_row, P.tokens_out, (size_t)m * 4, cudaMemcpyDeviceToDevice, c->stream));
  pl->passes[b] = k + 1;
  for (int i = 0; i < m; ++i) s->T0[b * m + i] += 1;
  return DLLM_OK;
}

int pipeline_ready(dllm_pipeline* pl) {
  dllm_ctx* c = pl->ctx;
  if (!pl->connected) return set_err(c, DLLM_EINVAL, "pipeline: not connected to the next stage");
  if (int rc = use_device(c)) return rc;
  return resolve(pl->st);
}
}  // namespace

int dllm_pipeline_run(dllm_pipeline* pl, int steps) {
  if (!pl) return DLLM_EINVAL;
  dllm_ctx* c = pl->ctx;
  if (steps < 1) return set_err(c, DLLM_EINVAL, "pipeline_run: invalid steps=%d", steps);
  if (int rc = pipeline_ready(pl)) return rc;
  const int B = pl->n_micro, m = pl->micro;
  const bool last = pl->rank == pl->world - 1;
  if (last && steps > pl->hist_cap) {
    CK(c, cudaStreamSynchronize(c->stream));
    dev_free(pl->hist);
    pl->hist = nullptr;
    pl->hist_cap = 0;
    if (int rc = dev_alloc(c, &pl->hist, (size_t)steps * B * m, "pipeline token history")) return rc;
    pl->hist_cap = steps;
  }
  for (int step = 0; step < steps; ++step)
    for (int b = 0; b < B; ++b)
      if (int rc = pipeline_pass(pl, b, last ? pl->hist + ((size_t)step * B + b) * m : nullptr)) return rc;
  pl->hist_steps = last ? steps : 0;
  return DLLM_OK;
}

int dllm_pipeline_set_host_tokens(dllm_pipeline* pl, int on) {
  if (!pl) return DLLM_EINVAL;
  if (int rc = use_device(pl->ctx)) return rc;
  CK(pl->ctx, cudaStreamSynchronize(pl->ctx->stream));
  pl->host_tokens = on != 0;
  return DLLM_OK;
}

int dllm_pipeline_run_micro(dllm_pipeline* pl, int b, const int32_t* tokens, int32_t* tokens_out) {
  if (!pl) return DLLM_EINVAL;
  dllm_ctx* c = pl->ctx;
  const int m = pl->micro;
  if (b < 0 || b >= pl->n_micro) return set_err(c, DLLM_EINVAL, "pipeline_run_micro: invalid micro-batch %d", b);
  const bool first = pl->rank == 0, last = pl->rank == pl->world - 1;
  if (first && pl->host_tokens && !tokens)
    return set_err(c, DLLM_EINVAL, "pipeline_run_micro: the first stage needs the micro-batch's tokens");
  if (last && !tokens_out) return set_err(c, DLLM_EINVAL, "pipeline_run_micro: the last stage returns tokens");
  if (int rc = pipeline_ready(pl)) return rc;
  if (first && tokens) {
    for (int i = 0; i < m; ++i)
      if (tokens[i] < 0 || tokens[i] >= c->cfg.vocab_size)
        return set_err(c, DLLM_EINVAL, "pipeline_run_micro: token %d out of range", tokens[i]);
    CK(c, cudaMemcpyAsync(rx_tok(pl, pl->rx, b), tokens, (size_t)m * 4, cudaMemcpyHostToDevice, c->stream));
  }
  if (int rc = pipeline_pass(pl, b, nullptr)) return rc;
  if (!last) return DLLM_OK;
  const int32_t* src = pl->world == 1 ? rx_tok(pl, pl->rx, b) : pl->tok_out + (size_t)b * m;
  CK(c, cudaMemcpyAsync(tokens_out, src, (size_t)m * 4, cudaMemcpyDeviceToHost, c->stream));
  return sync_check(c, kDefaultTimeoutMs);
}

int dllm_pipeline_read_tokens(dllm_pipeline* pl, int32_t* out, int steps) {
  if (!pl) return DLLM_EINVAL;
  dllm_ctx* c = pl->ctx;
  if (pl->rank != pl->world - 1) return set_err(c, DLLM_EINVAL, "pipeline_read_tokens: only the last stage samples");
  if (!out || steps < 1 || steps > pl->hist_steps)
    return set_err(c, DLLM_EINVAL, "pipeline_read_tokens: %d steps requested, %d run", steps, pl->hist_steps);
  if (int rc = use_device(c)) return rc;
  CK(c, cudaMemcpyAsync(out, pl->hist, (size_t)steps * pl->n_micro * pl->micro * 4, cudaMemcpyDeviceToHost, c->stream));
  return sync_check(c, std::max(kDefaultTimeoutMs, steps * 200));
}

int dllm_pipeline_synchronize(dllm_pipeline* pl, int timeout_ms) {
  if (!pl) return DLLM_EINVAL;
  if (int rc = use_device(pl->ctx)) return rc;
  return sync_check(pl->ctx, timeout_ms);
}

}  // extern "C"
