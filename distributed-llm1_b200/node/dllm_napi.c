/*
 * dllm_napi.c — Node-API addon over libdllm.so (include/dllm.h), so the
 * reference's JavaScript (kernels.js, pipeline.js) can run on the B200 path.
 * kernels.js / pipeline.js in this directory are the drop-in modules built on it.
 *
 * Handles (ctx, buffers, stages, leaders, pipelines) are napi externals. Buffers
 * are released by the garbage collector (dllm_buf_free), as GPUBuffers are;
 * ctx, stage, leader and pipeline have explicit destroy calls (the ctx stays
 * alive until its last buffer is gone: the library reference-counts it).
 * A non-zero status throws `new Error(dllm_last_error(ctx))` with `code` set to
 * the status name, as the reference throws (kernels.js:182,189,196,204,244).
 * Calls that hand data back to JavaScript block the calling thread for at most
 * the library's bounded wait (readF32's 15 s, kernels.js:201-207); the JS
 * modules wrap them in Promises where the reference is async.
 *
 * Build (not run in this repository: there is no Node.js here): node-gyp with
 * binding.gyp next to this file, after `make -C ../csrc`.
 */
#include <node_api.h>
#include <stdlib.h>
#include <string.h>

#include "dllm.h"

typedef struct {
  dllm_stage* st;
  dllm_ctx* ctx;
  int owned; /* 0: a leader's stage, destroyed with the leader */
} stage_ref;

typedef struct {
  dllm_leader* ld;
  dllm_ctx* ctx;
} leader_ref;

typedef struct {
  dllm_pipeline* pl;
  dllm_ctx* ctx;
} pipeline_ref;

static const char* status_name(int st) {
  switch (st) {
    case DLLM_EINVAL: return "DLLM_EINVAL";
    case DLLM_ENOMEM: return "DLLM_ENOMEM";
    case DLLM_ERANGE: return "DLLM_ERANGE";
    case DLLM_ETIMEOUT: return "DLLM_ETIMEOUT";
    case DLLM_ECUDA: return "DLLM_ECUDA";
    case DLLM_ENOTFOUND: return "DLLM_ENOTFOUND";
    case DLLM_EDEVICE: return "DLLM_EDEVICE";
    default: return "DLLM_ERROR";
  }
}

static napi_value fail(napi_env env, const dllm_ctx* ctx, int st) {
  napi_throw_error(env, status_name(st), ctx ? dllm_last_error(ctx) : dllm_status_string(st));
  return NULL;
}

static napi_value type_error(napi_env env, const char* msg) {
  napi_throw_type_error(env, NULL, msg);
  return NULL;
}

#define ARGS(n)                                                   \
  size_t argc = (n);                                              \
  napi_value argv[(n) > 0 ? (n) : 1];                             \
  if (napi_get_cb_info(env, info, &argc, argv, NULL, NULL) != napi_ok) return NULL

static void* ext(napi_env env, napi_value v) {
  void* p = NULL;
  if (napi_get_value_external(env, v, &p) != napi_ok) return NULL;
  return p;
}

static int32_t i32(napi_env env, napi_value v) {
  int32_t x = 0;
  napi_get_value_int32(env, v, &x);
  return x;
}

static double f64(napi_env env, napi_value v) {
  double x = 0;
  napi_get_value_double(env, v, &x);
  return x;
}

static napi_value undef(napi_env env) {
  napi_value u;
  napi_get_undefined(env, &u);
  return u;
}

static napi_value num(napi_env env, double x) {
  napi_value v;
  napi_create_double(env, x, &v);
  return v;
}

/* typed-array view: data pointer and element count (NULL on a type mismatch) */
static void* typed(napi_env env, napi_value v, napi_typedarray_type want, size_t* n) {
  bool is = false;
  napi_is_typedarray(env, v, &is);
  if (!is) return NULL;
  napi_typedarray_type t;
  void* data = NULL;
  napi_value ab;
  size_t off = 0;
  napi_get_typedarray_info(env, v, &t, n, &data, &ab, &off);
  return t == want ? data : NULL;
}

static napi_value new_typed(napi_env env, napi_typedarray_type t, size_t n, size_t esize, void** data) {
  napi_value ab, out;
  napi_create_arraybuffer(env, n * esize, data, &ab);
  napi_create_typedarray(env, t, n, ab, 0, &out);
  return out;
}

static void buf_finalize(napi_env env, void* data, void* hint) {
  (void)env;
  (void)hint;
  dllm_buf_free((dllm_buf*)data);
}

static napi_value wrap_buf(napi_env env, dllm_buf* b) {
  napi_value out;
  napi_create_external(env, b, buf_finalize, NULL, &out);
  return out;
}

static char* label_of(napi_env env, napi_value v, char* dst, size_t cap) {
  size_t len = 0;
  dst[0] = 0;
  napi_valuetype t;
  napi_typeof(env, v, &t);
  if (t == napi_string) napi_get_value_string_utf8(env, v, dst, cap, &len);
  return dst;
}

/* ---- initKernels(device[, cfg]) (kernels.js:5) --------------------------------- */
static void cfg_field(napi_env env, napi_value obj, const char* key, int32_t* dst) {
  bool has = false;
  napi_has_named_property(env, obj, key, &has);
  if (!has) return;
  napi_value v;
  napi_get_named_property(env, obj, key, &v);
  *dst = i32(env, v);
}

static void cfg_field_f(napi_env env, napi_value obj, const char* key, float* dst) {
  bool has = false;
  napi_has_named_property(env, obj, key, &has);
  if (!has) return;
  napi_value v;
  napi_get_named_property(env, obj, key, &v);
  *dst = (float)f64(env, v);
}

static napi_value InitKernels(napi_env env, napi_callback_info info) {
  ARGS(2);
  int32_t dev = argc > 0 ? i32(env, argv[0]) : 0;
  dllm_config cfg;
  dllm_config_default(&cfg); /* CFG of constants.js:10-23 */
  if (argc > 1) {
    napi_valuetype t;
    napi_typeof(env, argv[1], &t);
    if (t == napi_object) {
      napi_value o = argv[1];
      cfg_field(env, o, "vocabSize", &cfg.vocab_size);
      cfg_field(env, o, "hiddenSize", &cfg.hidden_size);
      cfg_field(env, o, "numLayers", &cfg.num_layers);
      cfg_field(env, o, "numQHeads", &cfg.num_q_heads);
      cfg_field(env, o, "numKVHeads", &cfg.num_kv_heads);
      cfg_field(env, o, "headDim", &cfg.head_dim);
      cfg_field(env, o, "intermediateSize", &cfg.intermediate_size);
      cfg_field_f(env, o, "ropeTheta", &cfg.rope_theta);
      cfg_field_f(env, o, "rmsNormEps", &cfg.rms_norm_eps);
      cfg_field(env, o, "tieWordEmbeddings", &cfg.tie_word_embeddings);
      cfg_field(env, o, "eosTokenId", &cfg.eos_token_id);
      cfg_field(env, o, "maxPos", &cfg.max_pos);
      cfg_field(env, o, "kvDtype", &cfg.kv_dtype);
      cfg_field(env, o, "kvPageSize", &cfg.kv_page_size);
      cfg_field(env, o, "maxSeqs", &cfg.max_seqs);
    }
  }
  dllm_ctx* ctx = NULL;
  int st = dllm_init_kernels(dev, &cfg, &ctx);
  if (st) return fail(env, NULL, st);
  napi_value out;
  napi_create_external(env, ctx, NULL, NULL, &out); /* released by ctxDestroy */
  return out;
}

static napi_value CtxDestroy(napi_env env, napi_callback_info info) {
  ARGS(1);
  dllm_ctx_destroy((dllm_ctx*)ext(env, argv[0]));
  return undef(env);
}

static napi_value GetConfig(napi_env env, napi_callback_info info) {
  ARGS(1);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  dllm_config c;
  int st = dllm_ctx_get_config(ctx, &c);
  if (st) return fail(env, ctx, st);
  napi_value o;
  napi_create_object(env, &o);
  napi_set_named_property(env, o, "vocabSize", num(env, c.vocab_size));
  napi_set_named_property(env, o, "hiddenSize", num(env, c.hidden_size));
  napi_set_named_property(env, o, "numLayers", num(env, c.num_layers));
  napi_set_named_property(env, o, "numQHeads", num(env, c.num_q_heads));
  napi_set_named_property(env, o, "numKVHeads", num(env, c.num_kv_heads));
  napi_set_named_property(env, o, "headDim", num(env, c.head_dim));
  napi_set_named_property(env, o, "intermediateSize", num(env, c.intermediate_size));
  napi_set_named_property(env, o, "maxPos", num(env, c.max_pos));
  napi_set_named_property(env, o, "eosTokenId", num(env, c.eos_token_id));
  napi_set_named_property(env, o, "tieWordEmbeddings", num(env, c.tie_word_embeddings));
  return o;
}

/* ---- buffers (kernels.js:181-211) ------------------------------------------------ */
static napi_value LoadWeightBits(napi_env env, napi_callback_info info) {
  ARGS(3);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  size_t n = 0;
  const uint32_t* bits = (const uint32_t*)typed(env, argv[1], napi_uint32_array, &n);
  if (!bits) return type_error(env, "loadWeightBits: expected a Uint32Array");
  char lab[128];
  dllm_buf* b = NULL;
  int st = dllm_load_weight_bits(ctx, bits, n, argc > 2 ? label_of(env, argv[2], lab, sizeof lab) : "weights", &b);
  if (st) return fail(env, ctx, st);
  return wrap_buf(env, b);
}

static napi_value LoadWeightBf16(napi_env env, napi_callback_info info) {
  ARGS(3);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  size_t n = 0;
  const uint16_t* v = (const uint16_t*)typed(env, argv[1], napi_uint16_array, &n);
  if (!v) return type_error(env, "loadWeightBf16: expected a Uint16Array");
  char lab[128];
  dllm_buf* b = NULL;
  int st = dllm_load_weight_bf16(ctx, v, n, argc > 2 ? label_of(env, argv[2], lab, sizeof lab) : "weights", &b);
  if (st) return fail(env, ctx, st);
  return wrap_buf(env, b);
}

static napi_value CreateF32(napi_env env, napi_callback_info info) {
  ARGS(3);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  double n = f64(env, argv[1]);
  char lab[128];
  if (!(n > 0)) return fail(env, NULL, DLLM_EINVAL);
  dllm_buf* b = NULL;
  int st = dllm_create_f32(ctx, (size_t)n, argc > 2 ? label_of(env, argv[2], lab, sizeof lab) : "", &b);
  if (st) return fail(env, ctx, st);
  return wrap_buf(env, b);
}

static napi_value WriteF32(napi_env env, napi_callback_info info) {
  ARGS(3);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  size_t n = 0;
  const float* src = (const float*)typed(env, argv[2], napi_float32_array, &n);
  if (!src) return type_error(env, "writeF32: expected a Float32Array");
  int st = dllm_write_f32(ctx, (dllm_buf*)ext(env, argv[1]), src, n);
  if (st) return fail(env, ctx, st);
  return undef(env);
}

static napi_value ReadF32(napi_env env, napi_callback_info info) {
  ARGS(4);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  double n = f64(env, argv[2]);
  char lab[128];
  if (!(n > 0)) return fail(env, NULL, DLLM_EINVAL);
  void* data = NULL;
  napi_value out = new_typed(env, napi_float32_array, (size_t)n, 4, &data);
  int st = dllm_read_f32(ctx, (const dllm_buf*)ext(env, argv[1]), (float*)data, (size_t)n,
                         argc > 3 ? label_of(env, argv[3], lab, sizeof lab) : "");
  if (st) return fail(env, ctx, st);
  return out;
}

/* ---- ops, one per shader (kernels.js:222-301) ------------------------------------- */
static napi_value Matmul(napi_env env, napi_callback_info info) {
  ARGS(6);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  dllm_buf* o = NULL;
  int st = dllm_matmul(ctx, (dllm_buf*)ext(env, argv[1]), (dllm_buf*)ext(env, argv[2]), i32(env, argv[3]),
                       i32(env, argv[4]), i32(env, argv[5]), &o);
  if (st) return fail(env, ctx, st);
  return wrap_buf(env, o);
}

static napi_value Rmsnorm(napi_env env, napi_callback_info info) {
  ARGS(4);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  dllm_buf* o = NULL;
  int st = dllm_rmsnorm(ctx, (dllm_buf*)ext(env, argv[1]), (dllm_buf*)ext(env, argv[2]), i32(env, argv[3]), &o);
  if (st) return fail(env, ctx, st);
  return wrap_buf(env, o);
}

static napi_value Rope(napi_env env, napi_callback_info info, int q) {
  ARGS(4);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  dllm_buf* x = (dllm_buf*)ext(env, argv[1]);
  int st = q ? dllm_rope_q(ctx, x, i32(env, argv[2]), i32(env, argv[3]))
             : dllm_rope_k(ctx, x, i32(env, argv[2]), i32(env, argv[3]));
  if (st) return fail(env, ctx, st);
  return argv[1]; /* in place, like ctx.ropeQ/ropeK */
}
static napi_value RopeQ(napi_env env, napi_callback_info info) { return Rope(env, info, 1); }
static napi_value RopeK(napi_env env, napi_callback_info info) { return Rope(env, info, 0); }

static napi_value Attention(napi_env env, napi_callback_info info) {
  ARGS(6);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  dllm_buf* o = NULL;
  int st = dllm_attention(ctx, (dllm_buf*)ext(env, argv[1]), (dllm_buf*)ext(env, argv[2]),
                          (dllm_buf*)ext(env, argv[3]), i32(env, argv[4]), i32(env, argv[5]), &o);
  if (st) return fail(env, ctx, st);
  return wrap_buf(env, o);
}

static napi_value SiluMul(napi_env env, napi_callback_info info) {
  ARGS(4);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  dllm_buf* o = NULL;
  int st = dllm_silu_mul(ctx, (dllm_buf*)ext(env, argv[1]), (dllm_buf*)ext(env, argv[2]), i32(env, argv[3]), &o);
  if (st) return fail(env, ctx, st);
  return wrap_buf(env, o);
}

static napi_value Add(napi_env env, napi_callback_info info) {
  ARGS(4);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  dllm_buf* o = NULL;
  int st = dllm_add(ctx, (dllm_buf*)ext(env, argv[1]), (dllm_buf*)ext(env, argv[2]), i32(env, argv[3]), &o);
  if (st) return fail(env, ctx, st);
  return wrap_buf(env, o);
}

static napi_value AddBias(napi_env env, napi_callback_info info) {
  ARGS(5);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  dllm_buf* o = NULL;
  int st = dllm_add_bias(ctx, (dllm_buf*)ext(env, argv[1]), (dllm_buf*)ext(env, argv[2]), i32(env, argv[3]),
                         i32(env, argv[4]), &o);
  if (st) return fail(env, ctx, st);
  return wrap_buf(env, o);
}

/* ---- Stage (pipeline.js:26-88) ---------------------------------------------------- */
static void stage_finalize(napi_env env, void* data, void* hint) {
  (void)env;
  (void)hint;
  stage_ref* r = (stage_ref*)data;
  if (r->owned && r->st) dllm_stage_destroy(r->st);
  free(r);
}

static napi_value wrap_stage(napi_env env, dllm_stage* st, dllm_ctx* ctx, int owned) {
  stage_ref* r = (stage_ref*)calloc(1, sizeof *r);
  r->st = st;
  r->ctx = ctx;
  r->owned = owned;
  napi_value out;
  napi_create_external(env, r, stage_finalize, NULL, &out);
  return out;
}

static napi_value StageCreate(napi_env env, napi_callback_info info) {
  ARGS(3);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  dllm_stage* st = NULL;
  int rc = dllm_stage_create(ctx, i32(env, argv[1]), i32(env, argv[2]), &st);
  if (rc) return fail(env, ctx, rc);
  return wrap_stage(env, st, ctx, 1);
}

static napi_value StageSetWeight(napi_env env, napi_callback_info info) {
  ARGS(3);
  stage_ref* r = (stage_ref*)ext(env, argv[0]);
  char name[256];
  int rc = dllm_stage_set_weight(r->st, label_of(env, argv[1], name, sizeof name), (dllm_buf*)ext(env, argv[2]));
  if (rc) return fail(env, r->ctx, rc);
  return undef(env);
}

static napi_value StageReset(napi_env env, napi_callback_info info) {
  ARGS(1);
  stage_ref* r = (stage_ref*)ext(env, argv[0]);
  int rc = dllm_stage_reset(r->st);
  if (rc) return fail(env, r->ctx, rc);
  return undef(env);
}

static napi_value StageGetT0(napi_env env, napi_callback_info info) {
  ARGS(2);
  stage_ref* r = (stage_ref*)ext(env, argv[0]);
  return num(env, dllm_stage_get_t0(r->st, argc > 1 ? i32(env, argv[1]) : 0));
}

static napi_value StageSetT0(napi_env env, napi_callback_info info) {
  ARGS(3);
  stage_ref* r = (stage_ref*)ext(env, argv[0]);
  int rc = dllm_stage_set_t0(r->st, i32(env, argv[1]), i32(env, argv[2]));
  if (rc) return fail(env, r->ctx, rc);
  return undef(env);
}

static napi_value StageForward(napi_env env, napi_callback_info info) {
  ARGS(4);
  stage_ref* r = (stage_ref*)ext(env, argv[0]);
  size_t n = 0;
  const float* h = (const float*)typed(env, argv[1], napi_float32_array, &n);
  if (!h) return type_error(env, "Stage.forward: expected a Float32Array");
  dllm_buf* o = NULL;
  int rc = dllm_stage_forward(r->st, h, i32(env, argv[2]), i32(env, argv[3]), &o);
  if (rc) return fail(env, r->ctx, rc);
  return wrap_buf(env, o);
}

static napi_value StageAppendKv(napi_env env, napi_callback_info info) {
  ARGS(5);
  stage_ref* r = (stage_ref*)ext(env, argv[0]);
  int rc = dllm_stage_append_kv(r->st, i32(env, argv[1]), (dllm_buf*)ext(env, argv[2]), (dllm_buf*)ext(env, argv[3]),
                                i32(env, argv[4]));
  if (rc) return fail(env, r->ctx, rc);
  return undef(env);
}

/* ---- LeaderPipeline (pipeline.js:91-282) ---------------------------------------------- */
static void leader_finalize(napi_env env, void* data, void* hint) {
  (void)env;
  (void)hint;
  leader_ref* r = (leader_ref*)data;
  if (r->ld) dllm_leader_destroy(r->ld);
  free(r);
}

static napi_value LeaderCreate(napi_env env, napi_callback_info info) {
  ARGS(3);
  dllm_ctx* ctx = (dllm_ctx*)ext(env, argv[0]);
  dllm_leader* ld = NULL;
  int rc = dllm_leader_create(ctx, i32(env, argv[1]), i32(env, argv[2]), &ld);
  if (rc) return fail(env, ctx, rc);
  leader_ref* r = (leader_ref*)calloc(1, sizeof *r);
  r->ld = ld;
  r->ctx = ctx;
  napi_value out;
  napi_create_external(env, r, leader_finalize, NULL, &out);
  return out;
}

static napi_value LeaderStage(napi_env env, napi_callback_info info) {
  ARGS(1);
  leader_ref* r = (leader_ref*)ext(env, argv[0]);
  return wrap_stage(env, dllm_leader_stage(r->ld), r->ctx, 0);
}

static napi_value LeaderSetWeights(napi_env env, napi_callback_info info) {
  ARGS(4);
  leader_ref* r = (leader_ref*)ext(env, argv[0]);
  dllm_buf* bufs[3] = {NULL, NULL, NULL};
  for (int i = 0; i < 3 && (size_t)(i + 1) < argc; ++i) bufs[i] = (dllm_buf*)ext(env, argv[i + 1]);
  int rc = dllm_leader_set_weights(r->ld, bufs[0], bufs[1], bufs[2]);
  if (rc) return fail(env, r->ctx, rc);
  return undef(env);
}

static napi_value LeaderEmbedTokens(napi_env env, napi_callback_info info) {
  ARGS(2);
  leader_ref* r = (leader_ref*)ext(env, argv[0]);
  size_t n = 0;
  const int32_t* t = (const int32_t*)typed(env, argv[1], napi_int32_array, &n);
  if (!t || n == 0) return type_error(env, "embedTokens: expected a non-empty Int32Array");
  dllm_config c;
  dllm_ctx_get_config(r->ctx, &c);
  void* data = NULL;
  napi_value out = new_typed(env, napi_float32_array, n * (size_t)c.hidden_size, 4, &data);
  int rc = dllm_leader_embed_tokens(r->ld, t, (int)n, (float*)data);
  if (rc) return fail(env, r->ctx, rc);
  return out;
}

static napi_value LeaderSampleLast(napi_env env, napi_callback_info info) {
  ARGS(2);
  leader_ref* r = (leader_ref*)ext(env, argv[0]);
  size_t n = 0;
  const float* h = (const float*)typed(env, argv[1], napi_float32_array, &n);
  if (!h) return type_error(env, "sampleLast: expected a Float32Array");
  int32_t tok = 0;
  int rc = dllm_leader_sample_last(r->ld, h, &tok, NULL);
  if (rc) return fail(env, r->ctx, rc);
  return num(env, tok);
}

static napi_value LeaderForward(napi_env env, napi_callback_info info) {
  ARGS(4);
  leader_ref* r = (leader_ref*)ext(env, argv[0]);
  size_t n = 0;
  const float* h = (const float*)typed(env, argv[1], napi_float32_array, &n);
  if (!h) return type_error(env, "forward: expected a Float32Array");
  dllm_config c;
  dllm_ctx_get_config(r->ctx, &c);
  void* data = NULL;
  napi_value out = new_typed(env, napi_float32_array, (size_t)c.hidden_size, 4, &data);
  int rc = dllm_leader_forward(r->ld, h, i32(env, argv[2]), i32(env, argv[3]), (float*)data);
  if (rc) return fail(env, r->ctx, rc);
  return out;
}

static napi_value LeaderGenerate(napi_env env, napi_callback_info info) {
  ARGS(3);
  leader_ref* r = (leader_ref*)ext(env, argv[0]);
  size_t n = 0;
  const int32_t* t = (const int32_t*)typed(env, argv[1], napi_int32_array, &n);
  int32_t max_new = i32(env, argv[2]);
  if (!t || n == 0 || max_new < 1) return type_error(env, "generate: expected tokens and maxNew >= 1");
  int32_t* buf = (int32_t*)malloc(sizeof(int32_t) * (size_t)max_new);
  int got = 0;
  int rc = dllm_leader_generate(r->ld, t, (int)n, max_new, buf, &got);
  if (rc) {
    free(buf);
    return fail(env, r->ctx, rc);
  }
  void* data = NULL;
  napi_value out = new_typed(env, napi_int32_array, (size_t)got, 4, &data);
  memcpy(data, buf, sizeof(int32_t) * (size_t)got);
  free(buf);
  return out;
}

/* ---- multi-GPU pipeline ----------------------------------------------------------------- */
static void pipeline_finalize(napi_env env, void* data, void* hint) {
  (void)env;
  (void)hint;
  pipeline_ref* r = (pipeline_ref*)data;
  if (r->pl) dllm_pipeline_destroy(r->pl);
  free(r);
}

static napi_value PipelineCreate(napi_env env, napi_callback_info info) {
  ARGS(5);
  stage_ref* s = (stage_ref*)ext(env, argv[0]);
  dllm_pipeline* pl = NULL;
  int rc = dllm_pipeline_create(s->st, i32(env, argv[1]), i32(env, argv[2]), i32(env, argv[3]), i32(env, argv[4]), &pl);
  if (rc) return fail(env, s->ctx, rc);
  pipeline_ref* r = (pipeline_ref*)calloc(1, sizeof *r);
  r->pl = pl;
  r->ctx = s->ctx;
  napi_value out;
  napi_create_external(env, r, pipeline_finalize, NULL, &out);
  return out;
}

static napi_value PipelineHandle(napi_env env, napi_callback_info info) {
  ARGS(1);
  pipeline_ref* r = (pipeline_ref*)ext(env, argv[0]);
  void* data = NULL;
  napi_value out = new_typed(env, napi_uint8_array, DLLM_PIPELINE_HANDLE_BYTES, 1, &data);
  int rc = dllm_pipeline_handle(r->pl, (uint8_t*)data);
  if (rc) return fail(env, r->ctx, rc);
  return out;
}

static napi_value PipelineConnect(napi_env env, napi_callback_info info) {
  ARGS(2);
  pipeline_ref* r = (pipeline_ref*)ext(env, argv[0]);
  size_t n = 0;
  const uint8_t* h = (const uint8_t*)typed(env, argv[1], napi_uint8_array, &n);
  if (!h || n != DLLM_PIPELINE_HANDLE_BYTES) return type_error(env, "pipeline connect: expected a 64-byte Uint8Array");
  int rc = dllm_pipeline_connect(r->pl, h);
  if (rc) return fail(env, r->ctx, rc);
  return undef(env);
}

static napi_value PipelineSetTokens(napi_env env, napi_callback_info info) {
  ARGS(2);
  pipeline_ref* r = (pipeline_ref*)ext(env, argv[0]);
  size_t n = 0;
  const int32_t* t = (const int32_t*)typed(env, argv[1], napi_int32_array, &n);
  if (!t) return type_error(env, "pipeline setTokens: expected an Int32Array");
  int rc = dllm_pipeline_set_tokens(r->pl, t, (int)n);
  if (rc) return fail(env, r->ctx, rc);
  return undef(env);
}

static napi_value PipelineRun(napi_env env, napi_callback_info info) {
  ARGS(2);
  pipeline_ref* r = (pipeline_ref*)ext(env, argv[0]);
  int rc = dllm_pipeline_run(r->pl, i32(env, argv[1]));
  if (rc) return fail(env, r->ctx, rc);
  return undef(env);
}

static napi_value PipelineReadTokens(napi_env env, napi_callback_info info) {
  ARGS(3);
  pipeline_ref* r = (pipeline_ref*)ext(env, argv[0]);
  int32_t steps = i32(env, argv[1]), per_step = i32(env, argv[2]);
  if (steps < 1 || per_step < 1) return type_error(env, "pipeline readTokens: steps and sequences must be >= 1");
  void* data = NULL;
  napi_value out = new_typed(env, napi_int32_array, (size_t)steps * per_step, 4, &data);
  int rc = dllm_pipeline_read_tokens(r->pl, (int32_t*)data, steps);
  if (rc) return fail(env, r->ctx, rc);
  return out;
}

/* ---- module ------------------------------------------------------------------------------ */
#define FN(name, fn) {name, NULL, fn, NULL, NULL, NULL, napi_default, NULL}

static napi_value Init(napi_env env, napi_value exports) {
  napi_property_descriptor props[] = {
      FN("initKernels", InitKernels), FN("ctxDestroy", CtxDestroy), FN("getConfig", GetConfig),
      FN("loadWeightBits", LoadWeightBits), FN("loadWeightBf16", LoadWeightBf16), FN("createF32", CreateF32),
      FN("writeF32", WriteF32), FN("readF32", ReadF32), FN("matmul", Matmul), FN("rmsnorm", Rmsnorm),
      FN("ropeQ", RopeQ), FN("ropeK", RopeK), FN("attention", Attention), FN("siluMul", SiluMul), FN("add", Add),
      FN("addBias", AddBias), FN("stageCreate", StageCreate), FN("stageSetWeight", StageSetWeight),
      FN("stageReset", StageReset), FN("stageGetT0", StageGetT0), FN("stageSetT0", StageSetT0),
      FN("stageForward", StageForward), FN("stageAppendKv", StageAppendKv), FN("leaderCreate", LeaderCreate),
      FN("leaderStage", LeaderStage), FN("leaderSetWeights", LeaderSetWeights),
      FN("leaderEmbedTokens", LeaderEmbedTokens), FN("leaderSampleLast", LeaderSampleLast),
      FN("leaderForward", LeaderForward), FN("leaderGenerate", LeaderGenerate),
      FN("pipelineCreate", PipelineCreate), FN("pipelineHandle", PipelineHandle),
      FN("pipelineConnect", PipelineConnect), FN("pipelineSetTokens", PipelineSetTokens),
      FN("pipelineRun", PipelineRun), FN("pipelineReadTokens", PipelineReadTokens),
  };
  napi_define_properties(env, exports, sizeof props / sizeof props[0], props);
  return exports;
}

NAPI_MODULE(NODE_GYP_MODULE_NAME, Init)
