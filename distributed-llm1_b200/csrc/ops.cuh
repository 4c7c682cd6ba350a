// ops.cuh — host launchers of the op-level kernels (one per reference shader,
// kernels.js:26-171) and of the utility kernels (weights, KV cache, argmax).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.cuh"

namespace dllm {

// Raise the dynamic shared-memory limits of the op kernels on the current device.
cudaError_t configure_op_kernels();

// out[t, j] = sum_k x[t, k] * W[j, k]   (MATMUL, kernels.js:26-44)
cudaError_t op_matmul(const float* x, const __nv_bfloat16* w, float* out, int n, int din, int dout, int sms,
                      cudaStream_t st);
// RMSNORM (kernels.js:46-63), rows of d
cudaError_t op_rmsnorm(const float* x, const __nv_bfloat16* g, float* out, int n, int d, float eps, cudaStream_t st);
// ROPE (kernels.js:66-83), in place on n rows of heads*hd
cudaError_t op_rope(float* x, int n, int heads, int hd, int pos0, const float* freq, cudaStream_t st);
// SILUMUL / ADD / ADDBIAS (kernels.js:134-171)
cudaError_t op_silu_mul(const float* a, const float* b, float* out, int total, cudaStream_t st);
cudaError_t op_add(const float* a, const float* b, float* out, int total, cudaStream_t st);
cudaError_t op_add_bias(const float* a, const __nv_bfloat16* bias, float* out, int total, int dout, cudaStream_t st);
// ATTENTION (kernels.js:86-132) over fp32 caches [max_pos, kvh*hd]; rows[t] = {0, pos, T0 + t}
struct AttnScratch {
  float* part_o;
  float* part_ml;
  unsigned int* arrive;
  int max_splits;
};
cudaError_t op_attention(const float* q, const float* kc, const float* vc, float* out, const RowDesc* rows, int n,
                         int nq, int kvh, int hd, int max_pos, float scale, const AttnScratch& sc, int* err, int sms,
                         cudaStream_t st);
// ATTENTION over a stage's paged KV cache (the stage kernel's attention phase as
// its own cooperative launch); A.kc/A.vc are the layer's pools, kv_dtype 0 fp32, 1 bf16
cudaError_t op_attention_paged(const AttnArgs& A, int kv_dtype, int hd, int sms, cudaStream_t st);
// addBias + ropeQ/ropeK + appendKv of n rows whose q|k|v projections are in q, k, v
cudaError_t op_qkv_post(float* q, const float* k, const float* v, const __nv_bfloat16* bq, const __nv_bfloat16* bk,
                        const __nv_bfloat16* bv, int n, int NQ, int KVH, int HD, const float* freq,
                        const RowDesc* rows, const KvLayout& kv, void* kc, void* vc, int kv_dtype, int* err,
                        cudaStream_t st);
// greedy token of each of `rows` rows of n logits (best: [rows] keys, zero between uses)
cudaError_t op_argmax_rows(const float* logits, int rows, int n, unsigned long long* best, int32_t* tokens,
                           cudaStream_t st);
// argmax over n logits into *best (zero it first); lowest index wins ties
cudaError_t op_argmax(const float* logits, int n, unsigned long long* best, cudaStream_t st);
// embedding gather: out[t] = bf16->f32(E[tokens[t]])
cudaError_t op_embed(const __nv_bfloat16* E, const int32_t* tokens, float* out, int n, int d, int vocab, int* err,
                     cudaStream_t st);
// synthetic data
cudaError_t op_fill_normal_bf16(__nv_bfloat16* p, size_t n, uint64_t seed, float std, cudaStream_t st);
cudaError_t op_fill_const_bf16(__nv_bfloat16* p, size_t n, float v, cudaStream_t st);
cudaError_t op_u32_to_bf16(const uint32_t* src, __nv_bfloat16* dst, size_t n, cudaStream_t st);
// KV cache utilities; kv_dtype 0 fp32, 1 bf16
cudaError_t op_kv_fill_random(const KvLayout& kv, void* k, void* v, int kv_dtype, int seq, int n_slots, int kvh, int hd,
                              uint64_t seed, cudaStream_t st);
cudaError_t op_kv_read(const KvLayout& kv, const void* pool, int kv_dtype, int seq, int slot0, int n, int kvh, int hd,
                       float* out, cudaStream_t st);
cudaError_t op_kv_write(const KvLayout& kv, void* pool, int kv_dtype, int seq, int slot0, int n, int kvh, int hd,
                        const float* src, cudaStream_t st);

}  // namespace dllm
