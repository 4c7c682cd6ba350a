// ops.cu — op-level kernels behind the ctx API of kernels.js (one launcher per
// shader) and utility kernels (synthetic weights, KV cache access, argmax).
// The matvec and attention ops reuse the phase code of the stage kernel.
#include <chrono>
#include <cmath>
#include <thread>

#include "dllm.h"
#include "kernels.cuh"
#include "ops.cuh"
#include "stage.cuh"

namespace dllm {

// ---- counter-based synthetic data (splitmix64 finalizer + Box-Muller) -----------
__host__ __device__ inline uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
DLLM_DEV float hash_normal(uint64_t seed, uint64_t i) {
  const uint64_t r = mix64(mix64(seed) ^ i);
  const float u1 = ((float)(r >> 40) + 1.0f) * 5.9604644775390625e-8f;  // (0, 1]
  const float u2 = (float)(r & 0xffffffull) * 5.9604644775390625e-8f;   // [0, 1)
  return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

template <typename T>
DLLM_DEV T cvt_out(float v);
template <>
DLLM_DEV float cvt_out<float>(float v) { return v; }
template <>
DLLM_DEV __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return f32_to_bf16(v); }
DLLM_DEV float cvt_in(float v) { return v; }
DLLM_DEV float cvt_in(__nv_bfloat16 v) { return bf16_to_f32(v); }

static inline unsigned int blocks_for(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  if (b > 0x7fffffffll) b = 0x7fffffffll;
  return (unsigned int)(b < 1 ? 1 : b);
}

// ---- MATMUL ---------------------------------------------------------------------
template <int M>
__global__ void __launch_bounds__(kThreads, 1)
    matmul_kernel(const float* x, const __nv_bfloat16* w, float* out, int n, int din, int dout) {
  extern __shared__ __align__(16) float smem[];
  __shared__ float red[32];
  const int m0 = blockIdx.y * M;
  const int mr = min(M, n - m0);
  const PhaseSmem sm{smem, kStageXsFloats, smem + kStageXsFloats, kStagePartFloats, red};
  const EpiStore e{w, out + (size_t)m0 * dout, dout};
  NoState ns;
  gemv_phase<EpiStore, M>(e, GemvIn{x + (size_t)m0 * din, din, mr, nullptr, 0.f}, dout, sm, blockIdx.x, gridDim.x,
                          ns);
}

template <int M>
static cudaError_t launch_matmul(const float* x, const __nv_bfloat16* w, float* out, int n, int din, int dout,
                                 int sms, cudaStream_t st) {
  dim3 grid(sms, (n + M - 1) / M);
  matmul_kernel<M><<<grid, kThreads, kStageSmemBytes, st>>>(x, w, out, n, din, dout);
  return cudaGetLastError();
}

cudaError_t op_matmul(const float* x, const __nv_bfloat16* w, float* out, int n, int din, int dout, int sms,
                      cudaStream_t st) {
  if (n <= 1) return launch_matmul<1>(x, w, out, n, din, dout, sms, st);
  if (n <= 2) return launch_matmul<2>(x, w, out, n, din, dout, sms, st);
  if (n <= 4) return launch_matmul<4>(x, w, out, n, din, dout, sms, st);
  return launch_matmul<8>(x, w, out, n, din, dout, sms, st);
}

// ---- RMSNORM --------------------------------------------------------------------
__global__ void rmsnorm_kernel(const float* x, const __nv_bfloat16* g, float* out, int d, float eps) {
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * d;
  float* orow = out + (size_t)blockIdx.x * d;
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float v = xr[i];
    ss = fmaf(v, v, ss);
  }
  const float tot = block_sum(ss, red);
  const float scale = 1.0f / sqrtf(tot / (float)d + eps);
  for (int i = threadIdx.x; i < d; i += blockDim.x) orow[i] = (xr[i] * scale) * bf16_to_f32(g[i]);
}

cudaError_t op_rmsnorm(const float* x, const __nv_bfloat16* g, float* out, int n, int d, float eps, cudaStream_t st) {
  rmsnorm_kernel<<<n, 256, 0, st>>>(x, g, out, d, eps);
  return cudaGetLastError();
}

// ---- ROPE -----------------------------------------------------------------------
__global__ void rope_kernel(float* x, int n, int heads, int hd, int pos0, const float* freq) {
  const int half_n = hd >> 1;
  const long long total = (long long)n * heads * half_n;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int half = (int)(i % half_n);
  const long long th = i / half_n;
  const int h = (int)(th % heads);
  const int t = (int)(th / heads);
  const float ang = __fmul_rn((float)(pos0 + t), freq[half]);
  float s, c;
  sincosf(ang, &s, &c);
  float* row = x + (size_t)t * heads * hd + (size_t)h * hd;
  const float x1 = row[half], x2 = row[half + half_n];
  row[half] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
  row[half + half_n] = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
}

cudaError_t op_rope(float* x, int n, int heads, int hd, int pos0, const float* freq, cudaStream_t st) {
  const long long total = (long long)n * heads * (hd / 2);
  rope_kernel<<<blocks_for(total, 256), 256, 0, st>>>(x, n, heads, hd, pos0, freq);
  return cudaGetLastError();
}

// ---- SILUMUL / ADD / ADDBIAS ------------------------------------------------------
__global__ void silu_mul_kernel(const float* a, const float* b, float* out, int total) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const float v = a[i];
  out[i] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), b[i]);
}
__global__ void add_kernel(const float* a, const float* b, float* out, int total) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < total) out[i] = __fadd_rn(a[i], b[i]);
}
__global__ void add_bias_kernel(const float* a, const __nv_bfloat16* bias, float* out, int total, int dout) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < total) out[i] = __fadd_rn(a[i], bf16_to_f32(bias[i % dout]));
}

cudaError_t op_silu_mul(const float* a, const float* b, float* out, int total, cudaStream_t st) {
  silu_mul_kernel<<<blocks_for(total, 256), 256, 0, st>>>(a, b, out, total);
  return cudaGetLastError();
}
cudaError_t op_add(const float* a, const float* b, float* out, int total, cudaStream_t st) {
  add_kernel<<<blocks_for(total, 256), 256, 0, st>>>(a, b, out, total);
  return cudaGetLastError();
}
cudaError_t op_add_bias(const float* a, const __nv_bfloat16* bias, float* out, int total, int dout, cudaStream_t st) {
  add_bias_kernel<<<blocks_for(total, 256), 256, 0, st>>>(a, bias, out, total, dout);
  return cudaGetLastError();
}

// ---- ATTENTION (reference cache layout) -------------------------------------------
template <int HD>
constexpr size_t attn_smem_bytes() {
  return sizeof(float) * (size_t)attn_smem_floats<float, HD>();
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1) attention_op_kernel(const AttnArgs A) {
  extern __shared__ __align__(16) float smem[];
  attn_phase<float, HD>(A, smem, blockIdx.x, gridDim.x);
}

// Cooperative launch: the CTAs holding the splits of one (row, kv head) wait for
// each other before merging, so all of them must be resident.
template <int HD>
static cudaError_t launch_attention(const AttnArgs& A, int sms, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = attn_smem_bytes<HD>();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attention_op_kernel<HD>, A);
}

// ---- ATTENTION over a stage's paged cache (wide passes) -----------------------------
template <typename KT, int HD>
__global__ void __launch_bounds__(kThreads, 1) attention_paged_kernel(const AttnArgs A) {
  extern __shared__ __align__(16) float smem[];
  attn_phase<KT, HD>(A, smem, blockIdx.x, gridDim.x);
}

template <typename KT, int HD>
static cudaError_t launch_attention_paged(const AttnArgs& A, int sms, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = sizeof(float) * (size_t)attn_smem_floats<KT, HD>();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // split CTAs of a (row, kv head) wait for each other
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attention_paged_kernel<KT, HD>, A);
}

cudaError_t op_attention_paged(const AttnArgs& A, int kv_dtype, int hd, int sms, cudaStream_t st) {
  if (kv_dtype == 0) {
    if (hd == 64) return launch_attention_paged<float, 64>(A, sms, st);
    if (hd == 128) return launch_attention_paged<float, 128>(A, sms, st);
  } else {
    if (hd == 64) return launch_attention_paged<__nv_bfloat16, 64>(A, sms, st);
    if (hd == 128) return launch_attention_paged<__nv_bfloat16, 128>(A, sms, st);
  }
  return cudaErrorInvalidValue;
}

// ---- q|k|v epilogue of a wide pass: addBias, ropeQ/ropeK, appendKv -------------------
// Thread per (row, head, half): the same arithmetic as the stage kernel's fused
// epilogue (pipeline.js:59-64, kernels.js:66-83 and :148-159); k and v go to the
// row's KV slot through the paged layout, q is rotated in place.
template <typename KT>
__global__ void qkv_post_kernel(float* q, const float* k, const float* v, const __nv_bfloat16* bq,
                                const __nv_bfloat16* bk, const __nv_bfloat16* bv, int n, int NQ, int KVH, int HD,
                                const float* freq, const RowDesc* rows, KvLayout kv, KT* kc, KT* vc, int* err) {
  const int half_n = HD >> 1;
  const int heads = NQ + 2 * KVH;
  const long long total = (long long)n * heads * half_n;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int half = (int)(i % half_n);
    const int hh = (int)((i / half_n) % heads);
    const int t = (int)(i / ((long long)half_n * heads));
    int kind, lh;
    if (hh < NQ) {
      kind = 0;
      lh = hh;
    } else if (hh < NQ + KVH) {
      kind = 1;
      lh = hh - NQ;
    } else {
      kind = 2;
      lh = hh - NQ - KVH;
    }
    const int j0 = lh * HD + half, j1 = j0 + half_n;
    const float* src = kind == 0 ? q + (size_t)t * NQ * HD : (kind == 1 ? k : v) + (size_t)t * KVH * HD;
    float x1 = src[j0], x2 = src[j1];
    const __nv_bfloat16* b = kind == 0 ? bq : (kind == 1 ? bk : bv);
    if (b) {
      x1 = __fadd_rn(x1, bf16_to_f32(b[j0]));
      x2 = __fadd_rn(x2, bf16_to_f32(b[j1]));
    }
    const RowDesc rd = rows[t];
    if (kind < 2) {
      const float ang = __fmul_rn((float)rd.pos, freq[half]);
      float sn, cs;
      sincosf(ang, &sn, &cs);
      const float o1 = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
      const float o2 = __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs));
      x1 = o1;
      x2 = o2;
    }
    if (kind == 0) {
      float* qr = q + (size_t)t * NQ * HD;
      qr[j0] = x1;
      qr[j1] = x2;
      continue;
    }
    if (rd.slot < 0 || rd.slot >= kv.max_slots || rd.seq < 0 || rd.seq >= kv.num_seqs) {
      atomicExch(err, kErrKvRange);
      continue;
    }
    KT* base = (kind == 1 ? kc : vc) + kv.offset(rd.seq, rd.slot, lh);
    base[half] = cvt_out<KT>(x1);
    base[half + half_n] = cvt_out<KT>(x2);
  }
}

cudaError_t op_qkv_post(float* q, const float* k, const float* v, const __nv_bfloat16* bq, const __nv_bfloat16* bk,
                        const __nv_bfloat16* bv, int n, int NQ, int KVH, int HD, const float* freq,
                        const RowDesc* rows, const KvLayout& kv, void* kc, void* vc, int kv_dtype, int* err,
                        cudaStream_t st) {
  const long long total = (long long)n * (NQ + 2 * KVH) * (HD / 2);
  const unsigned int b = blocks_for(total, 256);
  if (kv_dtype == 0)
    qkv_post_kernel<float><<<b, 256, 0, st>>>(q, k, v, bq, bk, bv, n, NQ, KVH, HD, freq, rows, kv, (float*)kc,
                                              (float*)vc, err);
  else
    qkv_post_kernel<__nv_bfloat16><<<b, 256, 0, st>>>(q, k, v, bq, bk, bv, n, NQ, KVH, HD, freq, rows, kv,
                                                      (__nv_bfloat16*)kc, (__nv_bfloat16*)vc, err);
  return cudaGetLastError();
}

// ---- greedy argmax of many rows (sampleLast per sequence, pipeline.js:159-162) --------
__global__ void argmax_rows_kernel(const float* logits, int n, unsigned long long* best) {
  __shared__ unsigned long long sb;
  const int row = blockIdx.y;
  if (threadIdx.x == 0) sb = 0ull;
  __syncthreads();
  unsigned long long k = 0ull;
  const float* x = logits + (size_t)row * n;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long kk = argmax_key(x[i], i);
    if (kk > k) k = kk;
  }
  if (k) atomicMax(&sb, k);
  __syncthreads();
  if (threadIdx.x == 0 && sb) atomicMax(best + row, sb);
}
__global__ void argmax_tokens_kernel(unsigned long long* best, int rows, int32_t* tokens) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows) {
    const unsigned long long k = best[r];
    tokens[r] = k == 0ull ? 0 : argmax_key_index(k);  // all-NaN row: index 0 (the reference's initial best)
    best[r] = 0ull;
  }
}

cudaError_t op_argmax_rows(const float* logits, int rows, int n, unsigned long long* best, int32_t* tokens,
                           cudaStream_t st) {
  argmax_rows_kernel<<<dim3(64, rows), 256, 0, st>>>(logits, n, best);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  argmax_tokens_kernel<<<(rows + 127) / 128, 128, 0, st>>>(best, rows, tokens);
  return cudaGetLastError();
}

cudaError_t configure_op_kernels() {
  const int mm = (int)kStageSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(matmul_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, mm);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(matmul_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, mm);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(matmul_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, mm);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(matmul_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, mm);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_op_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn_smem_bytes<64>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_op_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn_smem_bytes<128>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_paged_kernel<float, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(float) * attn_smem_floats<float, 64>()));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_paged_kernel<float, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(float) * attn_smem_floats<float, 128>()));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_paged_kernel<__nv_bfloat16, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(float) * attn_smem_floats<__nv_bfloat16, 64>()));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_paged_kernel<__nv_bfloat16, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(float) * attn_smem_floats<__nv_bfloat16, 128>()));
  return e;
}

cudaError_t op_attention(const float* q, const float* kc, const float* vc, float* out, const RowDesc* rows, int n,
                         int nq, int kvh, int hd, int max_pos, float scale, const AttnScratch& sc, int* err, int sms,
                         cudaStream_t st) {
  KvLayout kv{};
  kv.page_table = nullptr;
  kv.log2_page = 30;  // the whole cache is one page: slot-major rows [max_pos, kvh*hd]
  kv.max_pages = 1;
  kv.head_stride = hd;
  kv.row_stride = kvh * hd;
  kv.page_stride = 0;
  kv.max_slots = max_pos;
  kv.num_seqs = 1;
  AttnArgs A{q, out, kc, vc, kv, rows, n, nq, kvh, scale, sc.max_splits, sc.part_o, sc.part_ml, sc.arrive, err};
  if (hd == 64) return launch_attention<64>(A, sms, st);
  if (hd == 128) return launch_attention<128>(A, sms, st);
  return cudaErrorInvalidValue;
}

// ---- argmax -------------------------------------------------------------------------
__global__ void argmax_kernel(const float* x, int n, unsigned long long* best) {
  __shared__ unsigned long long sb;
  if (threadIdx.x == 0) sb = 0ull;
  __syncthreads();
  unsigned long long k = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long kk = argmax_key(x[i], i);
    if (kk > k) k = kk;
  }
  if (k) atomicMax(&sb, k);
  __syncthreads();
  if (threadIdx.x == 0 && sb) atomicMax(best, sb);
}

cudaError_t op_argmax(const float* logits, int n, unsigned long long* best, cudaStream_t st) {
  unsigned int blocks = blocks_for(n, 256);
  if (blocks > 1184) blocks = 1184;
  argmax_kernel<<<blocks, 256, 0, st>>>(logits, n, best);
  return cudaGetLastError();
}

// ---- embedding gather ----------------------------------------------------------------
__global__ void embed_kernel(const __nv_bfloat16* E, const int32_t* tokens, float* out, int n, int d, int vocab,
                             int* err) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)n * d) return;
  const int t = (int)(i / d), k = (int)(i % d);
  int tok = tokens[t];
  if (tok < 0 || tok >= vocab) {
    if (k == 0) atomicExch(err, kErrToken);
    tok = 0;
  }
  out[i] = bf16_to_f32(E[(size_t)tok * d + k]);
}

cudaError_t op_embed(const __nv_bfloat16* E, const int32_t* tokens, float* out, int n, int d, int vocab, int* err,
                     cudaStream_t st) {
  embed_kernel<<<blocks_for((long long)n * d, 256), 256, 0, st>>>(E, tokens, out, n, d, vocab, err);
  return cudaGetLastError();
}

// ---- synthetic weights -------------------------------------------------------------
__global__ void fill_normal_bf16_kernel(__nv_bfloat16* p, size_t n, uint64_t seed, float std) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    p[i] = f32_to_bf16(hash_normal(seed, i) * std);
}
__global__ void fill_const_bf16_kernel(__nv_bfloat16* p, size_t n, float v) {
  const __nv_bfloat16 b = f32_to_bf16(v);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = b;
}
__global__ void u32_to_bf16_kernel(const uint32_t* src, __nv_bfloat16* dst, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = __ushort_as_bfloat16((unsigned short)(src[i] & 0xffffu));
}

cudaError_t op_fill_normal_bf16(__nv_bfloat16* p, size_t n, uint64_t seed, float std, cudaStream_t st) {
  fill_normal_bf16_kernel<<<4096, 256, 0, st>>>(p, n, seed, std);
  return cudaGetLastError();
}
cudaError_t op_fill_const_bf16(__nv_bfloat16* p, size_t n, float v, cudaStream_t st) {
  fill_const_bf16_kernel<<<4096, 256, 0, st>>>(p, n, v);
  return cudaGetLastError();
}
cudaError_t op_u32_to_bf16(const uint32_t* src, __nv_bfloat16* dst, size_t n, cudaStream_t st) {
  u32_to_bf16_kernel<<<4096, 256, 0, st>>>(src, dst, n);
  return cudaGetLastError();
}

// ---- KV cache utilities -----------------------------------------------------------------
template <typename KT>
__global__ void kv_fill_random_kernel(KvLayout kv, KT* k, KT* v, int seq, int n_slots, int kvh, int hd,
                                      uint64_t seed) {
  const long long total = (long long)n_slots * kvh * hd;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % hd);
    const long long sh = i / hd;
    const int head = (int)(sh % kvh);
    const int slot = (int)(sh / kvh);
    const long long off = kv.offset(seq, slot, head) + d;
    k[off] = cvt_out<KT>(hash_normal(seed, 2ull * (uint64_t)i));
    v[off] = cvt_out<KT>(hash_normal(seed, 2ull * (uint64_t)i + 1ull));
  }
}
template <typename KT>
__global__ void kv_read_kernel(KvLayout kv, const KT* pool, int seq, int slot0, int n, int kvh, int hd, float* out) {
  const long long total = (long long)n * kvh * hd;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int d = (int)(i % hd);
  const long long sh = i / hd;
  const int head = (int)(sh % kvh);
  const int t = (int)(sh / kvh);
  out[i] = cvt_in(pool[kv.offset(seq, slot0 + t, head) + d]);
}
template <typename KT>
__global__ void kv_write_kernel(KvLayout kv, KT* pool, int seq, int slot0, int n, int kvh, int hd, const float* src) {
  const long long total = (long long)n * kvh * hd;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int d = (int)(i % hd);
  const long long sh = i / hd;
  const int head = (int)(sh % kvh);
  const int t = (int)(sh / kvh);
  pool[kv.offset(seq, slot0 + t, head) + d] = cvt_out<KT>(src[i]);
}

cudaError_t op_kv_fill_random(const KvLayout& kv, void* k, void* v, int kv_dtype, int seq, int n_slots, int kvh, int hd,
                              uint64_t seed, cudaStream_t st) {
  if (kv_dtype == 0)
    kv_fill_random_kernel<float><<<2048, 256, 0, st>>>(kv, (float*)k, (float*)v, seq, n_slots, kvh, hd, seed);
  else
    kv_fill_random_kernel<__nv_bfloat16>
        <<<2048, 256, 0, st>>>(kv, (__nv_bfloat16*)k, (__nv_bfloat16*)v, seq, n_slots, kvh, hd, seed);
  return cudaGetLastError();
}
cudaError_t op_kv_read(const KvLayout& kv, const void* pool, int kv_dtype, int seq, int slot0, int n, int kvh, int hd,
                       float* out, cudaStream_t st) {
  const unsigned int b = blocks_for((long long)n * kvh * hd, 256);
  if (kv_dtype == 0)
    kv_read_kernel<float><<<b, 256, 0, st>>>(kv, (const float*)pool, seq, slot0, n, kvh, hd, out);
  else
    kv_read_kernel<__nv_bfloat16><<<b, 256, 0, st>>>(kv, (const __nv_bfloat16*)pool, seq, slot0, n, kvh, hd, out);
  return cudaGetLastError();
}
cudaError_t op_kv_write(const KvLayout& kv, void* pool, int kv_dtype, int seq, int slot0, int n, int kvh, int hd,
                        const float* src, cudaStream_t st) {
  const unsigned int b = blocks_for((long long)n * kvh * hd, 256);
  if (kv_dtype == 0)
    kv_write_kernel<float><<<b, 256, 0, st>>>(kv, (float*)pool, seq, slot0, n, kvh, hd, src);
  else
    kv_write_kernel<__nv_bfloat16><<<b, 256, 0, st>>>(kv, (__nv_bfloat16*)pool, seq, slot0, n, kvh, hd, src);
  return cudaGetLastError();
}

}  // namespace dllm

// ---- attention without allocation -------------------------------------------------------
// Scratch of dllm_attention_noalloc: every GPU that loads this library keeps these
// bytes until the process exits. Calls share it, so calls that overlap on the GPU
// race; each call's first kernel clears the error word and the ticket counters
// before its attention kernel runs.
namespace dllm {

constexpr size_t kNoAllocScratchBytes = 4u << 20;  // 4 MiB
constexpr int kNoAllocMaxRows = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

__global__ void noalloc_attn_init(RowDesc* rows, unsigned int* arrive, int* err, int t0, int n, int kvh) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) rows[i] = RowDesc{0, t0 + i, t0 + i, 0};
  for (int i = threadIdx.x; i < 2 * n * kvh; i += blockDim.x) arrive[i] = 0u;  // arrivals, finishes
  if (threadIdx.x == 0) *err = 0;
}

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Byte layout of the scratch for n rows and `splits` attention splits. The error
// word sits at offset 0 whatever the shape, so dllm_attention_noalloc_status can
// read it without knowing the last call's arguments.
struct NoAllocLayout {
  size_t err, rows, arrive, part_ml, part_o, total;
};
static NoAllocLayout noalloc_layout(int n, int nq, int kvh, int hd, int splits) {
  NoAllocLayout L;
  size_t off = 0;
  L.err = off;
  off = align256(off + sizeof(int));
  L.rows = off;
  off = align256(off + sizeof(RowDesc) * (size_t)n);
  L.arrive = off;
  off = align256(off + sizeof(unsigned int) * 2 * (size_t)n * kvh);
  L.part_ml = off;
  off = align256(off + sizeof(float) * 2 * (size_t)n * nq * splits);
  L.part_o = off;
  off = align256(off + sizeof(float) * (size_t)n * nq * splits * hd);
  L.total = off;
  return L;
}

}  // namespace dllm

extern "C" int dllm_attention_noalloc(const float* q, const float* kcache, const float* vcache, float* out, int t0,
                                      int n, int num_q_heads, int num_kv_heads, int head_dim, int max_pos,
                                      void* cuda_stream) {
  using namespace dllm;
  if (!q || !kcache || !vcache || !out) return DLLM_EINVAL;
  if (n < 1 || t0 < 0 || max_pos < 1 || (long long)t0 + n > max_pos) return DLLM_EINVAL;
  if (head_dim != 64 && head_dim != 128) return DLLM_EINVAL;
  if (num_kv_heads < 1 || num_q_heads < 1 || num_q_heads % num_kv_heads || num_q_heads / num_kv_heads > kGMax)
    return DLLM_EINVAL;
  if (n > kNoAllocMaxRows) return DLLM_ERANGE;
  // Every call, with the caller's device current: the device address of the static
  // scratch in this context, the SM count, and the attention kernel's shared-memory
  // limit. None of these allocates, and nothing is cached between calls, so the
  // entry point stays valid across a device reset or a change of context.
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DLLM_ECUDA;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return DLLM_ECUDA;
  unsigned char* scratch = static_cast<unsigned char*>(p);
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) return DLLM_ECUDA;
  if (configure_op_kernels() != cudaSuccess) return DLLM_ECUDA;
  int splits = sms / ((n < 8 ? n : 8) * num_kv_heads);
  if (splits > 64) splits = 64;
  if (splits < 1) splits = 1;
  NoAllocLayout L = noalloc_layout(n, num_q_heads, num_kv_heads, head_dim, splits);
  while (L.total > kNoAllocScratchBytes && splits > 1) L = noalloc_layout(n, num_q_heads, num_kv_heads, head_dim, --splits);
  if (L.total > kNoAllocScratchBytes) return DLLM_ERANGE;
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  RowDesc* rows = reinterpret_cast<RowDesc*>(scratch + L.rows);
  unsigned int* arrive = reinterpret_cast<unsigned int*>(scratch + L.arrive);
  int* err = reinterpret_cast<int*>(scratch + L.err);
  noalloc_attn_init<<<1, 256, 0, st>>>(rows, arrive, err, t0, n, num_kv_heads);
  if (cudaGetLastError() != cudaSuccess) return DLLM_ECUDA;
  AttnScratch sc{reinterpret_cast<float*>(scratch + L.part_o), reinterpret_cast<float*>(scratch + L.part_ml), arrive,
                 splits};
  const float scale = (float)(1.0 / std::sqrt((double)head_dim));
  if (op_attention(q, kcache, vcache, out, rows, n, num_q_heads, num_kv_heads, head_dim, max_pos, scale, sc, err, sms,
                   st) != cudaSuccess)
    return DLLM_ECUDA;
  return DLLM_OK;
}

extern "C" int dllm_attention_noalloc_status(void* cuda_stream, int timeout_ms, int* device_error) {
  using namespace dllm;
  if (device_error) *device_error = 0;
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  // bounded wait for the stream (the same polling the ctx calls use)
  const auto t_end = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : 15000);
  for (;;) {
    const cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) return DLLM_ECUDA;
    if (std::chrono::steady_clock::now() > t_end) return DLLM_ETIMEOUT;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_noalloc_scratch, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return DLLM_ECUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return DLLM_ECUDA;
  if (device_error) *device_error = v;
  if (v == 0) return DLLM_OK;
  if (v == kErrBarrier) return DLLM_ETIMEOUT;
  if (v == kErrKvRange) return DLLM_ERANGE;
  return DLLM_EDEVICE;
}
