// stage.cuh — parameters of the persistent stage kernel and its host launcher.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"

namespace dllm {

// Weights and KV pools of one decoder layer (HF tensor names, weights.js:167-182).
struct LayerW {
  const __nv_bfloat16 *ln1, *ln2;         // input_layernorm, post_attention_layernorm
  const __nv_bfloat16 *wq, *wk, *wv, *wo; // self_attn.{q,k,v,o}_proj.weight [out, in]
  const __nv_bfloat16 *bq, *bk, *bv;      // self_attn.{q,k,v}_proj.bias (may be null)
  const __nv_bfloat16 *wg, *wu, *wd;      // mlp.{gate,up,down}_proj.weight
  void* kc;                               // K pool of this layer
  void* vc;                               // V pool of this layer
};

struct StageParams {
  int D, NQ, KVH, HD, I, V, log2_half;
  float eps, scale;
  int n_layers;
  const LayerW* layers;  // device array [n_layers]
  const float* freq;     // [HD/2]
  int m_rows;            // rows of this pass (<= template M)
  RowDesc* rows;         // [m_rows]
  float* h;              // [M][D] residual stream, in/out
  float* q;              // [M][NQ*HD]
  float* att;            // [M][NQ*HD]
  float* mid;            // [M][I]
  float* part_o;         // attention split partials
  float* part_ml;
  unsigned int* arrive;  // [2][M][KVH] attention split arrivals, finishes
  int max_splits;
  KvLayout kv;           // k/v bases unused (per layer in LayerW)
  // optional first phase: h[m] = embed[tokens_in[m]]
  const int32_t* tokens_in;
  const __nv_bfloat16* embed;
  // optional last phase: final norm + LM head + argmax
  const __nv_bfloat16* final_norm;
  const __nv_bfloat16* lm_head;
  unsigned long long* best;  // [M], zero between uses
  int32_t* tokens_out;       // [M]
  float* logits;             // [logits_cap][M][V] or null
  int logits_cap;
  int* step_count;           // steps completed (indexes logits/history), or null
  int32_t* history;          // [hist_cap][M] or null
  int hist_cap;
  int advance_rows;          // pos++ and slot++ for every row at the end
  unsigned int* bar_count;   // grid barrier arrivals, zeroed by launch_stage
  unsigned int* bar_epoch;   // unused
  int* err;
  int pref_bytes;            // per-CTA L2 prefetch budget for the next phase
  unsigned long long* trace; // optional: %globaltimer (ns) at kernel start and after every barrier
  int trace_cap;
  // Pipeline hop over NVLink peer memory (all optional). The pass first waits
  // (bounded) until *in_flag >= in_expect, the previous stage's signal that this
  // pass's input rows (or, on the first stage, tokens) have landed in local
  // memory. At the end it stores its output rows h (or, with a LM head, its
  // tokens) straight into the next stage's receive buffer in that GPU's memory
  // and then releases *out_flag = out_value there.
  const unsigned int* in_flag;
  unsigned int in_expect;
  float* out_h;              // peer [m_rows][D]
  int32_t* out_tok;          // peer [m_rows]
  unsigned int* out_flag;    // peer
  unsigned int out_value;
  // One-row split-K MLP: down_proj sums go into `acc` in fixed point (64-bit
  // atomics) and are folded into the next phase's input instead of a reduction
  // phase. acc must sit right after the barrier counter (bar_count + 4) so one
  // memset clears both before every launch; h2 holds the folded row for o_proj.
  long long* acc;            // [D]
  float* h2;                 // [D]
  int splitk;                // split-K MLP lanes per row group (16 or 32; 0: off), set by launch_stage
  int attn_kv_floats;        // attention K/V ring in shared memory (floats; 0: one round at a time)
  int xs_floats;             // dynamic smem partition
  int part_floats;
};

// Dynamic shared memory the stage kernel is launched with.
constexpr int kStageXsFloats = 32768;    // 128 KB of staged activations
constexpr int kStagePartFloats = 16384;  // 64 KB of segment partials
constexpr int kStageSmallPartFloats = 4096;  // 16 KB: the one-row split-K partition
constexpr size_t kStageSmemBytes = (size_t)(kStageXsFloats + kStagePartFloats) * sizeof(float);
// Attention K/V ring: 144 KB, i.e. up to 3-4 rounds in flight while one is
// computed, for stages whose attention items can hold more than kAttnRingSlots
// slots on average (max_pos * KV heads / SMs): long items make attention a large
// share of the pass; short ones (a round or two each) keep one round at a time
// and leave the shared memory to L1, which the weight streaming needs more.
constexpr int kAttnRingSlots = 256;
constexpr int kAttnKvLongFloats = 36864;

// Launches stage_kernel<KT, HD, M> with M the smallest of {1,2,4,8} >= m_rows,
// one CTA per SM, cooperative (all CTAs resident). kv_dtype: 0 fp32, 1 bf16.
cudaError_t launch_stage(const StageParams& p, int kv_dtype, int grid, cudaStream_t st);
// Raise the dynamic shared-memory limit of every stage kernel instantiation on
// the current device (call once per device, before any launch or capture).
cudaError_t configure_stage_kernels();

}  // namespace dllm
