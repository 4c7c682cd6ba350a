// stage_impl.cuh — the persistent decode-step kernel of one pipeline stage
// (template; instantiated per KV dtype in stage_f32.cu and stage_bf16.cu).
//
// One launch runs [embed] -> layers [start, end) -> [final norm + LM head +
// argmax] for up to 8 rows (sequences of a micro-batch, or prompt tokens of a
// prefill chunk). CTAs are one per SM and co-resident (cooperative launch);
// phases are separated by grid_barrier(). See kernels.cuh for the phases.
#pragma once
#include "kernels.cuh"
#include "stage.cuh"


namespace dllm {

DLLM_DEV AttnArgs attn_args(const StageParams& P, const LayerW& L) {
  return AttnArgs{P.q, P.att, L.kc, L.vc, P.kv, P.rows, P.m_rows, P.NQ, P.KVH, P.scale, P.max_splits,
                  P.part_o, P.part_ml, P.arrive, P.err, P.attn_kv_floats};
}

// SKL: lanes per row group of the split-K down projection (16: column slices of
// up to 128, 32: up to 256). RING: attention K/V staged through the multi-round
// ring (P.attn_kv_floats > 0, long contexts). Separate instantiations, so each
// kernel carries one variant of each.
template <typename KT, int HD, int M, int SKL = 16, bool RING = false>
__global__ void __launch_bounds__(kThreads, 1) stage_kernel(const StageParams P) {
  extern __shared__ __align__(16) float smem[];
  __shared__ float red[32];
  __shared__ unsigned long long sbest[kMaxRows];
  __shared__ AttnEarly s_early;
  const int cta = blockIdx.x, ncta = gridDim.x;
  const PhaseSmem sm{smem, P.xs_floats, smem + P.xs_floats, P.part_floats, red};
  NoState ns;
  const int D = P.D, QD = P.NQ * P.HD;
  const int qkv_units = (P.NQ + 2 * P.KVH) * (P.HD >> 1);
  int tr = 0;  // trace slot: CTA 0 stamps the global timer at start and after every barrier
  auto trace = [&]() {
    if (P.trace && cta == 0 && threadIdx.x == 0 && tr < P.trace_cap) P.trace[tr] = global_timer_ns();
    ++tr;
  };
  trace();

  // Pipeline hop: wait (bounded) for the previous stage's rows or tokens.
  if (P.in_flag && !wait_peer_flag(P.in_flag, P.in_expect, P.err)) return;

  // Weights never depend on earlier phases: warm L2 for the first matvec.
  if (P.n_layers > 0) {
    const LayerW L0 = P.layers[0];
    EpiQKV<KT> e0{L0.wq, L0.wk, L0.wv, nullptr, nullptr, nullptr, P.NQ, P.KVH, P.HD, P.log2_half};
    prefetch_phase(e0, D, qkv_units, cta, ncta, P.pref_bytes);
  }

  if (P.tokens_in) {
    // embedTokens (pipeline.js:121-128): bf16 row -> fp32, 8 elements per thread.
    const int chunks = D >> 3;
    const int c0 = (int)(((long long)cta * chunks) / ncta), c1 = (int)(((long long)(cta + 1) * chunks) / ncta);
    for (int m = 0; m < P.m_rows; ++m) {
      int tok = P.tokens_in[m];
      if (tok < 0 || tok >= P.V) {
        if (threadIdx.x == 0) atomicExch(P.err, kErrToken);
        tok = 0;
      }
      const uint4* src = reinterpret_cast<const uint4*>(P.embed + (size_t)tok * D);
      for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
        const uint4 w = __ldg(src + c);
        float4* dst = reinterpret_cast<float4*>(P.h + (size_t)m * D) + 2 * c;
        dst[0] = make_float4(bf16_lo(w.x), bf16_hi(w.x), bf16_lo(w.y), bf16_hi(w.y));
        dst[1] = make_float4(bf16_lo(w.z), bf16_hi(w.z), bf16_lo(w.w), bf16_hi(w.w));
      }
    }
    if (!grid_barrier(P.bar_count, P.err)) return;
    trace();
  }

  // One row with the split-K MLP: the down_proj sums of layer l wait in P.acc
  // (fixed point) until layer l+1's QKV phase folds them into its input; the
  // fold of this CTA's share also goes to P.h2, the residual o_proj adds to.
  const bool fused = M == 1 && P.splitk;
  for (int l = 0; l < P.n_layers; ++l) {
    const LayerW L = P.layers[l];
    const bool pending = fused && l > 0;  // layer l-1's down_proj sums
    // ---- QKV: rmsnorm -> q,k,v matmul -> addBias -> ropeQ/ropeK -> appendKv (pipeline.js:55-64)
    const EpiQKV<KT> eq{L.wq, L.wk, L.wv, L.bq, L.bk, L.bv, P.NQ, P.KVH, P.HD, P.log2_half, P.freq, P.q,
                        reinterpret_cast<KT*>(L.kc), reinterpret_cast<KT*>(L.vc), P.kv, P.rows, P.err};
    // (fused: the input is h + the pending sums; this CTA's share of it goes to h2)
    gemv_phase<EpiQKV<KT>, M>(eq, GemvIn{P.h, D, P.m_rows, L.ln1, P.eps, pending ? P.acc : nullptr,
                                         fused ? P.h2 : nullptr},
                              qkv_units, sm, cta, ncta, ns);
    // one row, one round at a time: this CTA's first attention rows (all but the
    // slot this pass appends) into shared memory, landing across the barrier
    // (measured: attention 11.9 -> 10.6 us per layer at 7B / 2k; the ring variant
    // already overlaps its first round and lost 1 % with it)
    int early = 0;
    if (M == 1 && !RING) {
      if (l == 0) attn_early_plan<KT, HD, RING>(attn_args(P, L), cta, ncta, &s_early);
      early = attn_early_issue<KT, HD>(s_early, L.kc, L.vc, P.kv.row_stride, smem);
    }
    const EpiResidual eo{L.wo, P.h, D, fused ? P.h2 : nullptr};
    prefetch_phase(eo, QD, D, cta, ncta, 2 * P.pref_bytes);
    if (!grid_barrier(P.bar_count, P.err)) return;
    trace();

    // ---- attention over slots [0, slot] (pipeline.js:65)
    if (pending) zero_share(P.acc, D, cta, ncta);  // every CTA has read the sums
    attn_phase<KT, HD, RING>(attn_args(P, L), smem, cta, ncta, early);
    if (!grid_barrier(P.bar_count, P.err)) return;
    trace();

    // ---- o_proj + residual (pipeline.js:66-67)
    gemv_phase<EpiResidual, M>(eo, GemvIn{P.att, QD, P.m_rows, nullptr, 0.f}, D, sm, cta, ncta, ns);
    const EpiSiluGate eg{L.wg, L.wu, P.mid, P.I};
    prefetch_phase(eg, D, P.I, cta, ncta, P.pref_bytes, fused ? 8 : 1);  // the MLP's unit ranges
    if (!grid_barrier(P.bar_count, P.err)) return;
    trace();

    // ---- rmsnorm -> gate, up -> siluMul (pipeline.js:69-72)
    if (fused) {
      // Split-K MLP (one row): each CTA keeps its 8-aligned slice of SiLU(gate)*up
      // in shared memory and multiplies it straight into its column slice of
      // down_proj for all rows (no barrier, no staging of the whole vector); the
      // per-CTA partials go into P.acc, summed by integer atomics.
      int k0, k1;
      unit_range(P.I, cta, ncta, 8, k0, k1);
      float* slice = smem + P.xs_floats - 256;
      EpiSiluGate eg{L.wg, L.wu, P.mid, P.I, slice, k0};
      const PhaseSmem sm_g{smem, P.xs_floats - 256, sm.part, sm.part_floats, red};  // staging stops short of the slice
      gemv_phase<EpiSiluGate, M>(eg, GemvIn{P.h, D, P.m_rows, L.ln2, P.eps}, P.I, sm_g, cta, ncta, ns, 8);
      // ---- down_proj (pipeline.js:73), this CTA's K-slice; + residual (:74) when folded
      down_partial<SKL>(L.wd, D, P.I, k0, k1 - k0, slice, P.acc);
    } else {
      gemv_phase<EpiSiluGate, M>(eg, GemvIn{P.h, D, P.m_rows, L.ln2, P.eps}, P.I, sm, cta, ncta, ns);
      const EpiResidual ed{L.wd, P.h, D};
      prefetch_phase(ed, P.I, D, cta, ncta, P.pref_bytes);
      if (!grid_barrier(P.bar_count, P.err)) return;
      trace();

      // ---- down_proj + residual (pipeline.js:73-74)
      gemv_phase<EpiResidual, M>(ed, GemvIn{P.mid, P.I, P.m_rows, nullptr, 0.f}, D, sm, cta, ncta, ns);
    }
    // the next layer's first q|k|v rows (or the LM head) into L2 across the barrier
    if (l + 1 < P.n_layers) {
      const LayerW Ln = P.layers[l + 1];
      const EpiQKV<KT> en{Ln.wq, Ln.wk, Ln.wv, nullptr, nullptr, nullptr, P.NQ, P.KVH, P.HD, P.log2_half};
      prefetch_phase(en, D, qkv_units, cta, ncta, P.pref_bytes);
    } else if (P.lm_head) {
      const EpiArgmax<M> ep{P.lm_head, P.V, nullptr};
      prefetch_phase(ep, D, P.V, cta, ncta, P.pref_bytes);
    }
    if (!grid_barrier(P.bar_count, P.err)) return;
    trace();
  }
  if (fused && P.n_layers > 0) {
    // ---- the last layer's down_proj sums + residual (pipeline.js:73-74) into h
    fold_residual(P.h, P.acc, P.h, D, cta, ncta, true);
    if (!grid_barrier(P.bar_count, P.err)) return;
    trace();
  }

  if (P.out_h) {
    // ---- hop (pipeline.js:226-253): this CTA's share of the output rows straight
    // into the next stage's receive buffer over NVLink, then one release of its flag
    const int n4 = (P.m_rows * D) >> 2;
    const int v0 = (int)(((long long)cta * n4) / ncta), v1 = (int)(((long long)(cta + 1) * n4) / ncta);
    const float4* src = reinterpret_cast<const float4*>(P.h);
    float4* dst = reinterpret_cast<float4*>(P.out_h);
    for (int i = v0 + threadIdx.x; i < v1; i += blockDim.x) dst[i] = __ldcg(src + i);
    __threadfence_system();
    if (!grid_barrier(P.bar_count, P.err)) return;
    if (cta == 0 && threadIdx.x == 0) {
      __threadfence_system();
      st_release_sys_u32(P.out_flag, P.out_value);
    }
  }

  if (P.lm_head) {
    // ---- sampleLast: rmsnorm(model.norm) -> LM head -> argmax (pipeline.js:147-169)
    float* logits = nullptr;
    if (P.logits) {
      const int step = P.step_count ? *P.step_count : 0;
      if (step < P.logits_cap) logits = P.logits + (size_t)step * M * P.V;
    }
    const EpiArgmax<M> ea{P.lm_head, P.V, logits};
    typename EpiArgmax<M>::State st;
#pragma unroll
    for (int i = 0; i < M; ++i) st.key[i] = 0ull;
    gemv_phase<EpiArgmax<M>, M>(ea, GemvIn{P.h, D, P.m_rows, P.final_norm, P.eps}, P.V, sm, cta, ncta, st);
    if (threadIdx.x < M) sbest[threadIdx.x] = 0ull;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < M; ++i)
      if (st.key[i]) atomicMax(&sbest[i], st.key[i]);
    __syncthreads();
    if (threadIdx.x < P.m_rows && sbest[threadIdx.x]) atomicMax(&P.best[threadIdx.x], sbest[threadIdx.x]);
    if (!grid_barrier(P.bar_count, P.err)) return;
    trace();
    if (cta == 0) {
      if (threadIdx.x < P.m_rows) {
        const int m = threadIdx.x;
        const unsigned long long k = atomicExch(&P.best[m], 0ull);
        const int tok = argmax_key_index(k);
        P.tokens_out[m] = tok;
        if (P.history) {
          const int step = P.step_count ? *P.step_count : 0;
          if (step < P.hist_cap) P.history[(size_t)step * P.m_rows + m] = tok;
        }
        if (P.advance_rows) {
          P.rows[m].pos += 1;
          P.rows[m].slot += 1;
        }
        if (P.out_tok) P.out_tok[m] = tok;  // the tokens go back to the first stage
      }
      if (P.out_tok) __threadfence_system();
      __syncthreads();
      if (threadIdx.x == 0 && P.step_count) atomicAdd(P.step_count, 1);
      if (threadIdx.x == 0 && P.out_tok) st_release_sys_u32(P.out_flag, P.out_value);
    }
  } else if (P.advance_rows && cta == 0 && threadIdx.x < P.m_rows) {
    P.rows[threadIdx.x].pos += 1;
    P.rows[threadIdx.x].slot += 1;
  }
}

template <typename KT, int HD, int M, int SKL = 16, bool RING = false>
static cudaError_t launch_one(const StageParams& p0, int grid, cudaStream_t st) {
  auto fn = stage_kernel<KT, HD, M, SKL, RING>;
  StageParams p = p0;
  if (M == 1 && p.splitk) {
    // One row with the split-K MLP: no phase stages more than a D- or
    // NQ*HD-long activation (mid is never staged), so a small shared-memory
    // partition suffices and the rest of the SM's 256 KB stays L1, which the
    // in-flight weight loads need.
    const int K = p.D > p.NQ * p.HD ? p.D : p.NQ * p.HD;
    int xs = ((K + 4095) / 4096) * 4096 + 256;  // staged x + the SiLU(gate)*up slice
    const int part = kStageSmallPartFloats;
    const int attn = attn_smem_floats<KT, HD>(RING ? p.attn_kv_floats : 0);
    if (xs + part < attn) xs = attn - part;
    xs = (xs + 3) & ~3;  // 16-byte aligned partial and slice areas
    if (xs + part < kStageXsFloats + kStagePartFloats) {
      p.xs_floats = xs;
      p.part_floats = part;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)(p.xs_floats + p.part_floats) * sizeof(float);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, p);
}

template <typename KT, int HD, bool RING>
static cudaError_t launch_m_ring(const StageParams& p, int grid, cudaStream_t st) {
  if (p.m_rows <= 1) {
    if constexpr (HD == 128)
      if (p.splitk == 32) return launch_one<KT, HD, 1, 32, RING>(p, grid, st);
    return launch_one<KT, HD, 1, 16, RING>(p, grid, st);
  }
  if (p.m_rows <= 2) return launch_one<KT, HD, 2, 16, RING>(p, grid, st);
  if (p.m_rows <= 4) return launch_one<KT, HD, 4, 16, RING>(p, grid, st);
  return launch_one<KT, HD, 8, 16, RING>(p, grid, st);
}

template <typename KT, int HD>
static cudaError_t launch_m(const StageParams& p, int grid, cudaStream_t st) {
  if (p.attn_kv_floats > 0) return launch_m_ring<KT, HD, true>(p, grid, st);
  return launch_m_ring<KT, HD, false>(p, grid, st);
}

template <typename KT, int HD, bool RING>
static cudaError_t configure_ring() {
  const int bytes = (int)kStageSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(stage_kernel<KT, HD, 1, 16, RING>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(stage_kernel<KT, HD, 2, 16, RING>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(stage_kernel<KT, HD, 4, 16, RING>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(stage_kernel<KT, HD, 8, 16, RING>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if constexpr (HD == 128)
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(stage_kernel<KT, HD, 1, 32, RING>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  return e;
}

template <typename KT, int HD>
static cudaError_t configure_hd() {
  cudaError_t e = configure_ring<KT, HD, false>();
  if (e == cudaSuccess) e = configure_ring<KT, HD, true>();
  return e;
}

}  // namespace dllm
