// kernels.cuh — device code of the decode path (sm_100a).
//
// The decode step of a pipeline stage runs as ONE persistent kernel
// (stage_kernel in stage.cu): one CTA per SM, all CTAs co-resident (cooperative
// launch), phases separated by a bounded grid barrier. Per decoder layer the
// phases are
//   QKV   : RMSNorm prologue + fused q|k|v matvec + bias + RoPE + KV-slot write
//   ATTN  : split-K GQA decode attention over the paged KV cache + merge
//   O     : o_proj matvec + residual add
//   GATEUP: RMSNorm prologue + gate|up matvec + SiLU(gate)*up
//   DOWN  : down_proj matvec + residual add
// which is the op order of Stage.forward (pipeline.js:52-75). Optional first
// and last phases gather the token embedding (pipeline.js:121-128) and run the
// final norm + LM head + greedy argmax (pipeline.js:141-174).
//
// Every matvec phase streams bf16 weights with 16-byte loads, accumulates in
// fp32, splits each row into K-segments spread over the CTA's 16 warps, and
// reduces the segment partials in shared memory in a fixed order, so results do
// not depend on scheduling. Work is split between CTAs by contiguous, equal
// unit ranges (a unit is one row, or the row pair an epilogue needs together).
// Before arriving at a barrier each CTA asks the TMA unit to prefetch the
// weights of its next phase into L2, so HBM keeps streaming through the barrier.
#pragma once

#include "common.cuh"

namespace dllm {

constexpr int kThreads = 512;            // 16 warps per CTA, one CTA per SM
constexpr int kWarps = kThreads / 32;
// 16-byte weight vectors each lane keeps in flight per task: 16 for single-row
// units, 8 per row for row pairs (16 either way), i.e. 8 KB per warp.
template <int R>
struct Seg {
  static constexpr int U = 16 / R;
  static constexpr int Chunks = 32 * U;  // 16-byte chunks per task segment
  static constexpr int Elems = Chunks * 8;
};
constexpr int kGMax = 8;                 // max query heads per KV head
constexpr int kAttnMaxSplits = 64;       // max attention splits per (row, kv head)
constexpr int kMaxRows = 8;              // max rows (sequences or prompt tokens) per pass

// ---- block helpers ---------------------------------------------------------------
DLLM_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < nw; ++w) t += red[w];  // same fixed order in every thread
  return t;
}

DLLM_DEV unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// GPU-scope atomic add that releases this thread's earlier writes (and, through a
// preceding __syncthreads, the CTA's) and acquires the writes released to it.
DLLM_DEV unsigned int atom_add_acq_rel_u32(unsigned int* p, unsigned int v) {
  unsigned int r;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(r) : "l"(p), "r"(v) : "memory");
  return r;
}
DLLM_DEV void st_release_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid-wide barrier for a cooperative (all-CTAs-resident) launch. The counter
// only grows within a launch (the launcher zeroes it before every launch), so
// barrier k completes when it reaches k * gridDim.x. After __syncthreads one
// thread per CTA arrives with a GPU-scope acq_rel atomic add (publishing the
// CTA's writes); the old value gives this barrier's target; the CTA whose
// arrival reaches it is released at once, the others poll with acquire loads.
// One round trip after the last arrival instead of a separate reset and
// release. The wait is bounded: after ~2^33 SM cycles (seconds) the CTA
// records an error and the caller leaves the kernel; the host reads the flag.
constexpr long long kBarrierTimeoutCycles = 1ll << 33;
constexpr int kErrBarrier = 2;
constexpr int kErrKvRange = 3;
constexpr int kErrToken = 4;

DLLM_DEV bool grid_barrier(unsigned int* count, int* err) {
  __syncthreads();
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const unsigned int n = gridDim.x;
    const unsigned int old = atom_add_acq_rel_u32(count, 1u);
    const unsigned int target = (old / n + 1u) * n;
    int ok = 1;
    if (old + 1u != target) {
      const long long t0 = clock64();
      while ((int)(ld_acquire_u32(count) - target) < 0) {
        if (clock64() - t0 > kBarrierTimeoutCycles) {
          atomicExch(err, kErrBarrier);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// System-scope (peer GPU) flag helpers for the pipeline hop over NVLink.
DLLM_DEV unsigned int ld_acquire_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
DLLM_DEV void st_release_sys_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
constexpr int kErrPeerWait = 6;

// Bounded wait of the whole CTA until *flag >= expect (written by another GPU).
DLLM_DEV bool wait_peer_flag(const unsigned int* flag, unsigned int expect, int* err) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    const long long t0 = clock64();
    while ((int)(ld_acquire_sys_u32(flag) - expect) < 0) {
      if (clock64() - t0 > kBarrierTimeoutCycles) {
        atomicExch(err, kErrPeerWait);
        ok = 0;
        break;
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// ---- activation staging (RMSNorm prologue, kernels.js:46-63) -----------------------
// Per row: ss = sum(x^2), scale = 1 / sqrt(ss / K + eps), x' = (x * scale) * g.
struct GemvIn {
  const float* x;               // [m_rows][K], written earlier in the same kernel: L2 reads
  int K;
  int m_rows;                   // valid rows (<= M)
  const __nv_bfloat16* norm_w;  // RMSNorm gamma [K] or null
  float eps;
  const long long* acc = nullptr;  // one row: pending fixed-point down_proj sums [K] added to x
  float* save = nullptr;           // optional [m_rows][K]: this CTA's share of the (summed) input rows
};

// ---- fixed-point residual sums (one-row split-K MLP) --------------------------------
// Each CTA's down_proj partial is rounded to a multiple of 2^-32 and added into a
// 64-bit integer accumulator with an atomic: integer addition is associative, so
// the sum is the same whatever order the 148 CTAs arrive in (deterministic), and
// it is exact up to the one rounding per partial (<= 2^-33 each). Range: partials
// below 2^31 in magnitude.
constexpr float kFixScale = 4294967296.0f;            // 2^32
constexpr float kFixInv = 2.3283064365386963e-10f;    // 2^-32
DLLM_DEV long long f32_to_fix(float v) { return __float2ll_rn(v * kFixScale); }
DLLM_DEV float fix_to_f32(long long a) { return __ll2float_rn(a) * kFixInv; }

// Elements [e, e+4) of row m of the phase input: x plus, when the input carries
// them, the pending fixed-point sums (e a multiple of 4).
DLLM_DEV float4 load_in4(const GemvIn& in, int m, int e) {
  float4 v = __ldcg(reinterpret_cast<const float4*>(in.x + (size_t)m * in.K + e));
  if (in.acc) {
    const longlong2* a = reinterpret_cast<const longlong2*>(in.acc + e);
    const longlong2 a0 = __ldcg(a), a1 = __ldcg(a + 1);
    v.x = __fadd_rn(v.x, fix_to_f32(a0.x));
    v.y = __fadd_rn(v.y, fix_to_f32(a0.y));
    v.z = __fadd_rn(v.z, fix_to_f32(a1.x));
    v.w = __fadd_rn(v.w, fix_to_f32(a1.y));
  }
  return v;
}

template <int M>
DLLM_DEV void row_scales(const GemvIn& in, float* red, float (&scale)[M]) {
#pragma unroll
  for (int m = 0; m < M; ++m) {
    scale[m] = 1.f;
    if (!in.norm_w || m >= in.m_rows) continue;
    float ss = 0.f;
    for (int i = threadIdx.x; i < (in.K >> 2); i += blockDim.x) {
      const float4 v = load_in4(in, m, 4 * i);
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
    const float tot = block_sum(ss, red);
    scale[m] = 1.0f / sqrtf(tot / (float)in.K + in.eps);
  }
}

// Stage columns [k0, k1) of every row into xs[m * xstride + (k - k0)]. With
// in.save, the elements of this CTA's share of the rows (K split evenly over the
// CTAs) are also written there, before normalisation.
template <int M>
DLLM_DEV void stage_x_block(const GemvIn& in, const float (&scale)[M], float* xs, int xstride, int k0, int k1,
                            int cta, int ncta) {
  const int w4 = (k1 - k0) >> 2;
  const int v0 = (int)(((long long)cta * in.K) / ncta), v1 = (int)(((long long)(cta + 1) * in.K) / ncta);
#pragma unroll
  for (int m = 0; m < M; ++m) {
    float4* dst = reinterpret_cast<float4*>(xs + (size_t)m * xstride);
    if (m >= in.m_rows) {
      for (int i = threadIdx.x; i < w4; i += blockDim.x) dst[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      continue;
    }
    const uint2* g = in.norm_w ? reinterpret_cast<const uint2*>(in.norm_w + k0) : nullptr;
    for (int i = threadIdx.x; i < w4; i += blockDim.x) {
      float4 v = load_in4(in, m, k0 + 4 * i);
      const int e0 = k0 + 4 * i;
      if (in.save && e0 + 3 >= v0 && e0 < v1) {
        float* sv = in.save + (size_t)m * in.K;
        const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (e0 + q >= v0 && e0 + q < v1) sv[e0 + q] = e[q];
      }
      if (g) {
        const uint2 gg = __ldg(g + i);
        v.x = (v.x * scale[m]) * bf16_lo(gg.x);
        v.y = (v.y * scale[m]) * bf16_hi(gg.x);
        v.z = (v.z * scale[m]) * bf16_lo(gg.y);
        v.w = (v.w * scale[m]) * bf16_hi(gg.y);
      }
      dst[i] = v;
    }
  }
  __syncthreads();
}

// in.save for a CTA without units in the phase: this CTA's share of every row.
DLLM_DEV void save_share(const GemvIn& in, int cta, int ncta) {
  const int v0 = (int)(((long long)cta * in.K) / ncta), v1 = (int)(((long long)(cta + 1) * in.K) / ncta);
  for (int m = 0; m < in.m_rows; ++m)
    for (int j = v0 + threadIdx.x; j < v1; j += blockDim.x) {
      float v = __ldcg(in.x + (size_t)m * in.K + j);
      if (in.acc) v = __fadd_rn(v, fix_to_f32(__ldcg(in.acc + j)));
      in.save[(size_t)m * in.K + j] = v;
    }
}

// Shared-memory budget a phase may use (floats).
struct PhaseSmem {
  float* xs;
  int xs_floats;
  float* part;
  int part_floats;
  float* red;  // >= 32 floats
};

// ---- matvec phase ----------------------------------------------------------------
// CTA `cta` of `ncta` owns units [u0, u1): equal contiguous ranges, or ranges
// whose bounds are multiples of `align` (the split-K MLP needs 16-byte aligned
// column slices of down_proj).
DLLM_DEV void unit_range(int units, int cta, int ncta, int align, int& u0, int& u1) {
  u0 = (int)(((long long)cta * units) / ncta);
  u1 = (int)(((long long)(cta + 1) * units) / ncta);
  if (align > 1) {
    u0 = u0 / align * align;
    u1 = cta + 1 == ncta ? units : u1 / align * align;
  }
}

// Epi supplies: R (rows per unit), unit_rows(u, K, p[R]) and unit(u, m, a[R], st).
// CTA `cta` of `ncta` owns units [cta*units/ncta, (cta+1)*units/ncta).
template <class Epi, int M>
DLLM_DEV void gemv_phase(const Epi& epi, const GemvIn& in, int units, const PhaseSmem& sm, int cta, int ncta,
                         typename Epi::State& st, int align = 1) {
  constexpr int R = Epi::R;
  constexpr int kU = Seg<R>::U;
  constexpr int kSegChunks = Seg<R>::Chunks;
  constexpr int kSegElems = Seg<R>::Elems;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int K = in.K, Kc = K >> 3;
  int u0, u1;
  unit_range(units, cta, ncta, align, u0, u1);
  const int nu = u1 - u0;
  const int nseg = (Kc + kSegChunks - 1) / kSegChunks;
  int seg_per_blk = sm.xs_floats / (M * kSegElems);
  if (seg_per_blk < 1) seg_per_blk = 1;
  if (seg_per_blk > nseg) seg_per_blk = nseg;
  const int nblk = (nseg + seg_per_blk - 1) / seg_per_blk;
  const int xstride = seg_per_blk * kSegElems;
  int ub = sm.part_floats / (nseg * R * M);
  if (ub < 1) ub = 1;

  float scale[M];
  row_scales<M>(in, sm.red, scale);
  if (nu <= 0) {
    if (in.save) save_share(in, cta, ncta);  // no staging here: write the share from L2
    return;
  }

  for (int b0 = 0; b0 < nu; b0 += ub) {
    const int nb = min(ub, nu - b0);
    for (int blk = 0; blk < nblk; ++blk) {
      const int s0 = blk * seg_per_blk, s1 = min(nseg, s0 + seg_per_blk);
      const int k0 = s0 * kSegElems, k1 = min(K, s1 * kSegElems);
      if (nblk > 1 || b0 == 0) {
        __syncthreads();  // previous readers of xs are done
        stage_x_block<M>(in, scale, sm.xs, xstride, k0, k1, cta, ncta);
      }
      const int nsb = s1 - s0;
      const int ntask = nb * nsb;
      for (int t = warp; t < ntask; t += nwarps) {
        const int ul = t / nsb, seg = s0 + (t - ul * nsb);
        const uint4* p[R];
        epi.unit_rows(u0 + b0 + ul, K, p);
        const int cbase = seg * kSegChunks + lane;
        uint4 w[kU][R];
#pragma unroll
        for (int i = 0; i < kU; ++i) {
          const int ci = cbase + 32 * i;
#pragma unroll
          for (int r = 0; r < R; ++r) {
            if (ci < Kc) w[i][r] = ld_stream16(p[r] + ci);
            else w[i][r] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        float acc[R][M];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
#pragma unroll
        for (int i = 0; i < kU; ++i) {
          const int ci = cbase + 32 * i;
          if (ci < Kc) {
            const int xo = ci * 8 - k0;
#pragma unroll
            for (int m = 0; m < M; ++m) {
              const float4* xr = reinterpret_cast<const float4*>(sm.xs + (size_t)m * xstride + xo);
              const float4 a = xr[0], b = xr[1];
#pragma unroll
              for (int r = 0; r < R; ++r) acc[r][m] = dot8(w[i][r], a, b, acc[r][m]);
            }
          }
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int m = 0; m < M; ++m) acc[r][m] = warp_sum(acc[r][m]);
        if (lane == 0) {
          float* dst = sm.part + ((size_t)ul * nseg + seg) * (R * M);
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int m = 0; m < M; ++m) dst[r * M + m] = acc[r][m];
        }
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nb * M; i += blockDim.x) {
      const int ul = i / M, m = i - ul * M;
      if (m >= in.m_rows) continue;
      float a[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float s = 0.f;
        for (int seg = 0; seg < nseg; ++seg) s += sm.part[((size_t)ul * nseg + seg) * (R * M) + r * M + m];
        a[r] = s;
      }
      epi.unit(u0 + b0 + ul, m, a, st);
    }
    __syncthreads();
  }
}

// Ask the TMA unit to pull rows of this CTA's units of a future matvec phase
// into L2: the units the phase will give CTA `cta` (the same unit_range split,
// `align` included), in the order the phase reads them, starting `skip` bytes
// into the CTA's share and covering up to `budget` bytes (whole units, at least
// one when budget > 0). Issued by warp 0; the copies run in the background.
template <class Epi>
DLLM_DEV void prefetch_phase(const Epi& epi, int K, int units, int cta, int ncta, int budget, int align = 1,
                             int skip = 0) {
  if (budget <= 0 || (threadIdx.x >> 5) != 0) return;
  const int lane = threadIdx.x & 31;
  int u0, u1;
  unit_range(units, cta, ncta, align, u0, u1);
  const int row_bytes = K * 2;
  const int unit_bytes = row_bytes * Epi::R;
  const int ubeg = u0 + skip / unit_bytes;
  const int uend = min(u1, ubeg + max(1, budget / unit_bytes));
  for (int u = ubeg + lane; u < uend; u += 32) {
    const uint4* p[Epi::R];
    epi.unit_rows(u, K, p);
#pragma unroll
    for (int r = 0; r < Epi::R; ++r) prefetch_l2_bulk(p[r], (uint32_t)row_bytes);
  }
}

// ---- epilogues ---------------------------------------------------------------------
struct NoState {};

// out[m][j] = x[m] . W[j]  (ctx.matmul, kernels.js:26-44)
struct EpiStore {
  static constexpr int R = 1;
  using State = NoState;
  const __nv_bfloat16* w;
  float* y;
  int N;
  DLLM_DEV void unit_rows(int u, int K, const uint4** p) const {
    p[0] = reinterpret_cast<const uint4*>(w + (size_t)u * K);
  }
  DLLM_DEV void unit(int u, int m, const float* a, State&) const { y[(size_t)m * N + u] = a[0]; }
};

// h[m][j] = src[m][j] + x[m] . W[j]  (o_proj / down_proj then ctx.add, pipeline.js:66-67,73-74);
// src is h itself unless the residual was folded into a separate buffer.
struct EpiResidual {
  static constexpr int R = 1;
  using State = NoState;
  const __nv_bfloat16* w;
  float* h;
  int N;
  const float* src = nullptr;
  DLLM_DEV void unit_rows(int u, int K, const uint4** p) const {
    p[0] = reinterpret_cast<const uint4*>(w + (size_t)u * K);
  }
  DLLM_DEV void unit(int u, int m, const float* a, State&) const {
    const size_t i = (size_t)m * N + u;
    h[i] = __fadd_rn(__ldcg((src ? src : h) + i), a[0]);
  }
};

// mid[m][j] = silu(x.Wg[j]) * (x.Wu[j])  (gate/up matmuls + ctx.siluMul, pipeline.js:70-72;
// SILUMUL kernels.js:134-145: a / (1 + exp(-a)) * b)
struct EpiSiluGate {
  static constexpr int R = 2;
  using State = NoState;
  const __nv_bfloat16* wg;
  const __nv_bfloat16* wu;
  float* out;
  int N;
  float* slice = nullptr;  // optional (one row): this CTA's values, slice[u - slice_base], in shared memory
  int slice_base = 0;
  DLLM_DEV void unit_rows(int u, int K, const uint4** p) const {
    p[0] = reinterpret_cast<const uint4*>(wg + (size_t)u * K);
    p[1] = reinterpret_cast<const uint4*>(wu + (size_t)u * K);
  }
  DLLM_DEV void unit(int u, int m, const float* a, State&) const {
    const float g = a[0];
    const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
    const float v = __fmul_rn(silu, a[1]);
    out[(size_t)m * N + u] = v;
    if (slice) slice[u - slice_base] = v;
  }
};

// q|k|v projection of one rotate-half pair (rows j and j + HD/2 of one head),
// + bias (ctx.addBias, kernels.js:148-159), + RoPE for q and k (ROPE,
// kernels.js:66-83), then q -> q buffer and k, v -> KV slot `slot` of the row's
// sequence (Stage.appendKv, pipeline.js:80-87).
template <typename KT>
struct EpiQKV {
  static constexpr int R = 2;
  using State = NoState;
  const __nv_bfloat16 *wq, *wk, *wv;
  const __nv_bfloat16 *bq, *bk, *bv;
  int NQ, KVH, HD, log2_half;
  const float* freq;  // [HD/2] RoPE inverse frequencies (f32)
  float* q_out;       // [m][NQ*HD]
  KT* kc;             // this layer's K pool
  KT* vc;             // this layer's V pool
  KvLayout kv;
  const RowDesc* rows;
  int* err;

  DLLM_DEV void locate(int u, int& kind, int& lh, int& half) const {
    const int hh = u >> log2_half;
    half = u & ((1 << log2_half) - 1);
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
  }
  DLLM_DEV void unit_rows(int u, int K, const uint4** p) const {
    int kind, lh, half;
    locate(u, kind, lh, half);
    const __nv_bfloat16* w = kind == 0 ? wq : (kind == 1 ? wk : wv);
    const size_t r0 = (size_t)lh * HD + half;
    p[0] = reinterpret_cast<const uint4*>(w + r0 * K);
    p[1] = reinterpret_cast<const uint4*>(w + (r0 + (HD >> 1)) * K);
  }
  DLLM_DEV void unit(int u, int m, const float* a, State&) const {
    int kind, lh, half;
    locate(u, kind, lh, half);
    const int j0 = lh * HD + half, j1 = j0 + (HD >> 1);
    float x1 = a[0], x2 = a[1];
    const __nv_bfloat16* b = kind == 0 ? bq : (kind == 1 ? bk : bv);
    if (b) {
      x1 = __fadd_rn(x1, bf16_to_f32(b[j0]));
      x2 = __fadd_rn(x2, bf16_to_f32(b[j1]));
    }
    const RowDesc rd = rows[m];
    if (kind < 2) {
      const float ang = __fmul_rn((float)rd.pos, freq[half]);
      float s, c;
      sincosf(ang, &s, &c);
      const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
      const float o2 = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
      x1 = o1;
      x2 = o2;
    }
    if (kind == 0) {
      float* q = q_out + (size_t)m * NQ * HD;
      q[j0] = x1;
      q[j1] = x2;
      return;
    }
    if (rd.slot < 0 || rd.slot >= kv.max_slots || rd.seq < 0 || rd.seq >= kv.num_seqs) {
      atomicExch(err, kErrKvRange);
      return;
    }
    KT* base = (kind == 1 ? kc : vc) + kv.offset(rd.seq, rd.slot, lh);
    store_kv(base + half, x1);
    store_kv(base + half + (HD >> 1), x2);
  }
  DLLM_DEV static void store_kv(float* p, float v) { *p = v; }
  DLLM_DEV static void store_kv(__nv_bfloat16* p, float v) { *p = f32_to_bf16(v); }
};

// Final norm + LM head + greedy argmax (sampleLast, pipeline.js:141-174). Each
// thread keeps the best (value, index) key per row; the CTA folds them with
// atomicMax into best[m]. Optionally writes the logits.
template <int M>
struct EpiArgmax {
  static constexpr int R = 1;
  struct State {
    unsigned long long key[M];
  };
  const __nv_bfloat16* w;
  int N;
  float* logits;  // [m][N] or null
  DLLM_DEV void unit_rows(int u, int K, const uint4** p) const {
    p[0] = reinterpret_cast<const uint4*>(w + (size_t)u * K);
  }
  DLLM_DEV void unit(int u, int m, const float* a, State& st) const {
    if (logits) logits[(size_t)m * N + u] = a[0];
    const unsigned long long k = argmax_key(a[0], u);
#pragma unroll
    for (int i = 0; i < M; ++i)
      if (i == m && k > st.key[i]) st.key[i] = k;
  }
};

// ---- split-K MLP down projection (one row) --------------------------------------------
// 16 values in 16 lanes (lanes of one half-warp, xor offsets 8..1): afterwards
// lane l (of its half) holds the sum of v[l] over the 16 lanes. Fixed order.
DLLM_DEV float transpose_reduce16(float (&v)[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = up ? v[i] : v[i + o];
      const float keep = up ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

// This CTA's share of down_proj for one row: p[j] = sum over t < S of
// Wd[j][k0 + t] * slice[t], for every output j < D, where slice is the CTA's own
// SiLU(gate)*up values for columns [k0, k0 + S) (still in shared memory), added
// to acc[j] in fixed point (f32_to_fix, one 64-bit atomic per output). A group of
// LANES lanes (16: a half-warp, S <= 128; 32: the warp, S <= 256) covers the S
// columns of a row, 8 per lane; each lane keeps 16 rows' 16-byte weight vectors
// in flight; the 16 row sums are transpose-reduced. k0 and the row length I
// multiples of 8.
template <int LANES>
DLLM_DEV void down_partial(const __nv_bfloat16* wd, int D, int I, int k0, int S, const float* slice,
                           long long* acc) {
  constexpr int U = 16;
  constexpr int GROUPS = 32 / LANES;  // row groups per warp
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int cl = lane & (LANES - 1), rsub = lane / LANES;
  const bool act = cl * 8 < S;
  float4 xa = make_float4(0.f, 0.f, 0.f, 0.f), xb = xa;
  if (act) {
    xa = *reinterpret_cast<const float4*>(slice + cl * 8);
    xb = *reinterpret_cast<const float4*>(slice + cl * 8 + 4);
  }
  const __nv_bfloat16* wcol = wd + k0 + cl * 8;
  for (int jb = 0; jb < D; jb += nwarps * GROUPS * U) {
    const int j0 = jb + warp * GROUPS * U + rsub * U;  // this group's 16 rows
    uint4 w[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      w[u] = (act && j0 + u < D) ? ld_stream16(wcol + (size_t)(j0 + u) * I) : make_uint4(0u, 0u, 0u, 0u);
    float acc_v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) acc_v[u] = dot8(w[u], xa, xb, 0.f);
    float tot = transpose_reduce16(acc_v);  // lane l of each half: row j0 + (l & 15), that half's columns
    if (LANES == 32) tot += __shfl_xor_sync(0xffffffffu, tot, 16);
    const int r = lane & 15;
    if ((LANES == 16 || lane < 16) && j0 + r < D)
      atomicAdd(reinterpret_cast<unsigned long long*>(acc + j0 + r), static_cast<unsigned long long>(f32_to_fix(tot)));
  }
}

// The hidden row with the pending down_proj sums folded in, for this CTA's
// share of the D elements: dst[j] = h[j] + acc[j] (the value load_in4 gives
// every CTA), or h[j] when nothing is pending (acc null). With zero_acc the
// share of acc is cleared (the next layer's sums start from zero).
DLLM_DEV void fold_residual(const float* h, long long* acc, float* dst, int D, int cta, int ncta, bool zero_acc) {
  const int v0 = (int)(((long long)cta * D) / ncta), v1 = (int)(((long long)(cta + 1) * D) / ncta);
  for (int j = v0 + threadIdx.x; j < v1; j += blockDim.x) {
    float v = __ldcg(h + j);
    if (acc) {
      v = __fadd_rn(v, fix_to_f32(__ldcg(acc + j)));
      if (zero_acc) acc[j] = 0ll;
    }
    dst[j] = v;
  }
}

// Clear this CTA's share of the accumulator.
DLLM_DEV void zero_share(long long* acc, int D, int cta, int ncta) {
  const int v0 = (int)(((long long)cta * D) / ncta), v1 = (int)(((long long)(cta + 1) * D) / ncta);
  for (int j = v0 + threadIdx.x; j < v1; j += blockDim.x) acc[j] = 0ll;
}

// ---- decode attention phase (ATTENTION, kernels.js:86-132) ------------------------------
// Row m's query attends to slots [0, slot_m] of its sequence. Work item =
// (row, kv head g, split s): a split is a contiguous range of slots; the CTA's
// warps take 32-slot sub-chunks. For the G query heads sharing kv head g
// (h / (NQ/KVH) == g, kernels.js:97) a lane owns one slot for q.k (no
// shuffles), then owns HD/32 dims for p.V. Online softmax per warp, combined
// across warps in shared memory and across splits by the last CTA to finish the
// (row, g) pair (atomic ticket, no waiting).
struct AttnArgs {
  const float* q;     // [M][NQ*HD]
  float* out;         // [M][NQ*HD]
  const void* kc;     // this layer's K pool
  const void* vc;
  KvLayout kv;
  const RowDesc* rows;
  int m_rows, NQ, KVH;
  float scale;        // f32(1/sqrt(HD)), applied after the dot (kernels.js:106)
  int max_splits;     // per (row, kv head)
  float* part_o;      // [M][NQ][max_splits][HD]
  float* part_ml;     // [M][NQ][max_splits][2]
  unsigned int* arrive;  // [2][m_rows][KVH] split arrivals then finishes, zero between uses
  int* err;
  int kv_floats = 0;  // attn_item_ring: shared memory for the K/V ring (floats)
};

// Splits of a row's slots [0, T): each split is a multiple of 32 slots and is
// worked on by `nsub` warps per query head (32 slots each per round).
DLLM_DEV int attn_splits(int T, int max_splits, int nsub, int* chunk_out) {
  int ns = (T + 32 * nsub - 1) / (32 * nsub);
  if (ns > max_splits) ns = max_splits;
  if (ns > kAttnMaxSplits) ns = kAttnMaxSplits;
  if (ns < 1) ns = 1;
  int chunk = (T + ns - 1) / ns;
  chunk = (chunk + 31) & ~31;
  ns = (T + chunk - 1) / chunk;
  *chunk_out = chunk;
  return ns;
}


// Slots of one K/V staging round of an attention item (a multiple of 32).
constexpr int kAttnRound = 64;
// attn_item_ring: rounds of 32 * cpr slots (cpr = 32-slot chunks per round, one
// per sub-warp of a query head, at most 4) in a ring of up to kAttnMaxStages
// rounds in shared memory, so later rounds' copies are in flight while one is
// computed; the item's KV pages (up to kAttnPageTab) are looked up once.
constexpr int kAttnMaxCpr = 4;
constexpr int kAttnMaxStages = 4;
constexpr int kAttnPageTab = 256;

template <typename KT, int HD>
__host__ __device__ constexpr int attn_round_floats(int cpr) {  // K and V rows of one round
  return (int)(2 * 32 * cpr * HD * sizeof(KT) / sizeof(float));
}
template <typename KT, int HD>
__host__ __device__ constexpr int attn_kv_default() {  // attn_item's single round
  return attn_round_floats<KT, HD>(kAttnRound / 32);
}
// chunks per round and ring depth for `nsub` sub-warps per head within kv_floats
template <typename KT, int HD>
DLLM_DEV void attn_ring(int nsub, int kv_floats, int& cpr, int& nst) {
  cpr = min(nsub, kAttnMaxCpr);
  while (cpr > 1 && attn_round_floats<KT, HD>(cpr) > kv_floats) --cpr;
  nst = kv_floats / attn_round_floats<KT, HD>(cpr);
  nst = max(1, min(kAttnMaxStages, nst));
}

// Shared-memory floats the attention of an item needs: the K/V rows (one round,
// or the ring of kv_floats), the per-warp softmax state and partial outputs, and
// the split-merge scratch.
template <typename KT, int HD>
__host__ __device__ constexpr int attn_smem_floats(int kv_floats = 0) {
  return (kv_floats > 0 ? kv_floats : attn_kv_default<KT, HD>()) + 2 * kWarps + kWarps * HD +
         2 * kGMax * kAttnMaxSplits + kGMax + 32 * 16;
}

// 16-byte asynchronous copy global -> shared (no register staging), cached in
// L2 only; completion is awaited with cp_async_wait_all().
DLLM_DEV void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gsrc)
               : "memory");
}
DLLM_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
DLLM_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most `pending` of this thread's committed groups are incomplete.
DLLM_DEV void cp_async_wait_pending(int pending) {
  switch (pending) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
  }
}

// DPL consecutive KV elements (shared memory) -> fp32.
template <typename KT, int DPL>
DLLM_DEV void kv_row_part(const KT* p, float (&v)[DPL]);
template <>
DLLM_DEV void kv_row_part<__nv_bfloat16, 4>(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 t = *reinterpret_cast<const uint2*>(p);
  v[0] = bf16_lo(t.x); v[1] = bf16_hi(t.x); v[2] = bf16_lo(t.y); v[3] = bf16_hi(t.y);
}
template <>
DLLM_DEV void kv_row_part<__nv_bfloat16, 2>(const __nv_bfloat16* p, float (&v)[2]) {
  const uint32_t t = *reinterpret_cast<const uint32_t*>(p);
  v[0] = bf16_lo(t); v[1] = bf16_hi(t);
}
template <>
DLLM_DEV void kv_row_part<float, 4>(const float* p, float (&v)[4]) {
  const float4 t = *reinterpret_cast<const float4*>(p);
  v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
template <>
DLLM_DEV void kv_row_part<float, 2>(const float* p, float (&v)[2]) {
  const float2 t = *reinterpret_cast<const float2*>(p);
  v[0] = t.x; v[1] = t.y;
}

// Lane l holds v[0..31] (partial sums for 32 slots); afterwards lane l holds the
// full sum for slot l. 31 shuffles, fixed order.
DLLM_DEV float transpose_reduce32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = up ? v[i] : v[i + o];
      const float keep = up ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

// Tail of an attention item, run by the whole CTA after every warp has written
// its (max, sum, acc[HD]) to wm/wl/wacc (warp c*G + h holds chunk group c of
// query head h): combine the groups per head, then either write the output
// (one split) or the split's partials, take the (row, kv head) ticket, and if
// this CTA is the last of the splits, merge them all (fixed order).
template <int HD>
DLLM_DEV void attn_finish(const AttnArgs& A, int m, int g, int s, int nsplit, int G, int nsub, const float* wm,
                          const float* wl, const float* wacc, float* mrg) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  // combine the sub-chunks of each head (warps c*G + h): thread per (h, d)
  float* out_row = A.out + (size_t)m * A.NQ * HD + (size_t)g * G * HD;
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
    const int hh = i / HD, d = i - hh * HD;
    float mx = -INFINITY;
    for (int cc = 0; cc < nsub; ++cc) mx = fmaxf(mx, wm[cc * G + hh]);
    float lt = 0.f, o = 0.f;
    for (int cc = 0; cc < nsub; ++cc) {
      const float mw = wm[cc * G + hh];
      if (mw == -INFINITY) continue;
      const float f = expf(mw - mx);
      lt = fmaf(wl[cc * G + hh], f, lt);
      o = fmaf(wacc[(cc * G + hh) * HD + d], f, o);
    }
    if (nsplit == 1) {
      out_row[hh * HD + d] = __fdiv_rn(o, lt);
    } else {
      const int hq = g * G + hh;
      A.part_o[(((size_t)m * A.NQ + hq) * A.max_splits + s) * HD + d] = o;
      if (d == 0) {
        float* ml = A.part_ml + (((size_t)m * A.NQ + hq) * A.max_splits + s) * 2;
        ml[0] = mx;
        ml[1] = lt;
      }
    }
  }
  if (nsplit == 1) {
    __syncthreads();
    return;
  }
  // All nsplit CTAs of this (row, kv head) are resident (cooperative launch)
  // and hold one split each (nsplit <= kAttnMaxSplits < grid), so they can wait
  // for each other: each arrives with an acq_rel add (publishing its partials),
  // waits (bounded) until every split has arrived, then merges a 1/nsplit share
  // of the G*HD outputs. The last CTA to finish resets both counters.
  __syncthreads();
  unsigned int* arr = A.arrive + m * A.KVH + g;
  unsigned int* fin = A.arrive + (A.m_rows + m) * A.KVH + g;
  __shared__ int s_go;
  if (threadIdx.x == 0) {
    atom_add_acq_rel_u32(arr, 1u);
    int ok = 1;
    const long long t0 = clock64();
    while (ld_acquire_u32(arr) < (unsigned int)nsplit) {
      if (clock64() - t0 > kBarrierTimeoutCycles) {
        atomicExch(A.err, kErrBarrier);
        ok = 0;
        break;
      }
    }
    s_go = ok;
  }
  __syncthreads();
  if (!s_go) return;
  const int nout = G * HD;
  const int per = (nout + nsplit - 1) / nsplit;
  const int o0 = s * per, o1 = min(nout, o0 + per);
  if (o0 < o1) {
    const int h0 = o0 / HD, h1 = (o1 - 1) / HD;  // heads this share touches
    const int nh = h1 - h0 + 1;
    float* sm_m = mrg;                        // [nh][nsplit]
    float* sm_w = sm_m + kGMax * nsplit;      // [nh][nsplit] split weights
    float* sm_den = sm_w + kGMax * nsplit;    // [nh]
    float* sm_p = sm_den + kGMax;             // [32][16] partial sums
    // one round of loads: the split maxima/sums of the heads, and up to 4 split
    // outputs per thread (thread = output i of a block of 32 x split group sg)
    for (int i = threadIdx.x; i < nh * nsplit; i += blockDim.x) {
      const int hh = i / nsplit, k = i - hh * nsplit;
      const float* ml = A.part_ml + (((size_t)m * A.NQ + g * G + h0 + hh) * A.max_splits + k) * 2;
      sm_m[i] = __ldcg(ml);
      sm_w[i] = __ldcg(ml + 1);
    }
    const int sg = threadIdx.x & 15, oi = threadIdx.x >> 4;  // 16 split groups x 32 outputs
    for (int ob = o0; ob < o1; ob += 32) {
      const int o = ob + oi;
      const bool has = o < o1;
      float v[kAttnMaxSplits / 16];
#pragma unroll
      for (int r = 0; r < kAttnMaxSplits / 16; ++r) {
        const int kk = sg + 16 * r;
        v[r] = (has && kk < nsplit)
                   ? __ldcg(A.part_o + (((size_t)m * A.NQ + g * G + o / HD) * A.max_splits + kk) * HD + (o % HD))
                   : 0.f;
      }
      __syncthreads();
      if (ob == o0) {
        // per head (one warp each): max over splits, weights exp(m_s - max), denominator
        for (int hh = warp; hh < nh; hh += nwarps) {
          float mx = -INFINITY;
          for (int k = lane; k < nsplit; k += 32) mx = fmaxf(mx, sm_m[hh * nsplit + k]);
          mx = warp_max(mx);
          float den = 0.f;
          for (int k = lane; k < nsplit; k += 32) {
            const float f = expf(sm_m[hh * nsplit + k] - mx);
            den = fmaf(sm_w[hh * nsplit + k], f, den);
            sm_w[hh * nsplit + k] = f;
          }
          den = warp_sum(den);
          if (lane == 0) sm_den[hh] = den;
        }
        __syncthreads();
      }
      float acc = 0.f;
      if (has) {
        const float* w = sm_w + (o / HD - h0) * nsplit;
#pragma unroll
        for (int r = 0; r < kAttnMaxSplits / 16; ++r) {
          const int kk = sg + 16 * r;
          if (kk < nsplit) acc = fmaf(w[kk], v[r], acc);
        }
      }
      sm_p[oi * 16 + sg] = acc;
      __syncthreads();
      if (threadIdx.x < 32 && ob + (int)threadIdx.x < o1) {
        const int oo = ob + threadIdx.x;
        float tot = 0.f;
        for (int q = 0; q < 16; ++q) tot += sm_p[threadIdx.x * 16 + q];  // fixed order
        out_row[oo] = __fdiv_rn(tot, sm_den[oo / HD - h0]);
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) {
    // every CTA of the group passed its wait before arriving here
    const unsigned int d = atom_add_acq_rel_u32(fin, 1u);
    if (d == (unsigned int)nsplit - 1) {
      *arr = 0u;
      *fin = 0u;
    }
  }
  __syncthreads();
}

// Attention for one work item (row m, kv head g, split s); called by the whole
// CTA. The item's slots are taken in rounds of kAttnRound: all threads copy the
// round's K and V rows into shared memory with cp.async (one memory round trip,
// each row read once for all G query heads), then warp w = c*G + h computes
// query head h over the round's 32-slot chunk c. q.k: lane l owns dims
// [DPL*l, DPL*l + DPL) of q_h; the 32 partial dot products are transpose-reduced
// so lane p holds slot p's score; online softmax per warp; p.V: lane l
// accumulates its dims. Chunk groups of a head are combined in attn_finish.
template <typename KT, int HD>
DLLM_DEV void attn_item(const AttnArgs& A, int m, int g, int s, int nsplit, int chunk, float* smem,
                        int skip = 0) {
  constexpr int DPL = HD / 32;
  constexpr int VPR = HD * (int)sizeof(KT) / 16;  // 16-byte vectors per K or V row
  constexpr int CPR = kAttnRound / 32;           // 32-slot chunks per round
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = A.NQ / A.KVH;
  const int nsub = max(1, kWarps / G);
  const int h = warp % G, c = warp / G;
  const bool active = c < min(nsub, CPR);
  const RowDesc rd = A.rows[m];
  const int T = rd.slot + 1;
  const int p0 = s * chunk, p1 = min(T, p0 + chunk);
  KT* ks = reinterpret_cast<KT*>(smem);        // [kAttnRound][HD]
  KT* vs = ks + kAttnRound * HD;               // [kAttnRound][HD]
  float* wm = smem + 2 * kAttnRound * HD * sizeof(KT) / sizeof(float);  // [kWarps]
  float* wl = wm + kWarps;                     // [kWarps]
  float* wacc = wl + kWarps;                   // [kWarps][HD]
  float* mrg = wacc + kWarps * HD;             // split merge scratch
  const KT* kc = reinterpret_cast<const KT*>(A.kc);
  const KT* vc = reinterpret_cast<const KT*>(A.vc);

  float q[DPL];
  if (active) {
    const float* qh = A.q + (size_t)m * A.NQ * HD + (size_t)(g * G + h) * HD + lane * DPL;
#pragma unroll
    for (int d = 0; d < DPL; ++d) q[d] = __ldcg(qh + d);
  }
  float mrun = -INFINITY, lsum = 0.f, acc[DPL];
#pragma unroll
  for (int d = 0; d < DPL; ++d) acc[d] = 0.f;

  for (int base = p0; base < p1; base += kAttnRound) {
    const int n = min(kAttnRound, p1 - base);
    __syncthreads();  // readers of the previous round are done
    // rows [base, base + n): chunk cc of 32 slots lies in one KV page
    const int nvec = ((n + 31) >> 5) * 32 * VPR;  // per K or V
    for (int i = threadIdx.x; i < 2 * nvec; i += blockDim.x) {
      const int which = i >= nvec;
      const int r = which ? i - nvec : i;
      const int j = r / VPR, v = r - j * VPR;
      if (base + j >= p1 || (base == p0 && j < skip)) continue;  // rows [p0, p0 + skip) are in flight already
      const long long off = A.kv.offset(rd.seq, base + (j & ~31), g) + (long long)(j & 31) * A.kv.row_stride;
      const KT* src = (which ? vc : kc) + off + v * (16 / (int)sizeof(KT));
      KT* dst = (which ? vs : ks) + j * HD + v * (16 / (int)sizeof(KT));
      cp_async16(dst, src);
    }
    cp_async_wait_all();
    __syncthreads();
    if (active) {
      for (int cc = c; cc * 32 < n; cc += nsub) {
        const int nvalid = min(32, n - cc * 32);
        const KT* kr = ks + (cc * 32) * HD + lane * DPL;
        const KT* vr = vs + (cc * 32) * HD + lane * DPL;
        float part[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float kv[DPL];
          kv_row_part<KT, DPL>(kr + j * HD, kv);
          float sdot = 0.f;
#pragma unroll
          for (int d = 0; d < DPL; ++d) sdot = fmaf(q[d], kv[d], sdot);
          part[j] = sdot;
        }
        const float sc = transpose_reduce32(part);  // lane = slot in the chunk
        const bool valid = lane < nvalid;
        const float sv = valid ? __fmul_rn(sc, A.scale) : -INFINITY;
        const float mnew = fmaxf(mrun, warp_max(sv));
        const float alpha = (mrun == -INFINITY) ? 0.f : expf(mrun - mnew);
        const float pv = valid ? expf(sv - mnew) : 0.f;
        lsum = fmaf(lsum, alpha, pv);
        mrun = mnew;
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[d] *= alpha;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float pj = __shfl_sync(0xffffffffu, pv, j);
          if (j < nvalid) {  // rows past the item were not copied
            float vv[DPL];
            kv_row_part<KT, DPL>(vr + j * HD, vv);
#pragma unroll
            for (int d = 0; d < DPL; ++d) acc[d] = fmaf(pj, vv[d], acc[d]);
          }
        }
      }
    }
  }
  const float l = warp_sum(lsum);
  if (lane == 0) {
    wm[warp] = active ? mrun : -INFINITY;
    wl[warp] = active ? l : 0.f;
  }
#pragma unroll
  for (int d = 0; d < DPL; ++d) wacc[warp * HD + lane * DPL + d] = active ? acc[d] : 0.f;
  __syncthreads();
  attn_finish<HD>(A, m, g, s, nsplit, G, min(nsub, CPR), wm, wl, wacc, mrg);
}

// attn_item for long contexts, staging K/V through a ring of A.kv_floats of
// shared memory: the item's slots are taken in rounds of 32 * cpr slots, copied
// (cp.async, each row read once for all G query heads) nst - 1 rounds ahead of
// the round being computed, so HBM latency overlaps the q.k / p.V work. The
// item's KV pages are looked up once (page_base), so a copy needs no dependent
// load. Per round the math is attn_item's: warp w = c*G + h computes query head
// h over the round's 32-slot chunk c.
template <typename KT, int HD>
DLLM_DEV void attn_item_ring(const AttnArgs& A, int m, int g, int s, int nsplit, int chunk, float* smem,
                             int skip = 0) {
  constexpr int DPL = HD / 32;
  constexpr int VPR = HD * (int)sizeof(KT) / 16;  // 16-byte vectors per K or V row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = A.NQ / A.KVH;
  const int nsub = max(1, kWarps / G);
  const int h = warp % G, c = warp / G;
  const int kvf = A.kv_floats;
  int cpr, nst;
  attn_ring<KT, HD>(nsub, kvf, cpr, nst);
  const int R = 32 * cpr;  // slots per round
  const bool active = c < min(nsub, cpr);
  const RowDesc rd = A.rows[m];
  const int T = rd.slot + 1;
  const int p0 = s * chunk, p1 = min(T, p0 + chunk);
  KT* ring = reinterpret_cast<KT*>(smem);      // per stage: [R][HD] K rows, then [R][HD] V rows
  float* wm = smem + kvf;                      // [kWarps]
  float* wl = wm + kWarps;                     // [kWarps]
  float* wacc = wl + kWarps;                   // [kWarps][HD]
  float* mrg = wacc + kWarps * HD;             // split merge scratch
  const KT* kc = reinterpret_cast<const KT*>(A.kc);
  const KT* vc = reinterpret_cast<const KT*>(A.vc);

  float q[DPL];
  if (active) {
    const float* qh = A.q + (size_t)m * A.NQ * HD + (size_t)(g * G + h) * HD + lane * DPL;
#pragma unroll
    for (int d = 0; d < DPL; ++d) q[d] = __ldcg(qh + d);
  }
  float mrun = -INFINITY, lsum = 0.f, acc[DPL];
#pragma unroll
  for (int d = 0; d < DPL; ++d) acc[d] = 0.f;

  // the item's pages: page_base[p] = element offset of slot 0 of logical page
  // lp0 + p for head g (in the split-merge scratch, free until attn_finish)
  long long* page_base = reinterpret_cast<long long*>(mrg);
  const int lp0 = p0 >> A.kv.log2_page;
  const int npg = p1 > p0 ? ((p1 - 1) >> A.kv.log2_page) - lp0 + 1 : 0;
  const bool tab = npg <= kAttnPageTab;
  if (tab && (int)threadIdx.x < npg)
    page_base[threadIdx.x] = A.kv.offset(rd.seq, (lp0 + (int)threadIdx.x) << A.kv.log2_page, g);
  __syncthreads();
  const int nr = (p1 - p0 + R - 1) / R;
  // copies of round r into its ring stage; a 32-slot chunk lies in one KV page
  auto issue = [&](int r) {
    const int base = p0 + r * R;
    const int n = min(R, p1 - base);
    KT* ks = ring + (size_t)(r % nst) * 2 * R * HD;
    KT* vs = ks + R * HD;
    const int nvec = ((n + 31) >> 5) * 32 * VPR;  // per K or V
    for (int i = threadIdx.x; i < 2 * nvec; i += blockDim.x) {
      const int which = i >= nvec;
      const int rr = which ? i - nvec : i;
      const int j = rr / VPR, v = rr - j * VPR;
      const int slot = base + j;
      if (slot >= p1 || (r == 0 && j < skip)) continue;  // rows [p0, p0 + skip) are in flight already
      const long long off =
          tab ? page_base[(slot >> A.kv.log2_page) - lp0] +
                    (long long)(slot & ((1 << A.kv.log2_page) - 1)) * A.kv.row_stride
              : A.kv.offset(rd.seq, base + (j & ~31), g) + (long long)(j & 31) * A.kv.row_stride;
      const KT* src = (which ? vc : kc) + off + v * (16 / (int)sizeof(KT));
      KT* dst = (which ? vs : ks) + j * HD + v * (16 / (int)sizeof(KT));
      cp_async16(dst, src);
    }
  };
  for (int r = 0; r < nst - 1; ++r) {
    if (r < nr) issue(r);
    cp_async_commit();
  }
  for (int r = 0; r < nr; ++r) {
    __syncthreads();  // readers of round r - 1 (whose stage round r + nst - 1 reuses) are done
    if (r + nst - 1 < nr) issue(r + nst - 1);
    cp_async_commit();
    cp_async_wait_pending(nst - 1);  // this thread's copies of round r have landed
    __syncthreads();                 // and every thread's
    const int n = min(R, p1 - (p0 + r * R));
    const KT* ks = ring + (size_t)(r % nst) * 2 * R * HD;
    const KT* vs = ks + R * HD;
    if (active) {
      for (int cc = c; cc * 32 < n; cc += nsub) {
        const int nvalid = min(32, n - cc * 32);
        const KT* kr = ks + (cc * 32) * HD + lane * DPL;
        const KT* vr = vs + (cc * 32) * HD + lane * DPL;
        float part[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float kv[DPL];
          kv_row_part<KT, DPL>(kr + j * HD, kv);
          float sdot = 0.f;
#pragma unroll
          for (int d = 0; d < DPL; ++d) sdot = fmaf(q[d], kv[d], sdot);
          part[j] = sdot;
        }
        const float sc = transpose_reduce32(part);  // lane = slot in the chunk
        const bool valid = lane < nvalid;
        const float sv = valid ? __fmul_rn(sc, A.scale) : -INFINITY;
        const float mnew = fmaxf(mrun, warp_max(sv));
        const float alpha = (mrun == -INFINITY) ? 0.f : expf(mrun - mnew);
        const float pv = valid ? expf(sv - mnew) : 0.f;
        lsum = fmaf(lsum, alpha, pv);
        mrun = mnew;
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[d] *= alpha;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float pj = __shfl_sync(0xffffffffu, pv, j);
          if (j < nvalid) {  // rows past the item were not copied
            float vv[DPL];
            kv_row_part<KT, DPL>(vr + j * HD, vv);
#pragma unroll
            for (int d = 0; d < DPL; ++d) acc[d] = fmaf(pj, vv[d], acc[d]);
          }
        }
      }
    }
  }
  cp_async_wait_pending(0);  // nothing in flight leaves the item (only empty groups remain)
  const float l = warp_sum(lsum);
  if (lane == 0) {
    wm[warp] = active ? mrun : -INFINITY;
    wl[warp] = active ? l : 0.f;
  }
#pragma unroll
  for (int d = 0; d < DPL; ++d) wacc[warp * HD + lane * DPL + d] = active ? acc[d] : 0.f;
  __syncthreads();
  attn_finish<HD>(A, m, g, s, nsplit, G, min(nsub, cpr), wm, wl, wacc, mrg);
}

// One-row passes: the rows of the first staging round of this CTA's first
// attention item that exist before the pass (every slot but the one the pass
// appends), located once per launch (the rows and page table do not change
// during it; the layer only changes the pool base). attn_early_issue copies them
// into the round's place in shared memory at the end of the QKV phase, so they
// land while the grid barrier completes; attn_phase then copies the rest.
struct AttnEarly {
  int n;              // rows to copy ahead (0: none)
  int R;              // rows of the item's first round (its stage-0 layout)
  long long coff[kAttnMaxCpr];  // element offset of each 32-slot chunk (head g)
};

template <typename KT, int HD, bool RING>
DLLM_DEV void attn_early_plan(const AttnArgs& A, int cta, int ncta, AttnEarly* plan) {
  if (threadIdx.x == 0) {
    plan->n = 0;
    const RowDesc rd = A.rows[0];
    if (A.m_rows == 1 && rd.slot >= 0 && rd.slot < A.kv.max_slots && rd.seq >= 0 && rd.seq < A.kv.num_seqs) {
      const int nsub = max(1, kWarps / (A.NQ / A.KVH));
      int chunk;
      const int ns = attn_splits(rd.slot + 1, A.max_splits, nsub, &chunk);
      if (cta < A.KVH * ns) {
        const int g = cta / ns, sp = cta - g * ns;
        int R = kAttnRound;
        if (RING) {
          int cpr, nst;
          attn_ring<KT, HD>(nsub, A.kv_floats, cpr, nst);
          R = 32 * cpr;
        }
        const int p0 = sp * chunk;
        const int n = min(R, min(rd.slot, p0 + chunk) - p0);  // rows before the appended slot
        if (n > 0) {
          plan->R = R;
          for (int c = 0; c * 32 < n; ++c) plan->coff[c] = A.kv.offset(rd.seq, p0 + 32 * c, g);
          plan->n = n;
        }
      }
    }
  }
  __syncthreads();
}

// Issue the planned copies into shared memory (one cp.async group) for this layer's pools.
template <typename KT, int HD>
DLLM_DEV int attn_early_issue(const AttnEarly& plan, const void* kc_, const void* vc_, int row_stride, float* smem) {
  constexpr int VPR = HD * (int)sizeof(KT) / 16;
  const int n = plan.n;
  if (n <= 0) return 0;
  const KT* kc = reinterpret_cast<const KT*>(kc_);
  const KT* vc = reinterpret_cast<const KT*>(vc_);
  KT* ks = reinterpret_cast<KT*>(smem);
  KT* vs = ks + plan.R * HD;
  const int nvec = n * VPR;
  for (int i = threadIdx.x; i < 2 * nvec; i += blockDim.x) {
    const int which = i >= nvec;
    const int r = which ? i - nvec : i;
    const int j = r / VPR, v = r - j * VPR;
    const long long off = plan.coff[j >> 5] + (long long)(j & 31) * row_stride;
    cp_async16((which ? vs : ks) + j * HD + v * (16 / (int)sizeof(KT)), (which ? vc : kc) + off + v * (16 / (int)sizeof(KT)));
  }
  cp_async_commit();
  return n;
}

// All attention work items of a pass, spread round-robin over the CTAs.
// RING: items go through attn_item_ring (A.kv_floats of shared memory).
template <typename KT, int HD, bool RING = false>
DLLM_DEV void attn_phase(const AttnArgs& A, float* smem, int cta, int ncta, int first_skip = 0) {
  // enumerate items: rows in order, kv heads, splits
  int item = 0;
  int skip = first_skip;  // rows of this CTA's first item issued ahead (attn_early_issue)
  for (int m = 0; m < A.m_rows; ++m) {
    const RowDesc rd = A.rows[m];
    if (rd.slot < 0 || rd.slot >= A.kv.max_slots || rd.seq < 0 || rd.seq >= A.kv.num_seqs) {
      if (cta == 0 && threadIdx.x == 0) atomicExch(A.err, kErrKvRange);
      continue;
    }
    int chunk;
    const int nsub = max(1, (int)(blockDim.x >> 5) / (A.NQ / A.KVH));
    const int ns = attn_splits(rd.slot + 1, A.max_splits, nsub, &chunk);
    const int n_items = A.KVH * ns;
    // this CTA's items of the row: global item index item + j == cta (mod ncta),
    // stepped directly (a scan over all items with a modulo each cost ~20 us)
    int j0 = (cta - item) % ncta;
    if (j0 < 0) j0 += ncta;
    for (int j = j0; j < n_items; j += ncta) {
      const int g = j / ns, s = j - g * ns;
      if constexpr (RING) attn_item_ring<KT, HD>(A, m, g, s, ns, chunk, smem, skip);
      else attn_item<KT, HD>(A, m, g, s, ns, chunk, smem, skip);
      skip = 0;
    }
    item += n_items;
  }
}

}  // namespace dllm
