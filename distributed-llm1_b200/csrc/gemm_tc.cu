// gemm_tc.cu — tcgen05 matmul for passes of many rows (see gemm_tc.cuh).
//
// One CTA = 4 warps computes a 128-row weight tile against all (padded) rows
// of the pass over a contiguous range of K (split-K when the tiles alone do not
// fill the GPU). Warp 0 lane 0 streams the weight tile and the activation tile
// of each 128-wide K block (two 64-wide boxes) into a shared-memory ring of 2-8
// stages with TMA
// (cp.async.bulk.tensor, 128-byte swizzle, completion on an mbarrier); warp 1
// lane 0 issues tcgen05.mma (kind::f16, bf16 in, fp32 accumulator in tensor
// memory) and frees each stage with tcgen05.commit; then all four warps read the
// accumulator back with tcgen05.ld (warp w owns TMEM lanes 32w..32w+31, i.e.
// weight rows) and write y, or the split's partial row, coalesced along N.
// Every mbarrier wait is bounded; a wait that runs out sets an error flag, and
// the CTA still waits (bounded) for its own copies and frees its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm_tc.cuh"

namespace dllm {
namespace {

constexpr int kBM = 128;      // weight rows per tile (MMA M)
constexpr int kBK = 64;       // K per box: 64 bf16 = 128 bytes, one swizzle row
constexpr int kBoxes = 2;     // boxes per stage: 256 contiguous bytes of each weight row per stage
constexpr int kBKS = kBK * kBoxes;  // K per stage
constexpr int kMaxStages = 8;   // deepest ring (one CTA per SM at 16-32 rows)
constexpr int kTcMaxTargets = 3;
constexpr int kTcThreads = 128;
constexpr int kABoxBytes = kBM * kBK * 2;              // 16 KB: one 128-row box
constexpr int kATileBytes = kABoxBytes * kBoxes;        // 32 KB per stage
constexpr long long kTcWaitCycles = 1ll << 32;        // ~2 s of SM cycles

DLLM_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

DLLM_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
DLLM_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Bounded wait for completion of the phase with parity `parity`.
DLLM_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const long long t0 = clock64();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > kTcWaitCycles) return false;
  }
}

// 2-D tiled TMA load of box (x = K offset, y = row offset) into shared memory,
// completing on `bar` (no multicast: the tensor always lies in this GPU's memory).
DLLM_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (stride
// byte offset 1024 >> 4), leading byte offset unused (1), descriptor version 1,
// layout type 2 (SWIZZLE_128B). The tile base must be 1024-byte aligned.
DLLM_DEV uint64_t umma_desc_sw128(const void* tile) {
  const uint64_t a = smem_u32(tile);
  return ((a & 0x3FFFFull) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// D[tmem] (+)= A[128 x 16] * B[N x 16]^T, bf16 inputs, fp32 accumulate.
DLLM_DEV void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Arrive on `bar` once every tcgen05.mma this thread issued so far has completed.
DLLM_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
DLLM_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DLLM_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 8 consecutive fp32 accumulator columns of this thread's TMEM lane.
DLLM_DEV void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
DLLM_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// One output matrix of a launch: weight tiles [tile_begin, tile_begin + tiles) of
// the grid belong to it. Several targets that share the activations (q|k|v,
// gate|up) go in one launch behind one hi/lo split.
struct TcTargetDev {
  float* out;           // y [rows][N], or partials [splits][rows][N]
  int N;
  int tile_begin;
  size_t split_stride;  // elements between splits' partials (0: out is y)
  int accumulate;       // y += (only when out is y)
};

struct TcArgs {
  int rows, K;
  int n_kblocks, kb_per_split;
  int stages;  // ring depth, <= kMaxStages, sized by the host to the shared memory
  int n_tgt;
  TcTargetDev t[kTcMaxTargets];
  int* err;
};

// RP = padded rows (16, 32, 64, 128); the MMA's N is 2 * RP (x_hi rows, x_lo rows).
template <int RP>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
                   const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ CUtensorMap tmX,
                   const TcArgs a) {
  constexpr int NMMA = 2 * RP;
  constexpr int kBBoxBytes = NMMA * kBK * 2;
  constexpr int kBTileBytes = kBBoxBytes * kBoxes;
  constexpr uint32_t kCols = NMMA < 32 ? 32 : NMMA;  // tensor-memory columns (a power of two >= 32)
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages], accum;
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_s;
  __shared__ int accum_ok_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.stages;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = base;                  // S x 16 KB
  uint8_t* sB = base + S * kATileBytes;  // S x kBTileBytes
  // which target this CTA's tile belongs to
  int m = 0;
  if (a.n_tgt > 1 && (int)blockIdx.x >= a.t[1].tile_begin) m = 1;
  if (a.n_tgt > 2 && (int)blockIdx.x >= a.t[2].tile_begin) m = 2;
  const TcTargetDev tg = a.t[m];
  const CUtensorMap* tmW = m == 0 ? &tmW0 : (m == 1 ? &tmW1 : &tmW2);
  const int tile = (int)blockIdx.x - tg.tile_begin;
  const int kb0 = blockIdx.y * a.kb_per_split;
  const int nkb = min(a.n_kblocks, kb0 + a.kb_per_split) - kb0;  // >= 1 (host sizes the splits)
  const int rot = (int)((blockIdx.x * 5u + blockIdx.y * 3u) % (unsigned)nkb);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&accum, 1);
    abort_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  int issued = 0;  // TMA stages issued (producer thread)
  if (warp == 0 && lane == 0) {
    // ---- producer: K blocks [kb0, kb0 + nkb) through the ring
    for (int i = 0; i < nkb; ++i) {
      const int s = i % S;
      const uint32_t ph = (uint32_t)(i / S) & 1u;
      if (!mbar_wait(&empty[s], ph ^ 1u)) {
        atomicExch(a.err, kErrTcWait);
        abort_s = 1;
        break;
      }
      if (abort_s) break;
      mbar_expect_tx(&full[s], (uint32_t)(kATileBytes + kBTileBytes));
      // K blocks in a per-tile rotated order: 148 tiles reading the same column
      // offset of rows a fixed stride apart crowd a few DRAM channels
      const int kx = (kb0 + (i + rot) % nkb) * kBKS;
#pragma unroll
      for (int b = 0; b < kBoxes; ++b) {
        tma_load_2d(sA + s * kATileBytes + b * kABoxBytes, tmW, kx + b * kBK, tile * kBM, &full[s]);
        tma_load_2d(sB + s * kBTileBytes + b * kBBoxBytes, &tmX, kx + b * kBK, 0, &full[s]);
      }
      issued = i + 1;
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer: 4 MMAs of K = 16 per stage, accumulator in tensor memory
    const uint32_t idesc = (1u << 4)                        // D fp32
                           | (1u << 7) | (1u << 10)         // A, B bf16
                           | ((uint32_t)(NMMA >> 3) << 17)  // N
                           | ((uint32_t)(kBM >> 4) << 24);  // M = 128; A and B K-major
    for (int i = 0; i < nkb; ++i) {
      const int s = i % S;
      const uint32_t ph = (uint32_t)(i / S) & 1u;
      if (!mbar_wait(&full[s], ph)) {
        atomicExch(a.err, kErrTcWait);
        abort_s = 1;
        break;
      }
      if (abort_s) break;
      tc_fence_after();
#pragma unroll
      for (int b = 0; b < kBoxes; ++b) {
        const uint64_t ad = umma_desc_sw128(sA + s * kATileBytes + b * kABoxBytes);
        const uint64_t bd = umma_desc_sw128(sB + s * kBTileBytes + b * kBBoxBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)  // +32 bytes along K inside the swizzled row
          umma_bf16(tmem, ad + 2ull * kk, bd + 2ull * kk, idesc, (uint32_t)((i | b | kk) != 0));
      }
      umma_commit(&empty[s]);
    }
    umma_commit(&accum);  // every MMA issued above has completed when this arrives
  }
  __syncwarp();

  // ---- epilogue: wait for the accumulator, then TMEM -> registers -> global
  if (threadIdx.x == 0) accum_ok_s = mbar_wait(&accum, 0) ? 1 : 0;
  __syncthreads();
  tc_fence_after();
  if (accum_ok_s && !abort_s) {
    const int j = tile * kBM + warp * 32 + lane;  // weight row = TMEM lane
    float* dst = tg.out + (size_t)blockIdx.y * tg.split_stride;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
    for (int c0 = 0; c0 < RP; c0 += 8) {
      uint32_t hi[8], lo[8];
      tmem_ld8(trow + (uint32_t)c0, hi);
      tmem_ld8(trow + (uint32_t)(RP + c0), lo);
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int r = c0 + q;
        if (r < a.rows && j < tg.N) {
          float* d = dst + (size_t)r * tg.N + j;
          const float v = __uint_as_float(hi[q]) + __uint_as_float(lo[q]);
          *d = tg.accumulate ? __fadd_rn(*d, v) : v;
        }
      }
    }
  } else if (threadIdx.x == 0 && !accum_ok_s) {
    atomicExch(a.err, kErrTcWait);
  }
  // ---- teardown: copies still in flight (only after an aborted wait) land
  // before the CTA exits, then the tensor memory is freed
  if (warp == 0 && lane == 0 && abort_s) {
    for (int i = max(0, issued - S); i < issued; ++i) mbar_wait(&full[i % S], (uint32_t)(i / S) & 1u);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
  }
}

// x (fp32 [rows][K]) -> xb (bf16 [2 RP][K]): row t < rows: xb[t] = bf16(x'), xb[RP + t]
// = bf16(x' - bf16(x')), where x' = (x * rsqrt(mean(x^2) + eps)) * g with a norm,
// else x; rows [rows, RP) are zero. Grid (K / kSplitChunk chunks, RP rows), 256
// threads x 8 elements each, 16-byte loads and stores: no thread walks a row
// (a strided loop over K is a chain of dependent round trips). With a norm each
// block first sums the squares of its whole row (float4 loads, block reduce), so
// every chunk of a row uses the same scale.
constexpr int kSplitThreads = 256;
constexpr int kSplitChunk = kSplitThreads * 8;

__global__ void __launch_bounds__(kSplitThreads) split_hilo_kernel(const float* x, int rows, int K,
                                                                   const __nv_bfloat16* norm_w, float eps, int rp,
                                                                   __nv_bfloat16* xb) {
  __shared__ float red[kSplitThreads / 32];
  const int t = blockIdx.y;
  const int k = blockIdx.x * kSplitChunk + threadIdx.x * 8;
  uint4* hi = reinterpret_cast<uint4*>(xb + (size_t)t * K + k);
  uint4* lo = reinterpret_cast<uint4*>(xb + (size_t)(rp + t) * K + k);
  if (t >= rows) {
    if (k < K) {
      *hi = make_uint4(0u, 0u, 0u, 0u);
      *lo = make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }
  const float* xr = x + (size_t)t * K;
  float scale = 1.f;
  if (norm_w) {
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    float ss = 0.f;
    for (int i = threadIdx.x; i < (K >> 2); i += kSplitThreads) {
      const float4 v = __ldg(x4 + i);
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < kSplitThreads / 32; ++i) tot += red[i];
    scale = 1.0f / sqrtf(tot / (float)K + eps);
  }
  if (k >= K) return;
  const float4 a = __ldg(reinterpret_cast<const float4*>(xr + k));
  const float4 b = __ldg(reinterpret_cast<const float4*>(xr + k + 4));
  float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  if (norm_w) {
    const uint4 g = __ldg(reinterpret_cast<const uint4*>(norm_w + k));
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[2 * q] = (v[2 * q] * scale) * bf16_lo(gw[q]);
      v[2 * q + 1] = (v[2 * q + 1] * scale) * bf16_hi(gw[q]);
    }
  }
  uint32_t h[4], l[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __nv_bfloat16 h0 = __float2bfloat16_rn(v[2 * q]), h1 = __float2bfloat16_rn(v[2 * q + 1]);
    const __nv_bfloat16 l0 = __float2bfloat16_rn(v[2 * q] - bf16_to_f32(h0));
    const __nv_bfloat16 l1 = __float2bfloat16_rn(v[2 * q + 1] - bf16_to_f32(h1));
    h[q] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
    l[q] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
  }
  *hi = make_uint4(h[0], h[1], h[2], h[3]);
  *lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// y[t][j] (=|+=) sum over splits s of part[s][t][j], in split order.
__global__ void splitk_reduce_kernel(const float* part, int splits, size_t stride, int rows, int N, float* y,
                                     int accumulate) {
  const size_t total = (size_t)rows * N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < splits; ++k) s += __ldcg(part + (size_t)k * stride + i);
    y[i] = accumulate ? __fadd_rn(y[i], s) : s;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Row-major bf16 [outer][inner] as a 2-D tensor map with a (64 x box_rows) box and
// the 128-byte swizzle; out-of-range boxes read zeros.
bool encode_rows(CUtensorMap* m, const void* base, int inner, int outer, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  const cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int padded_rows(int rows) { return rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 64 ? 64 : 128; }

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct Plan {
  int rp, n_tiles, n_kb, kb_per, splits, stages;
  size_t xb_bytes, part_bytes, smem;
};

// Tiles of all targets, K split until tiles x splits fills the SMs, and the ring
// depth: one wave -> one CTA per SM with the deepest ring that fits (up to 8
// stages, ~220 KB); several waves -> two CTAs per SM (~110 KB each), so one
// CTA's epilogue overlaps the other's loads.
Plan make_plan(int rows, int K, const int* Ns, int n, int sms) {
  Plan p;
  p.rp = padded_rows(rows);
  p.n_tiles = 0;
  int sumN = 0;
  for (int i = 0; i < n; ++i) {
    p.n_tiles += (Ns[i] + kBM - 1) / kBM;
    sumN += Ns[i];
  }
  p.n_kb = (K + kBKS - 1) / kBKS;
  int splits = sms / p.n_tiles;
  if (splits < 1) splits = 1;
  if (splits > p.n_kb) splits = p.n_kb;
  p.kb_per = (p.n_kb + splits - 1) / splits;
  p.splits = (p.n_kb + p.kb_per - 1) / p.kb_per;  // no empty split
  p.xb_bytes = align_up((size_t)2 * p.rp * K * 2, 1024);
  p.part_bytes = p.splits > 1 ? (size_t)p.splits * rows * sumN * 4 : 0;
  const size_t per_stage = (size_t)kATileBytes + (size_t)kBoxes * 2 * p.rp * kBK * 2;
  const bool one_wave = (long long)p.n_tiles * p.splits <= sms;
  // two CTAs per SM only when each still gets a double-buffered ring
  const bool two_per_sm = !one_wave && (110 * 1024 - 1024) / per_stage >= 2;
  const size_t budget = two_per_sm ? 110 * 1024 : 220 * 1024;
  int st = (int)((budget - 1024) / per_stage);
  p.stages = st < 2 ? 2 : (st > kMaxStages ? kMaxStages : st);
  p.smem = 1024 + (size_t)p.stages * per_stage;
  return p;
}

template <int RP>
cudaError_t launch_rp(const CUtensorMap* tw, const CUtensorMap& tx, const TcArgs& a, dim3 grid, size_t smem,
                      cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    const size_t most = 1024 + (size_t)kMaxStages * (kATileBytes + kBoxes * 2 * RP * kBK * 2);
    const size_t cap = 1024 + 220 * 1024;
    attr = cudaFuncSetAttribute(tc_gemm_kernel<RP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)(most < cap ? most : cap));
  });
  if (attr != cudaSuccess) return attr;
  tc_gemm_kernel<RP><<<grid, kTcThreads, smem, st>>>(tw[0], tw[1], tw[2], tx, a);
  return cudaGetLastError();
}

}  // namespace

bool tc_available() { return encode_fn() != nullptr; }

size_t tc_matmul_scratch_bytes(int rows, int K, int N, int sms) { return tc_matmul_multi_scratch_bytes(rows, K, &N, 1, sms); }

size_t tc_matmul_multi_scratch_bytes(int rows, int K, const int* Ns, int n, int sms) {
  const Plan p = make_plan(rows, K, Ns, n, sms);
  return p.xb_bytes + p.part_bytes;
}

cudaError_t tc_matmul_multi(const float* x, int rows, int K, const TcTarget* t, int n, const __nv_bfloat16* norm_w,
                            float eps, void* scratch, size_t scratch_bytes, int* err, int sms, cudaStream_t st) {
  if (rows < 1 || rows > kTcMaxRows || K < 8 || K % 8 != 0 || n < 1 || n > kTcMaxTargets || !x || !t || !scratch ||
      !err)
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(scratch) & 255) != 0) return cudaErrorMisalignedAddress;
  int Ns[kTcMaxTargets];
  for (int i = 0; i < n; ++i) {
    if (!t[i].w || !t[i].y || t[i].N < 1) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(t[i].w) & 15) != 0) return cudaErrorMisalignedAddress;
    Ns[i] = t[i].N;
  }
  const Plan p = make_plan(rows, K, Ns, n, sms);
  if (p.xb_bytes + p.part_bytes > scratch_bytes) return cudaErrorInvalidValue;
  __nv_bfloat16* xb = static_cast<__nv_bfloat16*>(scratch);
  float* part = reinterpret_cast<float*>(static_cast<char*>(scratch) + p.xb_bytes);
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0 || (norm_w && (reinterpret_cast<uintptr_t>(norm_w) & 15) != 0))
    return cudaErrorMisalignedAddress;
  split_hilo_kernel<<<dim3((K + kSplitChunk - 1) / kSplitChunk, p.rp), kSplitThreads, 0, st>>>(x, rows, K, norm_w,
                                                                                               eps, p.rp, xb);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  CUtensorMap tw[kTcMaxTargets], tx;
  TcArgs a = {};
  a.rows = rows;
  a.K = K;
  a.n_kblocks = p.n_kb;
  a.kb_per_split = p.kb_per;
  a.stages = p.stages;
  a.n_tgt = n;
  a.err = err;
  int tile = 0;
  size_t part_off = 0;
  for (int i = 0; i < n; ++i) {
    if (!encode_rows(&tw[i], t[i].w, K, t[i].N, kBM)) return cudaErrorInvalidValue;
    a.t[i].N = t[i].N;
    a.t[i].tile_begin = tile;
    tile += (t[i].N + kBM - 1) / kBM;
    if (p.splits > 1) {
      a.t[i].out = part + part_off;
      a.t[i].split_stride = (size_t)rows * t[i].N;
      a.t[i].accumulate = 0;
      part_off += (size_t)p.splits * rows * t[i].N;
    } else {
      a.t[i].out = t[i].y;
      a.t[i].split_stride = 0;
      a.t[i].accumulate = t[i].accumulate;
    }
  }
  for (int i = n; i < kTcMaxTargets; ++i) tw[i] = tw[0];  // unused parameters
  if (!encode_rows(&tx, xb, K, 2 * p.rp, 2 * p.rp)) return cudaErrorInvalidValue;
  const dim3 grid(p.n_tiles, p.splits);
  switch (p.rp) {
    case 16: e = launch_rp<16>(tw, tx, a, grid, p.smem, st); break;
    case 32: e = launch_rp<32>(tw, tx, a, grid, p.smem, st); break;
    case 64: e = launch_rp<64>(tw, tx, a, grid, p.smem, st); break;
    default: e = launch_rp<128>(tw, tx, a, grid, p.smem, st); break;
  }
  if (e != cudaSuccess || p.splits == 1) return e;
  for (int i = 0; i < n; ++i) {
    const size_t total = (size_t)rows * t[i].N;
    const unsigned int blocks = (unsigned int)std::min<size_t>((total + 255) / 256, (size_t)sms * 8);
    splitk_reduce_kernel<<<blocks, 256, 0, st>>>(a.t[i].out, p.splits, a.t[i].split_stride, rows, t[i].N, t[i].y,
                                                 t[i].accumulate);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t tc_matmul(const float* x, int rows, int K, const __nv_bfloat16* w, int N, float* y, int accumulate,
                      const __nv_bfloat16* norm_w, float eps, void* scratch, size_t scratch_bytes, int* err, int sms,
                      cudaStream_t st) {
  const TcTarget t{w, N, y, accumulate};
  return tc_matmul_multi(x, rows, K, &t, 1, norm_w, eps, scratch, scratch_bytes, err, sms, st);
}

}  // namespace dllm
