// common.cuh — device helpers shared by the sm_100a kernels of libdllm.
//
// Everything here is hand-written PTX for Blackwell (sm_100a) or plain CUDA C++:
//   * streaming 16-byte weight loads that bypass L1 (weights are read exactly once
//     per decode step, so they must not evict the activations L1 holds),
//   * the TMA engine's bulk L2 prefetch (cp.async.bulk.prefetch.L2),
//   * bf16 <-> fp32 bit helpers matching weights.js:153-164 (value = bits << 16).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define DLLM_DEV __device__ __forceinline__

namespace dllm {

// ---- memory -------------------------------------------------------------------
// 16-byte streaming load of read-only data: no L1 allocation, 256-byte L2 fetch.
DLLM_DEV uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Bulk prefetch of [p, p+bytes) into L2 by the TMA unit. p and bytes must be
// multiples of 16.
DLLM_DEV void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Nanosecond global timer (same clock on every SM).
DLLM_DEV unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---- bf16 bit helpers (weights.js:153-164: f32 bits = bf16 bits << 16) --------
DLLM_DEV float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
DLLM_DEV float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
DLLM_DEV float bf16_to_f32(__nv_bfloat16 b) { return __uint_as_float(((uint32_t)__bfloat16_as_ushort(b)) << 16); }

// fp32 -> bf16, round to nearest even (the storage rounding of the bf16 KV cache).
DLLM_DEV __nv_bfloat16 f32_to_bf16(float f) { return __float2bfloat16_rn(f); }

// ---- warp reductions ------------------------------------------------------------
DLLM_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
DLLM_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Dot product of 8 bf16 weights (one 16-byte vector) with 8 fp32 activations.
DLLM_DEV float dot8(uint4 w, float4 a, float4 b, float acc) {
  acc = fmaf(bf16_lo(w.x), a.x, acc);
  acc = fmaf(bf16_hi(w.x), a.y, acc);
  acc = fmaf(bf16_lo(w.y), a.z, acc);
  acc = fmaf(bf16_hi(w.y), a.w, acc);
  acc = fmaf(bf16_lo(w.z), b.x, acc);
  acc = fmaf(bf16_hi(w.z), b.y, acc);
  acc = fmaf(bf16_lo(w.w), b.z, acc);
  acc = fmaf(bf16_hi(w.w), b.w, acc);
  return acc;
}

// ---- greedy argmax key ----------------------------------------------------------
// (value, index) packed so that the u64 maximum is the largest value and, among
// equal values, the lowest index: the strict '>' scan of pipeline.js:159-162.
// NaN is mapped to -inf so it never wins (a NaN never compares greater in JS).
DLLM_DEV unsigned long long argmax_key(float v, int idx) {
  if (v != v) v = -INFINITY;
  uint32_t u = __float_as_uint(v);
  uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(~(uint32_t)idx);
}
DLLM_DEV int argmax_key_index(unsigned long long key) { return (int)(~(uint32_t)(key & 0xffffffffull)); }

// ---- per-row decode descriptor ----------------------------------------------------
// One row of a forward: which sequence it belongs to, the RoPE position, and
// the KV slot it writes (attention then covers slots [0, slot]). For
// Stage.forward(h, n, posStart) row t has pos = posStart + t and slot = T0 + t
// (pipeline.js:62-65; kernels.js:94 and :121).
struct RowDesc {
  int seq;
  int pos;
  int slot;
  int pad;
};

// KV cache addressing. A sequence's slot s lives in logical page s >> log2_page,
// mapped to a physical page through `page_table` (or the identity
// seq * max_pages + page when it is null). Element (slot, head, d) is at
//   phys * page_stride + head * head_stride + (s & (page-1)) * row_stride + d.
// The reference layout [maxPos, KVH*HD] (pipeline.js:38-43) is the special case
// of one page holding every slot: log2_page = 30, row_stride = KVH*HD,
// head_stride = HD. The stage's own paged cache is head-major inside a page
// (row_stride = HD), so 32 consecutive slots of one head are contiguous.
struct KvLayout {
  void* k;
  void* v;
  const int* page_table;
  int log2_page;
  int max_pages;  // pages per sequence
  int head_stride;
  int row_stride;
  long long page_stride;
  int max_slots;  // slots per sequence
  int num_seqs;

  DLLM_DEV long long offset(int seq, int slot, int head) const {
    const int lp = slot >> log2_page;
    const int off = slot & ((1 << log2_page) - 1);
    const int phys = page_table ? page_table[seq * max_pages + lp] : seq * max_pages + lp;
    return (long long)phys * page_stride + (long long)head * head_stride + (long long)off * row_stride;
  }
};

}  // namespace dllm
