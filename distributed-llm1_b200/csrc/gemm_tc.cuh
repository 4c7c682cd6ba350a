// gemm_tc.cuh — tensor-core (tcgen05) matmul for passes of many rows.
//
// MATMUL of kernels.js:26-44 (y[t, j] = sum_k x[t, k] * W[j, k]) when the rows
// of a pass make it a real GEMM (prefill chunks, wide micro-batches): weights
// bf16 [N, K] as the MMA's A operand (128 rows per tile, TMA-staged with the
// 128-byte swizzle), activations as the B operand. The reference computes in
// fp32; a bf16 copy of the activations would lose 16 mantissa bits, so each
// activation row x is split into x_hi = bf16(x) and x_lo = bf16(x - x_hi) and
// both go through the same MMA (B rows [0, Rp) hold x_hi, [Rp, 2 Rp) x_lo);
// the epilogue adds the two accumulator columns of a row. x_hi + x_lo carries
// 16 bits of x's 24-bit mantissa (the product with a bf16 weight is exact, the
// accumulation fp32), against 8 for a plain bf16 cast.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace dllm {

constexpr int kTcMinRows = 8;    // passes with fewer rows stay on the CUDA-core matvec (measured crossover)
constexpr int kTcMaxRows = 128;  // rows per launch (x_hi + x_lo = 256 MMA columns)
constexpr int kErrTcWait = 5;    // a tcgen05 kernel gave up waiting on an mbarrier

// Device bytes of scratch tc_matmul needs for `rows` rows of length K and N
// outputs on a GPU with `sms` SMs (split activations + split-K partials).
size_t tc_matmul_scratch_bytes(int rows, int K, int N, int sms);

// y[t, j] (=|+=) sum_k xn[t, k] * W[j, k] for t < rows (1..128), where xn is x
// with an optional RMSNorm (gamma `norm_w`, eps; kernels.js:46-63) applied per
// row. accumulate: 0 store, 1 add to y (the residual adds of pipeline.js:66-67,
// 73-74). K must be a multiple of 8 and w 16-byte aligned. `err` receives
// kErrTcWait if a bounded wait inside the kernel ran out.
cudaError_t tc_matmul(const float* x, int rows, int K, const __nv_bfloat16* w, int N, float* y, int accumulate,
                      const __nv_bfloat16* norm_w, float eps, void* scratch, size_t scratch_bytes, int* err, int sms,
                      cudaStream_t st);

// One output of a launch that shares its activations with the others (the
// q|k|v or gate|up projections of one RMSNorm'd input).
struct TcTarget {
  const __nv_bfloat16* w;  // [N, K] bf16, 16-byte aligned
  int N;
  float* y;                // [rows, N]
  int accumulate;          // 0 store, 1 add to y
};
// Up to 3 targets in one launch behind one hi/lo split of x (and one RMSNorm).
size_t tc_matmul_multi_scratch_bytes(int rows, int K, const int* Ns, int n, int sms);
cudaError_t tc_matmul_multi(const float* x, int rows, int K, const TcTarget* t, int n, const __nv_bfloat16* norm_w,
                            float eps, void* scratch, size_t scratch_bytes, int* err, int sms, cudaStream_t st);

// Whether the driver offers the tensor-map encoder (always true on a B200 driver).
bool tc_available();

}  // namespace dllm
