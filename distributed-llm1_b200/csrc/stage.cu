// stage.cu — dispatch of the stage kernel by KV dtype (instantiations live in
// stage_f32.cu and stage_bf16.cu so they compile in parallel).
#include "stage.cuh"

namespace dllm {

cudaError_t launch_stage_f32(const StageParams& p, int grid, cudaStream_t st);
cudaError_t launch_stage_bf16(const StageParams& p, int grid, cudaStream_t st);
cudaError_t configure_stage_f32();
cudaError_t configure_stage_bf16();

cudaError_t configure_stage_kernels() {
  cudaError_t e = configure_stage_f32();
  if (e == cudaSuccess) e = configure_stage_bf16();
  return e;
}

// The split-K MLP (one row) needs 8-aligned column slices of down_proj of at
// most 128 columns per CTA (16 lanes x 8 per row group) or, with head_dim 128,
// 256 (32 lanes x 8), and the accumulator after the barrier counter. Returns the
// lanes per row group, or 0 when the pass cannot use it.
static int splitk_lanes(const StageParams& p, int grid) {
  if (p.m_rows != 1 || !p.acc || !p.h2 || p.I % 8 != 0 || grid < 1) return 0;
  if (reinterpret_cast<const char*>(p.acc) != reinterpret_cast<const char*>(p.bar_count) + 16) return 0;
  int widest = 0;
  for (int c = 0; c < grid; ++c) {
    int u0 = (int)(((long long)c * p.I) / grid) / 8 * 8;
    int u1 = c + 1 == grid ? p.I : (int)(((long long)(c + 1) * p.I) / grid) / 8 * 8;
    if (u1 - u0 > widest) widest = u1 - u0;
  }
  if (widest <= 128) return 16;
  if (widest <= 256 && p.HD == 128) return 32;
  return 0;
}

cudaError_t launch_stage(const StageParams& p0, int kv_dtype, int grid, cudaStream_t st) {
  if (p0.m_rows < 1 || p0.m_rows > 8) return cudaErrorInvalidValue;
  StageParams p = p0;
  p.splitk = splitk_lanes(p, grid);
  // the grid barrier's counter (and, for the split-K MLP, the fixed-point
  // accumulator right after it) starts every launch at zero: one memset node
  // when the launch is captured into a graph
  const size_t clear = p.splitk ? 16 + sizeof(long long) * (size_t)p.D : sizeof(unsigned int);
  cudaError_t e = cudaMemsetAsync(p.bar_count, 0, clear, st);
  if (e != cudaSuccess) return e;
  return kv_dtype == 0 ? launch_stage_f32(p, grid, st) : launch_stage_bf16(p, grid, st);
}

}  // namespace dllm
