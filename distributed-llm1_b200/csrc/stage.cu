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

cudaError_t launch_stage(const StageParams& p, int kv_dtype, int grid, cudaStream_t st) {
  if (p.m_rows < 1 || p.m_rows > 8) return cudaErrorInvalidValue;
  // the grid barrier's counter starts every launch at zero (a memset node when
  // the launch is captured into a graph)
  cudaError_t e = cudaMemsetAsync(p.bar_count, 0, sizeof(unsigned int), st);
  if (e != cudaSuccess) return e;
  return kv_dtype == 0 ? launch_stage_f32(p, grid, st) : launch_stage_bf16(p, grid, st);
}

}  // namespace dllm
