// stage_f32.cu — stage kernel instantiations for the f32 KV cache.
#include "stage_impl.cuh"

namespace dllm {

cudaError_t launch_stage_f32(const StageParams& p, int grid, cudaStream_t st) {
  if (p.HD == 64) return launch_m<float, 64>(p, grid, st);
  if (p.HD == 128) return launch_m<float, 128>(p, grid, st);
  return cudaErrorInvalidValue;
}

cudaError_t configure_stage_f32() {
  cudaError_t e = configure_hd<float, 64>();
  if (e == cudaSuccess) e = configure_hd<float, 128>();
  return e;
}

}  // namespace dllm
