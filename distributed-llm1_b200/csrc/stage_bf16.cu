// stage_bf16.cu — stage kernel instantiations for the bf16 KV cache.
#include "stage_impl.cuh"

namespace dllm {

cudaError_t launch_stage_bf16(const StageParams& p, int grid, cudaStream_t st) {
  if (p.HD == 64) return launch_m<__nv_bfloat16, 64>(p, grid, st);
  if (p.HD == 128) return launch_m<__nv_bfloat16, 128>(p, grid, st);
  return cudaErrorInvalidValue;
}

cudaError_t configure_stage_bf16() {
  cudaError_t e = configure_hd<__nv_bfloat16, 64>();
  if (e == cudaSuccess) e = configure_hd<__nv_bfloat16, 128>();
  return e;
}

}  // namespace dllm
