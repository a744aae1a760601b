// kk3_kernel_nt1.cu - step kernel instantiation for batches of up to 8 rows (1 MMA n-tile(s) of 8),
// with its own launch helpers so no translation unit references another unit's kernel.
#include <cuda_runtime.h>

#include "kk3_kernel.cuh"

namespace kk3 {

// Raise (never lower) the kernel's dynamic shared memory limit to at least `smem`. The limit is per-function
// state shared by every context and by the allocation-free entry point, so lowering it for a smaller geometry
// would make the next launch of a live context with a larger need fail.
cudaError_t raise_smem_nt1(size_t smem) {
  cudaFuncAttributes attr;
  cudaError_t e = cudaFuncGetAttributes(&attr, kk3_step_kernel<1>);
  if (e != cudaSuccess) return e;
  if ((size_t)attr.maxDynamicSharedSizeBytes >= smem) return cudaSuccess;
  return cudaFuncSetAttribute(kk3_step_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

cudaError_t prepare_nt1(size_t smem, int* occupancy) {
  cudaError_t e = raise_smem_nt1(smem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occupancy, kk3_step_kernel<1>, kThreads, smem);
}

cudaError_t launch_nt1(const StepArgs* args, int grid, size_t smem, cudaStream_t stream) {
  void* params[] = {const_cast<StepArgs*>(args)};
  return cudaLaunchCooperativeKernel((const void*)kk3_step_kernel<1>, dim3(grid), dim3(kThreads), params, smem, stream);
}

}  // namespace kk3
