// q3s_warp.cu -- the warp-per-row kernels (q3s_warp.cuh) and their launcher,
// a translation unit of its own so that it compiles beside q3s_sampler.cu.
#include <cuda_runtime.h>

#include "q3s_args.cuh"
#include "q3s_warp.cuh"

namespace q3s {
namespace {

template <int R>
cudaError_t launch_warp(const SampleArgs& a, bool bf16, cudaStream_t st) {
  constexpr size_t dyn = warp_smem_bytes<R>();
  auto kern = bf16 ? sample_warp_kernel<R, true> : sample_warp_kernel<R, false>;
  // more than the 48 KB default of dynamic shared memory: opt in once per
  // (kernel, device)
  static bool granted[2][64] = {{false}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !granted[bf16 ? 1 : 0][dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) granted[bf16 ? 1 : 0][dev] = true;
  }
  const int grid = (a.B + WPB - 1) / WPB;
  kern<<<grid, WPB * 32, dyn, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_warp_rows(const SampleArgs& a, bool bf16, cudaStream_t st) {
  return a.V <= 2048 ? launch_warp<8>(a, bf16, st) : launch_warp<12>(a, bf16, st);
}

}  // namespace q3s
