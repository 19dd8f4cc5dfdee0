// q3s_warp.cu -- the shared-memory-resident row kernels (q3s_warp.cuh) and
// their launcher, a translation unit of its own so that it compiles beside
// q3s_sampler.cu.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "q3s_args.cuh"
#include "q3s_warp.cuh"

namespace q3s {
namespace {

template <int R, int W>
cudaError_t launch_smem(const SampleArgs& a, bool bf16, cudaStream_t st) {
  const size_t dyn = row_smem_bytes<R, W>(bf16);
  const bool proc = a.processed != nullptr;
  const int v = (bf16 ? 2 : 0) + (proc ? 1 : 0);
  using Kern = void (*)(const SampleArgs);
  const Kern kerns[4] = {sample_smem_kernel<R, W, false, false>, sample_smem_kernel<R, W, false, true>,
                         sample_smem_kernel<R, W, true, false>, sample_smem_kernel<R, W, true, true>};
  const Kern kern = kerns[v];
  // the shared-memory opt-in and the largest carveout (so that ~11 rows fit
  // per SM), set once per (variant, device): one bit per device; two threads
  // racing on a first launch both set the same attributes, which is harmless
  static std::atomic<uint64_t> done[4];
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
  if (!bit || !(done[v].load(std::memory_order_acquire) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    done[v].fetch_or(bit, std::memory_order_release);
  }
  return launch_maybe_pdl(kern, dim3(a.B), dim3(W * 32), dyn, st, a.pdl, a);
}

template <int R>
cudaError_t launch_r(const SampleArgs& a, bool bf16, cudaStream_t st, int w) {
  // the widest variant splits the rows' rounds (2R) into 2 per warp (R = 12)
  // or 1 per warp (R = 8)
  constexpr int WMAX = R == 12 ? 12 : 16;
  switch (w) {
    case 1: return launch_smem<R, 1>(a, bf16, st);
    case 2: return launch_smem<R, 2>(a, bf16, st);
    case 4: return launch_smem<R, 4>(a, bf16, st);
    case 8: return launch_smem<R, 8>(a, bf16, st);
    default: return launch_smem<R, WMAX>(a, bf16, st);
  }
}

}  // namespace

int smem_warps_for(int batch, int sm_count) {
  // measured on B200 (V=3072, configs 1/3/4): up to one row per SM a row is
  // latency-bound and takes the widest variant; up to two, 8 warps; beyond,
  // 4 warps per row (more rows side by side)
  if (batch <= sm_count) return 0;  // widest
  if (batch <= 2 * sm_count) return 8;
  return 4;
}

cudaError_t launch_warp_rows(const SampleArgs& a, bool bf16, cudaStream_t st, int warps) {
  return a.V <= 2048 ? launch_r<8>(a, bf16, st, warps) : launch_r<12>(a, bf16, st, warps);
}

}  // namespace q3s
