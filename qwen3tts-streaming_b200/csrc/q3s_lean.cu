// q3s_lean.cu -- the register-resident row kernels (q3s_lean.cuh) and their
// launcher, a translation unit of its own so that it compiles beside
// q3s_sampler.cu.
#include <cuda_runtime.h>

#include <cstdint>

#include "q3s_args.cuh"
#include "q3s_lean.cuh"

namespace q3s {
namespace {

template <int NT, int E>
cudaError_t launch_lean(const SampleArgs& a, bool bf16, cudaStream_t st) {
  const bool proc = a.processed != nullptr;
  auto kern = bf16 ? (proc ? sample_lean_kernel<NT, E, true, true> : sample_lean_kernel<NT, E, true, false>)
                   : (proc ? sample_lean_kernel<NT, E, false, true> : sample_lean_kernel<NT, E, false, false>);
  return launch_maybe_pdl(kern, dim3(a.B), dim3(NT), 0, st, a.pdl, a);
}

}  // namespace

cudaError_t launch_lean_rows(const SampleArgs& a, bool bf16, cudaStream_t st) {
  if (a.V <= 1024) return launch_lean<128, 8>(a, bf16, st);
  if (a.V <= 2048) return launch_lean<128, 16>(a, bf16, st);
  return launch_lean<128, 24>(a, bf16, st);
}

}  // namespace q3s
