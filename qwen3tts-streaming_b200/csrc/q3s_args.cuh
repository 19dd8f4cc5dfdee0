// q3s_args.cuh -- argument blocks passed by value to the kernels (shared by
// the translation units of libq3s_sampler.so).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q3s_sampler.h"

namespace q3s {

struct SampleArgs {
  int mode, B, V, K;
  int64_t row_stride;
  const void* logits;
  const int64_t* col_shift;
  const int64_t* token_counts;
  int64_t tc_stride;
  const int32_t* history;
  const int32_t* offsets;
  int64_t history_len;
  const int32_t* history_lengths;  // capacity layout: row b = [offsets[b], offsets[b] + len) inside its region
  const float* temperature;
  float temperature_default;
  const int32_t* top_k;
  const float* top_p;
  float top_p_default;
  const float* penalty;
  float penalty_default;
  const int32_t* min_new;
  int32_t min_new_default;
  const int32_t* cur_len;
  const float* noise;
  int64_t noise_stride;
  const float* uniforms;
  const uint8_t* suppress;
  int eos_id;
  int64_t* ids64;
  int32_t* ids32;
  int64_t* counts_out;
  int64_t co_stride;
  float* processed;
  int64_t proc_stride;
  int32_t* row_flags;
  int32_t* error_word;
  bool vec_logits;
  bool vec_counts;
  bool vec_suppress;
  bool vec_history;
  bool pdl;  // launched as a programmatic dependent: wait for the producing grid before touching logits
};

struct CpArgs {
  int mode, B, V, S, K, producer;
  const void* logits;
  int64_t row_stride, stage_stride;
  const int64_t* ids_init;
  const float* temperature;
  float temperature_default;
  const float* top_p;
  float top_p_default;
  const float* noise;
  int64_t noise_row_stride, noise_stage_stride;
  const float* uniforms;
  int64_t* ids_out;
  int32_t* row_flags;
  int32_t* error_word;
  bool bulk;
  uint32_t row_bytes;
  int nbuf;
};

// Shared-memory row kernels (q3s_warp.cu): icdf steps, 1024 < V <= 3072,
// V % 8 == 0; `warps` (1, 2, 4 or 8; anything else: the widest variant,
// 12 warps for V > 2048 and 16 below) warps per row.
cudaError_t launch_warp_rows(const SampleArgs& a, bool bf16, cudaStream_t st, int warps);
// Register-resident row kernels (q3s_lean.cu): icdf steps, V <= 3072,
// V % 8 == 0, one CTA of 128 threads per row.
cudaError_t launch_lean_rows(const SampleArgs& a, bool bf16, cudaStream_t st);
// q3s_sample's body; `pdl` launches the sampler as a programmatic dependent
// of the previous kernel on the stream (q3s_sampler.cu).
q3s_status sample_impl(const q3s_sample_desc* d, cudaStream_t stream, bool pdl);
// Record a failure for q3s_last_error_string (the calling thread's) and return s.
q3s_status report(q3s_status s, const char* fmt, ...);
// SM count of the current device (cached).
int sm_count();

// Warps per row for a batch size on `sm_count` SMs (0: the widest variant).
int smem_warps_for(int batch, int sm_count);
// Launch a kernel with the programmatic-stream-serialization attribute when
// `pdl` is set (the launch overlaps the previous kernel on the stream, which
// the kernel waits for with griddepcontrol.wait), plainly otherwise.
template <typename... Params, typename... Args>
cudaError_t launch_maybe_pdl(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                             Args&&... args) {
  if (!pdl) {
    kern<<<grid, block, smem, st>>>(static_cast<Args&&>(args)...);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&lc, kern, static_cast<Args&&>(args)...);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace q3s
