// q3s_philox.cuh -- device-side per-row uniforms / Gumbel noise.
//
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel Random Numbers: As Easy
// as 1, 2, 3", SC'11), written from the paper's round function: with
// multipliers M0, M1 and key (k0, k1),
//     (hi0, lo0) = M0 * x0,  (hi1, lo1) = M1 * x2,
//     x' = (hi1 ^ x1 ^ k0, lo1, hi0 ^ x3 ^ k1, lo0),
// the key bumped by the Weyl constants between rounds.  Counters and the
// float mapping are those of the host generator (q3s/philox.py row_uniforms),
// so both produce the same bits: block j of row key r at step s uses counter
// (j, r mod 2^32, s, 0xA5A5 ^ (r >> 32)) under key (seed mod 2^32,
// seed >> 32) -- all 64 bits of r, and for r < 2^32 the counter (j, r, s,
// 0xA5A5) -- and a 32-bit output x maps to (x >> 8) * 2^-24 in [0, 1).
// Per-row seeds (philox_seeds_kernel): block j of a row with 64-bit seed q
// at (step s, stage t) uses counter (j, s, t, 0x5EED) under key (q mod 2^32,
// q >> 32), so one row's numbers are its seed's alone.
//
// Replaces the reference's per-slot torch.rand calls and the noise transform
// -log(-log(clamp(u, 1e-8, 1))) (engine/backend/executor.py:3216-3295) with
// one launch over all rows.
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace q3s {

constexpr uint32_t PHILOX_M0 = 0xD2511F53u;
constexpr uint32_t PHILOX_M1 = 0xCD9E8D57u;
constexpr uint32_t PHILOX_W0 = 0x9E3779B9u;
constexpr uint32_t PHILOX_W1 = 0xBB67AE85u;

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k0 += PHILOX_W0;
      k1 += PHILOX_W1;
    }
    const uint32_t hi0 = __umulhi(PHILOX_M0, c.x), lo0 = PHILOX_M0 * c.x;
    const uint32_t hi1 = __umulhi(PHILOX_M1, c.z), lo1 = PHILOX_M1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
  }
  return c;
}

// (x >> 8) * 2^-24: exact in fp32, strictly below 1.
__device__ __forceinline__ float philox_unit(uint32_t x) {
  return __fmul_rn(__uint2float_rn(x >> 8), 0x1p-24f);
}

__device__ __forceinline__ void philox_store(const uint4 x, int j, int cols, int kind, float* o) {
  const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if (4 * j + e >= cols) break;
    float u = philox_unit(xs[e]);
    if (kind == 1) u = -logf(-logf(fminf(fmaxf(u, 1e-8f), 1.0f)));
    o[4 * j + e] = u;
  }
}

// One thread per (row, block of 4 columns); the key is the row's own 64-bit
// seed.  kind 0: uniforms; kind 1: Gumbel noise.
__global__ void philox_seeds_kernel(const uint64_t* seeds, uint32_t step, uint32_t stage, int rows, int cols,
                                    int kind, float* out, int64_t out_stride) {
  const int nblk = (cols + 3) / 4;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows) * nblk) return;
  const int i = static_cast<int>(idx / nblk), j = static_cast<int>(idx % nblk);
  const uint64_t q = seeds[i];
  const uint4 x = philox4x32_10(make_uint4(static_cast<uint32_t>(j), step, stage, 0x5EEDu), static_cast<uint32_t>(q),
                                static_cast<uint32_t>(q >> 32));
  philox_store(x, j, cols, kind, out + static_cast<int64_t>(i) * out_stride);
}

// One thread per (row, block of 4 columns).  kind 0: uniforms; kind 1:
// Gumbel noise -log(-log(max(u, 1e-8))) in fp32.
__global__ void philox_rows_kernel(uint32_t k0, uint32_t k1, uint32_t step, const int64_t* row_keys,
                                   int64_t row0, int rows, int cols, int kind, float* out,
                                   int64_t out_stride) {
  const int nblk = (cols + 3) / 4;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows) * nblk) return;
  const int i = static_cast<int>(idx / nblk), j = static_cast<int>(idx % nblk);
  const uint64_t r = static_cast<uint64_t>(row_keys ? row_keys[i] : row0 + i);
  const uint4 x = philox4x32_10(
      make_uint4(static_cast<uint32_t>(j), static_cast<uint32_t>(r), step, 0xA5A5u ^ static_cast<uint32_t>(r >> 32)),
      k0, k1);
  philox_store(x, j, cols, kind, out + static_cast<int64_t>(i) * out_stride);
}

}  // namespace q3s
