// q3s_device.cuh -- device building blocks of the codec-token sampler.
//
// Layout: one CTA owns one row of V logits.  Thread t holds the 8 contiguous
// vocabulary entries [8t, 8t+8) in registers for the whole step, so the row
// is read from HBM exactly once (16-byte vector loads) and every later pass
// (penalty, top-k select, top-p cut, CDF scan) runs on registers plus a few
// KB of shared memory.  All reductions use a fixed combination order, so a
// given input always produces bit-identical output.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q3s_sampler.h"

namespace q3s {

constexpr int E = 8;                      // vocabulary entries per thread
constexpr unsigned FULL = 0xffffffffu;
constexpr float NEG_SUPPRESS = -1e9f;     // talker_unified_modules.py:409
constexpr float BOUNDARY_EPS = 1e-6f;
constexpr int CAND = Q3S_MAX_TOPK;        // candidate buffer (exactly-K set, small top-p set)
constexpr int MASS_BITS = 38;             // fixed-point scale of top-p masses (weights <= 1)

#define Q3S_DEV __device__ __forceinline__

// ---------------------------------------------------------------------------
// scalar helpers
// ---------------------------------------------------------------------------

// Order-preserving float -> uint32 map (ascending).  -0 is folded onto +0 so
// that equal floats get equal keys, matching torch's comparisons.
Q3S_DEV uint32_t f2key(float x) {
  uint32_t u = __float_as_uint(x == 0.0f ? 0.0f : x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

Q3S_DEV float bf16_bits_to_f32(uint32_t h16) { return __uint_as_float(h16 << 16); }

// torch.argmax order: NaN beats everything (first NaN wins), then larger
// value, then lower tie-break key.
Q3S_DEV bool arg_better(float a, int ta, float b, int tb) {
  const bool na = a != a, nb = b != b;
  if (na | nb) return na && (!nb || ta < tb);
  return a > b || (a == b && ta < tb);
}

// exp(s - m) for the softmax weights; -inf (filtered) entries weigh 0.
Q3S_DEV float softmax_weight(float s, float m) {
  return (s == -INFINITY) ? 0.0f : expf(__fsub_rn(s, m));
}

Q3S_DEV uint4 ld_stream16(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

Q3S_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// per-CTA shared scratch
// ---------------------------------------------------------------------------

template <int NT>
struct alignas(16) Scratch {
  static constexpr int NW = NT / 32;
  unsigned long long red_q[32];
  unsigned long long mhist[256];
  float red_f[32];
  int red_i[32];
  uint32_t red_u[32];
  uint32_t hist[256];
  uint32_t cand_k[CAND];
  float cand_v[CAND];
  int cand_i[CAND];
  float cand_w[CAND];       // softmax weights (icdf) / Gumbel noise by rank (gumbel)
  uint8_t cand_keep[CAND];
  alignas(16) uint8_t seen[E * NT];  // presence flags built from a packed history
  int bc_i[4];
  uint32_t bc_u[4];
  unsigned long long bc_q[2];
};

// ---------------------------------------------------------------------------
// warp / block reductions (fixed order => deterministic)
// ---------------------------------------------------------------------------

Q3S_DEV float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
Q3S_DEV float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
  return v;
}
Q3S_DEV unsigned long long warp_sum_q(unsigned long long v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}

template <int NT>
Q3S_DEV float block_sum_f(float v, Scratch<NT>& sh) {
  v = warp_sum_f(v);
  if ((threadIdx.x & 31) == 0) sh.red_f[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += sh.red_f[i];
  __syncthreads();
  return r;
}

template <int NT>
Q3S_DEV float block_max_f(float v, Scratch<NT>& sh) {
  v = warp_max_f(v);
  if ((threadIdx.x & 31) == 0) sh.red_f[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = -INFINITY;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r = fmaxf(r, sh.red_f[i]);
  __syncthreads();
  return r;
}

template <int NT>
Q3S_DEV unsigned long long block_sum_q(unsigned long long v, Scratch<NT>& sh) {
  v = warp_sum_q(v);
  if ((threadIdx.x & 31) == 0) sh.red_q[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned long long r = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += sh.red_q[i];
  __syncthreads();
  return r;
}

template <int NT>
Q3S_DEV uint32_t block_sum_u(uint32_t v, Scratch<NT>& sh) {
  v = __reduce_add_sync(FULL, v);
  if ((threadIdx.x & 31) == 0) sh.red_u[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += sh.red_u[i];
  __syncthreads();
  return r;
}

template <int NT>
Q3S_DEV uint32_t block_min_u(uint32_t v, Scratch<NT>& sh) {
  v = __reduce_min_sync(FULL, v);
  if ((threadIdx.x & 31) == 0) sh.red_u[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = 0xffffffffu;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r = min(r, sh.red_u[i]);
  __syncthreads();
  return r;
}

template <int NT>
Q3S_DEV int block_min_i(int v, Scratch<NT>& sh) {
  v = __reduce_min_sync(FULL, v);
  if ((threadIdx.x & 31) == 0) sh.red_i[threadIdx.x >> 5] = v;
  __syncthreads();
  int r = 0x7fffffff;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r = min(r, sh.red_i[i]);
  __syncthreads();
  return r;
}

template <int NT>
Q3S_DEV int block_max_i(int v, Scratch<NT>& sh) {
  v = __reduce_max_sync(FULL, v);
  if ((threadIdx.x & 31) == 0) sh.red_i[threadIdx.x >> 5] = v;
  __syncthreads();
  int r = -0x7fffffff - 1;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r = max(r, sh.red_i[i]);
  __syncthreads();
  return r;
}

// Block argmax of (value, tie) under arg_better; returns the payload of the
// winner.  Threads without a candidate pass (-inf, INT_MAX, *).
template <int NT>
Q3S_DEV int block_argmax(float v, int tie, int payload, Scratch<NT>& sh) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(FULL, v, o);
    const int ot = __shfl_xor_sync(FULL, tie, o);
    const int op = __shfl_xor_sync(FULL, payload, o);
    if (arg_better(ov, ot, v, tie)) { v = ov; tie = ot; payload = op; }
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sh.red_f[w] = v;
    sh.red_i[w] = tie;
    sh.red_u[w] = static_cast<uint32_t>(payload);
  }
  __syncthreads();
  float bv = sh.red_f[0];
  int bt = sh.red_i[0];
  int bp = static_cast<int>(sh.red_u[0]);
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) {
    if (arg_better(sh.red_f[i], sh.red_i[i], bv, bt)) {
      bv = sh.red_f[i];
      bt = sh.red_i[i];
      bp = static_cast<int>(sh.red_u[i]);
    }
  }
  __syncthreads();
  return bp;
}

// Exclusive scan over threads (thread order = vocabulary order).
template <int NT>
Q3S_DEV uint32_t block_excl_scan_u(uint32_t v, uint32_t& total, Scratch<NT>& sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc += n;
  }
  if (lane == 31) sh.red_u[w] = inc;
  __syncthreads();
  uint32_t pre = 0, tot = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) {
    const uint32_t x = sh.red_u[i];
    pre += (i < w) ? x : 0u;
    tot += x;
  }
  __syncthreads();
  total = tot;
  return pre + inc - v;
}

template <int NT>
Q3S_DEV float block_excl_scan_f(float v, float& total, Scratch<NT>& sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float n = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc = __fadd_rn(inc, n);
  }
  float ex = __shfl_up_sync(FULL, inc, 1);
  if (lane == 0) ex = 0.0f;
  if (lane == 31) sh.red_f[w] = inc;
  __syncthreads();
  float pre = 0.0f, tot = 0.0f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) {
    const float x = sh.red_f[i];
    if (i < w) pre = __fadd_rn(pre, x);
    tot = __fadd_rn(tot, x);
  }
  __syncthreads();
  total = tot;
  return __fadd_rn(pre, ex);
}

// ---------------------------------------------------------------------------
// radix selection
// ---------------------------------------------------------------------------

// Key of the k-th largest entry (1-based k, multiplicity counted) among the
// entries flagged in `mask`.  MSB-first 8-bit digits with a shared-memory
// histogram; stops early once the selected bucket holds exactly the entries
// still needed (the answer is then that bucket's minimum).
template <int NT>
Q3S_DEV uint32_t select_kth_largest(const uint32_t (&key)[E], uint32_t mask, int k,
                                    Scratch<NT>& sh) {
  uint32_t prefix = 0, hmask = 0;
  int krem = k;
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += NT) sh.hist[i] = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (((mask >> j) & 1u) && (key[j] & hmask) == prefix)
        atomicAdd(&sh.hist[(key[j] >> shift) & 255u], 1u);
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      uint32_t c[8], s = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = sh.hist[lane * 8 + i];
        s += c[i];
      }
      uint32_t suf = s;  // entries in buckets >= this lane's first bucket
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_down_sync(FULL, suf, o);
        if (lane + o < 32) suf += n;
      }
      const uint32_t above = suf - s;
      if (above < static_cast<uint32_t>(krem) && static_cast<uint32_t>(krem) <= suf) {
        uint32_t acc = above;
        bool found = false;
#pragma unroll
        for (int i = 7; i >= 0; --i) {
          if (!found) {
            if (acc + c[i] >= static_cast<uint32_t>(krem)) {
              found = true;
              sh.bc_u[0] = static_cast<uint32_t>(lane * 8 + i);
              sh.bc_u[1] = c[i];
              sh.bc_i[0] = krem - static_cast<int>(acc);
            } else {
              acc += c[i];
            }
          }
        }
      }
    }
    __syncthreads();
    const uint32_t d = sh.bc_u[0];
    const uint32_t cnt = sh.bc_u[1];
    krem = sh.bc_i[0];
    prefix |= d << shift;
    hmask |= 255u << shift;
    if (shift > 0 && cnt == static_cast<uint32_t>(krem)) {
      uint32_t mn = 0xffffffffu;
#pragma unroll
      for (int j = 0; j < E; ++j)
        if (((mask >> j) & 1u) && (key[j] & hmask) == prefix) mn = min(mn, key[j]);
      return block_min_u<NT>(mn, sh);
    }
  }
  return prefix;
}

// Top-p cut by mass (ascending order = (value asc, index asc), the order of a
// stable ascending sort).  q are fixed-point weights; finds the smallest key v
// with  mass(key <= v) > tau.  Returns v and mass(key < v).
template <int NT>
Q3S_DEV void select_mass_cut(const uint32_t (&key)[E], const unsigned long long (&q)[E],
                             uint32_t mask, unsigned long long tau, Scratch<NT>& sh,
                             uint32_t& vstar, unsigned long long& below_out) {
  uint32_t prefix = 0, hmask = 0;
  unsigned long long below = 0;
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += NT) sh.mhist[i] = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (((mask >> j) & 1u) && q[j] != 0 && (key[j] & hmask) == prefix)
        atomicAdd(&sh.mhist[(key[j] >> shift) & 255u], q[j]);
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      unsigned long long c[8], s = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = sh.mhist[lane * 8 + i];
        s += c[i];
      }
      unsigned long long inc = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long n = __shfl_up_sync(FULL, inc, o);
        if (lane >= o) inc += n;
      }
      const unsigned long long lo = below + (inc - s);
      const unsigned long long hi = below + inc;
      if (lo <= tau && tau < hi) {
        unsigned long long acc = lo;
        bool found = false;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (!found) {
            if (acc + c[i] > tau) {
              found = true;
              sh.bc_u[0] = static_cast<uint32_t>(lane * 8 + i);
              sh.bc_q[0] = acc;
            } else {
              acc += c[i];
            }
          }
        }
      }
    }
    __syncthreads();
    // bc_* is rewritten only after the next pass's two barriers
    prefix |= sh.bc_u[0] << shift;
    below = sh.bc_q[0];
    hmask |= 255u << shift;
  }
  vstar = prefix;
  below_out = below;
}

}  // namespace q3s
