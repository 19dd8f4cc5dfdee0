// q3s_device.cuh -- device building blocks of the codec-token sampler.
//
// Layout: one CTA of NT threads owns one row of V logits.  Thread t holds the
// E contiguous vocabulary entries [E*t, E*t+E) in registers for the whole
// step (E = 8: one 16-byte bf16 load), so the row is read from HBM exactly
// once and every later pass (penalty, top-k select, top-p cut, CDF scan) runs
// on registers plus a few KB of shared memory.  Per-entry work is kept to the
// minimum (the top-k select works on pre-temperature keys; softmax weights and
// the draw touch only the survivors), and the number of barrier-separated
// block rounds is kept small: on B200 one such round costs ~200-600 cycles.
//
// All reductions combine in a fixed order, so a given input always produces
// bit-identical output.  Block reductions use double-buffered per-warp
// partials (one barrier each); radix passes use one 256-bin histogram that
// the scanning warp clears as it reads it (two barriers per pass).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q3s_sampler.h"

namespace q3s {

constexpr unsigned FULL = 0xffffffffu;
constexpr float NEG_SUPPRESS = -1e9f;     // talker_unified_modules.py:409
constexpr float BOUNDARY_EPS = 1e-6f;
constexpr int CAND = Q3S_MAX_TOPK;        // candidate records (exactly-K set, small top-p set)
constexpr int FINISH = 128;               // survivor count finished on a compact candidate list
constexpr int MASS_BITS = 36;             // fixed-point scale of top-p masses (weights <= 1)
constexpr int MASS_LO_BITS = 18;          // masses split into two 32-bit histograms
constexpr int NBINS = 256;                // radix digits of 8 bits

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

// Inverse of f2key.
Q3S_DEV float key2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// x / d rounded to nearest even, for a per-row divisor d with r = RN(1/d):
// two residual corrections of q0 = RN(x r) (Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990; Cornea, Harrison and Tang, "Scientific Computing on
// Itanium-based Systems", 2002): the first makes the quotient faithful, and
// with r the correctly rounded reciprocal the second, RN(q1 + r RN(x - d q1)),
// is the correctly rounded quotient while x, d, the quotient and the
// residuals stay normal (|x| and x/d within [2^-80, 2^100], d within
// [2^-20, 2^20]).  Finite x only.
Q3S_DEV float div_rn_row(float x, float d, float r) {
  const float q0 = __fmul_rn(x, r);
  const float q1 = __fmaf_rn(__fmaf_rn(-q0, d, x), r, q0);
  return __fmaf_rn(__fmaf_rn(-q1, d, x), r, q1);
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

Q3S_DEV unsigned long long mass_fixed(float w) {
  return __float2ull_rn(__fmul_rn(w, static_cast<float>(1ull << MASS_BITS)));
}

// Streaming 16-byte load, issued where it is written (volatile), not sunk to
// its first use.
Q3S_DEV uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

Q3S_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy helpers (every copy lands in the issuing CTA only)
// ---------------------------------------------------------------------------

Q3S_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
Q3S_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
Q3S_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Plain bulk copy global -> this CTA's shared memory (one destination).
Q3S_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
Q3S_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after ~2^20 polls (each poll itself blocks for a
// hardware-defined interval) instead of spinning forever.
Q3S_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < (1 << 20); ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// ---------------------------------------------------------------------------
// Capacity layout: the end of a row of `len` ids starting at `start` inside
// its region [start, region_end); -1 (an invalid end, flagged by the caller's
// offsets check) when len is negative or passes the region.
__device__ __forceinline__ int row_end_in_region(int start, int region_end, int len) {
  const long long e = static_cast<long long>(start) + len;
  return (len < 0 || e > region_end) ? -1 : static_cast<int>(e);
}

// per-CTA shared scratch
// ---------------------------------------------------------------------------

template <int NT, int E>
struct alignas(16) Scratch {
  static constexpr int NW = NT / 32;
  // radix histograms: [0] counts or mass high parts, [1] mass low parts.
  // Invariant: all zero between passes (the scanning warp clears what it reads).
  uint32_t hist[2][NBINS];
  uint4 cand[CAND];          // {key, index, value/weight bits, spare}
  float noise[CAND];         // Gumbel noise by rank
  alignas(16) float xs[CAND];  // candidate values by position (exactly-K ranks)
  unsigned long long part_q[2][32];
  float part_f[2][32];
  float part_f2[2][32];
  int part_i[2][32];
  uint32_t part_u[2][32];
  uint8_t keep[CAND];
  uint8_t surv[CAND];
  alignas(16) uint8_t seen[E * NT];  // presence flags built from a packed history
  uint32_t sel_u[4];
  unsigned long long sel_q[2];
  int flags;                 // row flags raised by any thread
};

// Zero the radix histograms (once per kernel, before the first barrier).
template <int NT, int E>
Q3S_DEV void clear_hist(Scratch<NT, E>& sh) {
  uint4* h = reinterpret_cast<uint4*>(&sh.hist[0][0]);
  for (int i = threadIdx.x; i < 2 * NBINS / 4; i += NT) h[i] = make_uint4(0, 0, 0, 0);
}

// ---------------------------------------------------------------------------
// warp / block reductions (fixed order => deterministic), one barrier each.
// `rb` alternates the partial buffers; every thread runs the same sequence.
// ---------------------------------------------------------------------------

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

template <int NT, int E>
Q3S_DEV unsigned long long block_sum_q(unsigned long long v, Scratch<NT, E>& sh, int& rb) {
  v = warp_sum_q(v);
  if ((threadIdx.x & 31) == 0) sh.part_q[rb][threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned long long r = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += sh.part_q[rb][i];
  rb ^= 1;
  return r;
}

template <int NT, int E>
Q3S_DEV uint32_t block_min_u(uint32_t v, Scratch<NT, E>& sh, int& rb) {
  v = __reduce_min_sync(FULL, v);
  if ((threadIdx.x & 31) == 0) sh.part_u[rb][threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = 0xffffffffu;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r = min(r, sh.part_u[rb][i]);
  rb ^= 1;
  return r;
}

template <int NT, int E>
Q3S_DEV int block_min_i(int v, Scratch<NT, E>& sh, int& rb) {
  v = __reduce_min_sync(FULL, v);
  if ((threadIdx.x & 31) == 0) sh.part_i[rb][threadIdx.x >> 5] = v;
  __syncthreads();
  int r = 0x7fffffff;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r = min(r, sh.part_i[rb][i]);
  rb ^= 1;
  return r;
}

template <int NT, int E>
Q3S_DEV int block_max_i(int v, Scratch<NT, E>& sh, int& rb) {
  v = __reduce_max_sync(FULL, v);
  if ((threadIdx.x & 31) == 0) sh.part_i[rb][threadIdx.x >> 5] = v;
  __syncthreads();
  int r = -0x7fffffff - 1;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r = max(r, sh.part_i[rb][i]);
  rb ^= 1;
  return r;
}

// Block argmax of (value, tie) under arg_better; returns the winner's payload.
// Threads without a candidate pass (-inf, INT_MAX, *).
template <int NT, int E>
Q3S_DEV int block_argmax(float v, int tie, int payload, Scratch<NT, E>& sh, int& rb) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(FULL, v, o);
    const int ot = __shfl_xor_sync(FULL, tie, o);
    const int op = __shfl_xor_sync(FULL, payload, o);
    if (arg_better(ov, ot, v, tie)) { v = ov; tie = ot; payload = op; }
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sh.part_f[rb][w] = v;
    sh.part_i[rb][w] = tie;
    sh.part_u[rb][w] = static_cast<uint32_t>(payload);
  }
  __syncthreads();
  float bv = sh.part_f[rb][0];
  int bt = sh.part_i[rb][0];
  int bp = static_cast<int>(sh.part_u[rb][0]);
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) {
    if (arg_better(sh.part_f[rb][i], sh.part_i[rb][i], bv, bt)) {
      bv = sh.part_f[rb][i];
      bt = sh.part_i[rb][i];
      bp = static_cast<int>(sh.part_u[rb][i]);
    }
  }
  rb ^= 1;
  return bp;
}

// Exclusive scan of a count over threads (thread order = vocabulary order),
// fused with a block max of `mx`.
template <int NT, int E>
Q3S_DEV uint32_t block_scan_count_max(uint32_t v, float mx, uint32_t& total, float& bmax, Scratch<NT, E>& sh,
                                      int& rb) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc += n;
  }
  mx = warp_max_f(mx);
  if (lane == 31) {
    sh.part_u[rb][w] = inc;
    sh.part_f[rb][w] = mx;
  }
  __syncthreads();
  uint32_t pre = 0, tot = 0;
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) {
    const uint32_t x = sh.part_u[rb][i];
    pre += (i < w) ? x : 0u;
    tot += x;
    m = fmaxf(m, sh.part_f[rb][i]);
  }
  rb ^= 1;
  total = tot;
  bmax = m;
  return pre + inc - v;
}

template <int NT, int E>
Q3S_DEV uint32_t block_excl_scan_u(uint32_t v, uint32_t& total, Scratch<NT, E>& sh, int& rb) {
  float ignore;
  return block_scan_count_max<NT, E>(v, -INFINITY, total, ignore, sh, rb);
}

// Exclusive fp32 scan over threads (vocabulary order); total = sum of all.
template <int NT, int E>
Q3S_DEV float block_excl_scan_f(float v, float& total, Scratch<NT, E>& sh, int& rb) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float n = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc = __fadd_rn(inc, n);
  }
  float ex = __shfl_up_sync(FULL, inc, 1);
  if (lane == 0) ex = 0.0f;
  if (lane == 31) sh.part_f2[rb][w] = inc;
  __syncthreads();
  float pre = 0.0f, tot = 0.0f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) {
    const float x = sh.part_f2[rb][i];
    if (i < w) pre = __fadd_rn(pre, x);
    tot = __fadd_rn(tot, x);
  }
  rb ^= 1;
  total = tot;
  return __fadd_rn(pre, ex);
}

// ---------------------------------------------------------------------------
// radix selection (8-bit digits, MSB first, 256-bin histograms)
// ---------------------------------------------------------------------------

// Warp 0: find the bin holding the krem-th largest counted entry.  Lane l
// owns bins [8l, 8l+8) (two 16-byte loads, kept in registers); a suffix scan
// over lanes picks the lane, which then walks its own 8 bins.  Clears the
// histogram.  sel = {bin, count in bin, rank left within the bin}.
Q3S_DEV void scan_count_desc(uint32_t* hist, uint32_t krem, uint32_t* sel) {
  const int lane = threadIdx.x;
  uint4* hb = reinterpret_cast<uint4*>(hist) + 2 * lane;
  const uint4 a = hb[0], b = hb[1];
  const uint32_t c[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  const uint32_t s = (c[0] + c[1]) + (c[2] + c[3]) + (c[4] + c[5]) + (c[6] + c[7]);
  uint32_t suf = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_down_sync(FULL, suf, o);
    if (lane + o < 32) suf += n;
  }
  const uint32_t above = suf - s;
  if (above < krem && krem <= suf) {
    uint32_t acc = above;
    bool found = false;
#pragma unroll
    for (int i = 7; i >= 0; --i) {
      if (!found && acc + c[i] >= krem) {
        found = true;
        sel[0] = static_cast<uint32_t>(8 * lane + i);
        sel[1] = c[i];
        sel[2] = krem - acc;
      }
      acc += c[i];
    }
  }
  hb[0] = make_uint4(0, 0, 0, 0);
  hb[1] = make_uint4(0, 0, 0, 0);
}

// As scan_count_desc, also recording the count of the next bin down in
// sel[3] (0 below bin 0); sel[0] = 0xffffffff when fewer than krem entries
// are counted.
Q3S_DEV void scan_count_desc_next(uint32_t* hist, uint32_t krem, uint32_t* sel) {
  const int lane = threadIdx.x;
  uint4* hb = reinterpret_cast<uint4*>(hist) + 2 * lane;
  const uint4 a = hb[0], b = hb[1];
  const uint32_t c[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  const uint32_t below0 = __shfl_up_sync(FULL, c[7], 1);  // bin 8 lane - 1
  const uint32_t s = (c[0] + c[1]) + (c[2] + c[3]) + (c[4] + c[5]) + (c[6] + c[7]);
  uint32_t suf = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_down_sync(FULL, suf, o);
    if (lane + o < 32) suf += n;
  }
  const uint32_t above = suf - s;
  const bool hit = above < krem && krem <= suf;
  if (hit) {
    uint32_t acc = above;
    bool found = false;
#pragma unroll
    for (int i = 7; i >= 0; --i) {
      if (!found && acc + c[i] >= krem) {
        found = true;
        sel[0] = static_cast<uint32_t>(8 * lane + i);
        sel[1] = c[i];
        sel[2] = krem - acc;
        sel[3] = i > 0 ? c[i > 0 ? i - 1 : 0] : (lane > 0 ? below0 : 0u);
      }
      acc += c[i];
    }
  }
  if (__ballot_sync(FULL, hit) == 0u && lane == 0) sel[0] = 0xffffffffu;
  hb[0] = make_uint4(0, 0, 0, 0);
  hb[1] = make_uint4(0, 0, 0, 0);
}

// Candidates for the k largest of the values xa (flagged in `mask`) from one
// histogram of d = max - xa in bins 1/8 wide over d < 32: every entry down to
// the bin below the one holding the k-th largest.  With every value in
// [-2000, 2000] an ulp is <= 2^-12, far inside a bin, so values within a few
// ulps of the ones ranked (approximate keys, temperature-quotient ties) stay
// in the set.  Returns false, leaving the histogram clear, when that does not
// apply (NaN, values outside the window, the k-th 32 or more below the top,
// or more than `stop` candidates); every thread returns the same.
template <int NT, int E>
Q3S_DEV bool select_bins8(const float (&xa)[E], uint32_t mask, int k, int stop, Scratch<NT, E>& sh, int& rb,
                          uint32_t& cmask) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float mx = -INFINITY;
  bool bad = false;
#pragma unroll
  for (int j = 0; j < E; ++j)
    if ((mask >> j) & 1u) {
      mx = fmaxf(mx, xa[j]);
      bad |= xa[j] != xa[j];
    }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
  const bool wbad = __any_sync(FULL, bad);
  if (lane == 0) {
    sh.part_f[rb][w] = mx;
    sh.part_i[rb][w] = wbad;
  }
  __syncthreads();
  float amax = sh.part_f[rb][0];
  int anyb = sh.part_i[rb][0];
#pragma unroll
  for (int i = 1; i < NW; ++i) {
    amax = fmaxf(amax, sh.part_f[rb][i]);
    anyb |= sh.part_i[rb][i];
  }
  rb ^= 1;
  if (anyb || !(fabsf(amax) <= 2000.0f)) return false;
#pragma unroll
  for (int j = 0; j < E; ++j)
    if ((mask >> j) & 1u) {
      const float e = __fmul_rn(__fsub_rn(amax, xa[j]), 8.0f);
      if (e < 256.0f) atomicAdd(&sh.hist[0][255u - static_cast<uint32_t>(e)], 1u);
    }
  __syncthreads();
  if (threadIdx.x < 32) scan_count_desc_next(sh.hist[0], static_cast<uint32_t>(k), sh.sel_u);
  __syncthreads();
  const uint32_t d = sh.sel_u[0];
  if (d == 0xffffffffu) return false;
  const uint32_t b8 = 255u - d;
  const uint32_t n8 = (static_cast<uint32_t>(k) - sh.sel_u[2]) + sh.sel_u[1] + sh.sel_u[3];
  if (b8 > 253u || n8 > static_cast<uint32_t>(stop)) return false;
  const float ecut = static_cast<float>(b8 + 2u);
  cmask = 0;
#pragma unroll
  for (int j = 0; j < E; ++j)
    if (((mask >> j) & 1u) && __fmul_rn(__fsub_rn(amax, xa[j]), 8.0f) < ecut) cmask |= 1u << j;
  return true;
}

// Key of the k-th largest entry (1-based k, multiplicity counted) among the
// entries flagged in `mask`.  Stops early once the chosen bucket holds exactly
// the entries still needed (the answer is then that bucket's minimum).
template <int NT, int E>
Q3S_DEV uint32_t select_kth_largest(const uint32_t (&key)[E], uint32_t mask, int k, Scratch<NT, E>& sh,
                                    int& rb) {
  uint32_t prefix = 0, hmask = 0;
  int krem = k;
  uint32_t* hist = sh.hist[0];
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (((mask >> j) & 1u) && (key[j] & hmask) == prefix) atomicAdd(&hist[(key[j] >> shift) & 255u], 1u);
    __syncthreads();
    if (threadIdx.x < 32) scan_count_desc(hist, static_cast<uint32_t>(krem), sh.sel_u);
    __syncthreads();
    const uint32_t d = sh.sel_u[0];
    const uint32_t cnt = sh.sel_u[1];
    krem = static_cast<int>(sh.sel_u[2]);
    prefix |= d << shift;
    hmask |= 255u << shift;
    if (shift > 0 && cnt == static_cast<uint32_t>(krem)) {
      uint32_t mn = 0xffffffffu;
#pragma unroll
      for (int j = 0; j < E; ++j)
        if (((mask >> j) & 1u) && (key[j] & hmask) == prefix) mn = min(mn, key[j]);
      return block_min_u<NT, E>(mn, sh, rb);
    }
  }
  return prefix;
}

// A key threshold with at least k flagged entries at or above it, and no more
// than `stop` when the radix passes allow stopping early: the lower edge of
// the bin holding the k-th largest key once that bin and everything above it
// hold <= stop entries (the exact k-th largest key otherwise).
template <int NT, int E>
Q3S_DEV uint32_t select_threshold(const uint32_t (&key)[E], uint32_t mask, int k, int stop, Scratch<NT, E>& sh,
                                  int& rb) {
  uint32_t prefix = 0, hmask = 0;
  int krem = k;
  uint32_t* hist = sh.hist[0];
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (((mask >> j) & 1u) && (key[j] & hmask) == prefix) atomicAdd(&hist[(key[j] >> shift) & 255u], 1u);
    __syncthreads();
    if (threadIdx.x < 32) scan_count_desc(hist, static_cast<uint32_t>(krem), sh.sel_u);
    __syncthreads();
    const uint32_t d = sh.sel_u[0];
    const uint32_t cnt = sh.sel_u[1];
    krem = static_cast<int>(sh.sel_u[2]);
    prefix |= d << shift;
    hmask |= 255u << shift;
    // entries strictly above the bin: k - krem; in it: cnt
    if (k - krem + static_cast<int>(cnt) <= stop) return prefix;
  }
  return prefix;
}

// Warp 0: first bin (ascending) where below + cumulative mass exceeds tau, in
// the mass histograms (high / low 32-bit parts).  Clears them.
// sel_u[0] = bin, sel_q[0] = mass before that bin.
Q3S_DEV void scan_mass_asc(uint32_t* hhi, uint32_t* hlo, unsigned long long below, unsigned long long tau,
                           uint32_t* sel_u, unsigned long long* sel_q) {
  const int lane = threadIdx.x;
  uint4* ph = reinterpret_cast<uint4*>(hhi) + 2 * lane;
  uint4* pl = reinterpret_cast<uint4*>(hlo) + 2 * lane;
  const uint4 h0 = ph[0], h1 = ph[1], l0 = pl[0], l1 = pl[1];
  const uint32_t hi[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  const uint32_t lo[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
  unsigned long long c[8], s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    c[i] = (static_cast<unsigned long long>(hi[i]) << MASS_LO_BITS) + lo[i];
    s += c[i];
  }
  unsigned long long inc = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long n = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc += n;
  }
  const unsigned long long lo0 = below + (inc - s);
  if (lo0 <= tau && tau < below + inc) {
    unsigned long long acc = lo0;
    bool found = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (!found && acc + c[i] > tau) {
        found = true;
        sel_u[0] = static_cast<uint32_t>(8 * lane + i);
        sel_q[0] = acc;
      }
      acc += c[i];
    }
  }
  ph[0] = make_uint4(0, 0, 0, 0);
  ph[1] = make_uint4(0, 0, 0, 0);
  pl[0] = make_uint4(0, 0, 0, 0);
  pl[1] = make_uint4(0, 0, 0, 0);
}

// Top-p cut by mass in ascending order (value asc, index asc -- a stable
// ascending sort).  w are the entries' softmax weights; finds the smallest
// key v with mass(key <= v) > tau, and mass(key < v).  Masses are fixed point,
// accumulated exactly in two 32-bit histograms (high and low parts), so the
// result does not depend on the order of the atomics.
template <int NT, int E>
Q3S_DEV void select_mass_cut(const uint32_t (&key)[E], const float (&w)[E], uint32_t mask,
                             unsigned long long tau, Scratch<NT, E>& sh, uint32_t& vstar,
                             unsigned long long& below_out) {
  uint32_t prefix = 0, hmask = 0;
  unsigned long long below = 0;
  uint32_t* hhi = sh.hist[0];
  uint32_t* hlo = sh.hist[1];
  constexpr uint32_t LO = (1u << MASS_LO_BITS) - 1u;
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const unsigned long long q = ((mask >> j) & 1u) ? mass_fixed(w[j]) : 0ull;
      if (q != 0 && (key[j] & hmask) == prefix) {
        const uint32_t bin = (key[j] >> shift) & 255u;
        atomicAdd(&hhi[bin], static_cast<uint32_t>(q >> MASS_LO_BITS));
        atomicAdd(&hlo[bin], static_cast<uint32_t>(q) & LO);
      }
    }
    __syncthreads();
    if (threadIdx.x < 32) scan_mass_asc(hhi, hlo, below, tau, sh.sel_u, sh.sel_q);
    __syncthreads();
    prefix |= sh.sel_u[0] << shift;
    below = sh.sel_q[0];
    hmask |= 255u << shift;
  }
  vstar = prefix;
  below_out = below;
}

}  // namespace q3s
