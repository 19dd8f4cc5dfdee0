// q3s_warp.cuh -- shared-memory-resident row sampler (icdf mode), one CTA of
// W warps per row (W = 1, 2, 4 or 8, chosen by the batch size).
//
// The row arrives with one bulk copy (cp.async.bulk, completion on an
// mbarrier) while the CTA scatters the row's history, and stays in shared
// memory; every pass over it is a rolled loop of 16-byte shared loads --
// lane l of warp w reads quad h = l + 32 r (entries [4h, 4h+4)) for the
// rounds r of its block [w RQ/W, (w+1) RQ/W), so a warp's load covers 512
// contiguous bytes without bank conflicts and each warp's block is a
// contiguous range of the vocabulary.  Vocabulary order is quad order:
// round r, then lane l, then entry j.  W = 1 takes no block barrier at all;
// W > 1 trades barriers for a W-times shorter chain of dependent work per
// row (small batches are latency-bound, large ones throughput-bound).
//
// The arithmetic and the tie rules are those of the CTA-per-row kernels in
// q3s_sampler.cu (HF LogitsProcessorList order, transformers
// generation/logits_process.py, as driven by the reference's
// qwen_tts/core/models/modeling_qwen3_tts.py:1591-1611 generate() call):
// suppress -> repetition penalty -> EOS gate -> temperature -> top-k (ties
// kept) -> top-p (stable ascending order) -> softmax -> inverse CDF.
#pragma once

#include <type_traits>

#include "q3s_args.cuh"
#include "q3s_device.cuh"

namespace q3s {

constexpr int WCAP = 256;              // candidate records per row
constexpr int COARSE_SHIFT = 19;       // coarse bin: exponent and top 4 mantissa bits of w (16 bins per octave)
constexpr int COARSE_BIN0 = (0x3f800000 >> COARSE_SHIFT) - 255;  // w = 1 -> bin 255; w < 2^-15.9 -> bin 0

Q3S_DEV int lane_id() { return static_cast<int>(threadIdx.x & 31u); }

// ---------------------------------------------------------------------------
// warp scans over a 256-bin histogram; each lane owns bins 8l..8l+7 and
// clears them after reading (the zero invariant of RowSmem::hist)
// ---------------------------------------------------------------------------

// Bin of the krem-th largest entry (bins descending): returns the bin, its
// count and the rank left inside it.
Q3S_DEV void warp_scan_count_desc(uint32_t* hist, uint32_t krem, uint32_t& d, uint32_t& cnt, uint32_t& knew) {
  const int lane = lane_id();
  uint4* hb = reinterpret_cast<uint4*>(hist) + 2 * lane;
  const uint4 a = hb[0], b = hb[1];
  const uint32_t c[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  const uint32_t s = (c[0] + c[1]) + (c[2] + c[3]) + (c[4] + c[5]) + (c[6] + c[7]);
  uint32_t suf = s;  // inclusive suffix sum over lanes >= this one
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_down_sync(FULL, suf, o);
    if (lane + o < 32) suf += n;
  }
  const uint32_t above = suf - s;
  const bool hit = above < krem && krem <= suf;
  uint32_t md = 0, mc = 0, mk = 0;
  if (hit) {
    uint32_t acc = above;
    bool found = false;
#pragma unroll
    for (int i = 7; i >= 0; --i) {
      if (!found && acc + c[i] >= krem) {
        found = true;
        md = static_cast<uint32_t>(8 * lane + i);
        mc = c[i];
        mk = krem - acc;
      }
      acc += c[i];
    }
  }
  hb[0] = make_uint4(0, 0, 0, 0);
  hb[1] = make_uint4(0, 0, 0, 0);
  const int src = (__ffs(__ballot_sync(FULL, hit)) - 1) & 31;
  d = __shfl_sync(FULL, md, src);
  cnt = __shfl_sync(FULL, mc, src);
  knew = __shfl_sync(FULL, mk, src);
  __syncwarp();
}

// As warp_scan_count_desc, without clearing the bins (several warps may scan
// the same histogram).
Q3S_DEV void warp_scan_count_desc_keep(const uint32_t* hist, uint32_t krem, uint32_t& d, uint32_t& knew) {
  const int lane = lane_id();
  const uint4* hb = reinterpret_cast<const uint4*>(hist) + 2 * lane;
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
  const bool hit = above < krem && krem <= suf;
  uint32_t md = 0, mk = 0;
  if (hit) {
    uint32_t acc = above;
    bool found = false;
#pragma unroll
    for (int i = 7; i >= 0; --i) {
      if (!found && acc + c[i] >= krem) {
        found = true;
        md = static_cast<uint32_t>(8 * lane + i);
        mk = krem - acc;
      }
      acc += c[i];
    }
  }
  const int src = (__ffs(__ballot_sync(FULL, hit)) - 1) & 31;
  d = __shfl_sync(FULL, md, src);
  knew = __shfl_sync(FULL, mk, src);
}

// Exact fixed-point masses (hi/lo histograms), bins ascending: the first bin
// where below + mass up to it exceeds tau, and the mass before it.
Q3S_DEV void warp_scan_mass_asc(uint32_t* hhi, uint32_t* hlo, unsigned long long below, unsigned long long tau,
                                uint32_t& d, unsigned long long& before) {
  const int lane = lane_id();
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
  const bool hit = lo0 <= tau && tau < below + inc;
  uint32_t md = 0;
  unsigned long long mb = 0;
  if (hit) {
    unsigned long long acc = lo0;
    bool found = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (!found && acc + c[i] > tau) {
        found = true;
        md = static_cast<uint32_t>(8 * lane + i);
        mb = acc;
      }
      acc += c[i];
    }
  }
  ph[0] = make_uint4(0, 0, 0, 0);
  ph[1] = make_uint4(0, 0, 0, 0);
  pl[0] = make_uint4(0, 0, 0, 0);
  pl[1] = make_uint4(0, 0, 0, 0);
  const int src = (__ffs(__ballot_sync(FULL, hit)) - 1) & 31;
  d = __shfl_sync(FULL, md, src);
  before = __shfl_sync(FULL, mb, src);
  __syncwarp();
}

Q3S_DEV float warp_excl_scan_f(float v, float& total) {
  const int lane = lane_id();
  float inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float n = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc = __fadd_rn(inc, n);
  }
  float ex = __shfl_up_sync(FULL, inc, 1);
  if (lane == 0) ex = 0.0f;
  total = __shfl_sync(FULL, inc, 31);
  return ex;
}

Q3S_DEV uint32_t warp_excl_scan_u(uint32_t v, uint32_t& total) {
  const int lane = lane_id();
  uint32_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc += n;
  }
  total = __shfl_sync(FULL, inc, 31);
  return inc - v;
}

Q3S_DEV unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// candidate lists (positions in vocabulary order)
// ---------------------------------------------------------------------------

// Inverse CDF over a list's kept weights in vocabulary order: the first
// position whose running sum exceeds u * total.  Lane l owns positions
// [l P, l P + P), P = ceil(n / 32) <= 8 (n <= WCAP) -- the association order
// of the CTA kernels' warp-0 finisher, so both produce the same sums.  wk[p]
// is the weight of position p, 0 for removed entries and for n <= p < 32 P.
// Each lane reads its weights once, into registers.
Q3S_DEV int warp_draw_list(const float* wk, int n, float u, int& flags) {
  const int lane = lane_id();
  const int P = (n + 31) / 32;
  float w[WCAP / 32];
#pragma unroll
  for (int r = 0; r < WCAP / 32; ++r) w[r] = r < P ? wk[lane * P + r] : 0.0f;
  // adding the +0 weights past P leaves every sum unchanged
  float a = 0.0f;
#pragma unroll
  for (int r = 0; r < WCAP / 32; ++r) a = __fadd_rn(a, w[r]);
  float W;
  const float pre = warp_excl_scan_f(a, W);
  const float thr = __fmul_rn(u, W);
  // cumulative weight through position l P + r: pre + (w_0 + ... + w_r)
  int r_first = -1, r_last = -1;
  float part = 0.0f, cdf_f = 0.0f, prev_f = 0.0f, cdf_l = 0.0f, prev_l = 0.0f;
#pragma unroll
  for (int r = 0; r < WCAP / 32; ++r) {
    const float before = __fadd_rn(pre, part);
    part = __fadd_rn(part, w[r]);
    const float c = __fadd_rn(pre, part);
    if (w[r] > 0.0f) {
      r_last = r;
      cdf_l = c;
      prev_l = before;
      if (r_first < 0 && c > thr) {
        r_first = r;
        cdf_f = c;
        prev_f = before;
      }
    }
  }
  const unsigned hit = __ballot_sync(FULL, r_first >= 0);
  int src, rsel;
  if (hit) {
    src = __ffs(hit) - 1;
    rsel = __shfl_sync(FULL, r_first, src);
  } else {
    const unsigned any = __ballot_sync(FULL, r_last >= 0);
    src = any ? 31 - __clz(any) : 0;
    rsel = any ? __shfl_sync(FULL, r_last, src) : 0;
    flags |= Q3S_ROW_FALLBACK;
  }
  const float cdf = hit ? cdf_f : cdf_l, prev = hit ? prev_f : prev_l;
  const float tol = BOUNDARY_EPS * W;
  const int near = (__fsub_rn(cdf, thr) < tol) || (__fsub_rn(thr, prev) < tol);
  if (__shfl_sync(FULL, near, src)) flags |= Q3S_ROW_DRAW_BOUNDARY;
  return src * P + rsel;
}

// Exclusive prefix over the lanes of a small count (0..7) and the warp total,
// from three ballots.
Q3S_DEV uint32_t warp_excl_small(uint32_t c, uint32_t& total) {
  const uint32_t lt = (1u << lane_id()) - 1u;
  const unsigned b0 = __ballot_sync(FULL, c & 1u), b1 = __ballot_sync(FULL, c & 2u), b2 = __ballot_sync(FULL, c & 4u);
  total = __popc(b0) + 2u * __popc(b1) + 4u * __popc(b2);
  return __popc(b0 & lt) + 2u * __popc(b1 & lt) + 4u * __popc(b2 & lt);
}

// Exact fixed-point masses in a coarse histogram (hi/lo parts), bins
// ascending: the total Zq, tau = floor(frac * Zq), the first bin where the
// running mass exceeds tau and the mass before it (d = 255, before = Zq when
// tau >= Zq).  Clears the bins.
Q3S_DEV void warp_scan_mass_total(uint32_t* hhi, uint32_t* hlo, float frac, unsigned long long& Zq,
                                  unsigned long long& tau, uint32_t& d, unsigned long long& before) {
  const int lane = lane_id();
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
  Zq = __shfl_sync(FULL, inc, 31);
  tau = __double2ull_rd(static_cast<double>(frac) * static_cast<double>(Zq));
  const unsigned long long lo0 = inc - s;
  const bool hit = lo0 <= tau && tau < inc;
  uint32_t md = 0;
  unsigned long long mb = 0;
  if (hit) {
    unsigned long long acc = lo0;
    bool found = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (!found && acc + c[i] > tau) {
        found = true;
        md = static_cast<uint32_t>(8 * lane + i);
        mb = acc;
      }
      acc += c[i];
    }
  }
  ph[0] = make_uint4(0, 0, 0, 0);
  ph[1] = make_uint4(0, 0, 0, 0);
  pl[0] = make_uint4(0, 0, 0, 0);
  pl[1] = make_uint4(0, 0, 0, 0);
  const unsigned bal = __ballot_sync(FULL, hit);
  d = bal ? __shfl_sync(FULL, md, __ffs(bal) - 1) : 255u;
  before = bal ? __shfl_sync(FULL, mb, __ffs(bal) - 1) : Zq;
  __syncwarp();
}

// Bin of an entry d >= 0 below the row's largest approximate value, bins of
// width 1/scale from d0 on: floor((d - d0) * scale), 255 from 255/scale on
// (entries above d0 -- d < d0 -- are not binned).  Monotone in d.
Q3S_DEV uint32_t top_bin(float d, float d0, float scale) {
  const float e = __fmul_rn(__fsub_rn(d, d0), scale);
  return e < 255.0f ? static_cast<uint32_t>(e) : 255u;
}

// As warp_scan_mass_total, without clearing the bins (several warps may scan
// the same histogram).
Q3S_DEV void warp_scan_mass_total_keep(const uint32_t* hhi, const uint32_t* hlo, float frac, unsigned long long& Zq,
                                       unsigned long long& tau, uint32_t& d, unsigned long long& before) {
  const int lane = lane_id();
  const uint4* ph = reinterpret_cast<const uint4*>(hhi) + 2 * lane;
  const uint4* pl = reinterpret_cast<const uint4*>(hlo) + 2 * lane;
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
  Zq = __shfl_sync(FULL, inc, 31);
  tau = __double2ull_rd(static_cast<double>(frac) * static_cast<double>(Zq));
  const unsigned long long lo0 = inc - s;
  const bool hit = lo0 <= tau && tau < inc;
  uint32_t md = 0;
  unsigned long long mb = 0;
  if (hit) {
    unsigned long long acc = lo0;
    bool found = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (!found && acc + c[i] > tau) {
        found = true;
        md = static_cast<uint32_t>(8 * lane + i);
        mb = acc;
      }
      acc += c[i];
    }
  }
  const unsigned bal = __ballot_sync(FULL, hit);
  d = bal ? __shfl_sync(FULL, md, __ffs(bal) - 1) : 255u;
  before = bal ? __shfl_sync(FULL, mb, __ffs(bal) - 1) : Zq;
}

Q3S_DEV uint32_t coarse_bin(float w) {
  const int e = static_cast<int>(__float_as_uint(w) >> COARSE_SHIFT) - COARSE_BIN0;
  return static_cast<uint32_t>(min(255, max(0, e)));
}

// ---------------------------------------------------------------------------
// per-row shared memory and the CTA-level steps (W warps share one row)
// ---------------------------------------------------------------------------

template <int R, int W>
struct alignas(16) RowSmem {
  static constexpr int RQ = 2 * R;       // rounds of one quad (4 entries) per lane
  static constexpr int RPW = RQ / W;     // rounds per warp
  static constexpr int VMAX = 128 * RQ;  // entries the row buffer holds
  float4 row[32 * RQ];                   // quad h: logits as loaded -> x' -> s -> softmax weights
  uint32_t hist[2][NBINS];               // counts / mass high parts, mass low parts; zero between uses
  union {
    uint8_t seen[VMAX];                  // presence flags from the packed history (dead after the first pass)
    uint4 cand[WCAP];                    // candidate records {s bits, index, x' bits, weight bits}
    float ex[32 * RQ];                   // draw: cumulative weight before each quad, within its warp's block
  } u;
  uint8_t appb[32 * RQ];                 // quad h: presence bits (low 4), suppress bits (high 4)
  uint8_t cmask[32 * RQ];                // candidate bits of quad h (low 4 bits)
  uint8_t keep[WCAP];
  float xf[2][W];                        // cross-warp exchange, double-buffered
  float xf2[2][W];
  int xi[2][W];
  unsigned long long xq[2][W];
  unsigned long long xq2[2][W];
  uint32_t sel[4];                       // a leader warp's results
  unsigned long long selq[4];
  int res[4];
  int lcnt[2];                           // list counters (band, crossing-bin entries)
  uint64_t bar;                          // completion of the logits bulk copy
};

template <int W>
Q3S_DEV void row_sync() {
  if (W == 1)
    __syncwarp();
  else
    __syncthreads();
}

// CTA-wide exchanges: each takes one barrier (none for W = 1) and combines
// the per-warp values in warp order, so the results are reproducible.
template <int R, int W>
struct RowX {
  RowSmem<R, W>& sh;
  int wi, lane, tg = 0;
  Q3S_DEV float max_f(float v) {
    v = warp_max_f(v);
    if (W == 1) return v;
    if (lane == 0) sh.xf[tg][wi] = v;
    __syncthreads();
    float m = sh.xf[tg][0];
#pragma unroll
    for (int i = 1; i < W; ++i) m = fmaxf(m, sh.xf[tg][i]);
    tg ^= 1;
    return m;
  }
  Q3S_DEV float min_f(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fminf(v, __shfl_xor_sync(FULL, v, o));
    if (W == 1) return v;
    if (lane == 0) sh.xf[tg][wi] = v;
    __syncthreads();
    float m = sh.xf[tg][0];
#pragma unroll
    for (int i = 1; i < W; ++i) m = fminf(m, sh.xf[tg][i]);
    tg ^= 1;
    return m;
  }
  Q3S_DEV unsigned long long min_q(unsigned long long v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long ov = __shfl_xor_sync(FULL, v, o);
      v = ov < v ? ov : v;
    }
    if (W == 1) return v;
    if (lane == 0) sh.xq[tg][wi] = v;
    __syncthreads();
    unsigned long long m = sh.xq[tg][0];
#pragma unroll
    for (int k = 1; k < W; ++k) m = sh.xq[tg][k] < m ? sh.xq[tg][k] : m;
    tg ^= 1;
    return m;
  }
  Q3S_DEV int max_i(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(FULL, v, o));
    if (W == 1) return v;
    if (lane == 0) sh.xi[tg][wi] = v;
    __syncthreads();
    int m = sh.xi[tg][0];
#pragma unroll
    for (int i = 1; i < W; ++i) m = max(m, sh.xi[tg][i]);
    tg ^= 1;
    return m;
  }
  Q3S_DEV int min_i(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = min(v, __shfl_xor_sync(FULL, v, o));
    if (W == 1) return v;
    if (lane == 0) sh.xi[tg][wi] = v;
    __syncthreads();
    int m = sh.xi[tg][0];
#pragma unroll
    for (int i = 1; i < W; ++i) m = min(m, sh.xi[tg][i]);
    tg ^= 1;
    return m;
  }
  // torch.argmax order over (value, index) pairs
  Q3S_DEV void argmax(float& v, int& i) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(FULL, v, o);
      const int oi = __shfl_xor_sync(FULL, i, o);
      if (arg_better(ov, oi, v, i)) {
        v = ov;
        i = oi;
      }
    }
    if (W == 1) return;
    if (lane == 0) {
      sh.xf[tg][wi] = v;
      sh.xi[tg][wi] = i;
    }
    __syncthreads();
    v = sh.xf[tg][0];
    i = sh.xi[tg][0];
#pragma unroll
    for (int k = 1; k < W; ++k)
      if (arg_better(sh.xf[tg][k], sh.xi[tg][k], v, i)) {
        v = sh.xf[tg][k];
        i = sh.xi[tg][k];
      }
    tg ^= 1;
  }
  // exclusive prefix (warp order) of one uint per warp; total out
  Q3S_DEV uint32_t prefix_u(uint32_t warp_total, uint32_t& total) {
    if (W == 1) {
      total = warp_total;
      return 0u;
    }
    if (lane == 0) sh.xi[tg][wi] = static_cast<int>(warp_total);
    __syncthreads();
    uint32_t pre = 0, tot = 0;
#pragma unroll
    for (int k = 0; k < W; ++k) {
      const uint32_t t = static_cast<uint32_t>(sh.xi[tg][k]);
      if (k < wi) pre += t;
      tot += t;
    }
    tg ^= 1;
    total = tot;
    return pre;
  }
  // exclusive prefix (warp order, sequential fp32 adds) of one float per warp
  Q3S_DEV float prefix_f(float warp_total, float& total) {
    if (W == 1) {
      total = warp_total;
      return 0.0f;
    }
    if (lane == 0) sh.xf[tg][wi] = warp_total;
    __syncthreads();
    float pre = 0.0f, tot = 0.0f;
#pragma unroll
    for (int k = 0; k < W; ++k) {
      if (k == wi) pre = tot;
      tot = __fadd_rn(tot, sh.xf[tg][k]);
    }
    tg ^= 1;
    total = tot;
    return pre;
  }
  Q3S_DEV unsigned long long max_q(unsigned long long v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long ov = __shfl_xor_sync(FULL, v, o);
      v = ov > v ? ov : v;
    }
    if (W == 1) return v;
    if (lane == 0) sh.xq[tg][wi] = v;
    __syncthreads();
    unsigned long long m = sh.xq[tg][0];
#pragma unroll
    for (int k = 1; k < W; ++k) m = sh.xq[tg][k] > m ? sh.xq[tg][k] : m;
    tg ^= 1;
    return m;
  }
  // two maxima in one exchange
  Q3S_DEV void max2_q(unsigned long long& a0, unsigned long long& a1) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long o0 = __shfl_xor_sync(FULL, a0, o), o1 = __shfl_xor_sync(FULL, a1, o);
      a0 = o0 > a0 ? o0 : a0;
      a1 = o1 > a1 ? o1 : a1;
    }
    if (W == 1) return;
    if (lane == 0) {
      sh.xq[tg][wi] = a0;
      sh.xq2[tg][wi] = a1;
    }
    __syncthreads();
    a0 = sh.xq[tg][0];
    a1 = sh.xq2[tg][0];
#pragma unroll
    for (int k = 1; k < W; ++k) {
      a0 = sh.xq[tg][k] > a0 ? sh.xq[tg][k] : a0;
      a1 = sh.xq2[tg][k] > a1 ? sh.xq2[tg][k] : a1;
    }
    tg ^= 1;
  }
  Q3S_DEV void max2_f(float& a0, float& a1) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      a0 = fmaxf(a0, __shfl_xor_sync(FULL, a0, o));
      a1 = fmaxf(a1, __shfl_xor_sync(FULL, a1, o));
    }
    if (W == 1) return;
    if (lane == 0) {
      sh.xf[tg][wi] = a0;
      sh.xf2[tg][wi] = a1;
    }
    __syncthreads();
    a0 = sh.xf[tg][0];
    a1 = sh.xf2[tg][0];
#pragma unroll
    for (int k = 1; k < W; ++k) {
      a0 = fmaxf(a0, sh.xf[tg][k]);
      a1 = fmaxf(a1, sh.xf2[tg][k]);
    }
    tg ^= 1;
  }
  Q3S_DEV unsigned long long sum_q(unsigned long long v) {
    v = warp_sum_u64(v);
    if (W == 1) return v;
    if (lane == 0) sh.xq[tg][wi] = v;
    __syncthreads();
    unsigned long long s = 0;
#pragma unroll
    for (int k = 0; k < W; ++k) s += sh.xq[tg][k];
    tg ^= 1;
    return s;
  }
};

// Radix select over the row (8-bit digits, most significant first), like
// select_threshold for a CTA: the k-th largest key, or earlier, once the
// entries at or above the current bin number at most `stop`, that bin's lower
// edge.  Each warp adds its block's keys to the shared histogram (qk(r, key)
// fills the keys of this lane's quad of round r and returns the mask of
// entries that take part), warp 0 scans it.
template <int R, int W, typename QuadKeys>
Q3S_DEV uint32_t row_select(RowSmem<R, W>& sh, int wi, int k, int stop, QuadKeys qk) {
  constexpr int RPW = RowSmem<R, W>::RPW;
  const int lane = lane_id();
  uint32_t prefix = 0, hmask = 0;
  uint32_t krem = static_cast<uint32_t>(k);
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll 2
    for (int r = wi * RPW; r < (wi + 1) * RPW; ++r) {
      uint32_t key[4];
      const uint32_t act = qk(r, key);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (((act >> j) & 1u) && (key[j] & hmask) == prefix) atomicAdd(&sh.hist[0][(key[j] >> shift) & 255u], 1u);
    }
    row_sync<W>();
    if (wi == 0) {
      uint32_t d, cnt, knew;
      warp_scan_count_desc(sh.hist[0], krem, d, cnt, knew);
      if (lane == 0) {
        sh.sel[0] = d;
        sh.sel[1] = cnt;
        sh.sel[2] = knew;
      }
    }
    row_sync<W>();
    const uint32_t d = sh.sel[0], cnt = sh.sel[1];
    krem = sh.sel[2];
    prefix |= d << shift;
    hmask |= 255u << shift;
    // entries strictly above the bin: k - krem (krem = rank left inside it);
    // in it: cnt
    if (static_cast<int>(static_cast<uint32_t>(k) - krem + cnt) <= stop) return prefix;
  }
  return prefix;
}

// HF TopPLogitsWarper's cut over a candidate list by all-pairs masses, every
// thread of the row taking list positions t, t + 32W, ...: an entry of the
// list (part[p] set) is removed when the exact fixed-point mass at or below
// it in stable ascending order (s asc, index asc), plus `below0` (the mass of
// everything under the list, all removed), is <= tau.  cand[p] = {s bits,
// index, -, -}; mq[q] = the mass of participant q (0 for others and for the
// padding up to n4).  Writes kept flags to kout[p]; ORs Q3S_ROW_TOPP_BOUNDARY
// into *flag_word when a cumulative mass (or below0) lies within eps of tau.
template <int W>
Q3S_DEV void row_cut_list(const uint4* cand, const uint8_t* part, const unsigned long long* mq, uint8_t* kout,
                          int n, int n4, unsigned long long tau, unsigned long long below0, unsigned long long eps,
                          int* flag_word) {
  const int t = static_cast<int>(threadIdx.x);
  bool near = t == 0 && tau - below0 < eps;
  for (int p = t; p < n; p += 32 * W) {
    if (!part[p]) {
      kout[p] = 0;
      continue;
    }
    const uint4 me = cand[p];
    const float sp = __uint_as_float(me.x);
    unsigned long long cum = below0;
    for (int q = 0; q < n4; q += 4) {
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint4 o = cand[q + v];
        const float so = __uint_as_float(o.x);
        const bool before = (so < sp) | ((so == sp) & (o.y <= me.y));
        cum += before ? mq[q + v] : 0ull;
      }
    }
    const bool kp = cum > tau;
    kout[p] = kp;
    near |= kp ? (cum - tau < eps) : (tau - cum < eps);
  }
  if (near) atomicOr(flag_word, Q3S_ROW_TOPP_BOUNDARY);
}

// Kept weights of a list into the draw's transposed layout (positions
// p < 32 ceil(n/32)), then the draw in warp 0.  Returns the chosen position
// in every thread (through res[0]) and ORs the draw's flags into res[1].
template <int R, int W>
Q3S_DEV int row_draw_list(RowSmem<R, W>& sh, const uint8_t* kout, float* wk, int n, float u) {
  const int t = static_cast<int>(threadIdx.x);
  const int P = (n + 31) / 32;
  for (int p = t; p < 32 * P; p += 32 * W)
    wk[p] = (p < n && kout[p]) ? __uint_as_float(sh.u.cand[p].w) : 0.0f;
  row_sync<W>();
  if (t < 32) {
    int lflags = 0;
    const int pos = warp_draw_list(wk, n, u, lflags);
    if (t == 0) {
      sh.res[0] = pos;
      sh.res[1] = lflags;
    }
  }
  row_sync<W>();
  return sh.res[0];
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

// Dynamic shared memory per row: RowSmem, then (bf16 rows) the row as loaded.
template <int R, int W>
constexpr size_t row_smem_bytes(bool bf16) {
  return sizeof(RowSmem<R, W>) + (bf16 ? 2 * RowSmem<R, W>::VMAX : 0);
}

// Resident rows per SM each variant is compiled for (its register budget):
// 64 registers for 16 and 8 warps and for 4-warp bf16 rows, 72 for 4-warp
// fp32 rows and 2 warps, ~120 for one warp; the widest variants run one row
// per SM.  Pinned so that code changes do not move the occupancy.
constexpr int row_min_blocks(int W, bool bf16) {
  return W >= 12 ? 2 : W == 8 ? 4 : W == 4 ? (bf16 ? 8 : 7) : W == 2 ? 14 : 17;
}

// PROC adds the verification-only processed-logits output (the row as HF's
// processors hand it to the draw: x'/T with the entries top-k and top-p
// remove at -inf; greedy rows x'); the timed variants carry none of it.
template <int R, int W, bool BF16, bool PROC>
__global__ void __launch_bounds__(W * 32, row_min_blocks(W, BF16)) sample_smem_kernel(const SampleArgs a) {
  extern __shared__ __align__(16) unsigned char q3s_row_smem[];
  using Smem = RowSmem<R, W>;
  constexpr int RPW = Smem::RPW;
  constexpr int NT = 32 * W;
  Smem& sh = *reinterpret_cast<Smem*>(q3s_row_smem);
  uint16_t* const stage = reinterpret_cast<uint16_t*>(q3s_row_smem + sizeof(Smem));  // bf16 row as loaded
  const int t = static_cast<int>(threadIdx.x);
  const int wi = t >> 5;
  const int lane = t & 31;
  const int b = blockIdx.x;
  const int rb0 = wi * RPW, rb1 = rb0 + RPW;  // this warp's rounds
  float* rowf = reinterpret_cast<float*>(sh.row);  // entry v at rowf[v]
  const int V = a.V;
  uint32_t err = 0;
  RowX<R, W> X{sh, wi, lane};
  // fields read inside loops and lambdas, as locals: nothing may take the
  // address of the parameter block (its loads would then stay in the loops)
  const uint8_t* const suppress = a.suppress;
  const int32_t* const history = a.history;
  const int eos_id = a.eos_id;
  const int esz = BF16 ? 2 : 4;
  const uint32_t row_bytes = static_cast<uint32_t>(V * esz);
  const unsigned char* grow = static_cast<const unsigned char*>(a.logits) + static_cast<int64_t>(b) * a.row_stride * esz;

  // ---- first loads: offsets and the suppress words of this warp's quads
  //      (L2-resident: every row reads them) ---------------------------------
  int o0 = 0, o1 = 0, olen = -1;
  if (history) {
    o0 = __ldg(a.offsets + b);
    o1 = __ldg(a.offsets + b + 1);  // the row's end, or (capacity layout) its region's end
    if (a.history_lengths) olen = __ldg(a.history_lengths + b);
  }
  const float T = a.temperature ? __ldg(a.temperature + b) : a.temperature_default;
  const float pen = a.penalty ? __ldg(a.penalty + b) : a.penalty_default;
  const float top_p = a.top_p ? __ldg(a.top_p + b) : a.top_p_default;
  const int kk = a.top_k ? __ldg(a.top_k + b) : a.K;
  const int min_new = a.min_new ? __ldg(a.min_new + b) : a.min_new_default;
  const float u = a.uniforms ? __ldg(a.uniforms + b) : 0.0f;
  const int cur_given = a.cur_len ? __ldg(a.cur_len + b) : -1;
  uint32_t supw[RPW];
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int h = lane + 32 * (rb0 + i);
    supw[i] = (suppress && 4 * h < V) ? __ldg(reinterpret_cast<const uint32_t*>(suppress + 4 * h)) : 0u;
  }
  // ---- the row's logits stream into shared memory (one plain bulk copy
  //      into this CTA's memory, issued before anything else so that it
  //      overlaps the parameter loads and the history scatter): fp32 rows
  //      straight into the row buffer, bf16 rows into their staging buffer
  //      (kept: the exact values of candidates are read back from it) -------
  // (launched behind the kernel that writes the logits -- a programmatic
  //  dependent -- the copy waits until after the history scatter, below)
  const bool pdl = a.pdl;
  if (t == 0) {
    mbar_init(&sh.bar, 1);
    fence_mbar_init();
    if (!pdl) {
      mbar_expect_tx(&sh.bar, row_bytes);
      bulk_g2s(BF16 ? static_cast<void*>(stage) : static_cast<void*>(sh.row), grow, row_bytes, &sh.bar);
    }
  }
  {
    // zero the histograms and the presence flags (the copy writes neither)
    uint4* hz = reinterpret_cast<uint4*>(&sh.hist[0][0]);
    for (int i = t; i < 2 * NBINS / 4; i += NT) hz[i] = make_uint4(0, 0, 0, 0);
    uint4* sz = reinterpret_cast<uint4*>(sh.u.seen);
    for (int i = t; i < Smem::VMAX / 16; i += NT) sz[i] = make_uint4(0, 0, 0, 0);
  }
  row_sync<W>();

  // presence scatter from the packed history (RepetitionPenalty's gather
  // set); racing stores of the same byte need no atomics
  int hist_len = 0;
  if (history) {
    if (a.history_lengths) o1 = row_end_in_region(o0, o1, olen);
    if (o0 < 0 || o1 < o0 || static_cast<int64_t>(o1) > a.history_len) {
      err |= Q3S_DEVERR_OFFSETS;
      o0 = o1 = 0;
    }
    hist_len = o1 - o0;
    const int32_t* hp = history;
    int mid0 = o0, mid1 = o0;
    if (a.vec_history) {
      mid0 = min(o1, (o0 + 3) & ~3);
      mid1 = mid0 + ((o1 - mid0) & ~3);
    }
    const int nhead = mid0 - o0;
    const int nrest = nhead + (o1 - mid1);
    const int nwork = nrest + (mid1 - mid0) / 4;  // scalar ids first, then 16-byte groups
    constexpr int U = 8;
    constexpr int ST = NT;  // scattering threads
    const int ts = t;
    for (int r0 = ts; r0 < nwork; r0 += U * ST) {
      int4 ids[U];
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int rr = r0 + q * ST;
        ids[q] = make_int4(-1, -1, -1, -1);
        if (rr < nrest)
          ids[q].x = __ldg(hp + (rr < nhead ? o0 + rr : mid1 + (rr - nhead)));
        else if (rr < nwork)
          ids[q] = __ldg(reinterpret_cast<const int4*>(hp + mid0) + (rr - nrest));
      }
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int rr = r0 + q * ST;
        if (rr >= nwork) continue;
        const int nid = rr < nrest ? 1 : 4;
        const int idv[4] = {ids[q].x, ids[q].y, ids[q].z, ids[q].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (i >= nid) break;
          if (static_cast<unsigned>(idv[i]) < static_cast<unsigned>(V))
            sh.u.seen[idv[i]] = 1;
          else
            err |= Q3S_DEVERR_HISTORY_ID;
        }
      }
    }
  }
  const int cur = a.cur_len ? cur_given : hist_len;
  const bool gate = eos_id >= 0 && eos_id < V && cur < min_new;
  if (pdl) {
    // the history and parameters are in; now wait for the grid that writes
    // the logits (its writes are visible after this) and fetch the row
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (t == 0) {
      mbar_expect_tx(&sh.bar, row_bytes);
      bulk_g2s(BF16 ? static_cast<void*>(stage) : static_cast<void*>(sh.row), grow, row_bytes, &sh.bar);
    }
  }

  int id = 0, flags = 0;
  // how the row was finished (read by the processed-logits output only)
  bool list_row = false;             // by the candidate list (non-greedy)
  bool wv_topk = false, wv_cut = false, wv_single = false, wv_nomass = false;
  uint32_t wv_kth = 0;
  const bool greedy = !(T > 0.0f);
  const int K = greedy ? 1 : kk;
  const bool few = greedy || (kk > 0 && kk < V);
  // the candidate path's approximate keys need a penalty and a temperature in
  // the normal window, and room for K plus its margin in WCAP
  const bool window_ok = (pen >= 0x1p-20f && pen <= 0x1p20f) &&
                         (greedy || (T >= 0x1p-20f && T <= 0x1p20f)) && K <= WCAP / 2;
  const bool cand_path = few && window_ok;
  const bool divT = !greedy && T != 1.0f;  // x / 1 == x exactly

  // the presence flags are complete (the mbarrier's initialisation was
  // published by the first barrier); every thread waits for the row
  // (bounded) and all see the same outcome
  row_sync<W>();
  const bool arrived = mbar_wait_bounded(&sh.bar, 0);
  bool all_arrived;
  if (W == 1)
    all_arrived = __all_sync(FULL, arrived);
  else
    all_arrived = __syncthreads_and(arrived) != 0;
  if (!all_arrived) {
    // the copy did not complete in time: report, wait once more (bounded)
    // so that no copy is left writing into a retired CTA's memory, give up
    (void)mbar_wait_bounded(&sh.bar, 0);
    if (t == 0) {
      if (a.ids64) a.ids64[b] = 0;
      if (a.ids32) a.ids32[b] = 0;
      if (a.row_flags) a.row_flags[b] = Q3S_ROW_FALLBACK;
      if (a.error_word) atomicOr(a.error_word, static_cast<int>(err | Q3S_DEVERR_WAIT_TIMEOUT));
    }
    return;
  }

  // the exact x' of entry v (suppress, EOS gate, repetition penalty) and
  // s = x'/T, recomputed from the logits in global memory (L2-resident)
  auto exact_x = [&](int v) -> float {
    float x = BF16 ? bf16_bits_to_f32(stage[v]) : reinterpret_cast<const float*>(grow)[v];
    const uint32_t ab = sh.appb[v >> 2] >> (v & 3);
    if ((ab >> 4) & 1u) x = NEG_SUPPRESS;
    if (gate && v == eos_id) x = -INFINITY;
    if (ab & 1u) x = x > 0.0f ? __fdiv_rn(x, pen) : __fmul_rn(x, pen);
    return x;
  };
  auto exact_s = [&](int v) -> float {
    const float x = exact_x(v);
    return divT ? __fdiv_rn(x, T) : x;
  };
  float lm = -INFINITY, gv = -INFINITY;  // running max of s; torch.argmax of s (greedy rows)
  int gi = 0x7fffffff;
  // candidate rows: the largest approximate value (x * RN(1/pen) for the
  // entries still to divide) and whether any is NaN, seen in the first pass
  const float rpen = __frcp_rn(pen);
  float amax = -INFINITY;
  bool anan = false;

  // ---- first pass: suppress (-1e9, talker_unified_modules.py:409), the EOS
  //      gate (-inf), the repetition penalty.  Candidate rows defer the
  //      division of present entries > 0 (x * RN(1/pen) keys select first);
  //      whole-vocabulary rows compute s = x'/T here.  Branch-free per entry:
  //      the selects replace data-dependent branches; the row's path picks
  //      one of two loops, so neither carries the other's arithmetic -------
  auto first_pass = [&](auto cand_tag, auto divt_tag, auto greedy_tag) {
    constexpr bool IS_CAND = decltype(cand_tag)::value;
    constexpr bool DIVT = decltype(divt_tag)::value, GREEDY = decltype(greedy_tag)::value;
    const uint2* stg = reinterpret_cast<const uint2*>(stage);  // bf16 quad h at stg[h]
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int h = lane + 32 * (rb0 + i);
      const bool in = 4 * h < V;
      float v[4];
      if (BF16) {
        const uint2 q = in ? stg[h] : make_uint2(0u, 0u);
        v[0] = bf16_bits_to_f32(q.x & 0xffffu);
        v[1] = bf16_bits_to_f32(q.x >> 16);
        v[2] = bf16_bits_to_f32(q.y & 0xffffu);
        v[3] = bf16_bits_to_f32(q.y >> 16);
      } else {
        const float4 q = in ? sh.row[h] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        v[0] = q.x;
        v[1] = q.y;
        v[2] = q.z;
        v[3] = q.w;
      }
      if (in) {
        const uint32_t f = history ? *reinterpret_cast<const uint32_t*>(&sh.u.seen[4 * h]) : 0u;
        uint32_t app = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const bool ap = ((f >> (8 * j)) & 0xffu) != 0u;
          app |= (ap ? 1u : 0u) << j;
          const bool sup = ((supw[i] >> (8 * j)) & 0xffu) != 0u;
          app |= (sup ? 16u : 0u) << j;
          float x = sup ? NEG_SUPPRESS : v[j];
          x = (gate && 4 * h + j == eos_id) ? -INFINITY : x;
          if constexpr (IS_CAND) {
            // the approximate value: x * pen for present entries <= 0 (exact),
            // x * RN(1/pen) for present entries > 0 (within 2 ulps of x / pen)
            x = ap ? __fmul_rn(x, x > 0.0f ? rpen : pen) : x;
            amax = fmaxf(amax, x);
            anan |= x != x;
          } else {
            const float dv = __fdiv_rn(x, pen), mv = __fmul_rn(x, pen);
            x = ap ? (x > 0.0f ? dv : mv) : x;
            if constexpr (DIVT) x = __fdiv_rn(x, T);
            lm = fmaxf(lm, x);
            if (GREEDY && arg_better(x, 4 * h + j, gv, gi)) {
              gv = x;
              gi = 4 * h + j;
            }
          }
          v[j] = x;
        }
        sh.row[h] = make_float4(v[0], v[1], v[2], v[3]);
        sh.appb[h] = static_cast<uint8_t>(app);
      }
    }
  };
  if (cand_path)
    first_pass(std::true_type{}, std::false_type{}, std::false_type{});
  else if (greedy)
    first_pass(std::false_type{}, std::false_type{}, std::true_type{});
  else if (divT)
    first_pass(std::false_type{}, std::true_type{}, std::false_type{});
  else
    first_pass(std::false_type{}, std::false_type{}, std::false_type{});
  row_sync<W>();  // the row is processed; the presence flags are dead

  bool done = false;
  if (cand_path) {
    // ---- few survivors: the row holds approximate values (x * RN(1/pen)
    //      instead of x / pen for present entries > 0, within 2 ulps); select
    //      a threshold on them, resolve exactly on the candidates ------------
    //
    // Histograms of d = max - value: bins 1/8 wide over d < 32 when that
    // locates the K-th largest tightly enough, else bins 1 wide over d < 255
    // and then bins 1/64 wide over the two unit bins from the one holding the
    // K-th largest.  With every value in [-2000, 2000] an ulp is <= 2^-12, so
    // the approximation error plus any temperature-tie window (a few ulps)
    // stays far inside one bin: every entry above the bin holding the K-th
    // largest, in it, or in the next one down is a candidate.  Otherwise
    // (wider values, NaN, the K-th below d = 253) a radix select on the
    // approximate keys with a 40-unit margin.
    amax = X.max_f(anan ? INFINITY : amax);
    auto dist = [&](float v) -> float { return __fsub_rn(amax, v); };
    bool linear = fabsf(amax) <= 2000.0f;
    // counts of the entries with (d - d0) * scale in [0, lim), by bin
    // 255 - floor((d - d0) * scale) (the scans run from the top down)
    auto bin_pass = [&](uint32_t* hist, float d0, float scale, float lim) {
#pragma unroll 2
      for (int r = rb0; r < rb1; ++r) {
        const int h = lane + 32 * r;
        if (4 * h >= V) continue;
        const float4 q = sh.row[h];
        const float v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float e = __fmul_rn(__fsub_rn(dist(v[j]), d0), scale);
          if (e >= 0.0f && e < lim) atomicAdd(&hist[255u - static_cast<uint32_t>(e)], 1u);
        }
      }
    };
    // candidates: d < dcut, or (d - dcut) * dsc < ecut
    float dcut = 0.0f, dsc = 8.0f, ecut = 0.0f;
    if (linear) {
      // Bins 1/8 wide over d < 32: when the K-th largest lies there and the
      // entries down to the bin below its own number at most WCAP, they are
      // the candidates.  Every warp scans the histogram itself (no
      // broadcast) and reaches the same decision.
      bin_pass(sh.hist[0], 0.0f, 8.0f, 256.0f);
      row_sync<W>();
      uint32_t d8, k8;
      warp_scan_count_desc_keep(sh.hist[0], static_cast<uint32_t>(K), d8, k8);
      const uint32_t b8 = 255u - d8;
      uint32_t n8 = WCAP + 1;
      if (b8 <= 253u) n8 = (static_cast<uint32_t>(K) - k8) + sh.hist[0][255u - b8] + sh.hist[0][254u - b8];
      if (n8 <= static_cast<uint32_t>(WCAP)) {
        ecut = static_cast<float>(b8 + 2u);
      } else {
        // Otherwise bins 1 wide over d < 255, then bins 1/64 wide over the
        // two unit bins from the one holding the K-th largest.
        row_sync<W>();
        for (int i = t; i < NBINS; i += NT) sh.hist[0][i] = 0u;
        row_sync<W>();
        bin_pass(sh.hist[0], 0.0f, 1.0f, 255.0f);
        row_sync<W>();
        uint32_t da, krem;
        warp_scan_count_desc_keep(sh.hist[0], static_cast<uint32_t>(K), da, krem);
        const uint32_t ba = 255u - da;
        linear = ba <= 253u;
        if (linear) {
          bin_pass(sh.hist[1], static_cast<float>(ba), 64.0f, 128.0f);
          row_sync<W>();
          uint32_t db, kb;
          warp_scan_count_desc_keep(sh.hist[1], krem, db, kb);
          dcut = static_cast<float>(ba);
          dsc = 64.0f;
          ecut = static_cast<float>(255u - db + 2u);  // fine bins <= the K-th's + 1
        }
      }
      // every warp has read the histograms once all pass the compaction's
      // exchange below; the histograms are cleared after it
    }
    uint32_t lo = 0;
    if (!linear) {
      // the histograms back to zero for the radix passes
      row_sync<W>();
      for (int i = t; i < 2 * NBINS; i += NT) (&sh.hist[0][0])[i] = 0u;
      row_sync<W>();
      const uint32_t thr = row_select<R, W>(sh, wi, K, WCAP / 2 + K / 2, [&](int r, uint32_t (&key)[4]) -> uint32_t {
        const int h = lane + 32 * r;
        if (4 * h >= V) {
#pragma unroll
          for (int j = 0; j < 4; ++j) key[j] = 0u;
          return 0u;
        }
        const float4 q = sh.row[h];
        key[0] = f2key(q.x);
        key[1] = f2key(q.y);
        key[2] = f2key(q.z);
        key[3] = f2key(q.w);
        return 15u;
      });
      lo = thr > 40u ? thr - 40u : 0u;
    }
    // candidates: masks per quad (one loop per selection kind, picked once
    // per row), then records in vocabulary order
    uint32_t cnt = 0;
    auto mask_pass = [&](auto linear_tag) {
      constexpr bool LIN = decltype(linear_tag)::value;
#pragma unroll 2
      for (int r = rb0; r < rb1; ++r) {
        const int h = lane + 32 * r;
        uint32_t cm = 0;
        if (4 * h < V) {
          const float4 q = sh.row[h];
          const float v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            bool c;
            if constexpr (LIN) {
              const float d = dist(v[j]);
              c = d < dcut || __fmul_rn(__fsub_rn(d, dcut), dsc) < ecut;
            } else {
              c = f2key(v[j]) >= lo;
            }
            cm |= (c ? 1u : 0u) << j;
          }
        }
        sh.cmask[h] = static_cast<uint8_t>(cm);
        cnt += __popc(cm);
      }
    };
    if (linear)
      mask_pass(std::true_type{});
    else
      mask_pass(std::false_type{});
#pragma unroll
    for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(FULL, cnt, o);
    uint32_t n32;
    uint32_t base = X.prefix_u(cnt, n32);
    const int n = static_cast<int>(n32);
    const int n4 = (n + 3) & ~3;
    // past the exchange every warp is done with the histograms: zero them
    for (int i = t; i < 2 * NBINS; i += NT) (&sh.hist[0][0])[i] = 0u;
    if (n <= WCAP) {
      // records {0, index, 0, 0}; the list's next step fills in x' and s
#pragma unroll 2
      for (int r = rb0; r < rb1; ++r) {
        const int h = lane + 32 * r;
        const uint32_t cm = sh.cmask[h];
        uint32_t tot;
        uint32_t p = base + warp_excl_small(__popc(cm), tot);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if ((cm >> j) & 1u) {
            sh.u.cand[p] = make_uint4(0u, static_cast<uint32_t>(4 * h + j), 0u, 0u);
            ++p;
          }
        base += tot;
      }
    }
    row_sync<W>();
    if (n <= WCAP) {
      // ---- the list, all threads: exact x' (recomputed from the staged row
      //      or L2, one load round trip for all candidates at once) and s per
      //      candidate, s again by position in the row buffer (dead past the
      //      compaction; NaN padding never compares), the list's maximum and
      //      the proof window -- one exchange -------------------------------
      float* sf = rowf;
      float m = -INFINITY, bad = 0.0f;
      // the K-th largest s (slot n - K below); with fewer than K candidates
      // every one is kept
      if (t == 0) *reinterpret_cast<float*>(&sh.sel[0]) = -INFINITY;
      for (int p = t; p < n4; p += NT) {
        if (p < n) {
          const uint32_t v = sh.u.cand[p].y;
          const float x = exact_x(static_cast<int>(v));
          const float s = greedy ? x : __fdiv_rn(x, T);
          sh.u.cand[p] = make_uint4(__float_as_uint(s), v, __float_as_uint(x), 0u);
          sf[p] = s;
          m = fmaxf(m, s);
          const float ap = fabsf(s);
          bad = (ap >= 0x1p-100f && ap <= 0x1p100f) ? bad : 1.0f;
        } else {
          sf[p] = __int_as_float(0x7fc00000);
        }
      }
      X.max2_f(m, bad);
      if (W == 1) __syncwarp();
      if (greedy) {
        // argmax of x' (torch.argmax order: lowest index on ties)
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int p = t; p < n; p += NT) {
          const float xv = __uint_as_float(sh.u.cand[p].z);
          const int iv = static_cast<int>(sh.u.cand[p].y);
          if (arg_better(xv, iv, bv, bi)) {
            bv = xv;
            bi = iv;
          }
        }
        X.argmax(bv, bi);
        id = bi;
        flags = Q3S_ROW_GREEDY;
        done = true;
      } else if (m != -INFINITY && bad == 0.0f) {
        // Quotients far from 1 may merge more than one fine bin (or 40 key
        // units) of x': the candidate set is proven complete only while
        // every candidate's |s| stays inside the window checked above.
        //
        // ---- exact order by all pairs: per candidate (LP threads each, the
        //      list split between them), its stable ascending slot (s asc,
        //      index asc); the entry in slot n - K is the K-th largest, and
        //      HF TopK keeps s >= it (ties kept).  The slot of a kept
        //      entry orders HF TopP's cumulative masses; entries TopK drops
        //      take the lowest slots (they are strictly below every kept one)
        //      and weigh nothing.  Kept softmax weights by position for the
        //      draw; with top-p, exact fixed-point masses by ascending slot
        //      and the slot of each position ---------------------------------
        const bool cut = top_p < 1.0f;
        const int P = (n + 31) >> 5;
        float* wk = reinterpret_cast<float*>(sh.hist);                                 // 32 P <= 256
        unsigned long long* mqa = reinterpret_cast<unsigned long long*>(rowf + WCAP);  // by ascending slot
        uint8_t* asca = sh.cmask;                                                      // slot by position
        const float4* sf4 = reinterpret_cast<const float4*>(sf);
        constexpr int LP = W >= 16 ? 4 : (W >= 8 ? 2 : 1);
        const int sl = t & (LP - 1);
        float* skth = reinterpret_cast<float*>(&sh.sel[0]);  // the K-th largest s
        for (int pb = 0; pb < 32 * P; pb += NT / LP) {
          // the ascending slot of p: entries below it, counting equal s at
          // lower positions -- s <= sp in quads wholly before p's (s < spu,
          // spu the next float up: every |s| here is normal and finite),
          // s < sp elsewhere, then p's own quad's earlier equal entries
          const int p = pb + t / LP;  // warp-uniform trip count: every lane shuffles
          const bool act = p < n;
          const float sp = act ? sf[p] : __int_as_float(0x7fc00000);
          const float spu = __uint_as_float(__float_as_uint(sp) + (sp > 0.0f ? 1u : 0xffffffffu));
          const int p4 = p >> 2;
          int c = 0;
#pragma unroll 4
          for (int q4 = sl; q4 < (n4 >> 2); q4 += LP) {
            const float4 f = sf4[q4];
            const float th = q4 < p4 ? spu : sp;
            c += (f.x < th) + (f.y < th) + (f.z < th) + (f.w < th);
          }
#pragma unroll
          for (int o = 1; o < LP; o <<= 1) c += __shfl_xor_sync(FULL, c, o);
          if (act && sl == 0) {
            for (int j = 4 * p4; j < p; ++j) c += sf[j] == sp;
            asca[p] = static_cast<uint8_t>(c);
            if (c == n - K) *skth = sp;  // ascending slot n - K: the K-th largest
          }
        }
        row_sync<W>();
        // kept by TopK: s >= the K-th largest (ties kept)
        const float sK = *skth;
        for (int p = t; p < 32 * P; p += NT) {
          float w = 0.0f;
          if (p < n) {
            const float sp = sf[p];
            w = sp >= sK ? softmax_weight(sp, m) : 0.0f;
            if (cut) mqa[asca[p]] = mass_fixed(w);
          }
          wk[p] = w;
        }
        row_sync<W>();
        // ---- warp 0 alone from here: top-p over the ascending slots, the
        //      draw over positions (vocabulary order) ------------------------
        if (wi == 0) {
          int lflags = 0;
          if (cut) {
            // HF TopPLogitsWarper: slot i goes when the mass of slots <= i is
            // <= tau = floor((1-p) Zq); the last slot stays
            const float frac = __fsub_rn(1.0f, top_p);
            const int i0 = 8 * lane;
            unsigned long long c[8], sum = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              c[j] = i0 + j < n ? mqa[i0 + j] : 0ull;
              sum += c[j];
            }
            unsigned long long inc = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const unsigned long long y = __shfl_up_sync(FULL, inc, o);
              if (lane >= o) inc += y;
            }
            const unsigned long long Zq = __shfl_sync(FULL, inc, 31);
            const unsigned long long tau = __double2ull_rd(static_cast<double>(frac) * static_cast<double>(Zq));
            const unsigned long long eps = Zq / 1000000ull;
            // The removed slots are a prefix (cumulative masses only grow):
            // every slot of the lanes before the first whose inclusive sum
            // passes tau, and that lane's slots up to tau.  That lane also
            // holds the cumulative masses on either side of tau (the
            // boundary check).  icut slots go; the last one always stays.
            const unsigned over = __ballot_sync(FULL, inc > tau);
            const int lc = over ? __ffs(over) - 1 : 31;
            int below = 0;
            bool near = false;
            if (lane == lc) {
              unsigned long long cum = inc - sum, lo = cum, hi = ~0ull;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                cum += c[j];
                if (cum <= tau) {
                  ++below;
                  lo = cum;
                } else if (hi == ~0ull && i0 + j < n - 1) {
                  hi = cum;
                }
              }
              near = tau < Zq && (tau - lo < eps || (hi != ~0ull && hi - tau < eps));
            }
            const int icut = min(8 * lc + __shfl_sync(FULL, below, lc), n - 1);
            if (__shfl_sync(FULL, near, lc)) lflags |= Q3S_ROW_TOPP_BOUNDARY;
            if constexpr (PROC) {
              if (lane == 0) sh.res[2] = icut;
            }
            int sa[WCAP / 32];
#pragma unroll
            for (int r = 0; r < WCAP / 32; ++r) sa[r] = r < P && lane * P + r < n ? asca[lane * P + r] : WCAP;
#pragma unroll
            for (int r = 0; r < WCAP / 32; ++r)
              if (sa[r] < icut) wk[lane * P + r] = 0.0f;
            __syncwarp();
          }
          if constexpr (PROC) {
            if (!cut && lane == 0) sh.res[2] = 0;
          }
          const int pos = warp_draw_list(wk, n, u, lflags);
          id = static_cast<int>(sh.u.cand[pos].y);
          flags = lflags;
        }
        done = true;
        list_row = true;
        if constexpr (PROC) {
          if (t == 0) sh.lcnt[0] = n;
        }
      }
    }
    if (!done) {
      // the candidate set overflowed or left the proven window: exact s for
      // the whole row, recomputed from the logits (the row holds approximate
      // values); the histograms, used as the list's scratch, back to zero
      for (int i = t; i < 2 * NBINS; i += NT) (&sh.hist[0][0])[i] = 0u;
#pragma unroll 1
      for (int r = rb0; r < rb1; ++r) {
        const int h = lane + 32 * r;
        if (4 * h >= V) continue;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float x = exact_s(4 * h + j);
          lm = fmaxf(lm, x);
          if (greedy && arg_better(x, 4 * h + j, gv, gi)) {
            gv = x;
            gi = 4 * h + j;
          }
          v[j] = x;
        }
        sh.row[h] = make_float4(v[0], v[1], v[2], v[3]);
      }
      flags = 0;
      row_sync<W>();
    }
  }
  if (!done) {
    // ---- whole-vocabulary rows: the row holds s -------------------------
    flags = 0;
    if (greedy) {
      X.argmax(gv, gi);
      id = gi;
      flags = Q3S_ROW_GREEDY;
    } else {
      const float m = X.max_f(lm);
      if (m == -INFINITY) {
        // nothing finite: report it and take the lowest index
        wv_nomass = true;
        err |= Q3S_DEVERR_NO_MASS;
        flags = Q3S_ROW_FALLBACK;
        id = 0;
      } else {
        // top-k survivors: s >= the k-th largest s (ties kept)
        const bool topk = kk > 0 && kk < V;
        uint32_t kth = 0;
        if (topk) {
          kth = row_select<R, W>(sh, wi, kk, kk, [&](int r, uint32_t (&key)[4]) -> uint32_t {
            const int h = lane + 32 * r;
            if (4 * h >= V) {
#pragma unroll
              for (int j = 0; j < 4; ++j) key[j] = 0u;
              return 0u;
            }
            const float4 f = sh.row[h];
            key[0] = f2key(f.x);
            key[1] = f2key(f.y);
            key[2] = f2key(f.z);
            key[3] = f2key(f.w);
            return 15u;
          });
        }
        // ---- softmax weights in place; exact fixed-point masses into a
        //      coarse histogram by the weight's exponent and top 4 mantissa
        //      bits (monotone in s) ------------------------------------------
        const bool cut = top_p < 1.0f;
        wv_topk = topk;
        wv_kth = kth;
        wv_cut = cut;
        constexpr uint32_t LO = (1u << MASS_LO_BITS) - 1u;
        // one loop per (top-k, top-p) combination, picked once per row
        auto weights_pass = [&](auto topk_tag, auto cut_tag) {
          constexpr bool TOPK = decltype(topk_tag)::value, CUT = decltype(cut_tag)::value;
#pragma unroll 2
          for (int r = rb0; r < rb1; ++r) {
            const int h = lane + 32 * r;
            if (4 * h >= V) continue;
            const float4 f = sh.row[h];
            const float sv[4] = {f.x, f.y, f.z, f.w};
            float wv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const bool surv = !TOPK || f2key(sv[j]) >= kth;
              wv[j] = surv ? softmax_weight(sv[j], m) : 0.0f;
              if constexpr (CUT) {
                const unsigned long long q = mass_fixed(wv[j]);
                if (q) {
                  const uint32_t bn = coarse_bin(wv[j]);
                  atomicAdd(&sh.hist[0][bn], static_cast<uint32_t>(q >> MASS_LO_BITS));
                  atomicAdd(&sh.hist[1][bn], static_cast<uint32_t>(q) & LO);
                }
              }
            }
            sh.row[h] = make_float4(wv[0], wv[1], wv[2], wv[3]);
          }
        };
        if (topk) {
          if (cut) weights_pass(std::true_type{}, std::true_type{});
          else weights_pass(std::true_type{}, std::false_type{});
        } else {
          if (cut) weights_pass(std::false_type{}, std::true_type{});
          else weights_pass(std::false_type{}, std::false_type{});
        }
        row_sync<W>();
        bool single = false;
        if (cut) {
          const float frac = __fsub_rn(1.0f, top_p);
          if (wi == 0) {
            unsigned long long Zq, tau, before;
            uint32_t bstar;
            warp_scan_mass_total(sh.hist[0], sh.hist[1], frac, Zq, tau, bstar, before);
            if (lane == 0) {
              sh.selq[0] = Zq;
              sh.selq[1] = tau;
              sh.selq[2] = before;
              sh.sel[3] = bstar;
            }
          }
          row_sync<W>();
          const unsigned long long Zq = sh.selq[0], tau = sh.selq[1], below = sh.selq[2];
          const uint32_t bstar = sh.sel[3];
          const unsigned long long eps = Zq / 1000000ull;
          if (tau >= Zq) {
            // everything but the ascending-last entry (largest s, then largest
            // index) goes; its weight is exp(0) = 1
            int last = -1;
#pragma unroll 1
            for (int r = rb0; r < rb1; ++r) {
              const int h = lane + 32 * r;
              if (4 * h >= V) continue;
              const float4 f = sh.row[h];
              const float wv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (wv[j] == 1.0f && exact_s(4 * h + j) == m) last = 4 * h + j;
            }
            id = X.max_i(last);
            single = true;
            wv_single = true;
          } else {
            // entries below the crossing bin go (their weights are zeroed),
            // entries above it stay; the crossing bin's entries are resolved
            // exactly as a list
            uint32_t cnt = 0;
#pragma unroll 2
            for (int r = rb0; r < rb1; ++r) {
              const int h = lane + 32 * r;
              uint32_t cm = 0;
              if (4 * h < V) {
                const float4 f = sh.row[h];
                float wv[4] = {f.x, f.y, f.z, f.w};
                bool zeroed = false;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  if (wv[j] > 0.0f) {
                    const uint32_t bn = coarse_bin(wv[j]);
                    if (bn < bstar) {
                      wv[j] = 0.0f;
                      zeroed = true;
                    } else if (bn == bstar) {
                      cm |= 1u << j;
                    }
                  }
                }
                if (zeroed) sh.row[h] = make_float4(wv[0], wv[1], wv[2], wv[3]);
              }
              sh.cmask[h] = static_cast<uint8_t>(cm);
              cnt += __popc(cm);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(FULL, cnt, o);
            uint32_t n32;
            uint32_t base = X.prefix_u(cnt, n32);
            const int n = static_cast<int>(n32);
            if (n <= WCAP) {
#pragma unroll 2
              for (int r = rb0; r < rb1; ++r) {
                const int h = lane + 32 * r;
                const uint32_t cm = sh.cmask[h];
                uint32_t tot;
                uint32_t p = base + warp_excl_small(__popc(cm), tot);
                if (cm) {
                  const float4 f = sh.row[h];
                  const float wv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
                  for (int j = 0; j < 4; ++j)
                    if ((cm >> j) & 1u) {
                      sh.u.cand[p] = make_uint4(0u, static_cast<uint32_t>(4 * h + j), 0u, __float_as_uint(wv[j]));
                      sh.keep[p] = 1;
                      ++p;
                    }
                }
                base += tot;
              }
              row_sync<W>();
              // exact s of the crossing bin's entries, the exact cut over
              // them, and the removed entries' weights zeroed in the row
              const int n4 = (n + 3) & ~3;
              unsigned long long* mq = reinterpret_cast<unsigned long long*>(sh.hist);  // (the histogram is done)
              if (t == 0) sh.res[3] = 0;
              for (int p = t; p < n4; p += NT) {
                if (p < n) {
                  sh.u.cand[p].x = __float_as_uint(exact_s(static_cast<int>(sh.u.cand[p].y)));
                  mq[p] = mass_fixed(__uint_as_float(sh.u.cand[p].w));
                } else {
                  sh.u.cand[p] = make_uint4(0xff800000u, 0x7fffffffu, 0u, 0u);
                  mq[p] = 0ull;
                }
                sh.keep[p] = p < n;
              }
              row_sync<W>();
              uint8_t* kout = sh.cmask;
              row_cut_list<W>(sh.u.cand, sh.keep, mq, kout, n, n4, tau, below, eps, &sh.res[3]);
              for (int p = t; p < n; p += NT)
                if (!kout[p]) rowf[sh.u.cand[p].y] = 0.0f;
              row_sync<W>();
              flags |= sh.res[3];
            } else {
              // the crossing bin holds too many entries: an exact radix cut
              // over the survivors of that bin and above, keys from the exact
              // s recomputed per entry
              auto skey = [&](int v) -> uint32_t { return f2key(exact_s(v)); };
              uint32_t prefix = 0, hmask = 0;
              unsigned long long bl = below;
#pragma unroll 1
              for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll 1
                for (int r = rb0; r < rb1; ++r) {
                  const int h = lane + 32 * r;
                  if (4 * h >= V) continue;
                  const float4 f = sh.row[h];
                  const float wv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    const unsigned long long q1 = mass_fixed(wv[j]);
                    if (q1 == 0 || coarse_bin(wv[j]) != bstar) continue;
                    const uint32_t key = skey(4 * h + j);
                    if ((key & hmask) == prefix) {
                      atomicAdd(&sh.hist[0][(key >> shift) & 255u], static_cast<uint32_t>(q1 >> MASS_LO_BITS));
                      atomicAdd(&sh.hist[1][(key >> shift) & 255u], static_cast<uint32_t>(q1) & LO);
                    }
                  }
                }
                row_sync<W>();
                if (wi == 0) {
                  uint32_t d;
                  unsigned long long bef;
                  warp_scan_mass_asc(sh.hist[0], sh.hist[1], bl, tau, d, bef);
                  if (lane == 0) {
                    sh.sel[0] = d;
                    sh.selq[3] = bef;
                  }
                }
                row_sync<W>();
                prefix |= sh.sel[0] << shift;
                hmask |= 255u << shift;
                bl = sh.selq[3];
              }
              const uint32_t vstar = prefix;
              // the entries at vstar share one s, one weight and one mass
              unsigned long long qs = 0;
#pragma unroll 1
              for (int r = rb0; r < rb1; ++r) {
                const int h = lane + 32 * r;
                if (4 * h >= V) continue;
                const float4 f = sh.row[h];
                const float wv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  if (mass_fixed(wv[j]) != 0 && coarse_bin(wv[j]) == bstar && skey(4 * h + j) == vstar)
                    qs = mass_fixed(wv[j]);
              }
              qs = X.max_q(qs);
              qs = qs ? qs : 1ull;
              const unsigned long long nrem = (tau - bl) / qs;  // ties removed, lowest index first
              const unsigned long long first_kept = bl + (nrem + 1) * qs;
              const unsigned long long last_removed = bl + nrem * qs;
              if ((first_kept - tau) < eps || (tau - last_removed) < eps) flags |= Q3S_ROW_TOPP_BOUNDARY;
              // tie ranks in vocabulary order: per-round warp scans, warp
              // blocks offset by the earlier warps' tie counts
              uint32_t tcount = 0;
#pragma unroll 1
              for (int r = rb0; r < rb1; ++r) {
                const int h = lane + 32 * r;
                if (4 * h >= V) continue;
                const float4 f = sh.row[h];
                const float wv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  if (mass_fixed(wv[j]) != 0 && coarse_bin(wv[j]) == bstar && skey(4 * h + j) == vstar) ++tcount;
              }
#pragma unroll
              for (int o = 16; o; o >>= 1) tcount += __shfl_xor_sync(FULL, tcount, o);
              uint32_t ttot;
              unsigned long long tb = X.prefix_u(tcount, ttot);
#pragma unroll 1
              for (int r = rb0; r < rb1; ++r) {
                const int h = lane + 32 * r;
                const bool in = 4 * h < V;
                float wv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                uint32_t key[4] = {0u, 0u, 0u, 0u};
                uint32_t ce = 0, inb = 0;
                if (in) {
                  const float4 f = sh.row[h];
                  wv[0] = f.x;
                  wv[1] = f.y;
                  wv[2] = f.z;
                  wv[3] = f.w;
#pragma unroll
                  for (int j = 0; j < 4; ++j)
                    if (wv[j] > 0.0f && coarse_bin(wv[j]) == bstar) {
                      inb |= 1u << j;
                      key[j] = skey(4 * h + j);
                      if (mass_fixed(wv[j]) != 0 && key[j] == vstar) ce |= 1u << j;
                    }
                }
                uint32_t tot;
                uint32_t t_in = warp_excl_scan_u(__popc(ce), tot);
                if (in && inb) {
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    if (!((inb >> j) & 1u)) continue;
                    bool kp = false;
                    if (key[j] > vstar) {
                      kp = true;
                    } else if ((ce >> j) & 1u) {
                      kp = tb + t_in >= nrem;
                      ++t_in;
                    }
                    if (!kp) wv[j] = 0.0f;
                  }
                  sh.row[h] = make_float4(wv[0], wv[1], wv[2], wv[3]);
                }
                tb += tot;
              }
              row_sync<W>();
            }
          }
        }
        if (!single) {
          // ---- inverse CDF in vocabulary order: cumulative weight before each
          //      quad (round scans within each warp's block, warp blocks in
          //      order), the first quad whose running sum passes u * total,
          //      then the entry inside it --------------------------------------
          float carry = 0.0f;
          int lastv = -1;
#pragma unroll 1
          for (int r = rb0; r < rb1; ++r) {
            const int h = lane + 32 * r;
            float qsum = 0.0f;
            if (4 * h < V) {
              const float4 f = sh.row[h];
              const float wv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                qsum = __fadd_rn(qsum, wv[j]);
                if (wv[j] > 0.0f) lastv = 4 * h + j;
              }
            }
            float tot;
            const float exs = warp_excl_scan_f(qsum, tot);
            sh.u.ex[h] = __fadd_rn(carry, exs);
            carry = __fadd_rn(carry, tot);
          }
          float Wt;
          const float off = X.prefix_f(carry, Wt);
          const float thr = __fmul_rn(u, Wt);
          int firstq = 0x7fffffff;
#pragma unroll 1
          for (int r = rb0; r < rb1; ++r) {
            const int h = lane + 32 * r;
            if (4 * h >= V) break;
            const float4 f = sh.row[h];
            const float wv[4] = {f.x, f.y, f.z, f.w};
            float acc = __fadd_rn(off, sh.u.ex[h]);
            bool hit = false;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              acc = __fadd_rn(acc, wv[j]);
              hit |= wv[j] > 0.0f && acc > thr;
            }
            if (hit) {
              firstq = h;
              break;
            }
          }
          // quads in vocabulary order are h = l + 32 r ascending
          firstq = X.min_i(firstq);
          lastv = X.max_i(lastv);
          if (firstq == 0x7fffffff) {
            id = lastv;
            flags |= Q3S_ROW_FALLBACK;
          } else {
            const int ow = (firstq >> 5) / RPW;
            if (wi == ow && lane == (firstq & 31)) {
              const float4 f = sh.row[firstq];
              const float wv[4] = {f.x, f.y, f.z, f.w};
              const float pre = __fadd_rn(off, sh.u.ex[firstq]);
              float acc = pre, prev = pre, cdf = pre;
              int pick = 4 * firstq;
              bool found = false;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float before = acc;
                acc = __fadd_rn(acc, wv[j]);
                if (!found && wv[j] > 0.0f && acc > thr) {
                  found = true;
                  pick = 4 * firstq + j;
                  prev = before;
                  cdf = acc;
                }
              }
              const float tol = BOUNDARY_EPS * Wt;
              sh.res[0] = pick;
              sh.res[1] = ((__fsub_rn(cdf, thr) < tol) || (__fsub_rn(thr, prev) < tol)) ? Q3S_ROW_DRAW_BOUNDARY : 0;
            }
            row_sync<W>();
            id = sh.res[0];
            flags |= sh.res[1];
          }
        }
      }
    }
  }
  if constexpr (PROC) {
    // Verification output, written after the row is decided: every entry's
    // exact processed value where top-k and top-p keep it, -inf elsewhere
    // (greedy rows: x' everywhere, the input of torch.argmax).  List rows
    // write -inf for all entries, then (after a barrier) the kept candidates.
    row_sync<W>();
    float* const prow = a.processed + static_cast<int64_t>(b) * a.proc_stride;
#pragma unroll 1
    for (int r = rb0; r < rb1; ++r) {
      const int h = lane + 32 * r;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int v = 4 * h + j;
        if (v >= V) continue;
        float o;
        if (greedy) {
          o = exact_x(v);
        } else if (list_row) {
          o = -INFINITY;
        } else {
          const float s = exact_s(v);
          bool kept;
          if (wv_nomass) kept = true;
          else if (wv_single) kept = v == id;
          else if (wv_cut) kept = rowf[v] > 0.0f;
          else kept = !wv_topk || f2key(s) >= wv_kth;
          o = kept ? s : -INFINITY;
        }
        prow[v] = o;
      }
    }
    if (list_row) {
      row_sync<W>();
      const float sK = *reinterpret_cast<const float*>(&sh.sel[0]);
      const int icut = sh.res[2], n = sh.lcnt[0];
      const uint8_t* asca = sh.cmask;
      for (int p = t; p < n; p += NT) {
        const uint4 c = sh.u.cand[p];
        const float s = __uint_as_float(c.x);
        if (s >= sK && static_cast<int>(asca[p]) >= icut) prow[c.y] = s;
      }
    }
  }
  if (t == 0) {
    if (a.ids64) a.ids64[b] = id;
    if (a.ids32) a.ids32[b] = id;
    if (a.row_flags) a.row_flags[b] = flags;
  }
  if (err && a.error_word) atomicOr(a.error_word, static_cast<int>(err));
}

}  // namespace q3s
