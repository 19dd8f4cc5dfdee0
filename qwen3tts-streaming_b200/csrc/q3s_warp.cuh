// q3s_warp.cuh -- warp-per-row sampler (icdf mode) for batched steps.
//
// One warp owns one row and keeps it in its own slice of shared memory: the
// row arrives with one bulk copy (cp.async.bulk, completion on an mbarrier)
// while the warp scatters the row's history, and every pass over it after
// that is a rolled loop of 16-byte shared loads -- lane l reads quad
// h = l + 32 r (entries [4h, 4h+4)) in round r, so a warp's load covers 512
// contiguous bytes without bank conflicts.  Reductions are warp shuffles; no
// block barrier is taken, and three CTAs of four warps share an SM.
// Vocabulary order is quad order: round r, then lane l, then entry j.
//
// The arithmetic and the tie rules are those of the CTA-per-row kernels in
// q3s_sampler.cu (HF LogitsProcessorList order, transformers
// generation/logits_process.py, as driven by the reference's
// qwen_tts/core/models/modeling_qwen3_tts.py:1591-1611 generate() call):
// suppress -> repetition penalty -> EOS gate -> temperature -> top-k (ties
// kept) -> top-p (stable ascending order) -> softmax -> inverse CDF.
#pragma once

#include "q3s_args.cuh"
#include "q3s_device.cuh"

namespace q3s {

constexpr int WPB = 4;                 // warps (rows) per CTA
constexpr int WCAP = 256;              // candidate records per warp
constexpr int COARSE_SCALE_BITS = 20;  // coarse masses floor(w * 2^20): a row (V <= 3072, w <= 1) sums below 2^32
constexpr int COARSE_SHIFT = 19;       // coarse bin: exponent and top 4 mantissa bits of w (16 bins per octave)
constexpr int COARSE_BIN0 = (0x3f800000 >> COARSE_SHIFT) - 255;  // w = 1 -> bin 255; w < 2^-15.9 -> bin 0

template <int R>
struct alignas(16) WarpSmem {
  static constexpr int RQ = 2 * R;       // rounds of one quad (4 entries) per lane
  static constexpr int VMAX = 128 * RQ;  // entries the row buffer holds
  float4 row[32 * RQ];                   // quad h: logits as loaded -> x' -> s -> softmax weights
  uint32_t hist[2][NBINS];               // counts / mass high parts, mass low parts; zero between uses
  union {
    uint8_t seen[VMAX];                  // presence flags from the packed history (dead after the first pass)
    uint4 cand[WCAP];                    // candidate records {s bits, index, x' bits, weight bits}
    float ex[32 * RQ];                   // draw: cumulative weight before each quad
  } u;
  uint8_t appb[16 * RQ];                 // presence bits: byte (r/2)*32 + l, nibble r%2 = quad of round r
  uint8_t keep[WCAP];
  uint64_t bar;                          // completion of the logits bulk copy
};

Q3S_DEV int lane_id() { return static_cast<int>(threadIdx.x & 31u); }

// ---------------------------------------------------------------------------
// warp scans over a 256-bin histogram; each lane owns bins 8l..8l+7 and
// clears them after reading (the zero invariant of WarpSmem::hist)
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

// Coarse u32 masses, bins ascending: the first bin where the running sum
// exceeds tau (tau < total).
Q3S_DEV uint32_t warp_scan_coarse_asc(uint32_t* hist, uint32_t tau) {
  const int lane = lane_id();
  uint4* hb = reinterpret_cast<uint4*>(hist) + 2 * lane;
  const uint4 a = hb[0], b = hb[1];
  const uint32_t c[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  const uint32_t s = (c[0] + c[1]) + (c[2] + c[3]) + (c[4] + c[5]) + (c[6] + c[7]);
  uint32_t inc = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc += n;
  }
  const uint32_t lo0 = inc - s;
  const bool hit = lo0 <= tau && tau < inc;
  uint32_t md = 0;
  if (hit) {
    uint32_t acc = lo0;
    bool found = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (!found && acc + c[i] > tau) {
        found = true;
        md = static_cast<uint32_t>(8 * lane + i);
      }
      acc += c[i];
    }
  }
  hb[0] = make_uint4(0, 0, 0, 0);
  hb[1] = make_uint4(0, 0, 0, 0);
  const unsigned bal = __ballot_sync(FULL, hit);
  const uint32_t d = bal ? __shfl_sync(FULL, md, __ffs(bal) - 1) : 255u;
  __syncwarp();
  return d;
}

// Radix select over the row (8-bit digits, most significant first), like
// select_threshold for a CTA: the k-th largest key, or earlier, once the
// entries at or above the current bin number at most `stop`, that bin's lower
// edge.  qk(r, key) fills the keys of this lane's quad of round r and returns
// the mask of entries that take part.
template <int RQ, typename QuadKeys>
Q3S_DEV uint32_t warp_select_rows(uint32_t* hist, int k, int stop, QuadKeys qk) {
  uint32_t prefix = 0, hmask = 0;
  uint32_t krem = static_cast<uint32_t>(k);
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll 2
    for (int r = 0; r < RQ; ++r) {
      uint32_t key[4];
      const uint32_t act = qk(r, key);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (((act >> j) & 1u) && (key[j] & hmask) == prefix) atomicAdd(&hist[(key[j] >> shift) & 255u], 1u);
    }
    __syncwarp();
    uint32_t d, cnt, knew;
    warp_scan_count_desc(hist, krem, d, cnt, knew);
    prefix |= d << shift;
    hmask |= 255u << shift;
    krem = knew;
    // entries strictly above the bin: k - krem (krem = rank left inside it);
    // in it: cnt
    if (static_cast<int>(static_cast<uint32_t>(k) - krem + cnt) <= stop) return prefix;
  }
  return prefix;
}

// Radix select of the k-th largest key over a candidate list (positions
// lane + 32 i); stop as above.
Q3S_DEV uint32_t warp_select_list(const uint4* cand, int n, uint32_t* hist, int k, int stop) {
  const int lane = lane_id();
  return warp_select_rows<WCAP / 128>(hist, k, stop, [&](int r, uint32_t (&key)[4]) -> uint32_t {
    uint32_t act = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int p = lane + 32 * (4 * r + j);
      key[j] = p < n ? f2key(__uint_as_float(cand[p].x)) : 0u;
      act |= (p < n ? 1u : 0u) << j;
    }
    return act;
  });
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
// candidate lists (positions in vocabulary order; lane l owns l + 32 q)
// ---------------------------------------------------------------------------

// HF TopPLogitsWarper's cut among the participating (keep[i]) entries of a
// list, given the mass `below0` of everything under the list (every entry
// below the list is removed, every entry above it kept): an entry is removed
// when the mass at or below it, in stable ascending order (s asc, index asc),
// is <= tau.  Requires below0 <= tau < below0 + list mass.  Masses are exact
// fixed point.  Returns Q3S_ROW_TOPP_BOUNDARY when the cut lies within eps of
// a cumulative-mass edge.
Q3S_DEV int warp_mass_cut_list(const uint4* cand, uint8_t* keep, int n, unsigned long long tau,
                               unsigned long long below0, unsigned long long eps, uint32_t* hhi, uint32_t* hlo) {
  const int lane = lane_id();
  constexpr int Q = WCAP / 32;
  constexpr uint32_t LO = (1u << MASS_LO_BITS) - 1u;
  uint32_t key[Q];
  unsigned long long q[Q];
#pragma unroll
  for (int i = 0; i < Q; ++i) {
    const int p = lane + 32 * i;
    const bool on = p < n && keep[p];
    key[i] = on ? f2key(__uint_as_float(cand[p].x)) : 0u;
    q[i] = on ? mass_fixed(__uint_as_float(cand[p].w)) : 0ull;
  }
  uint32_t prefix = 0, hmask = 0;
  unsigned long long below = below0;
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll
    for (int i = 0; i < Q; ++i)
      if (q[i] != 0 && (key[i] & hmask) == prefix) {
        const uint32_t bin = (key[i] >> shift) & 255u;
        atomicAdd(&hhi[bin], static_cast<uint32_t>(q[i] >> MASS_LO_BITS));
        atomicAdd(&hlo[bin], static_cast<uint32_t>(q[i]) & LO);
      }
    __syncwarp();
    uint32_t d;
    unsigned long long bef;
    warp_scan_mass_asc(hhi, hlo, below, tau, d, bef);
    prefix |= d << shift;
    hmask |= 255u << shift;
    below = bef;
  }
  const uint32_t vstar = prefix;
  // all entries at vstar share one s, hence one weight and one mass
  unsigned long long qs = 0;
#pragma unroll
  for (int i = 0; i < Q; ++i)
    if (q[i] != 0 && key[i] == vstar) qs = q[i];
  const unsigned bq = __ballot_sync(FULL, qs != 0);
  qs = __shfl_sync(FULL, qs, bq ? __ffs(bq) - 1 : 0);
  qs = qs ? qs : 1ull;
  const unsigned long long nrem = (tau - below) / qs;  // ties removed, lowest index first
  const unsigned long long first_kept = below + (nrem + 1) * qs;
  const unsigned long long last_removed = below + nrem * qs;
  const int flags = ((first_kept - tau) < eps || (tau - last_removed) < eps) ? Q3S_ROW_TOPP_BOUNDARY : 0;
  unsigned long long ties_before = 0;
#pragma unroll
  for (int i = 0; i < Q; ++i) {
    const int p = lane + 32 * i;
    const bool on = p < n && keep[p];
    const bool tie = on && q[i] != 0 && key[i] == vstar;
    const unsigned bal = __ballot_sync(FULL, tie);
    const unsigned long long rank = ties_before + __popc(bal & ((1u << lane) - 1u));
    // zero-mass entries follow their key: kept above vstar, removed at or below
    const bool kp = on && (key[i] > vstar || (tie && rank >= nrem));
    ties_before += __popc(bal);
    if (p < n) keep[p] = kp;
  }
  __syncwarp();
  return flags;
}

// Keep only the ascending-last participating entry of a list: largest s,
// then largest index (everything else has mass at or below it <= tau).
Q3S_DEV void warp_keep_last_list(const uint4* cand, uint8_t* keep, int n) {
  const int lane = lane_id();
  constexpr int Q = WCAP / 32;
  uint32_t bk = 0, bi = 0;
  int bp = -1;
#pragma unroll
  for (int i = 0; i < Q; ++i) {
    const int p = lane + 32 * i;
    if (p < n && keep[p]) {
      const uint32_t k = f2key(__uint_as_float(cand[p].x));
      if (bp < 0 || k > bk || (k == bk && cand[p].y > bi)) {
        bk = k;
        bi = cand[p].y;
        bp = p;
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const uint32_t ok = __shfl_xor_sync(FULL, bk, o);
    const uint32_t oi = __shfl_xor_sync(FULL, bi, o);
    const int op = __shfl_xor_sync(FULL, bp, o);
    if (op >= 0 && (bp < 0 || ok > bk || (ok == bk && oi > bi))) {
      bk = ok;
      bi = oi;
      bp = op;
    }
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < Q; ++i) {
    const int p = lane + 32 * i;
    if (p < n) keep[p] = (p == bp);
  }
  __syncwarp();
}

// Inverse CDF over a list's kept weights in vocabulary order: the first
// position whose running sum exceeds u * total.  Lane l owns positions
// [l P, l P + P), P = ceil(n / 32) -- the association order of the CTA
// kernels' warp-0 finisher, so both produce the same sums.
Q3S_DEV int warp_draw_list(const uint4* cand, const uint8_t* keep, int n, float u, int& flags) {
  const int lane = lane_id();
  const int P = (n + 31) / 32;
  float a = 0.0f;
  for (int r = 0; r < P; ++r) {
    const int i = lane * P + r;
    if (i < n && keep[i]) a = __fadd_rn(a, __uint_as_float(cand[i].w));
  }
  float W;
  const float pre = warp_excl_scan_f(a, W);
  const float thr = __fmul_rn(u, W);
  int r_first = -1, r_last = -1;
  float acc = 0.0f;
  for (int r = 0; r < P; ++r) {
    const int i = lane * P + r;
    const float w = (i < n && keep[i]) ? __uint_as_float(cand[i].w) : 0.0f;
    acc = __fadd_rn(acc, w);
    if (w > 0.0f) {
      r_last = r;
      if (r_first < 0 && __fadd_rn(pre, acc) > thr) r_first = r;
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
  int near = 0;
  if (lane == src) {
    float cdf = pre, prev = pre, a2 = 0.0f;
    for (int r = 0; r <= rsel; ++r) {
      const int i = lane * P + r;
      const float w = (i < n && keep[i]) ? __uint_as_float(cand[i].w) : 0.0f;
      a2 = __fadd_rn(a2, w);
      if (r < rsel) prev = __fadd_rn(pre, a2);
      cdf = __fadd_rn(pre, a2);
    }
    const float tol = BOUNDARY_EPS * W;
    near = (__fsub_rn(cdf, thr) < tol) || (__fsub_rn(thr, prev) < tol);
  }
  if (__shfl_sync(FULL, near, src)) flags |= Q3S_ROW_DRAW_BOUNDARY;
  return src * P + rsel;
}

Q3S_DEV uint32_t coarse_bin(float w) {
  const int e = static_cast<int>(__float_as_uint(w) >> COARSE_SHIFT) - COARSE_BIN0;
  return static_cast<uint32_t>(min(255, max(0, e)));
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

template <int R>
constexpr size_t warp_smem_bytes() {
  return static_cast<size_t>(WPB) * sizeof(WarpSmem<R>);
}

template <int R, bool BF16>
__global__ void __launch_bounds__(WPB * 32, 3) sample_warp_kernel(const SampleArgs a) {
  extern __shared__ __align__(16) unsigned char q3s_warp_smem[];
  constexpr int RQ = WarpSmem<R>::RQ;
  const int wi = static_cast<int>(threadIdx.x >> 5);
  const int lane = lane_id();
  const int b = blockIdx.x * WPB + wi;
  if (b >= a.B) return;  // whole warps leave; no block-wide synchronisation follows
  WarpSmem<R>& sh = reinterpret_cast<WarpSmem<R>*>(q3s_warp_smem)[wi];
  float* rowf = reinterpret_cast<float*>(sh.row);  // entry v at rowf[v]
  const int V = a.V;
  uint32_t err = 0;
  // fields read inside loops and lambdas, as locals: nothing may take the
  // address of the parameter block (its loads would then stay in the loops)
  const uint8_t* const suppress = a.suppress;
  const int32_t* const history = a.history;
  const int eos_id = a.eos_id;

  // ---- the row's logits stream into shared memory (one bulk copy, no
  //      multicast) while the history is scattered ---------------------------
  const int esz = BF16 ? 2 : 4;
  const uint32_t row_bytes = static_cast<uint32_t>(V * esz);
  // bf16 rows land in the upper half of the buffer and are widened in place
  constexpr uint32_t stage_off = BF16 ? static_cast<uint32_t>(sizeof(sh.row) / 2) : 0u;
  const unsigned char* grow = static_cast<const unsigned char*>(a.logits) + static_cast<int64_t>(b) * a.row_stride * esz;
  if (lane == 0) {
    mbar_init(&sh.bar, 1);
    fence_mbar_init();
    mbar_expect_tx(&sh.bar, row_bytes);
    bulk_g2s(reinterpret_cast<unsigned char*>(sh.row) + stage_off, grow, row_bytes, &sh.bar);
  }
  int o0 = 0, o1 = 0;
  if (history) {
    o0 = __ldg(a.offsets + b);
    o1 = __ldg(a.offsets + b + 1);
  }
  {
    // zero the histograms and the presence flags
    uint4* hz = reinterpret_cast<uint4*>(&sh.hist[0][0]);
#pragma unroll
    for (int i = 0; i < 2 * NBINS / 4 / 32; ++i) hz[lane + 32 * i] = make_uint4(0, 0, 0, 0);
    uint4* sz = reinterpret_cast<uint4*>(sh.u.seen);
#pragma unroll
    for (int i = 0; i < WarpSmem<R>::VMAX / 16 / 32; ++i) sz[lane + 32 * i] = make_uint4(0, 0, 0, 0);
  }
  __syncwarp();

  // ---- presence scatter from the packed history (RepetitionPenalty's gather
  //      set); racing stores of the same byte need no atomics ---------------
  int hist_len = 0;
  if (history) {
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
    for (int r0 = lane; r0 < nwork; r0 += U * 32) {
      int4 ids[U];
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int rr = r0 + q * 32;
        ids[q] = make_int4(-1, -1, -1, -1);
        if (rr < nrest)
          ids[q].x = __ldg(hp + (rr < nhead ? o0 + rr : mid1 + (rr - nhead)));
        else if (rr < nwork)
          ids[q] = __ldg(reinterpret_cast<const int4*>(hp + mid0) + (rr - nrest));
      }
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int rr = r0 + q * 32;
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
    __syncwarp();
  }
  const float T = a.temperature ? __ldg(a.temperature + b) : a.temperature_default;
  const float pen = a.penalty ? __ldg(a.penalty + b) : a.penalty_default;
  const float top_p = a.top_p ? __ldg(a.top_p + b) : a.top_p_default;
  const int kk = a.top_k ? __ldg(a.top_k + b) : a.K;
  const int min_new = a.min_new ? __ldg(a.min_new + b) : a.min_new_default;
  const float u = a.uniforms ? __ldg(a.uniforms + b) : 0.0f;
  const int cur = a.cur_len ? __ldg(a.cur_len + b) : hist_len;
  const bool gate = eos_id >= 0 && eos_id < V && cur < min_new;

  int id = 0, flags = 0;
  const bool greedy = !(T > 0.0f);
  const int K = greedy ? 1 : kk;
  const bool few = greedy || (kk > 0 && kk < V);
  // the candidate path's approximate keys need a penalty and a temperature in
  // the normal window, and room for K plus its margin in WCAP
  const bool window_ok = (pen >= 0x1p-20f && pen <= 0x1p20f) &&
                         (greedy || (T >= 0x1p-20f && T <= 0x1p20f)) && K <= WCAP / 2;
  const bool cand_path = few && window_ok;
  const bool divT = !greedy && T != 1.0f;  // x / 1 == x exactly

  if (!mbar_wait_bounded(&sh.bar, 0)) {
    // the copy did not complete in time: report, wait once more (bounded)
    // so that no copy is left writing into a retired CTA's memory, give up
    (void)mbar_wait_bounded(&sh.bar, 0);
    if (lane == 0) {
      if (a.ids64) a.ids64[b] = 0;
      if (a.ids32) a.ids32[b] = 0;
      if (a.row_flags) a.row_flags[b] = Q3S_ROW_FALLBACK;
      if (a.error_word) atomicOr(a.error_word, static_cast<int>(err | Q3S_DEVERR_WAIT_TIMEOUT));
    }
    return;
  }

  auto app_nib = [&](int r) -> uint32_t { return (sh.appb[(r >> 1) * 32 + lane] >> (4 * (r & 1))) & 15u; };
  // the exact s of entry v: the processors of the first pass and s = x'/T,
  // recomputed from the logits in global memory
  auto exact_s = [&](int v) -> float {
    float x = BF16 ? bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(grow)[v])
                   : reinterpret_cast<const float*>(grow)[v];
    if (suppress && suppress[v]) x = NEG_SUPPRESS;
    if (gate && v == eos_id) x = -INFINITY;
    const int h = v >> 2, r = h >> 5, l = h & 31;
    const uint32_t app = (sh.appb[(r >> 1) * 32 + l] >> (4 * (r & 1) + (v & 3))) & 1u;
    if (app) x = x > 0.0f ? __fdiv_rn(x, pen) : __fmul_rn(x, pen);
    return divT ? __fdiv_rn(x, T) : x;
  };
  // running maximum of s (and the last index holding it) and torch.argmax of
  // s (first index) over this lane's entries, vocabulary order
  float lm = -INFINITY, gv = -INFINITY;
  int llast = -1, gi = 0x7fffffff;
  auto track = [&](float s, int v) {
    if (s > lm) {
      lm = s;
      llast = v;
    } else if (s == lm) {
      llast = v;
    }
    if (arg_better(s, v, gv, gi)) {
      gv = s;
      gi = v;
    }
  };

  // ---- first pass: suppress (-1e9, talker_unified_modules.py:409), the EOS
  //      gate (-inf), the repetition penalty (x * pen for entries <= 0; the
  //      division of present entries > 0 and the temperature wait for the
  //      whole-vocabulary path, which does them here) ------------------------
  {
    const uint2* stg = reinterpret_cast<const uint2*>(reinterpret_cast<const unsigned char*>(sh.row) + stage_off);
    uint32_t nib = 0;
#pragma unroll 2
    for (int r = 0; r < RQ; ++r) {
      const int h = lane + 32 * r;
      const bool in = 4 * h < V;
      float v[4];
      if (BF16) {
        // widening in place: round r reads bf16 bytes [stage_off + 256 r,
        // +256) and writes fp32 bytes [512 r, +512); stage_off = 256 RQ, so
        // the writes end where the next round's reads begin, at the latest
        uint2 q = make_uint2(0u, 0u);
        if (in) q = stg[h];
        __syncwarp();
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
      uint32_t app = 0;
      if (in) {
        if (suppress) {
          const uint32_t m4 = __ldg(reinterpret_cast<const uint32_t*>(suppress + 4 * h));
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if ((m4 >> (8 * j)) & 0xffu) v[j] = NEG_SUPPRESS;
        }
        if (history) {
          const uint32_t f = *reinterpret_cast<const uint32_t*>(&sh.u.seen[4 * h]);
#pragma unroll
          for (int j = 0; j < 4; ++j) app |= (((f >> (8 * j)) & 0xffu) ? 1u : 0u) << j;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (gate && 4 * h + j == eos_id) v[j] = -INFINITY;
          if ((app >> j) & 1u) {
            if (v[j] > 0.0f) {
              if (!cand_path) v[j] = __fdiv_rn(v[j], pen);
            } else {
              v[j] = __fmul_rn(v[j], pen);
            }
          }
          if (!cand_path) {
            if (divT) v[j] = __fdiv_rn(v[j], T);
            track(v[j], 4 * h + j);
          }
        }
        sh.row[h] = make_float4(v[0], v[1], v[2], v[3]);
      }
      nib |= app << (4 * (r & 1));
      if (r & 1) {
        sh.appb[(r >> 1) * 32 + lane] = static_cast<uint8_t>(nib);
        nib = 0;
      }
      if (BF16) __syncwarp();
    }
  }
  __syncwarp();  // every presence read is done before the union is reused

  bool done = false;
  if (cand_path) {
    // ---- few survivors: select on approximate keys (x * RN(1/pen) instead
    //      of x / pen, within a few ulps), resolve exactly on the candidates
    //      within 40 key units of the threshold or above ----------------------
    const float rpen = __frcp_rn(pen);
    auto akeys = [&](int r, uint32_t (&key)[4]) -> uint32_t {
      const int h = lane + 32 * r;
      if (4 * h >= V) {
#pragma unroll
        for (int j = 0; j < 4; ++j) key[j] = 0u;
        return 0u;
      }
      const float4 q = sh.row[h];
      const float v[4] = {q.x, q.y, q.z, q.w};
      const uint32_t app = app_nib(r);
#pragma unroll
      for (int j = 0; j < 4; ++j) key[j] = f2key((((app >> j) & 1u) && v[j] > 0.0f) ? __fmul_rn(v[j], rpen) : v[j]);
      return 15u;
    };
    const uint32_t thr = warp_select_rows<RQ>(sh.hist[0], K, WCAP / 2 + K / 2, akeys);
    const uint32_t lo = thr > 40u ? thr - 40u : 0u;
    // candidate records {0, index, x' (not yet divided by pen), 1 if x / pen
    // is due}, in vocabulary order; two rounds per scan (counts <= 4 each)
    uint32_t base = 0;
#pragma unroll 1
    for (int r = 0; r < RQ; r += 2) {
      uint32_t key0[4], key1[4];
      const uint32_t act0 = akeys(r, key0), act1 = akeys(r + 1, key1);
      uint32_t cm0 = 0, cm1 = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (((act0 >> j) & 1u) && key0[j] >= lo) cm0 |= 1u << j;
        if (((act1 >> j) & 1u) && key1[j] >= lo) cm1 |= 1u << j;
      }
      uint32_t tot;
      const uint32_t ex = warp_excl_scan_u(__popc(cm0) | (__popc(cm1) << 16), tot);
      const uint32_t t0 = tot & 0xffffu, t1 = tot >> 16;
      if (base + t0 + t1 <= static_cast<uint32_t>(WCAP)) {
        uint32_t p0 = base + (ex & 0xffffu), p1 = base + t0 + (ex >> 16);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint32_t cm = q ? cm1 : cm0;
          if (!cm) continue;
          const int rr = r + q;
          const int h = lane + 32 * rr;
          const float4 f = sh.row[h];
          const float v[4] = {f.x, f.y, f.z, f.w};
          const uint32_t app = app_nib(rr);
          uint32_t& p = q ? p1 : p0;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if ((cm >> j) & 1u) {
              sh.u.cand[p] = make_uint4(0u, static_cast<uint32_t>(4 * h + j), __float_as_uint(v[j]),
                                        (((app >> j) & 1u) && v[j] > 0.0f) ? 1u : 0u);
              ++p;
            }
        }
      }
      base += t0 + t1;
    }
    const int n = static_cast<int>(base);
    if (n <= WCAP) {
      __syncwarp();
      constexpr int Q = WCAP / 32;
      // exact x' = x / pen for the flagged candidates
#pragma unroll 1
      for (int i = 0; i < Q; ++i) {
        const int p = lane + 32 * i;
        if (p < n && sh.u.cand[p].w) {
          sh.u.cand[p].z = __float_as_uint(__fdiv_rn(__uint_as_float(sh.u.cand[p].z), pen));
          sh.u.cand[p].w = 0u;
        }
      }
      __syncwarp();
      if (greedy) {
        // argmax of x' (torch.argmax order: lowest index on ties)
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < Q; ++i) {
          const int p = lane + 32 * i;
          if (p < n) {
            const float xv = __uint_as_float(sh.u.cand[p].z);
            const int iv = static_cast<int>(sh.u.cand[p].y);
            if (arg_better(xv, iv, bv, bi)) {
              bv = xv;
              bi = iv;
            }
          }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          const float ov = __shfl_xor_sync(FULL, bv, o);
          const int oi = __shfl_xor_sync(FULL, bi, o);
          if (arg_better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
          }
        }
        id = bi;
        flags = Q3S_ROW_GREEDY;
        done = true;
      } else {
        // s = x'/T; HF TopK keeps s >= the K-th largest s (ties kept)
        float m = -INFINITY;
#pragma unroll 1
        for (int i = 0; i < Q; ++i) {
          const int p = lane + 32 * i;
          if (p < n) {
            const float s = __fdiv_rn(__uint_as_float(sh.u.cand[p].z), T);
            sh.u.cand[p].x = __float_as_uint(s);
            m = fmaxf(m, s);
          }
        }
        m = warp_max_f(m);
        __syncwarp();
        const uint32_t ks = warp_select_list(sh.u.cand, n, sh.hist[0], K, K);
        // quotients far from 1 may merge more than 40 key units of x': the
        // candidate set is proven complete only inside this window
        const float sk = fabsf(key2f(ks));
        if (m != -INFINITY && sk >= 0x1p-100f && sk <= 0x1p100f) {
          unsigned long long lq = 0;
#pragma unroll
          for (int i = 0; i < Q; ++i) {
            const int p = lane + 32 * i;
            if (p < n) {
              const float s = __uint_as_float(sh.u.cand[p].x);
              const bool sv = f2key(s) >= ks;
              const float wgt = sv ? softmax_weight(s, m) : 0.0f;
              sh.keep[p] = sv;
              sh.u.cand[p].w = __float_as_uint(wgt);
              lq += sv ? mass_fixed(wgt) : 0ull;
            }
          }
          __syncwarp();
          if (top_p < 1.0f) {
            const unsigned long long Zq = warp_sum_u64(lq);
            const float frac = __fsub_rn(1.0f, top_p);
            const unsigned long long tau = __double2ull_rd(static_cast<double>(frac) * static_cast<double>(Zq));
            if (tau >= Zq)
              warp_keep_last_list(sh.u.cand, sh.keep, n);
            else
              flags |= warp_mass_cut_list(sh.u.cand, sh.keep, n, tau, 0ull, Zq / 1000000ull, sh.hist[0], sh.hist[1]);
          }
          const int pos = warp_draw_list(sh.u.cand, sh.keep, n, u, flags);
          id = static_cast<int>(sh.u.cand[pos].y);
          done = true;
        }
      }
      __syncwarp();
    }
    if (!done) {
      // the candidate set overflowed or left the proven window: finish s for
      // the whole row in place
#pragma unroll 2
      for (int r = 0; r < RQ; ++r) {
        const int h = lane + 32 * r;
        if (4 * h >= V) continue;
        const float4 f = sh.row[h];
        float v[4] = {f.x, f.y, f.z, f.w};
        const uint32_t app = app_nib(r);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (((app >> j) & 1u) && v[j] > 0.0f) v[j] = __fdiv_rn(v[j], pen);
          if (divT) v[j] = __fdiv_rn(v[j], T);
          track(v[j], 4 * h + j);
        }
        sh.row[h] = make_float4(v[0], v[1], v[2], v[3]);
      }
      __syncwarp();
    }
  }

  if (!done) {
    // ---- whole-vocabulary rows: the row holds s -------------------------
    flags = 0;
    const float m = warp_max_f(lm);
    if (greedy) {
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, gv, o);
        const int oi = __shfl_xor_sync(FULL, gi, o);
        if (arg_better(ov, oi, gv, gi)) {
          gv = ov;
          gi = oi;
        }
      }
      id = gi;
      flags = Q3S_ROW_GREEDY;
    } else if (m == -INFINITY) {
      // nothing finite: report it and take the lowest index
      err |= Q3S_DEVERR_NO_MASS;
      flags = Q3S_ROW_FALLBACK;
      id = 0;
    } else {
      // the ascending-last entry: largest s, then largest index (it survives
      // top-k, which keeps ties at the top)
      int last = lm == m ? llast : -1;
#pragma unroll
      for (int o = 16; o; o >>= 1) last = max(last, __shfl_xor_sync(FULL, last, o));
      // top-k survivors: s >= the k-th largest s (ties kept)
      const bool topk = kk > 0 && kk < V;
      uint32_t kth = 0;
      if (topk) {
        kth = warp_select_rows<RQ>(sh.hist[0], kk, kk, [&](int r, uint32_t (&key)[4]) -> uint32_t {
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
      // ---- softmax weights in place; exact total mass; coarse histogram of
      //      approximate masses by the weight's exponent and top 4 mantissa
      //      bits (monotone in s) ----------------------------------------------
      const bool cut = top_p < 1.0f;
      unsigned long long lq = 0;
      uint32_t lc = 0;
#pragma unroll 2
      for (int r = 0; r < RQ; ++r) {
        const int h = lane + 32 * r;
        if (4 * h >= V) continue;
        const float4 f = sh.row[h];
        const float sv[4] = {f.x, f.y, f.z, f.w};
        float wv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const bool surv = !topk || f2key(sv[j]) >= kth;
          wv[j] = surv ? softmax_weight(sv[j], m) : 0.0f;
          if (cut && wv[j] > 0.0f) {
            lq += mass_fixed(wv[j]);
            const uint32_t c = __float2uint_rd(__fmul_rn(wv[j], static_cast<float>(1u << COARSE_SCALE_BITS)));
            lc += c;
            if (c) atomicAdd(&sh.hist[0][coarse_bin(wv[j])], c);
          }
        }
        sh.row[h] = make_float4(wv[0], wv[1], wv[2], wv[3]);
      }
      __syncwarp();
      uint32_t blo = 0;  // the draw counts weights in coarse bins >= blo
      bool single = false;
      if (cut) {
        const unsigned long long Zq = warp_sum_u64(lq);
        const float frac = __fsub_rn(1.0f, top_p);
        const unsigned long long tau = __double2ull_rd(static_cast<double>(frac) * static_cast<double>(Zq));
        const unsigned long long eps = Zq / 1000000ull;
        uint32_t Zc = lc;
#pragma unroll
        for (int o = 16; o; o >>= 1) Zc += __shfl_xor_sync(FULL, Zc, o);
        const uint32_t tau_c = min(__double2uint_rd(static_cast<double>(frac) * static_cast<double>(Zc)),
                                   Zc > 0 ? Zc - 1 : 0u);
        const uint32_t bstar = warp_scan_coarse_asc(sh.hist[0], tau_c);
        if (tau >= Zq) {
          // everything but the ascending-last entry goes
          id = last;
          single = true;
        } else {
          // exact masses below and inside the coarse window [wlo, whi];
          // window entries become candidate records in vocabulary order
          const uint32_t wlo = bstar > 0 ? bstar - 1 : 0u;
          const uint32_t whi = bstar < 255 ? bstar + 1 : 255u;
          unsigned long long lb = 0, lw = 0;
          uint32_t base = 0;
#pragma unroll 1
          for (int r = 0; r < RQ; r += 2) {
            uint32_t cm[2] = {0u, 0u};
            float wq[2][4];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const int h = lane + 32 * (r + q);
              const float4 f = (4 * h < V) ? sh.row[h] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
              wq[q][0] = f.x;
              wq[q][1] = f.y;
              wq[q][2] = f.z;
              wq[q][3] = f.w;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float w1 = wq[q][j];
                if (w1 > 0.0f) {
                  const uint32_t bn = coarse_bin(w1);
                  const unsigned long long q1 = mass_fixed(w1);
                  if (bn < wlo) {
                    lb += q1;
                  } else if (bn <= whi) {
                    lw += q1;
                    cm[q] |= 1u << j;
                  }
                }
              }
            }
            uint32_t tot;
            const uint32_t ex = warp_excl_scan_u(__popc(cm[0]) | (__popc(cm[1]) << 16), tot);
            const uint32_t t0 = tot & 0xffffu, t1 = tot >> 16;
            if (base + t0 + t1 <= static_cast<uint32_t>(WCAP)) {
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                uint32_t p = base + (q ? t0 + (ex >> 16) : (ex & 0xffffu));
                const int h = lane + 32 * (r + q);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  if ((cm[q] >> j) & 1u) {
                    sh.u.cand[p] = make_uint4(0u, static_cast<uint32_t>(4 * h + j), 0u, __float_as_uint(wq[q][j]));
                    sh.keep[p] = 1;
                    ++p;
                  }
              }
            }
            base += t0 + t1;
          }
          const unsigned long long below = warp_sum_u64(lb);
          const unsigned long long wmass = warp_sum_u64(lw);
          const int n = static_cast<int>(base);
          __syncwarp();
          if (below <= tau && tau < below + wmass && n <= WCAP) {
            // the cut lies inside the window: exact s of its entries, the
            // exact cut, and removed entries' weights zeroed in the row
#pragma unroll 1
            for (int i = 0; i < WCAP / 32; ++i) {
              const int p = lane + 32 * i;
              if (p < n) sh.u.cand[p].x = __float_as_uint(exact_s(static_cast<int>(sh.u.cand[p].y)));
            }
            __syncwarp();
            flags |= warp_mass_cut_list(sh.u.cand, sh.keep, n, tau, below, eps, sh.hist[0], sh.hist[1]);
#pragma unroll 1
            for (int i = 0; i < WCAP / 32; ++i) {
              const int p = lane + 32 * i;
              if (p < n && !sh.keep[p]) rowf[sh.u.cand[p].y] = 0.0f;
            }
            blo = wlo;
          } else {
            // the coarse window missed (approximate masses) or holds too many
            // entries: an exact radix cut over every survivor, keys from the
            // exact s recomputed per entry
            auto skey = [&](int v) -> uint32_t { return f2key(exact_s(v)); };
            uint32_t prefix = 0, hmask = 0;
            unsigned long long bl = 0;
            constexpr uint32_t LO = (1u << MASS_LO_BITS) - 1u;
#pragma unroll 1
            for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll 1
              for (int r = 0; r < RQ; ++r) {
                const int h = lane + 32 * r;
                if (4 * h >= V) continue;
                const float4 f = sh.row[h];
                const float wv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const unsigned long long q1 = mass_fixed(wv[j]);
                  if (q1 == 0) continue;
                  const uint32_t key = skey(4 * h + j);
                  if ((key & hmask) == prefix) {
                    atomicAdd(&sh.hist[0][(key >> shift) & 255u], static_cast<uint32_t>(q1 >> MASS_LO_BITS));
                    atomicAdd(&sh.hist[1][(key >> shift) & 255u], static_cast<uint32_t>(q1) & LO);
                  }
                }
              }
              __syncwarp();
              uint32_t d;
              unsigned long long bef;
              warp_scan_mass_asc(sh.hist[0], sh.hist[1], bl, tau, d, bef);
              prefix |= d << shift;
              hmask |= 255u << shift;
              bl = bef;
            }
            const uint32_t vstar = prefix;
            // the entries at vstar share one s, one weight and one mass
            unsigned long long qs = 0;
#pragma unroll 1
            for (int r = 0; r < RQ; ++r) {
              const int h = lane + 32 * r;
              if (4 * h >= V) continue;
              const float4 f = sh.row[h];
              const float wv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (mass_fixed(wv[j]) != 0 && skey(4 * h + j) == vstar) qs = mass_fixed(wv[j]);
            }
            const unsigned bq = __ballot_sync(FULL, qs != 0);
            qs = __shfl_sync(FULL, qs, bq ? __ffs(bq) - 1 : 0);
            qs = qs ? qs : 1ull;
            const unsigned long long nrem = (tau - bl) / qs;  // ties removed, lowest index first
            const unsigned long long first_kept = bl + (nrem + 1) * qs;
            const unsigned long long last_removed = bl + nrem * qs;
            if ((first_kept - tau) < eps || (tau - last_removed) < eps) flags |= Q3S_ROW_TOPP_BOUNDARY;
            unsigned long long tb = 0;  // ties in earlier rounds
#pragma unroll 1
            for (int r = 0; r < RQ; ++r) {
              const int h = lane + 32 * r;
              const bool in = 4 * h < V;
              float wv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
              uint32_t key[4] = {0u, 0u, 0u, 0u};
              uint32_t ce = 0;
              if (in) {
                const float4 f = sh.row[h];
                wv[0] = f.x;
                wv[1] = f.y;
                wv[2] = f.z;
                wv[3] = f.w;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  key[j] = wv[j] > 0.0f ? skey(4 * h + j) : 0u;
                  if (mass_fixed(wv[j]) != 0 && key[j] == vstar) ce |= 1u << j;
                }
              }
              uint32_t tot;
              uint32_t t_in = warp_excl_scan_u(__popc(ce), tot);
              if (in) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  bool kp = false;
                  if (wv[j] > 0.0f) {
                    if (key[j] > vstar) {
                      kp = true;
                    } else if ((ce >> j) & 1u) {
                      kp = tb + t_in >= nrem;
                      ++t_in;
                    }
                  }
                  if (!kp) wv[j] = 0.0f;
                }
                sh.row[h] = make_float4(wv[0], wv[1], wv[2], wv[3]);
              }
              tb += tot;
            }
            blo = 0;
          }
          __syncwarp();
        }
      }
      if (!single) {
        // ---- inverse CDF in vocabulary order: cumulative weight before each
        //      quad (round scans), then the first quad whose running sum
        //      passes u * total, then the entry inside it -------------------
        float carry = 0.0f;
        int lastv = -1;
#pragma unroll 1
        for (int r = 0; r < RQ; ++r) {
          const int h = lane + 32 * r;
          float qsum = 0.0f;
          if (4 * h < V) {
            const float4 f = sh.row[h];
            const float wv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float w1 = (wv[j] > 0.0f && coarse_bin(wv[j]) >= blo) ? wv[j] : 0.0f;
              qsum = __fadd_rn(qsum, w1);
              if (w1 > 0.0f) lastv = 4 * h + j;
            }
          }
          float tot;
          const float exs = warp_excl_scan_f(qsum, tot);
          sh.u.ex[r * 32 + lane] = __fadd_rn(carry, exs);
          carry = __fadd_rn(carry, tot);
        }
        __syncwarp();
        const float W = carry;
        const float thr = __fmul_rn(u, W);
        // this lane's first quad (vocabulary order) whose running sum > thr
        int firstq = 0x7fffffff;
#pragma unroll 1
        for (int r = 0; r < RQ; ++r) {
          const int h = lane + 32 * r;
          if (4 * h >= V) break;
          const float4 f = sh.row[h];
          const float wv[4] = {f.x, f.y, f.z, f.w};
          float acc = sh.u.ex[r * 32 + lane];
          bool hit = false;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float w1 = (wv[j] > 0.0f && coarse_bin(wv[j]) >= blo) ? wv[j] : 0.0f;
            acc = __fadd_rn(acc, w1);
            hit |= w1 > 0.0f && acc > thr;
          }
          if (hit) {
            firstq = r * 32 + lane;
            break;
          }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          firstq = min(firstq, __shfl_xor_sync(FULL, firstq, o));
          lastv = max(lastv, __shfl_xor_sync(FULL, lastv, o));
        }
        if (firstq == 0x7fffffff) {
          id = lastv;
          flags |= Q3S_ROW_FALLBACK;
        } else {
          const int ol = firstq & 31, orr = firstq >> 5;
          int pick = 0, near = 0;
          if (lane == ol) {
            const int h = lane + 32 * orr;
            const float4 f = sh.row[h];
            const float wv[4] = {f.x, f.y, f.z, f.w};
            const float pre = sh.u.ex[orr * 32 + lane];
            float acc = pre, prev = pre, cdf = pre;
            bool found = false;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float w1 = (wv[j] > 0.0f && coarse_bin(wv[j]) >= blo) ? wv[j] : 0.0f;
              const float before = acc;
              acc = __fadd_rn(acc, w1);
              if (!found && w1 > 0.0f && acc > thr) {
                found = true;
                pick = 4 * h + j;
                prev = before;
                cdf = acc;
              }
            }
            const float tol = BOUNDARY_EPS * W;
            near = (__fsub_rn(cdf, thr) < tol) || (__fsub_rn(thr, prev) < tol);
          }
          id = __shfl_sync(FULL, pick, ol);
          if (__shfl_sync(FULL, near, ol)) flags |= Q3S_ROW_DRAW_BOUNDARY;
        }
      }
    }
  }
  if (lane == 0) {
    if (a.ids64) a.ids64[b] = id;
    if (a.ids32) a.ids32[b] = id;
    if (a.row_flags) a.row_flags[b] = flags;
  }
  if (err && a.error_word) atomicOr(a.error_word, static_cast<int>(err));
}

}  // namespace q3s
