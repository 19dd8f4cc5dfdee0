// q3s_core.cuh -- the register-resident exact sampler core shared by the
// CTA-per-row kernel (q3s_sampler.cu) and the register-resident row kernel
// (q3s_lean.cu): row loads, suppress / presence masks, sample_exact (rows
// that keep the whole vocabulary, and the exact fallback) and sample_core
// (the per-row sampler over E entries a thread).
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "q3s_args.cuh"
#include "q3s_device.cuh"

namespace q3s {

// ---------------------------------------------------------------------------
// loads
// ---------------------------------------------------------------------------

// The E logits of vocabulary entries [v0, v0+E) of one row, as fp32.  `shift`
// (in [0,V)) reads column v at (v + shift) mod V.  Entries >= V are -inf and
// cleared from `vmask`.
template <bool BF16, int E>
Q3S_DEV void load_logits(const void* base, int64_t row_off, int V, int v0, int shift, bool vec, float (&x)[E],
                         uint32_t& vmask) {
  vmask = 0;
  if (shift == 0 && vec && v0 + E <= V) {
    if (BF16) {
      const uint16_t* p = static_cast<const uint16_t*>(base) + row_off + v0;
#pragma unroll
      for (int c = 0; c < E / 8; ++c) {
        const uint4 r = ld_stream16(p + 8 * c);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          x[8 * c + 2 * i] = bf16_bits_to_f32(w[i] & 0xffffu);
          x[8 * c + 2 * i + 1] = bf16_bits_to_f32(w[i] >> 16);
        }
      }
    } else {
      const float* p = static_cast<const float*>(base) + row_off + v0;
#pragma unroll
      for (int c = 0; c < E / 4; ++c) {
        const uint4 r = ld_stream16(p + 4 * c);
        x[4 * c] = __uint_as_float(r.x);
        x[4 * c + 1] = __uint_as_float(r.y);
        x[4 * c + 2] = __uint_as_float(r.z);
        x[4 * c + 3] = __uint_as_float(r.w);
      }
    }
    vmask = (E == 32) ? 0xffffffffu : ((1u << E) - 1u);
    return;
  }
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const int v = v0 + j;
    x[j] = -INFINITY;
    if (v < V) {
      int q = v + shift;
      if (q >= V) q -= V;
      if (BF16)
        x[j] = bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(base) + row_off + q));
      else
        x[j] = __ldg(static_cast<const float*>(base) + row_off + q);
      vmask |= 1u << j;
    }
  }
}

// E byte flags (nonzero = set), 8-byte aligned -> bitmask.
template <int E>
Q3S_DEV uint32_t bytes_to_mask(const uint8_t* p) {
  uint32_t m = 0;
#pragma unroll
  for (int c = 0; c < E / 8; ++c) {
    const uint2 f = *reinterpret_cast<const uint2*>(p + 8 * c);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      m |= (((f.x >> (8 * j)) & 0xffu) ? 1u : 0u) << (8 * c + j);
      m |= (((f.y >> (8 * j)) & 0xffu) ? 1u : 0u) << (8 * c + j + 4);
    }
  }
  return m;
}

Q3S_DEV int norm_shift(int64_t s, int V) {
  int64_t r = s % V;
  if (r < 0) r += V;
  return static_cast<int>(r);
}

// ---------------------------------------------------------------------------
// the shared per-row sampler
// ---------------------------------------------------------------------------

struct RowCfg {
  int mode;
  bool greedy;
  float T;
  int k;            // gumbel: K; icdf: top-k (<=0 or >=V: off)
  float top_p;
  float u;
  const float* noise;  // gumbel noise of this row, indexed by rank
};

// Exact path: samples one id from the processed logits v (post suppress /
// penalty / EOS gate, every entry exact; v is overwritten).  Used for rows
// that keep the whole vocabulary and as the fallback of sample_core.  Every
// thread returns the same id; `flags` is complete in the thread that owns the
// id (v0 <= id < v0+E).  `processed` (optional) receives the row handed to
// the draw: g0 (gumbel), the filtered s (icdf), x (greedy).  Needs sh.hist
// all-zero on entry and leaves it so.
template <int NT, int E, int MODE>
Q3S_DEV int sample_exact(float (&v)[E], uint32_t vmask, int V, const RowCfg& c, Scratch<NT, E>& sh,
                         float* processed, int& flags, uint32_t& err) {
  const int t = threadIdx.x;
  const int v0 = t * E;
  int rb = 0;
  flags = 0;
  if (t == 0) sh.flags = 0;  // published by the first barrier below

  if (c.greedy) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (((vmask >> j) & 1u) && arg_better(v[j], v0 + j, bv, bi)) {
        bv = v[j];
        bi = v0 + j;
      }
    if (processed) {
#pragma unroll
      for (int j = 0; j < E; ++j)
        if ((vmask >> j) & 1u) processed[v0 + j] = v[j];
    }
    flags = Q3S_ROW_GREEDY;
    return block_argmax<NT, E>(bv, bi, bi, sh, rb);
  }

  if (MODE == Q3S_DRAW_GUMBEL) {
    // talker_unified_modules.py:415-420 / utils.py:1189-1193
    const int K = c.k;
    const int K4 = (K + 3) & ~3;
    for (int r = t; r < K; r += NT) sh.noise[r] = __ldg(c.noise + r);
    for (int r = K + t; r < K4; r += NT) sh.cand[r] = make_uint4(0u, 0x7fffffffu, 0u, 0u);  // never outranks
    if (processed) {
#pragma unroll
      for (int j = 0; j < E; ++j)
        if ((vmask >> j) & 1u) processed[v0 + j] = v[j];
    }
    uint32_t key[E];
#pragma unroll
    for (int j = 0; j < E; ++j) key[j] = f2key(v[j]);
    const uint32_t kth = select_kth_largest<NT, E>(key, vmask, K, sh, rb);
    uint32_t cg = 0, ce = 0;
#pragma unroll
    for (int j = 0; j < E; ++j)
      if ((vmask >> j) & 1u) {
        cg += key[j] > kth;
        ce += key[j] == kth;
      }
    uint32_t tot;
    const uint32_t ex = block_excl_scan_u<NT, E>((cg << 16) | ce, tot, sh, rb);
    const uint32_t gt_tot = tot >> 16;
    const uint32_t need = static_cast<uint32_t>(K) - gt_tot;  // ties admitted, lowest index first
    uint32_t pg = ex >> 16, pe = ex & 0xffffu;
#pragma unroll
    for (int j = 0; j < E; ++j) {
      if (!((vmask >> j) & 1u)) continue;
      int slot = -1;
      if (key[j] > kth) {
        slot = static_cast<int>(pg++);
      } else if (key[j] == kth) {
        if (pe < need) slot = static_cast<int>(gt_tot + pe);
        ++pe;
      }
      if (slot >= K) {  // cannot happen when kth is exact; never write past the set
        err |= Q3S_DEVERR_CANDIDATES;
        slot = -1;
      }
      if (slot >= 0) sh.cand[slot] = make_uint4(key[j], static_cast<uint32_t>(v0 + j), __float_as_uint(v[j]), 0u);
    }
    __syncthreads();
    float bs = -INFINITY;
    int br = 0x7fffffff, bid = 0x7fffffff;
    for (int ci = t; ci < K; ci += NT) {
      const uint4 me = sh.cand[ci];
      const int ic = static_cast<int>(me.y);
      int rank = 0;
      for (int o = 0; o < K4; o += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 ot = sh.cand[o + u];
          rank += (ot.x > me.x) | ((ot.x == me.x) & (static_cast<int>(ot.y) < ic));
        }
      }
      const float score = __fadd_rn(__fdiv_rn(__uint_as_float(me.z), c.T), sh.noise[rank]);
      if (arg_better(score, rank, bs, br)) {
        bs = score;
        br = rank;
        bid = ic;
      }
    }
    return block_argmax<NT, E>(bs, br, bid, sh, rb);
  }

  // ---- icdf: Temperature -> TopK -> TopP -> softmax -> inverse CDF ----------
  uint32_t key[E];
  uint32_t smask = vmask;
  if (c.k > 0 && c.k < V) {
    // HF TopKLogitsWarper keeps s >= (k-th largest s), s = x / T.  Division
    // by T > 0 is monotone, so the k-th largest s is RN(x_k / T) with x_k the
    // k-th largest x, and the survivors are {x >= x_k} plus entries just below
    // x_k whose quotient rounds onto it.  While quotients stay normal, one
    // quotient's preimage spans < 2.0001 ulps of x, so only the 4 floats below
    // x_k are divided to check; otherwise every entry is divided.
#pragma unroll
    for (int j = 0; j < E; ++j) key[j] = f2key(v[j]);
    const uint32_t kx = select_kth_largest<NT, E>(key, vmask, c.k, sh, rb);
    const float sk = __fdiv_rn(key2f(kx), c.T);
    const float ask = fabsf(sk);
    const bool window = ask >= 0x1p-100f && ask <= 0x1p100f && c.T >= 0x1p-20f && c.T <= 0x1p20f;
    smask = 0;
#pragma unroll
    for (int j = 0; j < E; ++j) {
      if (!((vmask >> j) & 1u)) continue;
      if (key[j] >= kx) {
        v[j] = __fdiv_rn(v[j], c.T);
        smask |= 1u << j;
      } else if (!window || kx - key[j] <= 4u) {
        const float sj = __fdiv_rn(v[j], c.T);
        if (sj == sk) {
          v[j] = sj;
          smask |= 1u << j;
        }
      }
    }
  } else if (c.T != 1.0f) {  // x / 1 == x exactly
#pragma unroll
    for (int j = 0; j < E; ++j)
      if ((vmask >> j) & 1u) v[j] = __fdiv_rn(v[j], c.T);
  }
  float lm = -INFINITY;
#pragma unroll
  for (int j = 0; j < E; ++j)
    if ((smask >> j) & 1u) lm = fmaxf(lm, v[j]);
  uint32_t n;
  float m;
  const uint32_t pos0 = block_scan_count_max<NT, E>(__popc(smask), lm, n, m, sh, rb);
  if (m == -INFINITY) {
    // nothing finite survived: report and take the lowest index
    err |= Q3S_DEVERR_NO_MASS;
    flags = Q3S_ROW_FALLBACK;
    int first = 0x7fffffff;
#pragma unroll
    for (int j = E - 1; j >= 0; --j)
      if ((vmask >> j) & 1u) first = v0 + j;
    return block_min_i<NT, E>(first, sh, rb);
  }

  if (n <= static_cast<uint32_t>(FINISH < NT ? FINISH : NT)) {
    // ---- few survivors (every top-k row): finish on a compact list --------
    // Candidate records in vocabulary order; top-p by all-pairs masses (one
    // candidate per thread); the draw runs in warp 0 alone.
    const int n4 = (static_cast<int>(n) + 3) & ~3;
    uint32_t pos = pos0;
#pragma unroll
    for (int j = 0; j < E; ++j)
      if ((smask >> j) & 1u) {
        sh.cand[pos] = make_uint4(f2key(v[j]), static_cast<uint32_t>(v0 + j),
                                  __float_as_uint(softmax_weight(v[j], m)), 0u);
        ++pos;
      }
    if (t >= static_cast<int>(n) && t < n4) sh.cand[t] = make_uint4(0u, 0x7fffffffu, 0u, 0u);  // weightless
    if (t < n4) sh.keep[t] = 1;
    __syncthreads();
    if (c.top_p < 1.0f) {
      // HF TopPLogitsWarper over a stable ascending order (value asc, index
      // asc): remove an entry when the softmax mass at-or-below it is <= 1-p;
      // the ascending-last entry always stays.
      const float frac = __fsub_rn(1.0f, c.top_p);
      if (t < static_cast<int>(n)) {
        const uint4 me = sh.cand[t];
        const int ic = static_cast<int>(me.y);
        float cum = 0.0f, Z = 0.0f;
        int after = 0;
        for (int o = 0; o < n4; o += 4) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint4 ot = sh.cand[o + u];
            const float w = __uint_as_float(ot.z);
            const bool before = (ot.x < me.x) | ((ot.x == me.x) & (static_cast<int>(ot.y) <= ic));
            cum = __fadd_rn(cum, before ? w : 0.0f);
            Z = __fadd_rn(Z, w);
            after += (!before) & (static_cast<int>(ot.y) != 0x7fffffff);
          }
        }
        const float thr = __fmul_rn(frac, Z);
        sh.keep[t] = (after == 0) || !(cum <= thr);
        if (after != 0 && fabsf(__fsub_rn(cum, thr)) < BOUNDARY_EPS * Z) atomicOr(&sh.flags, Q3S_ROW_TOPP_BOUNDARY);
      }
      __syncthreads();
    }
    if (t < 32) {
      // inverse CDF over the kept candidates: lane l owns positions 4l..4l+3
      const int lane = t;
      float w[4], acc[4], a = 0.0f;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int i = 4 * lane + r;
        w[r] = (i < static_cast<int>(n) && sh.keep[i]) ? __uint_as_float(sh.cand[i].z) : 0.0f;
        a = __fadd_rn(a, w[r]);
        acc[r] = a;
      }
      float inc = a;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float nb = __shfl_up_sync(FULL, inc, o);
        if (lane >= o) inc = __fadd_rn(inc, nb);
      }
      float pre = __shfl_up_sync(FULL, inc, 1);
      if (lane == 0) pre = 0.0f;
      const float W = __shfl_sync(FULL, inc, 31);
      const float thr = __fmul_rn(c.u, W);
      int r_first = -1;
#pragma unroll
      for (int r = 3; r >= 0; --r)
        if (w[r] > 0.0f && __fadd_rn(pre, acc[r]) > thr) r_first = r;
      const unsigned hit = __ballot_sync(FULL, r_first >= 0);
      int src, rsel;
      bool fallback = false;
      if (hit) {
        src = __ffs(hit) - 1;
        rsel = __shfl_sync(FULL, r_first, src);
      } else {
        int r_last = -1;
#pragma unroll
        for (int r = 0; r < 4; ++r)
          if (w[r] > 0.0f) r_last = r;
        const unsigned any = __ballot_sync(FULL, r_last >= 0);
        src = any ? 31 - __clz(any) : 0;
        rsel = any ? __shfl_sync(FULL, r_last, src) : 0;
        fallback = true;
      }
      if (lane == src) {
        const int i = 4 * lane + rsel;
        float cdf = pre, prev = pre;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          if (r == rsel) cdf = __fadd_rn(pre, acc[r]);
          if (r < rsel) prev = __fadd_rn(pre, acc[r]);
        }
        int fl = fallback ? Q3S_ROW_FALLBACK : 0;
        const float tol = BOUNDARY_EPS * W;
        if ((__fsub_rn(cdf, thr) < tol) || (__fsub_rn(thr, prev) < tol)) fl |= Q3S_ROW_DRAW_BOUNDARY;
        if (fl) atomicOr(&sh.flags, fl);
        sh.sel_u[3] = sh.cand[i].y;
      }
    }
    __syncthreads();
    const int id = static_cast<int>(sh.sel_u[3]);
    flags = sh.flags;
    if (processed) {
      uint32_t p2 = pos0;
#pragma unroll
      for (int j = 0; j < E; ++j) {
        if (!((vmask >> j) & 1u)) continue;
        float out = -INFINITY;
        if ((smask >> j) & 1u) {
          if (sh.keep[p2]) out = v[j];
          ++p2;
        }
        processed[v0 + j] = out;
      }
    }
    return id;
  }

  // ---- many survivors (top-k off): block-wide top-p and draw -------------
#pragma unroll
  for (int j = 0; j < E; ++j) key[j] = f2key(v[j]);
  if (c.top_p < 1.0f) {
    // HF TopPLogitsWarper over a stable ascending order (value asc, index
    // asc): remove an entry when the softmax mass at-or-below it is <= 1-p;
    // the ascending-last entry always stays.
    const float frac = __fsub_rn(1.0f, c.top_p);
    {
      float w[E];
      unsigned long long lq = 0;
#pragma unroll
      for (int j = 0; j < E; ++j) {
        w[j] = ((smask >> j) & 1u) ? softmax_weight(v[j], m) : 0.0f;
        lq += ((smask >> j) & 1u) ? mass_fixed(w[j]) : 0ull;
      }
      const unsigned long long Zq = block_sum_q<NT, E>(lq, sh, rb);
      const unsigned long long tau = __double2ull_rd(static_cast<double>(frac) * static_cast<double>(Zq));
      if (tau >= Zq) {
        // everything but the ascending-last entry goes
        int last = -1;
#pragma unroll
        for (int j = 0; j < E; ++j)
          if (((smask >> j) & 1u) && v[j] == m) last = v0 + j;
        last = block_max_i<NT, E>(last, sh, rb);
        smask = (last >= v0 && last < v0 + E) ? (1u << (last - v0)) : 0u;
      } else {
        uint32_t vstar;
        unsigned long long below;
        select_mass_cut<NT, E>(key, w, smask, tau, sh, vstar, below);
        uint32_t ce = 0;
        unsigned long long qstar = 1;
#pragma unroll
        for (int j = 0; j < E; ++j)
          if (((smask >> j) & 1u) && key[j] == vstar) {
            ++ce;
            qstar = mass_fixed(w[j]);
          }
        uint32_t cet;
        uint32_t tr = block_excl_scan_u<NT, E>(ce, cet, sh, rb);
        qstar = qstar ? qstar : 1ull;
        const unsigned long long nrem = (tau - below) / qstar;  // ties removed (lowest index first)
        const unsigned long long eps = Zq / 1000000ull;
        uint32_t nm = 0;
        bool near = false;
#pragma unroll
        for (int j = 0; j < E; ++j) {
          if (!((smask >> j) & 1u)) continue;
          if (key[j] > vstar) {
            nm |= 1u << j;
          } else if (key[j] == vstar) {
            if (tr >= nrem) nm |= 1u << j;
            ++tr;
            const unsigned long long first_kept = below + (nrem + 1) * qstar;
            const unsigned long long last_removed = below + nrem * qstar;
            near = (first_kept - tau) < eps || (tau - last_removed) < eps;
          }
        }
        if (near) atomicOr(&sh.flags, Q3S_ROW_TOPP_BOUNDARY);
        smask = nm;
      }
    }
  }

  // inverse CDF in vocabulary order over the surviving softmax weights
  float lsum = 0.0f;
#pragma unroll
  for (int j = 0; j < E; ++j) lsum = __fadd_rn(lsum, ((smask >> j) & 1u) ? softmax_weight(v[j], m) : 0.0f);
  float W;
  const float pre = block_excl_scan_f<NT, E>(lsum, W, sh, rb);
  const float thr = __fmul_rn(c.u, W);
  int first = 0x7fffffff;
  {
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const float w = ((smask >> j) & 1u) ? softmax_weight(v[j], m) : 0.0f;
      acc = __fadd_rn(acc, w);
      if (first == 0x7fffffff && w > 0.0f && __fadd_rn(pre, acc) > thr) first = v0 + j;
    }
  }
  int id = block_min_i<NT, E>(first, sh, rb);
  bool fallback = false;
  if (id == 0x7fffffff) {
    int last = -1;
#pragma unroll
    for (int j = 0; j < E; ++j)
      if ((smask >> j) & 1u) last = v0 + j;
    id = block_max_i<NT, E>(last, sh, rb);
    fallback = true;
  }
  flags = sh.flags | (fallback ? Q3S_ROW_FALLBACK : 0);
  if (id >= v0 && id < v0 + E) {
    // owner: is the draw within 1e-6 (relative) of a CDF edge?
    float acc = 0.0f, prev = pre, cdf = pre;
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const float w = ((smask >> j) & 1u) ? softmax_weight(v[j], m) : 0.0f;
      acc = __fadd_rn(acc, w);
      const float cur = __fadd_rn(pre, acc);
      if (v0 + j == id) cdf = cur;
      if (v0 + j < id) prev = cur;
    }
    const float tol = BOUNDARY_EPS * W;
    if ((__fsub_rn(cdf, thr) < tol) || (__fsub_rn(thr, prev) < tol)) flags |= Q3S_ROW_DRAW_BOUNDARY;
  }
  if (processed) {
#pragma unroll
    for (int j = 0; j < E; ++j)
      if ((vmask >> j) & 1u) processed[v0 + j] = ((smask >> j) & 1u) ? v[j] : -INFINITY;
  }
  return id;
}

// Full sampler for one row.  x: logits after suppress and the EOS gate, before
// the repetition penalty, which applies to the entries flagged in `pmask`
// (x > 0 ? x / pen : x * pen).  Every thread returns the same id; `flags`
// is complete in the thread that owns the id (v0 <= id < v0+E).
//
// Rows that keep a few entries (top-k rows, Gumbel exactly-K rows, greedy
// rows) select on approximate keys -- the penalty division replaced by a
// multiply with RN(1/pen), within a few ulps of it -- and resolve exactly on
// a small candidate set: every entry whose approximate key is within 40 ulps
// of the selected threshold or above.  That set holds every entry of the
// exact top K (keys move by at most ~4 ulps), every entry below it sits at
// least 8 ulps under the exact K-th value, so no temperature-quotient tie can
// reach outside the set, and only its entries are divided exactly.  Rows that
// keep the whole vocabulary, or whose candidate set overflows (massive ties),
// take sample_exact.
template <int NT, int E, int MODE>
Q3S_DEV int sample_core(float (&x)[E], uint32_t vmask, uint32_t pmask, float pen, int V, const RowCfg& c,
                        Scratch<NT, E>& sh, float* processed, int& flags, uint32_t& err) {
  const int t = threadIdx.x;
  const int v0 = t * E;
  // negative penalised entries are exact products; dmask = entries still to divide
  uint32_t dmask = 0;
#pragma unroll
  for (int j = 0; j < E; ++j)
    if ((pmask >> j) & 1u) {
      if (x[j] > 0.0f)
        dmask |= 1u << j;
      else
        x[j] = __fmul_rn(x[j], pen);
    }
  const bool topk_row = c.greedy || MODE == Q3S_DRAW_GUMBEL || (c.k > 0 && c.k < V);
  const bool window_ok = c.greedy || MODE == Q3S_DRAW_GUMBEL || (c.T >= 0x1p-20f && c.T <= 0x1p20f);
  if (!topk_row || !window_ok) {
#pragma unroll
    for (int j = 0; j < E; ++j)
      if ((dmask >> j) & 1u) x[j] = __fdiv_rn(x[j], pen);
    return sample_exact<NT, E, MODE>(x, vmask, V, c, sh, processed, flags, err);
  }

  int rb = 0;
  flags = 0;
  if (t == 0) sh.flags = 0;  // published by the first barrier below
  const int K = c.greedy ? 1 : c.k;
  if (MODE == Q3S_DRAW_GUMBEL && !c.greedy) {
    for (int r = t; r < K; r += NT) sh.noise[r] = __ldg(c.noise + r);
  }
  float xa[E];
  {
    const float rpen = __frcp_rn(pen);
#pragma unroll
    for (int j = 0; j < E; ++j) xa[j] = ((dmask >> j) & 1u) ? __fmul_rn(x[j], rpen) : x[j];
  }
  // candidates: one 1/8-unit histogram below the largest value where that
  // locates the K-th tightly, else a radix threshold with a 40-ulp margin
  uint32_t cmask = 0;
  if (!select_bins8<NT, E>(xa, vmask, K, FINISH + K, sh, rb, cmask)) {
    uint32_t key[E];
#pragma unroll
    for (int j = 0; j < E; ++j) key[j] = f2key(xa[j]);
    const uint32_t thr = select_threshold<NT, E>(key, vmask, K, FINISH + K / 2, sh, rb);
    const uint32_t lo = thr > 40u ? thr - 40u : 0u;
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (((vmask >> j) & 1u) && key[j] >= lo) cmask |= 1u << j;
  }
  uint32_t n;
  const uint32_t pos0 = block_excl_scan_u<NT, E>(__popc(cmask), n, sh, rb);
  if (n > static_cast<uint32_t>(CAND)) {
#pragma unroll
    for (int j = 0; j < E; ++j)
      if ((dmask >> j) & 1u) x[j] = __fdiv_rn(x[j], pen);
    __syncthreads();  // shared state of this path is reused by sample_exact
    return sample_exact<NT, E, MODE>(x, vmask, V, c, sh, processed, flags, err);
  }
  // candidate records in vocabulary order: {s or x' bits, index, x' bits, weight bits}
  const int n4 = (static_cast<int>(n) + 3) & ~3;
  bool nonfinite = false;
  {
    uint32_t pos = pos0;
#pragma unroll
    for (int j = 0; j < E; ++j)
      if ((cmask >> j) & 1u) {
        const float xe = ((dmask >> j) & 1u) ? __fdiv_rn(x[j], pen) : x[j];
        sh.cand[pos] = make_uint4(0u, static_cast<uint32_t>(v0 + j), __float_as_uint(xe), 0u);
        sh.xs[pos] = xe;
        nonfinite |= !isfinite(xe);
        ++pos;
      }
    for (int i = static_cast<int>(n) + t; i < n4; i += NT) {
      sh.cand[i] = make_uint4(0xff800000u, 0x7fffffffu, 0xff800000u, 0u);  // -inf, never outranks
      sh.xs[i] = -INFINITY;
    }
  }
  nonfinite = __syncthreads_or(nonfinite) != 0;

  if (MODE == Q3S_DRAW_GUMBEL || c.greedy) {
    // exactly-K by (x' desc, index asc) (talker_unified_modules.py:415,
    // utils.py:1189); score x'/T + noise[rank]; argmax, lowest rank on ties.
    // Positions are in vocabulary order, so the rank of position i counts
    // x >= x_i before it and x > x_i after it: with every x' finite, one
    // compare per entry -- x > (the float below x_i) in quads wholly before
    // i's, x > x_i elsewhere, then the equal entries earlier in i's quad.
    float bs = -INFINITY;
    int br = 0x7fffffff, bid = 0x7fffffff;
    const float4* xs4 = reinterpret_cast<const float4*>(sh.xs);
    for (int i = t; i < static_cast<int>(n); i += NT) {
      const uint4 me = sh.cand[i];
      const float xi = __uint_as_float(me.z);
      const int ii = static_cast<int>(me.y);
      int rank = 0;
      if (!nonfinite) {
        const uint32_t bi = __float_as_uint(xi);
        const float xd = xi > 0.0f ? __uint_as_float(bi - 1u) : (xi < 0.0f ? __uint_as_float(bi + 1u) : -0x1p-149f);
        const int p4 = i >> 2;
#pragma unroll 4
        for (int q4 = 0; q4 < (n4 >> 2); ++q4) {
          const float4 f = xs4[q4];
          const float th = q4 < p4 ? xd : xi;
          rank += (f.x > th) + (f.y > th) + (f.z > th) + (f.w > th);
        }
        for (int q = 4 * p4; q < i; ++q) rank += sh.xs[q] == xi;
      } else {
        for (int o = 0; o < n4; o += 4) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint4 ot = sh.cand[o + u];
            const float xo = __uint_as_float(ot.z);
            rank += (xo > xi) | ((xo == xi) & (static_cast<int>(ot.y) < ii));
          }
        }
      }
      if (rank < K) {
        const float score = c.greedy ? -static_cast<float>(rank)
                                     : __fadd_rn(__fdiv_rn(xi, c.T), sh.noise[rank]);
        if (arg_better(score, rank, bs, br)) {
          bs = score;
          br = rank;
          bid = ii;
        }
      }
    }
    const int id = block_argmax<NT, E>(bs, br, bid, sh, rb);
    flags = c.greedy ? Q3S_ROW_GREEDY : 0;
    if (processed) {
#pragma unroll
      for (int j = 0; j < E; ++j)
        if ((vmask >> j) & 1u) processed[v0 + j] = ((dmask >> j) & 1u) ? __fdiv_rn(x[j], pen) : x[j];
    }
    return id;
  }

  if constexpr (MODE == Q3S_DRAW_ICDF) {
    // ---- icdf: HF top-k survivors among the candidates, top-p, draw --------
    // s = x'/T; an entry survives when fewer than k entries have a larger s
    for (int i = t; i < static_cast<int>(n); i += NT)
      sh.cand[i].x = __float_as_uint(__fdiv_rn(__uint_as_float(sh.cand[i].z), c.T));
    __syncthreads();
    for (int i = t; i < static_cast<int>(n); i += NT) {
      const float si = __uint_as_float(sh.cand[i].x);
      int above = 0;
      float m = -INFINITY;
      for (int o = 0; o < n4; o += 4) {
  #pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float so = __uint_as_float(sh.cand[o + u].x);
          above += so > si;
          m = fmaxf(m, so);
        }
      }
      const bool surv = above < K;
      sh.surv[i] = surv;
      sh.keep[i] = surv;
      sh.cand[i].w = __float_as_uint(surv ? softmax_weight(si, m) : 0.0f);
    }
    __syncthreads();
    if (c.top_p < 1.0f) {
      // HF TopPLogitsWarper over a stable ascending order (value asc, index
      // asc): remove a survivor when the softmax mass at-or-below it is <= 1-p;
      // the ascending-last survivor always stays.
      const float frac = __fsub_rn(1.0f, c.top_p);
      for (int i = t; i < static_cast<int>(n); i += NT) {
        if (!sh.surv[i]) continue;
        const uint4 me = sh.cand[i];
        const float si = __uint_as_float(me.x);
        const int ii = static_cast<int>(me.y);
        float cum = 0.0f, Z = 0.0f;
        int after = 0;
        for (int o = 0; o < n4; o += 4) {
  #pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint4 ot = sh.cand[o + u];
            const float so = __uint_as_float(ot.x);
            const float w = __uint_as_float(ot.w);
            const bool sv = o + u < static_cast<int>(n) && sh.surv[o + u];
            const bool before = (so < si) | ((so == si) & (static_cast<int>(ot.y) <= ii));
            cum = __fadd_rn(cum, (sv && before) ? w : 0.0f);
            Z = __fadd_rn(Z, sv ? w : 0.0f);
            after += sv && !before;
          }
        }
        const float thr_m = __fmul_rn(frac, Z);
        sh.keep[i] = (after == 0) || !(cum <= thr_m);
        if (after != 0 && fabsf(__fsub_rn(cum, thr_m)) < BOUNDARY_EPS * Z) atomicOr(&sh.flags, Q3S_ROW_TOPP_BOUNDARY);
      }
      __syncthreads();
    }
    if (t < 32) {
      // inverse CDF over the kept candidates (vocabulary order): lane l owns
      // positions [l*P, l*P + P) for P = ceil(n/32) <= 16
      const int lane = t;
      const int P = (static_cast<int>(n) + 31) / 32;
      float a = 0.0f;
      for (int r = 0; r < P; ++r) {
        const int i = lane * P + r;
        if (i < static_cast<int>(n) && sh.keep[i]) a = __fadd_rn(a, __uint_as_float(sh.cand[i].w));
      }
      float inc = a;
  #pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float nb = __shfl_up_sync(FULL, inc, o);
        if (lane >= o) inc = __fadd_rn(inc, nb);
      }
      float pre = __shfl_up_sync(FULL, inc, 1);
      if (lane == 0) pre = 0.0f;
      const float W = __shfl_sync(FULL, inc, 31);
      const float thr_u = __fmul_rn(c.u, W);
      int r_first = -1, r_last = -1;
      float acc = 0.0f;
      for (int r = 0; r < P; ++r) {
        const int i = lane * P + r;
        const float w = (i < static_cast<int>(n) && sh.keep[i]) ? __uint_as_float(sh.cand[i].w) : 0.0f;
        acc = __fadd_rn(acc, w);
        if (w > 0.0f) {
          r_last = r;
          if (r_first < 0 && __fadd_rn(pre, acc) > thr_u) r_first = r;
        }
      }
      const unsigned hit = __ballot_sync(FULL, r_first >= 0);
      int src, rsel;
      bool fallback = false;
      if (hit) {
        src = __ffs(hit) - 1;
        rsel = __shfl_sync(FULL, r_first, src);
      } else {
        const unsigned any = __ballot_sync(FULL, r_last >= 0);
        src = any ? 31 - __clz(any) : 0;
        rsel = any ? __shfl_sync(FULL, r_last, src) : 0;
        fallback = true;
      }
      if (lane == src) {
        float cdf = pre, prev = pre, a2 = 0.0f;
        for (int r = 0; r <= rsel; ++r) {
          const int i = lane * P + r;
          const float w = (i < static_cast<int>(n) && sh.keep[i]) ? __uint_as_float(sh.cand[i].w) : 0.0f;
          a2 = __fadd_rn(a2, w);
          if (r < rsel) prev = __fadd_rn(pre, a2);
          cdf = __fadd_rn(pre, a2);
        }
        int fl = fallback ? Q3S_ROW_FALLBACK : 0;
        const float tol = BOUNDARY_EPS * W;
        if ((__fsub_rn(cdf, thr_u) < tol) || (__fsub_rn(thr_u, prev) < tol)) fl |= Q3S_ROW_DRAW_BOUNDARY;
        if (fl) atomicOr(&sh.flags, fl);
        sh.sel_u[3] = sh.cand[lane * P + rsel].y;
      }
    }
    __syncthreads();
    const int id = static_cast<int>(sh.sel_u[3]);
    flags = sh.flags;
    if (processed) {
      uint32_t p2 = pos0;
  #pragma unroll
      for (int j = 0; j < E; ++j) {
        if (!((vmask >> j) & 1u)) continue;
        float out = -INFINITY;
        if ((cmask >> j) & 1u) {
          if (sh.keep[p2]) out = __uint_as_float(sh.cand[p2].x);
          ++p2;
        }
        processed[v0 + j] = out;
      }
    }
    return id;
  } else {
    return 0;  // not reached: gumbel rows return above
  }
}

}  // namespace q3s
