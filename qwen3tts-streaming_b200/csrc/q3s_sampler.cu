// q3s_sampler.cu -- sm_100a kernels and the C ABI of include/q3s_sampler.h.
//
// sample_rows_kernel   one CTA per row: load -> suppress / presence penalty /
//                      EOS gate -> (greedy | gumbel exactly-K | icdf top-k,
//                      top-p, inverse-CDF) -> id (+ count update).
// cp_frame_kernel      persistent: each CTA walks its rows through all S
//                      code-predictor stages; stage rows are prefetched into a
//                      shared-memory ring with cp.async.bulk + mbarrier, and
//                      stage j's logits are read through the producer map
//                      (rotation by stage j-1's id).
//
// Reference arithmetic followed (file:line in X-Square-Robot/Qwen3TTS-Streaming):
//   suppress/penalty/top-k/Gumbel/argmax/count update
//       scripts/export/talker_unified_modules.py:384-389, 407-422
//   code-predictor stage select   scripts/export/utils.py:1178-1193, 1218-1237
//   HF processor chain            tools/validation/prefill_compare.py:383-399
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "q3s_device.cuh"
#include "q3s_sampler.h"

namespace q3s {

// ---------------------------------------------------------------------------
// argument blocks passed by value to the kernels
// ---------------------------------------------------------------------------

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

constexpr int MAX_NBUF = 8;

// ---------------------------------------------------------------------------
// loads
// ---------------------------------------------------------------------------

// The 8 logits of vocabulary entries [v0, v0+8) of one row, fp32.  `shift`
// (in [0,V)) reads column v at (v + shift) mod V.  Entries >= V are -inf and
// cleared from `vmask`.
template <bool BF16>
Q3S_DEV void load_logits8(const void* base, int64_t row_off, int V, int v0, int shift,
                          bool vec, float (&x)[E], uint32_t& vmask) {
  vmask = 0;
  if (shift == 0 && vec && v0 + E <= V) {
    if (BF16) {
      const uint4 r = ld_stream16(static_cast<const uint16_t*>(base) + row_off + v0);
      const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        x[2 * i] = bf16_bits_to_f32(w[i] & 0xffffu);
        x[2 * i + 1] = bf16_bits_to_f32(w[i] >> 16);
      }
    } else {
      const float* p = static_cast<const float*>(base) + row_off + v0;
      const uint4 r0 = ld_stream16(p), r1 = ld_stream16(p + 4);
      x[0] = __uint_as_float(r0.x); x[1] = __uint_as_float(r0.y);
      x[2] = __uint_as_float(r0.z); x[3] = __uint_as_float(r0.w);
      x[4] = __uint_as_float(r1.x); x[5] = __uint_as_float(r1.y);
      x[6] = __uint_as_float(r1.z); x[7] = __uint_as_float(r1.w);
    }
    vmask = 0xffu;
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

// Samples one id from the processed logits x (post suppress/penalty/EOS gate).
// Every thread returns the same id and flags.  `processed` (optional) receives
// the row handed to the draw: g0 (gumbel), the filtered s (icdf), x (greedy).
template <int NT>
Q3S_DEV int sample_core(const float (&x)[E], uint32_t vmask, int V, const RowCfg& c,
                        Scratch<NT>& sh, float* processed, int& flags, uint32_t& err) {
  const int t = threadIdx.x;
  const int v0 = t * E;
  flags = 0;

  if (c.greedy) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (((vmask >> j) & 1u) && arg_better(x[j], v0 + j, bv, bi)) {
        bv = x[j];
        bi = v0 + j;
      }
    if (processed) {
#pragma unroll
      for (int j = 0; j < E; ++j)
        if ((vmask >> j) & 1u) processed[v0 + j] = x[j];
    }
    flags = Q3S_ROW_GREEDY;
    return block_argmax<NT>(bv, bi, bi, sh);
  }

  if (c.mode == Q3S_DRAW_GUMBEL) {
    // talker_unified_modules.py:415-420 / utils.py:1189-1193
    const int K = c.k;
    for (int r = t; r < K; r += NT) sh.cand_w[r] = __ldg(c.noise + r);
    uint32_t key[E];
#pragma unroll
    for (int j = 0; j < E; ++j) key[j] = f2key(x[j]);
    const uint32_t kth = select_kth_largest<NT>(key, vmask, K, sh);
    uint32_t cg = 0, ce = 0;
#pragma unroll
    for (int j = 0; j < E; ++j)
      if ((vmask >> j) & 1u) {
        cg += key[j] > kth;
        ce += key[j] == kth;
      }
    uint32_t tot;
    const uint32_t ex = block_excl_scan_u<NT>((cg << 16) | ce, tot, sh);
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
      if (slot >= 0) {
        sh.cand_k[slot] = key[j];
        sh.cand_v[slot] = x[j];
        sh.cand_i[slot] = v0 + j;
      }
    }
    __syncthreads();
    float bs = -INFINITY;
    int br = 0x7fffffff, bid = 0x7fffffff;
    for (int ci = t; ci < K; ci += NT) {
      const uint32_t kc = sh.cand_k[ci];
      const int ic = sh.cand_i[ci];
      int rank = 0;
      for (int o = 0; o < K; ++o) {
        const uint32_t ko = sh.cand_k[o];
        rank += (ko > kc) || (ko == kc && sh.cand_i[o] < ic);
      }
      const float score = __fadd_rn(__fdiv_rn(sh.cand_v[ci], c.T), sh.cand_w[rank]);
      if (arg_better(score, rank, bs, br)) {
        bs = score;
        br = rank;
        bid = ic;
      }
    }
    if (processed) {
#pragma unroll
      for (int j = 0; j < E; ++j)
        if ((vmask >> j) & 1u) processed[v0 + j] = x[j];
    }
    return block_argmax<NT>(bs, br, bid, sh);
  }

  // ---- icdf: Temperature -> TopK -> TopP -> softmax -> inverse CDF ----------
  float s[E];
  uint32_t key[E];
#pragma unroll
  for (int j = 0; j < E; ++j) {
    s[j] = ((vmask >> j) & 1u) ? __fdiv_rn(x[j], c.T) : -INFINITY;
    key[j] = f2key(s[j]);
  }
  uint32_t smask = vmask;
  if (c.k > 0 && c.k < V) {
    // HF TopKLogitsWarper: drop s < (k-th largest value); ties at it survive.
    const uint32_t kth = select_kth_largest<NT>(key, vmask, c.k, sh);
    smask = 0;
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (((vmask >> j) & 1u) && key[j] >= kth) smask |= 1u << j;
  }
  float lm = -INFINITY;
#pragma unroll
  for (int j = 0; j < E; ++j)
    if ((smask >> j) & 1u) lm = fmaxf(lm, s[j]);
  const float m = block_max_f<NT>(lm, sh);
  if (m == -INFINITY) {
    // nothing finite survived: report and fall back to the lowest index
    err |= Q3S_DEVERR_NO_MASS;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (((vmask >> j) & 1u) && arg_better(x[j], v0 + j, bv, bi)) {
        bv = x[j];
        bi = v0 + j;
      }
    flags = Q3S_ROW_FALLBACK;
    return block_argmax<NT>(bv, bi, bi, sh);
  }

  if (c.top_p < 1.0f) {
    // HF TopPLogitsWarper over a stable ascending order (value asc, index
    // asc): remove an entry when the softmax mass at-or-below it is <= 1-p;
    // the ascending-last entry always stays.
    const float frac = __fsub_rn(1.0f, c.top_p);
    uint32_t n;
    const uint32_t pos0 = block_excl_scan_u<NT>(__popc(smask), n, sh);
    bool near = false;
    if (n <= static_cast<uint32_t>(NT)) {
      uint32_t pos = pos0;
#pragma unroll
      for (int j = 0; j < E; ++j)
        if ((smask >> j) & 1u) {
          sh.cand_k[pos] = key[j];
          sh.cand_i[pos] = v0 + j;
          sh.cand_w[pos] = softmax_weight(s[j], m);
          ++pos;
        }
      __syncthreads();
      float wc = 0.0f, cum = 0.0f;
      int after = 0;
      if (t < static_cast<int>(n)) {
        const uint32_t kc = sh.cand_k[t];
        const int ic = sh.cand_i[t];
        wc = sh.cand_w[t];
        for (int o = 0; o < static_cast<int>(n); ++o) {
          const uint32_t ko = sh.cand_k[o];
          const int io = sh.cand_i[o];
          if (ko < kc || (ko == kc && io <= ic))
            cum = __fadd_rn(cum, sh.cand_w[o]);
          else
            ++after;
        }
      }
      const float Z = block_sum_f<NT>(wc, sh);
      const float thr = __fmul_rn(frac, Z);
      if (t < static_cast<int>(n)) {
        sh.cand_keep[t] = (after == 0) || !(cum <= thr);
        near = (after != 0) && fabsf(__fsub_rn(cum, thr)) < BOUNDARY_EPS * Z;
      }
      if (__syncthreads_or(near)) flags |= Q3S_ROW_TOPP_BOUNDARY;
      uint32_t nm = 0;
      pos = pos0;
#pragma unroll
      for (int j = 0; j < E; ++j)
        if ((smask >> j) & 1u) {
          if (sh.cand_keep[pos]) nm |= 1u << j;
          ++pos;
        }
      smask = nm;
      __syncthreads();  // cand_* reused by later phases
    } else {
      unsigned long long q[E], lq = 0;
#pragma unroll
      for (int j = 0; j < E; ++j) {
        q[j] = ((smask >> j) & 1u)
                   ? __float2ull_rn(__fmul_rn(softmax_weight(s[j], m), static_cast<float>(1ull << MASS_BITS)))
                   : 0ull;
        lq += q[j];
      }
      const unsigned long long Zq = block_sum_q<NT>(lq, sh);
      const unsigned long long tau = __double2ull_rd(static_cast<double>(frac) * static_cast<double>(Zq));
      if (tau >= Zq) {
        // everything but the ascending-last entry goes
        int last = -1;
#pragma unroll
        for (int j = 0; j < E; ++j)
          if (((smask >> j) & 1u) && s[j] == m) last = v0 + j;
        last = block_max_i<NT>(last, sh);
        smask = (last >= v0 && last < v0 + E) ? (1u << (last - v0)) : 0u;
      } else {
        uint32_t vstar;
        unsigned long long below;
        select_mass_cut<NT>(key, q, smask, tau, sh, vstar, below);
        uint32_t ce = 0;
        unsigned long long qstar = 1;
#pragma unroll
        for (int j = 0; j < E; ++j)
          if (((smask >> j) & 1u) && key[j] == vstar) {
            ++ce;
            qstar = q[j];
          }
        uint32_t cet;
        uint32_t tr = block_excl_scan_u<NT>(ce, cet, sh);
        qstar = qstar ? qstar : 1ull;
        const unsigned long long nrem = (tau - below) / qstar;  // ties removed (lowest index first)
        const unsigned long long eps = Zq / 1000000ull;
        uint32_t nm = 0;
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
        if (__syncthreads_or(near)) flags |= Q3S_ROW_TOPP_BOUNDARY;
        smask = nm;
      }
    }
  }

  // inverse CDF in vocabulary order over the surviving softmax weights
  float w[E], lc[E], lsum = 0.0f;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    w[j] = ((smask >> j) & 1u) ? softmax_weight(s[j], m) : 0.0f;
    lsum = __fadd_rn(lsum, w[j]);
    lc[j] = lsum;
  }
  float W;
  const float pre = block_excl_scan_f<NT>(lsum, W, sh);
  const float thr = __fmul_rn(c.u, W);
  int first = 0x7fffffff;
#pragma unroll
  for (int j = E - 1; j >= 0; --j)
    if (w[j] > 0.0f && __fadd_rn(pre, lc[j]) > thr) first = v0 + j;
  int id = block_min_i<NT>(first, sh);
  if (id == 0x7fffffff) {
    int last = -1;
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (w[j] > 0.0f) last = v0 + j;
    id = block_max_i<NT>(last, sh);
    flags |= Q3S_ROW_FALLBACK;
  }
  bool near = false;
  float prev = pre;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const float cdf = __fadd_rn(pre, lc[j]);
    if (v0 + j == id) {
      const float tol = BOUNDARY_EPS * W;
      near = (__fsub_rn(cdf, thr) < tol) || (__fsub_rn(thr, prev) < tol);
    }
    prev = cdf;
  }
  if (__syncthreads_or(near)) flags |= Q3S_ROW_DRAW_BOUNDARY;
  if (processed) {
#pragma unroll
    for (int j = 0; j < E; ++j)
      if ((vmask >> j) & 1u) processed[v0 + j] = ((smask >> j) & 1u) ? s[j] : -INFINITY;
  }
  return id;
}

// ---------------------------------------------------------------------------
// one sampling step, one CTA per row
// ---------------------------------------------------------------------------

template <int NT, bool BF16>
__global__ void __launch_bounds__(NT) sample_rows_kernel(const SampleArgs a) {
  __shared__ Scratch<NT> sh;
  const int b = blockIdx.x;
  const int t = threadIdx.x;
  const int v0 = t * E;
  const int V = a.V;
  uint32_t err = 0;

  // issue every independent load first
  const int shift = a.col_shift ? norm_shift(__ldg(a.col_shift + b), V) : 0;
  float x[E];
  uint32_t vmask;
  load_logits8<BF16>(a.logits, static_cast<int64_t>(b) * a.row_stride, V, v0, shift, a.vec_logits, x,
                     vmask);

  uint32_t app = 0;
  if (a.token_counts) {
    const int64_t* tc = a.token_counts + static_cast<int64_t>(b) * a.tc_stride + v0;
    if (a.vec_counts && v0 + E <= V) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 r = ld_stream16(tc + 2 * i);
        const int64_t c0 = static_cast<int64_t>((static_cast<uint64_t>(r.y) << 32) | r.x);
        const int64_t c1 = static_cast<int64_t>((static_cast<uint64_t>(r.w) << 32) | r.z);
        app |= (c0 > 0 ? 1u : 0u) << (2 * i);
        app |= (c1 > 0 ? 1u : 0u) << (2 * i + 1);
      }
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j)
        if (v0 + j < V && __ldg(tc + j) > 0) app |= 1u << j;
    }
  }
  uint32_t sup = 0;
  if (a.suppress) {
    if (a.vec_suppress && v0 + E <= V) {
      const uint2 m = __ldg(reinterpret_cast<const uint2*>(a.suppress + v0));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sup |= (((m.x >> (8 * j)) & 0xffu) ? 1u : 0u) << j;
        sup |= (((m.y >> (8 * j)) & 0xffu) ? 1u : 0u) << (j + 4);
      }
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j)
        if (v0 + j < V && __ldg(a.suppress + v0 + j)) sup |= 1u << j;
    }
  }
  const float T = a.temperature ? __ldg(a.temperature + b) : a.temperature_default;
  const float pen = a.penalty ? __ldg(a.penalty + b) : a.penalty_default;
  const float top_p = a.top_p ? __ldg(a.top_p + b) : a.top_p_default;
  const int kk = (a.mode == Q3S_DRAW_ICDF && a.top_k) ? __ldg(a.top_k + b) : a.K;
  const int min_new = a.min_new ? __ldg(a.min_new + b) : a.min_new_default;
  const float u = a.uniforms ? __ldg(a.uniforms + b) : 0.0f;

  int hist_len = 0;
  if (a.history) {
    int o0 = __ldg(a.offsets + b), o1 = __ldg(a.offsets + b + 1);
    if (o0 < 0 || o1 < o0 || static_cast<int64_t>(o1) > a.history_len) {
      err |= Q3S_DEVERR_OFFSETS;
      o0 = o1 = 0;
    }
    hist_len = o1 - o0;
    *reinterpret_cast<uint2*>(&sh.seen[v0]) = make_uint2(0u, 0u);
    __syncthreads();
    // presence scatter: racing stores of the same byte need no atomics
    for (int i = o0 + t; i < o1; i += 4 * NT) {
      int id[4];
      bool in[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        in[r] = i + r * NT < o1;
        id[r] = in[r] ? __ldg(a.history + i + r * NT) : 0;
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        if (!in[r]) continue;
        if (static_cast<unsigned>(id[r]) < static_cast<unsigned>(V))
          sh.seen[id[r]] = 1;
        else
          err |= Q3S_DEVERR_HISTORY_ID;
      }
    }
    __syncthreads();
    const uint2 f = *reinterpret_cast<const uint2*>(&sh.seen[v0]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      app |= (((f.x >> (8 * j)) & 0xffu) ? 1u : 0u) << j;
      app |= (((f.y >> (8 * j)) & 0xffu) ? 1u : 0u) << (j + 4);
    }
  }
  const int cur = a.cur_len ? __ldg(a.cur_len + b) : hist_len;
  const bool gate = a.eos_id >= 0 && a.eos_id < V && cur < min_new;

  // suppress (-1e9) -> presence penalty -> EOS gate
#pragma unroll
  for (int j = 0; j < E; ++j) {
    if (!((vmask >> j) & 1u)) continue;
    float v = x[j];
    if ((sup >> j) & 1u) v = NEG_SUPPRESS;
    if ((app >> j) & 1u) v = (v > 0.0f) ? __fdiv_rn(v, pen) : __fmul_rn(v, pen);
    if (gate && v0 + j == a.eos_id) v = -INFINITY;
    x[j] = v;
  }

  RowCfg c;
  c.mode = a.mode;
  c.greedy = (a.mode == Q3S_DRAW_ICDF) ? !(T > 0.0f) : (a.noise == nullptr);
  c.T = T;
  c.k = kk;
  c.top_p = top_p;
  c.u = u;
  c.noise = a.noise ? a.noise + static_cast<int64_t>(b) * a.noise_stride : nullptr;
  float* proc = a.processed ? a.processed + static_cast<int64_t>(b) * a.proc_stride : nullptr;
  int flags;
  const int id = sample_core<NT>(x, vmask, V, c, sh, proc, flags, err);

  const bool owner = id >= v0 && id < v0 + E;
  if (owner) {
    if (a.ids64) a.ids64[b] = id;
    if (a.ids32) a.ids32[b] = id;
    if (a.row_flags) a.row_flags[b] = flags;
  }
  if (a.counts_out) {
    int64_t* co = a.counts_out + static_cast<int64_t>(b) * a.co_stride;
    if (a.counts_out == a.token_counts && a.co_stride == a.tc_stride) {
      if (owner) co[id] += 1;  // in-place: the row was read before any write
    } else {
      const int64_t* tc = a.token_counts + static_cast<int64_t>(b) * a.tc_stride;
#pragma unroll
      for (int j = 0; j < E; ++j)
        if (v0 + j < V) co[v0 + j] = __ldg(tc + v0 + j) + (v0 + j == id ? 1 : 0);
    }
  }
  if (err && a.error_word) atomicOr(a.error_word, static_cast<int>(err));
}

// ---------------------------------------------------------------------------
// code-predictor frame: persistent, cp.async.bulk-prefetched stage rows
// ---------------------------------------------------------------------------

Q3S_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
Q3S_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
Q3S_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Plain (non-multicast) bulk copy global -> this CTA's shared memory.
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

template <int NT, bool BF16>
__global__ void __launch_bounds__(NT) cp_frame_kernel(const CpArgs a) {
  __shared__ Scratch<NT> sh;
  __shared__ __align__(8) uint64_t bars[MAX_NBUF];
  extern __shared__ __align__(128) unsigned char ring[];
  const int t = threadIdx.x;
  const int v0 = t * E;
  const int V = a.V, S = a.S;
  const int nrows = (a.B - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                    static_cast<int>(gridDim.x);
  const int nitems = nrows * S;
  const int esz = BF16 ? 2 : 4;

  auto issue = [&](int g) {
    const int i = g / S, j = g % S;
    const int b = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
    const unsigned char* src = static_cast<const unsigned char*>(a.logits) +
                               (static_cast<int64_t>(j) * a.stage_stride + static_cast<int64_t>(b) * a.row_stride) * esz;
    const int slot = g % a.nbuf;
    mbar_expect_tx(&bars[slot], a.row_bytes);
    bulk_g2s(ring + static_cast<size_t>(slot) * a.row_bytes, src, a.row_bytes, &bars[slot]);
  };

  if (a.bulk) {
    if (t == 0) {
      for (int s = 0; s < a.nbuf; ++s) mbar_init(&bars[s], 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (t == 0)
      for (int g = 0; g < min(a.nbuf, nitems); ++g) issue(g);
  }

  for (int i = 0; i < nrows; ++i) {
    const int b = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
    int64_t prev = (a.producer == Q3S_CP_ROTATE) ? __ldg(a.ids_init + b) : 0;
    const float T = a.temperature ? __ldg(a.temperature + b) : a.temperature_default;
    const float top_p = a.top_p ? __ldg(a.top_p + b) : a.top_p_default;
    for (int j = 0; j < S; ++j) {
      const int g = i * S + j;
      const int shift = (a.producer == Q3S_CP_ROTATE) ? norm_shift(prev, V) : 0;
      float x[E];
      uint32_t vmask = 0;
      if (a.bulk) {
        const int slot = g % a.nbuf;
        const bool ok = mbar_wait_bounded(&bars[slot], static_cast<uint32_t>((g / a.nbuf) & 1));
        if (__syncthreads_or(!ok)) {
          // give up: report, wait (bounded) for this CTA's copies still in
          // flight so none lands after exit, then leave
          if (t == 0) {
            if (a.error_word) atomicOr(a.error_word, Q3S_DEVERR_WAIT_TIMEOUT);
            for (int h = g; h < min(g + a.nbuf, nitems); ++h)
              (void)mbar_wait_bounded(&bars[h % a.nbuf], static_cast<uint32_t>((h / a.nbuf) & 1));
          }
          return;
        }
        const unsigned char* row = ring + static_cast<size_t>(slot) * a.row_bytes;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int v = v0 + e;
          x[e] = -INFINITY;
          if (v < V) {
            int q = v + shift;
            if (q >= V) q -= V;
            x[e] = BF16 ? bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(row)[q])
                        : reinterpret_cast<const float*>(row)[q];
            vmask |= 1u << e;
          }
        }
        __syncthreads();  // every thread has read the slot
        if (t == 0 && g + a.nbuf < nitems) issue(g + a.nbuf);
      } else {
        load_logits8<BF16>(a.logits, static_cast<int64_t>(j) * a.stage_stride + static_cast<int64_t>(b) * a.row_stride,
                           V, v0, shift, false, x, vmask);
      }
      RowCfg c;
      c.mode = a.mode;
      c.greedy = (a.mode == Q3S_DRAW_ICDF) ? !(T > 0.0f) : (a.noise == nullptr);
      c.T = T;
      c.k = a.K;
      c.top_p = top_p;
      c.u = a.uniforms ? __ldg(a.uniforms + static_cast<int64_t>(b) * S + j) : 0.0f;
      c.noise = a.noise ? a.noise + static_cast<int64_t>(b) * a.noise_row_stride + static_cast<int64_t>(j) * a.noise_stage_stride
                        : nullptr;
      int flags;
      uint32_t err = 0;
      const int id = sample_core<NT>(x, vmask, V, c, sh, nullptr, flags, err);
      if (t == 0) {
        a.ids_out[static_cast<int64_t>(b) * S + j] = id;
        if (a.row_flags) a.row_flags[static_cast<int64_t>(b) * S + j] = flags;
      }
      if (err && a.error_word) atomicOr(a.error_word, static_cast<int>(err));
      prev = id;
    }
  }
}

}  // namespace q3s

// ===========================================================================
// host side: validation, dispatch, C ABI
// ===========================================================================

namespace {

thread_local char g_last_error[512] = "";

q3s_status fail(q3s_status s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return s;
}

q3s_status ok() {
  g_last_error[0] = '\0';
  return Q3S_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int pick_threads(int V) {
  const int need = (V + q3s::E - 1) / q3s::E;
  static const int sizes[] = {64, 128, 256, 384, 512, 768, 1024};
  for (int s : sizes)
    if (s >= need) return s;
  return -1;
}

template <int NT>
q3s_status launch_rows(const q3s::SampleArgs& a, bool bf16, cudaStream_t st) {
  if (bf16)
    q3s::sample_rows_kernel<NT, true><<<a.B, NT, 0, st>>>(a);
  else
    q3s::sample_rows_kernel<NT, false><<<a.B, NT, 0, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_sample launch failed: %s", cudaGetErrorString(e));
  return ok();
}

int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

template <int NT, bool BF16>
q3s_status launch_cp_t(const q3s::CpArgs& a, cudaStream_t st) {
  const size_t dyn = a.bulk ? static_cast<size_t>(a.nbuf) * a.row_bytes : 0;
  auto kern = q3s::cp_frame_kernel<NT, BF16>;
  if (dyn > 0) {
    // static + dynamic shared memory may pass the 48 KB default: opt in.
    // Idempotent per (kernel, device); the value only ever grows.
    static int granted[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || granted[dev] < static_cast<int>(dyn)) {
      const cudaError_t e =
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn));
      if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_sample_cp_frame smem attribute: %s", cudaGetErrorString(e));
      if (dev >= 0 && dev < 64) granted[dev] = static_cast<int>(dyn);
    }
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NT, dyn) != cudaSuccess || per_sm <= 0) per_sm = 1;
  const int grid = std::min(a.B, device_sm_count() * per_sm);
  kern<<<grid, NT, dyn, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_sample_cp_frame launch failed: %s", cudaGetErrorString(e));
  return ok();
}

template <int NT>
q3s_status launch_cp(const q3s::CpArgs& a, bool bf16, cudaStream_t st) {
  return bf16 ? launch_cp_t<NT, true>(a, st) : launch_cp_t<NT, false>(a, st);
}

}  // namespace

extern "C" {

const char* q3s_last_error_string(void) { return g_last_error; }

int32_t q3s_abi_version(void) { return Q3S_ABI_VERSION; }

uint32_t q3s_desc_size(int32_t which) {
  if (which == 0) return static_cast<uint32_t>(sizeof(q3s_sample_desc));
  if (which == 1) return static_cast<uint32_t>(sizeof(q3s_cp_frame_desc));
  return 0;
}

q3s_status q3s_sample(const q3s_sample_desc* d, void* stream) {
  if (!d) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: desc is NULL");
  if (d->struct_size != sizeof(q3s_sample_desc))
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: struct_size %u != %u (ABI mismatch)", d->struct_size,
                static_cast<unsigned>(sizeof(q3s_sample_desc)));
  if (d->mode != Q3S_DRAW_GUMBEL && d->mode != Q3S_DRAW_ICDF)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: unknown mode %d", d->mode);
  if (d->logits_dtype != Q3S_DTYPE_F32 && d->logits_dtype != Q3S_DTYPE_BF16)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: unknown logits dtype %d", d->logits_dtype);
  if (d->batch < 0) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: batch %d < 0", d->batch);
  if (d->vocab < 1 || d->vocab > Q3S_MAX_VOCAB)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: vocab %d outside [1, %d]", d->vocab, Q3S_MAX_VOCAB);
  if (d->batch == 0) return ok();
  const int V = d->vocab;
  if (!d->logits) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: logits is NULL");
  if (d->logits_row_stride < V)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: logits_row_stride %lld < vocab %d",
                static_cast<long long>(d->logits_row_stride), V);
  if (!d->ids_i64 && !d->ids_i32) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: no ids output given");
  if (d->token_counts && d->history)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: give token_counts or history, not both");
  if (d->token_counts && d->token_counts_row_stride < V)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: token_counts_row_stride < vocab");
  if (d->history && (!d->offsets || d->history_len < 0))
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: packed history needs offsets and history_len >= 0");
  if (d->counts_out && !d->token_counts)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: counts_out needs token_counts");
  if (d->counts_out && d->counts_out_row_stride < V)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: counts_out_row_stride < vocab");
  if (d->processed_logits && d->processed_row_stride < V)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: processed_row_stride < vocab");
  if (!d->penalty && !(d->penalty_default > 0.0f))
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: penalty_default must be > 0");
  if (d->mode == Q3S_DRAW_GUMBEL) {
    const int kmax = std::min(V, Q3S_MAX_TOPK);
    if (d->gumbel_noise && (d->topk < 1 || d->topk > kmax))
      return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: gumbel topk %d outside [1, %d]", d->topk, kmax);
    if (d->gumbel_noise && d->gumbel_row_stride < d->topk)
      return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: gumbel_row_stride < topk");
  } else {
    const bool all_greedy = !d->temperature && !(d->temperature_default > 0.0f);
    if (!d->uniforms && !all_greedy)
      return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: icdf mode needs uniforms");
  }
  const int nt = pick_threads(V);
  if (nt < 0) return fail(Q3S_ERR_UNSUPPORTED, "q3s_sample: vocab %d too large", V);
  const bool bf16 = d->logits_dtype == Q3S_DTYPE_BF16;
  const int esz = bf16 ? 2 : 4;

  q3s::SampleArgs a;
  memset(&a, 0, sizeof(a));
  a.mode = d->mode;
  a.B = d->batch;
  a.V = V;
  a.K = (d->mode == Q3S_DRAW_GUMBEL) ? std::min(d->topk, V) : d->topk;
  a.row_stride = d->logits_row_stride;
  a.logits = d->logits;
  a.col_shift = d->col_shift;
  a.token_counts = d->token_counts;
  a.tc_stride = d->token_counts_row_stride;
  a.history = d->history;
  a.offsets = d->offsets;
  a.history_len = d->history_len;
  a.temperature = d->temperature;
  a.temperature_default = d->temperature_default;
  a.top_k = d->top_k;
  a.top_p = d->top_p;
  a.top_p_default = d->top_p_default;
  a.penalty = d->penalty;
  a.penalty_default = d->penalty_default;
  a.min_new = d->min_new_tokens;
  a.min_new_default = d->min_new_tokens_default;
  a.cur_len = d->cur_len;
  a.noise = (d->mode == Q3S_DRAW_GUMBEL) ? d->gumbel_noise : nullptr;
  a.noise_stride = d->gumbel_row_stride;
  a.uniforms = d->uniforms;
  a.suppress = d->suppress_mask;
  a.eos_id = d->eos_id;
  a.ids64 = d->ids_i64;
  a.ids32 = d->ids_i32;
  a.counts_out = d->counts_out;
  a.co_stride = d->counts_out_row_stride;
  a.processed = d->processed_logits;
  a.proc_stride = d->processed_row_stride;
  a.row_flags = d->row_flags;
  a.error_word = d->error_word;
  a.vec_logits = aligned16(d->logits) && ((d->logits_row_stride * esz) % 16 == 0);
  a.vec_counts = d->token_counts && aligned16(d->token_counts) && (d->token_counts_row_stride % 2 == 0);
  a.vec_suppress = d->suppress_mask && ((reinterpret_cast<uintptr_t>(d->suppress_mask) & 7u) == 0);

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (nt) {
    case 64: return launch_rows<64>(a, bf16, st);
    case 128: return launch_rows<128>(a, bf16, st);
    case 256: return launch_rows<256>(a, bf16, st);
    case 384: return launch_rows<384>(a, bf16, st);
    case 512: return launch_rows<512>(a, bf16, st);
    case 768: return launch_rows<768>(a, bf16, st);
    default: return launch_rows<1024>(a, bf16, st);
  }
}

q3s_status q3s_sample_cp_frame(const q3s_cp_frame_desc* d, void* stream) {
  if (!d) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: desc is NULL");
  if (d->struct_size != sizeof(q3s_cp_frame_desc))
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: struct_size %u != %u (ABI mismatch)",
                d->struct_size, static_cast<unsigned>(sizeof(q3s_cp_frame_desc)));
  if (d->mode != Q3S_DRAW_GUMBEL && d->mode != Q3S_DRAW_ICDF)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: unknown mode %d", d->mode);
  if (d->logits_dtype != Q3S_DTYPE_F32 && d->logits_dtype != Q3S_DTYPE_BF16)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: unknown logits dtype %d", d->logits_dtype);
  if (d->producer != Q3S_CP_DIRECT && d->producer != Q3S_CP_ROTATE)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: unknown producer %d", d->producer);
  if (d->batch < 0) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: batch < 0");
  if (d->vocab < 1 || d->vocab > Q3S_MAX_VOCAB)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: vocab %d outside [1, %d]", d->vocab, Q3S_MAX_VOCAB);
  if (d->stages < 1 || d->stages > Q3S_MAX_CP_STAGES)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: stages %d outside [1, %d]", d->stages,
                Q3S_MAX_CP_STAGES);
  if (d->batch == 0) return ok();
  const int V = d->vocab;
  if (!d->logits || !d->ids_out) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: logits/ids_out NULL");
  if (d->logits_row_stride < V) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: row stride < vocab");
  if (d->stages > 1 && d->logits_stage_stride < static_cast<int64_t>(d->batch - 1) * d->logits_row_stride + V)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: stage stride overlaps rows");
  if (d->producer == Q3S_CP_ROTATE && !d->ids_init)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: ROTATE needs ids_init");
  if (d->mode == Q3S_DRAW_GUMBEL) {
    const int kmax = std::min(V, Q3S_MAX_TOPK);
    if (d->gumbel_noise && (d->topk < 1 || d->topk > kmax))
      return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: topk %d outside [1, %d]", d->topk, kmax);
    if (d->gumbel_noise && (d->gumbel_row_stride < static_cast<int64_t>(d->stages - 1) * d->gumbel_stage_stride + d->topk ||
                            d->gumbel_stage_stride < d->topk))
      return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: gumbel strides too small");
  } else {
    const bool all_greedy = !d->temperature && !(d->temperature_default > 0.0f);
    if (!d->uniforms && !all_greedy)
      return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample_cp_frame: icdf mode needs uniforms");
  }
  const int nt = pick_threads(V);
  if (nt < 0) return fail(Q3S_ERR_UNSUPPORTED, "q3s_sample_cp_frame: vocab %d too large", V);
  const bool bf16 = d->logits_dtype == Q3S_DTYPE_BF16;
  const int esz = bf16 ? 2 : 4;

  q3s::CpArgs a;
  memset(&a, 0, sizeof(a));
  a.mode = d->mode;
  a.B = d->batch;
  a.V = V;
  a.S = d->stages;
  a.K = (d->mode == Q3S_DRAW_GUMBEL) ? std::min(d->topk, V) : d->topk;
  a.producer = d->producer;
  a.logits = d->logits;
  a.row_stride = d->logits_row_stride;
  a.stage_stride = d->logits_stage_stride;
  a.ids_init = d->ids_init;
  a.temperature = d->temperature;
  a.temperature_default = d->temperature_default;
  a.top_p = d->top_p;
  a.top_p_default = d->top_p_default;
  a.noise = (d->mode == Q3S_DRAW_GUMBEL) ? d->gumbel_noise : nullptr;
  a.noise_row_stride = d->gumbel_row_stride;
  a.noise_stage_stride = d->gumbel_stage_stride;
  a.uniforms = d->uniforms;
  a.ids_out = d->ids_out;
  a.row_flags = d->row_flags;
  a.error_word = d->error_word;
  a.row_bytes = static_cast<uint32_t>(V * esz);
  a.bulk = aligned16(d->logits) && (a.row_bytes % 16 == 0) && ((d->logits_row_stride * esz) % 16 == 0) &&
           ((d->logits_stage_stride * esz) % 16 == 0);
  // ring of stage rows in flight: ~16 KB (4 x 4 KB rows at V=2048 bf16), 2..8 slots
  a.nbuf = a.bulk ? std::max(2, std::min(q3s::MAX_NBUF, static_cast<int>((16u * 1024u) / a.row_bytes))) : 0;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (nt) {
    case 64: return launch_cp<64>(a, bf16, st);
    case 128: return launch_cp<128>(a, bf16, st);
    case 256: return launch_cp<256>(a, bf16, st);
    case 384: return launch_cp<384>(a, bf16, st);
    case 512: return launch_cp<512>(a, bf16, st);
    case 768: return launch_cp<768>(a, bf16, st);
    default: return launch_cp<1024>(a, bf16, st);
  }
}

}  // extern "C"
