// q3s_cp.cuh -- code-predictor frame for the engine graph's stage sampler
// (CodePredictorUnrolled._select_token, scripts/export/utils.py:1178-1193,
// looped at :1218-1237) in Gumbel mode: one CTA of 256 threads per row runs
// all S stages, each a short fixed chain of five barriers.
//
// A frame is latency-bound (one row per SM at the engine's batch sizes), so
// a stage does only what exactly-K top-k + Gumbel needs, with thread t
// holding entries t, t + 256, ... of the row (read from a ring of bulk-copied
// stage rows, the producer's rotation applied on the read):
//   1. the row maximum (one integer reduction of order-preserving keys per
//      warp, one exchange);
//   2. one histogram of d = max - v in bins 1/8 wide over d < 32 (shared
//      atomics; floor((max - v) * 8) is monotone in v, so every entry at or
//      above the K-th largest lies in the bin holding it or an earlier one);
//      warp 0 finds that bin and turns the counts into exclusive prefixes;
//   3. those entries placed by bin (a counting sort: each takes its bin's
//      cursor, advanced atomically), so every bin is a contiguous range;
//   4. each candidate's exact rank (value desc, index asc) = its bin's start
//      plus its rank among the few entries of its own bin (bins are monotone
//      in the value and equal values share a bin), counted over one 64-bit
//      word per entry that orders like (value desc, index asc); the first K
//      score v / T + noise[rank] (v / T correctly rounded through the row's
//      reciprocal; the noise of this stage was fetched during the previous
//      one); the argmax (lowest rank on ties).
// Rows outside that pattern -- the K-th largest 32 or more below the maximum,
// more than 256 entries down to its bin (massive ties) -- take the general
// CTA sampler core on the row re-read in that core's layout (thread t holding
// entries [8t, 8t+8)).
#pragma once

#include "q3s_args.cuh"
#include "q3s_device.cuh"

namespace q3s {

constexpr int CPF_NT = 256;
constexpr int CPF_E = 8;
constexpr int CPF_CAP = 256;  // fast-path candidates (one per thread)

// MINB CTAs per SM: 1 leaves the stage all the registers it wants, 2 caps
// them (a few spilled) so that two rows share an SM.
template <bool BF16, int MINB>
__global__ void __launch_bounds__(CPF_NT, MINB) cp_fast_kernel(const CpArgs a) {
  constexpr int NT = CPF_NT, E = CPF_E, NW = NT / 32;
  __shared__ Scratch<NT, E> sh;
  __shared__ __align__(8) uint64_t bars[MAX_NBUF];
  __shared__ __align__(16) uint32_t wmax[NW];  // the warps' maxima as order-preserving keys
  __shared__ float wbs[NW];
  __shared__ int wbr[NW], wbi[NW];
  // candidate slot -> (f2key(value) << 32) | ~index: one word that orders
  // like (value desc, index asc) when compared as an integer
  __shared__ unsigned long long ckey[CPF_CAP];
  __shared__ int sel[2];
  extern __shared__ __align__(128) unsigned char cpf_ring[];
  const int t = static_cast<int>(threadIdx.x), w = t >> 5, lane = t & 31;
  const int v0 = t * E;
  const int V = a.V, S = a.S, K = a.K;
  const int esz = BF16 ? 2 : 4;
  const int nrows = (a.B - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                    static_cast<int>(gridDim.x);
  const int nitems = nrows * S;

  auto issue = [&](int g) {
    const int i = g / S, j = g % S;
    const int b = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
    const unsigned char* src = static_cast<const unsigned char*>(a.logits) +
                               (static_cast<int64_t>(j) * a.stage_stride + static_cast<int64_t>(b) * a.row_stride) * esz;
    const int slot = g % a.nbuf;
    mbar_expect_tx(&bars[slot], a.row_bytes);
    bulk_g2s(cpf_ring + static_cast<size_t>(slot) * a.row_bytes, src, a.row_bytes, &bars[slot]);
  };
  // noise of item g (row i, stage j) by rank into half (g & 1) of sh.noise
  // noise of item g (row i, stage j), entry t of its K, from global memory
  // (0 past the end): fetched into a register at a stage's start and stored
  // at its end, so the load's latency overlaps the stage instead of holding
  // the fetching warps (and with them the stage's first barrier)
  auto fetch_noise = [&](int g) -> float {
    if (g >= nitems || t >= K) return 0.0f;
    const int i = g / S, j = g % S;
    const int b = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
    return __ldg(a.noise + static_cast<int64_t>(b) * a.noise_row_stride + static_cast<int64_t>(j) * a.noise_stage_stride + t);
  };
  // ... into half (g & 1) of sh.noise (by rank)
  auto stash_noise = [&](int g, float nz) {
    if (g < nitems && t < K) sh.noise[(g & 1) * CPF_CAP + t] = nz;
  };

  clear_hist<NT, E>(sh);
  if (t == 0) {
    for (int s = 0; s < a.nbuf; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  stash_noise(0, fetch_noise(0));
  __syncthreads();
  if (t == 0)
    for (int g = 0; g < min(a.nbuf, nitems); ++g) issue(g);

  for (int i = 0; i < nrows; ++i) {
    const int b = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
    int64_t prev = (a.producer == Q3S_CP_ROTATE) ? __ldg(a.ids_init + b) : 0;
    const float T = a.temperature ? __ldg(a.temperature + b) : a.temperature_default;
    // v / T by the per-row reciprocal where that is the correctly rounded
    // quotient (normal operands: |v| in [2^-60, 2^60], T in [2^-20, 2^20]),
    // else by the division itself
    const bool t_ok = T >= 0x1p-20f && T <= 0x1p20f;
    const float rT = __frcp_rn(t_ok ? T : 1.0f);
    for (int j = 0; j < S; ++j) {
      const int g = i * S + j;
      const int shift = (a.producer == Q3S_CP_ROTATE) ? norm_shift(prev, V) : 0;
      const int slot = g % a.nbuf;
      // each thread waits for the row itself; whether any wait gave up is
      // agreed on at barrier (1), the first the stage takes (nothing before
      // it stores to shared memory but the warps' maxima)
      const bool ok = mbar_wait_bounded(&bars[slot], static_cast<uint32_t>((g / a.nbuf) & 1));
      // prefetch the next stage's noise (the previous stage's slot is
      // refilled below, off the critical path)
      const float nz_next = fetch_noise(g + 1);
      const unsigned char* row = cpf_ring + static_cast<size_t>(slot) * a.row_bytes;
      // entries v = t + NT e, e < E (the producer's rotation applied on the
      // read): a warp's loads are consecutive words, free of bank conflicts
      auto load_row = [&](float (&xr)[E], uint32_t& vm, int first, int step) {
        vm = 0;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int v = first + step * e;
          xr[e] = -INFINITY;
          if (v < V) {
            int q = v + shift;
            q -= q >= V ? V : 0;
            xr[e] = BF16 ? bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(row)[q])
                         : reinterpret_cast<const float*>(row)[q];
            vm |= 1u << e;
          }
        }
      };
      float x[E];
      uint32_t vmask;
      load_row(x, vmask, t, NT);

      // 1. the row maximum: the thread's (NaN dropped), then one integer
      //    reduction of order-preserving keys per warp (key 0, below every
      //    key, for a thread whose entries are all NaN)
      float tm = x[0];
#pragma unroll
      for (int e = 1; e < E; ++e) tm = fmaxf(tm, x[e]);
      const uint32_t wk_max = __reduce_max_sync(FULL, tm != tm ? 0u : f2key(tm));
      if (lane == 0) wmax[w] = wk_max;
      if (__syncthreads_or(!ok)) {  // (1) a wait gave up: report, wait (bounded) for copies in flight
        if (t == 0) {
          if (a.error_word) atomicOr(a.error_word, Q3S_DEVERR_WAIT_TIMEOUT);
          const int issued = g == 0 ? a.nbuf : a.nbuf - 1;
          for (int h = g; h < min(g + issued, nitems); ++h)
            (void)mbar_wait_bounded(&bars[h % a.nbuf], static_cast<uint32_t>((h / a.nbuf) & 1));
        }
        return;
      }
      float m;
      {
        static_assert(NW == 8, "two 16-byte reads of the warps' keys");
        const uint4 k0 = reinterpret_cast<const uint4*>(wmax)[0], k1 = reinterpret_cast<const uint4*>(wmax)[1];
        const uint32_t mk = max(max(max(k0.x, k0.y), max(k0.z, k0.w)), max(max(k1.x, k1.y), max(k1.z, k1.w)));
        m = key2f(mk);  // NaN when no warp had a number: every bin test fails, the row takes the core
      }
      // 2. histogram of floor((m - v) * 8) over d < 32 (each entry's bin
      //    kept; 256 = beyond)
      int eb[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float ev = __fmul_rn(__fsub_rn(m, x[e]), 8.0f);
        eb[e] = ev < 256.0f ? static_cast<int>(ev) : 256;
        if (eb[e] < 256) atomicAdd(&sh.hist[0][eb[e]], 1u);
      }
      __syncthreads();  // (2)
      // while warp 0 scans: refill the previous stage's slot
      if (t == 32 && g > 0 && g - 1 + a.nbuf < nitems) issue(g - 1 + a.nbuf);
      if (w == 0) {
        // the bin holding the K-th largest and the count through it; every
        // bin's count becomes its exclusive prefix (the placement cursor)
        uint4* hb = reinterpret_cast<uint4*>(sh.hist[0]) + 2 * lane;
        const uint4 h0 = hb[0], h1 = hb[1];
        const uint32_t c[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        uint32_t sum = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) sum += c[k];
        uint32_t inc = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(FULL, inc, o);
          if (lane >= o) inc += y;
        }
        uint32_t pre[8];
        uint32_t run = inc - sum;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          pre[k] = run;
          run += c[k];
        }
        hb[0] = make_uint4(pre[0], pre[1], pre[2], pre[3]);
        hb[1] = make_uint4(pre[4], pre[5], pre[6], pre[7]);
        const uint32_t kk = static_cast<uint32_t>(K);
        const unsigned hit = __ballot_sync(FULL, inc >= kk && inc - sum < kk);
        if (lane == 0) {
          sel[0] = 256;
          sel[1] = 0;
        }
        __syncwarp();
        if (hit && lane == __ffs(hit) - 1) {
          uint32_t acc = inc - sum;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            acc += c[k];
            if (acc >= kk) {
              sel[0] = 8 * lane + k;
              sel[1] = static_cast<int>(acc);
              break;
            }
          }
        }
      }
      __syncthreads();  // (3)
      const int bK = sel[0], n = sel[1];
      int id, flags = 0;
      if (bK >= 256 || n > CPF_CAP) {
        // outside the fast pattern: the general CTA core, on the row again in
        // its layout (thread t holds entries [E t, E t + E)), the histogram
        // (now cursors) back to zero first
        for (int i = t; i < NBINS; i += NT) sh.hist[0][i] = 0u;
        load_row(x, vmask, v0, 1);
        __syncthreads();
        RowCfg c;
        c.mode = Q3S_DRAW_GUMBEL;
        c.greedy = false;
        c.T = T;
        c.k = K;
        c.top_p = 1.0f;
        c.u = 0.0f;
        c.noise = a.noise + static_cast<int64_t>(b) * a.noise_row_stride + static_cast<int64_t>(j) * a.noise_stage_stride;
        uint32_t err = 0;
        id = sample_core<NT, E, Q3S_DRAW_GUMBEL>(x, vmask, 0u, 1.0f, V, c, sh, nullptr, flags, err);
        if (err && a.error_word) atomicOr(a.error_word, static_cast<int>(err));
        // every thread holds the same id; the owner (complete flags) writes it
        if (id >= v0 && id < v0 + E) {
          a.ids_out[static_cast<int64_t>(b) * S + j] = id;
          if (a.row_flags) a.row_flags[static_cast<int64_t>(b) * S + j] = flags;
        }
        prev = id;
        // the core loads its own noise into sh.noise[0, K): store the next
        // stage's once every thread is done with the core
        __syncthreads();
        stash_noise(g + 1, nz_next);
        continue;
      }
      // 3. the candidates (bins 0..bK) placed by bin (a counting sort: slot =
      //    the bin's cursor, advanced atomically), so each bin is a
      //    contiguous range of the list
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (eb[e] <= bK) {
          const uint32_t slot = atomicAdd(&sh.hist[0][eb[e]], 1u);
          sh.xs[slot] = x[e];
          ckey[slot] = (static_cast<unsigned long long>(f2key(x[e])) << 32) | ~static_cast<uint32_t>(t + NT * e);
        }
      __syncthreads();  // (4)
      // 4. exact rank (value desc, index asc): the bins are monotone in the
      //    value and equal values share a bin, so the rank is the bin's start
      //    plus the rank inside the bin; the first K score v / T +
      //    noise[rank]; the argmax (lowest rank on ties).  A bin's cursor now
      //    holds the next bin's start.
      float bs = -INFINITY;
      int br = 0x7fffffff, bi = 0;
      if (t < n) {
        const float vp = sh.xs[t];
        const unsigned long long me = ckey[t];
        // the bin again, by the same arithmetic as in 2.
        const uint32_t k = static_cast<uint32_t>(__fmul_rn(__fsub_rn(m, vp), 8.0f));
        const uint32_t start = k ? sh.hist[0][k - 1] : 0u, end = sh.hist[0][k];
        int r = static_cast<int>(start);
        for (uint32_t q = start; q < end; ++q) r += ckey[q] > me;
        if (r < K) {
          const float av = fabsf(vp);
          const float sc = t_ok && av >= 0x1p-60f && av <= 0x1p60f ? div_rn_row(vp, T, rT) : __fdiv_rn(vp, T);
          bs = __fadd_rn(sc, sh.noise[(g & 1) * CPF_CAP + r]);
          br = r;
          bi = static_cast<int>(~static_cast<uint32_t>(me));
        }
      }
      // argmax (score desc, rank asc) by two warp reductions: the largest
      // order-preserving score key, then the lowest rank among the lanes
      // holding it (ranks are distinct); lanes without a score hold key 0
      auto warp_best = [&](uint32_t key, uint32_t rank, int idv, uint32_t& bkey, uint32_t& brank, int& bid) {
        bkey = __reduce_max_sync(FULL, key);
        brank = __reduce_min_sync(FULL, key == bkey ? rank : 0xffffffffu);
        const unsigned hit = __ballot_sync(FULL, key == bkey && rank == brank);
        bid = __shfl_sync(FULL, idv, hit ? __ffs(hit) - 1 : 0);
      };
      uint32_t wk, wr;
      int wi;
      warp_best(br != 0x7fffffff ? f2key(bs) : 0u, static_cast<uint32_t>(br), bi, wk, wr, wi);
      if (lane == 0) {
        wbs[w] = __uint_as_float(wk);  // the key's bits
        wbr[w] = static_cast<int>(wr);
        wbi[w] = wi;
      }
      __syncthreads();  // (5)
      for (int i = t; i < NBINS; i += NT) sh.hist[0][i] = 0u;  // the zero invariant, for the next stage
      {
        // the same reduction over the warps' results (lanes 0..NW-1)
        const bool in = lane < NW;
        uint32_t fk, fr;
        warp_best(in ? __float_as_uint(wbs[lane]) : 0u, in ? static_cast<uint32_t>(wbr[lane]) : 0xffffffffu,
                  in ? wbi[lane] : 0, fk, fr, id);
      }
      if (t == 0) {
        a.ids_out[static_cast<int64_t>(b) * S + j] = id;
        if (a.row_flags) a.row_flags[static_cast<int64_t>(b) * S + j] = 0;
      }
      prev = id;
      stash_noise(g + 1, nz_next);  // half (g + 1) & 1: last read in the previous stage
    }
  }
}

}  // namespace q3s
