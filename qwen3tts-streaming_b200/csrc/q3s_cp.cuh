// q3s_cp.cuh -- code-predictor frame, one warp per row: all S stages of the
// engine graph's stage sampler (CodePredictorUnrolled._select_token,
// scripts/export/utils.py:1178-1193, looped at :1218-1237) for one row, with
// no block-wide barrier at all -- a stage is a short chain of warp-synchronous
// steps, which is what bounds a frame at one row per SM.
//
// Per stage (V <= 2048 entries, NP = V / 32 per lane, lane l holding entries
// l + 32 i in registers, read from a ring of bulk-copied stage rows with the
// producer's rotation applied on the read):
//   greedy (no noise): torch.argmax of the row (lowest index on ties);
//   Gumbel: exactly-K top-k ordered (value desc, index asc), scores
//   v / T + noise[rank], argmax (lowest rank on ties):
//     1. the row maximum (warp shuffles);
//     2. one histogram of d = max - v in bins 1/8 wide over d < 32 (shared
//        atomics); a warp scan finds the bin holding the K-th largest --
//        every entry at or above it falls in that bin or an earlier one
//        (floor((max - v) * 8) is monotone in v);
//     3. those entries compacted in index order by ballots (at most 256;
//        otherwise, or when the K-th lies 32 or more below the maximum, an
//        exact bitwise select of the K-th key and the first ties by index);
//     4. each candidate's exact descending rank by all pairs (the list is in
//        index order, so earlier position = lower index breaks ties);
//     5. the K ranked candidates' scores, the warp argmax.
// The noise of the next stage is loaded while the current one computes.
#pragma once

#include "q3s_args.cuh"
#include "q3s_device.cuh"

namespace q3s {

constexpr int CPW_CAP = 256;  // candidate list

// Index of the first entry with the larger value (torch.argmax order).
Q3S_DEV void warp_argmax_vi(float& v, int& i) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(FULL, v, o);
    const int oi = __shfl_xor_sync(FULL, i, o);
    if (arg_better(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
}

template <int NP, bool BF16>
__global__ void __launch_bounds__(32) cp_warp_kernel(const CpArgs a) {
  extern __shared__ __align__(128) unsigned char cpw_ring[];
  __shared__ __align__(16) uint32_t hist[256];
  __shared__ float cval[CPW_CAP];
  __shared__ int cidx[CPW_CAP];
  __shared__ __align__(8) uint64_t bars[MAX_NBUF];
  const int lane = static_cast<int>(threadIdx.x);
  const int b = static_cast<int>(blockIdx.x);
  const int V = a.V, S = a.S, K = a.K;
  const int esz = BF16 ? 2 : 4;
  const bool greedy = a.noise == nullptr;
  const uint32_t lt = (1u << lane) - 1u;

  auto issue = [&](int j) {
    const int slot = j % a.nbuf;
    const unsigned char* src = static_cast<const unsigned char*>(a.logits) +
                               (static_cast<int64_t>(j) * a.stage_stride + static_cast<int64_t>(b) * a.row_stride) * esz;
    mbar_expect_tx(&bars[slot], a.row_bytes);
    bulk_g2s(cpw_ring + static_cast<size_t>(slot) * a.row_bytes, src, a.row_bytes, &bars[slot]);
  };
  if (lane == 0) {
    for (int s = 0; s < a.nbuf; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    for (int j = 0; j < min(a.nbuf, S); ++j) issue(j);
  }
  __syncwarp();

  int64_t prev = (a.producer == Q3S_CP_ROTATE) ? __ldg(a.ids_init + b) : 0;
  const float T = a.temperature ? __ldg(a.temperature + b) : a.temperature_default;
  constexpr int KP = CPW_CAP / 32;  // noise values per lane (K <= CPW_CAP)
  float gz[KP];
  auto load_noise = [&](int j) {
#pragma unroll
    for (int q = 0; q < KP; ++q) {
      const int r = lane + 32 * q;
      gz[q] = (!greedy && r < K) ? __ldg(a.noise + static_cast<int64_t>(b) * a.noise_row_stride +
                                         static_cast<int64_t>(j) * a.noise_stage_stride + r)
                                 : 0.0f;
    }
  };
  if (!greedy) load_noise(0);

  for (int j = 0; j < S; ++j) {
    const int slot = j % a.nbuf;
    const int shift = (a.producer == Q3S_CP_ROTATE) ? norm_shift(prev, V) : 0;
    if (!__all_sync(FULL, mbar_wait_bounded(&bars[slot], static_cast<uint32_t>((j / a.nbuf) & 1)))) {
      // give up: report, wait (bounded) for the copies still in flight, leave
      if (lane == 0) {
        if (a.error_word) atomicOr(a.error_word, Q3S_DEVERR_WAIT_TIMEOUT);
        for (int h = j; h < min(j + a.nbuf, S); ++h)
          (void)mbar_wait_bounded(&bars[h % a.nbuf], static_cast<uint32_t>((h / a.nbuf) & 1));
      }
      return;
    }
    const unsigned char* row = cpw_ring + static_cast<size_t>(slot) * a.row_bytes;
    float x[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const int v = lane + 32 * i;
      int q = v + shift;
      q -= q >= V ? V : 0;
      x[i] = v < V ? (BF16 ? bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(row)[q])
                           : reinterpret_cast<const float*>(row)[q])
                   : -INFINITY;
    }
    __syncwarp();
    if (lane == 0 && j + a.nbuf < S) issue(j + a.nbuf);  // every lane has read the slot

    int id = 0, flags = 0;
    float gcur[KP];
#pragma unroll
    for (int q = 0; q < KP; ++q) gcur[q] = gz[q];
    if (!greedy && j + 1 < S) load_noise(j + 1);  // in flight while this stage computes
    if (greedy) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        const int v = lane + 32 * i;
        if (v < V && arg_better(x[i], v, bv, bi)) {
          bv = x[i];
          bi = v;
        }
      }
      warp_argmax_vi(bv, bi);
      id = bi;
      flags = Q3S_ROW_GREEDY;
    } else {
      float m = x[0];
#pragma unroll
      for (int i = 1; i < NP; ++i) m = fmaxf(m, x[i]);
      m = warp_max_f(m);
      // histogram of floor((m - v) * 8) over d < 32
      reinterpret_cast<uint4*>(hist)[2 * lane] = make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(hist)[2 * lane + 1] = make_uint4(0, 0, 0, 0);
      __syncwarp();
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        const float e = __fmul_rn(__fsub_rn(m, x[i]), 8.0f);
        if (e < 256.0f) atomicAdd(&hist[static_cast<uint32_t>(e)], 1u);
      }
      __syncwarp();
      // the bin of the K-th largest: bins ascending in d = descending values
      const uint4 h0 = reinterpret_cast<const uint4*>(hist)[2 * lane];
      const uint4 h1 = reinterpret_cast<const uint4*>(hist)[2 * lane + 1];
      const uint32_t c[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
      uint32_t sum = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) sum += c[i];
      uint32_t inc = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(FULL, inc, o);
        if (lane >= o) inc += y;
      }
      const uint32_t kk = static_cast<uint32_t>(K);
      const unsigned hitb = __ballot_sync(FULL, inc >= kk && inc - sum < kk);
      int bK = 256;
      uint32_t cnt = 0;
      if (hitb) {
        const int src = __ffs(hitb) - 1;
        int mb = 0;
        uint32_t mc = 0;
        if (lane == src) {
          uint32_t acc = inc - sum;
          bool found = false;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            acc += c[i];
            if (!found && acc >= kk) {
              found = true;
              mb = 8 * lane + i;
              mc = acc;
            }
          }
        }
        bK = __shfl_sync(FULL, mb, src);
        cnt = __shfl_sync(FULL, mc, src);
      }
      int n = 0;
      if (bK < 256 && cnt <= static_cast<uint32_t>(CPW_CAP)) {
        // candidates: every entry in bins 0..bK, in index order
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          const float e = __fmul_rn(__fsub_rn(m, x[i]), 8.0f);
          const bool cnd = lane + 32 * i < V && e < static_cast<float>(bK + 1);
          const unsigned bal = __ballot_sync(FULL, cnd);
          if (cnd) {
            const int p = n + __popc(bal & lt);
            cval[p] = x[i];
            cidx[p] = lane + 32 * i;
          }
          n += __popc(bal);
        }
      } else {
        // exact: the K-th largest key bit by bit, then the entries above it
        // and the first ties by index (exactly K of them)
        uint32_t key[NP];
#pragma unroll
        for (int i = 0; i < NP; ++i) key[i] = lane + 32 * i < V ? f2key(x[i]) : 0u;
        uint32_t prefix = 0;
#pragma unroll 1
        for (int bit = 31; bit >= 0; --bit) {
          const uint32_t want = prefix | (1u << bit);
          uint32_t ge = 0;
#pragma unroll
          for (int i = 0; i < NP; ++i) ge += key[i] >= want;
#pragma unroll
          for (int o = 16; o; o >>= 1) ge += __shfl_xor_sync(FULL, ge, o);
          if (ge >= kk) prefix = want;  // the K-th largest key is >= want
        }
        uint32_t above = 0;
#pragma unroll
        for (int i = 0; i < NP; ++i) above += key[i] > prefix;
#pragma unroll
        for (int o = 16; o; o >>= 1) above += __shfl_xor_sync(FULL, above, o);
        int ties = 0;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          const bool over = key[i] > prefix, tie = lane + 32 * i < V && key[i] == prefix;
          const unsigned bt = __ballot_sync(FULL, tie);
          const bool take = over || (tie && ties + __popc(bt & lt) < K - static_cast<int>(above));
          const unsigned bal = __ballot_sync(FULL, take);
          if (take) {
            const int p = n + __popc(bal & lt);
            cval[p] = x[i];
            cidx[p] = lane + 32 * i;
          }
          n += __popc(bal);
          ties += __popc(bt);
        }
      }
      __syncwarp();
      // exact descending ranks by all pairs; scores of the first K; argmax
      float bs = -INFINITY;
      int br = 0x7fffffff, bidx = 0;
      for (int pb = 0; pb < n; pb += 32) {
        const int p = pb + lane;
        const bool act = p < n;
        const float vp = act ? cval[p] : 0.0f;
        int r = 0;
        if (act)
          for (int q = 0; q < n; ++q) {
            const float vq = cval[q];
            r += (vq > vp) || (vq == vp && q < p);
          }
        float g = 0.0f;
#pragma unroll
        for (int q = 0; q < KP; ++q) {
          const float gv = __shfl_sync(FULL, gcur[q], r & 31);
          if (q == (r >> 5)) g = gv;
        }
        if (act && r < K) {
          const float s = __fadd_rn(__fdiv_rn(vp, T), g);
          if (s > bs || (s == bs && r < br)) {
            bs = s;
            br = r;
            bidx = cidx[p];
          }
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float os = __shfl_xor_sync(FULL, bs, o);
        const int orr = __shfl_xor_sync(FULL, br, o), oi = __shfl_xor_sync(FULL, bidx, o);
        if (os > bs || (os == bs && orr < br)) {
          bs = os;
          br = orr;
          bidx = oi;
        }
      }
      id = bidx;
      __syncwarp();  // the candidate list and histogram are reused next stage
    }
    if (lane == 0) {
      a.ids_out[static_cast<int64_t>(b) * S + j] = id;
      if (a.row_flags) a.row_flags[static_cast<int64_t>(b) * S + j] = flags;
    }
    prev = id;
  }
}

}  // namespace q3s
