// q3s_lean.cuh -- register-resident row sampler for large batches (icdf mode).
//
// One CTA of NT threads per row; thread t holds vocabulary entries
// [t E, t E + E) in registers for the whole step, so every pass over the row
// is register arithmetic (no shared-memory row traffic) and a thread's
// entries are contiguous in vocabulary order (one sequential sum per thread,
// one block scan, for the inverse CDF).
//
// The per-entry work is kept to a few instructions by working on approximate
// processed values and recovering exactness on a short list:
//
//   pass 1   suppress (-1e9), repetition penalty as x * RN(1/pen) for present
//            entries > 0 (within 2 ulps of x / pen; x * pen and untouched
//            entries are exact), row maximum (NaN-propagating);
//   few-survivor rows (top-k, greedy):
//   pass 2   histogram of the distance to the maximum in bins 1/8 wide (a
//            float add on 2^23 makes the bin an integer without F2I);
//   pass 3   candidates: every entry down to one bin below the bin of the
//            K-th largest; with |values| <= 2000 the approximation error
//            and any temperature-quotient merge are < 2^-9, far inside a
//            bin, so the set holds every entry HF TopK keeps;
//   list     exact x' and s = x'/T per candidate (IEEE division), a counting
//            sort by exact bins plus ranks inside each bin (s desc, index
//            desc), TopK with ties kept, TopP on exact fixed-point masses in
//            ascending order, inverse CDF over the kept list in vocabulary
//            order;
//   whole-vocabulary rows (top-k off, top-p < 1):
//   pass 2   softmax weights; a count histogram by the weight's exponent and
//            top 4 mantissa bits (16 bins per octave) locates the top-p cut
//            to within a bin from count x midpoint-weight estimates;
//   pass 3   entries below a 5-bin bracket around that bin are removed (their
//            mass summed), bracket entries form the list;
//   list     exact s per list entry, the same counting sort, the exact cut
//            (HF TopP: ascending (s, index), cumulative mass <= (1-p) Z goes),
//            verified against the bracket (a wrong bracket takes the exact
//            path); then the inverse CDF over the whole row.
//
// Rows the fast paths cannot decide exactly (values beyond |2000|, NaN or
// infinite maxima, candidate lists over LCAP, a top-p cut outside the
// bracket, K > KMAX, extreme penalties or temperatures) re-run on the exact
// register-resident core (sample_core), so every row has one result
// whatever its values.
//
// The arithmetic follows the reference's processor chain
// (tools/validation/prefill_compare.py:383-399: RepetitionPenalty ->
// Temperature -> TopK -> TopP -> softmax -> draw, with the suppress mask of
// scripts/export/talker_unified_modules.py:384-389,409 and HF
// MinNewTokensLengthLogitsProcessor's EOS gate).
#pragma once

#include <type_traits>

#include "q3s_core.cuh"

namespace q3s {
namespace lean {

constexpr int LCAP = 256;              // list capacity (records in Scratch::cand)
constexpr int KMAX = 128;              // largest top-k the candidate path takes
constexpr uint32_t F23 = 0x4B000000u;  // bits of 2^23
constexpr float LOG2E = 1.4426950408889634f;

// List positions a thread takes (positions t PP .. t PP + PP - 1).
__host__ __device__ constexpr int pp(int NT) { return (LCAP + NT - 1) / NT; }

// Resident CTAs per SM each variant is compiled for (64 registers a thread).
__host__ __device__ constexpr int min_blocks(int NT) { return NT <= 128 ? 8 : 4; }

// max with NaN propagation (PTX max.NaN): a NaN anywhere makes the row max
// NaN, which sends the row to the exact path.
Q3S_DEV float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// 2^x (PTX ex2.approx, subnormal results flushed to zero).
Q3S_DEV float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Byte i (0..7) of an 8-byte word is nonzero.
Q3S_DEV bool byte_set(const uint2& w, int i) { return ((i < 4 ? w.x : w.y) & (0xffu << (8 * (i & 3)))) != 0u; }

// div_rn_row on the two lanes of packed fp32x2 arithmetic (the same roundings).
Q3S_DEV float2 div2_rn_row(float2 x, float d, float r) {
  const float2 dd = make_float2(-d, -d), rr = make_float2(r, r);
  const float2 q0 = __fmul2_rn(x, rr);
  const float2 q1 = __ffma2_rn(__ffma2_rn(q0, dd, x), rr, q0);
  return __ffma2_rn(__ffma2_rn(q1, dd, x), rr, q1);
}

// Integer bin of a value below a reference: RN(c0 - c v) - 2^23 as the
// float's bits, clamped to 255, with c0 = RN(c ref + 2^23 + 1).  One fused
// multiply-add rounds once, so the bin is a monotone non-increasing function
// of v (a float's bits order like its value), and v <= ref gives a result
// >= 2^23, i.e. a bin >= 0.  Needs |c ref| <= 2^21.
Q3S_DEV uint32_t ref_bin(float v, float c, float c0) {
  return min(__float_as_uint(__fmaf_rn(v, -c, c0)) - F23, 255u);
}
Q3S_DEV float ref_c0(float c, float ref) { return __fadd_rn(__fmul_rn(c, ref), 8388609.0f); }

// Bin of a softmax weight w in [0, 1 + 2^-23]: 16 bins per octave by the exponent and
// the top 4 mantissa bits (bin 0: w in [1, 1 + 1/16)), 255 for w < 2^-15.9
// and w = 0.  Monotone non-increasing in w.
Q3S_DEV uint32_t wbin(float w) { return min(2032u - (__float_as_uint(w) >> 19), 255u); }
// The midpoint weight of a wbin bin (an estimate of each entry's weight).
Q3S_DEV float wbin_mid(uint32_t k) { return __uint_as_float(((2032u - k) << 19) | (1u << 18)); }

// Warp-wide exclusive prefix over 256 bins held 8 per lane (bins 8l..8l+7):
// returns the prefix before each of the lane's bins in pre[], the total.
Q3S_DEV uint32_t warp_bins_prefix(const uint32_t* hist, uint32_t (&c)[8], uint32_t (&pre)[8]) {
  const int lane = threadIdx.x & 31;
  const uint4 a = reinterpret_cast<const uint4*>(hist)[2 * lane], b = reinterpret_cast<const uint4*>(hist)[2 * lane + 1];
  c[0] = a.x; c[1] = a.y; c[2] = a.z; c[3] = a.w; c[4] = b.x; c[5] = b.y; c[6] = b.z; c[7] = b.w;
  uint32_t s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += c[i];
  uint32_t inc = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc += n;
  }
  uint32_t run = inc - s;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    pre[i] = run;
    run += c[i];
  }
  return __shfl_sync(FULL, inc, 31);
}

// The first bin (ascending) whose inclusive prefix reaches k (k >= 1), and
// the prefix after the next bin (the count down to one bin further); 256 when
// the bins hold fewer than k.
Q3S_DEV void warp_bin_of_rank(const uint32_t* hist, uint32_t k, uint32_t& bin, uint32_t& through_next) {
  uint32_t c[8], pre[8];
  const uint32_t total = warp_bins_prefix(hist, c, pre);
  const int lane = threadIdx.x & 31;
  uint32_t mine = 256u, nxt = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (mine == 256u && pre[i] + c[i] >= k) {
      mine = static_cast<uint32_t>(8 * lane + i);
      nxt = pre[i] + c[i] + (i < 7 ? c[i + 1] : 0u);
    }
  const unsigned hit = __ballot_sync(FULL, mine != 256u);
  if (!hit || total < k) {
    bin = 256u;
    through_next = total;
    return;
  }
  const int src = __ffs(hit) - 1;
  bin = __shfl_sync(FULL, mine, src);
  // when the next bin starts on the following lane, add its count there
  const uint32_t c0n = __shfl_sync(FULL, c[0], (src + 1) & 31);
  through_next = __shfl_sync(FULL, nxt, src) + ((bin & 7u) == 7u && bin < 255u ? c0n : 0u);
}


// ---------------------------------------------------------------------------
// the list: records sh.cand[p] = {s bits, vocabulary index, weight bits, bin}
// in vocabulary order (p < n <= LCAP); sorted positions by (s desc, index
// desc) in sh.xs (sorted position -> p) and sh.noise (p -> sorted position)
// ---------------------------------------------------------------------------

template <int NT, int E>
Q3S_DEV uint32_t* list_inv(Scratch<NT, E>& sh) { return reinterpret_cast<uint32_t*>(sh.xs); }
template <int NT, int E>
Q3S_DEV uint32_t* list_pos(Scratch<NT, E>& sh) { return reinterpret_cast<uint32_t*>(sh.noise); }

// (s, index) of q comes before p in descending order
Q3S_DEV bool desc_before(const uint4& q, float sp, uint32_t ip) {
  const float sq = __uint_as_float(q.x);
  return sq > sp || (sq == sp && q.y > ip);
}

// Counting sort of the list by its bins (ascending bin = descending s; the
// bin is a monotone function of s, so bins never disagree with the order),
// then ranks inside each bin.  Entry: every record's bin is set and counted
// in sh.hist[0] (visible: a barrier after the counting).  Exit (after a
// barrier): the sorted positions; sh.hist[0] zero, sh.hist[1] garbage.
template <int NT, int E>
Q3S_DEV void list_sort_desc(Scratch<NT, E>& sh, int n) {
  const int t = threadIdx.x;
  uint32_t* inv = list_inv(sh);
  uint32_t* pos = list_pos(sh);
  uint32_t* tmp = reinterpret_cast<uint32_t*>(sh.keep);  // LCAP 16-bit slots fit in keep + surv
  uint16_t* slot16 = reinterpret_cast<uint16_t*>(tmp);
  if (t < 32) {
    uint32_t c[8], pre[8];
    (void)warp_bins_prefix(sh.hist[0], c, pre);
    uint4* h1 = reinterpret_cast<uint4*>(sh.hist[1]) + 2 * t;
    h1[0] = make_uint4(pre[0], pre[1], pre[2], pre[3]);
    h1[1] = make_uint4(pre[4], pre[5], pre[6], pre[7]);
    uint4* h0 = reinterpret_cast<uint4*>(sh.hist[0]) + 2 * t;
    h0[0] = make_uint4(0u, 0u, 0u, 0u);
    h0[1] = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
  for (int p = t; p < n; p += NT) {
    const uint32_t k = sh.cand[p].w;
    slot16[atomicAdd(&sh.hist[1][k], 1u)] = static_cast<uint16_t>(p);
  }
  __syncthreads();
  for (int p = t; p < n; p += NT) {
    const uint4 me = sh.cand[p];
    const uint32_t k = me.w;
    const uint32_t start = k ? sh.hist[1][k - 1] : 0u, end = sh.hist[1][k];
    const float sp = __uint_as_float(me.x);
    uint32_t r = 0;
    for (uint32_t i = start; i < end; ++i) r += desc_before(sh.cand[slot16[i]], sp, me.y);
    inv[start + r] = static_cast<uint32_t>(p);
    pos[p] = start + r;
  }
  __syncthreads();
}

// Block suffix sums of fixed-point masses over sorted positions [0, n):
// thread t takes positions t PP .. t PP + PP - 1 (PP = ceil(LCAP / NT)); returns in
// suf[i] the sum over positions >= its position, and the total.  One barrier.
template <int NT, int E>
Q3S_DEV void block_suffix_q(const unsigned long long (&q)[pp(NT)], unsigned long long (&suf)[pp(NT)],
                            unsigned long long& total, Scratch<NT, E>& sh, int& rb) {
  constexpr int PP = pp(NT);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  unsigned long long s = 0;
#pragma unroll
  for (int i = 0; i < PP; ++i) s += q[i];
  unsigned long long inc = s;  // inclusive suffix over lanes >= this one
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long x = __shfl_down_sync(FULL, inc, o);
    if (lane + o < 32) inc += x;
  }
  if (lane == 0) sh.part_q[rb][w] = inc;
  __syncthreads();
  unsigned long long after = 0, tot = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) {
    if (i > w) after += sh.part_q[rb][i];
    tot += sh.part_q[rb][i];
  }
  total = tot;
  rb ^= 1;
  unsigned long long run = after + inc;  // sum over positions >= this thread's first
#pragma unroll
  for (int i = 0; i < PP; ++i) {
    suf[i] = run;
    run -= q[i];
  }
}

// Inverse CDF over list positions in vocabulary order: w[i] is the kept
// weight of position t PP + i (0 for removed and padding).  Returns the chosen
// position in every thread (-1: nothing positive); `owner` is set in the one
// thread that holds it, whose `flags` then carry the draw's flags.  Two
// barriers (three when nothing passes u * total).
template <int NT, int E>
Q3S_DEV int list_draw(const float (&w)[pp(NT)], float u, Scratch<NT, E>& sh, int& rb, int& flags, bool& owner) {
  constexpr int PP = pp(NT);
  const int t = threadIdx.x;
  float loc = 0.0f;
#pragma unroll
  for (int i = 0; i < PP; ++i) loc = __fadd_rn(loc, w[i]);
  float W;
  const float pre = block_excl_scan_f<NT, E>(loc, W, sh, rb);
  const float thr = __fmul_rn(u, W);
  int pick = 0x7fffffff, last = -1;
  float cdf = 0.0f, prev = 0.0f, acc = pre;
#pragma unroll
  for (int i = 0; i < PP; ++i) {
    const float before = acc;
    acc = __fadd_rn(acc, w[i]);
    if (w[i] > 0.0f) {
      last = t * PP + i;
      if (pick == 0x7fffffff && acc > thr) {
        pick = t * PP + i;
        cdf = acc;
        prev = before;
      }
    }
  }
  const int first = block_min_i<NT, E>(pick, sh, rb);
  if (first != 0x7fffffff) {
    owner = pick == first;
    const float tol = BOUNDARY_EPS * W;
    if (owner && ((__fsub_rn(cdf, thr) < tol) || (__fsub_rn(thr, prev) < tol))) flags |= Q3S_ROW_DRAW_BOUNDARY;
    return first;
  }
  const int lst = block_max_i<NT, E>(last, sh, rb);
  owner = lst >= 0 ? last == lst : t == 0;
  if (owner) flags |= Q3S_ROW_FALLBACK;
  return lst;
}

// Exclusive block scan of a count (thread order) fused with a fixed-order
// block sum of a float.  One barrier.
template <int NT, int E>
Q3S_DEV uint32_t block_scan_count_sum(uint32_t v, float f, uint32_t& total, float& fsum, Scratch<NT, E>& sh,
                                      int& rb) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc += n;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) f = __fadd_rn(f, __shfl_xor_sync(FULL, f, o));
  if (lane == 31) sh.part_u[rb][w] = inc;
  if (lane == 0) sh.part_f2[rb][w] = f;
  __syncthreads();
  uint32_t pre = 0, tot = 0;
  float fs = 0.0f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) {
    const uint32_t x = sh.part_u[rb][i];
    pre += (i < w) ? x : 0u;
    tot += x;
    fs = __fadd_rn(fs, sh.part_f2[rb][i]);
  }
  rb ^= 1;
  total = tot;
  fsum = fs;
  return pre + inc - v;
}

// Block max with NaN propagation.  One barrier.
template <int NT, int E>
Q3S_DEV float block_max_nan(float v, Scratch<NT, E>& sh, int& rb) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = max_nan(v, __shfl_xor_sync(FULL, v, o));
  if ((threadIdx.x & 31) == 0) sh.part_f[rb][threadIdx.x >> 5] = v;
  __syncthreads();
  float m = sh.part_f[rb][0];
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) m = max_nan(m, sh.part_f[rb][i]);
  rb ^= 1;
  return m;
}

// Fixed-order block sum of a float.  One barrier.
template <int NT, int E>
Q3S_DEV float block_sum_f(float v, Scratch<NT, E>& sh, int& rb) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(FULL, v, o));
  if ((threadIdx.x & 31) == 0) sh.part_f2[rb][threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) s = __fadd_rn(s, sh.part_f2[rb][i]);
  rb ^= 1;
  return s;
}

// Block suffix sums of floats over sorted positions (as block_suffix_q):
// suf[i] = the sum over positions >= t PP + i, in a fixed order.  One barrier.
template <int NT, int E>
Q3S_DEV void block_suffix_f(const float (&q)[pp(NT)], float (&suf)[pp(NT)], Scratch<NT, E>& sh, int& rb) {
  constexpr int PP = pp(NT);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  // suffix inside the thread, then across lanes, then across warps
  float ins[PP];
  float run = 0.0f;
#pragma unroll
  for (int i = PP - 1; i >= 0; --i) {
    run = __fadd_rn(q[i], run);
    ins[i] = run;
  }
  float inc = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float x = __shfl_down_sync(FULL, inc, o);
    if (lane + o < 32) inc = __fadd_rn(inc, x);
  }
  float after_lane = __shfl_down_sync(FULL, inc, 1);
  if (lane == 31) after_lane = 0.0f;
  if (lane == 0) sh.part_f2[rb][w] = inc;
  __syncthreads();
  float after = 0.0f;
#pragma unroll
  for (int i = NT / 32 - 1; i >= 0; --i)
    if (i > w) after = __fadd_rn(sh.part_f2[rb][i], after);
  rb ^= 1;
  const float base = __fadd_rn(after_lane, after);
#pragma unroll
  for (int i = 0; i < PP; ++i) suf[i] = __fadd_rn(ins[i], base);
}

}  // namespace lean
}  // namespace q3s

namespace q3s {

// 16-byte read-only load with L1 allocation, issued where it is written
// (volatile: not sunk to its first use).
Q3S_DEV uint4 ld_nc16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// The row's logits as fp32 into registers, entries [v0, v0 + E) (-inf past V),
// through the read-only path with L1 allocation, so that the exact re-reads of
// single candidates hit L1.
template <bool BF16, int E>
Q3S_DEV void lean_load(const void* base, int64_t row_off, int V, int v0, bool vec, float (&x)[E], uint32_t& vmask) {
  if (vec && v0 + E <= V) {
    if (BF16) {
      const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + row_off + v0);
      uint4 r[E / 8];
#pragma unroll
      for (int c = 0; c < E / 8; ++c) r[c] = ld_nc16(p + c);
#pragma unroll
      for (int c = 0; c < E / 8; ++c) {
        const uint32_t w[4] = {r[c].x, r[c].y, r[c].z, r[c].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          x[8 * c + 2 * i] = __uint_as_float(w[i] << 16);
          x[8 * c + 2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
      }
    } else {
      const uint4* p = reinterpret_cast<const uint4*>(static_cast<const float*>(base) + row_off + v0);
      uint4 r[E / 4];
#pragma unroll
      for (int c = 0; c < E / 4; ++c) r[c] = ld_nc16(p + c);
#pragma unroll
      for (int c = 0; c < E / 4; ++c) {
        x[4 * c] = __uint_as_float(r[c].x);
        x[4 * c + 1] = __uint_as_float(r[c].y);
        x[4 * c + 2] = __uint_as_float(r[c].z);
        x[4 * c + 3] = __uint_as_float(r[c].w);
      }
    }
    vmask = (E == 32) ? 0xffffffffu : ((1u << E) - 1u);
    return;
  }
  vmask = 0;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const int v = v0 + j;
    x[j] = -INFINITY;
    if (v < V) {
      x[j] = BF16 ? bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(base) + row_off + v))
                  : __ldg(static_cast<const float*>(base) + row_off + v);
      vmask |= 1u << j;
    }
  }
}

// The exact register-resident core for one row (sample_core): the row's
// logits re-read, suppress and the EOS gate applied, presence from the
// shared-memory map.  Needs sh.hist zero.  Every thread returns the id; the
// flags are complete in the thread that owns it.
template <int NT, int E, bool BF16>
__device__ __noinline__ int lean_exact_row(const void* logits, int64_t row_off, int V, bool vec, const uint8_t* suppress,
                                           bool history, bool gate, int eos_id, bool greedy, float T, float pen, int kk,
                                           float top_p, float u, float* proc, Scratch<NT, E>& sh, int& flags,
                                           uint32_t& err) {
  const int v0 = static_cast<int>(threadIdx.x) * E;
  float xr[E];
  uint32_t vm;
  lean_load<BF16, E>(logits, row_off, V, v0, vec, xr, vm);
  uint32_t pmask = 0;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const int v = v0 + j;
    if (v >= V) continue;
    if (suppress && __ldg(suppress + v)) xr[j] = NEG_SUPPRESS;
    if (gate && v == eos_id) xr[j] = -INFINITY;
    if (history && sh.seen[v]) pmask |= 1u << j;
  }
  RowCfg c;
  c.mode = Q3S_DRAW_ICDF;
  c.greedy = greedy;
  c.T = T;
  c.k = kk;
  c.top_p = top_p;
  c.u = u;
  c.noise = nullptr;
  return sample_core<NT, E, Q3S_DRAW_ICDF>(xr, vm, pmask & vm, pen, V, c, sh, proc, flags, err);
}

// PROC adds the verification-only processed-logits output (x'/T where top-k
// and top-p keep the entry, -inf elsewhere; x' for greedy rows).
template <int NT, int E, bool BF16, bool PROC>
__global__ void __launch_bounds__(NT, lean::min_blocks(NT)) sample_lean_kernel(const SampleArgs a) {
  using namespace lean;
  constexpr int PP = pp(NT);
  __shared__ Scratch<NT, E> sh;
  __shared__ uint32_t maxkey;  // largest exact key on the list
  __shared__ int top_above;    // whole-vocabulary rows: bit 0 / 1 -- the cut clears the bracket's lower / upper guard
  __shared__ int brk[4];       // whole-vocabulary rows: the bracket (lo, hi bins), entries above it, usable
  __shared__ uint8_t dummy_byte;  // the history scatter's target for ids outside [0, V)
  const int t = static_cast<int>(threadIdx.x);
  const int b = static_cast<int>(blockIdx.x);
  const int v0 = t * E;
  const int V = a.V;
  uint32_t err = 0;
  int rb = 0;

  // ---- parameters, the suppress bytes of this thread's entries ------------
  int o0 = 0, o1 = 0, olen = -1;
  if (a.history) {
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
  const uint8_t* const suppress = a.suppress;
  uint2 supb[E / 8];
#pragma unroll
  for (int c = 0; c < E / 8; ++c) {
    const int vb = v0 + 8 * c;
    if (suppress && a.vec_suppress && vb + 8 <= V) {
      supb[c] = __ldg(reinterpret_cast<const uint2*>(suppress + vb));
    } else {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t f = (suppress && vb + i < V && __ldg(suppress + vb + i)) ? 1u : 0u;
        if (i < 4) lo |= f << (8 * i);
        else hi |= f << (8 * (i - 4));
      }
      supb[c] = make_uint2(lo, hi);
    }
  }
  // the row's logits: issued first (ahead of the history scatter), unless the
  // kernel that writes them may still be running (programmatic dependent)
  float x[E];
  uint32_t vmask = 0;
  const int64_t row_off = static_cast<int64_t>(b) * a.row_stride;
  if (!a.pdl) lean_load<BF16, E>(a.logits, row_off, V, v0, a.vec_logits, x, vmask);
  clear_hist<NT, E>(sh);
  if (t == 0) {
    sh.flags = 0;
    maxkey = 0u;
  }
  if (a.history) {
#pragma unroll
    for (int c = 0; c < E / 8; ++c) *reinterpret_cast<uint2*>(&sh.seen[v0 + 8 * c]) = make_uint2(0u, 0u);
  }
  __syncthreads();

  // ---- presence scatter from the packed history (racing stores of the same
  //      byte need no atomics); 16-byte loads over the aligned middle ------
  int hist_len = 0;
  if (a.history) {
    if (a.history_lengths) o1 = row_end_in_region(o0, o1, olen);
    if (o0 < 0 || o1 < o0 || static_cast<int64_t>(o1) > a.history_len) {
      err |= Q3S_DEVERR_OFFSETS;
      o0 = o1 = 0;
    }
    hist_len = o1 - o0;
    // the aligned middle by 16-byte loads (4 in flight a thread), the ragged
    // ends (at most 3 ids each, all of them without 16-byte alignment) by
    // scalar loads
    const int32_t* h = a.history;
    int mid0 = o0, mid1 = o0;
    if (a.vec_history) {
      mid0 = min(o1, (o0 + 3) & ~3);
      mid1 = mid0 + ((o1 - mid0) & ~3);
    }
    // branch-free: an id outside [0, V) is stored to a dummy byte and reported
    bool bad = false;
    auto put = [&](int idv) {
      const bool ok = static_cast<unsigned>(idv) < static_cast<unsigned>(V);
      bad |= !ok;
      *(ok ? &sh.seen[idv] : &dummy_byte) = 1;
    };
    const int nv = (mid1 - mid0) >> 2;
    const int4* hv = reinterpret_cast<const int4*>(h + mid0);
    for (int i = t; i < nv; i += 4 * NT) {
      int4 q[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) q[k] = i + k * NT < nv ? __ldg(hv + i + k * NT) : make_int4(0, 0, 0, 0);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (i + k * NT < nv) {
          put(q[k].x);
          put(q[k].y);
          put(q[k].z);
          put(q[k].w);
        }
    }
    for (int r = o0 + t; r < mid0; r += NT) put(__ldg(h + r));
    for (int r = mid1 + t; r < o1; r += NT) put(__ldg(h + r));
    if (bad) err |= Q3S_DEVERR_HISTORY_ID;
  }
  // launched behind the kernel that writes the logits: wait for it here,
  // then load the row (otherwise the row's loads went out before the scatter)
  if (a.pdl) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    lean_load<BF16, E>(a.logits, row_off, V, v0, a.vec_logits, x, vmask);
  }
  __syncthreads();  // presence complete
  uint2 prw[E / 8];
#pragma unroll
  for (int c = 0; c < E / 8; ++c)
    prw[c] = a.history ? *reinterpret_cast<const uint2*>(&sh.seen[v0 + 8 * c]) : make_uint2(0u, 0u);
  const int cur = a.cur_len ? cur_given : hist_len;
  const int eos_id = a.eos_id;
  const bool gate = eos_id >= 0 && eos_id < V && cur < min_new;

  // exact x' of entry v (suppress, EOS gate, repetition penalty), re-read
  auto exact_x = [&](int v) -> float {
    float xv = BF16 ? bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(a.logits) + row_off + v))
                    : __ldg(static_cast<const float*>(a.logits) + row_off + v);
    if (suppress && __ldg(suppress + v)) xv = NEG_SUPPRESS;
    if (gate && v == eos_id) xv = -INFINITY;
    if (a.history && sh.seen[v]) xv = xv > 0.0f ? __fdiv_rn(xv, pen) : __fmul_rn(xv, pen);
    return xv;
  };

  // ---- pass 1: suppress, EOS gate, repetition penalty, row maximum -------
  //      few-survivor rows: x * RN(1/pen) for present entries > 0 (within 2
  //      ulps; the list recomputes exact values); whole-vocabulary rows: the
  //      correctly rounded quotient, and s = x'/T likewise (their weights
  //      come from these values)
  const bool greedy = !(T > 0.0f);
  const bool topk = kk > 0 && kk < V;
  const int K = greedy ? 1 : kk;
  const bool few = greedy || (topk && K <= KMAX);
  const bool cut = top_p < 1.0f;
  const float rpen = __frcp_rn(pen);
  const float rT = __frcp_rn(T);
  const bool divT = !few && T != 1.0f;
  if (gate && eos_id >= v0 && eos_id < v0 + E) {
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (v0 + j == eos_id) x[j] = -INFINITY;
  }
  float m = -INFINITY;
  if (few) {
#pragma unroll
    for (int c = 0; c < E / 8; ++c) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int j = 8 * c + i;
        float y = byte_set(supb[c], i) ? NEG_SUPPRESS : x[j];
        const float f = byte_set(prw[c], i) ? (y > 0.0f ? rpen : pen) : 1.0f;
        y = __fmul_rn(y, f);
        x[j] = y;
        m = max_nan(m, y);
      }
    }
  } else {
    // branch-free: both penalty branches for every entry, two entries per
    // packed fp32x2 operation; the temperature division in its own variant
    auto vocab_pass = [&](auto divt_tag) {
      constexpr bool DIVT = decltype(divt_tag)::value;
#pragma unroll
      for (int c = 0; c < E / 8; ++c) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const int j = 8 * c + i;
          float y0 = byte_set(supb[c], i) ? NEG_SUPPRESS : x[j];
          float y1 = byte_set(supb[c], i + 1) ? NEG_SUPPRESS : x[j + 1];
          const float2 q = div2_rn_row(make_float2(y0, y1), pen, rpen);
          const float2 py = __fmul2_rn(make_float2(y0, y1), make_float2(pen, pen));
          if (byte_set(prw[c], i)) y0 = y0 > 0.0f ? q.x : py.x;
          if (byte_set(prw[c], i + 1)) y1 = y1 > 0.0f ? q.y : py.y;
          if constexpr (DIVT) {
            const float2 st = div2_rn_row(make_float2(y0, y1), T, rT);
            y0 = y0 == -INFINITY ? y0 : st.x;
            y1 = y1 == -INFINITY ? y1 : st.y;
          }
          x[j] = y0;
          x[j + 1] = y1;
          m = max_nan(m, max_nan(y0, y1));
        }
      }
    };
    if (divT)
      vocab_pass(std::true_type{});
    else
      vocab_pass(std::false_type{});
  }
  m = block_max_nan<NT, E>(m, sh, rb);
  // the fast paths' window: finite values within +-2000, penalty and
  // temperature within [2^-20, 2^20] (NaN and infinite maxima fail here)
  const bool win = pen >= 0x1p-20f && pen <= 0x1p20f && (greedy || (T >= 0x1p-20f && T <= 0x1p20f)) &&
                   fabsf(m) <= 2000.0f;
  int path = 0;  // 0: exact core, 1: candidate list, 2: whole vocabulary
  if (win && few) path = 1;
  else if (win && !greedy && !topk) path = 2;

  int id = 0, flags = 0;
  bool owner = t == 0;
  bool fast_done = false;
  int n = 0;                        // list length
  uint32_t rmask = 0, bbits = 0;    // whole-vocabulary rows: list entries the cut removed, entries below the bracket
  const uint32_t* inv = list_inv(sh);

  // List records: the owners write each list entry's vocabulary index at its
  // position (vocabulary order), then every thread completes positions t,
  // t + NT, ... (balanced whatever the owners' counts).
  auto write_indices = [&](uint32_t cbits, uint32_t pos0) {
    uint32_t cb = cbits, p = pos0;
    while (cb) {
      const int j = __ffs(cb) - 1;
      cb &= cb - 1u;
      sh.cand[p].y = static_cast<uint32_t>(v0 + j);
      ++p;
    }
  };

  if (path == 1) {
    // ==== few survivors: top-k (or greedy) candidates, exact on the list ====
    // pass 2: distance bins 1/8 wide below the maximum (bin 255: the rest)
    const float c0 = ref_c0(8.0f, m);
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const uint32_t k = ref_bin(x[j], 8.0f, c0);
      if (k < 255u) atomicAdd(&sh.hist[0][k], 1u);  // bin 255 (the rest) is never read
    }
    __syncthreads();
    uint32_t kb, nthru;
    warp_bin_of_rank(sh.hist[0], static_cast<uint32_t>(K), kb, nthru);  // every warp, same answer
    if (kb <= 253u && nthru <= static_cast<uint32_t>(LCAP)) {
      // pass 3: candidates down to one bin below the K-th largest's bin
      // (bin <= lim exactly when the bin's float is <= 2^23 + lim)
      const float rlim = __uint_as_float(F23 + kb + 1u);
      uint32_t cbits = 0;
#pragma unroll
      for (int j = 0; j < E; ++j) cbits |= (__fmaf_rn(x[j], -8.0f, c0) <= rlim ? 1u : 0u) << j;
      uint32_t n32;
      float ign;
      const uint32_t pos0 = block_scan_count_max<NT, E>(__popc(cbits), -INFINITY, n32, ign, sh, rb);
      n = static_cast<int>(n32);
      // every warp has read the histogram: zero it for the list's bins
      for (int i = t; i < NBINS; i += NT) sh.hist[0][i] = 0u;
      write_indices(cbits, pos0);
      __syncthreads();
      // exact x' and s = x'/T per list entry
      for (int p = t; p < n; p += NT) {
        const int v = static_cast<int>(sh.cand[p].y);
        const float xe = exact_x(v);
        const float sv = (greedy || T == 1.0f) ? xe : __fdiv_rn(xe, T);
        sh.cand[p] = make_uint4(__float_as_uint(sv), static_cast<uint32_t>(v), __float_as_uint(xe), 0u);
        atomicMax(&maxkey, f2key(sv));
      }
      __syncthreads();
      if (greedy) {
        // torch.argmax of x' (lowest index on ties)
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int p = t; p < n; p += NT) {
          const uint4 r = sh.cand[p];
          if (arg_better(__uint_as_float(r.z), static_cast<int>(r.y), bv, bi)) {
            bv = __uint_as_float(r.z);
            bi = static_cast<int>(r.y);
          }
        }
        id = block_argmax<NT, E>(bv, bi, bi, sh, rb);
        flags = Q3S_ROW_GREEDY;
        owner = t == 0;
        fast_done = true;
      } else {
        // exact bins (1/8 of x' per bin, from the list's largest s), counting
        // sort, ranks inside each bin
        const float ms = key2f(maxkey);
        const float cs = __fmul_rn(8.0f, T);
        const float c0s = ref_c0(cs, ms);
        for (int p = t; p < n; p += NT) {
          const uint32_t k = ref_bin(__uint_as_float(sh.cand[p].x), cs, c0s);
          sh.cand[p].w = k;
          atomicAdd(&sh.hist[0][k], 1u);
        }
        __syncthreads();
        list_sort_desc<NT, E>(sh, n);
        // HF TopK: s >= the K-th largest (ties kept): sorted positions [0, nk)
        const float sK = __uint_as_float(sh.cand[inv[K - 1]].x);
        float wv[PP];
        unsigned long long q[PP];
        bool kp[PP];
        uint32_t pl[PP];
#pragma unroll
        for (int i = 0; i < PP; ++i) {
          const int P = t * PP + i;
          kp[i] = false;
          wv[i] = 0.0f;
          q[i] = 0ull;
          pl[i] = 0u;
          if (P < n) {
            pl[i] = inv[P];
            const float sv = __uint_as_float(sh.cand[pl[i]].x);
            kp[i] = sv >= sK;
            wv[i] = kp[i] ? softmax_weight(sv, ms) : 0.0f;
            q[i] = mass_fixed(wv[i]);
          }
        }
        if (cut) {
          // HF TopP over the kept entries in ascending order (the reverse of
          // the sorted positions): a position goes when the mass at or below
          // it is <= tau = floor((1-p) Zq); position 0 (the ascending-last)
          // always stays
          unsigned long long suf[PP], Zq;
          block_suffix_q<NT, E>(q, suf, Zq, sh, rb);
          const float frac = __fsub_rn(1.0f, top_p);
          const unsigned long long tau = __double2ull_rd(static_cast<double>(frac) * static_cast<double>(Zq));
          const unsigned long long eps = Zq / 1000000ull;
          bool near = false;
#pragma unroll
          for (int i = 0; i < PP; ++i) {
            const int P = t * PP + i;
            if (P < n && kp[i]) {
              const bool rm = P != 0 && suf[i] <= tau;
              if (tau < Zq) near |= rm ? (tau - suf[i] < eps) : (suf[i] > tau && suf[i] - tau < eps);
              kp[i] = !rm;
            }
          }
          if (near) atomicOr(&sh.flags, Q3S_ROW_TOPP_BOUNDARY);
        }
#pragma unroll
        for (int i = 0; i < PP; ++i) {
          const int P = t * PP + i;
          if (P < n) {
            sh.cand[pl[i]].z = __float_as_uint(kp[i] ? wv[i] : 0.0f);
            sh.surv[pl[i]] = kp[i] ? 1 : 0;
          }
        }
        __syncthreads();
        // inverse CDF over the kept list in vocabulary order
        float wl[PP];
#pragma unroll
        for (int i = 0; i < PP; ++i) {
          const int p = t * PP + i;
          wl[i] = p < n ? __uint_as_float(sh.cand[p].z) : 0.0f;
        }
        int dflags = 0;
        bool down = false;
        const int pp = list_draw<NT, E>(wl, u, sh, rb, dflags, down);
        id = pp >= 0 ? static_cast<int>(sh.cand[pp].y) : 0;
        owner = down;
        flags = dflags | (down ? sh.flags : 0);
        fast_done = true;
      }
    }
  }
  else if (path == 2) {
    // ==== whole vocabulary: top-k off; x holds exact s ======================
    // pass 2: softmax weights 2^((s - m) log2 e) (stored over s), their sum
    // (two interleaved partial sums), and (top-p) a count histogram by the
    // weight's bits
    const float mL = __fmul_rn(m, LOG2E);
    float2 zs = make_float2(0.0f, 0.0f);
    auto weights_pass = [&](auto cut_tag) {
      constexpr bool CUT = decltype(cut_tag)::value;
#pragma unroll
      for (int j = 0; j < E; j += 2) {
        const float2 arg = __ffma2_rn(make_float2(x[j], x[j + 1]), make_float2(LOG2E, LOG2E), make_float2(-mL, -mL));
        const float w0 = ex2(arg.x), w1 = ex2(arg.y);
        x[j] = w0;
        x[j + 1] = w1;
        zs = __fadd2_rn(zs, make_float2(w0, w1));
        if constexpr (CUT) {
          // bin 255 (weights < 2^-15.9 and zeros) is not counted
          const uint32_t k0 = wbin(w0), k1 = wbin(w1);
          if (k0 < 255u) atomicAdd(&sh.hist[0][k0], 1u);
          if (k1 < 255u) atomicAdd(&sh.hist[0][k1], 1u);
        }
      }
    };
    if (cut)
      weights_pass(std::true_type{});
    else
      weights_pass(std::false_type{});
    float loc = __fadd_rn(zs.x, zs.y);  // this thread's kept weight (the draw's per-thread total)
    const float Z = block_sum_f<NT, E>(loc, sh, rb);  // also publishes the histogram
    bool ok = true;
    if (cut) {
      // warp 0: estimated ascending masses (count x bin midpoint; weights
      // < 2^-15.9 are not counted), the bin where they pass tau, a 5-bin
      // bracket around it
      const float frac = __fsub_rn(1.0f, top_p);
      const float tau = __fmul_rn(frac, Z);
      if (t < 32) {
        const int lane = t;
        uint32_t c[8], pre[8];
        (void)warp_bins_prefix(sh.hist[0], c, pre);
        float sl[8], run = 0.0f;
#pragma unroll
        for (int i = 7; i >= 0; --i) {
          const uint32_t k = static_cast<uint32_t>(8 * lane + i);
          run = __fadd_rn(run, __fmul_rn(static_cast<float>(c[i]), wbin_mid(k)));  // bin 255 holds no counts
          sl[i] = run;
        }
        float inc = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_down_sync(FULL, inc, o);
          if (lane + o < 32) inc = __fadd_rn(inc, y);
        }
        float after = __shfl_down_sync(FULL, inc, 1);
        if (lane == 31) after = 0.0f;
        int jh = -1;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (__fadd_rn(sl[i], after) > tau) jh = 8 * lane + i;
        jh = __reduce_max_sync(FULL, jh);
        const int lo = max(jh - 2, 0), hi = min(jh + 2, 254);
        uint32_t inb = 0, abv = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int k = 8 * lane + i;
          inb += (k >= lo && k <= hi) ? c[i] : 0u;
          abv += k < lo ? c[i] : 0u;
        }
        inb = __reduce_add_sync(FULL, inb);
        abv = __reduce_add_sync(FULL, abv);
        if (lane == 0) {
          brk[0] = lo;
          brk[1] = hi;
          brk[2] = static_cast<int>(abv);
          brk[3] = jh >= 0 && jh <= 254 && inb <= static_cast<uint32_t>(LCAP);
          top_above = 0;
        }
      }
      __syncthreads();
      const int lo = brk[0], hi = brk[1];
      const uint32_t abv = static_cast<uint32_t>(brk[2]);
      ok = brk[3] != 0;
      if (ok) {
        // pass 3: below the bracket (w under the bottom edge of bin hi)
        // removed, its mass summed; bracket entries (w under the top edge of
        // bin lo) -> list; the kept weights' per-thread sums for the draw
        const float wlo = __uint_as_float((2032u - static_cast<uint32_t>(hi)) << 19);
        const float whi = __uint_as_float((2033u - static_cast<uint32_t>(lo)) << 19);
        float blo = 0.0f;
        float2 ls = make_float2(0.0f, 0.0f);
        uint32_t cbits = 0;
#pragma unroll
        for (int j = 0; j < E; j += 2) {
          float w[2] = {x[j], x[j + 1]};
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const bool below = w[e] < wlo;
            blo = __fadd_rn(blo, below ? w[e] : 0.0f);
            cbits |= ((!below && w[e] < whi) ? 1u : 0u) << (j + e);
            bbits |= (below ? 1u : 0u) << (j + e);
            w[e] = below ? 0.0f : w[e];
          }
          x[j] = w[0];
          x[j + 1] = w[1];
          ls = __fadd2_rn(ls, make_float2(w[0], w[1]));
        }
        loc = __fadd_rn(ls.x, ls.y);
        uint32_t n32;
        float blo_tot;
        const uint32_t pos0 = block_scan_count_sum<NT, E>(__popc(cbits), blo, n32, blo_tot, sh, rb);
        n = static_cast<int>(n32);
        for (int i = t; i < NBINS; i += NT) sh.hist[0][i] = 0u;
        write_indices(cbits, pos0);
        __syncthreads();
        // exact s and its weight per list entry
        for (int p = t; p < n; p += NT) {
          const int v = static_cast<int>(sh.cand[p].y);
          const float xe = exact_x(v);
          const float sv = T == 1.0f ? xe : __fdiv_rn(xe, T);
          const float w = ex2(__fmaf_rn(sv, LOG2E, -mL));
          sh.cand[p] = make_uint4(__float_as_uint(sv), static_cast<uint32_t>(v), __float_as_uint(w), 0u);
          atomicMax(&maxkey, f2key(sv));
        }
        __syncthreads();
        // exact bins over the bracket's span (~0.3 of s in 768ths), counting
        // sort, ranks inside each bin
        const float msl = key2f(maxkey);
        const float c0l = ref_c0(768.0f, msl);
        for (int p = t; p < n; p += NT) {
          const uint32_t k = ref_bin(__uint_as_float(sh.cand[p].x), 768.0f, c0l);
          sh.cand[p].w = k;
          atomicAdd(&sh.hist[0][k], 1u);
        }
        __syncthreads();
        list_sort_desc<NT, E>(sh, n);
        // HF TopP: ascending (s, index) = descending positions reversed;
        // cumulative mass = everything below the bracket + the list's
        // suffix; a position goes when that is <= tau
        float wq[PP], suf[PP];
#pragma unroll
        for (int i = 0; i < PP; ++i) {
          const int P = t * PP + i;
          wq[i] = P < n ? __uint_as_float(sh.cand[inv[P]].z) : 0.0f;
        }
        block_suffix_f<NT, E>(wq, suf, sh, rb);
        const float tol = BOUNDARY_EPS * Z;
        // guards: the bracket's lower / upper edge weights moved inward by
        // 2^-7, far more than the weights' own error (a few ulps)
        const float g_lo = __fmul_rn(wlo, 1.0078125f);
        const float g_hi = __fmul_rn(whi, 0.9921875f);
        bool near = t == 0 && blo_tot <= tau && __fsub_rn(tau, blo_tot) < tol;
        int seen_ok = 0;
#pragma unroll
        for (int i = 0; i < PP; ++i) {
          const int P = t * PP + i;
          if (P < n) {
            const float cum = __fadd_rn(blo_tot, suf[i]);
            bool rm = cum <= tau;
            if (P == 0 && abv == 0u) rm = false;  // the ascending-last entry of the row stays
            near |= rm ? (__fsub_rn(tau, cum) < tol) : (__fsub_rn(cum, tau) < tol);
            // the cut lies inside the bracket, clear of its edges: some
            // removed entry above the lower guard, some kept one below the
            // upper guard
            if (rm && wq[i] >= g_lo) seen_ok |= 1;
            if (!rm && wq[i] <= g_hi) seen_ok |= 2;
            sh.surv[inv[P]] = rm ? 0 : 1;
          }
        }
        if (seen_ok) atomicOr(&top_above, seen_ok);
        if (near) atomicOr(&sh.flags, Q3S_ROW_TOPP_BOUNDARY);
        __syncthreads();
        // entries outside the bracket are then on the same side of the cut
        // in exact order as in the classification above
        ok = (top_above & 1) && (abv == 0u || (top_above & 2));
        if (ok) {
          // this thread's list entries the cut removed: out of its total
          uint32_t cb = cbits, p = pos0;
          while (cb) {
            const int j = __ffs(cb) - 1;
            cb &= cb - 1u;
            if (!sh.surv[p]) {
              rmask |= 1u << j;
              loc = __fsub_rn(loc, __uint_as_float(sh.cand[p].z));
            }
            ++p;
          }
        }
      }
    }
    if (ok) {
      // ---- inverse CDF over the row in vocabulary order: block scan of the
      //      per-thread totals; only the threads whose range reaches u * W
      //      walk their entries (all of them, in the rare case none picks)
      float W;
      const float pre = block_excl_scan_f<NT, E>(fmaxf(loc, 0.0f), W, sh, rb);
      const float thr = __fmul_rn(u, W);
      int pick = 0x7fffffff, last = -1;
      float cdf = 0.0f, prev = 0.0f;
      auto walk = [&]() {
        float acc = pre;
#pragma unroll
        for (int j = 0; j < E; ++j) {
          const float w = ((rmask >> j) & 1u) ? 0.0f : x[j];
          const float before = acc;
          acc = __fadd_rn(acc, w);
          if (w > 0.0f) {
            last = v0 + j;
            if (pick == 0x7fffffff && acc > thr) {
              pick = v0 + j;
              cdf = acc;
              prev = before;
            }
          }
        }
      };
      const float dl = __fmul_rn(thr, 0x1p-16f);
      if (pre <= __fadd_rn(thr, dl) && __fadd_rn(pre, loc) >= __fsub_rn(thr, dl)) walk();
      int first = block_min_i<NT, E>(pick, sh, rb);
      if (first == 0x7fffffff) {
        pick = 0x7fffffff;
        walk();
        first = block_min_i<NT, E>(pick, sh, rb);
      }
      if (first != 0x7fffffff) {
        id = first;
        owner = pick == first;
        if (owner) {
          flags = sh.flags;
          const float dtol = BOUNDARY_EPS * W;
          if ((__fsub_rn(cdf, thr) < dtol) || (__fsub_rn(thr, prev) < dtol)) flags |= Q3S_ROW_DRAW_BOUNDARY;
        }
      } else {
        const int lst = block_max_i<NT, E>(last, sh, rb);
        id = lst >= 0 ? lst : 0;
        owner = lst >= 0 ? last == lst : t == 0;
        if (owner) flags = sh.flags | Q3S_ROW_FALLBACK;
      }
      fast_done = true;
    }
  }
  if (!fast_done) {
    // ==== the exact core (rare rows), out of line so that its registers
    //      stay off the fast paths ==========================================
    __syncthreads();
    clear_hist<NT, E>(sh);
    __syncthreads();
    float* proc = PROC ? a.processed + static_cast<int64_t>(b) * a.proc_stride : nullptr;
    id = lean_exact_row<NT, E, BF16>(a.logits, row_off, V, a.vec_logits, suppress, a.history != nullptr, gate, eos_id,
                                     greedy, T, pen, kk, top_p, u, proc, sh, flags, err);
    owner = (id >= v0 && id < v0 + E) || (t == 0 && (id < 0 || id >= V));
    flags |= Q3S_ROW_EXACT_CORE;
  } else if constexpr (PROC) {
    // verification output: x'/T where kept, -inf elsewhere (greedy: x')
    float* const prow = a.processed + static_cast<int64_t>(b) * a.proc_stride;
    if (path == 1 && !greedy) {
#pragma unroll
      for (int j = 0; j < E; ++j)
        if (v0 + j < V) prow[v0 + j] = -INFINITY;
      __syncthreads();
      for (int p = t; p < n; p += NT)
        if (sh.surv[p]) prow[sh.cand[p].y] = __uint_as_float(sh.cand[p].x);
    } else {
#pragma unroll 1
      for (int j = 0; j < E; ++j) {
        const int v = v0 + j;
        if (v >= V) continue;
        const float xe = exact_x(v);
        float o = xe;
        if (!greedy) {
          const bool kept = !((bbits >> j) & 1u) && !((rmask >> j) & 1u);
          o = kept ? (T == 1.0f ? xe : __fdiv_rn(xe, T)) : -INFINITY;
        }
        prow[v] = o;
      }
    }
  }
  if (owner) {
    if (a.ids64) a.ids64[b] = id;
    if (a.ids32) a.ids32[b] = id;
    if (a.row_flags) a.row_flags[b] = flags;
  }
  if (err && a.error_word) atomicOr(a.error_word, static_cast<int>(err));
}

}  // namespace q3s
