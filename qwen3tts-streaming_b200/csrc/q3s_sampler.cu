// q3s_sampler.cu -- sm_100a kernels and the C ABI of include/q3s_sampler.h.
//
// sample_rows_kernel   one CTA per row: load -> suppress / presence penalty /
//                      EOS gate -> (greedy | gumbel exactly-K | icdf top-k,
//                      top-p, inverse-CDF) -> id (+ count update).
// sample_warp_kernel   one warp per row (q3s_warp.cuh), icdf steps of large
//                      batches: no block barriers, ~12 rows in flight per SM.
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
#include <atomic>
#include <type_traits>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "q3s_args.cuh"
#include "q3s_device.cuh"
#include "q3s_philox.cuh"
#include "q3s_step.cuh"
#include "q3s_core.cuh"
#include "q3s_sampler.h"

namespace q3s {

constexpr int MAX_NBUF = 16;

// ---------------------------------------------------------------------------
// one sampling step, one CTA per row
// ---------------------------------------------------------------------------

template <int NT, int E, bool BF16, int MODE>
__global__ void __launch_bounds__(NT) sample_rows_kernel(const SampleArgs a) {
  __shared__ Scratch<NT, E> sh;
  const int b = blockIdx.x;
  const int t = threadIdx.x;
  const int v0 = t * E;
  const int V = a.V;
  uint32_t err = 0;

  // launched behind the kernel that writes the logits: wait for it first
  if (a.pdl) asm volatile("griddepcontrol.wait;" ::: "memory");
  // issue every independent load first
  const int shift = a.col_shift ? norm_shift(__ldg(a.col_shift + b), V) : 0;
  float x[E];
  uint32_t vmask;
  load_logits<BF16, E>(a.logits, static_cast<int64_t>(b) * a.row_stride, V, v0, shift, a.vec_logits, x, vmask);
  int o0 = 0, o1 = 0, olen = -1;
  if (a.history) {
    o0 = __ldg(a.offsets + b);
    o1 = __ldg(a.offsets + b + 1);  // the row's end, or (capacity layout) its region's end
    if (a.history_lengths) olen = __ldg(a.history_lengths + b);
  }
  uint32_t app = 0;
  if (a.token_counts) {
    const int64_t* tc = a.token_counts + static_cast<int64_t>(b) * a.tc_stride + v0;
    if (a.vec_counts && v0 + E <= V) {
#pragma unroll
      for (int i = 0; i < E / 2; ++i) {
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
      sup = bytes_to_mask<E>(a.suppress + v0);
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
  clear_hist<NT, E>(sh);
  // suppress now: waiting for the logits here overlaps the offsets round trip
  // (otherwise the compiler may sink the logits load past the history phase)
#pragma unroll
  for (int j = 0; j < E; ++j)
    if ((sup >> j) & 1u) x[j] = NEG_SUPPRESS;

  int hist_len = 0;
  if (a.history) {
    if (a.history_lengths) o1 = row_end_in_region(o0, o1, olen);
    if (o0 < 0 || o1 < o0 || static_cast<int64_t>(o1) > a.history_len) {
      err |= Q3S_DEVERR_OFFSETS;
      o0 = o1 = 0;
    }
    hist_len = o1 - o0;
#pragma unroll
    for (int c = 0; c < E / 8; ++c) *reinterpret_cast<uint2*>(&sh.seen[v0 + 8 * c]) = make_uint2(0u, 0u);
    __syncthreads();
    // presence scatter (racing stores of the same byte need no atomics):
    // 16-byte loads over the aligned middle of the row's ids, scalar loads for
    // the ragged head [o0, mid0) and tail [mid1, o1); each thread issues up to
    // U loads before its first store, so the ids arrive in one round trip
    const int32_t* h = a.history;
    int mid0 = o0, mid1 = o0;
    if (a.vec_history) {
      mid0 = min(o1, (o0 + 3) & ~3);
      mid1 = mid0 + ((o1 - mid0) & ~3);
    }
    const int nhead = mid0 - o0;
    const int nrest = nhead + (o1 - mid1);
    const int nwork = nrest + (mid1 - mid0) / 4;  // scalar ids first, then 16-byte chunks
    constexpr int U = 8;
    for (int r = t; r < nwork; r += U * NT) {
      int4 ids[U];
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int rr = r + q * NT;
        ids[q] = make_int4(-1, -1, -1, -1);
        if (rr < nrest)
          ids[q].x = __ldg(h + (rr < nhead ? o0 + rr : mid1 + (rr - nhead)));
        else if (rr < nwork)
          ids[q] = __ldg(reinterpret_cast<const int4*>(h + mid0) + (rr - nrest));
      }
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int rr = r + q * NT;
        if (rr >= nwork) continue;
        const int nid = rr < nrest ? 1 : 4;
        const int idv[4] = {ids[q].x, ids[q].y, ids[q].z, ids[q].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (i >= nid) break;
          if (static_cast<unsigned>(idv[i]) < static_cast<unsigned>(V))
            sh.seen[idv[i]] = 1;
          else
            err |= Q3S_DEVERR_HISTORY_ID;
        }
      }
    }
    __syncthreads();
    app |= bytes_to_mask<E>(&sh.seen[v0]);
  }
  const int cur = a.cur_len ? __ldg(a.cur_len + b) : hist_len;
  const bool gate = a.eos_id >= 0 && a.eos_id < V && cur < min_new;

  // EOS gate (-inf is unchanged by the penalty that sample_core applies)
  if (gate && a.eos_id >= v0 && a.eos_id < v0 + E) {
#pragma unroll
    for (int j = 0; j < E; ++j)
      if (v0 + j == a.eos_id) x[j] = -INFINITY;
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
  const int id = sample_core<NT, E, MODE>(x, vmask, app & vmask, pen, V, c, sh, proc, flags, err);

  const bool owner = (id >= v0 && id < v0 + E) || (t == 0 && (id < 0 || id >= V));
  if (owner) {
    if (a.ids64) a.ids64[b] = id;
    if (a.ids32) a.ids32[b] = id;
    if (a.row_flags) a.row_flags[b] = flags;
  }
  if (a.counts_out) {
    int64_t* co = a.counts_out + static_cast<int64_t>(b) * a.co_stride;
    if (a.counts_out == a.token_counts && a.co_stride == a.tc_stride) {
      if (owner && id >= 0 && id < V) co[id] += 1;  // in-place: the row was read before any write
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

template <int NT, int E, bool BF16, int MODE>
__global__ void __launch_bounds__(NT) cp_frame_kernel(const CpArgs a) {
  __shared__ Scratch<NT, E> sh;
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

  clear_hist<NT, E>(sh);
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
            const int issued = g == 0 ? a.nbuf : a.nbuf - 1;  // items g .. g + issued - 1
            for (int h = g; h < min(g + issued, nitems); ++h)
              (void)mbar_wait_bounded(&bars[h % a.nbuf], static_cast<uint32_t>((h / a.nbuf) & 1));
          }
          return;
        }
        // every thread has passed this barrier after reading the previous
        // stage's slot: it takes the item nbuf - 1 stages ahead
        if (t == 0 && g > 0 && g - 1 + a.nbuf < nitems) issue(g - 1 + a.nbuf);
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
      } else {
        // every thread is done with the previous stage's shared state
        __syncthreads();
        load_logits<BF16, E>(a.logits,
                             static_cast<int64_t>(j) * a.stage_stride + static_cast<int64_t>(b) * a.row_stride, V, v0,
                             shift, false, x, vmask);
      }
      RowCfg c;
      c.mode = a.mode;
      c.greedy = (a.mode == Q3S_DRAW_ICDF) ? !(T > 0.0f) : (a.noise == nullptr);
      c.T = T;
      c.k = a.K;
      c.top_p = top_p;
      c.u = a.uniforms ? __ldg(a.uniforms + static_cast<int64_t>(b) * S + j) : 0.0f;
      c.noise = a.noise ? a.noise + static_cast<int64_t>(b) * a.noise_row_stride +
                              static_cast<int64_t>(j) * a.noise_stage_stride
                        : nullptr;
      int flags;
      uint32_t err = 0;
      const int id = sample_core<NT, E, MODE>(x, vmask, 0u, 1.0f, V, c, sh, nullptr, flags, err);
      if (id >= v0 && id < v0 + E) {  // the owner holds the complete flags
        a.ids_out[static_cast<int64_t>(b) * S + j] = id;
        if (a.row_flags) a.row_flags[static_cast<int64_t>(b) * S + j] = flags;
      }
      if (err && a.error_word) atomicOr(a.error_word, static_cast<int>(err));
      prev = id;
    }
  }
}

}  // namespace q3s

#include "q3s_cp.cuh"

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

// Threads per row and entries per thread for a vocabulary size: 8 entries per
// thread (one 16-byte bf16 load) up to V = 4096.
bool pick_shape(int V, int& nt, int& e) {
  if (V <= 512) { nt = 64; e = 8; }
  else if (V <= 1024) { nt = 128; e = 8; }
  else if (V <= 2048) { nt = 256; e = 8; }
  else if (V <= 3072) { nt = 384; e = 8; }
  else if (V <= 4096) { nt = 512; e = 8; }
  else if (V <= Q3S_MAX_VOCAB) { nt = 512; e = 16; }
  else return false;
  return true;
}

template <int NT, int E>
q3s_status launch_rows(const q3s::SampleArgs& a, bool bf16, cudaStream_t st) {
  const bool g = a.mode == Q3S_DRAW_GUMBEL;
  auto kern = bf16 ? (g ? q3s::sample_rows_kernel<NT, E, true, Q3S_DRAW_GUMBEL>
                        : q3s::sample_rows_kernel<NT, E, true, Q3S_DRAW_ICDF>)
                   : (g ? q3s::sample_rows_kernel<NT, E, false, Q3S_DRAW_GUMBEL>
                        : q3s::sample_rows_kernel<NT, E, false, Q3S_DRAW_ICDF>);
  const cudaError_t e = q3s::launch_maybe_pdl(kern, dim3(a.B), dim3(NT), 0, st, a.pdl, a);
  if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_sample launch failed: %s", cudaGetErrorString(e));
  return ok();
}

// Process-wide kernel policy (q3s_set_kernel_policy).
int g_policy = Q3S_POLICY_AUTO;

int device_sm_count() {
  // per-device cache; racing first readers store the same value
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// The widest cluster step_fused_kernel<NT> gets on this device: 16 CTAs
// (non-portable, opted in) where the device can place one, else the portable
// 8.  Per-device cache; racing first callers store the same value.
template <int NT>
int fused_cluster_max() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return q3s::FUSED_MAX_CTAS;
  int m = cache[dev].load(std::memory_order_relaxed);
  if (m == 0) {
    m = q3s::FUSED_MAX_CTAS;
    const auto kern = q3s::step_fused_kernel<NT>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t lc = {};
      lc.gridDim = dim3(q3s::FUSED_WIDE_CTAS);
      lc.blockDim = dim3(NT);
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = q3s::FUSED_WIDE_CTAS;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      lc.attrs = at;
      lc.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &lc) == cudaSuccess && n >= 1) m = q3s::FUSED_WIDE_CTAS;
    }
    (void)cudaGetLastError();  // a refused opt-in or query leaves the portable width
    cache[dev].store(m, std::memory_order_relaxed);
  }
  return m;
}

template <int NT>
cudaError_t launch_step_fused(const q3s::StepArgs& a, int rpt, int n_cta, cudaStream_t st) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(static_cast<unsigned>(n_cta));
  lc.blockDim = dim3(NT);
  lc.dynamicSmemBytes = 0;
  lc.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = static_cast<unsigned>(n_cta);
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, q3s::step_fused_kernel<NT>, a, rpt);
}

template <int NT, int E, bool BF16, int MODE>
q3s_status launch_cp_t(const q3s::CpArgs& a, cudaStream_t st) {
  const size_t dyn = a.bulk ? static_cast<size_t>(a.nbuf) * a.row_bytes : 0;
  auto kern = q3s::cp_frame_kernel<NT, E, BF16, MODE>;
  if (dyn > 0) {
    // static + dynamic shared memory may pass the 48 KB default: opt in.
    // Idempotent per (kernel, device); the value only ever grows.
    static std::atomic<int> granted[64];
    int dev = 0;
    cudaGetDevice(&dev);
    const bool known = dev >= 0 && dev < 64;
    if (!known || granted[dev].load(std::memory_order_acquire) < static_cast<int>(dyn)) {
      const cudaError_t e =
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn));
      if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_sample_cp_frame smem attribute: %s", cudaGetErrorString(e));
      if (known) {
        // keep the largest grant: a racing smaller one must not lower it
        int cur = granted[dev].load(std::memory_order_relaxed);
        while (cur < static_cast<int>(dyn) &&
               !granted[dev].compare_exchange_weak(cur, static_cast<int>(dyn), std::memory_order_release)) {
        }
      }
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

template <int NT, int E>
q3s_status launch_cp(const q3s::CpArgs& a, bool bf16, cudaStream_t st) {
  if (a.mode == Q3S_DRAW_GUMBEL)
    return bf16 ? launch_cp_t<NT, E, true, Q3S_DRAW_GUMBEL>(a, st) : launch_cp_t<NT, E, false, Q3S_DRAW_GUMBEL>(a, st);
  return bf16 ? launch_cp_t<NT, E, true, Q3S_DRAW_ICDF>(a, st) : launch_cp_t<NT, E, false, Q3S_DRAW_ICDF>(a, st);
}

}  // namespace

namespace q3s {

q3s_status report(q3s_status s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return s;
}

int sm_count() { return device_sm_count(); }

}  // namespace q3s

extern "C" {

const char* q3s_last_error_string(void) { return g_last_error; }

int32_t q3s_abi_version(void) { return Q3S_ABI_VERSION; }

int32_t q3s_set_kernel_policy(int32_t policy) {
  if (policy < Q3S_POLICY_AUTO || policy > Q3S_POLICY_LEAN) return -1;
  return __atomic_exchange_n(&g_policy, policy, __ATOMIC_RELAXED);
}

q3s_status q3s_philox_rows(uint64_t seed, uint32_t step, const int64_t* row_keys, int64_t row0, int32_t rows,
                           int32_t cols, int32_t kind, float* out, int64_t out_row_stride, void* stream) {
  if (rows < 0 || cols < 0) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_philox_rows: rows=%d cols=%d", rows, cols);
  if (kind != Q3S_PHILOX_UNIFORM && kind != Q3S_PHILOX_GUMBEL)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_philox_rows: unknown kind %d", kind);
  if (rows == 0 || cols == 0) return ok();
  if (!out) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_philox_rows: out is NULL");
  if (out_row_stride < cols)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_philox_rows: out_row_stride %lld < cols %d",
                static_cast<long long>(out_row_stride), cols);
  const int64_t threads = static_cast<int64_t>(rows) * ((cols + 3) / 4);
  const int nt = 256;
  const int64_t grid = (threads + nt - 1) / nt;
  if (grid > 0x7fffffffLL) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_philox_rows: too many rows x columns");
  q3s::philox_rows_kernel<<<static_cast<unsigned>(grid), nt, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32), step, row_keys, row0, rows, cols, kind, out,
      out_row_stride);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_philox_rows launch failed: %s", cudaGetErrorString(e));
  return ok();
}

q3s_status q3s_philox_seeds(const uint64_t* row_seeds, uint32_t step, uint32_t stage, int32_t rows, int32_t cols,
                            int32_t kind, float* out, int64_t out_row_stride, void* stream) {
  if (rows < 0 || cols < 0) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_philox_seeds: rows=%d cols=%d", rows, cols);
  if (kind != Q3S_PHILOX_UNIFORM && kind != Q3S_PHILOX_GUMBEL)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_philox_seeds: unknown kind %d", kind);
  if (rows == 0 || cols == 0) return ok();
  if (!out || !row_seeds) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_philox_seeds: out / row_seeds is NULL");
  if (out_row_stride < cols)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_philox_seeds: out_row_stride %lld < cols %d",
                static_cast<long long>(out_row_stride), cols);
  const int64_t threads = static_cast<int64_t>(rows) * ((cols + 3) / 4);
  const int nt = 256;
  const int64_t grid = (threads + nt - 1) / nt;
  if (grid > 0x7fffffffLL) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_philox_seeds: too many rows x columns");
  q3s::philox_seeds_kernel<<<static_cast<unsigned>(grid), nt, 0, static_cast<cudaStream_t>(stream)>>>(
      row_seeds, step, stage, rows, cols, kind, out, out_row_stride);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_philox_seeds launch failed: %s", cudaGetErrorString(e));
  return ok();
}

uint32_t q3s_desc_size(int32_t which) {
  if (which == 0) return static_cast<uint32_t>(sizeof(q3s_sample_desc));
  if (which == 1) return static_cast<uint32_t>(sizeof(q3s_cp_frame_desc));
  if (which == 2) return static_cast<uint32_t>(sizeof(q3s_step_desc));
  if (which == 3) return static_cast<uint32_t>(sizeof(q3s_head_desc));
  return 0;
}

q3s_status q3s_step_update(const q3s_step_desc* d, void* stream) {
  if (!d) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_step_update: desc is NULL");
  if (d->struct_size != sizeof(q3s_step_desc))
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_step_update: struct_size %u != %u (ABI mismatch)", d->struct_size,
                static_cast<unsigned>(sizeof(q3s_step_desc)));
  const int B = d->batch;
  if (B < 0 || B >= (1 << 23)) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_step_update: batch %d outside [0, 2^23)", B);
  if (B == 0) return ok();
  if ((d->ids_i64 == nullptr) == (d->ids_i32 == nullptr))
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_step_update: give exactly one of ids_i64 / ids_i32");
  q3s::StepArgs a{};
  a.batch = B;
  a.eos_id = d->eos_id;
  a.ids_i64 = d->ids_i64;
  a.ids_i32 = d->ids_i32;
  // threshold normalisation of EngineLoop.__init__ (engine/backend/engine_loop.py:372-387)
  a.abort = std::max(0, d->abort_frames);
  const int suspect = std::max(0, d->suspect_frames), emergency = std::max(0, d->emergency_frames);
  a.suspect = (suspect > 0 && a.abort > 0) ? std::min(suspect, a.abort) : 0;
  a.emergency = (emergency > 0 && a.abort > 0) ? std::max(emergency, a.abort) : 0;
  const double ratio = d->min_audio_text_ratio;
  if (ratio != ratio) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_step_update: min_audio_text_ratio is NaN");
  a.min_ratio = ratio > 0.0 ? ratio : 0.0;
  if (a.abort > 0) {
    if (!d->loop_token || !d->loop_run || !d->loop_max_run || !d->loop_suspect_count || !d->loop_recovery_count)
      return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_step_update: the loop guard is on but a guard state array is NULL");
    if (a.min_ratio > 0.0 && (!d->frame_idx || !d->decode_start_frame || !d->text_tokens_consumed || !d->input_complete))
      return fail(Q3S_ERR_INVALID_ARGUMENT,
                  "q3s_step_update: the progress gate needs frame_idx, decode_start_frame, text_tokens_consumed and "
                  "input_complete");
  }
  if (d->event_list && !d->event_count)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_step_update: event_list needs event_count");
  if (d->event_count && !d->events)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_step_update: event_list / event_count are compacted from events");
  const bool in_place = d->history_lengths != nullptr;
  const bool append = d->history_out != nullptr && !in_place;
  if (in_place) {
    if (!d->history_out || static_cast<const void*>(d->history_out) != static_cast<const void*>(d->history) ||
        !d->offsets)
      return fail(Q3S_ERR_INVALID_ARGUMENT,
                  "q3s_step_update: the in-place append (history_lengths) needs offsets and history_out == history");
    if (d->history_out_capacity < 0 || d->history_out_capacity > INT32_MAX)
      return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_step_update: history_out_capacity %lld outside [0, 2^31)",
                  static_cast<long long>(d->history_out_capacity));
  }
  if (append) {
    if ((!d->history && d->history_len > 0) || !d->offsets || !d->offsets_out)
      return fail(Q3S_ERR_INVALID_ARGUMENT,
                  "q3s_step_update: the history append needs history (unless empty), offsets and offsets_out");
    if (d->history_len < 0 || d->history_out_capacity < d->history_len + B || d->history_out_capacity > INT32_MAX)
      return fail(Q3S_ERR_INVALID_ARGUMENT,
                  "q3s_step_update: history_out_capacity %lld must lie in [history_len + batch, 2^31) (history_len %lld)",
                  static_cast<long long>(d->history_out_capacity), static_cast<long long>(d->history_len));
    const uintptr_t i0 = reinterpret_cast<uintptr_t>(d->history), i1 = i0 + 4 * static_cast<uintptr_t>(d->history_len);
    const uintptr_t o0 = reinterpret_cast<uintptr_t>(d->history_out),
                    o1 = o0 + 4 * static_cast<uintptr_t>(d->history_out_capacity);
    if (i0 < o1 && o0 < i1)
      return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_step_update: history_out overlaps history (rows shift right)");
    const uintptr_t f0 = reinterpret_cast<uintptr_t>(d->offsets), f1 = f0 + 4 * static_cast<uintptr_t>(B + 1);
    const uintptr_t g0 = reinterpret_cast<uintptr_t>(d->offsets_out), g1 = g0 + 4 * static_cast<uintptr_t>(B + 1);
    if (f0 < g1 && g0 < f1) return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_step_update: offsets_out overlaps offsets");
  }
  a.history = d->history;
  a.offsets = d->offsets;
  a.history_len = d->history_len;
  a.history_out = d->history_out;
  a.offsets_out = d->offsets_out;
  a.history_out_capacity = d->history_out_capacity;
  a.loop_token = d->loop_token;
  a.loop_run = d->loop_run;
  a.loop_max_run = d->loop_max_run;
  a.loop_suspect_count = d->loop_suspect_count;
  a.loop_recovery_count = d->loop_recovery_count;
  a.frame_idx = d->frame_idx;
  a.decode_start_frame = d->decode_start_frame;
  a.text_tokens = d->text_tokens_consumed;
  a.input_complete = d->input_complete;
  a.events = d->events;
  a.event_run = d->event_run;
  a.event_list = d->event_list;
  a.event_count = d->event_count;
  a.error_word = d->error_word;
  a.history_lengths = d->history_lengths;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  // One cluster: the narrowest CTA (128 .. 1024 threads) that covers the
  // batch with a row per thread in 16 CTAs, so that the rows spread over as
  // many SMs as the cluster allows (the launch is bound by the rows each SM
  // serves); past 16 x 1024 rows, up to 4 rows a thread.
  int fused_nt = 128;
  while (fused_nt < 1024 && B > q3s::FUSED_WIDE_CTAS * fused_nt) fused_nt *= 2;
  const int max_cta = fused_nt == 128   ? fused_cluster_max<128>()
                      : fused_nt == 256 ? fused_cluster_max<256>()
                      : fused_nt == 512 ? fused_cluster_max<512>()
                                        : fused_cluster_max<1024>();
  const int fused_rows = max_cta * fused_nt;
  const bool fused = !append && B <= fused_rows * q3s::FUSED_MAX_RPT;
  cudaError_t e = cudaSuccess;
  if (fused) {
    // rows per thread first, so that every CTA of the cluster has work
    const int rpt = (B + fused_rows - 1) / fused_rows;
    const int n_cta = (B + fused_nt * rpt - 1) / (fused_nt * rpt);
    e = fused_nt == 128   ? launch_step_fused<128>(a, rpt, n_cta, st)
        : fused_nt == 256 ? launch_step_fused<256>(a, rpt, n_cta, st)
        : fused_nt == 512 ? launch_step_fused<512>(a, rpt, n_cta, st)
                          : launch_step_fused<1024>(a, rpt, n_cta, st);
  } else if (append) {
    q3s::step_rows_kernel<<<static_cast<unsigned>(B), q3s::APPEND_NT, 0, st>>>(a);
  } else {
    q3s::step_lite_kernel<<<static_cast<unsigned>((B + q3s::LITE_NT - 1) / q3s::LITE_NT), q3s::LITE_NT, 0, st>>>(a);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e == cudaSuccess && !fused && (d->event_list || d->event_count)) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(1);
    lc.blockDim = dim3(q3s::COMPACT_NT);
    lc.dynamicSmemBytes = 0;
    lc.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    e = cudaLaunchKernelEx(&lc, q3s::step_compact_kernel, a);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_step_update launch failed: %s", cudaGetErrorString(e));
  return ok();
}

q3s_status q3s_sample(const q3s_sample_desc* d, void* stream) {
  return q3s::sample_impl(d, static_cast<cudaStream_t>(stream), false);
}

}  // extern "C"

namespace q3s {

q3s_status sample_impl(const q3s_sample_desc* d, cudaStream_t stream, bool pdl) {
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
  if (d->history_lengths && !d->history)
    return fail(Q3S_ERR_INVALID_ARGUMENT, "q3s_sample: history_lengths (capacity layout) needs history and offsets");
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
  int nt = 0, ne = 0;
  if (!pick_shape(V, nt, ne)) return fail(Q3S_ERR_UNSUPPORTED, "q3s_sample: vocab %d too large", V);
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
  a.history_lengths = d->history_lengths;
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
  a.vec_history = d->history && aligned16(d->history);
  a.pdl = pdl;

  cudaStream_t st = stream;
  const bool warp_ok = a.mode == Q3S_DRAW_ICDF && !a.token_counts && !a.col_shift &&
                       !a.counts_out && V % 8 == 0 && V > 1024 && V <= 3072 && a.vec_logits &&
                       (!a.suppress || a.vec_suppress);
  const int policy = __atomic_load_n(&g_policy, __ATOMIC_RELAXED);
  // the register-resident kernel: the same steps as the shared-memory one,
  // any vocabulary up to 3072 that is a multiple of 8
  const bool lean_ok = a.mode == Q3S_DRAW_ICDF && !a.token_counts && !a.col_shift && !a.counts_out &&
                       V % 8 == 0 && V <= 3072 && (!a.suppress || a.vec_suppress);
  // AUTO: the register-resident kernel beyond two rows per SM, where it is
  // the fastest measured (B200, configs 3 and 4); the shared-memory row
  // kernel below that (latency-bound batches)
  const bool lean_auto = policy == Q3S_POLICY_AUTO && a.B > 2 * device_sm_count();
  if (lean_ok && (policy == Q3S_POLICY_LEAN || lean_auto)) {
    const cudaError_t e = q3s::launch_lean_rows(a, bf16, st);
    if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_sample lean launch failed: %s", cudaGetErrorString(e));
    return ok();
  }
  if (warp_ok && policy != Q3S_POLICY_CTA && policy != Q3S_POLICY_LEAN) {
    int warps = q3s::smem_warps_for(a.B, device_sm_count());
    if (policy == Q3S_POLICY_ROW_W1) warps = 1;
    if (policy == Q3S_POLICY_ROW_W2) warps = 2;
    if (policy == Q3S_POLICY_ROW_W4) warps = 4;
    if (policy == Q3S_POLICY_ROW_W8) warps = 8;
    if (policy == Q3S_POLICY_ROW_WMAX) warps = 0;
    const cudaError_t e = q3s::launch_warp_rows(a, bf16, st, warps);
    if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_sample warp launch failed: %s", cudaGetErrorString(e));
    return ok();
  }
  if (ne == 16) return launch_rows<512, 16>(a, bf16, st);
  switch (nt) {
    case 64: return launch_rows<64, 8>(a, bf16, st);
    case 128: return launch_rows<128, 8>(a, bf16, st);
    case 256: return launch_rows<256, 8>(a, bf16, st);
    case 384: return launch_rows<384, 8>(a, bf16, st);
    default: return launch_rows<512, 8>(a, bf16, st);
  }
}

}  // namespace q3s

extern "C" {

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
  int nt = 0, ne = 0;
  if (!pick_shape(V, nt, ne)) return fail(Q3S_ERR_UNSUPPORTED, "q3s_sample_cp_frame: vocab %d too large", V);
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
  // ring of stage rows in flight: up to 64 KB, 2..16 slots -- a whole
  // 15-stage frame of 4 KB rows (V = 2048 bf16), so that every stage row of
  // a CTA's first row is requested at once and later stages never wait
  a.nbuf = a.bulk ? std::max(2, std::min(q3s::MAX_NBUF, static_cast<int>((64u * 1024u) / a.row_bytes))) : 0;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Gumbel frames (the engine graph's stages) with rows of at most 2048
  // entries and K <= 256: the lean stage chain of q3s_cp.cuh; the CTA policy
  // keeps the general CTA-per-row kernel
  const int policy = __atomic_load_n(&g_policy, __ATOMIC_RELAXED);
  if (a.mode == Q3S_DRAW_GUMBEL && a.noise && a.bulk && V <= q3s::CPF_NT * q3s::CPF_E && a.K <= q3s::CPF_CAP &&
      policy != Q3S_POLICY_CTA) {
    const size_t dyn = static_cast<size_t>(a.nbuf) * a.row_bytes;
    // one CTA per SM holds the whole register budget of the stage (rows that
    // fit on the SMs at once); with more rows than SMs two CTAs share an SM
    // (fewer registers each), so that two rows' stage chains interleave
    const bool wide = a.B > device_sm_count();
    auto kern = bf16 ? (wide ? q3s::cp_fast_kernel<true, 2> : q3s::cp_fast_kernel<true, 1>)
                     : (wide ? q3s::cp_fast_kernel<false, 2> : q3s::cp_fast_kernel<false, 1>);
    const int ki = (bf16 ? 2 : 0) + (wide ? 1 : 0);
    {
      // the ring may pass the 48 KB default: opt in (idempotent per kernel
      // and device; the value only ever grows)
      static std::atomic<int> granted[4][64];
      int dev = 0;
      cudaGetDevice(&dev);
      const bool known = dev >= 0 && dev < 64;
      if (!known || granted[ki][dev].load(std::memory_order_acquire) < static_cast<int>(dyn)) {
        const cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn));
        if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_sample_cp_frame smem attribute: %s", cudaGetErrorString(e));
        if (known) {
          int cur = granted[ki][dev].load(std::memory_order_relaxed);
          while (cur < static_cast<int>(dyn) &&
                 !granted[ki][dev].compare_exchange_weak(cur, static_cast<int>(dyn), std::memory_order_release)) {
          }
        }
      }
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, q3s::CPF_NT, dyn) != cudaSuccess || per_sm <= 0)
      per_sm = 1;
    const int grid = std::min(a.B, device_sm_count() * per_sm);
    kern<<<grid, q3s::CPF_NT, dyn, st>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(Q3S_ERR_CUDA, "q3s_sample_cp_frame launch failed: %s", cudaGetErrorString(e));
    return ok();
  }
  if (ne == 16) return launch_cp<512, 16>(a, bf16, st);
  switch (nt) {
    case 64: return launch_cp<64, 8>(a, bf16, st);
    case 128: return launch_cp<128, 8>(a, bf16, st);
    case 256: return launch_cp<256, 8>(a, bf16, st);
    case 384: return launch_cp<384, 8>(a, bf16, st);
    default: return launch_cp<512, 8>(a, bf16, st);
  }
}

}  // extern "C"
