// q3s_step.cuh -- the per-step codec-0 epilogue on the device (q3s_step_update).
//
// What it replaces (file:line in X-Square-Robot/Qwen3TTS-Streaming):
//   EOS detection: the host reads every row's codebook-0 id back and compares
//       it with the codec EOS id          engine/backend/executor.py:532-546
//   frame counter: frame_idx += 1 on non-EOS rows, before the guard
//                                         engine/backend/engine_loop.py:2749-2750
//   two-stage token loop guard: run / recovery / suspect bookkeeping, the
//       generation-progress gate, deferred / confirmed / emergency decisions
//                                         engine/backend/engine_loop.py:2863-3080
//   history append: the packed-history form of token_counts + one_hot(id)
//                                         scripts/export/talker_unified_modules.py:421-422
//
// Launches on the caller's stream:
//   step_fused_kernel    (capacity layout or no append, B <= 65536) ONE
//                        launch, a cluster of <= 16 CTAs of 128 .. 1024
//                        threads: one thread per row
//                        (up to 4) runs the guard and the in-place append
//                        (history[offsets[b] + len[b]] = ids[b], len[b] += 1),
//                        then the CTAs place the ordered event list through
//                        distributed shared memory;
//   step_lite_kernel     the same per-row work for larger batches, followed
//                        by step_compact_kernel;
//   step_rows_kernel     (packed layout, copied append) CTA b: thread 0 runs row b's guard (events[b],
//                        event_run[b], state) while the CTA copies history row
//                        b to its shifted place in the output
//                        (offsets_out[b] = offsets[b] + b) and appends ids[b];
//                        register-light so 8 CTAs stay resident per SM;
//   step_compact_kernel  one CTA: ordered compaction of events[] into
//                        (row << 8) | bits entries and the count (only when
//                        the caller asks for the list or the count); a
//                        programmatic dependent launch, so its launch overlaps
//                        the row kernel and griddepcontrol.wait orders it.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q3s_device.cuh"
#include "q3s_sampler.h"

namespace q3s {

struct StepArgs {
  int batch;
  int eos_id;
  const int64_t* ids_i64;
  const int32_t* ids_i32;
  const int32_t* history;
  const int32_t* offsets;
  int64_t history_len;
  int32_t* history_out;
  int32_t* offsets_out;
  int64_t history_out_capacity;
  int suspect, abort, emergency;  // normalised
  double min_ratio;               // clamped at 0
  int32_t* loop_token;
  int32_t* loop_run;
  int32_t* loop_max_run;
  int32_t* loop_suspect_count;
  int32_t* loop_recovery_count;
  int32_t* frame_idx;
  const int32_t* decode_start_frame;
  const int32_t* text_tokens;
  const uint8_t* input_complete;
  int32_t* events;
  int32_t* event_run;
  int32_t* event_list;
  int32_t* event_count;
  int32_t* error_word;
  int32_t* history_lengths;       // capacity layout: in-place append into history_out
};

__device__ __forceinline__ int64_t step_id(const StepArgs& a, int b) {
  return a.ids_i64 ? a.ids_i64[b] : static_cast<int64_t>(a.ids_i32[b]);
}

// Per-row inputs of the guard.
struct GuardRow {
  int64_t id;
  int frame, token, run, max_run, suspects, recoveries, start, text;
  bool complete;
};

__device__ __forceinline__ void guard_load(const StepArgs& a, int b, GuardRow& r) {
  r = GuardRow{};
  r.id = step_id(a, b);
  r.frame = a.frame_idx ? a.frame_idx[b] : 0;
  if (a.abort > 0) {
    r.token = a.loop_token[b];
    r.run = a.loop_run[b];
    r.max_run = a.loop_max_run[b];
    r.suspects = a.loop_suspect_count[b];
    r.recoveries = a.loop_recovery_count[b];
    if (a.min_ratio > 0.0) {
      r.start = a.decode_start_frame[b];
      r.text = a.text_tokens[b];
      r.complete = a.input_complete[b] != 0;
    }
  }
}

// The guard of one row (state written back); returns its event bits.
__device__ __forceinline__ int guard_apply(const StepArgs& a, int b, GuardRow& r, int& ev_run) {
  ev_run = 0;
  if (r.id == a.eos_id) return Q3S_EVT_EOS;  // segment ends; no counter, no guard
  r.frame += 1;
  if (a.frame_idx) a.frame_idx[b] = r.frame;
  if (a.abort <= 0) return 0;
  int bits = 0;
  if (r.id == static_cast<int64_t>(r.token)) {
    r.run += 1;
  } else {
    if (a.suspect > 0 && r.run >= a.suspect) {
      r.recoveries += 1;
      bits |= Q3S_EVT_RECOVERED;
      ev_run = r.run;
    }
    r.token = static_cast<int>(r.id);
    r.run = 1;
  }
  r.max_run = max(r.max_run, r.run);
  if (a.suspect > 0 && r.run == a.suspect) {
    r.suspects += 1;
    bits |= Q3S_EVT_SUSPECT;
  }
  bool ready = true;
  if (a.min_ratio > 0.0) {
    const int64_t steps = max(static_cast<int64_t>(0), static_cast<int64_t>(r.frame) - r.start);
    const int text = max(0, r.text);
    // Python's int / int: one correctly rounded double division (both exact).
    const double ratio = text > 0 ? static_cast<double>(steps) / static_cast<double>(text) : 0.0;
    ready = r.complete && (text == 0 || ratio >= a.min_ratio);
  }
  if (r.run == a.abort && !ready) bits |= Q3S_EVT_DEFERRED;
  if (r.run >= a.abort && ready) {
    bits |= Q3S_EVT_ABORT_PROGRESS;
    ev_run = r.run;
  } else if (a.emergency > 0 && r.run >= a.emergency) {
    bits |= Q3S_EVT_ABORT_EMERGENCY;
    ev_run = r.run;
  }
  a.loop_token[b] = r.token;
  a.loop_run[b] = r.run;
  a.loop_max_run[b] = r.max_run;
  a.loop_suspect_count[b] = r.suspects;
  a.loop_recovery_count[b] = r.recoveries;
  return bits;
}

// History row b -> history_out[offsets[b] + b ...], then ids[b]; thread 0
// runs row b's guard meanwhile.  One CTA of APPEND_NT threads per row,
// APPEND_U loads in flight per thread; held to 32 registers so 8 CTAs (2048
// threads) stay resident per SM and enough rows are in flight to cover DRAM
// latency.  Without the append the CTA is one warp and only the guard runs.
constexpr int APPEND_NT = 256;
constexpr int APPEND_U = 8;

__global__ void __launch_bounds__(APPEND_NT, 8) step_rows_kernel(const StepArgs a) {
  // let the compaction kernel (a programmatic dependent launch) be scheduled
  // now; it still waits for this whole grid before reading events
  asm volatile("griddepcontrol.launch_dependents;");
  const int b = blockIdx.x;
  if (threadIdx.x == 0) {
    GuardRow r;
    guard_load(a, b, r);
    int ev_run;
    const int bits = guard_apply(a, b, r, ev_run);
    if (a.events) a.events[b] = bits;
    if (a.event_run) a.event_run[b] = ev_run;
  }
  if (!a.history_out) return;
  const int64_t s = a.offsets[b], e = a.offsets[b + 1];
  const int64_t d = s + b, n = e - s;
  if (threadIdx.x == 0) {
    a.offsets_out[b] = static_cast<int32_t>(d);
    if (b == a.batch - 1) a.offsets_out[a.batch] = static_cast<int32_t>(e + a.batch);
  }
  const bool ok = s >= 0 && n >= 0 && e <= a.history_len && d + n + 1 <= a.history_out_capacity;
  if (!ok) {
    if (threadIdx.x == 0 && a.error_word) atomicOr(a.error_word, Q3S_DEVERR_OFFSETS);
    return;
  }
  const int32_t* src = a.history + s;
  int32_t* dst = a.history_out + d;
  const int n32 = static_cast<int>(n);  // n <= history_len < 2^31 (checked on the host)
  for (int i0 = 0; i0 < n32; i0 += APPEND_U * APPEND_NT) {
    int32_t v[APPEND_U];
#pragma unroll
    for (int u = 0; u < APPEND_U; ++u) {
      const int i = i0 + u * APPEND_NT + static_cast<int>(threadIdx.x);
      if (i < n32) v[u] = __ldcs(src + i);
    }
#pragma unroll
    for (int u = 0; u < APPEND_U; ++u) {
      const int i = i0 + u * APPEND_NT + static_cast<int>(threadIdx.x);
      if (i < n32) dst[i] = v[u];
    }
  }
  if (threadIdx.x == 0) dst[n] = static_cast<int32_t>(step_id(a, b));
}

// Row b of the lite form: the guard, and with the capacity layout the
// in-place append of ids[b] at the end of row b inside its region
// [offsets[b], offsets[b+1]) of history_out.  A full region gets nothing (and
// Q3S_DEVERR_HISTORY_FULL), an inconsistent one Q3S_DEVERR_OFFSETS.  Returns
// the row's event bits.
__device__ __forceinline__ int lite_row(const StepArgs& a, int b) {
  GuardRow r;
  guard_load(a, b, r);
  // the row's region is read with the guard inputs, before any store, so all
  // of the row's loads share one trip to memory
  int64_t s = 0, e = 0;
  int len = 0;
  if (a.history_lengths) {
    s = a.offsets[b];
    e = a.offsets[b + 1];
    len = a.history_lengths[b];
  }
  int ev_run;
  const int bits = guard_apply(a, b, r, ev_run);
  if (a.events) a.events[b] = bits;
  if (a.event_run) a.event_run[b] = ev_run;
  if (!a.history_lengths) return bits;
  if (s < 0 || e < s || e > a.history_out_capacity || len < 0 || s + len > e) {
    if (a.error_word) atomicOr(a.error_word, Q3S_DEVERR_OFFSETS);
  } else if (s + len == e) {
    if (a.error_word) atomicOr(a.error_word, Q3S_DEVERR_HISTORY_FULL);
  } else {
    a.history_out[s + len] = static_cast<int32_t>(r.id);
    a.history_lengths[b] = len + 1;
  }
  return bits;
}

// One thread per row, followed by step_compact_kernel (rows beyond what one
// cluster of step_fused_kernel covers).
constexpr int LITE_NT = 128;

__global__ void __launch_bounds__(LITE_NT) step_lite_kernel(const StepArgs a) {
  asm volatile("griddepcontrol.launch_dependents;");
  const int b = static_cast<int>(blockIdx.x) * LITE_NT + static_cast<int>(threadIdx.x);
  if (b >= a.batch) return;
  lite_row(a, b);
}

// The lite form and the ordered event list in ONE launch: a cluster of up to
// FUSED_WIDE_CTAS CTAs of NT threads, thread t of CTA c taking rows
// (c * NT + t) * rpt ... + rpt - 1, so thread order is row order.  Each CTA
// scans its per-thread event counts and sends its total to slot c of every
// CTA of the cluster with st.async, which completes on the receiving CTA's
// mbarrier (4 bytes from each CTA expected); each CTA then adds up its own
// slots (the totals of the CTAs before it, and of all) and writes its entries
// of event_list; CTA 0 writes event_count.  No thread fences its global
// stores and no CTA waits for the others to finish: the only cluster barrier
// (every CTA has started and initialised its mbarrier before any st.async
// reaches it) is arrived at entry and waited on after the row work.  The
// mbarrier wait is bounded; if it gives up the CTA sets
// Q3S_DEVERR_WAIT_TIMEOUT and writes no entries.  (Every CTA sends its totals
// unconditionally right after the cluster barrier, with no wait in between,
// so a late send, not a missing one, is the only way to reach that branch.)
// No global scratch, no second launch.
constexpr int FUSED_MAX_CTAS = 8;    // portable cluster size
constexpr int FUSED_WIDE_CTAS = 16;  // non-portable, where the device grants it
constexpr int FUSED_MAX_RPT = 4;

// st.async of one int32 into CTA `rank`'s copy of `slot`, completing 4 bytes
// on that CTA's copy of `bar`.
__device__ __forceinline__ void step_send_total(int* slot, uint64_t* bar, unsigned rank, int v) {
  unsigned rs, rb;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rs) : "r"(smem_u32(slot)), "r"(rank));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rb) : "r"(smem_u32(bar)), "r"(rank));
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(rs), "r"(v),
               "r"(rb)
               : "memory");
}

template <int NT>
__global__ void __launch_bounds__(NT, 1) step_fused_kernel(const StepArgs a, int rpt) {
  __shared__ int warp_tot[NT / 32];
  __shared__ int cta_tot[FUSED_WIDE_CTAS];  // slot c: the event count of CTA c
  __shared__ __align__(8) uint64_t tot_bar;
  const bool want_list = a.event_list || a.event_count;  // uniform over the grid
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned me = blockIdx.x, n_cta = gridDim.x;
  if (want_list) {
    if (tid == 0) {
      mbar_init(&tot_bar, 1);
      mbar_expect_tx(&tot_bar, 4u * n_cta);  // the one arrival; the bytes may land before or after it
      fence_mbar_init();
    }
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  }
  const int b0 = (static_cast<int>(me) * NT + tid) * rpt;
  uint32_t evp = 0;  // the event bits (< 2^8) of row b0 + k in byte k
  int c = 0;
#pragma unroll
  for (int k = 0; k < FUSED_MAX_RPT; ++k) {
    const int bits = k < rpt && b0 + k < a.batch ? lite_row(a, b0 + k) : 0;
    evp |= static_cast<uint32_t>(bits) << (8 * k);
    c += bits != 0;
  }
  if (!want_list) return;
  int incl = c;  // inclusive warp scan of the per-thread counts
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int pre = incl - c, tot = 0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) {
    const int t = warp_tot[w];
    pre += w < warp ? t : 0;
    tot += t;
  }
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA has started
  if (tid < static_cast<int>(n_cta)) step_send_total(&cta_tot[me], &tot_bar, static_cast<unsigned>(tid), tot);
  if (!mbar_wait_bounded(&tot_bar, 0)) {
    if (tid == 0 && a.error_word) atomicOr(a.error_word, Q3S_DEVERR_WAIT_TIMEOUT);
    return;
  }
  int base = 0, all = 0;
  for (unsigned j = 0; j < n_cta; ++j) {
    const int t = cta_tot[j];
    base += j < me ? t : 0;
    all += t;
  }
  pre += base;
  if (a.event_list) {
#pragma unroll
    for (int k = 0; k < FUSED_MAX_RPT; ++k) {
      const int bits = static_cast<int>((evp >> (8 * k)) & 0xFFu);
      if (bits) a.event_list[pre++] = ((b0 + k) << 8) | bits;
    }
  }
  if (me == 0 && tid == 0 && a.event_count) *a.event_count = all;
}

// Ordered compaction of events[0, B) into event_list ((row << 8) | bits for
// rows with any bit, ascending) and event_count.  One CTA: thread t takes
// COMPACT_RPT consecutive rows of each chunk, so thread order is row order and
// one block scan of per-thread counts places every entry.
constexpr int COMPACT_NT = 1024;
constexpr int COMPACT_RPT = 4;

__global__ void __launch_bounds__(COMPACT_NT) step_compact_kernel(const StepArgs a) {
  // launched as a programmatic dependent of step_rows_kernel: wait until that
  // grid has completed and its writes (events) are visible
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ int warp_tot[COMPACT_NT / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int base = 0;
  for (int r0 = 0; r0 < a.batch; r0 += COMPACT_NT * COMPACT_RPT) {
    const int b0 = r0 + tid * COMPACT_RPT;
    int ev[COMPACT_RPT];
    int c = 0;
#pragma unroll
    for (int k = 0; k < COMPACT_RPT; ++k) {
      ev[k] = b0 + k < a.batch ? a.events[b0 + k] : 0;
      c += ev[k] != 0;
    }
    int incl = c;  // inclusive warp scan of the per-thread counts
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int pre = base + incl - c, tot = 0;
    for (int w = 0; w < COMPACT_NT / 32; ++w) {
      const int t = warp_tot[w];
      pre += w < warp ? t : 0;
      tot += t;
    }
    if (a.event_list) {
#pragma unroll
      for (int k = 0; k < COMPACT_RPT; ++k)
        if (ev[k]) a.event_list[pre++] = ((b0 + k) << 8) | ev[k];
    }
    base += tot;
    __syncthreads();  // warp_tot is rewritten by the next chunk
  }
  if (tid == 0 && a.event_count) *a.event_count = base;
}

}  // namespace q3s
