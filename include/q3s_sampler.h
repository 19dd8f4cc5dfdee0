/*
 * q3s_sampler.h -- C ABI of the B200 (sm_100a) codec-token sampler.
 *
 * One call samples one token per row for a batch of streams: the talker's
 * codebook-0 step, or one / all fifteen code-predictor stages.  The reference
 * (X-Square-Robot/Qwen3TTS-Streaming) has no standalone sampler API; its
 * sampler is a sub-graph of the fused TensorRT decode engine, fed by name
 * through TRTEngine.infer (engine/backend/executor.py:323-453) with the inputs
 * built in Executor._build_fused_inputs (engine/backend/executor.py:3376-3475).
 * The entry points below replace those sub-graphs:
 *
 *   q3s_sample           scripts/export/talker_unified_modules.py:407-422
 *                        (codebook 0: suppress -> repetition penalty ->
 *                        top-k 50 -> /T -> +Gumbel -> argmax -> one-hot count
 *                        update), scripts/export/utils.py:1178-1193
 *                        (CodePredictorUnrolled._select_token, one stage), and
 *                        tools/validation/prefill_compare.py:383-399
 *                        (_sample_token: the HF processor chain + multinomial,
 *                        here an inverse-CDF draw from a caller uniform).
 *   q3s_sample_cp_frame  scripts/export/utils.py:1218-1237 (the 15-stage
 *                        sampling loop of CodePredictorUnrolled.forward), as
 *                        one persistent kernel per frame.
 *
 * Conventions
 *   - Every pointer in a descriptor is a DEVICE pointer (except the
 *     descriptor itself).  NULL per-row parameter arrays fall back to the
 *     scalar *_default field.
 *   - Calls are asynchronous on `stream` (a cudaStream_t passed as void*;
 *     NULL = the legacy default stream), never allocate, never synchronise,
 *     and are re-entrant.  The library's only mutable state: per-device
 *     caches of the SM count and of kernel attributes already set (atomics;
 *     racing first calls store the same values), the process-wide kernel
 *     policy of q3s_set_kernel_policy (an atomic int), and a thread-local
 *     error string.
 *   - Arguments are validated on the host before any CUDA call; a bad
 *     argument returns Q3S_ERR_INVALID_ARGUMENT and launches nothing.
 *     q3s_last_error_string() explains the most recent failure of the
 *     calling thread.
 *   - Data problems only visible on the device (history ids outside
 *     [0,vocab), bad offsets, too many candidates) are OR-ed into the
 *     optional device word `error_word` (Q3S_DEVERR_* bits); the row is still
 *     sampled with the offending entries ignored.
 *   - Nothing here faults on purpose: every device-side wait is bounded and
 *     reports Q3S_DEVERR_WAIT_TIMEOUT instead of hanging.
 */
#ifndef Q3S_SAMPLER_H
#define Q3S_SAMPLER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q3S_ABI_VERSION 2
#define Q3S_MAX_VOCAB 8192     /* one CTA holds a whole row on chip */
#define Q3S_MAX_TOPK 512       /* largest exactly-K candidate set (gumbel mode) */
#define Q3S_MAX_CP_STAGES 64

typedef enum q3s_status {
  Q3S_OK = 0,
  Q3S_ERR_INVALID_ARGUMENT = 1,
  Q3S_ERR_UNSUPPORTED = 2,
  Q3S_ERR_CUDA = 3
} q3s_status;

typedef enum q3s_draw_mode {
  /* engine graph: exactly-K top-k ordered (value desc, index asc), scores
   * v/T + gumbel_noise[rank], argmax (lowest rank on ties). */
  Q3S_DRAW_GUMBEL = 0,
  /* validation chain: HF top-k (ties at the k-th value kept), top-p (stable
   * ascending order), softmax, first index with cdf > u * cdf_last. */
  Q3S_DRAW_ICDF = 1
} q3s_draw_mode;

typedef enum q3s_dtype { Q3S_DTYPE_F32 = 0, Q3S_DTYPE_BF16 = 1 } q3s_dtype;

/* row_flags bits written per row (optional output) */
#define Q3S_ROW_DRAW_BOUNDARY 1   /* draw within 1e-6 (relative) of a CDF edge */
#define Q3S_ROW_TOPP_BOUNDARY 2   /* a top-p cumulative mass within 1e-6 of 1-p */
#define Q3S_ROW_GREEDY 4          /* argmax path taken */
#define Q3S_ROW_FALLBACK 8        /* u*total reached the total: last positive id taken */
#define Q3S_ROW_EXACT_CORE 16     /* register-resident row kernel: the row was decided by the exact
                                     whole-row core (values beyond its fast paths' proven window) */

/* error_word bits (device side, OR-ed) */
#define Q3S_DEVERR_HISTORY_ID 1        /* history id outside [0,vocab): ignored */
#define Q3S_DEVERR_OFFSETS 2           /* offsets not monotone / beyond history_len */
#define Q3S_DEVERR_NO_MASS 4           /* no finite logit survived (id = argmax) */
#define Q3S_DEVERR_WAIT_TIMEOUT 8      /* a bounded device wait gave up */
#define Q3S_DEVERR_CANDIDATES 16       /* exactly-K candidate set overflow */
#define Q3S_DEVERR_HISTORY_FULL 32     /* capacity layout: a row's region is full (id not appended) */

/* One sampling step over B rows (codebook 0, or one code-predictor stage). */
typedef struct q3s_sample_desc {
  uint32_t struct_size;        /* = sizeof(q3s_sample_desc) */
  int32_t mode;                /* q3s_draw_mode */
  int32_t batch;               /* B >= 0 (0 = no-op) */
  int32_t vocab;               /* V, 1..Q3S_MAX_VOCAB */
  int32_t topk;                /* gumbel: K candidates (1..min(V,Q3S_MAX_TOPK));
                                  icdf: default top-k when top_k == NULL (<=0 or >=V: off) */
  int32_t logits_dtype;        /* q3s_dtype */
  int64_t logits_row_stride;   /* elements between rows (>= V) */
  const void* logits;          /* [B, stride] */
  const int64_t* col_shift;    /* optional [B]: row b, column v is read at
                                  logits[b, (v + col_shift[b]) mod V] */

  /* presence history: token_counts layout OR packed ragged layout (or none) */
  const int64_t* token_counts; /* [B, token_counts_row_stride] int64, count > 0 = appeared */
  int64_t token_counts_row_stride;
  const int32_t* history;      /* packed ids; row b = history[offsets[b] .. offsets[b+1])
                                  (capacity layout: see history_lengths at the end) */
  const int32_t* offsets;      /* [B+1] */
  int64_t history_len;         /* entries in `history` (bounds check) */

  /* per-row parameters (NULL = scalar default) */
  const float* temperature;    float temperature_default;   /* icdf: <= 0 = greedy */
  const int32_t* top_k;        /* icdf only; NULL = `topk` for every row */
  const float* top_p;          float top_p_default;         /* icdf: >= 1 = off */
  const float* penalty;        float penalty_default;       /* 1 = off */
  const int32_t* min_new_tokens; int32_t min_new_tokens_default;
  const int32_t* cur_len;      /* NULL: history length (packed) or 0 */

  /* randomness, supplied by the caller */
  const float* gumbel_noise;   /* gumbel: [B, gumbel_row_stride], column r pairs with rank r;
                                  NULL = greedy argmax over the full row (utils.py:1185-1186) */
  int64_t gumbel_row_stride;
  const float* uniforms;       /* icdf: [B] in [0,1) */

  /* special-token masking */
  const uint8_t* suppress_mask; /* optional bool [V]: true -> logit = -1e9 */
  int32_t eos_id;               /* EOS id for min-new-tokens gating (-1 = none) */
  int32_t reserved0;

  /* outputs */
  int64_t* ids_i64;            /* [B] (either or both of ids_i64 / ids_i32) */
  int32_t* ids_i32;
  int64_t* counts_out;         /* optional [B, counts_out_row_stride]: token_counts +
                                  one_hot(id); may equal token_counts (in-place +1) */
  int64_t counts_out_row_stride;
  float* processed_logits;     /* optional [B, processed_row_stride] fp32 (verification) */
  int64_t processed_row_stride;
  int32_t* row_flags;          /* optional [B], Q3S_ROW_* bits */
  int32_t* error_word;         /* optional single device int32, Q3S_DEVERR_* bits */

  /* capacity layout of the history (optional): row b's ids are
   * history[offsets[b] .. offsets[b] + history_lengths[b]) inside its region
   * [offsets[b], offsets[b+1]), so that q3s_step_update can append in place.
   * NULL: the packed layout above. */
  const int32_t* history_lengths; /* [B] */
} q3s_sample_desc;

/* Stage producer of the code-predictor frame. */
typedef enum q3s_cp_producer {
  Q3S_CP_DIRECT = 0,  /* stage j reads logits[j] as given */
  Q3S_CP_ROTATE = 1   /* stage j reads logits[j][b][(v + id_{j-1}[b]) mod V], id_{-1} = ids_init */
} q3s_cp_producer;

/* All code-predictor stages of one frame for B rows, one persistent kernel. */
typedef struct q3s_cp_frame_desc {
  uint32_t struct_size;        /* = sizeof(q3s_cp_frame_desc) */
  int32_t mode;                /* q3s_draw_mode */
  int32_t batch;
  int32_t vocab;
  int32_t stages;              /* S, 1..Q3S_MAX_CP_STAGES (reference: 15) */
  int32_t topk;                /* K (reference: min(50, V)) */
  int32_t logits_dtype;
  int32_t producer;            /* q3s_cp_producer */
  const void* logits;          /* [S, B, V] with the strides below */
  int64_t logits_row_stride;   /* elements */
  int64_t logits_stage_stride; /* elements */
  const int64_t* ids_init;     /* [B], ROTATE only */
  const float* temperature;    float temperature_default;
  const float* top_p;          float top_p_default;          /* icdf only */
  const float* gumbel_noise;   /* gumbel: [B, S, >=K] (cp_gumbel_noise layout); NULL = greedy */
  int64_t gumbel_row_stride;   /* elements between rows */
  int64_t gumbel_stage_stride; /* elements between stages */
  const float* uniforms;       /* icdf: [B, S] */
  int64_t* ids_out;            /* [B, S] int64 (reference cp_tokens layout) */
  int32_t* row_flags;          /* optional [B, S] */
  int32_t* error_word;         /* optional */
} q3s_cp_frame_desc;

/* Sample one token per row.  Replaces talker_unified_modules.py:407-422,
 * utils.py:1178-1193 and prefill_compare.py:383-399 (see above). */
q3s_status q3s_sample(const q3s_sample_desc* desc, void* stream);

/* Sample all stages of a code-predictor frame in one persistent launch.
 * Replaces the sampling loop of utils.py:1218-1237. */
q3s_status q3s_sample_cp_frame(const q3s_cp_frame_desc* desc, void* stream);

/* Message for the calling thread's most recent non-OK status ("" if none). */
const char* q3s_last_error_string(void);

/* Q3S_ABI_VERSION of the loaded library. */
int32_t q3s_abi_version(void);

/* sizeof() of the descriptors as compiled into the library, so a binding can
 * check its own struct layout (which: 0 = sample, 1 = cp_frame, 2 = step,
 * 3 = head). */
uint32_t q3s_desc_size(int32_t which);

/* Per-row randomness on the device (the next step after the sampler: the
 * reference draws it per slot on the host side of the launch,
 * engine/backend/executor.py:3216-3295 -- one torch.rand per slot and step,
 * then -log(-log(clamp(u, 1e-8, 1))) for the Gumbel noise).  One launch fills
 * out[i, 0..cols) for rows i = 0..rows-1 from Philox4x32-10 keyed by `seed`:
 * block j of row key r (row_keys[i], or row0 + i when row_keys is NULL) at
 * `step` uses counter (j, r mod 2^32, step, 0xA5A5 ^ (r >> 32)) -- all 64
 * bits of the key take part; below 2^32 the counter is (j, r, step, 0xA5A5)
 * --; a 32-bit output x becomes the uniform (x >> 8) * 2^-24 in [0, 1).  The same bits as the host
 * generator q3s/philox.py (row_uniforms), so a row's numbers do not depend on
 * which batch or shard it sits in.  `out` and `row_keys` are device
 * pointers; asynchronous on `stream`. */
#define Q3S_PHILOX_UNIFORM 0   /* uniforms in [0, 1) (one per row for the icdf draw) */
#define Q3S_PHILOX_GUMBEL 1    /* -log(-log(max(u, 1e-8))) in fp32 (gumbel_noise) */
q3s_status q3s_philox_rows(uint64_t seed, uint32_t step, const int64_t* row_keys, int64_t row0, int32_t rows,
                           int32_t cols, int32_t kind, float* out, int64_t out_row_stride, void* stream);

/* The same with one 64-bit seed per row as the Philox key: block j of row i
 * at (step, stage) uses counter (j, step, stage, 0x5EED) under key
 * (row_seeds[i] mod 2^32, row_seeds[i] >> 32).  This maps the reference's
 * per-slot generators one to one: each slot's generator is seeded with the
 * 63-bit blake2b digest of (base seed, request identity, segment[, retry])
 * (_stable_sampling_seed, engine/backend/executor.py:79-86, used per slot at
 * :3216-3254), so the host computes that seed once per segment (a retry gets
 * its salted seed) and the device draws every step's numbers from it; `stage`
 * separates the codebook-0 noise (e.g. 0) from the code-predictor stages.
 * Host generator: q3s/philox.py seeded_uniforms. */
q3s_status q3s_philox_seeds(const uint64_t* row_seeds, uint32_t step, uint32_t stage, int32_t rows, int32_t cols,
                            int32_t kind, float* out, int64_t out_row_stride, void* stream);

/* Per-step codec-0 epilogue on the device: EOS, frame counter, token loop
 * guard, packed history append.  The reference reads every row's codebook-0
 * id back to the host each step (engine/backend/executor.py:532-546) and runs
 * these checks per slot in Python (engine/backend/engine_loop.py:2749-2750,
 * 2863-3080, thresholds normalised at :372-387); the count update it feeds is
 * talker_unified_modules.py:421-422.  The kernels do them for all rows and
 * leave a compact event list, so the host reads one word per step (the
 * event count) and the listed rows only when it is non-zero: one cluster
 * launch with the in-place append (history_lengths) or none, up to 65536
 * rows; otherwise a per-row launch (guard + history copy) and an event
 * compaction launch when the list or the count is asked for. */
#define Q3S_EVT_EOS 1              /* id == eos_id: segment ends, guard skipped */
#define Q3S_EVT_SUSPECT 2          /* loop_run reached the suspect threshold */
#define Q3S_EVT_RECOVERED 4        /* token changed after a run >= suspect */
#define Q3S_EVT_DEFERRED 8         /* run == abort without generation progress */
#define Q3S_EVT_ABORT_PROGRESS 16  /* run >= abort with progress ("progress" mode) */
#define Q3S_EVT_ABORT_EMERGENCY 32 /* run >= emergency ("emergency" mode) */

typedef struct q3s_step_desc {
  uint32_t struct_size;        /* = sizeof(q3s_step_desc) */
  int32_t batch;               /* B >= 0 (0 = no-op), < 2^23 */
  const int64_t* ids_i64;      /* [B] sampled codebook-0 ids: exactly one of the two */
  const int32_t* ids_i32;
  int32_t eos_id;              /* codec EOS id (reference: 2150) */
  int32_t reserved0;

  /* packed history append (history_out NULL = skipped).  Row b of the output
   * is row b of the input followed by ids[b]; offsets_out[b] = offsets[b] + b.
   * history_out must not overlap history. */
  const int32_t* history;      /* packed ids (NULL allowed when history_len is 0); row b = history[offsets[b] .. offsets[b+1]) */
  const int32_t* offsets;      /* [B+1] */
  int64_t history_len;         /* entries in `history` (bounds check) */
  int32_t* history_out;        /* capacity history_out_capacity entries (>= history_len + B) */
  int32_t* offsets_out;        /* [B+1] */
  int64_t history_out_capacity;

  /* loop guard thresholds as given to the engine (normalised inside as the
   * engine does: abort <= 0 turns the guard off) */
  int32_t suspect_frames;
  int32_t abort_frames;
  int32_t emergency_frames;
  int32_t reserved1;
  double min_audio_text_ratio; /* <= 0: no progress gate */

  /* per-row guard state [B], read and updated in place (the engine keeps it
   * per segment / slot; a new or retried segment starts at loop_token = -1 and
   * zeros).  Required when the guard is on; frame_idx is optional otherwise. */
  int32_t* loop_token;
  int32_t* loop_run;
  int32_t* loop_max_run;
  int32_t* loop_suspect_count;
  int32_t* loop_recovery_count;
  int32_t* frame_idx;          /* +1 on every non-EOS row */
  /* progress inputs [B] (required when the guard is on and min ratio > 0) */
  const int32_t* decode_start_frame;
  const int32_t* text_tokens_consumed;
  const uint8_t* input_complete;

  /* outputs (all optional) */
  int32_t* events;             /* [B] Q3S_EVT_* bits (required with event_list / event_count) */
  int32_t* event_run;          /* [B] ended run on RECOVERED, run on an abort, else 0 */
  int32_t* event_list;         /* [B] (row << 8) | bits for rows with any bit, ascending row */
  int32_t* event_count;        /* one int32: entries written to event_list (required with it) */
  int32_t* error_word;         /* Q3S_DEVERR_OFFSETS on bad offsets / capacity (row skipped);
                                  Q3S_DEVERR_WAIT_TIMEOUT if the bounded wait of the one-launch
                                  event-list exchange gave up (that CTA's entries not written) */

  /* in-place append into the capacity layout (optional; then history_out
   * must equal history and offsets_out is not used): row b's region is
   * [offsets[b], offsets[b+1]) of history_out, its ids the first
   * history_lengths[b] entries; ids[b] goes to history_out[offsets[b] +
   * history_lengths[b]] and the length grows by one.  A full region gets
   * nothing appended and sets Q3S_DEVERR_HISTORY_FULL.  O(B) bytes a step
   * instead of the packed copy's O(sum of lengths). */
  int32_t* history_lengths;    /* [B], read and updated */
} q3s_step_desc;

/* One epilogue step over B rows; asynchronous on `stream`, no allocation.
 * Without the packed copy (history_out NULL, or the capacity layout's
 * in-place append) one thread runs each row. */
q3s_status q3s_step_update(const q3s_step_desc* desc, void* stream);

/* The codec head and the sampler in one call: logits = hidden @ weight^T on
 * the tensor cores (bf16 operands, fp32 accumulation, bf16 logits), then --
 * when `sample` is given -- one q3s_sample step over those logits, launched
 * behind the head as a programmatic dependent so that its history and
 * parameter loads overlap the GEMM and it reads the logits while they sit in
 * L2.  Replaces codec_head(hidden) (scripts/export/talker_unified_modules.py:
 * 345, nn.Linear(hidden_size, vocab, bias=False) applied to the last
 * position) or a code predictor's lm_heads[stage] (scripts/export/utils.py:
 * 1223) followed by the sampling sub-graph (:407-422 / utils.py:1178-1193).
 * The logits are an output, as the fused engine outputs them. */
typedef struct q3s_head_desc {
  uint32_t struct_size;        /* = sizeof(q3s_head_desc) */
  int32_t batch;               /* B >= 0 (0 = no-op) */
  int32_t hidden_size;         /* H: a positive multiple of 256 */
  int32_t vocab;               /* V: a positive multiple of 64, <= Q3S_MAX_VOCAB */
  const void* hidden;          /* bf16 [B, hidden_row_stride], 16-byte aligned rows */
  int64_t hidden_row_stride;   /* elements, >= H, a multiple of 8 */
  const void* weight;          /* bf16 [V, weight_row_stride]: the Linear's weight (out x in) */
  int64_t weight_row_stride;   /* elements, >= H, a multiple of 8 */
  void* logits;                /* bf16 [B, logits_row_stride] output */
  int64_t logits_row_stride;   /* elements, >= V, a multiple of 8 */
  const q3s_sample_desc* sample; /* optional sampling step over the logits; its batch, vocab, logits,
                                    logits_dtype and logits_row_stride are taken from here */
  int32_t* error_word;         /* optional: Q3S_DEVERR_WAIT_TIMEOUT if a bounded device wait gave up */
  int32_t reserved0;
} q3s_head_desc;

q3s_status q3s_head_sample(const q3s_head_desc* desc, void* stream);

/* Kernel family for icdf steps that either family can serve (process-wide;
 * a tuning and test knob with no counterpart in the reference interface):
 * the register-resident CTA-per-row kernel, the shared-memory-resident row
 * kernel with W warps per row (W chosen from the batch size, or forced), or
 * the register-resident row kernel that resolves each row exactly on a short
 * list (LEAN, 128 threads a row).  AUTO takes LEAN for batches of more than
 * two rows per SM and the shared-memory kernel below that, wherever they
 * apply.  All return the same ids, except that a draw or a top-p cut within
 * 1e-6 of a cumulative-mass edge (flagged in row_flags) may land on either
 * side.  Steps that need token_counts, col_shift or counts_out, Gumbel mode,
 * or a vocabulary not a multiple of 8 always take CTA-per-row; the
 * shared-memory kernel also needs 1024 < V <= 3072, LEAN V <= 3072. */
typedef enum {
  Q3S_POLICY_AUTO = 0,
  Q3S_POLICY_CTA = 1,
  Q3S_POLICY_WARP = 2,   /* shared-memory row kernel, W from the batch size */
  Q3S_POLICY_ROW_W1 = 3, /* shared-memory row kernel, W forced to 1, 2, 4, 8 */
  Q3S_POLICY_ROW_W2 = 4,
  Q3S_POLICY_ROW_W4 = 5,
  Q3S_POLICY_ROW_W8 = 6,
  Q3S_POLICY_ROW_WMAX = 7, /* W = 12 (V > 2048) or 16 (V <= 2048) */
  Q3S_POLICY_LEAN = 8      /* register-resident row kernel (128 threads a row) */
} q3s_kernel_policy;

/* Set the policy; returns the previous one, or -1 (unchanged) for an unknown
 * value. */
int32_t q3s_set_kernel_policy(int32_t policy);

#ifdef __cplusplus
}
#endif

#endif /* Q3S_SAMPLER_H */
