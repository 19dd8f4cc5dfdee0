"""CPU oracle for the codec-token sampling hot path -- TEST INFRASTRUCTURE ONLY.

This file is a restatement, in plain torch-CPU / numpy operations, of the
reference's sampler arithmetic.  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / ``--impl reference`` legs may import it, and
only as the checker or the timed CPU baseline; the product path (the CUDA
kernels behind ``include/q3s_sampler.h``) never calls it.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
code (``TalkerUnifiedFusedONNX.forward`` with stub sub-modules,
``CodePredictorUnrolled._select_token``, and ``_sample_token`` from
``tools/validation/prefill_compare.py`` with its multinomial draw driven by
supplied uniforms) and commits the results as ``tests/golden/*.npz``;
``tests/test_oracle_golden.py`` checks this file against them.

Two draw modes share one logits-processor core:

* ``gumbel`` -- the engine graph: suppress (-1e9) -> presence repetition
  penalty -> exactly-K top-k -> /T -> +noise -> argmax -> gather -> one-hot
  count update.  Reference: scripts/export/talker_unified_modules.py:407-422
  (codebook 0) and scripts/export/utils.py:1178-1193 (code-predictor stage).
* ``icdf`` -- the validation sampler chain: suppress (-1e9) ->
  RepetitionPenalty -> MinNewTokens(EOS=-inf) -> Temperature -> TopK (ties at
  the k-th value kept) -> TopP -> softmax -> inverse-CDF draw from one
  supplied uniform.  Reference: tools/validation/prefill_compare.py:383-399,
  with the TopP / MinNewTokens steps of the same ``transformers`` logits
  processors (transformers 5.5.0 here; the reference pins no version).

Tie rules (documented deviations, both deterministic):

* gumbel top-k orders its K candidates by (value desc, index asc); the
  reference's ``torch.topk`` leaves tie order unspecified, and the Gumbel noise
  is paired with candidates by rank, so tie order can change the sampled id.
  ``raw_topk_ids`` reports what plain ``torch.topk`` gives, to count those rows.
* top-p sorts ascending with a *stable* sort, i.e. (value asc, index asc);
  ``TopPLogitsWarper`` calls ``torch.sort`` without ``stable=True``.
"""
from __future__ import annotations

import numpy as np
import torch

NEG_SUPPRESS = -1e9  # talker_unified_modules.py:409, prefill_compare.py:395
BOUNDARY_EPS = 1e-6  # draws / top-p cuts this close to an edge are counted, not failed

ROW_DRAW_BOUNDARY = 1
ROW_TOPP_BOUNDARY = 2
ROW_GREEDY = 4


# --------------------------------------------------------------------------
# inputs
# --------------------------------------------------------------------------

def suppress_mask(vocab_size: int = 3072, eos_id: int = 2150) -> np.ndarray:
    """bool[V]: ids in [V-1024, V) except EOS.
    Reference: talker_unified_modules.py:384-389 (and prefill_compare.py:280-284)."""
    m = np.zeros(vocab_size, dtype=bool)
    m[max(0, vocab_size - 1024):] = True
    if 0 <= eos_id < vocab_size:
        m[eos_id] = False
    return m


def row_spans(offsets: np.ndarray, lengths: np.ndarray | None = None) -> list[tuple[int, int]]:
    """[start, end) of every row: offsets[b]..offsets[b+1] (packed), or the
    first lengths[b] entries of the region offsets[b]..offsets[b+1]
    (capacity layout)."""
    o = np.asarray(offsets, np.int64)
    if lengths is None:
        return [(int(o[b]), int(o[b + 1])) for b in range(len(o) - 1)]
    n = np.asarray(lengths, np.int64)
    return [(int(o[b]), int(o[b] + n[b])) for b in range(len(o) - 1)]


def appeared_from_packed(history: np.ndarray, offsets: np.ndarray, vocab: int,
                         lengths: np.ndarray | None = None) -> np.ndarray:
    """Presence matrix bool[B,V] from a packed ragged history (or its
    capacity layout, ``lengths`` given).  Ids outside [0,V) are ignored (the
    kernel flags them in its error word)."""
    spans = row_spans(offsets, lengths)
    B = len(spans)
    out = np.zeros((B, vocab), dtype=bool)
    for b, (s0, s1) in enumerate(spans):
        ids = np.asarray(history[s0:s1], dtype=np.int64)
        ids = ids[(ids >= 0) & (ids < vocab)]
        out[b, ids] = True
    return out


def _as_f32(logits) -> torch.Tensor:
    """bf16 inputs are upcast to fp32 once, before any processing."""
    t = torch.as_tensor(logits)
    return t.float().clone()


def _row_param(x, B: int, default, dtype) -> torch.Tensor:
    if x is None:
        return torch.full((B,), default, dtype=dtype)
    t = torch.as_tensor(np.asarray(x)).to(dtype).reshape(-1)
    assert t.numel() == B
    return t


# --------------------------------------------------------------------------
# shared logits-processor core
# --------------------------------------------------------------------------

def _apply_suppress_penalty(s: torch.Tensor, appeared: torch.Tensor | None,
                            penalty: torch.Tensor, suppress: np.ndarray | None) -> torch.Tensor:
    """suppress -> presence repetition penalty.

    Reference: talker_unified_modules.py:409-413 (``where(g0>0, g0/p, g0*p)``
    where ``token_counts>0``).  HF ``RepetitionPenaltyLogitsProcessor`` uses
    ``where(x<0, x*p, x/p)``: the two agree for every x (x==0 gives 0 either way)."""
    if suppress is not None:
        s = s.masked_fill(torch.as_tensor(suppress), NEG_SUPPRESS)
    if appeared is not None:
        pen = penalty.reshape(-1, 1)
        penalized = torch.where(s > 0, s / pen, s * pen)
        s = torch.where(torch.as_tensor(appeared), penalized, s)
    return s


def _apply_eos_gate(s: torch.Tensor, eos_id: int | None, min_new: torch.Tensor | None,
                    cur_len: torch.Tensor | None) -> torch.Tensor:
    """HF ``MinNewTokensLengthLogitsProcessor``: EOS -> -inf while the row's
    current length is below ``min_new_tokens``."""
    if eos_id is None or min_new is None or eos_id < 0 or eos_id >= s.shape[1]:
        return s
    gate = cur_len < min_new
    if bool(gate.any()):
        s = s.clone()
        s[gate, eos_id] = float("-inf")
    return s


def _canonical_desc_order(x: torch.Tensor) -> torch.Tensor:
    """Indices sorting each row by (value desc, index asc)."""
    # stable descending sort keeps equal values in index order
    return torch.sort(x, dim=-1, descending=True, stable=True).indices


# --------------------------------------------------------------------------
# gumbel mode (the engine graph)
# --------------------------------------------------------------------------

def sample_gumbel(logits, *, gumbel_noise, temperature, penalty,
                  token_counts=None, history=None, offsets=None,
                  suppress: np.ndarray | None = None, topk: int = 50,
                  eos_id: int | None = None, min_new_tokens=None, cur_len=None) -> dict:
    """Codebook-0 sampler of the fused graph.

    Reference: talker_unified_modules.py:407-422::

        g0 = g0.masked_fill(suppress_mask, -1e9)
        g0 = where(token_counts>0, where(g0>0, g0/penalty, g0*penalty), g0)
        topk_vals, topk_idx = g0.topk(50)
        selected = (topk_vals / temperature + gumbel_noise).argmax(-1)
        codec_token_0 = topk_idx.gather(1, selected)
        updated_token_counts = token_counts + one_hot(codec_token_0)

    ``token_counts`` (int64 [B,V]) or a packed ``history``/``offsets`` gives
    the presence set.  Returns ids, updated counts (counts layout only), the
    processed row ``g0`` and the ids plain ``torch.topk`` would give."""
    s = _as_f32(logits)
    B, V = s.shape
    K = min(int(topk), V)
    T = _row_param(temperature, B, 1.0, torch.float32)
    pen = _row_param(penalty, B, 1.0, torch.float32)
    appeared = None
    if token_counts is not None:
        appeared = torch.as_tensor(np.asarray(token_counts)) > 0
    elif history is not None:
        appeared = torch.as_tensor(appeared_from_packed(history, offsets, V))
    g0 = _apply_suppress_penalty(s, appeared, pen, suppress)
    if min_new_tokens is not None:
        if cur_len is None:
            cur_len = (np.diff(offsets) if offsets is not None else np.zeros(B, np.int32))
        g0 = _apply_eos_gate(g0, eos_id, _row_param(min_new_tokens, B, 0, torch.int64),
                             _row_param(cur_len, B, 0, torch.int64))
    noise = torch.as_tensor(np.asarray(gumbel_noise, dtype=np.float32))[:, :K]

    order = _canonical_desc_order(g0)[:, :K]
    vals = g0.gather(1, order)
    sel = (vals / T.reshape(-1, 1) + noise).argmax(dim=-1)
    ids = order.gather(1, sel.unsqueeze(1)).squeeze(1)

    rv, ri = g0.topk(K, dim=-1)
    rsel = (rv / T.reshape(-1, 1) + noise).argmax(dim=-1)
    raw_ids = ri.gather(1, rsel.unsqueeze(1)).squeeze(1)

    out = {"ids": ids.numpy().astype(np.int64), "processed": g0.numpy(),
           "raw_topk_ids": raw_ids.numpy().astype(np.int64)}
    if token_counts is not None:
        tc = torch.as_tensor(np.asarray(token_counts, dtype=np.int64))
        out["updated_counts"] = (tc + torch.nn.functional.one_hot(ids, V).to(tc.dtype)).numpy()
    return out


def select_token_cp(logits, *, temperature=None, gumbel_noise=None, topk: int = 50) -> np.ndarray:
    """Code-predictor stage sampler.

    Reference: utils.py:1178-1193 -- greedy ``argmax`` over the full row when
    no noise is given; otherwise top-min(K,V) -> /T -> +noise[:, :K] ->
    argmax -> gather, with no penalty and no suppress."""
    s = _as_f32(logits)
    if s.dim() == 3:
        s = s.squeeze(1)
    B, V = s.shape
    if gumbel_noise is None:
        return s.argmax(dim=-1).numpy().astype(np.int64)
    K = min(int(topk), V)
    T = _row_param(temperature, B, 1.0, torch.float32)
    noise = torch.as_tensor(np.asarray(gumbel_noise, dtype=np.float32))[:, :K]
    order = _canonical_desc_order(s)[:, :K]
    vals = s.gather(1, order)
    sel = (vals / T.reshape(-1, 1) + noise).argmax(dim=-1)
    return order.gather(1, sel.unsqueeze(1)).squeeze(1).numpy().astype(np.int64)


# --------------------------------------------------------------------------
# icdf mode (validation sampler chain + inverse-CDF on supplied uniforms)
# --------------------------------------------------------------------------

def _top_k_filter(s: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """HF ``TopKLogitsWarper`` with a per-row k: remove ``s < kth value``
    (ties at the k-th value are kept).  k<=0 or k>=V disables the row."""
    B, V = s.shape
    active = (k > 0) & (k < V)
    if not bool(active.any()):
        return s
    kmax = int(k[active].max())
    top = torch.topk(s, kmax, dim=-1).values
    kk = torch.where(active, k, torch.ones_like(k)).clamp(1, kmax) - 1
    thr = top.gather(1, kk.reshape(-1, 1).long())
    remove = (s < thr) & active.reshape(-1, 1)
    return s.masked_fill(remove, float("-inf"))


def _top_p_filter(s: torch.Tensor, p: torch.Tensor):
    """HF ``TopPLogitsWarper`` with a per-row p and a stable ascending sort.

    Returns (filtered scores, boundary rows): a row is a boundary row when the
    float64 cumulative probability of some element lies within 1e-6 of
    ``1-p``, so an fp32 implementation may legitimately cut one element more
    or less there."""
    B, V = s.shape
    active = p < 1.0
    boundary = torch.zeros(B, dtype=torch.bool)
    if not bool(active.any()):
        return s, boundary
    out = s.clone()
    rows = torch.nonzero(active).reshape(-1)
    sub = s[rows]
    sorted_logits, sorted_idx = torch.sort(sub, dim=-1, descending=False, stable=True)
    cum = sorted_logits.softmax(dim=-1).cumsum(dim=-1)
    thr = (1 - p[rows]).reshape(-1, 1)
    remove = cum <= thr
    remove[:, -1] = False
    rm = remove.scatter(1, sorted_idx, remove)
    out[rows] = sub.masked_fill(rm, float("-inf"))
    cum64 = torch.softmax(sorted_logits.double(), dim=-1).cumsum(dim=-1)
    near = (cum64 - thr.double()).abs() < BOUNDARY_EPS
    near[:, -1] = False
    boundary[rows] = near.any(dim=-1) | ((cum64 <= thr.double()) != remove).any(dim=-1)
    return out, boundary


def inverse_cdf_draw(s: np.ndarray, u: np.ndarray):
    """Draw ``id`` = first index with ``cdf > u * cdf[-1]``, the cdf being the
    inclusive sum, in vocabulary order, of ``exp(s - max)`` over finite s
    (float64, batched).  Returns (ids, boundary rows): a row is a boundary row
    when ``u * cdf[-1]`` lies within 1e-6 (relative) of the chosen CDF edge."""
    s64 = torch.as_tensor(np.asarray(s, dtype=np.float32)).double()
    B, V = s64.shape
    m = s64.max(dim=1, keepdim=True).values
    w = torch.exp(s64 - m)
    w = torch.where(torch.isnan(w), torch.zeros_like(w), w)
    cdf = w.cumsum(dim=1)
    tot = cdf[:, -1:]
    thr = torch.as_tensor(np.asarray(u, dtype=np.float32)).double().reshape(B, 1) * tot
    ids = torch.searchsorted(cdf, thr, right=True).reshape(B)
    over = ids >= V
    if bool(over.any()):
        pos = (w > 0).double() * torch.arange(1, V + 1, dtype=torch.float64)
        ids = torch.where(over, pos.argmax(dim=1), ids)
    hi = cdf.gather(1, ids.reshape(B, 1))
    lo = torch.where(ids.reshape(B, 1) > 0, cdf.gather(1, (ids - 1).clamp(min=0).reshape(B, 1)),
                     torch.zeros_like(hi))
    eps = BOUNDARY_EPS * tot
    bnd = ((hi - thr).abs() < eps) | ((thr - lo).abs() < eps)
    return ids.numpy().astype(np.int64), bnd.reshape(B).numpy()


def sample_icdf(logits, *, uniforms, temperature=None, top_k=None, top_p=None, penalty=None,
                history=None, offsets=None, token_counts=None, history_lengths=None,
                suppress: np.ndarray | None = None, eos_id: int | None = None,
                min_new_tokens=None, cur_len=None,
                temperature_default=1.0, top_k_default=0, top_p_default=1.0,
                penalty_default=1.0, min_new_default=0) -> dict:
    """Batched restatement of ``_sample_token`` (prefill_compare.py:383-399)
    with per-row parameters, the BASELINE TopP / MinNewTokens steps, and the
    ``torch.multinomial`` draw replaced by inverse-CDF on ``uniforms``.

    A row with temperature <= 0 is greedy: argmax (lowest index on ties) of the
    suppressed / penalised / EOS-gated row.  ``cur_len`` defaults to the row's
    history length."""
    s = _as_f32(logits)
    B, V = s.shape
    T = _row_param(temperature, B, temperature_default, torch.float32)
    K = _row_param(top_k, B, top_k_default, torch.int64)
    P = _row_param(top_p, B, top_p_default, torch.float32)
    pen = _row_param(penalty, B, penalty_default, torch.float32)
    mn = _row_param(min_new_tokens, B, min_new_default, torch.int64)
    if cur_len is None:
        if history_lengths is not None:
            cur_len = np.asarray(history_lengths, np.int64)
        else:
            cur_len = np.diff(np.asarray(offsets)) if offsets is not None else np.zeros(B, np.int64)
    cl = _row_param(cur_len, B, 0, torch.int64)
    appeared = None
    if token_counts is not None:
        appeared = torch.as_tensor(np.asarray(token_counts)) > 0
    elif history is not None:
        appeared = torch.as_tensor(appeared_from_packed(history, offsets, V, history_lengths))
    x = _apply_suppress_penalty(s, appeared, pen, suppress)
    x = _apply_eos_gate(x, eos_id, mn, cl)

    greedy = T <= 0
    Tsafe = torch.where(greedy, torch.ones_like(T), T)
    y = x / Tsafe.reshape(-1, 1)
    y = _top_k_filter(y, torch.where(greedy, torch.zeros_like(K), K))
    y, topp_bnd = _top_p_filter(y, torch.where(greedy, torch.ones_like(P), P))
    ids, draw_bnd = inverse_cdf_draw(y.numpy(), np.asarray(uniforms, dtype=np.float32).reshape(-1))
    if bool(greedy.any()):
        g = torch.nonzero(greedy).reshape(-1)
        ids[g.numpy()] = x[g].argmax(dim=-1).numpy()
        draw_bnd[g.numpy()] = False
    processed = torch.where(greedy.reshape(-1, 1), x, y)
    flags = (draw_bnd.astype(np.int32) * ROW_DRAW_BOUNDARY
             | topp_bnd.numpy().astype(np.int32) * ROW_TOPP_BOUNDARY
             | greedy.numpy().astype(np.int32) * ROW_GREEDY)
    return {"ids": ids, "processed": processed.numpy(), "flags": flags,
            "boundary": (flags & (ROW_DRAW_BOUNDARY | ROW_TOPP_BOUNDARY)) != 0}


# --------------------------------------------------------------------------
# code-predictor frame (15 dependent stages)
# --------------------------------------------------------------------------

def rotate_rows(base: np.ndarray, shift: np.ndarray) -> np.ndarray:
    """``out[b, v] = base[b, (v + shift[b]) mod V]`` -- the synthetic stage
    producer of the code-predictor benchmark: stage j's logits are a fixed
    function of stage j-1's sampled ids, so the stages must run in order."""
    base = np.asarray(base)
    B, V = base.shape
    idx = (np.arange(V)[None, :] + np.asarray(shift, dtype=np.int64).reshape(-1, 1)) % V
    return np.take_along_axis(base, idx, axis=1)


def cp_frame(base, *, mode: str, ids_init=None, rotate: bool = True, temperature=None,
             topk: int = 50, top_p=None, gumbel_noise=None, uniforms=None) -> dict:
    """Run the stage chain of ``CodePredictorUnrolled.forward``'s sampling
    (utils.py:1218-1237) over ``base`` [S,B,V].  With ``rotate``, stage j reads
    ``rotate_rows(base[j], ids[j-1])`` (``ids[-1] = ids_init``).  ``mode`` is
    ``gumbel`` (noise [B,S,>=K]; ``None`` = greedy argmax) or ``icdf``
    (uniforms [B,S]).  Returns ids [B,S] and per-stage boundary flags."""
    base = np.asarray(base)
    S, B, V = base.shape
    prev = np.zeros(B, np.int64) if ids_init is None else np.asarray(ids_init, np.int64)
    ids = np.zeros((B, S), np.int64)
    bnd = np.zeros((B, S), bool)
    for j in range(S):
        lg = rotate_rows(base[j], prev) if rotate else base[j]
        lg = torch.from_numpy(np.ascontiguousarray(lg))
        if mode == "gumbel":
            nz = None if gumbel_noise is None else np.asarray(gumbel_noise)[:, j, :]
            ids[:, j] = select_token_cp(lg, temperature=temperature, gumbel_noise=nz, topk=topk)
        else:
            r = sample_icdf(lg, uniforms=np.asarray(uniforms)[:, j], temperature=temperature,
                            top_k=None, top_k_default=topk, top_p=top_p)
            ids[:, j] = r["ids"]
            bnd[:, j] = r["boundary"]
        prev = ids[:, j]
    return {"ids": ids, "boundary": bnd}


# ---------------------------------------------------------------------------
# per-step codec-0 epilogue: EOS, frame counter, token loop guard, history append
# ---------------------------------------------------------------------------

EVT_EOS, EVT_SUSPECT, EVT_RECOVERED, EVT_DEFERRED = 1, 2, 4, 8
EVT_ABORT_PROGRESS, EVT_ABORT_EMERGENCY = 16, 32
GUARD_FIELDS = ("loop_token", "loop_run", "loop_max_run", "loop_suspect_count", "loop_recovery_count", "frame_idx")


def guard_thresholds(suspect: int, abort: int, emergency: int) -> tuple[int, int, int]:
    """Threshold normalisation of EngineLoop.__init__
    (engine/backend/engine_loop.py:372-387): abort clamped at 0; suspect kept
    only with both stages on and then clamped to abort; emergency kept only
    with both on and then raised to abort."""
    abort = max(0, int(abort))
    suspect = max(0, int(suspect))
    suspect = min(suspect, abort) if suspect > 0 and abort > 0 else 0
    emergency = max(0, int(emergency))
    emergency = max(emergency, abort) if emergency > 0 and abort > 0 else 0
    return suspect, abort, emergency


def step_update(ids, *, eos_id: int, state: dict, suspect: int = 0, abort: int = 0, emergency: int = 0,
                min_ratio: float = 0.0, decode_start_frame=None, text_tokens=None, input_complete=None,
                history=None, offsets=None, history_lengths=None):
    """One step of the per-row codec-0 epilogue, row by row.

    * EOS: ``id == eos_id`` (engine/backend/executor.py:532-546); an EOS row
      ends its segment and skips the guard (engine_loop.py:2838-2839).
    * frame counter: ``frame_idx += 1`` on non-EOS rows, before the guard
      (engine_loop.py:2749-2750).
    * two-stage loop guard (engine_loop.py:2863-2966 and the decisions at
      :2968-3080): run / recovery / suspect bookkeeping, the generation
      progress gate ``audio_steps / text_tokens >= min_ratio`` (Python true
      division of two ints = one correctly rounded double division), deferred
      at ``run == abort`` without progress, abort by progress (confirmed) or
      by the emergency stage.
    * history append: row b of the packed history gains ``ids[b]`` (the packed
      counterpart of ``token_counts + one_hot(id)``,
      scripts/export/talker_unified_modules.py:421-422, applied to every row);
      ``offsets_out[b] = offsets[b] + b``.  With ``history_lengths`` (the
      capacity layout: row b is the first lengths[b] entries of its region
      offsets[b]..offsets[b+1]) the id goes in place after the row's last
      one and the length grows by one; a full region gets nothing (the
      kernel reports Q3S_DEVERR_HISTORY_FULL).  Then history_out is the
      updated copy of ``history`` and offsets_out the updated lengths.

    ``state`` maps GUARD_FIELDS to int arrays [B], updated in place.  Returns
    (events [B] int32, run [B] int32 -- the ended run on RECOVERED, the run on
    an abort, else 0 --, history_out or None, offsets_out or None).
    """
    ids = np.asarray(ids, np.int64)
    B = ids.shape[0]
    suspect, abort, emergency = guard_thresholds(suspect, abort, emergency)
    min_ratio = max(0.0, float(min_ratio))
    events = np.zeros(B, np.int32)
    runs = np.zeros(B, np.int32)
    st = {k: state[k] for k in GUARD_FIELDS}
    for b in range(B):
        tok = int(ids[b])
        if tok == eos_id:
            events[b] = EVT_EOS
            continue
        st["frame_idx"][b] += 1
        if abort <= 0:
            continue
        bits = 0
        if tok == st["loop_token"][b]:
            st["loop_run"][b] += 1
        else:
            if suspect > 0 and st["loop_run"][b] >= suspect:
                st["loop_recovery_count"][b] += 1
                bits |= EVT_RECOVERED
                runs[b] = st["loop_run"][b]
            st["loop_token"][b] = tok
            st["loop_run"][b] = 1
        run = int(st["loop_run"][b])
        st["loop_max_run"][b] = max(int(st["loop_max_run"][b]), run)
        if suspect > 0 and run == suspect:
            st["loop_suspect_count"][b] += 1
            bits |= EVT_SUSPECT
        audio_steps = max(0, int(st["frame_idx"][b]) - int(decode_start_frame[b] if decode_start_frame is not None else 0))
        text = max(0, int(text_tokens[b] if text_tokens is not None else 0))
        ratio = audio_steps / text if text > 0 else 0.0
        complete = bool(input_complete[b]) if input_complete is not None else False
        ready = min_ratio <= 0.0 or (complete and (text == 0 or ratio >= min_ratio))
        confirmed = run >= abort and ready
        emerg = emergency > 0 and run >= emergency
        if run == abort and not ready:
            bits |= EVT_DEFERRED
        if confirmed:
            bits |= EVT_ABORT_PROGRESS
            runs[b] = run
        elif emerg:
            bits |= EVT_ABORT_EMERGENCY
            runs[b] = run
        events[b] = bits
    hist_out = off_out = None
    if history is not None and history_lengths is not None:
        hist_out = np.array(history, np.int32, copy=True)
        o = np.asarray(offsets, np.int64)
        off_out = np.array(history_lengths, np.int32, copy=True)
        for b in range(B):
            if o[b] + off_out[b] < o[b + 1]:
                hist_out[o[b] + off_out[b]] = ids[b]
                off_out[b] += 1
        return events, runs, hist_out, off_out
    if history is not None:
        history = np.asarray(history, np.int32)
        offsets = np.asarray(offsets, np.int64)
        off_out = (offsets + np.arange(B + 1)).astype(np.int32)
        hist_out = np.empty(int(off_out[-1]), np.int32)
        for b in range(B):
            s, e = int(offsets[b]), int(offsets[b + 1])
            hist_out[off_out[b]:off_out[b] + (e - s)] = history[s:e]
            hist_out[off_out[b] + (e - s)] = ids[b]
    return events, runs, hist_out, off_out


def event_list(events: np.ndarray) -> np.ndarray:
    """Rows with any event, ascending, packed as (row << 8) | bits."""
    rows = np.nonzero(events)[0]
    return ((rows.astype(np.int64) << 8) | events[rows]).astype(np.int32)
