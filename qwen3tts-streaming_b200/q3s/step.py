"""Host side of the per-step codec-0 epilogue (``q3s_step_update``).

The reference copies every row's codebook-0 id to the host each step to test
it against the codec EOS id (engine/backend/executor.py:532-546), then runs the
frame counter and the two-stage token loop guard per slot in Python
(engine/backend/engine_loop.py:2749-2750, 2863-3080).  ``StepGuard`` keeps that
per-slot state on the GPU -- the fields of ``EngineSegment`` (loop_token,
loop_run, loop_max_run, loop_suspect_count, loop_recovery_count,
engine_loop.py:184-192) and the slot's frame_idx -- and runs the step over
all rows on the device, which also appends the sampled ids to the rows'
history (the history form of ``token_counts + one_hot(id)``,
scripts/export/talker_unified_modules.py:421-422): in place into a
``RowHistory`` (capacity layout, O(B) bytes a step, one launch up to 64 K
rows), or as a copy of a packed history with one id more per row (two
launches).  The host then reads one
int32 (the event count) per step, and the compact event list only when it is
not zero.

The thresholds take the engine's constructor arguments and are normalised by
the library exactly as ``EngineLoop.__init__`` does (engine_loop.py:372-387).
Decisions that need host state (retry vs. abort, audio health, logging) stay
with the caller; each event row carries the bits that tell it which branch of
the reference the row took.
"""
from __future__ import annotations

import ctypes as C
from contextlib import nullcontext as _nullcontext
from typing import Optional, Sequence, Union

import torch

from . import _lib
from .ops import DEFAULT_EOS, _need_cuda, _stream_handle

EVENT_NAMES = {
    _lib.EVT_EOS: "eos",
    _lib.EVT_SUSPECT: "loop_suspect",
    _lib.EVT_RECOVERED: "loop_recovered",
    _lib.EVT_DEFERRED: "loop_deferred",
    _lib.EVT_ABORT_PROGRESS: "loop_abort_progress",
    _lib.EVT_ABORT_EMERGENCY: "loop_abort_emergency",
}
GUARD_FIELDS = ("loop_token", "loop_run", "loop_max_run", "loop_suspect_count", "loop_recovery_count", "frame_idx")


class StepGuard:
    """Per-slot EOS / loop-guard state for ``batch`` rows on one GPU.

    ``token_loop_*`` are the engine's scheduler settings (defaults: the
    reference SchedulerConfig, engine/config.py:179-193).  Rows start as a new
    segment (loop_token -1, counters 0, frame_idx 0); ``reset_rows`` is the
    reset a retried segment gets (engine_loop.py:3486-3490).
    """

    def __init__(self, batch: int, *, eos_id: int = DEFAULT_EOS, token_loop_suspect_frames: int = 4,
                 token_loop_abort_frames: int = 10, token_loop_min_audio_text_ratio: float = 2.0,
                 token_loop_emergency_abort_frames: int = 20, device: Union[str, torch.device, None] = None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise ValueError("StepGuard state lives on a CUDA device")
        self.batch = int(batch)
        B = max(self.batch, 1)
        i32 = dict(dtype=torch.int32, device=self.device)
        self.state = {k: torch.zeros(B, **i32) for k in GUARD_FIELDS}
        self.state["loop_token"].fill_(-1)
        self.decode_start_frame = torch.zeros(B, **i32)
        self.text_tokens_consumed = torch.zeros(B, **i32)
        self.input_complete = torch.zeros(B, dtype=torch.uint8, device=self.device)
        self.events = torch.zeros(B, **i32)
        self.event_run = torch.zeros(B, **i32)
        self.event_list = torch.zeros(B, **i32)
        self.event_count = torch.zeros(1, **i32)
        self.error_word = torch.zeros(1, **i32)
        d = _lib.StepDesc()
        d.struct_size = C.sizeof(_lib.StepDesc)
        d.batch = self.batch
        d.eos_id = int(eos_id)
        d.suspect_frames = int(token_loop_suspect_frames)
        d.abort_frames = int(token_loop_abort_frames)
        d.emergency_frames = int(token_loop_emergency_abort_frames)
        d.min_audio_text_ratio = float(token_loop_min_audio_text_ratio)
        for k in GUARD_FIELDS:
            setattr(d, k, self.state[k].data_ptr())
        d.decode_start_frame = self.decode_start_frame.data_ptr()
        d.text_tokens_consumed = self.text_tokens_consumed.data_ptr()
        d.input_complete = self.input_complete.data_ptr()
        d.events = self.events.data_ptr()
        d.event_run = self.event_run.data_ptr()
        d.event_list = self.event_list.data_ptr()
        d.event_count = self.event_count.data_ptr()
        d.error_word = self.error_word.data_ptr()
        self._desc = d
        self._lib = _lib.load()

    # -- host-side segment bookkeeping -------------------------------------
    def reset_rows(self, rows: Union[Sequence[int], torch.Tensor],
                   stream: Optional[torch.cuda.Stream] = None) -> None:
        """A new or retried segment in these rows: loop_token -1, counters 0.
        The writes go on ``stream`` (the current stream if None): pass the
        stream the next ``step`` runs on, so they are ordered before it."""
        with torch.cuda.stream(stream) if stream is not None else _nullcontext():
            idx = torch.as_tensor(rows, dtype=torch.long, device=self.device)
            for k in GUARD_FIELDS[:-1]:
                self.state[k].index_fill_(0, idx, -1 if k == "loop_token" else 0)

    def set_progress(self, rows: Union[Sequence[int], torch.Tensor, None] = None, *,
                     frame_idx=None, decode_start_frame=None, text_tokens_consumed=None, input_complete=None,
                     stream: Optional[torch.cuda.Stream] = None) -> None:
        """Write the progress inputs of the given rows (all rows if None).

        The reference changes a segment's progress while it streams:
        ``text_tokens_consumed`` grows as text arrives
        (engine/backend/engine_loop.py:930-1000) and ``input_complete`` is set
        when the input ends (:1027).  The guard's progress gate reads them at
        every step, so call this whenever either changes, before the next
        ``step``, with that step's ``stream`` (the writes are then ordered
        before the launch; the current stream if None)."""
        with torch.cuda.stream(stream) if stream is not None else _nullcontext():
            idx = (torch.arange(self.batch, device=self.device) if rows is None
                   else torch.as_tensor(rows, dtype=torch.long, device=self.device))
            for t, v in ((self.state["frame_idx"], frame_idx), (self.decode_start_frame, decode_start_frame),
                         (self.text_tokens_consumed, text_tokens_consumed), (self.input_complete, input_complete)):
                if v is not None:
                    t[idx] = torch.as_tensor(v, device=self.device).to(t.dtype)

    # -- the step ------------------------------------------------------------
    def step(self, ids: torch.Tensor, *, history: Optional[torch.Tensor] = None,
             offsets: Optional[torch.Tensor] = None, history_out: Optional[torch.Tensor] = None,
             offsets_out: Optional[torch.Tensor] = None, rows: Optional["RowHistory"] = None,
             stream: Optional[torch.cuda.Stream] = None) -> None:
        """Launch the epilogue for this step's ids ([B] int64 or int32).

        With ``rows`` (a ``RowHistory``) each row's id is appended in place
        (O(B) bytes).  With ``history_out`` given instead, row b of the packed
        ``history`` / ``offsets`` is written to ``history_out`` followed by
        ``ids[b]``, and ``offsets_out = offsets + arange(B+1)``;
        ``history_out`` needs ``len(history) + B`` entries and must not
        overlap ``history``.  Asynchronous on ``stream``; read results with
        ``read_events``.
        """
        _need_cuda(ids, "ids", self.device)
        if ids.numel() != self.batch:
            raise ValueError(f"ids has {ids.numel()} values for {self.batch} rows")
        ids = ids.reshape(self.batch)
        if ids.dtype not in (torch.int64, torch.int32):
            raise ValueError(f"ids dtype {ids.dtype} unsupported (int64 or int32)")
        if not ids.is_contiguous():
            ids = ids.contiguous()
        d = self._desc
        d.ids_i64 = ids.data_ptr() if ids.dtype == torch.int64 else None
        d.ids_i32 = ids.data_ptr() if ids.dtype == torch.int32 else None
        d.history_lengths = None
        if rows is not None:
            if history_out is not None or history is not None:
                raise ValueError("give rows (in-place append) or the packed history / history_out, not both")
            if rows.batch != self.batch or rows.ids.device != self.device:
                raise ValueError(f"rows holds {rows.batch} rows on {rows.ids.device}; the guard {self.batch} on "
                                 f"{self.device}")
            d.history = d.history_out = rows.ids.data_ptr()
            d.offsets = rows.offsets.data_ptr()
            d.history_len = d.history_out_capacity = rows.ids.numel()
            d.offsets_out = None
            d.history_lengths = rows.lengths.data_ptr()
        elif history_out is not None:
            for t, n in ((history, "history"), (offsets, "offsets"), (history_out, "history_out"),
                         (offsets_out, "offsets_out")):
                if t is None:
                    raise ValueError(f"the history append needs {n}")
                _need_cuda(t, n, self.device)
                if t.dtype != torch.int32 or not t.is_contiguous():
                    raise ValueError(f"{n} must be a contiguous int32 tensor")
            if offsets.numel() != self.batch + 1 or offsets_out.numel() != self.batch + 1:
                raise ValueError(f"offsets / offsets_out need {self.batch + 1} entries")
            d.history, d.offsets, d.history_len = history.data_ptr(), offsets.data_ptr(), history.numel()
            d.history_out, d.offsets_out = history_out.data_ptr(), offsets_out.data_ptr()
            d.history_out_capacity = history_out.numel()
        else:
            d.history = d.offsets = d.history_out = d.offsets_out = None
            d.history_len = d.history_out_capacity = 0
        _lib.check(self._lib.q3s_step_update(C.byref(d), _stream_handle(stream)), "q3s_step_update")
        # keep the ids alive until the launch has been issued on the stream
        self._ids = ids
        self._stream = stream

    def read_events(self) -> list[tuple[int, int]]:
        """Synchronise and return [(row, bits)] of this step's rows with events,
        ascending by row: one 4-byte read, plus the list when it is non-empty."""
        if getattr(self, "_stream", None) is not None:
            self._stream.synchronize()  # the step ran on a stream other than the current one
        n = int(self.event_count.item())
        if n == 0:
            return []
        packed = self.event_list[:n].cpu()
        return [(int(v) >> 8, int(v) & 0xFF) for v in packed]

    def fields(self) -> dict[str, torch.Tensor]:
        """The per-row guard state (device tensors, updated in place)."""
        return {k: v[: self.batch] for k, v in self.state.items()}


def algorithmic_bytes_in_place(batch: int) -> int:
    """Bytes one q3s_step_update launch must move with the in-place append of
    the capacity layout: int64 ids (8 B), region offsets (4 (B + 1)), the
    lengths read and written (8 B), one id written per row (4 B), the guard
    state (48 B), progress inputs (9 B), events and event runs (8 B), the
    event count (4)."""
    B = int(batch)
    return 8 * B + 4 * (B + 1) + 8 * B + 4 * B + 48 * B + 9 * B + 8 * B + 4


class RowHistory:
    """Every row's token history in the capacity layout: row b owns the
    region ``ids[offsets[b] : offsets[b+1]]`` and its history is the first
    ``lengths[b]`` entries of it.  The sampler reads it through
    ``sampler_kwargs()`` (the repetition penalty's presence set) and
    ``StepGuard.step(ids, rows=...)`` appends each step's ids in place, so a
    step moves O(B) bytes where the packed layout re-copies every row -- the
    device-side form of the reference's count write-back
    (engine/backend/engine_loop.py:2617-2625, 2746-2747;
    scripts/export/talker_unified_modules.py:421-422).  A full region takes
    no more ids and reports Q3S_DEVERR_HISTORY_FULL in the guard's error
    word."""

    def __init__(self, batch: int, capacity: Union[int, Sequence[int]], *,
                 device: Union[str, torch.device, None] = None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.batch = int(batch)
        caps = torch.as_tensor([capacity] * self.batch if isinstance(capacity, int) else list(capacity),
                               dtype=torch.int64)
        if caps.numel() != self.batch or bool((caps < 0).any()):
            raise ValueError("one non-negative capacity per row")
        offs = torch.zeros(self.batch + 1, dtype=torch.int64)
        offs[1:] = torch.cumsum(caps, 0)
        if int(offs[-1]) >= 2 ** 31:
            raise ValueError("total capacity must stay below 2^31 entries")
        self.offsets = offs.to(torch.int32).to(self.device)
        self.ids = torch.zeros(max(1, int(offs[-1])), dtype=torch.int32, device=self.device)
        self.lengths = torch.zeros(self.batch, dtype=torch.int32, device=self.device)

    @classmethod
    def from_packed(cls, history: torch.Tensor, offsets: torch.Tensor, capacity: Union[int, Sequence[int]], *,
                    device: Union[str, torch.device, None] = None) -> "RowHistory":
        """A capacity layout holding the rows of a packed history (set-up,
        not a per-step operation)."""
        offsets = torch.as_tensor(offsets).to(torch.int64).cpu()
        B = offsets.numel() - 1
        rh = cls(B, capacity, device=device if device is not None else history.device)
        lens = offsets[1:] - offsets[:-1]
        if bool((lens > (rh.offsets[1:] - rh.offsets[:-1]).cpu()).any()):
            raise ValueError("a row is longer than its capacity")
        if int(lens.sum()):
            row = torch.repeat_interleave(torch.arange(B), lens)
            pos = torch.arange(int(lens.sum())) - offsets[:-1][row] + rh.offsets.cpu().to(torch.int64)[row]
            rh.ids[pos.to(rh.device)] = torch.as_tensor(history).to(rh.device, torch.int32).reshape(-1)
        rh.lengths.copy_(lens.to(torch.int32))
        return rh

    def reset_rows(self, rows: Union[Sequence[int], torch.Tensor],
                   stream: Optional[torch.cuda.Stream] = None) -> None:
        """Empty these rows' histories (a new segment in the slot), on
        ``stream`` (the current stream if None)."""
        with torch.cuda.stream(stream) if stream is not None else _nullcontext():
            self.lengths[torch.as_tensor(rows, dtype=torch.long, device=self.device)] = 0

    def sampler_kwargs(self) -> dict:
        """history / offsets / history_lengths for ``SamplePlan``."""
        return {"history": self.ids, "offsets": self.offsets, "history_lengths": self.lengths}

    def packed(self) -> tuple[torch.Tensor, torch.Tensor]:
        """The same rows as a packed history and offsets (host tensors; for
        checks)."""
        ids, offs, lens = self.ids.cpu(), self.offsets.cpu().long(), self.lengths.cpu().long()
        rows = [ids[int(offs[b]):int(offs[b] + lens[b])] for b in range(self.batch)]
        po = torch.zeros(self.batch + 1, dtype=torch.int32)
        po[1:] = torch.cumsum(lens, 0).to(torch.int32)
        return (torch.cat(rows) if rows else torch.zeros(0, dtype=torch.int32)), po


def algorithmic_bytes(batch: int, history_len: int) -> int:
    """Bytes one q3s_step_update launch must move with the history append on:
    history read (4 L) and written with one id more per row (4 (L + B)),
    offsets in and out (8 (B + 1)), int64 ids (8 B), six int32 guard fields
    read and written (48 B), the progress inputs (9 B), events and event runs
    (8 B), the event count (4).  The event list (at most 4 B) is not counted."""
    B, L = int(batch), int(history_len)
    return 4 * L + 4 * (L + B) + 8 * (B + 1) + 8 * B + 48 * B + 9 * B + 8 * B + 4


def step_update(ids: torch.Tensor, guard: StepGuard, **kw) -> list[tuple[int, int]]:
    """One epilogue step, synchronously: launch, then read the event list."""
    guard.step(ids, **kw)
    return guard.read_events()
