"""Host side of the per-step codec-0 epilogue (``q3s_step_update``).

The reference copies every row's codebook-0 id to the host each step to test
it against the codec EOS id (engine/backend/executor.py:532-546), then runs the
frame counter and the two-stage token loop guard per slot in Python
(engine/backend/engine_loop.py:2749-2750, 2863-3080).  ``StepGuard`` keeps that
per-slot state on the GPU -- the fields of ``EngineSegment`` (loop_token,
loop_run, loop_max_run, loop_suspect_count, loop_recovery_count,
engine_loop.py:184-192) and the slot's frame_idx -- and runs two launches per
step over all rows, which also append the sampled ids to a packed history
(the packed form of ``token_counts + one_hot(id)``,
scripts/export/talker_unified_modules.py:421-422).  The host then reads one
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
    def reset_rows(self, rows: Union[Sequence[int], torch.Tensor]) -> None:
        """A new or retried segment in these rows: loop_token -1, counters 0."""
        idx = torch.as_tensor(rows, dtype=torch.long, device=self.device)
        for k in GUARD_FIELDS[:-1]:
            self.state[k].index_fill_(0, idx, -1 if k == "loop_token" else 0)

    def set_progress(self, rows: Union[Sequence[int], torch.Tensor, None] = None, *,
                     frame_idx=None, decode_start_frame=None, text_tokens_consumed=None, input_complete=None) -> None:
        """Write the progress inputs of the given rows (all rows if None)."""
        idx = (torch.arange(self.batch, device=self.device) if rows is None
               else torch.as_tensor(rows, dtype=torch.long, device=self.device))
        for t, v in ((self.state["frame_idx"], frame_idx), (self.decode_start_frame, decode_start_frame),
                     (self.text_tokens_consumed, text_tokens_consumed), (self.input_complete, input_complete)):
            if v is not None:
                t[idx] = torch.as_tensor(v, device=self.device).to(t.dtype)

    # -- the step ------------------------------------------------------------
    def step(self, ids: torch.Tensor, *, history: Optional[torch.Tensor] = None,
             offsets: Optional[torch.Tensor] = None, history_out: Optional[torch.Tensor] = None,
             offsets_out: Optional[torch.Tensor] = None, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Launch the epilogue for this step's ids ([B] int64 or int32).

        With ``history_out`` given, row b of the packed ``history`` /
        ``offsets`` is written to ``history_out`` followed by ``ids[b]``, and
        ``offsets_out = offsets + arange(B+1)``; ``history_out`` needs
        ``len(history) + B`` entries and must not overlap ``history``.
        Asynchronous on ``stream``; read results with ``read_events``.
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
        if history_out is not None:
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
