"""Generate tests/golden/guard_steps.npz from the reference engine loop itself.

The per-step codec-0 epilogue of the reference -- EOS detection
(engine/backend/executor.py:532-546), the frame counter
(engine/backend/engine_loop.py:2749-2750) and the two-stage token loop guard
(engine/backend/engine_loop.py:2863-3080, thresholds normalised at :372-387)
-- is run here by driving ``EngineLoop._process_step_output`` with synthetic
``StepOutput`` batches, in the way the reference's own guard tests do
(tests/unit/engine_core/test_engine_loop_pipeline.py:807-860): a CPU
``KVCachePool``, a stub executor, one session per stream.  Every stream is a
segment 0 of its own session, so an abort never takes the retry path (a retry
needs an earlier live segment, engine_loop.py:3443-3450) and ends the stream.

The last scenarios (DYNAMIC) also change each stream's generation progress
mid-run, as the reference does while a segment streams in
(engine/backend/engine_loop.py:930-1000 raises text_tokens_consumed,
:1027 sets input_complete): before step t the segment gets that step's text
count and completion flag, recorded as s<i>_progress [STEPS, STREAMS, 2].

Recorded per scenario, step t and stream s: whether s was active before the
step, the codec-0 token fed, the events the reference emitted (read from its
log records: "Loop suspect", "Loop recovered", "Loop deferred", "Loop
abort ... mode=progress|emergency"; EOS from the eos flag), the run length an
abort reported and the recovered run, and the segment/slot guard fields after
the step (loop_token, loop_run, loop_max_run, loop_suspect_count,
loop_recovery_count, frame_idx).

Needs the reference tree (read-only) and runs in this container only; the GPU
box uses the committed .npz.  Modules the engine imports but this path never
calls (soxr, wetext, pypinyin) are stubbed as empty modules.

    python tests/golden/make_guard_golden.py <reference checkout>   (or Q3S_REFERENCE=...)
"""
from __future__ import annotations

import asyncio
import logging
import os
import queue
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
EOS_ID = 2150

# event bits (same values as Q3S_EVT_* in include/q3s_sampler.h)
EVT_EOS, EVT_SUSPECT, EVT_RECOVERED, EVT_DEFERRED, EVT_ABORT_PROGRESS, EVT_ABORT_EMERGENCY = 1, 2, 4, 8, 16, 32

# (suspect, abort, min_audio_text_ratio, emergency) as given to EngineLoop
SCENARIOS = [
    (4, 10, 2.0, 20),   # SchedulerConfig defaults (engine/config.py:179-193)
    (4, 4, 0.0, 0),     # test_loop_abort_after_threshold_*: abort at 4, no progress gate
    (0, 6, 0.0, 0),     # suspect stage off
    (3, 8, 1.5, 12),
    (9, 5, 1.0, 3),     # suspect clamped to abort, emergency raised to abort
    (4, 0, 2.0, 20),    # guard off: only EOS and the frame counter
    (2, 7, 3.25, 0),    # progress gate, no emergency stage
]
# scenarios whose text count and completion flag change between steps
DYNAMIC = [
    (4, 10, 2.0, 20),
    (3, 6, 1.0, 0),
    (2, 5, 0.5, 12),
]
STREAMS = 16
STEPS = 64


def _progress_schedule(rng: np.random.Generator, text0: int, complete0: bool):
    """Per-step (text_tokens_consumed, input_complete) of one stream: text
    arrives in bursts until the input completes at a random step (or was
    complete from the start)."""
    text = np.empty(STEPS, np.int64)
    comp = np.empty(STEPS, np.int64)
    t_done = 0 if complete0 else int(rng.integers(1, STEPS + 8))
    cur = text0
    for t in range(STEPS):
        done = t >= t_done
        if not done and rng.random() < 0.35:
            cur += int(rng.integers(1, 4))
        text[t], comp[t] = cur, int(done)
    return text, comp


def _import_reference(root: Path):
    for name in ("soxr", "wetext", "pypinyin"):
        if name not in sys.modules:
            sys.modules[name] = types.ModuleType(name)
    for p in (root / "client" / "src", root):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))
    import torch  # noqa: F401  (the engine imports it)
    from engine.backend.engine_loop import EngineLoop, EngineSegment
    from engine.backend.executor import StepOutput
    from engine.backend.kv_cache_pool import KVCachePool, ModelConfig
    from engine.core.types import EngineRequest, RequestType

    return EngineLoop, EngineSegment, StepOutput, KVCachePool, ModelConfig, EngineRequest, RequestType


class _Events(logging.Handler):
    """Collects the guard's log records per session id."""

    def __init__(self):
        super().__init__(level=logging.DEBUG)
        self.rows: dict[str, list[tuple[int, int]]] = {}

    def emit(self, record):
        msg = record.msg if isinstance(record.msg, str) else ""
        args = record.args if isinstance(record.args, tuple) else ()
        if not args:
            return
        sid = args[0]
        if msg.startswith("Loop suspect"):
            self.rows.setdefault(sid, []).append((EVT_SUSPECT, 0))
        elif msg.startswith("Loop recovered"):
            self.rows.setdefault(sid, []).append((EVT_RECOVERED, int(args[3])))  # recovered run
        elif msg.startswith("Loop deferred"):
            self.rows.setdefault(sid, []).append((EVT_DEFERRED, 0))
        elif msg.startswith("Loop abort"):
            mode = args[7]
            bit = EVT_ABORT_PROGRESS if mode == "progress" else EVT_ABORT_EMERGENCY
            self.rows.setdefault(sid, []).append((bit, int(args[3])))  # run at abort


def _stream_inputs(rng: np.random.Generator):
    """Per-stream constants and a token sequence with runs and returns."""
    frame0 = int(rng.integers(0, 120))
    start = int(rng.integers(0, frame0 + 1))
    text = int(rng.choice([0, 1, int(rng.integers(2, 40)), int(rng.integers(40, 200))]))
    complete = bool(rng.random() < 0.7)
    p_repeat = float(rng.choice([0.3, 0.75, 0.92, 0.985]))
    p_eos = float(rng.choice([0.0, 0.0, 0.01, 0.04]))
    alphabet = rng.choice(2048, size=int(rng.integers(2, 7)), replace=False)
    toks = np.empty(STEPS, np.int64)
    prev = int(rng.choice(alphabet))
    for t in range(STEPS):
        if rng.random() < p_eos:
            toks[t] = EOS_ID
            continue
        if rng.random() >= p_repeat:
            prev = int(rng.choice(alphabet))
        toks[t] = prev
    return frame0, start, text, complete, toks


def run_scenario(ref, scen, seed, dynamic=False):
    EngineLoop, EngineSegment, StepOutput, KVCachePool, ModelConfig, EngineRequest, RequestType = ref
    import torch

    suspect, abort, ratio, emergency = scen
    rng = np.random.default_rng(seed)
    mc = ModelConfig(num_layers=2, kv_heads=2, head_dim=4, max_seq_len=4096, n_c2w_layers=2, c2w_kv_heads=2,
                     c2w_head_dim=4, c2w_sliding_window=8)
    pool = KVCachePool(max_slots=STREAMS, config=mc, device=torch.device("cpu"), preallocate=False)

    class StubExecutor:
        kv_pool = pool
        _device = torch.device("cpu")
        _config = mc

    loop = asyncio.new_event_loop()
    el = EngineLoop(engine_inbox=queue.Queue(), async_loop=loop, executor=StubExecutor(), max_batch_size=STREAMS,
                    token_loop_suspect_frames=suspect, token_loop_abort_frames=abort,
                    token_loop_min_audio_text_ratio=ratio, token_loop_emergency_abort_frames=emergency,
                    token_loop_max_retries=0)
    audio = (np.ones(1920, dtype=np.float32) * 0.25).tobytes()
    segs, slots = [], []
    consts = np.zeros((STREAMS, 4), np.int64)  # frame0, decode_start_frame, text_tokens, input_complete
    tokens = np.zeros((STEPS, STREAMS), np.int64)
    prng = np.random.default_rng(seed + 50000)  # progress schedules (dynamic scenarios only)
    prog_text = np.zeros((STEPS, STREAMS), np.int64)
    prog_comp = np.zeros((STEPS, STREAMS), np.int64)
    for s in range(STREAMS):
        sid = f"s{s}"
        el._handle_request(EngineRequest(type=RequestType.NEW_SESSION, session_id=sid, result_queue=queue.Queue()))
        slot = pool.allocate(f"{sid}:0")
        seg = EngineSegment(sid, 0)
        seg.slot = slot
        seg.state = "active"
        el._groups[sid].segments[0] = seg
        el._seg_by_slot[slot.slot_id] = seg
        frame0, start, text, complete, toks = _stream_inputs(rng)
        slot.frame_idx = frame0
        seg.decode_start_frame = start
        seg.text_tokens_consumed = text
        seg.input_complete = complete
        consts[s] = (frame0, start, text, int(complete))
        tokens[:, s] = toks
        if dynamic:
            prog_text[:, s], prog_comp[:, s] = _progress_schedule(prng, text, complete)
        segs.append(seg)
        slots.append(slot)

    handler = _Events()
    lg = logging.getLogger("engine.backend.engine_loop")
    old_level = lg.level
    lg.setLevel(logging.DEBUG)
    lg.addHandler(handler)
    active = np.zeros((STEPS, STREAMS), np.uint8)
    events = np.zeros((STEPS, STREAMS), np.int32)
    runs = np.zeros((STEPS, STREAMS), np.int32)   # recovered run (RECOVERED) or run at abort
    state = np.zeros((STEPS, STREAMS, 6), np.int64)
    alive = [True] * STREAMS
    try:
        for t in range(STEPS):
            rows = [s for s in range(STREAMS) if alive[s]]
            if not rows:
                break
            handler.rows.clear()
            if dynamic:
                for s in rows:
                    segs[s].text_tokens_consumed = int(prog_text[t, s])
                    segs[s].input_complete = bool(prog_comp[t, s])
            out = StepOutput(slots=[slots[s] for s in rows],
                             eos_flags=[bool(tokens[t, s] == EOS_ID) for s in rows],
                             tokens=[int(tokens[t, s]) for s in rows], audio_chunks=[audio for _ in rows],
                             split_c2w_conv=[[] for _ in rows], split_c2w_transconv=[[] for _ in rows])
            el._process_step_output(out)
            for s in rows:
                active[t, s] = 1
                bits = EVT_EOS if tokens[t, s] == EOS_ID else 0
                for bit, r in handler.rows.get(f"s{s}", []):
                    bits |= bit
                    if bit in (EVT_RECOVERED, EVT_ABORT_PROGRESS, EVT_ABORT_EMERGENCY):
                        runs[t, s] = r
                events[t, s] = bits
                seg, slot = segs[s], slots[s]
                state[t, s] = (seg.loop_token, seg.loop_run, seg.loop_max_run, seg.loop_suspect_count,
                               seg.loop_recovery_count, slot.frame_idx)
                if bits & (EVT_EOS | EVT_ABORT_PROGRESS | EVT_ABORT_EMERGENCY):
                    assert seg.state == "done", (scen, t, s, bits, seg.state)
                    alive[s] = False
                else:
                    assert seg.state == "active", (scen, t, s, bits, seg.state)
    finally:
        lg.removeHandler(handler)
        lg.setLevel(old_level)
        loop.close()
    r = dict(consts=consts, tokens=tokens, active=active, events=events, runs=runs, state=state)
    if dynamic:
        r["progress"] = np.stack([prog_text, prog_comp], axis=-1)
    return r


def main():
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("Q3S_REFERENCE")
    if not arg:
        sys.exit("usage: make_guard_golden.py <reference checkout> (or set Q3S_REFERENCE)")
    root = Path(arg)
    ref = _import_reference(root)
    allscen = SCENARIOS + DYNAMIC
    out = {"scenarios": np.array(allscen, np.float64), "eos_id": np.int64(EOS_ID),
           "dynamic": np.array([0] * len(SCENARIOS) + [1] * len(DYNAMIC), np.int64)}
    for i, scen in enumerate(allscen):
        dyn = i >= len(SCENARIOS)
        r = run_scenario(ref, scen, seed=(7100 + i) if not dyn else (7300 + i), dynamic=dyn)
        for k, v in r.items():
            out[f"s{i}_{k}"] = v
        ev = r["events"]
        print(f"scenario {scen}{' (progress changes mid-run)' if dyn else ''}: eos={int((ev & EVT_EOS).astype(bool).sum())} "
              f"suspect={int((ev & EVT_SUSPECT).astype(bool).sum())} "
              f"recovered={int((ev & EVT_RECOVERED).astype(bool).sum())} "
              f"deferred={int((ev & EVT_DEFERRED).astype(bool).sum())} "
              f"abort_p={int((ev & EVT_ABORT_PROGRESS).astype(bool).sum())} "
              f"abort_e={int((ev & EVT_ABORT_EMERGENCY).astype(bool).sum())}")
    np.savez_compressed(HERE / "guard_steps.npz", **out)


if __name__ == "__main__":
    main()
