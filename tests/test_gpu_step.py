"""GPU parity of the per-step codec-0 epilogue (q3s_step_update) -- bit-exact.

* the reference engine loop's own decisions (tests/golden/guard_steps.npz,
  made by tests/golden/make_guard_golden.py from EngineLoop._process_step_output)
  replayed step by step with the state kept on the device;
* the oracle (oracle/q3s_oracle.py step_update) on large random batches:
  events, event runs, state, the ordered event list, and the packed history
  append (history_out / offsets_out bit-exact);
* edge cases: int32 ids, guard off, empty history rows, several guard chunks,
  a row with bad offsets (error bit, other rows intact).
"""
import numpy as np
import pytest
import torch

import q3s_oracle as O
from conftest import load_golden

pytestmark = pytest.mark.gpu


def _guard(q3s, B, dev, su, ab, ra, em):
    return q3s.StepGuard(B, eos_id=2150, token_loop_suspect_frames=su, token_loop_abort_frames=ab,
                         token_loop_min_audio_text_ratio=ra, token_loop_emergency_abort_frames=em, device=dev)


@pytest.mark.parametrize("i", range(10))
def test_step_guard_matches_reference_engine_loop(q3s_lib, cuda_device, i):
    """Scenarios 7-9 change the text count and the completion flag between
    steps (the reference raises them while a segment streams in); the host
    calls set_progress before each step, as the integration guide says."""
    import q3s
    g = load_golden("guard_steps")
    prog = g.get(f"s{i}_progress")
    su, ab, ra, em = g["scenarios"][i]
    c, tok, act = g[f"s{i}_consts"], g[f"s{i}_tokens"], g[f"s{i}_active"].astype(bool)
    S = c.shape[0]
    gd = _guard(q3s, S, cuda_device, int(su), int(ab), float(ra), int(em))
    gd.set_progress(frame_idx=c[:, 0], decode_start_frame=c[:, 1], text_tokens_consumed=c[:, 2],
                    input_complete=c[:, 3])
    stream = torch.cuda.Stream(device=cuda_device)
    for t in range(tok.shape[0]):
        ids = torch.from_numpy(tok[t]).to(cuda_device)
        if prog is not None:
            # written on the step's stream: ordered before the launch
            gd.set_progress(text_tokens_consumed=prog[t, :, 0], input_complete=prog[t, :, 1], stream=stream)
        gd.step(ids, stream=stream)
        got = gd.read_events()
        ev = gd.events.cpu().numpy()[:S]
        runs = gd.event_run.cpu().numpy()[:S]
        a = act[t]
        np.testing.assert_array_equal(ev[a], g[f"s{i}_events"][t][a], err_msg=f"step {t}")
        np.testing.assert_array_equal(runs[a], g[f"s{i}_runs"][t][a], err_msg=f"step {t}")
        assert got == [(r, int(ev[r])) for r in np.nonzero(ev)[0]]
        live = a & ((g[f"s{i}_events"][t] & (O.EVT_EOS | O.EVT_ABORT_PROGRESS | O.EVT_ABORT_EMERGENCY)) == 0)
        st = np.stack([gd.state[k].cpu().numpy()[:S] for k in O.GUARD_FIELDS], 1)
        np.testing.assert_array_equal(st[live], g[f"s{i}_state"][t][live], err_msg=f"step {t}")
    assert int(gd.error_word.item()) == 0


def _random_case(rng, B, max_len):
    lens = rng.integers(0, max_len + 1, B)
    lens[rng.random(B) < 0.05] = 0
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    hist = rng.integers(0, 3072, int(offs[-1])).astype(np.int32)
    return hist, offs


@pytest.mark.parametrize("B,steps,max_len,ids_dtype", [
    (128, 6, 2048, torch.int64),    # config-1 sizes
    (4096, 3, 4096, torch.int64),   # config-4 sizes: two guard chunks
    (2049, 4, 64, torch.int32),     # one row past a chunk; int32 ids
    (1, 5, 0, torch.int64),
])
def test_step_update_matches_oracle(q3s_lib, cuda_device, B, steps, max_len, ids_dtype):
    import q3s
    rng = np.random.default_rng(B + steps)
    su, ab, ra, em = 3, 6, 1.5, 9
    gd = _guard(q3s, B, cuda_device, su, ab, ra, em)
    frame0 = rng.integers(0, 50, B)
    start = rng.integers(0, 50, B)
    text = rng.integers(0, 30, B)
    comp = (rng.random(B) < 0.7).astype(np.int64)
    gd.set_progress(frame_idx=frame0, decode_start_frame=start, text_tokens_consumed=text, input_complete=comp)
    state = {k: np.zeros(B, np.int64) for k in O.GUARD_FIELDS}
    state["loop_token"][:] = -1
    state["frame_idx"][:] = frame0
    hist, offs = _random_case(rng, B, max_len)
    prev = rng.integers(0, 4, B)
    for t in range(steps):
        change = rng.random(B) < 0.3
        prev = np.where(change, rng.integers(0, 4, B), prev)
        ids = np.where(rng.random(B) < 0.02, 2150, prev + 100)
        dh, do = torch.from_numpy(hist).to(cuda_device), torch.from_numpy(offs).to(cuda_device)
        h_out = torch.full((hist.size + B,), -7, dtype=torch.int32, device=cuda_device)
        o_out = torch.empty(B + 1, dtype=torch.int32, device=cuda_device)
        gd.step(torch.from_numpy(ids).to(cuda_device, ids_dtype), history=dh, offsets=do, history_out=h_out,
                offsets_out=o_out)
        got = gd.read_events()
        ev, runs, h2, o2 = O.step_update(ids, eos_id=2150, state=state, suspect=su, abort=ab, emergency=em,
                                         min_ratio=ra, decode_start_frame=start, text_tokens=text,
                                         input_complete=comp, history=hist, offsets=offs)
        np.testing.assert_array_equal(gd.events.cpu().numpy()[:B], ev)
        np.testing.assert_array_equal(gd.event_run.cpu().numpy()[:B], runs)
        for k in O.GUARD_FIELDS:
            np.testing.assert_array_equal(gd.state[k].cpu().numpy()[:B], state[k], err_msg=k)
        assert got == [(int(v) >> 8, int(v) & 0xFF) for v in O.event_list(ev)]
        np.testing.assert_array_equal(h_out.cpu().numpy(), h2)
        np.testing.assert_array_equal(o_out.cpu().numpy(), o2)
        hist, offs = h2, o2
    assert int(gd.error_word.item()) == 0


def test_step_update_guard_off_counts_frames_and_eos(q3s_lib, cuda_device):
    import q3s
    gd = _guard(q3s, 5, cuda_device, 4, 0, 2.0, 20)
    ids = torch.tensor([7, 2150, 7, 7, 2150], device=cuda_device)
    for _ in range(3):
        gd.step(ids)
        assert gd.read_events() == [(1, 1), (4, 1)]
    assert gd.state["frame_idx"].cpu().tolist()[:5] == [3, 0, 3, 3, 0]
    assert gd.state["loop_run"].cpu().tolist()[:5] == [0] * 5


def test_step_update_bad_offsets_flag_only_that_row(q3s_lib, cuda_device):
    import q3s
    gd = _guard(q3s, 3, cuda_device, 4, 10, 0.0, 20)
    hist = torch.arange(10, dtype=torch.int32, device=cuda_device)
    offs = torch.tensor([0, 4, 3, 10], dtype=torch.int32, device=cuda_device)  # row 1 ends before it starts
    h_out = torch.full((13,), -7, dtype=torch.int32, device=cuda_device)
    o_out = torch.empty(4, dtype=torch.int32, device=cuda_device)
    gd.step(torch.tensor([50, 51, 52], device=cuda_device), history=hist, offsets=offs, history_out=h_out,
            offsets_out=o_out)
    torch.cuda.synchronize()
    assert int(gd.error_word.item()) & 2  # Q3S_DEVERR_OFFSETS
    assert o_out.cpu().tolist() == [0, 5, 5, 13]
    # row 0 and row 2 appended; row 1 skipped (nothing written for it)
    assert h_out.cpu().tolist() == [0, 1, 2, 3, 50, 3, 4, 5, 6, 7, 8, 9, 52]


# ---------------------------------------------------------------------------
# capacity layout: in-place append (RowHistory), O(B) bytes a step
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("B,steps,max_len,cap_extra", [
    (128, 6, 2048, 8),    # config-1 sizes: one 128-thread CTA
    (4096, 3, 4096, 4),   # config-4 sizes: one cluster of 16 x 256 threads, a row per thread
    (3, 5, 2, 2),
    (513, 3, 64, 2),      # five 128-thread CTAs, the last with one row
    (1100, 2, 64, 2),     # nine 128-thread CTAs
    (9000, 2, 64, 4),     # 1024-thread CTAs
    (20000, 2, 16, 4),    # two rows per thread
    (40000, 2, 8, 4),     # three rows per thread
    (70000, 2, 8, 4),     # past one cluster: row kernel + compaction kernel
])
def test_in_place_append_matches_oracle(q3s_lib, cuda_device, B, steps, max_len, cap_extra):
    """Guard + in-place append over several steps against the oracle; the
    rows whose region fills up stop growing and set HISTORY_FULL."""
    import q3s
    rng = np.random.default_rng(7 * B + steps)
    su, ab, ra, em = 3, 6, 1.5, 9
    gd = _guard(q3s, B, cuda_device, su, ab, ra, em)
    frame0, start, text = rng.integers(0, 50, B), rng.integers(0, 50, B), rng.integers(0, 30, B)
    comp = (rng.random(B) < 0.7).astype(np.int64)
    gd.set_progress(frame_idx=frame0, decode_start_frame=start, text_tokens_consumed=text, input_complete=comp)
    state = {k: np.zeros(B, np.int64) for k in O.GUARD_FIELDS}
    state["loop_token"][:] = -1
    state["frame_idx"][:] = frame0
    hist, offs = _random_case(rng, B, max_len)
    lens0 = np.diff(offs)
    caps = lens0 + rng.integers(0, cap_extra + 1, B)  # some rows fill up within the test
    rows = q3s.RowHistory.from_packed(torch.from_numpy(hist).to(cuda_device), torch.from_numpy(offs), caps.tolist(),
                                      device=cuda_device)
    reg = rows.offsets.cpu().numpy()
    buf = rows.ids.cpu().numpy().copy()
    lens = lens0.astype(np.int32)
    full = False
    prev = rng.integers(0, 4, B)
    for t in range(steps):
        prev = np.where(rng.random(B) < 0.3, rng.integers(0, 4, B), prev)
        ids = np.where(rng.random(B) < 0.02, 2150, prev + 100)
        gd.step(torch.from_numpy(ids).to(cuda_device), rows=rows)
        got = gd.read_events()
        ev, runs, buf, lens = O.step_update(ids, eos_id=2150, state=state, suspect=su, abort=ab, emergency=em,
                                           min_ratio=ra, decode_start_frame=start, text_tokens=text,
                                           input_complete=comp, history=buf, offsets=reg, history_lengths=lens)
        full = full or bool(((reg[:-1] + lens) == reg[1:]).any())
        np.testing.assert_array_equal(gd.events.cpu().numpy()[:B], ev)
        np.testing.assert_array_equal(gd.event_run.cpu().numpy()[:B], runs)
        for k in O.GUARD_FIELDS:
            np.testing.assert_array_equal(gd.state[k].cpu().numpy()[:B], state[k], err_msg=k)
        assert got == [(int(v) >> 8, int(v) & 0xFF) for v in O.event_list(ev)]
        np.testing.assert_array_equal(rows.lengths.cpu().numpy(), lens)
        np.testing.assert_array_equal(rows.ids.cpu().numpy()[: buf.size], buf)
    err = int(gd.error_word.item())
    assert (err & ~32) == 0
    # a row that reached its capacity reports HISTORY_FULL once it is asked to grow
    if full:
        gd.step(torch.full((B,), 5, dtype=torch.int64, device=cuda_device), rows=rows)
        torch.cuda.synchronize()
        assert int(gd.error_word.item()) & 32


def test_in_place_append_bad_region_flags_only_that_row(q3s_lib, cuda_device):
    import q3s
    gd = _guard(q3s, 3, cuda_device, 4, 10, 0.0, 20)
    rows = q3s.RowHistory(3, 4, device=cuda_device)
    rows.lengths.copy_(torch.tensor([1, 9, 0], dtype=torch.int32))  # row 1 claims more than its region
    gd.step(torch.tensor([50, 51, 52], device=cuda_device), rows=rows)
    torch.cuda.synchronize()
    assert int(gd.error_word.item()) & 2  # Q3S_DEVERR_OFFSETS
    assert rows.lengths.cpu().tolist() == [2, 9, 1]
    assert rows.ids.cpu().tolist()[:9] == [0, 50, 0, 0, 0, 0, 0, 0, 52]
