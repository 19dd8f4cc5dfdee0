"""The CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py).  CPU only."""
import numpy as np
import torch

import q3s_oracle as O
from conftest import load_golden


def _counts(hist, offs, B, V):
    tc = np.zeros((B, V), np.int64)
    for b in range(B):
        np.add.at(tc[b], hist[offs[b]:offs[b + 1]], 1)
    return tc


def test_suppress_mask_matches_reference_rule():
    m = O.suppress_mask(3072, 2150)
    assert m.sum() == 1023 and not m[2150] and m[2048] and m[3071] and not m[2047]


def test_gumbel_codebook0_f32_matches_reference_exactly():
    g = load_golden("gumbel_cb0_f32")
    B, V = g["logits"].shape
    tc = _counts(g["history"], g["offsets"], B, V)
    out = O.sample_gumbel(g["logits"], gumbel_noise=g["gumbel_noise"], temperature=g["temperature"],
                          penalty=g["penalty"], token_counts=tc, suppress=O.suppress_mask(V), topk=50)
    assert not g["tie_rows"].any()
    np.testing.assert_array_equal(out["ids"], g["ids"])
    np.testing.assert_array_equal(out["raw_topk_ids"], g["ids"])
    delta = out["updated_counts"] - tc
    np.testing.assert_array_equal(np.argwhere(delta != 0), g["delta_rc"])
    np.testing.assert_array_equal(delta[delta != 0], g["delta_val"])


def test_gumbel_codebook0_bf16_ties_counted():
    g = load_golden("gumbel_cb0_bf16")
    B, V = g["logits"].shape
    tc = _counts(g["history"], g["offsets"], B, V)
    out = O.sample_gumbel(g["logits"], gumbel_noise=g["gumbel_noise"], temperature=g["temperature"],
                          penalty=g["penalty"], token_counts=tc, suppress=O.suppress_mask(V), topk=50)
    # plain torch.topk on the oracle's processed row reproduces the reference on every row
    np.testing.assert_array_equal(out["raw_topk_ids"], g["ids"])
    # the canonical (value desc, index asc) rule differs only on tie-affected rows
    ok = ~g["tie_rows"]
    np.testing.assert_array_equal(out["ids"][ok], g["ids"][ok])
    # same presence-penalty input given as a packed history
    out2 = O.sample_gumbel(g["logits"], gumbel_noise=g["gumbel_noise"], temperature=g["temperature"],
                           penalty=g["penalty"], history=g["history"], offsets=g["offsets"],
                           suppress=O.suppress_mask(V), topk=50)
    np.testing.assert_array_equal(out2["ids"], out["ids"])


def test_cp_select_matches_reference():
    g = load_golden("cp_select")
    ids = O.select_token_cp(g["logits"], temperature=g["temperature"], gumbel_noise=g["gumbel_noise"], topk=50)
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_array_equal(O.select_token_cp(g["logits"]), g["greedy_ids"])


def test_icdf_matches_reference_sample_token():
    g = load_golden("icdf_sample_token")
    B, V = g["logits"].shape
    out = O.sample_icdf(g["logits"], uniforms=g["uniforms"], temperature=g["temperature"], top_k=g["top_k"],
                        top_p=None, penalty=g["penalty"], history=g["history"], offsets=g["offsets"],
                        suppress=O.suppress_mask(V), eos_id=2150)
    # processed logits: bit-exact with the reference chain's softmax input
    np.testing.assert_array_equal(out["processed"], g["processed"])
    ok = ~out["boundary"]
    assert ok.sum() >= B - 1
    np.testing.assert_array_equal(out["ids"][ok], g["ids"][ok])


def test_icdf_matches_hf_extended_chain():
    g = load_golden("icdf_hf_extended")
    B, V = g["logits"].shape
    out = O.sample_icdf(g["logits"], uniforms=g["uniforms"], temperature=g["temperature"], top_k=g["top_k"],
                        top_p=g["top_p"], penalty=g["penalty"], history=g["history"], offsets=g["offsets"],
                        min_new_tokens=g["min_new_tokens"], suppress=O.suppress_mask(V), eos_id=2150)
    ok = ~out["boundary"]
    np.testing.assert_array_equal(out["processed"][ok], g["processed"][ok])
    np.testing.assert_array_equal(out["ids"][ok], g["ids"][ok])
    # EOS gating: rows still below min_new_tokens must carry -inf at EOS
    lens = np.diff(g["offsets"])
    gated = lens < g["min_new_tokens"]
    assert gated.any()
    assert np.all(np.isneginf(out["processed"][gated, 2150]))


def test_icdf_greedy_rows_take_lowest_index_argmax():
    x = np.zeros((2, 16), np.float32)
    x[:, [3, 7]] = 5.0
    out = O.sample_icdf(x, uniforms=[0.5, 0.5], temperature=[0.0, 0.0])
    np.testing.assert_array_equal(out["ids"], [3, 3])
    assert np.all(out["flags"] & O.ROW_GREEDY)


def test_inverse_cdf_edges():
    s = np.log(np.array([[0.25, 0.25, 0.5]], np.float64)).astype(np.float32)
    ids, _ = O.inverse_cdf_draw(s, np.array([0.0], np.float32))
    assert ids[0] == 0
    ids, _ = O.inverse_cdf_draw(s, np.array([np.float32(1) - np.float32(2**-24)], np.float32))
    assert ids[0] == 2
    ids, bnd = O.inverse_cdf_draw(s, np.array([0.5], np.float32))
    assert ids[0] == 2 and bnd[0]  # exactly on a CDF edge: counted as a boundary draw


def test_rotate_rows_is_the_documented_producer():
    base = np.arange(12).reshape(2, 6)
    out = O.rotate_rows(base, np.array([1, 5]))
    np.testing.assert_array_equal(out[0], [1, 2, 3, 4, 5, 0])
    np.testing.assert_array_equal(out[1], [11, 6, 7, 8, 9, 10])


def test_cp_frame_chain_depends_on_previous_ids():
    rng = np.random.default_rng(0)
    base = (rng.standard_normal((3, 4, 64)) * 2.5).astype(np.float32)
    init = np.array([0, 1, 2, 3])
    a = O.cp_frame(base, mode="gumbel", ids_init=init, rotate=True)["ids"]
    for j in range(3):
        prev = init if j == 0 else a[:, j - 1]
        np.testing.assert_array_equal(a[:, j], O.rotate_rows(base[j], prev).argmax(-1))
    assert torch.is_tensor(torch.from_numpy(a))


# ---- per-step epilogue: EOS, frame counter, loop guard (reference engine loop) ----

def _replay_guard(g, i, fn):
    """Feed scenario i of guard_steps.npz step by step through ``fn`` and
    compare events, event runs and state with what the reference engine loop
    recorded (rows compared while they are active; state of rows the step
    ended is not compared)."""
    su, ab, ra, em = g["scenarios"][i]
    c, tok, act = g[f"s{i}_consts"], g[f"s{i}_tokens"], g[f"s{i}_active"].astype(bool)
    S = c.shape[0]
    state = {k: np.zeros(S, np.int64) for k in O.GUARD_FIELDS}
    state["loop_token"][:] = -1
    state["frame_idx"][:] = c[:, 0]
    cfg = dict(suspect=int(su), abort=int(ab), emergency=int(em), min_ratio=float(ra), decode_start_frame=c[:, 1],
               text_tokens=c[:, 2], input_complete=c[:, 3])
    prog = g.get(f"s{i}_progress")
    for t in range(tok.shape[0]):
        if prog is not None:  # the text count / completion the engine had at this step
            cfg = dict(cfg, text_tokens=prog[t, :, 0], input_complete=prog[t, :, 1])
        ev, runs = fn(tok[t], state, cfg)
        a = act[t]
        np.testing.assert_array_equal(ev[a], g[f"s{i}_events"][t][a], err_msg=f"scenario {i} step {t}")
        np.testing.assert_array_equal(runs[a], g[f"s{i}_runs"][t][a], err_msg=f"scenario {i} step {t}")
        live = a & ((g[f"s{i}_events"][t] & (O.EVT_EOS | O.EVT_ABORT_PROGRESS | O.EVT_ABORT_EMERGENCY)) == 0)
        st = np.stack([state[k] for k in O.GUARD_FIELDS], 1)
        np.testing.assert_array_equal(st[live], g[f"s{i}_state"][t][live], err_msg=f"scenario {i} step {t}")


def test_step_guard_oracle_matches_reference_engine_loop():
    g = load_golden("guard_steps")
    seen = 0
    for i in range(len(g["scenarios"])):
        def fn(ids, state, cfg):
            ev, runs, _, _ = O.step_update(ids, eos_id=int(g["eos_id"]), state=state, **cfg)
            return ev, runs
        _replay_guard(g, i, fn)
        seen |= int(np.bitwise_or.reduce(g[f"s{i}_events"].ravel()))
    assert seen == 63  # every event kind occurs in the fixture


def test_step_guard_thresholds_normalised_like_engine():
    assert O.guard_thresholds(4, 10, 20) == (4, 10, 20)
    assert O.guard_thresholds(9, 5, 3) == (5, 5, 5)
    assert O.guard_thresholds(4, 0, 20) == (0, 0, 0)
    assert O.guard_thresholds(-1, 6, -2) == (0, 6, 0)


def test_step_history_append_oracle():
    rng = np.random.default_rng(3)
    lens = rng.integers(0, 9, 7)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    hist = rng.integers(0, 3072, offs[-1]).astype(np.int32)
    ids = rng.integers(0, 3072, 7)
    state = {k: np.zeros(7, np.int64) for k in O.GUARD_FIELDS}
    _, _, h2, o2 = O.step_update(ids, eos_id=2150, state=state, history=hist, offsets=offs)
    for b in range(7):
        row = h2[o2[b]:o2[b + 1]]
        np.testing.assert_array_equal(row[:-1], hist[offs[b]:offs[b + 1]])
        assert row[-1] == ids[b]
    assert o2[-1] == offs[-1] + 7


def test_step_update_shards_by_rows():
    """Rows are independent: running the epilogue per rank on its row block
    (q3s.shard.row_range, offsets rebased) and shifting each rank's event rows
    by its first row reproduces the single-batch events, state and history."""
    from q3s import shard

    rng = np.random.default_rng(11)
    B, world = 37, 4
    lens = rng.integers(0, 20, B)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    hist = rng.integers(0, 3072, offs[-1]).astype(np.int32)
    cfg = dict(suspect=2, abort=3, emergency=5, min_ratio=1.0, decode_start_frame=rng.integers(0, 5, B),
               text_tokens=rng.integers(0, 4, B), input_complete=rng.integers(0, 2, B))

    def fresh(n):
        st = {k: np.zeros(n, np.int64) for k in O.GUARD_FIELDS}
        st["loop_token"][:] = -1
        return st

    full, parts = fresh(B), [fresh(shard.row_range(r, world, B)[1] - shard.row_range(r, world, B)[0])
                             for r in range(world)]
    for _ in range(6):
        ids = np.where(rng.random(B) < 0.1, 2150, rng.integers(0, 3, B) + 500)
        ev, runs, h_full, o_full = O.step_update(ids, eos_id=2150, state=full, history=hist, offsets=offs, **cfg)
        got_list, got_hist = [], []
        for r in range(world):
            a, b = shard.row_range(r, world, B)
            sub = {k: (v[a:b] if isinstance(v, np.ndarray) else v) for k, v in cfg.items()}
            o = offs[a:b + 1] - offs[a]
            e, ru, h, _ = O.step_update(ids[a:b], eos_id=2150, state=parts[r], history=hist[offs[a]:offs[b]],
                                        offsets=o, **sub)
            np.testing.assert_array_equal(e, ev[a:b])
            np.testing.assert_array_equal(ru, runs[a:b])
            for k in O.GUARD_FIELDS:
                np.testing.assert_array_equal(parts[r][k], full[k][a:b])
            got_list += [(int(v) >> 8) + a for v in O.event_list(e)]
            got_hist.append(h)
        assert got_list == [int(v) >> 8 for v in O.event_list(ev)]
        np.testing.assert_array_equal(np.concatenate(got_hist), h_full)
        hist, offs = h_full, o_full.astype(np.int64)
