"""CUDA kernels (through the C ABI) against the CPU oracle and the reference's
golden vectors.

Tolerances (stated by the benchmark contract):
  * sampled ids bit-exact, except rows the oracle or the kernel flags as a
    boundary draw (within 1e-6 of a CDF edge or of the top-p cut), which are
    counted and bounded;
  * processed logits within 1e-5 relative in fp32 (they are in fact compared
    bit-exactly where both sides apply the same IEEE operations).
"""
import numpy as np
import pytest
import torch

import q3s
import q3s_oracle as O
from conftest import load_golden
from q3s import _lib, workloads

pytestmark = pytest.mark.gpu

RTOL = 1e-5
MAX_BOUNDARY_FRACTION = 0.02
# the shared-memory row kernel with 1, 2, 4, 8 and 12 or 16 warps per row
WARP_POLICIES = ["w1", "w2", "w4", "w8", "wmax", "lean"]


def _dev(x, dev):
    return torch.as_tensor(np.ascontiguousarray(x)).to(dev)


def _proc_close(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    same_inf = np.isinf(a) == np.isinf(b)
    fin = np.isfinite(a) & np.isfinite(b)
    return bool(np.all(same_inf) and np.all(a[np.isinf(a)] == b[np.isinf(a)])
                and np.all(np.abs(a[fin] - b[fin]) <= RTOL * np.abs(b[fin]) + 1e-30))


def run_icdf_batch(b: workloads.Batch, dev, *, processed=True):
    g = b.to(dev)
    B, V = g.B, g.V
    proc = torch.empty(B, V, dtype=torch.float32, device=dev) if processed else None
    flags = torch.zeros(B, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ids = q3s.sample_packed(g.logits, g.history, g.offsets, uniforms=g.uniforms, temperature=g.temperature,
                            top_k=g.top_k, top_p=g.top_p, penalty=g.penalty, min_new_tokens=g.min_new_tokens,
                            suppress=g.suppress, eos_id=g.eos_id, processed=proc, row_flags=flags,
                            error_word=err)
    torch.cuda.synchronize()
    return (ids.cpu().numpy(), None if proc is None else proc.cpu().numpy(), flags.cpu().numpy(),
            int(err.item()))


def oracle_icdf(b: workloads.Batch):
    return O.sample_icdf(b.logits, uniforms=b.uniforms.numpy(), temperature=b.temperature.numpy(),
                         top_k=b.top_k.numpy(), top_p=b.top_p.numpy(), penalty=b.penalty.numpy(),
                         history=b.history.numpy(), offsets=b.offsets.numpy(),
                         min_new_tokens=b.min_new_tokens.numpy(), suppress=b.suppress.numpy(), eos_id=b.eos_id)


def assert_ids_match(ids, ref, kflags, label, max_frac=None):
    """Bit-exact ids except on boundary rows (flagged by the oracle or the
    kernel); a boundary row that differs must still pick an id the oracle's
    processed row kept.  ``max_frac`` bounds the boundary share for random
    inputs (edge-case tests sit on CDF edges by construction)."""
    bnd = ref["boundary"] | ((kflags & (_lib.ROW_DRAW_BOUNDARY | _lib.ROW_TOPP_BOUNDARY)) != 0)
    bad = (ids != ref["ids"]) & ~bnd
    assert not bad.any(), f"{label}: {bad.sum()} non-boundary mismatches at rows {np.nonzero(bad)[0][:10]}"
    diff = np.nonzero((ids != ref["ids"]) & bnd)[0]
    if "processed" in ref:
        for r in diff:
            assert np.isfinite(ref["processed"][r, ids[r]]), f"{label}: row {r} drew a filtered id {ids[r]}"
    if max_frac is not None:
        assert bnd.mean() <= max_frac + 1.0 / len(ids), f"{label}: {bnd.sum()} boundary rows"
    return int(bnd.sum()), int(len(diff))


# ---------------------------------------------------------------------------
# golden vectors from the reference
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", ["gumbel_cb0_f32", "gumbel_cb0_bf16"])
@pytest.mark.parametrize("inplace", [False, True])
def test_codebook0_gumbel_matches_reference_golden(cuda_device, q3s_lib, name, inplace):
    g = load_golden(name)
    B, V = g["logits"].shape
    tc = np.zeros((B, V), np.int64)
    for b in range(B):
        np.add.at(tc[b], g["history"][g["offsets"][b]:g["offsets"][b + 1]], 1)
    logits = g["logits_bf16"].to(cuda_device) if "logits_bf16" in g else _dev(g["logits"], cuda_device)
    tcd = _dev(tc, cuda_device)
    sampler = q3s.CodecSampler(device=cuda_device)
    ids, upd = sampler.codebook0(logits, tcd, _dev(g["gumbel_noise"], cuda_device),
                                 _dev(g["temperature"].reshape(B, 1), cuda_device),
                                 _dev(g["penalty"].reshape(B, 1), cuda_device), inplace=inplace)
    ids = ids.cpu().numpy()
    ok = ~g["tie_rows"]
    np.testing.assert_array_equal(ids[ok], g["ids"][ok])
    oracle = O.sample_gumbel(g["logits"], gumbel_noise=g["gumbel_noise"], temperature=g["temperature"],
                             penalty=g["penalty"], token_counts=tc, suppress=O.suppress_mask(V), topk=50)
    np.testing.assert_array_equal(ids, oracle["ids"])  # canonical tie rule on every row
    np.testing.assert_array_equal(upd.cpu().numpy(), oracle["updated_counts"])
    if inplace:
        assert upd.data_ptr() == tcd.data_ptr()


def test_cp_select_matches_reference_golden(cuda_device, q3s_lib):
    g = load_golden("cp_select")
    B = g["logits"].shape[0]
    lg = _dev(g["logits"], cuda_device).reshape(B, 1, -1)
    ids = q3s.select_token(lg, temperature=_dev(g["temperature"].reshape(B, 1), cuda_device),
                           gumbel_noise=_dev(g["gumbel_noise"], cuda_device))
    np.testing.assert_array_equal(ids.cpu().numpy(), g["ids"])
    np.testing.assert_array_equal(q3s.select_token(lg).cpu().numpy(), g["greedy_ids"])


def test_icdf_matches_reference_sample_token_golden(cuda_device, q3s_lib):
    g = load_golden("icdf_sample_token")
    B, V = g["logits"].shape
    ref = O.sample_icdf(g["logits"], uniforms=g["uniforms"], temperature=g["temperature"], top_k=g["top_k"],
                        penalty=g["penalty"], history=g["history"], offsets=g["offsets"],
                        suppress=O.suppress_mask(V), eos_id=2150)
    proc = torch.empty(B, V, dtype=torch.float32, device=cuda_device)
    flags = torch.zeros(B, dtype=torch.int32, device=cuda_device)
    ids = q3s.sample_packed(g["logits_bf16"].to(cuda_device), _dev(g["history"], cuda_device),
                            _dev(g["offsets"], cuda_device), uniforms=_dev(g["uniforms"], cuda_device),
                            temperature=_dev(g["temperature"], cuda_device), top_k=_dev(g["top_k"], cuda_device),
                            top_p=1.0, penalty=_dev(g["penalty"], cuda_device), min_new_tokens=0,
                            suppress=q3s.suppress_mask(V, 2150, cuda_device), processed=proc, row_flags=flags)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(proc.cpu().numpy(), g["processed"])  # bit-exact
    assert_ids_match(ids.cpu().numpy(), {"ids": g["ids"], "boundary": ref["boundary"]}, flags.cpu().numpy(),
                     "sample_token golden")


def test_icdf_matches_hf_extended_golden(cuda_device, q3s_lib):
    g = load_golden("icdf_hf_extended")
    B, V = g["logits"].shape
    ref = O.sample_icdf(g["logits"], uniforms=g["uniforms"], temperature=g["temperature"], top_k=g["top_k"],
                        top_p=g["top_p"], penalty=g["penalty"], history=g["history"], offsets=g["offsets"],
                        min_new_tokens=g["min_new_tokens"], suppress=O.suppress_mask(V), eos_id=2150)
    proc = torch.empty(B, V, dtype=torch.float32, device=cuda_device)
    flags = torch.zeros(B, dtype=torch.int32, device=cuda_device)
    ids = q3s.sample_packed(g["logits_bf16"].to(cuda_device), _dev(g["history"], cuda_device),
                            _dev(g["offsets"], cuda_device), uniforms=_dev(g["uniforms"], cuda_device),
                            temperature=_dev(g["temperature"], cuda_device), top_k=_dev(g["top_k"], cuda_device),
                            top_p=_dev(g["top_p"], cuda_device), penalty=_dev(g["penalty"], cuda_device),
                            min_new_tokens=_dev(g["min_new_tokens"], cuda_device),
                            suppress=q3s.suppress_mask(V, 2150, cuda_device), processed=proc, row_flags=flags)
    torch.cuda.synchronize()
    kf = flags.cpu().numpy()
    ok = ~(ref["boundary"] | ((kf & 3) != 0))
    assert _proc_close(proc.cpu().numpy()[ok], g["processed"][ok])
    assert_ids_match(ids.cpu().numpy(), {"ids": g["ids"], "boundary": ~ok}, kf, "hf extended golden")


# ---------------------------------------------------------------------------
# benchmark configurations against the oracle
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("cfg,rows", [(0, None), (1, None), (3, None), (4, None)])
def test_configs_match_oracle(cuda_device, q3s_lib, cfg, rows):
    b = workloads.make_batch(cfg, rows=rows)
    ids, proc, kf, err = run_icdf_batch(b, cuda_device)
    ref = oracle_icdf(b)
    assert err == 0
    nb, nbm = assert_ids_match(ids, ref, kf, f"config {cfg}", max_frac=MAX_BOUNDARY_FRACTION)
    ok = ~(ref["boundary"] | ((kf & 3) != 0))
    assert _proc_close(proc[ok], ref["processed"][ok])
    greedy = b.temperature.numpy() <= 0
    assert np.all((kf[greedy] & _lib.ROW_GREEDY) != 0)
    print(f"config {cfg}: {len(ids)} rows, {nb} boundary rows, {nbm} of them differ")


def test_gumbel_packed_matches_oracle(cuda_device, q3s_lib):
    b = workloads.make_batch(1)
    g = b.to(cuda_device)
    ids = q3s.sample_packed(g.logits, g.history, g.offsets, mode="gumbel", topk=50, gumbel_noise=g.gumbel_noise,
                            temperature=g.temperature, penalty=g.penalty, suppress=g.suppress, eos_id=b.eos_id,
                            min_new_tokens=g.min_new_tokens)
    ref = O.sample_gumbel(b.logits, gumbel_noise=b.gumbel_noise.numpy(), temperature=b.temperature.numpy(),
                          penalty=b.penalty.numpy(), history=b.history.numpy(), offsets=b.offsets.numpy(),
                          suppress=b.suppress.numpy(), topk=50, eos_id=b.eos_id,
                          min_new_tokens=b.min_new_tokens.numpy())
    np.testing.assert_array_equal(ids.cpu().numpy(), ref["ids"])


def test_deterministic_across_runs(cuda_device, q3s_lib):
    b = workloads.make_batch(4, rows=(0, 256))
    a1, p1, f1, _ = run_icdf_batch(b, cuda_device)
    a2, p2, f2, _ = run_icdf_batch(b, cuda_device)
    np.testing.assert_array_equal(a1, a2)
    np.testing.assert_array_equal(p1.view(np.uint32), p2.view(np.uint32))
    np.testing.assert_array_equal(f1, f2)


# ---------------------------------------------------------------------------
# edge cases
# ---------------------------------------------------------------------------

def _icdf_case(dev, logits, *, T=1.0, k=0, p=1.0, pen=1.0, hist=None, u=None, mn=0, eos=-1, suppress=None):
    logits = np.asarray(logits, np.float32)
    B, V = logits.shape
    rng = np.random.default_rng(0)
    u = rng.random(B).astype(np.float32) if u is None else np.asarray(u, np.float32)
    if hist is None:
        hist = [np.zeros(0, np.int32)] * B
    offs = np.zeros(B + 1, np.int32)
    offs[1:] = np.cumsum([len(h) for h in hist])
    flat = np.concatenate(hist).astype(np.int32) if offs[-1] else np.zeros(1, np.int32)
    ref = O.sample_icdf(logits, uniforms=u, temperature=np.full(B, T, np.float32), top_k=np.full(B, k),
                        top_p=np.full(B, p, np.float32), penalty=np.full(B, pen, np.float32),
                        history=flat[:offs[-1]], offsets=offs, min_new_tokens=np.full(B, mn),
                        suppress=suppress, eos_id=eos)
    proc = torch.empty(B, V, dtype=torch.float32, device=dev)
    flags = torch.zeros(B, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ids = q3s.sample_packed(_dev(logits, dev), _dev(flat, dev), _dev(offs, dev), uniforms=_dev(u, dev),
                            temperature=T, top_k=k, top_p=p, penalty=pen, min_new_tokens=mn, eos_id=eos,
                            suppress=None if suppress is None else _dev(suppress, dev), processed=proc,
                            row_flags=flags, error_word=err)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), proc.cpu().numpy(), flags.cpu().numpy(), int(err.item()), ref


@pytest.mark.parametrize("V", [1, 7, 64, 1000, 2048, 3072, 4100, 8192])
@pytest.mark.parametrize("k,p", [(0, 1.0), (50, 1.0), (50, 0.9), (0, 0.95), (1, 1.0)])
def test_vocab_sizes_and_filters(cuda_device, q3s_lib, V, k, p):
    rng = np.random.default_rng(V * 7 + k)
    x = (rng.standard_normal((6, V)) * 2.0).astype(np.float32)
    ids, proc, kf, err, ref = _icdf_case(cuda_device, x, T=0.8, k=k, p=p)
    assert err == 0
    assert_ids_match(ids, ref, kf, f"V={V} k={k} p={p}", max_frac=0.5)
    ok = ~(ref["boundary"] | ((kf & 3) != 0))
    assert _proc_close(proc[ok], ref["processed"][ok])


def test_heavy_ties_and_top_k_boundary_ties(cuda_device, q3s_lib):
    x = np.zeros((4, 512), np.float32)
    x[:, :100] = 1.0           # 100-way tie across the k=50 boundary: HF keeps all of them
    x[1] = 0.0                 # a fully flat row
    x[2, ::3] = -np.inf
    ids, proc, kf, err, ref = _icdf_case(cuda_device, x, k=50, p=0.7)
    assert_ids_match(ids, ref, kf, "ties")
    ok = ~(ref["boundary"] | ((kf & 3) != 0))
    assert _proc_close(proc[ok], ref["processed"][ok])


def test_extreme_uniforms_and_tiny_top_p(cuda_device, q3s_lib):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((6, 3072)) * 3).astype(np.float32)
    u = np.array([0.0, 0.0, np.float32(1 - 2**-24), np.float32(1 - 2**-24), 0.5, 0.25], np.float32)
    ids, _, kf, _, ref = _icdf_case(cuda_device, x, k=0, p=1e-4, u=u)
    np.testing.assert_array_equal(ids, x.argmax(-1))  # top-p this small keeps only the top entry
    ids, _, kf, _, ref = _icdf_case(cuda_device, x, k=100, p=1.0, u=u)
    assert_ids_match(ids, ref, kf, "extreme uniforms")


def test_penalty_eos_gate_and_suppress(cuda_device, q3s_lib):
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((8, 3072)) * 3).astype(np.float32)
    x[:, 2150] = 50.0  # EOS would win everywhere unless gated
    hist = [rng.integers(0, 3072, n).astype(np.int32) for n in (0, 1, 5, 9, 30, 64, 65, 200)]
    sup = O.suppress_mask(3072, 2150)
    ids, proc, kf, err, ref = _icdf_case(cuda_device, x, T=0.9, k=50, p=0.9, pen=1.3, hist=hist, mn=64,
                                         eos=2150, suppress=sup)
    assert err == 0
    assert_ids_match(ids, ref, kf, "penalty/eos")
    lens = np.array([len(h) for h in hist])
    assert np.all(ids[lens < 64] != 2150) and np.all(ids[lens >= 64] == 2150)
    ok = ~(ref["boundary"] | ((kf & 3) != 0))
    assert _proc_close(proc[ok], ref["processed"][ok])


def test_bad_history_is_reported_not_faulted(cuda_device, q3s_lib):
    x = np.zeros((2, 256), np.float32)
    hist = [np.array([5, 300, -1], np.int32), np.array([7], np.int32)]
    ids, _, _, err, _ = _icdf_case(cuda_device, x, hist=hist)
    assert err & _lib.DEVERR_HISTORY_ID
    dev = cuda_device
    err_t = torch.zeros(1, dtype=torch.int32, device=dev)
    bad_offs = torch.tensor([0, 5, 2], dtype=torch.int32, device=dev)  # non-monotone
    q3s.sample_packed(torch.zeros(2, 256, device=dev), torch.zeros(5, dtype=torch.int32, device=dev), bad_offs,
                      uniforms=torch.zeros(2, device=dev), error_word=err_t)
    torch.cuda.synchronize()
    assert int(err_t.item()) & _lib.DEVERR_OFFSETS


def test_strided_and_3d_logits(cuda_device, q3s_lib):
    dev = cuda_device
    rng = np.random.default_rng(5)
    full = (rng.standard_normal((4, 3, 3072)) * 3).astype(np.float32)
    noise = rng.gumbel(size=(4, 50)).astype(np.float32)
    tc = np.zeros((4, 3072), np.int64)
    ids, _ = q3s.sample_codebook0(_dev(full, dev), _dev(tc, dev), _dev(noise, dev), 0.9, 1.05)
    ref = O.sample_gumbel(full[:, -1, :], gumbel_noise=noise, temperature=np.full(4, 0.9, np.float32),
                          penalty=np.full(4, 1.05, np.float32), token_counts=tc, topk=50)
    np.testing.assert_array_equal(ids.cpu().numpy(), ref["ids"])


def test_col_shift_reads_rotated_rows(cuda_device, q3s_lib):
    dev = cuda_device
    rng = np.random.default_rng(6)
    base = torch.from_numpy((rng.standard_normal((16, 2048)) * 2.5).astype(np.float32)).to(torch.bfloat16)
    shift = rng.integers(0, 2048, 16)
    noise = rng.gumbel(size=(16, 50)).astype(np.float32)
    plan = q3s.SamplePlan(base.to(dev), mode="gumbel", topk=50, temperature=0.9,
                          gumbel_noise=_dev(noise, dev), col_shift=_dev(shift, dev))
    plan.launch()
    ref = O.select_token_cp(O.rotate_rows(base.float().numpy(), shift), temperature=np.full(16, 0.9, np.float32),
                            gumbel_noise=noise, topk=50)
    np.testing.assert_array_equal(plan.ids.cpu().numpy(), ref)


# ---------------------------------------------------------------------------
# code-predictor frame
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("mode", ["gumbel", "icdf", "greedy"])
@pytest.mark.parametrize("rotate", [True, False])
def test_cp_frame_matches_oracle_chain(cuda_device, q3s_lib, mode, rotate):
    f = workloads.make_cp_frame()
    g = f.to(cuda_device)
    flags = torch.zeros(f.B, f.S, dtype=torch.int32, device=cuda_device)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ids = q3s.sample_cp_frame(g.base, mode="icdf" if mode == "icdf" else "gumbel", ids_init=g.ids_init,
                              rotate=rotate, temperature=g.temperature, topk=50, top_p=1.0,
                              gumbel_noise=g.gumbel_noise if mode == "gumbel" else None,
                              uniforms=g.uniforms, row_flags=flags, error_word=err).cpu().numpy()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = O.cp_frame(f.base.float().numpy(), mode="icdf" if mode == "icdf" else "gumbel",
                     ids_init=f.ids_init.numpy(), rotate=rotate, temperature=f.temperature.numpy(), topk=50,
                     gumbel_noise=f.gumbel_noise.numpy() if mode == "gumbel" else None,
                     uniforms=f.uniforms.numpy())
    if mode == "icdf":
        # a boundary draw in stage j legitimately changes every later stage of that row
        kf = flags.cpu().numpy()
        bnd = ref["boundary"] | ((kf & 3) != 0)
        first_bnd = np.where(bnd.any(1), bnd.argmax(1), f.S)
        for b in range(f.B):
            np.testing.assert_array_equal(ids[b, :first_bnd[b]], ref["ids"][b, :first_bnd[b]])
        assert (first_bnd < f.S).mean() < 0.1
    else:
        np.testing.assert_array_equal(ids, ref["ids"])


def test_cp_frame_equals_fifteen_single_stage_launches(cuda_device, q3s_lib):
    f = workloads.make_cp_frame()
    g = f.to(cuda_device)
    frame = q3s.sample_cp_frame(g.base, mode="gumbel", ids_init=g.ids_init, rotate=True,
                                temperature=g.temperature, topk=50, gumbel_noise=g.gumbel_noise)
    prev = g.ids_init.clone()
    outs = []
    for j in range(f.S):
        plan = q3s.SamplePlan(g.base[j], mode="gumbel", topk=50, temperature=g.temperature,
                              gumbel_noise=g.gumbel_noise[:, j, :], col_shift=prev)
        plan.launch()
        prev = plan.ids
        outs.append(prev)
    np.testing.assert_array_equal(torch.stack(outs, 1).cpu().numpy(), frame.cpu().numpy())


@pytest.mark.parametrize("case", ["ties", "spread", "mixed", "fp32", "tiny", "extreme_t", "wide"])
def test_cp_frame_fast_path_and_its_fallbacks(cuda_device, q3s_lib, case):
    """The Gumbel frame kernel (auto policy) against the oracle chain and the
    CTA-per-row frame kernel, on rows that leave its fast pattern: massive
    ties (more than 256 entries down to the K-th's bin) and widely spread
    values (the K-th 32 or more below the maximum), alone and mixed with
    ordinary rows, bf16 and fp32; on candidates whose v / T leaves the
    reciprocal's window (tiny and signed-zero values, temperatures outside
    [2^-20, 2^20]); and on more rows than SMs (two CTAs per SM)."""
    rng = np.random.default_rng({"ties": 1, "spread": 2, "mixed": 3, "fp32": 4, "tiny": 5, "extreme_t": 6,
                                 "wide": 7}[case])
    S, B, V = 5, (400 if case == "wide" else 40), 2048
    base = (rng.standard_normal((S, B, V)) * 2.5).astype(np.float32)
    if case == "tiny":
        # rows far below zero with 80 planted entries at tiny magnitudes and
        # both zeros, all of them inside the top 50's reach
        base[:, ::2, :] -= 30.0
        tiny = np.array([1e-20, -1e-20, 3e-19, -7e-22, 0.0, -0.0, 2e-30, -5e-25], np.float32)
        base[:, ::2, 100:180] = np.resize(tiny, 80)
    if case in ("ties", "mixed"):
        rows = slice(None) if case == "ties" else slice(0, B, 3)
        base[:, rows, :] = np.round(base[:, rows, :] * 2) / 2  # a few hundred entries share each top value
        base[:, rows, :600] = np.maximum(base[:, rows, :600], 4.0)
    if case in ("spread", "mixed"):
        rows = slice(None) if case == "spread" else slice(1, B, 3)
        base[:, rows, :] *= 40.0
    bf16 = case != "fp32"
    bt = torch.from_numpy(base)
    if bf16:
        bt = bt.to(torch.bfloat16)
        base = bt.float().numpy()
    init = rng.integers(0, V, B)
    T = rng.uniform(0.6, 1.0, B).astype(np.float32)
    if case == "extreme_t":
        T[::3] = 1e-7
        T[1::3] = 3e6
    u = rng.random((B, S, 50)).astype(np.float32)
    from q3s.philox import gumbel_from_uniforms
    noise = gumbel_from_uniforms(u)
    ref = O.cp_frame(base, mode="gumbel", ids_init=init, rotate=True, temperature=T, gumbel_noise=noise)
    outs = {}
    for policy in ("auto", "cta"):
        err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        with q3s.kernel_policy(policy):
            ids = q3s.sample_cp_frame(bt.to(cuda_device), mode="gumbel", ids_init=_dev(init, cuda_device), rotate=True,
                                      temperature=_dev(T, cuda_device), topk=50,
                                      gumbel_noise=_dev(noise, cuda_device), error_word=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0, policy
        outs[policy] = ids.cpu().numpy()
    np.testing.assert_array_equal(outs["auto"], ref["ids"])
    np.testing.assert_array_equal(outs["cta"], ref["ids"])


# ---------------------------------------------------------------------------
# warp-per-row kernels (forced by policy; "auto" picks them for large batches)
# ---------------------------------------------------------------------------

def _packed_args(b: workloads.Batch, dev):
    g = b.to(dev)
    return g, dict(uniforms=g.uniforms, temperature=g.temperature, top_k=g.top_k, top_p=g.top_p,
                   penalty=g.penalty, min_new_tokens=g.min_new_tokens, suppress=g.suppress, eos_id=g.eos_id)


def _run_policy(policy, g, kw, dev, processed=False):
    flags = torch.zeros(g.B, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    proc = torch.full((g.B, g.V), float("nan"), dtype=torch.float32, device=dev) if processed else None
    with q3s.kernel_policy(policy):
        ids = q3s.sample_packed(g.logits, g.history, g.offsets, row_flags=flags, error_word=err, processed=proc,
                                **kw)
    torch.cuda.synchronize()
    out = (ids.cpu().numpy(), flags.cpu().numpy(), int(err.item()))
    return out + (proc.cpu().numpy(),) if processed else out


@pytest.fixture(scope="module")
def oracle_configs():
    """The oracle's result per benchmark configuration (computed once)."""
    cache = {}

    def get(cfg):
        if cfg not in cache:
            b = workloads.make_batch(cfg)
            cache[cfg] = (b, oracle_icdf(b))
        return cache[cfg]
    return get


@pytest.mark.parametrize("policy", ["warp"] + WARP_POLICIES)
@pytest.mark.parametrize("cfg", [1, 3, 4])
def test_warp_kernel_configs_match_oracle_and_cta(cuda_device, q3s_lib, oracle_configs, cfg, policy):
    """Every row-kernel width on the whole of configs 1, 3 and 4: ids against
    the oracle and the CTA kernel, processed logits against the oracle within
    RTOL (1e-5 relative) on every non-boundary row."""
    b, ref = oracle_configs(cfg)
    g, kw = _packed_args(b, cuda_device)
    ids_w, kf_w, err_w, proc_w = _run_policy(policy, g, kw, cuda_device, processed=True)
    ids_c, kf_c, err_c = _run_policy("cta", g, kw, cuda_device)
    assert err_w == 0 and err_c == 0
    nb, nbm = assert_ids_match(ids_w, ref, kf_w, f"warp config {cfg}", max_frac=MAX_BOUNDARY_FRACTION)
    ok = ~(ref["boundary"] | ((kf_w & 3) != 0))
    assert not np.isnan(proc_w).any(), "processed row not fully written"
    assert _proc_close(proc_w[ok], ref["processed"][ok]), f"{policy} config {cfg}: processed logits differ"
    # the processed output does not change the sampled ids
    ids_np, kf_np, _ = _run_policy(policy, g, kw, cuda_device)
    np.testing.assert_array_equal(ids_np, ids_w)
    np.testing.assert_array_equal(kf_np, kf_w)
    # both kernel families agree wherever neither flags a boundary
    bnd = ((kf_w | kf_c) & (_lib.ROW_DRAW_BOUNDARY | _lib.ROW_TOPP_BOUNDARY)) != 0
    np.testing.assert_array_equal(ids_w[~bnd], ids_c[~bnd])
    np.testing.assert_array_equal(kf_w & _lib.ROW_GREEDY, kf_c & _lib.ROW_GREEDY)
    print(f"warp config {cfg}: {len(ids_w)} rows, {nb} boundary rows, {nbm} differ from the oracle")


def _warp_case(dev, logits, bf16=False, policy="warp", **kw):
    with q3s.kernel_policy(policy):
        logits = np.asarray(logits, np.float32)
        B, V = logits.shape
        rng = np.random.default_rng(1)
        u = kw.pop("u", None)
        u = rng.random(B).astype(np.float32) if u is None else np.asarray(u, np.float32)
        hist = kw.pop("hist", None) or [np.zeros(0, np.int32)] * B
        T, k, p = kw.get("T", 1.0), kw.get("k", 0), kw.get("p", 1.0)
        pen, mn, eos, sup = kw.get("pen", 1.0), kw.get("mn", 0), kw.get("eos", -1), kw.get("suppress")
        offs = np.zeros(B + 1, np.int32)
        offs[1:] = np.cumsum([len(h) for h in hist])
        flat = np.concatenate(hist).astype(np.int32) if offs[-1] else np.zeros(1, np.int32)
        x_t = torch.from_numpy(logits)
        if bf16:
            x_t = x_t.to(torch.bfloat16)
            logits = x_t.float().numpy()
        Tv = np.broadcast_to(np.asarray(T, np.float32), (B,)).copy()
        kv = np.broadcast_to(np.asarray(k, np.int32), (B,)).copy()
        ref = O.sample_icdf(logits, uniforms=u, temperature=Tv, top_k=kv, top_p=np.full(B, p, np.float32),
                            penalty=np.full(B, pen, np.float32), history=flat[:offs[-1]], offsets=offs,
                            min_new_tokens=np.full(B, mn), suppress=sup, eos_id=eos)
        outs = []
        for want_proc in (False, True):
            flags = torch.zeros(B, dtype=torch.int32, device=dev)
            err = torch.zeros(1, dtype=torch.int32, device=dev)
            proc = torch.full((B, V), float("nan"), dtype=torch.float32, device=dev) if want_proc else None
            ids = q3s.sample_packed(x_t.to(dev), _dev(flat, dev), _dev(offs, dev), uniforms=_dev(u, dev),
                                    temperature=_dev(Tv, dev), top_k=_dev(kv, dev), top_p=p, penalty=pen,
                                    min_new_tokens=mn, eos_id=eos, suppress=None if sup is None else _dev(sup, dev),
                                    row_flags=flags, error_word=err, processed=proc)
            torch.cuda.synchronize()
            outs.append((ids.cpu().numpy(), flags.cpu().numpy(), int(err.item()),
                         None if proc is None else proc.cpu().numpy()))
        (ids, kf, e, _), (ids_p, kf_p, e_p, proc) = outs
        # the processed-logits variant samples the same ids, and its rows
        # match the oracle's processed rows wherever no boundary is flagged
        np.testing.assert_array_equal(ids_p, ids)
        np.testing.assert_array_equal(kf_p, kf)
        assert e_p == e
        ok = ~(ref["boundary"] | ((kf & 3) != 0))
        assert not np.isnan(proc).any(), "processed row not fully written"
        assert _proc_close(proc[ok], ref["processed"][ok]), f"{policy}: processed logits differ"
        return ids, kf, e, ref


@pytest.mark.parametrize("V", [1032, 2048, 2056, 3072])
@pytest.mark.parametrize("k,p", [(0, 1.0), (50, 1.0), (50, 0.9), (0, 0.95), (0, 0.5), (1, 1.0), (300, 0.9)])
@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("policy", WARP_POLICIES)
def test_warp_kernel_vocab_sizes_and_filters(cuda_device, q3s_lib, V, k, p, bf16, policy):
    rng = np.random.default_rng(V * 11 + k)
    x = (rng.standard_normal((40, V)) * 2.0).astype(np.float32)
    T = np.where(np.arange(40) % 10 == 3, 0.0, 0.8).astype(np.float32)  # some greedy rows
    ids, kf, err, ref = _warp_case(cuda_device, x, bf16=bf16, policy=policy, T=T, k=k, p=p)
    assert err == 0
    assert_ids_match(ids, ref, kf, f"{policy} V={V} k={k} p={p} bf16={bf16}", max_frac=0.25)


@pytest.mark.parametrize("policy", WARP_POLICIES)
def test_warp_kernel_ties_overflow_and_flat_rows(cuda_device, q3s_lib, policy):
    x = np.zeros((6, 3072), np.float32)
    x[0, :100] = 1.0          # 100-way tie across the k=50 boundary: HF keeps all of them
    x[2, ::3] = -np.inf
    x[3, :600] = 2.0          # 600-way tie: the candidate list overflows, the exact path runs
    x[4] = np.linspace(-1, 1, 3072, dtype=np.float32)
    x[5, 7] = 1e30            # one dominant entry
    for k, p in ((50, 0.7), (50, 1.0), (0, 0.9), (100, 0.3)):
        ids, kf, err, ref = _warp_case(cuda_device, x, policy=policy, k=k, p=p)
        assert err == 0
        assert_ids_match(ids, ref, kf, f"{policy} ties k={k} p={p}")


@pytest.mark.parametrize("policy", WARP_POLICIES)
def test_warp_kernel_extreme_uniforms_temperatures_and_top_p(cuda_device, q3s_lib, policy):
    rng = np.random.default_rng(13)
    x = (rng.standard_normal((8, 3072)) * 3).astype(np.float32)
    u = np.array([0.0, 0.0, np.float32(1 - 2**-24), np.float32(1 - 2**-24), 0.5, 0.25, 0.75, 0.1], np.float32)
    ids, kf, _, ref = _warp_case(cuda_device, x, policy=policy, k=0, p=1e-4, u=u)
    np.testing.assert_array_equal(ids, x.argmax(-1))
    ids, kf, _, ref = _warp_case(cuda_device, x, policy=policy, k=100, p=1.0, u=u)
    assert_ids_match(ids, ref, kf, "warp extreme uniforms")
    # temperatures outside the candidate window take the exact path
    T = np.array([1e-7, 3e6, 1e-30, 0.5, 2.0, 1e-6, 1e7, 1.0], np.float32)
    for k, p in ((50, 0.9), (0, 0.9)):
        ids, kf, err, ref = _warp_case(cuda_device, x, policy=policy, T=T, k=k, p=p, u=u)
        assert err == 0
        assert_ids_match(ids, ref, kf, f"warp extreme T k={k}")


@pytest.mark.parametrize("policy", WARP_POLICIES)
def test_warp_kernel_penalty_eos_gate_and_suppress(cuda_device, q3s_lib, policy):
    rng = np.random.default_rng(14)
    x = (rng.standard_normal((8, 3072)) * 3).astype(np.float32)
    x[:, 2150] = 50.0
    hist = [rng.integers(0, 3072, n).astype(np.int32) for n in (0, 1, 5, 9, 30, 64, 65, 4000)]
    sup = O.suppress_mask(3072, 2150)
    for k, p in ((50, 0.9), (0, 0.95)):
        ids, kf, err, ref = _warp_case(cuda_device, x, policy=policy, T=0.9, k=k, p=p, pen=1.3, hist=list(hist),
                                       mn=64, eos=2150, suppress=sup)
        assert err == 0
        assert_ids_match(ids, ref, kf, f"warp penalty/eos k={k}")
        lens = np.array([len(h) for h in hist])
        assert np.all(ids[lens < 64] != 2150) and np.all(ids[lens >= 64] == 2150)


@pytest.mark.parametrize("policy", WARP_POLICIES)
def test_warp_kernel_bad_history_is_reported(cuda_device, q3s_lib, policy):
    x = np.zeros((2, 2048), np.float32)
    hist = [np.array([5, 3000, -1], np.int32), np.array([7], np.int32)]
    _, _, err, _ = _warp_case(cuda_device, x, policy=policy, hist=hist)
    assert err & _lib.DEVERR_HISTORY_ID


@pytest.mark.parametrize("policy", WARP_POLICIES)
@pytest.mark.parametrize("bf16", [False, True])
def test_warp_kernel_threshold_paths(cuda_device, q3s_lib, policy, bf16):
    """Rows that take each way of locating the K-th largest in the row kernel:
    bins 1/8 wide near the top, unit bins then 1/64 bins (the K-th 32 or more
    below the top, or too many entries near it for 1/8 bins), the radix
    select (values beyond +-2000), and the exact whole-row path."""
    rng = np.random.default_rng(21)
    V = 3072
    x = (rng.standard_normal((10, V)) * 3).astype(np.float32)   # rows 0-1: 1/8 bins
    x[2] = rng.standard_normal(V)
    x[2, 11] = 60.0                                             # K-th ~60 below the top
    x[3] = rng.standard_normal(V) * 0.1                         # dense: 1/64 bins needed
    x[4] = rng.standard_normal(V) * 0.1 + 500.0                 # dense, offset
    x[5] = rng.standard_normal(V) * 0.004                       # denser still: exact path
    x[6] = rng.standard_normal(V) * 1000.0                      # beyond +-2000: radix select
    x[7, :40] = -1e9                                            # a suppressed block at the top positions
    x[8] = np.round(rng.standard_normal(V) * 8) / 8             # many exact ties on the 1/8 grid
    x[9] = rng.standard_normal(V) * 20.0                        # wide spread
    T = np.array([0.7, 1.3, 0.9, 0.9, 0.9, 0.9, 0.9, 0.8, 0.9, 1.0], np.float32)
    for k, p in ((20, 1.0), (50, 0.9), (100, 0.95), (128, 0.8)):
        ids, kf, err, ref = _warp_case(cuda_device, x, bf16=bf16, policy=policy, T=T, k=k, p=p)
        assert err == 0
        assert_ids_match(ids, ref, kf, f"{policy} threshold paths k={k} p={p} bf16={bf16}", max_frac=0.25)


@pytest.mark.parametrize("bf16", [False, True])
def test_gumbel_candidate_paths(cuda_device, q3s_lib, bf16):
    """Exactly-K Gumbel rows through each way the CTA sampler finds its
    candidates (1/8-unit bins below the row maximum, the radix threshold for
    values beyond +-2000, NaN-free rows too dense or too peaked for the bins),
    with ties across the K boundary (lowest index first), -inf and suppressed
    entries, and a repetition penalty over a packed history."""
    rng = np.random.default_rng(31)
    B, V = 12, 3072
    x = (rng.standard_normal((B, V)) * 3).astype(np.float32)
    x[1, :120] = 4.0                                   # 120-way tie across K = 50
    x[2] = rng.standard_normal(V) * 0.01               # dense: radix threshold
    x[3] = rng.standard_normal(V); x[3, 9] = 60.0      # K-th far below the top
    x[4] = rng.standard_normal(V) * 1000.0             # beyond +-2000
    x[5, ::2] = -np.inf                                # half the row -inf
    x[6, 7] = 1e30                                     # one dominant entry
    x[7] = np.round(rng.standard_normal(V) * 8) / 8    # many exact ties
    x[8, :3000] = -1e9                                 # suppressed block: fewer than K above it
    xt = torch.from_numpy(x)
    if bf16:
        xt = xt.to(torch.bfloat16)
        x = xt.float().numpy()
    noise = (-np.log(-np.log(rng.random((B, 50)).clip(1e-12, 1 - 1e-7)))).astype(np.float32)
    T = np.full(B, 0.9, np.float32)
    pen = np.full(B, 1.15, np.float32)
    hist = [rng.integers(0, V, int(n)).astype(np.int32) for n in rng.integers(0, 600, B)]
    offs = np.zeros(B + 1, np.int32)
    offs[1:] = np.cumsum([len(h) for h in hist])
    flat = np.concatenate(hist).astype(np.int32)
    ids = q3s.sample_packed(xt.to(cuda_device), _dev(flat, cuda_device), _dev(offs, cuda_device), mode="gumbel",
                            topk=50, gumbel_noise=_dev(noise, cuda_device), temperature=_dev(T, cuda_device),
                            penalty=_dev(pen, cuda_device), eos_id=-1)
    ref = O.sample_gumbel(x, gumbel_noise=noise, temperature=T, penalty=pen, history=flat, offsets=offs,
                          topk=50, eos_id=-1)
    np.testing.assert_array_equal(ids.cpu().numpy(), ref["ids"])


def test_philox_rows_match_host_generator(cuda_device, q3s_lib):
    """Device-side per-row uniforms are bit-identical to the host generator
    (q3s/philox.py row_uniforms) for contiguous and arbitrary row keys, steps
    and column counts; the Gumbel transform agrees with the torch fp32
    transform of the same uniforms within 1e-6 (relative and absolute: both
    use a correctly-rounded-within-1-ulp log)."""
    from q3s import philox as P
    rng = np.random.default_rng(41)
    cases = [(0, 0, 1, 1, 0), (2**40 + 12345, 7, 128, 50, 0), (2**64 - 1, 3, 1000, 3, 5000),
             (987654321, 0, 128, 750, 0), (5, 2**32 - 1, 33, 4, 2**33 + 17)]
    for seed, step, rows, cols, row0 in cases:
        keys = np.arange(row0, row0 + rows, dtype=np.int64)
        want = P.row_uniforms(seed, keys, cols=cols, step=step)
        got = q3s.philox_rows(seed, rows, cols, step=step, row0=row0, device=cuda_device).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
        g = q3s.philox_rows(seed, rows, cols, step=step, row0=row0, kind="gumbel", device=cuda_device).cpu().numpy()
        np.testing.assert_allclose(g, P.gumbel_from_uniforms(want), rtol=1e-6, atol=1e-6)
    # arbitrary slot keys (engine slots), including keys past 2^32
    keys = rng.integers(0, 2**40, 257).astype(np.int64)
    want = P.row_uniforms(77, keys, cols=15 * 50, step=9)
    got = q3s.philox_rows(77, 257, 15 * 50, step=9, row_keys=_dev(keys, cuda_device)).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    assert float(got.min()) >= 0.0 and float(got.max()) < 1.0
    # keys r and r + 2^32 give different streams (all 64 bits of the key)
    two = q3s.philox_rows(77, 2, 8, row_keys=_dev(np.array([9, 9 + 2**32], np.int64), cuda_device)).cpu().numpy()
    assert not np.array_equal(two[0], two[1])


def test_philox_seeds_match_host_generator(cuda_device, q3s_lib):
    """One 64-bit seed per row (the reference's per-slot seeds): the device
    draws the host generator's bits (q3s/philox.py seeded_uniforms) for any
    seed, step and stage, Gumbel noise within 1e-6."""
    from q3s import philox as P
    rng = np.random.default_rng(43)
    seeds = [int(x) for x in rng.integers(0, 2**63, 300)] + [0, 2**64 - 1, 2**63, 2**32, 2**32 + 1]
    dseeds = torch.tensor([x - 2**64 if x >= 2**63 else x for x in seeds], dtype=torch.int64, device=cuda_device)
    for cols, step, stage in ((50, 0, 0), (750, 17, 3), (1, 2**32 - 1, 2**31), (3, 5, 0)):
        want = P.seeded_uniforms(seeds, cols, step=step, stage=stage)
        got = q3s.philox_seeds(dseeds, cols, step=step, stage=stage).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
        g = q3s.philox_seeds(dseeds, cols, step=step, stage=stage, kind="gumbel").cpu().numpy()
        np.testing.assert_allclose(g, P.gumbel_from_uniforms(want), rtol=1e-6, atol=1e-6)
    # a row's numbers follow its seed, not its position in the batch
    a = q3s.philox_seeds(dseeds[:8], 50, step=1).cpu().numpy()
    b = q3s.philox_seeds(dseeds[:8].flip(0), 50, step=1).cpu().numpy()
    np.testing.assert_array_equal(a, b[::-1])


# ---------------------------------------------------------------------------
# capacity layout of the history (RowHistory): the same ids as packed
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("policy", ["auto", "cta", "w4", "wmax", "lean"])
@pytest.mark.parametrize("cfg", [1, 3])
def test_capacity_layout_matches_packed_and_oracle(cuda_device, q3s_lib, oracle_configs, cfg, policy):
    """Rows in regions with spare capacity: ids, flags and processed logits
    equal the packed layout's, and the oracle's (on the used prefixes)."""
    b, ref = oracle_configs(cfg)
    g, kw = _packed_args(b, cuda_device)
    lens = np.diff(b.offsets.numpy())
    caps = (lens + np.random.default_rng(cfg).integers(0, 64, b.B)).tolist()
    rows = q3s.RowHistory.from_packed(g.history, b.offsets, caps, device=cuda_device)
    outs = {}
    for name, hk in (("packed", dict(history=g.history, offsets=g.offsets)), ("capacity", rows.sampler_kwargs())):
        flags = torch.zeros(g.B, dtype=torch.int32, device=cuda_device)
        err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        proc = torch.empty(g.B, g.V, dtype=torch.float32, device=cuda_device)
        with q3s.kernel_policy(policy):
            plan = q3s.SamplePlan(g.logits, mode="icdf", processed=proc, row_flags=flags, error_word=err, **hk,
                                  **{k: v for k, v in kw.items() if k not in ("eos_id", "suppress")},
                                  suppress_mask=g.suppress, eos_id=g.eos_id)
            plan.launch()
        torch.cuda.synchronize()
        outs[name] = (plan.ids.cpu().numpy(), flags.cpu().numpy(), int(err.item()), proc.cpu().numpy())
    (ip, fp, ep, pp), (ic, fc, ec, pc) = outs["packed"], outs["capacity"]
    assert ep == 0 and ec == 0
    np.testing.assert_array_equal(ic, ip)
    np.testing.assert_array_equal(fc, fp)
    np.testing.assert_array_equal(pc, pp)
    ph, po = rows.packed()
    ref2 = O.sample_icdf(b.logits, uniforms=b.uniforms.numpy(), temperature=b.temperature.numpy(),
                         top_k=b.top_k.numpy(), top_p=b.top_p.numpy(), penalty=b.penalty.numpy(),
                         history=rows.ids.cpu().numpy(), offsets=rows.offsets.cpu().numpy(),
                         history_lengths=rows.lengths.cpu().numpy(), min_new_tokens=b.min_new_tokens.numpy(),
                         suppress=b.suppress.numpy(), eos_id=b.eos_id)
    np.testing.assert_array_equal(ref2["ids"], ref["ids"])
    np.testing.assert_array_equal(ph.numpy(), b.history.numpy())
    assert_ids_match(ic, ref2, fc, f"capacity layout config {cfg} {policy}", max_frac=MAX_BOUNDARY_FRACTION)


def test_capacity_layout_bad_length_is_reported(cuda_device, q3s_lib):
    """A length past its region is flagged (OFFSETS) and the row sampled
    without a history, on both kernel families."""
    rng = np.random.default_rng(3)
    B, V = 4, 3072
    x = torch.from_numpy((rng.standard_normal((B, V)) * 2).astype(np.float32)).to(cuda_device)
    rows = q3s.RowHistory(B, 16, device=cuda_device)
    rows.ids.copy_(torch.from_numpy(rng.integers(0, V, rows.ids.numel()).astype(np.int32)))
    rows.lengths.copy_(torch.tensor([3, 17, 0, 16], dtype=torch.int32))
    for policy in ("cta", "auto"):
        err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        with q3s.kernel_policy(policy):
            plan = q3s.SamplePlan(x, mode="icdf", uniforms=torch.full((B,), 0.5, device=cuda_device), topk=50,
                                  penalty=1.3, error_word=err, **rows.sampler_kwargs())
            plan.launch()
        torch.cuda.synchronize()
        assert int(err.item()) & _lib.DEVERR_OFFSETS, policy


# ---------------------------------------------------------------------------
# the lean kernel's fast paths and its exact core
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("cfg", [1, 3, 4])
def test_lean_fast_paths_decide_benchmark_rows(cuda_device, q3s_lib, oracle_configs, cfg):
    """Every row of the benchmark configurations is decided on the lean
    kernel's fast paths (no Q3S_ROW_EXACT_CORE flag), with the oracle's ids."""
    b, ref = oracle_configs(cfg)
    g, kw = _packed_args(b, cuda_device)
    ids, kf, err = _run_policy("lean", g, kw, cuda_device)
    assert err == 0
    assert not np.any(kf & _lib.ROW_EXACT_CORE), f"config {cfg}: rows {np.nonzero(kf & _lib.ROW_EXACT_CORE)[0][:8]}"
    assert_ids_match(ids, ref, kf, f"lean config {cfg}", max_frac=MAX_BOUNDARY_FRACTION)


def test_lean_rows_outside_the_window_take_the_exact_core(cuda_device, q3s_lib):
    """Rows the fast paths cannot prove exact -- a logit beyond +-2000, a
    top-k beyond the candidate path's 128, a 600-way tie that overflows the
    list -- are flagged Q3S_ROW_EXACT_CORE and still match the oracle; an
    ordinary row beside them is not flagged."""
    rng = np.random.default_rng(31)
    x = (rng.standard_normal((4, 3072)) * 3).astype(np.float32)
    x[0, 17] = 5000.0        # beyond the fast window
    x[2, :600] = 50.0        # a 600-way tie at the top (list overflow for k = 50)
    T = np.full(4, 0.9, np.float32)
    for k, p, exact_rows in ((50, 0.9, (0, 2)), (300, 0.9, (0, 1, 2, 3))):
        ids, kf, err, ref = _warp_case(cuda_device, x, policy="lean", T=T, k=k, p=p)
        assert err == 0
        assert_ids_match(ids, ref, kf, f"lean exact core k={k}")
        flagged = set(np.nonzero(kf & _lib.ROW_EXACT_CORE)[0].tolist())
        assert flagged == set(exact_rows), f"k={k}: exact-core rows {sorted(flagged)}"
