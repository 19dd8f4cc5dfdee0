"""``torch.ops.q3s.*`` on the GPU against the reference's golden vectors and
the oracle (the same tolerances as test_gpu_parity.py: ids bit-exact outside
counted boundary rows)."""
import numpy as np
import pytest
import torch

import q3s
import q3s_oracle as O
from conftest import load_golden
from q3s import workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda_device):
    return q3s.load_torch_ops()


def _dev(x, dev):
    return torch.as_tensor(np.ascontiguousarray(x)).to(dev)


def _counts(g, B, V):
    tc = np.zeros((B, V), np.int64)
    for b in range(B):
        np.add.at(tc[b], g["history"][g["offsets"][b]:g["offsets"][b + 1]], 1)
    return tc


@pytest.mark.parametrize("name", ["gumbel_cb0_f32", "gumbel_cb0_bf16"])
def test_sample_codebook0_op_matches_reference_golden(cuda_device, ops, name):
    g = load_golden(name)
    B, V = g["logits"].shape
    tc = _counts(g, B, V)
    logits = g["logits_bf16"].to(cuda_device) if "logits_bf16" in g else _dev(g["logits"], cuda_device)
    sup = q3s.suppress_mask(V, 2150, cuda_device)
    T = _dev(g["temperature"].reshape(B, 1), cuda_device)
    P = _dev(g["penalty"].reshape(B, 1), cuda_device)
    noise = _dev(g["gumbel_noise"], cuda_device)
    tcd = _dev(tc, cuda_device)
    ids, upd = torch.ops.q3s.sample_codebook0(logits, tcd, noise, T, P, sup, 50)
    oracle = O.sample_gumbel(g["logits"], gumbel_noise=g["gumbel_noise"], temperature=g["temperature"],
                             penalty=g["penalty"], token_counts=tc, suppress=O.suppress_mask(V), topk=50)
    ok = ~g["tie_rows"]
    np.testing.assert_array_equal(ids.cpu().numpy()[ok], g["ids"][ok])
    np.testing.assert_array_equal(ids.cpu().numpy(), oracle["ids"])
    np.testing.assert_array_equal(upd.cpu().numpy(), oracle["updated_counts"])
    np.testing.assert_array_equal(tcd.cpu().numpy(), tc)  # functional: input untouched
    # the in-place form updates token_counts and returns the same ids
    ids2 = torch.ops.q3s.sample_codebook0_(logits, tcd, noise, T, P, sup, 50)
    np.testing.assert_array_equal(ids2.cpu().numpy(), ids.cpu().numpy())
    np.testing.assert_array_equal(tcd.cpu().numpy(), oracle["updated_counts"])
    # [B,S,V] engine output: the last position is sampled
    l3 = torch.stack([torch.zeros_like(logits), logits], dim=1)
    ids3, _ = torch.ops.q3s.sample_codebook0(l3, _dev(tc, cuda_device), noise, T, P, sup, 50)
    np.testing.assert_array_equal(ids3.cpu().numpy(), ids.cpu().numpy())


def test_sample_cp_stage_op_matches_reference_golden(cuda_device, ops):
    g = load_golden("cp_select")
    B = g["logits"].shape[0]
    lg = _dev(g["logits"], cuda_device).reshape(B, 1, -1)
    ids = torch.ops.q3s.sample_cp_stage(lg, _dev(g["temperature"].reshape(B, 1), cuda_device),
                                        _dev(g["gumbel_noise"], cuda_device), 50)
    np.testing.assert_array_equal(ids.cpu().numpy(), g["ids"])
    greedy = torch.ops.q3s.sample_cp_stage(lg, None, None, 50)
    np.testing.assert_array_equal(greedy.cpu().numpy(), g["greedy_ids"])


def test_sample_codebook0_packed_op_matches_reference_golden(cuda_device, ops):
    g = load_golden("icdf_hf_extended")
    B, V = g["logits"].shape
    ref = O.sample_icdf(g["logits"], uniforms=g["uniforms"], temperature=g["temperature"], top_k=g["top_k"],
                        top_p=g["top_p"], penalty=g["penalty"], history=g["history"], offsets=g["offsets"],
                        min_new_tokens=g["min_new_tokens"], suppress=O.suppress_mask(V), eos_id=2150)
    d = {k: _dev(g[k], cuda_device) for k in ("history", "offsets", "uniforms", "temperature", "top_k", "top_p",
                                               "penalty", "min_new_tokens")}
    ids = torch.ops.q3s.sample_codebook0_packed(g["logits_bf16"].to(cuda_device), d["history"], d["offsets"],
                                                d["uniforms"], d["temperature"], d["top_k"], d["top_p"],
                                                d["penalty"], d["min_new_tokens"],
                                                q3s.suppress_mask(V, 2150, cuda_device), 2150)
    got = ids.cpu().numpy()
    bad = (got != g["ids"]) & ~ref["boundary"]
    assert not bad.any(), f"rows {np.nonzero(bad)[0][:10]}"


def test_sample_codebook0_packed_op_matches_oracle_on_config1(cuda_device, ops):
    b = workloads.make_batch(1)
    gd = b.to(cuda_device)
    ids = torch.ops.q3s.sample_codebook0_packed(gd.logits, gd.history, gd.offsets, gd.uniforms, gd.temperature,
                                                gd.top_k, gd.top_p, gd.penalty, gd.min_new_tokens, gd.suppress,
                                                b.eos_id)
    ref = O.sample_icdf(b.logits, uniforms=b.uniforms.numpy(), temperature=b.temperature.numpy(),
                        top_k=b.top_k.numpy(), top_p=b.top_p.numpy(), penalty=b.penalty.numpy(),
                        history=b.history.numpy(), offsets=b.offsets.numpy(),
                        min_new_tokens=b.min_new_tokens.numpy(), suppress=b.suppress.numpy(), eos_id=b.eos_id)
    got = ids.cpu().numpy()
    assert not ((got != ref["ids"]) & ~ref["boundary"]).any()
    # the same ids through the plan API
    np.testing.assert_array_equal(got, q3s.sample_packed(gd.logits, gd.history, gd.offsets, uniforms=gd.uniforms,
                                                         temperature=gd.temperature, top_k=gd.top_k,
                                                         top_p=gd.top_p, penalty=gd.penalty,
                                                         min_new_tokens=gd.min_new_tokens, suppress=gd.suppress,
                                                         eos_id=b.eos_id).cpu().numpy())


@pytest.mark.parametrize("greedy", [False, True])
def test_sample_cp_frame_op_matches_oracle_chain(cuda_device, ops, greedy):
    f = workloads.make_cp_frame(rows=(0, 32))
    fd = f.to(cuda_device)
    noise = None if greedy else fd.gumbel_noise
    ids = torch.ops.q3s.sample_cp_frame(fd.base, fd.temperature.reshape(-1, 1), noise, 50)
    ref = O.cp_frame(f.base.float().numpy(), mode="gumbel", rotate=False,
                     temperature=f.temperature.numpy(),
                     gumbel_noise=None if greedy else f.gumbel_noise.numpy())
    np.testing.assert_array_equal(ids.cpu().numpy(), ref["ids"])


def test_torch_ops_reject_bad_inputs(cuda_device, ops):
    x = torch.zeros(4, 3072, device=cuda_device)
    with pytest.raises(RuntimeError, match="token_counts"):
        torch.ops.q3s.sample_codebook0(x, torch.zeros(4, 3071, dtype=torch.int64, device=cuda_device),
                                       torch.zeros(4, 50, device=cuda_device), torch.ones(4, 1, device=cuda_device),
                                       torch.ones(4, 1, device=cuda_device), None, 50)
    with pytest.raises(RuntimeError, match="offsets"):
        torch.ops.q3s.sample_codebook0_packed(x, torch.zeros(8, dtype=torch.int32, device=cuda_device),
                                              torch.zeros(3, dtype=torch.int32, device=cuda_device),
                                              *([torch.ones(4, device=cuda_device)] * 6), None, 2150)
