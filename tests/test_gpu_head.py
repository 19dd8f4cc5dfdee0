"""The codec head on the tensor cores (q3s_head_sample): logits against torch's
fp32 matmul of the same bf16 operands, and the sampler launched behind it
against the same sampler run on those logits and against the oracle.

Tolerance for the logits: the kernel accumulates in fp32 in its own order
(a 16-wide MMA sum per K step, then 8 K slices added in order), torch's fp32
GEMM in cuBLAS's.  Against the float64 product of the same bf16 operands both
are within one bf16 unit in the last place of the larger magnitude plus the
fp32 accumulation error (|d| <= 2^-7 max(|got|, |ref|) + 1e-3; near zero the
accumulation error dominates a bf16 ulp -- cuBLAS's fp32 result shows the same),
and at least 99% of the kernel's logits equal the rounded float64 product.
Sampled ids are bit-exact against the plain sampler on the head's own logits,
and against the oracle on those logits outside counted boundary rows."""
import numpy as np
import pytest
import torch

import q3s
import q3s_oracle as O
from q3s import workloads

pytestmark = pytest.mark.gpu


def _operands(dev, B, H, V, seed):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(B, H, generator=g).to(torch.bfloat16)
    weight = (torch.randn(V, H, generator=g) * (3.0 / H ** 0.5)).to(torch.bfloat16)
    return hidden.to(dev), weight.to(dev)


def _check_logits(logits, hidden, weight):
    ref = hidden.double() @ weight.double().t()
    got = logits.double()
    d = (got - ref).abs()
    tol = torch.maximum(got.abs(), ref.abs()) * 2.0 ** -7 + 1e-3
    assert bool((d <= tol).all()), f"max |d| {float(d.max())}"
    same = float((logits == ref.to(torch.bfloat16)).float().mean())
    assert same >= 0.99, f"only {same:.4f} of the logits equal the rounded reference"


@pytest.mark.parametrize("B,H,V", [(1, 512, 256), (5, 2048, 3072), (128, 2048, 3072), (200, 2048, 2048),
                                   (300, 1024, 3072), (129, 4096, 512), (64, 768, 192), (128, 2048, 320)])
def test_head_logits_match_torch(cuda_device, q3s_lib, B, H, V):
    hidden, weight = _operands(cuda_device, B, H, V, B + H + V)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    logits = torch.full((B, V), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    q3s.HeadPlan(hidden, weight, logits, error_word=err).launch()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert not bool(torch.isnan(logits.float()).any())
    _check_logits(logits, hidden, weight)
    # the last position of [B, S, H] hidden states, and a strided logits buffer
    h3 = torch.stack([torch.zeros_like(hidden), hidden], dim=1)
    wide = torch.zeros(B, V + 64, dtype=torch.bfloat16, device=cuda_device)
    q3s.HeadPlan(h3, weight, wide[:, :V]).launch()
    torch.cuda.synchronize()
    assert torch.equal(wide[:, :V], logits)
    assert not bool(wide[:, V:].float().abs().sum())


@pytest.mark.parametrize("B", [1, 128, 300])
def test_head_then_sampler_matches_plain_sampler_and_oracle(cuda_device, q3s_lib, B):
    """Config-1 parameters over the head's logits: the dependent launch gives
    the ids the stand-alone sampler gives on those logits (both kernel
    families), and the oracle's outside boundary rows."""
    H, V = 2048, 3072
    b = workloads.make_batch(1, total_rows=B)
    g = b.to(cuda_device)
    hidden, weight = _operands(cuda_device, B, H, V, 7 * B)
    kw = dict(mode="icdf", history=g.history, offsets=g.offsets, uniforms=g.uniforms, temperature=g.temperature,
              top_k=g.top_k, top_p=g.top_p, penalty=g.penalty, min_new_tokens=g.min_new_tokens,
              suppress_mask=g.suppress, eos_id=g.eos_id)
    for policy in ("auto", "cta"):
        with q3s.kernel_policy(policy):
            logits = torch.empty(B, V, dtype=torch.bfloat16, device=cuda_device)
            flags = torch.zeros(B, dtype=torch.int32, device=cuda_device)
            plan = q3s.SamplePlan(logits, row_flags=flags, **kw)
            q3s.HeadPlan(hidden, weight, logits, sample=plan).launch()
            torch.cuda.synchronize()
            ids = plan.ids.clone()
            again = q3s.SamplePlan(logits.clone(), **kw)
            again.launch()
            torch.cuda.synchronize()
            assert torch.equal(ids, again.ids), policy
        _check_logits(logits, hidden, weight)
        ref = O.sample_icdf(logits.float().cpu().numpy(), uniforms=b.uniforms.numpy(),
                            temperature=b.temperature.numpy(), top_k=b.top_k.numpy(), top_p=b.top_p.numpy(),
                            penalty=b.penalty.numpy(), history=b.history.numpy(), offsets=b.offsets.numpy(),
                            min_new_tokens=b.min_new_tokens.numpy(), suppress=b.suppress.numpy(), eos_id=b.eos_id)
        bnd = ref["boundary"] | ((flags.cpu().numpy() & 3) != 0)
        bad = (ids.cpu().numpy() != ref["ids"]) & ~bnd
        assert not bad.any(), f"{policy}: rows {np.nonzero(bad)[0][:8]}"


def test_head_then_gumbel_counts_engine_layout(cuda_device, q3s_lib):
    """The engine's own layout behind the head (gumbel, token_counts updated in
    place): the same ids and counts as the stand-alone call on the logits."""
    B, H, V = 64, 2048, 3072
    b = workloads.make_batch(1, total_rows=B)
    g = b.to(cuda_device)
    hidden, weight = _operands(cuda_device, B, H, V, 99)
    counts = g.token_counts()
    counts2 = counts.clone()
    logits = torch.empty(B, V, dtype=torch.bfloat16, device=cuda_device)
    plan = q3s.SamplePlan(logits, mode="gumbel", topk=50, token_counts=counts, counts_out=counts,
                          temperature=g.temperature, penalty=g.penalty, gumbel_noise=g.gumbel_noise,
                          suppress_mask=g.suppress)
    q3s.HeadPlan(hidden, weight, logits, sample=plan).launch()
    ids, upd = q3s.sample_codebook0(logits, counts2, g.gumbel_noise, g.temperature.reshape(-1, 1),
                                    g.penalty.reshape(-1, 1), suppress=g.suppress, inplace=True)
    torch.cuda.synchronize()
    assert torch.equal(plan.ids, ids)
    assert torch.equal(counts, counts2)
