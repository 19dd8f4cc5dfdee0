"""Generate golden sampler vectors by running the REFERENCE's own code.

Run in a container where the reference checkout is available (it is not on
the GPU box; the fixtures it writes are committed instead):

    python tests/golden/make_golden.py --reference /path/to/Qwen3TTS-Streaming
    python tests/golden/make_golden.py --reference ... --time   # CPU baseline (i)

Cases (inputs are seeded synthetic tensors; outputs come from the reference):

* gumbel_cb0_f32 / gumbel_cb0_bf16 -- ``TalkerUnifiedFusedONNX.forward``
  (scripts/export/talker_unified_modules.py:397-440) with stub backbone / code
  predictor / codec-sum modules that return the given logits; records
  ``codec_token_0`` (= full_codec[:,0]) and ``updated_token_counts``.  The bf16
  case has top-k ties; rows whose id depends on ``torch.topk``'s unspecified
  tie order are marked ``tie_rows``.
* cp_select -- ``CodePredictorUnrolled._select_token``
  (scripts/export/utils.py:1178-1193), Gumbel and greedy.
* icdf_sample_token -- ``_sample_token`` (tools/validation/
  prefill_compare.py:383-399) with ``torch.multinomial`` replaced, for the
  duration of the call, by an inverse-CDF draw on a supplied uniform, and
  ``torch.softmax`` wrapped to record the processed logits it receives.
* icdf_hf_extended -- the same transformers processors plus TopP and
  MinNewTokens (the benchmark's extensions), applied per row; rows where
  ``torch.sort``'s unstable tie order changes the TopP cut are marked.
"""
from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "qwen3tts-streaming_b200"))

from q3s.philox import gumbel_from_uniforms, row_uniforms  # noqa: E402

V = 3072
CPV = 2048
EOS = 2150
K = 50


def bf16_round(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(x).to(torch.bfloat16).float().numpy()


def to_u16(x: np.ndarray) -> np.ndarray:
    """fp32 values that are exactly bf16 -> their bf16 bit patterns."""
    t = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16)
    return t.view(torch.int16).numpy().view(np.uint16)


def make_logits(rng, B, vocab, scale, mask_high):
    x = (rng.standard_normal((B, vocab)) * scale).astype(np.float32)
    for b in range(B):
        x[b, rng.choice(min(vocab, 2048), 5, replace=False)] += 8.0
    if mask_high:
        hi = np.arange(vocab - 1024, vocab)
        x[:, hi[hi != EOS]] = -np.inf
    return x


def make_hist(rng, B, lo, hi):
    lens = rng.integers(lo, hi + 1, B)
    offs = np.zeros(B + 1, np.int32)
    offs[1:] = np.cumsum(lens)
    hist = rng.integers(0, 2048, int(offs[-1])).astype(np.int32)
    return hist, offs


def counts_from(hist, offs, B, vocab):
    tc = np.zeros((B, vocab), np.int64)
    for b in range(B):
        np.add.at(tc[b], hist[offs[b]:offs[b + 1]], 1)
    return tc


# ---------------------------------------------------------------------------

def ref_paths(ref: Path):
    for p in (ref / "scripts" / "export", ref / "scripts" / "python", ref / "tools" / "validation"):
        sys.path.insert(0, str(p))


class _StubTalker(nn.Module):
    num_layers = 0

    def __init__(self, logits):
        super().__init__()
        self.logits = logits

    def forward(self, input_embeds, position_ids, *inputs):
        B = self.logits.shape[0]
        return (torch.zeros(B, 1, 4), self.logits)


class _StubCP(nn.Module):
    def forward(self, past_hidden, codec_token_0, cp_gumbel_noise=None, temperature=None):
        return torch.zeros(codec_token_0.shape[0], 15, dtype=torch.long)


class _StubSum(nn.Module):
    def forward(self, full_codec):
        return torch.zeros(full_codec.shape[0], 4)


def run_fused_sampler(logits, token_counts, noise, temperature, penalty):
    from talker_unified_modules import TalkerUnifiedFusedONNX

    B = logits.shape[0]
    fused = TalkerUnifiedFusedONNX(_StubTalker(torch.from_numpy(logits).reshape(B, 1, -1)),
                                   _StubCP(), _StubSum(), vocab_size=logits.shape[1],
                                   codec_eos_token_id=EOS).eval()
    with torch.no_grad():
        out = fused(torch.zeros(B, 1, 4), torch.zeros(B, 3, 1, 1, dtype=torch.long),
                    torch.from_numpy(token_counts), torch.from_numpy(noise),
                    torch.zeros(B, 15, K), torch.from_numpy(temperature).reshape(B, 1),
                    torch.from_numpy(penalty).reshape(B, 1))
    full_codec, updated = out[1], out[4]
    return full_codec[:, 0].numpy().astype(np.int64), updated.numpy()


def canonical_gumbel(logits, token_counts, noise, temperature, penalty):
    """The canonical (value desc, index asc) variant, to mark tie rows."""
    g0 = torch.from_numpy(logits).clone()
    sup = torch.zeros(g0.shape[1], dtype=torch.bool)
    sup[g0.shape[1] - 1024:] = True
    sup[EOS] = False
    g0 = g0.masked_fill(sup, -1e9)
    pen = torch.from_numpy(penalty).reshape(-1, 1)
    g0 = torch.where(torch.from_numpy(token_counts) > 0, torch.where(g0 > 0, g0 / pen, g0 * pen), g0)
    order = torch.sort(g0, dim=-1, descending=True, stable=True).indices[:, :K]
    vals = g0.gather(1, order)
    sel = (vals / torch.from_numpy(temperature).reshape(-1, 1) + torch.from_numpy(noise)).argmax(-1)
    return order.gather(1, sel[:, None])[:, 0].numpy()


def case_gumbel(seed, B, bf16):
    rng = np.random.default_rng(seed)
    logits = make_logits(rng, B, V, 3.0, True)
    if bf16:
        logits = bf16_round(logits)
    hist, offs = make_hist(rng, B, 16, 600)
    tc = counts_from(hist, offs, B, V)
    T = rng.uniform(0.6, 1.0, B).astype(np.float32)
    P = rng.uniform(1.0, 1.2, B).astype(np.float32)
    noise = gumbel_from_uniforms(row_uniforms(seed, B, cols=K))
    ids, updated = run_fused_sampler(logits, tc, noise, T, P)
    canon = canonical_gumbel(logits, tc, noise, T, P)
    delta = updated - tc
    nz = np.argwhere(delta != 0)
    return dict(logits_u16=to_u16(logits) if bf16 else None, logits=None if bf16 else logits,
                history=hist, offsets=offs, temperature=T, penalty=P, gumbel_noise=noise,
                ids=ids, tie_rows=(canon != ids), delta_rc=nz.astype(np.int64),
                delta_val=delta[delta != 0].astype(np.int64))


def case_cp_select(seed, B):
    from utils import CodePredictorUnrolled

    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((B, 1, CPV)) * 2.5).astype(np.float32)
    T = np.full(B, 0.9, np.float32)
    noise = gumbel_from_uniforms(row_uniforms(seed, B, cols=K))
    fake_self = types.SimpleNamespace(logits_topk=K)
    with torch.no_grad():
        ids = CodePredictorUnrolled._select_token(fake_self, torch.from_numpy(logits),
                                                  temperature=torch.from_numpy(T).reshape(B, 1),
                                                  gumbel_noise=torch.from_numpy(noise))
        greedy = CodePredictorUnrolled._select_token(fake_self, torch.from_numpy(logits))
    return dict(logits=logits.reshape(B, CPV), temperature=T, gumbel_noise=noise,
                ids=ids.numpy().astype(np.int64), greedy_ids=greedy.numpy().reshape(-1).astype(np.int64))


def _icdf_from_probs(probs: torch.Tensor, u: float) -> int:
    cdf = np.cumsum(probs.double().reshape(-1).numpy())
    i = int(np.searchsorted(cdf, u * cdf[-1], side="right"))
    if i >= cdf.shape[0]:
        i = int(np.nonzero(probs.reshape(-1).numpy() > 0)[0][-1])
    return i


def case_icdf_sample_token(seed, B):
    import prefill_compare as pc

    rng = np.random.default_rng(seed)
    logits = bf16_round(make_logits(rng, B, V, 3.0, True))
    hist, offs = make_hist(rng, B, 16, 600)
    T = rng.uniform(0.6, 1.0, B).astype(np.float32)
    TK = rng.choice([20, 50, 100], B).astype(np.int32)
    PEN = rng.uniform(1.0, 1.2, B).astype(np.float32)
    u = row_uniforms(seed, B, cols=1).reshape(-1)
    suppress = [i for i in range(V - 1024, V) if i != EOS]
    ids = np.zeros(B, np.int64)
    proc = np.zeros((B, V), np.float32)
    real_mn, real_sm = torch.multinomial, torch.softmax
    for b in range(B):
        seen = {}

        def fake_softmax(s, dim=-1, **kw):
            seen["s"] = s.detach().clone()
            return real_sm(s, dim=dim, **kw)

        def fake_multinomial(probs, num_samples=1, **kw):
            return torch.tensor([[_icdf_from_probs(probs, float(u[b]))]], dtype=torch.long)

        torch.multinomial, torch.softmax = fake_multinomial, fake_softmax
        try:
            h = torch.from_numpy(hist[offs[b]:offs[b + 1]].astype(np.int64)).reshape(1, -1)
            # scalar parameters as the reference passes them: Python floats / ints
            tok = pc._sample_token(torch.from_numpy(logits[b:b + 1]), h, top_k=int(TK[b]),
                                   temperature=float(T[b]), rep_pen=float(PEN[b]), suppress=suppress)
        finally:
            torch.multinomial, torch.softmax = real_mn, real_sm
        ids[b] = int(tok.reshape(-1)[0])
        proc[b] = seen["s"].reshape(-1).numpy()
    return dict(logits_u16=to_u16(logits), history=hist, offsets=offs, temperature=T, top_k=TK,
                penalty=PEN, uniforms=u, ids=ids, processed=proc)


def case_icdf_hf_extended(seed, B):
    from transformers.generation.logits_process import (
        MinNewTokensLengthLogitsProcessor, RepetitionPenaltyLogitsProcessor, TemperatureLogitsWarper,
        TopKLogitsWarper, TopPLogitsWarper)

    rng = np.random.default_rng(seed)
    logits = bf16_round(make_logits(rng, B, V, 3.0, True))
    hist, offs = make_hist(rng, B, 0, 80)
    T = rng.uniform(0.6, 1.0, B).astype(np.float32)
    TK = rng.choice([0, 20, 50, 100], B).astype(np.int32)
    TP = rng.uniform(0.8, 1.0, B).astype(np.float32)
    PEN = rng.uniform(1.0, 1.2, B).astype(np.float32)
    MN = rng.integers(0, 65, B).astype(np.int32)
    u = row_uniforms(seed, B, cols=1).reshape(-1)
    ids = np.zeros(B, np.int64)
    proc = np.zeros((B, V), np.float32)
    sort_tie = np.zeros(B, bool)
    real_sort = torch.sort
    for b in range(B):
        h = torch.from_numpy(hist[offs[b]:offs[b + 1]].astype(np.int64)).reshape(1, -1)
        s = torch.from_numpy(logits[b:b + 1]).float().clone()
        s[..., [i for i in range(V - 1024, V) if i != EOS]] = -1e9
        s = RepetitionPenaltyLogitsProcessor(float(PEN[b]))(h, s)
        s = MinNewTokensLengthLogitsProcessor(0, int(MN[b]), EOS)(h, s)
        s = TemperatureLogitsWarper(float(T[b]))(h, s)
        if TK[b] > 0:
            s = TopKLogitsWarper(int(TK[b]))(h, s)
        s_unstable = TopPLogitsWarper(float(TP[b]))(h, s)
        torch.sort = lambda *a, **k: real_sort(*a, **{**k, "stable": True})
        try:
            s_stable = TopPLogitsWarper(float(TP[b]))(h, s)
        finally:
            torch.sort = real_sort
        sort_tie[b] = not torch.equal(torch.isinf(s_unstable), torch.isinf(s_stable))
        s = s_stable
        probs = torch.softmax(s, dim=-1)
        ids[b] = _icdf_from_probs(probs, float(u[b]))
        proc[b] = s.reshape(-1).numpy()
    return dict(logits_u16=to_u16(logits), history=hist, offsets=offs, temperature=T, top_k=TK,
                top_p=TP, penalty=PEN, min_new_tokens=MN, uniforms=u, ids=ids, processed=proc,
                sort_tie_rows=sort_tie)


def time_reference(configs=(1, 4), iters=50, warmup=5):
    """CPU baseline (i): the reference's own sampler fragment timed on this
    host -- ``TalkerUnifiedFusedONNX.forward`` with the stub modules on each
    codebook-0 config's synthetic inputs (logits, token_counts built from the
    rows' histories, Gumbel noise of the shared uniforms, per-row temperature
    and penalty), and ``CodePredictorUnrolled._select_token`` 15 times in
    sequence on config 2's stage logits.  p50 over ``iters`` steps after
    ``warmup``; one JSON line per config."""
    import json
    import platform
    import time

    from talker_unified_modules import TalkerUnifiedFusedONNX
    from utils import CodePredictorUnrolled

    from q3s import workloads

    cpu = platform.processor() or platform.machine()
    try:
        with open("/proc/cpuinfo") as fh:
            cpu = next((ln.split(":", 1)[1].strip() for ln in fh if ln.startswith("model name")), cpu)
    except OSError:
        pass
    host = dict(cores=os.cpu_count(), torch_threads=torch.get_num_threads(), cpu=cpu)

    def p50(fn):
        for _ in range(warmup):
            fn()
        ts = []
        for _ in range(iters):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return float(np.median(ts))

    for cfg in configs:
        b = workloads.make_batch(cfg)
        B, Vb = b.B, b.V
        logits = b.logits.float().reshape(B, 1, Vb)
        hist, offs = b.history.numpy(), b.offsets.numpy().astype(np.int64)
        tc = torch.from_numpy(counts_from(hist, offs, B, Vb))
        fused = TalkerUnifiedFusedONNX(_StubTalker(logits), _StubCP(), _StubSum(), vocab_size=Vb,
                                       codec_eos_token_id=EOS).eval()
        args_ = (torch.zeros(B, 1, 4), torch.zeros(B, 3, 1, 1, dtype=torch.long), tc, b.gumbel_noise.float(),
                 torch.zeros(B, 15, K), b.temperature.reshape(B, 1), b.penalty.reshape(B, 1))

        def step():
            with torch.no_grad():
                fused(*args_)

        t = p50(step)
        print(json.dumps({"baseline": "(i) reference TalkerUnifiedFusedONNX.forward, stub modules",
                          "config": cfg, "B": B, "V": Vb, "p50_step_us": round(1e6 * t, 1),
                          "tokens_per_s": round(B / t, 1), "iters": iters, **host}), flush=True)
    f = workloads.make_cp_frame()
    S, B = f.base.shape[0], f.base.shape[1]
    stages = [f.base[j].float().reshape(B, 1, -1) for j in range(S)]
    T = f.temperature.reshape(B, 1)
    fake_self = types.SimpleNamespace(logits_topk=K)

    def frame():
        with torch.no_grad():
            for j in range(S):
                CodePredictorUnrolled._select_token(fake_self, stages[j], temperature=T,
                                                    gumbel_noise=f.gumbel_noise[:, j, :])

    t = p50(frame)
    print(json.dumps({"baseline": "(i) reference CodePredictorUnrolled._select_token x 15", "config": 2,
                      "B": B, "V": int(stages[0].shape[-1]), "p50_frame_us": round(1e6 * t, 1),
                      "tokens_per_s": round(B * S / t, 1), "iters": iters, **host}), flush=True)


def save(name, d):
    d = {k: v for k, v in d.items() if v is not None}
    np.savez_compressed(HERE / f"{name}.npz", **d)
    print(f"wrote {name}.npz", {k: getattr(v, 'shape', None) for k, v in d.items()})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("Q3S_REFERENCE"),
                    help="reference checkout (default: $Q3S_REFERENCE)")
    ap.add_argument("--time", action="store_true",
                    help="instead of writing fixtures, time the reference's sampler fragment on this host "
                         "(CPU baseline (i)) with every host thread")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <reference checkout> or set Q3S_REFERENCE")
    ref_paths(Path(args.reference))
    if args.time:
        torch.set_num_threads(os.cpu_count() or 1)
        time_reference()
        return
    torch.set_num_threads(1)
    save("gumbel_cb0_f32", case_gumbel(11, 8, bf16=False))
    save("gumbel_cb0_bf16", case_gumbel(12, 16, bf16=True))
    save("cp_select", case_cp_select(13, 8))
    save("icdf_sample_token", case_icdf_sample_token(14, 12))
    save("icdf_hf_extended", case_icdf_hf_extended(15, 16))


if __name__ == "__main__":
    main()
