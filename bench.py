#!/usr/bin/env python
"""Benchmark of the codec-token sampling step (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl q3s|reference]

Workload (the configuration the metric is quoted on): config 1, the
codebook-0 step of a 128-stream continuous batch -- bf16 logits [128,3072],
packed ragged histories U[16,2048], per-row temperature / top-k / top-p /
repetition penalty / min-new-tokens, one Philox uniform per row, inverse-CDF
draw.  With N GPUs every rank samples its own 128 rows of a 128*N-row batch
(weak scaling, no collective on the data path).

Timing (everything that is replayed is captured before the timed region):

* ``value`` / ``ms_per_step``: K launches back to back, replayed from CUDA
  graphs that rotate over G input copies whose footprint is > 3x the 126 MB
  L2.  Inside the barrier + synchronize bracket, ahead of the first event,
  the warm-up replays and an untimed rotation over every copy are enqueued:
  the timed launches read inputs that left L2 long before, and the GPU is
  busy while the host submits, so no host latency lands in the timed region.
  CUDA events on the launching stream, max over ranks.
* ``p50_step_us``: the median, over 9 timed passes of the same K launches
  (the first is the pass ``value`` reports), of the per-launch time.
  ``event_pair_p50_step_us``: up to 256 launches after the same lead-in, each
  a single-launch graph replay between its own event pair (an upper bound:
  the pair adds event records and a graph launch to every step).
  ``cold_isolated_p50_step_us``: K launches each after its own L2 flush (a 2x
  L2 write and a 2x L2 read), the cold-start latency of a lone step.
* ``e2e``: the same metric through the public API (a q3s.SamplePlan bound to
  persistent device buffers, as an engine binds them) with that step's inputs
  copied from pinned host memory and the ids read back every step.

The ids of every timed launch are compared with each other and, after the
timed region, with the CPU oracle on the whole (gathered) batch: bit-exact
except rows flagged as CDF / top-p boundary rows.  A failed check exits 1.

``--impl reference`` times the CPU restatement of the reference sampler (the
oracle) on the host cores with every host thread, on the same configuration.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
import types
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qwen3tts-streaming_b200"))

METRIC = "sampled tokens/sec/GPU at B=128,V=3072 and B=4096; p50 sampling-step µs"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
ROWS_PER_GPU = 128
WORKLOAD = ("cfg1 codebook-0 step: B=128 per GPU, V=3072 bf16, icdf draw with per-row "
            "T/top-k/top-p/penalty/min_new_tokens over packed ragged histories")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["q3s", "reference"], default="q3s")
    ap.add_argument("--no-extra", action="store_true", help="skip the per-config extra measurements")
    ap.add_argument("--extra-steps", type=int, default=200, help="timed launches per extra configuration")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="bound on the CPU-baseline sample")
    ap.add_argument("--e2e-steps", type=int, default=400)
    ap.add_argument("--profile-config", type=int, default=None,
                    help="plain eager launches of one config (0-4; 2 = code-predictor frame) for ncu; "
                         "prints no bench value")
    ap.add_argument("--profile-step", action="store_true",
                    help="with --profile-config 1 or 4: the launches are q3s_step_update appending in place "
                         "into that config's history (capacity layout)")
    ap.add_argument("--profile-packed", action="store_true",
                    help="with --profile-step: the packed layout instead (every row copied with its new id)")
    ap.add_argument("--profile-head", action="store_true",
                    help="with --profile-config 1: the codec head GEMM alone (hidden [B,2048] x W^T, V=3072)")
    ap.add_argument("--profile-gumbel", action="store_true",
                    help="with --profile-config 1: the engine layout (gumbel, token_counts, in-place counts)")
    return ap.parse_args()


def headline_config(world: int) -> dict:
    """The `config` object, identical in both arms."""
    return {"workload": WORKLOAD, "global_batch": ROWS_PER_GPU * world, "rows_per_gpu": ROWS_PER_GPU,
            "parallelism": f"rows sharded over {world} GPU(s), no collective on the data path"}


# ---------------------------------------------------------------------------
# environment helpers
# ---------------------------------------------------------------------------

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def peaks_tflops():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text()).get("bf16_tflops", 0.0)) or None
    return 1590.0


def profile_traffic(name: str):
    """dram bytes per launch from the committed ncu summary, if present."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            return float(line.split(":", 1)[1].split()[0])
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank: int):
        self.samples = []
        self.proc = None
        vis = [x.strip() for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip()]
        self.gpu = vis[local_rank] if local_rank < len(vis) else str(local_rank)
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.time(), parts))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0: float, t1: float):
        win = [p for (t, p) in self.samples if t0 <= t <= t1]
        where = "timed"
        if not win:  # timed region shorter than the sampling period: nearest samples
            win = [p for (t, p) in self.samples if t0 - 0.5 <= t <= t1 + 0.5]
            where = "around_timed"
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(p[1]) for p in win if num(p[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for p in win for n, v in zip(names, p[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(win[0][2]),
                "reasons": reasons, "samples": len(win), "window": where,
                "power_w_max": max((num(p[3]) or 0.0) for p in win)}


# ---------------------------------------------------------------------------
# timing machinery
# ---------------------------------------------------------------------------

class L2Flush:
    """Evicts the 126 MB L2: a write of 2x L2 (leaves dirty lines), then a read
    of another 2x L2 (writes those back and leaves only clean lines), so no
    write-back of the flush lands inside a timed launch."""

    def __init__(self, dev):
        import torch

        n = 2 * L2_BYTES
        self.w = torch.empty(n, dtype=torch.uint8, device=dev)
        self.r = torch.ones(n // 4, dtype=torch.float32, device=dev)
        self.acc = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self):
        import torch

        self.w.zero_()
        torch.sum(self.r, dim=0, out=self.acc)


def barrier(world):
    import torch.distributed as dist

    if world > 1:
        dist.barrier()


def max_ranks(x, world, dev):
    if world == 1:
        return x
    from q3s.shard import max_over_ranks

    return max_over_ranks(x, dev)


class GraphSteps:
    """K launches, back to back, replayed from CUDA graphs that are all
    captured here (before any timing), over G input copies whose footprint is
    > 3x L2: ``rot`` launches every copy once (the untimed lead-in of each
    timed pass: it leaves the copies the timed launches read long out of L2
    and keeps the GPU busy while the host submits); ``graph`` launches the
    first n = min(K, G) copies, replayed K // n times, and ``rem`` the first
    K % n; ``singles`` holds one single-launch graph per copy for the
    per-step pass."""

    MAX_SINGLES = 256

    def __init__(self, plans, stream, steps: int, singles: bool = True):
        import torch

        self.stream = stream
        self.K = steps
        self.G = len(plans)
        self.n = min(steps, self.G)
        self.reps, rem = divmod(steps, self.n)
        with torch.cuda.stream(stream):
            for p in plans[: min(3, self.n)]:
                p.launch(stream)  # module load, attributes, before capture
        stream.synchronize()

        def capture(ps):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for p in ps:
                    p.launch(stream)
            return g

        self.rot = capture(plans)
        self.graph = capture(plans[: self.n])
        self.rem = capture(plans[:rem]) if rem else None
        self.singles = [capture([p]) for p in plans[: min(self.n, self.MAX_SINGLES)]] if singles else []
        stream.synchronize()

    def warm(self, warmup: int, sync: bool = True):
        """Replays the timed graphs (each at least once, >= warmup launches)."""
        import torch

        with torch.cuda.stream(self.stream):
            for _ in range(max(1, math.ceil(warmup / self.n))):
                self.graph.replay()
            if self.rem is not None:
                self.rem.replay()
            self.rot.replay()
        if sync:
            self.stream.synchronize()

    def run(self):
        import torch

        with torch.cuda.stream(self.stream):
            for _ in range(self.reps):
                self.graph.replay()
            if self.rem is not None:
                self.rem.replay()

    def release(self):
        self.rot = self.graph = self.rem = None
        self.singles = []


def timed_back_to_back(gs: GraphSteps, stream, world, dev, warmup: int = 3) -> float:
    """Device ms of gs.K launches, max over ranks.  Inside the barrier +
    synchronize bracket the warm-up replays and the rotation over every copy
    are enqueued ahead of the first event: the GPU stays busy (and at its
    clocks) while the host submits the timed graph, and the timed launches
    read copies that left L2 long before."""
    import torch

    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gs.warm(warmup, sync=False)
    a.record(stream)
    gs.run()
    b.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_ranks(a.elapsed_time(b), world, dev)


def timed_per_step(gs: GraphSteps, stream, world, dev, warmup: int = 3) -> list:
    """Per-launch device ms of the first min(K, G, 256) launches, back to back:
    an event pair around each single-launch graph replay.  The warm-up and
    the rotation over every copy head the pass (milliseconds of GPU work), so
    the host stays ahead of the GPU and no submission latency lands inside an
    event pair; launch i reads copy i, out of L2 since the rotation."""
    import torch

    barrier(world)
    torch.cuda.synchronize()
    gs.warm(warmup, sync=False)
    evs = []
    with torch.cuda.stream(stream):
        for g in gs.singles:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            g.replay()
            b.record(stream)
            evs.append((a, b))
    torch.cuda.synchronize()
    barrier(world)
    return [a.elapsed_time(b) for a, b in evs]


def timed_isolated(launch, steps: int, flush: L2Flush, stream, world, dev, after=None) -> list:
    """Per-launch device ms of `steps` isolated launches, the L2 flushed before
    each (outside its event pair)."""
    import torch

    evs = []
    barrier(world)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(steps):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            launch(stream)
            b.record(stream)
            evs.append((a, b))
            if after is not None:
                after(i)
    torch.cuda.synchronize()
    barrier(world)
    return [a.elapsed_time(b) for a, b in evs]


def p50_over_ranks(times_ms: list, world, dev) -> float:
    return max_ranks(statistics.median(times_ms), world, dev)


def n_copies(bytes_per_copy: int) -> int:
    return max(2, min(4096, math.ceil(3 * L2_BYTES / max(1, bytes_per_copy))))


# ---------------------------------------------------------------------------
# q3s arm
# ---------------------------------------------------------------------------

def clone_batch(b):
    import torch

    kw = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in b.__dict__.items()}
    return type(b)(**kw)


def plan_for(g, **kw):
    import q3s

    return q3s.SamplePlan(g.logits, mode="icdf", history=g.history, offsets=g.offsets, uniforms=g.uniforms,
                          temperature=g.temperature, top_k=g.top_k, top_p=g.top_p, penalty=g.penalty,
                          min_new_tokens=g.min_new_tokens, suppress_mask=g.suppress, eos_id=g.eos_id, **kw)


def gumbel_plan_for(g, counts, **kw):
    """The engine's layout (talker_unified_modules.py:407-422): gumbel noise,
    int64 token_counts updated in place, the suppress buffer."""
    import q3s

    return q3s.SamplePlan(g.logits, mode="gumbel", topk=50, token_counts=counts, counts_out=counts,
                          temperature=g.temperature, penalty=g.penalty, gumbel_noise=g.gumbel_noise,
                          suppress_mask=g.suppress, **kw)


def copies_for(steps: int, base, bytes_step: int) -> list:
    """G copies of one step's inputs, G * bytes > 3x L2 (the timed launches
    rotate through them)."""
    return [base] + [clone_batch(base) for _ in range(n_copies(bytes_step) - 1)]


PASSES = 9  # timed passes behind each p50 (the first is the one `value` reports)


def repeat_passes(gs: GraphSteps, stream, world, dev, warmup: int, first_ms: float, passes: int = PASSES) -> float:
    """p50 (ms per launch) over `passes` timed passes of gs.K launches, the
    first being the pass already timed (``first_ms`` per launch)."""
    per = [first_ms] + [timed_back_to_back(gs, stream, world, dev, warmup) / gs.K for _ in range(passes - 1)]
    return statistics.median(per)


def measure(plans, stream, steps, warmup, world, dev):
    """Back-to-back mean (ms per launch, the first timed pass) and its p50
    over repeated passes of one workload."""
    gs = GraphSteps(plans, stream, steps, singles=False)
    gs.warm(warmup)
    ms = timed_back_to_back(gs, stream, world, dev, warmup) / steps
    p50 = repeat_passes(gs, stream, world, dev, warmup, ms)
    gs.release()
    return ms, p50, None


def measure_config(cfg, rows, total_rows, world, dev, stream, steps, warmup):
    from q3s import workloads

    b = workloads.make_batch(cfg, rows=rows, total_rows=total_rows)
    base = b.to(dev)
    bytes_step = b.algorithmic_bytes()
    plans = [plan_for(g) for g in copies_for(steps, base, bytes_step)]
    ms, p50, _ = measure(plans, stream, steps, warmup, world, dev)
    return ms, p50, bytes_step, b.B


def measure_gumbel_counts(cfg, rows, total_rows, world, dev, stream, steps, warmup):
    """The engine layout on config `cfg`'s logits and histories (as counts)."""
    from q3s import workloads

    b = workloads.make_batch(cfg, rows=rows, total_rows=total_rows)
    base = b.to(dev)
    counts = base.token_counts()
    B, V = b.B, b.V
    # logits, counts read, one count written, T / penalty, noise (K = 50), ids, suppress mask
    bytes_step = B * V * b.logits.element_size() + 8 * B * V + 8 * B + 8 * B + 4 * 50 * B + 8 * B + V
    copies = copies_for(steps, base, bytes_step)
    plans = [gumbel_plan_for(g, counts.clone()) for g in copies]
    ms, p50, _ = measure(plans, stream, steps, warmup, world, dev)
    return ms, p50, bytes_step, B


class _StepPlan:
    """One q3s_step_update launch over its own history copy (the launch
    writes history_out / offsets_out; the guard state is shared)."""

    def __init__(self, guard, ids, history, offsets):
        import torch

        self.guard, self.ids, self.history, self.offsets = guard, ids, history, offsets
        self.h_out = torch.empty(history.numel() + ids.numel(), dtype=torch.int32, device=history.device)
        self.o_out = torch.empty(offsets.numel(), dtype=torch.int32, device=history.device)

    def launch(self, stream=None):
        self.guard.step(self.ids, history=self.history, offsets=self.offsets, history_out=self.h_out,
                        offsets_out=self.o_out, stream=stream)


class _InPlacePlan:
    """One q3s_step_update launch appending in place (capacity layout), with
    its own guard state and row lengths; the id buffer is shared."""

    def __init__(self, guard, ids, rows):
        self.guard, self.ids, self.rows = guard, ids, rows

    def launch(self, stream=None):
        self.guard.step(self.ids, rows=self.rows, stream=stream)


def measure_step(cfg, rows, total_rows, world, dev, stream, steps, warmup, in_place=True):
    """q3s_step_update (EOS + loop guard + the history append) on the history
    of one codebook-0 config: in place into the capacity layout (every launch
    its own guard state and lengths, rotated through > 3x L2), or as the
    packed copy (every launch its own history copy)."""
    import copy

    import numpy as np
    import torch

    import q3s
    from q3s import step as qstep
    from q3s import workloads

    b = workloads.make_batch(cfg, rows=rows, total_rows=total_rows).to(dev)
    B, L = b.B, b.history.numel()
    rng = np.random.default_rng(4242 + cfg)
    progress = dict(frame_idx=rng.integers(0, 200, B), decode_start_frame=rng.integers(0, 50, B),
                    text_tokens_consumed=rng.integers(0, 100, B), input_complete=rng.random(B) < 0.7)
    ids = torch.from_numpy(rng.integers(0, 2048, B)).to(dev)

    def new_guard():
        g = q3s.StepGuard(B, device=dev)  # reference SchedulerConfig thresholds (4 / 10 / 2.0 / 20)
        g.set_progress(**progress)
        return g

    if in_place:
        bytes_step = qstep.algorithmic_bytes_in_place(B)
        n = min(1024, n_copies(bytes_step))
        lens = b.offsets[1:].cpu().long() - b.offsets[:-1].cpu().long()
        base_rows = q3s.RowHistory.from_packed(b.history, b.offsets.cpu(), (lens + 256).tolist(), device=dev)
        plans = []
        for _ in range(n):
            r = copy.copy(base_rows)
            r.lengths = base_rows.lengths.clone()
            plans.append(_InPlacePlan(new_guard(), ids, r))
    else:
        bytes_step = qstep.algorithmic_bytes(B, L)
        n = n_copies(bytes_step)
        guard = new_guard()
        plans = [_StepPlan(guard, ids, b.history, b.offsets)]
        plans += [_StepPlan(guard, ids, b.history.clone(), b.offsets.clone()) for _ in range(n - 1)]
    ms, p50, _ = measure(plans, stream, steps, warmup, world, dev)
    return ms, p50, bytes_step, B


def measure_cp(rows, total_rows, world, dev, stream, frames, warmup):
    """Code-predictor frame: persistent kernel vs 15 single-stage launches."""
    import torch

    import q3s
    from q3s import workloads

    f = workloads.make_cp_frame(rows=rows, total_rows=total_rows)
    base = f.to(dev)
    nbytes = f.algorithmic_bytes()
    R = n_copies(nbytes)
    bases = [base.base] + [base.base.clone() for _ in range(R - 1)]
    frame_plans = [q3s.CpFramePlan(x, mode="gumbel", topk=50, ids_init=base.ids_init, rotate=True,
                                   temperature=base.temperature, gumbel_noise=base.gumbel_noise) for x in bases]
    ms_p, p50_p, _ = measure(frame_plans, stream, frames, warmup, world, dev)

    class Chain:
        def __init__(self, x):
            self.ids = [torch.empty(f.B, dtype=torch.int64, device=dev) for _ in range(f.S)]
            self.stage = []
            prev = base.ids_init
            for j in range(f.S):
                self.stage.append(q3s.SamplePlan(x[j], mode="gumbel", topk=50, temperature=base.temperature,
                                                 gumbel_noise=base.gumbel_noise[:, j, :], col_shift=prev,
                                                 ids=self.ids[j]))
                prev = self.ids[j]

        def launch(self, stream=None):
            for p in self.stage:
                p.launch(stream)

    chains = [Chain(x) for x in bases]
    ms_15, p50_15, _ = measure(chains, stream, frames, warmup, world, dev)
    same = all(torch.equal(torch.stack(c.ids, 1), frame_plans[0].ids) for c in chains[:1])
    return ms_p, p50_p, ms_15, p50_15, nbytes, f.B, same


HEAD_H = 2048  # talker hidden size (engine/backend/kv_cache_pool.py ModelConfig.hidden_size)


class _SeparateHead:
    """cuBLAS (torch.mm) for the head, then the sampler: the unfused path."""

    def __init__(self, hidden, weight, logits, plan):
        self.hidden, self.weight, self.logits, self.plan = hidden, weight, logits, plan

    def launch(self, stream=None):
        import torch

        with torch.cuda.stream(stream) if stream is not None else torch.cuda.stream(torch.cuda.current_stream()):
            torch.mm(self.hidden, self.weight.t(), out=self.logits)
        if self.plan is not None:
            self.plan.launch(stream)


def measure_head(rows, total_rows, world, dev, stream, steps, warmup):
    """The codec head (hidden [B, 2048] x W^T, W [3072, 2048] bf16) and the
    config-1 sampling step over its logits: fused (the tcgen05 head kernel,
    the sampler launched behind it as a programmatic dependent) against
    separate (cuBLAS GEMM, then the sampler); and each GEMM alone."""
    import torch

    import q3s
    from q3s import workloads

    b = workloads.make_batch(1, rows=rows, total_rows=total_rows)
    B, V = b.B, b.V
    g = torch.Generator().manual_seed(2024)
    hidden0 = torch.randn(B, HEAD_H, generator=g).to(torch.bfloat16)
    weight0 = (torch.randn(V, HEAD_H, generator=g) * (3.0 / HEAD_H ** 0.5)).to(torch.bfloat16)
    gemm_bytes = 2 * V * HEAD_H + 2 * B * HEAD_H + 2 * B * V
    bytes_step = gemm_bytes + b.algorithmic_bytes() - B * V * b.logits.element_size() + 2 * B * V
    flops = 2 * B * V * HEAD_H
    G = n_copies(bytes_step)
    sets = []
    for i in range(G):
        gb = b.to(dev)
        logits = torch.empty(B, V, dtype=torch.bfloat16, device=dev)
        sets.append((hidden0.to(dev), weight0.to(dev), logits, gb))

    def sample_plan(logits, gb):
        return plan_for(gb.__class__(**dict(gb.__dict__, logits=logits)))

    fused = [q3s.HeadPlan(h, w, lg, sample=sample_plan(lg, gb)) for h, w, lg, gb in sets]
    separate = [_SeparateHead(h, w, lg, sample_plan(lg, gb)) for h, w, lg, gb in sets]
    head_only = [q3s.HeadPlan(h, w, lg) for h, w, lg, _ in sets]
    cublas_only = [_SeparateHead(h, w, lg, None) for h, w, lg, _ in sets]
    out = {}
    for name, plans in (("fused", fused), ("separate", separate), ("head_gemm", head_only),
                        ("cublas_gemm", cublas_only)):
        ms, p50, _ = measure(plans, stream, steps, warmup, world, dev)
        out[name] = (ms, p50)
    # the fused ids equal the stand-alone sampler's on the head's own logits
    with torch.cuda.stream(stream):
        fused[0].launch(stream)
    stream.synchronize()
    chk = sample_plan(sets[0][2].clone(), sets[0][3])
    with torch.cuda.stream(stream):
        chk.launch(stream)
    stream.synchronize()
    same = bool(torch.equal(chk.ids, fused[0].ids))
    return out, gemm_bytes, bytes_step, flops, B, same


def oracle_icdf_check(batch, ids, flags):
    """The CPU oracle on the whole batch (the checker): returns (rows,
    mismatches, boundary rows, unexplained mismatches)."""
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import q3s_oracle as O

    ref = O.sample_icdf(batch.logits, uniforms=batch.uniforms.numpy(), temperature=batch.temperature.numpy(),
                        top_k=batch.top_k.numpy(), top_p=batch.top_p.numpy(), penalty=batch.penalty.numpy(),
                        history=batch.history.numpy(), offsets=batch.offsets.numpy(),
                        min_new_tokens=batch.min_new_tokens.numpy(), suppress=batch.suppress.numpy(),
                        eos_id=batch.eos_id)
    got = np.asarray(ids)
    bnd = ref["boundary"] | ((np.asarray(flags) & 3) != 0)
    mism = got != ref["ids"]
    return int(got.size), int(mism.sum()), int(bnd.sum()), int((mism & ~bnd).sum())


def cpu_baseline_sample(cfg, seconds, rows=None):
    """Time the oracle (CPU restatement of the reference sampler) on host
    cores: whole-batch steps of config `cfg` until `seconds` have elapsed."""
    import torch

    sys.path.insert(0, str(ROOT / "oracle"))
    import q3s_oracle as O
    from q3s import workloads

    b = workloads.make_batch(cfg, rows=rows)
    args = dict(uniforms=b.uniforms.numpy(), temperature=b.temperature.numpy(), top_k=b.top_k.numpy(),
                top_p=b.top_p.numpy(), penalty=b.penalty.numpy(), history=b.history.numpy(),
                offsets=b.offsets.numpy(), min_new_tokens=b.min_new_tokens.numpy(),
                suppress=b.suppress.numpy(), eos_id=b.eos_id)
    O.sample_icdf(b.logits, **args)  # warm
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        O.sample_icdf(b.logits, **args)
        times.append(time.perf_counter() - t0)
        if len(times) >= 10000:
            break
    p50 = statistics.median(times)
    return {"rows": b.B, "p50_s": p50, "steps": len(times), "threads": torch.get_num_threads()}


def run_q3s(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    import q3s
    from q3s import shard, workloads

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    q3s.load_library()
    stream = torch.cuda.Stream(device=dev)
    K, W = max(1, args.steps), max(3, args.warmup)
    flush = L2Flush(dev)

    # ---- headline: config 1, 128 rows per GPU -----------------------------
    total = ROWS_PER_GPU * world
    r0, r1 = shard.row_range(rank, world, total)
    batch = workloads.make_batch(1, rows=(r0, r1), total_rows=total)
    base = batch.to(dev)
    bytes_step = batch.algorithmic_bytes()
    copies = copies_for(K, base, bytes_step)
    plans = [plan_for(g) for g in copies]
    gs = GraphSteps(plans, stream, K)
    gs.warm(W)

    clocks = ClockSampler(local).start()
    time.sleep(0.3)
    t0 = time.time()
    ms_total = timed_back_to_back(gs, stream, world, dev, W)
    t1 = time.time()
    time.sleep(0.25)
    clocks.stop()
    ms_step = ms_total / K
    launched = plans[: gs.n]
    # the same K launches in further timed passes (p50 over passes), and the
    # first launches again with an event pair around each one
    p50_ms = repeat_passes(gs, stream, world, dev, W, ms_step)
    per = timed_per_step(gs, stream, world, dev, W)
    n_per = len(per)
    gs.release()
    ev_p50_ms = p50_over_ranks(per, world, dev)
    same = all(torch.equal(p.ids, plans[0].ids) for p in launched) and bool((plans[0].ids >= 0).all())

    # cold isolated launches: the L2 flushed before each (the launch also
    # meets cold TLBs and caches), ids kept per launch
    iso_ids = torch.empty(K, r1 - r0, dtype=torch.int64, device=dev)
    iso = timed_isolated(plans[0].launch, K, flush, stream, world, dev,
                         after=lambda i: iso_ids[i].copy_(plans[0].ids))
    iso_p50_ms = p50_over_ranks(iso, world, dev)
    same = same and bool((iso_ids == plans[0].ids.unsqueeze(0)).all())

    # verification launch (row flags) on the same inputs, outside the timed region
    vflags = torch.zeros(r1 - r0, dtype=torch.int32, device=dev)
    verr = torch.zeros(1, dtype=torch.int32, device=dev)
    vplan = plan_for(base, row_flags=vflags, error_word=verr)
    with torch.cuda.stream(stream):
        vplan.launch(stream)
    stream.synchronize()
    same = same and torch.equal(vplan.ids, plans[0].ids)
    ids_all = shard.gather_ids(plans[0].ids, total) if world > 1 else plans[0].ids
    flags_all = shard.gather_ids(vflags, total) if world > 1 else vflags
    same_t = torch.tensor([1 if same else 0], device=dev)
    if world > 1:
        dist.all_reduce(same_t, op=dist.ReduceOp.MIN)
    same = bool(same_t.item())
    err_word = int(verr.item())

    # ---- e2e through the public API with pinned host buffers --------------
    # The engine-style integration: a SamplePlan bound once to persistent
    # device input buffers (as the reference binds its engine's buffers); per
    # step, that step's inputs go host -> device in one copy from a packed
    # pinned buffer, the plan launches, and the ids come back to pinned host
    # memory before the next step.  The per-call API (sample_packed, which
    # builds its descriptor and copies each input separately) is timed too.
    in_keys = ["logits", "history", "offsets", "temperature", "top_k", "top_p", "penalty", "min_new_tokens",
               "uniforms"]
    host = {k: batch.__dict__[k].contiguous() for k in in_keys}
    segs, off = {}, 0
    for k in in_keys:
        nb = host[k].numel() * host[k].element_size()
        segs[k] = (off, nb)
        off += (nb + 255) // 256 * 256
    h_pack = torch.empty(off, dtype=torch.uint8).pin_memory()
    d_pack = torch.empty(off, dtype=torch.uint8, device=dev)
    dview = {}
    for k in in_keys:
        o, nb = segs[k]
        h_pack[o:o + nb].copy_(host[k].reshape(-1).view(torch.uint8))
        dview[k] = d_pack[o:o + nb].view(host[k].dtype).view(host[k].shape)
    h2d = sum(nb for _, nb in segs.values())
    e2e_plan = q3s.SamplePlan(dview["logits"], mode="icdf", history=dview["history"], offsets=dview["offsets"],
                              uniforms=dview["uniforms"], temperature=dview["temperature"], top_k=dview["top_k"],
                              top_p=dview["top_p"], penalty=dview["penalty"],
                              min_new_tokens=dview["min_new_tokens"], suppress_mask=base.suppress,
                              eos_id=batch.eos_id)
    # the plan reads the copied buffers themselves (no conversion copies)
    assert all(getattr(e2e_plan.desc, k) == dview[k].data_ptr() for k in in_keys), "plan not bound to d_pack"
    h_ids = torch.empty(r1 - r0, dtype=torch.int64).pin_memory()
    E = max(1, min(args.e2e_steps, max(K, 200)))

    def e2e_step():
        d_pack.copy_(h_pack, non_blocking=True)
        e2e_plan.launch(stream)
        h_ids.copy_(e2e_plan.ids, non_blocking=True)
        stream.synchronize()
        return h_ids

    pk_host = {k: (v.pin_memory() if isinstance(v, torch.Tensor) else v) for k, v in batch.__dict__.items()}
    pk_dev = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in base.__dict__.items()}

    ops = q3s.load_torch_ops()

    def per_call_step():
        for k in in_keys:
            pk_dev[k].copy_(pk_host[k], non_blocking=True)
        out = ops.sample_codebook0_packed(pk_dev["logits"], pk_dev["history"], pk_dev["offsets"],
                                          pk_dev["uniforms"], pk_dev["temperature"], pk_dev["top_k"],
                                          pk_dev["top_p"], pk_dev["penalty"], pk_dev["min_new_tokens"],
                                          pk_dev["suppress"], batch.eos_id)
        return out.cpu()

    def time_host_loop(step):
        with torch.cuda.stream(stream):
            for _ in range(min(W, 20)):
                step()
            torch.cuda.synchronize()
            barrier(world)
            ta = time.perf_counter()
            for _ in range(E):
                res = step()
            tb = time.perf_counter()
        barrier(world)
        return max_ranks(tb - ta, world, dev), res.clone()

    e2e_s, got = time_host_loop(e2e_step)
    e2e_ok = torch.equal(got, plans[0].ids.cpu())
    pc_s, got_pc = time_host_loop(per_call_step)
    e2e_ok = e2e_ok and torch.equal(got_pc, plans[0].ids.cpu())

    # ---- extra configurations -------------------------------------------------
    extra = {}
    peak = peaks()[0]
    S = max(1, args.extra_steps)
    if not args.no_extra:
        ms0, p0, _, _ = measure_config(0, None, None, world, dev, stream, S, 10)
        extra["cfg0_B1_f32"] = {"us_per_step": round(1000 * ms0, 3), "p50_us": round(1000 * p0, 3),
                                "tokens_per_s": round(1 / (ms0 / 1000))}
        for cfg, n in ((3, 1024), (4, 4096)):
            rr = shard.row_range(rank, world, n)
            ms, p50, by, bb = measure_config(cfg, rr, n, world, dev, stream, S, 10)
            gbs = by / (ms / 1000) / 1e9
            extra[f"cfg{cfg}_B{n}"] = {"us_per_step": round(1000 * ms, 3), "p50_us": round(1000 * p50, 3),
                                       "tokens_per_s": round(n / (ms / 1000)), "rows_per_gpu": bb,
                                       "algorithmic_bytes_per_gpu": by, "achieved_gbs_per_gpu": round(gbs, 1),
                                       "frac_of_measured_hbm": round(gbs / peak, 4)}
        ms, p50, by, bb = measure_gumbel_counts(1, (r0, r1), total, world, dev, stream, S, 10)
        gbs = by / (ms / 1000) / 1e9
        extra["cfg1_gumbel_counts"] = {
            "layout": "engine graph: gumbel exactly-K 50, int64 token_counts [B,V] updated in place, suppress mask",
            "us_per_step": round(1000 * ms, 3), "p50_us": round(1000 * p50, 3), "rows_per_gpu": bb,
            "tokens_per_s": round(total / (ms / 1000)), "algorithmic_bytes_per_gpu": by,
            "achieved_gbs_per_gpu": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 4)}
        for cfg, n, in_place in ((1, total, True), (4, 4096, True), (4, 4096, False)):
            rr = shard.row_range(rank, world, n)
            ms, p50, by, bb = measure_step(cfg, rr, n, world, dev, stream, S, 10, in_place=in_place)
            gbs = by / (ms / 1000) / 1e9
            key = f"step_update_cfg{cfg}_B{n}" + ("" if in_place else "_packed_copy")
            extra[key] = {"history": "capacity layout, in-place append (RowHistory)" if in_place else
                          "packed layout, every row copied with its new id",
                          "us_per_step": round(1000 * ms, 3), "p50_us": round(1000 * p50, 3), "rows_per_gpu": bb,
                          "algorithmic_bytes_per_gpu": by, "achieved_gbs_per_gpu": round(gbs, 1),
                          "frac_of_measured_hbm": round(gbs / peak, 4), "d2h_bytes_per_step": 4}
        hd, gb_, hb_, fl_, hB, h_same = measure_head((r0, r1), total, world, dev, stream, S, 10)
        peak_tf = peaks_tflops()
        extra["cfg1_head_sample_B128"] = {
            "what": "codec head hidden[B,2048] x W[3072,2048]^T (bf16, fp32 accumulation) + the config-1 "
                    "sampling step over its logits",
            "fused_us": round(1000 * hd["fused"][0], 3), "fused_p50_us": round(1000 * hd["fused"][1], 3),
            "separate_cublas_plus_sampler_us": round(1000 * hd["separate"][0], 3),
            "separate_p50_us": round(1000 * hd["separate"][1], 3),
            "head_gemm_us": round(1000 * hd["head_gemm"][0], 3),
            "cublas_gemm_us": round(1000 * hd["cublas_gemm"][0], 3),
            "head_gemm_achieved_gbs": round(gb_ / (hd["head_gemm"][0] / 1000) / 1e9, 1),
            "head_gemm_frac_of_measured_hbm": round(gb_ / (hd["head_gemm"][0] / 1000) / 1e9 / peak, 4),
            "head_gemm_tflops": round(fl_ / (hd["head_gemm"][0] / 1000) / 1e12, 1),
            "head_gemm_frac_of_measured_bf16": round(fl_ / (hd["head_gemm"][0] / 1000) / 1e12 / peak_tf, 4)
            if peak_tf else None,
            "gemm_bytes": gb_, "fused_bytes": hb_, "gemm_flops": fl_, "rows_per_gpu": hB,
            "fused_ids_equal_sampler_on_head_logits": h_same}
        msp, p50p, ms15, p5015, cpb, cb, cp_same = measure_cp((r0, r1), total, world, dev, stream, S, 10)
        extra["cfg2_cp_frame_B128"] = {"persistent_us_per_frame": round(1000 * msp, 3),
                                       "persistent_p50_us": round(1000 * p50p, 3),
                                       "fifteen_launches_us_per_frame": round(1000 * ms15, 3),
                                       "fifteen_launches_p50_us": round(1000 * p5015, 3),
                                       "tokens_per_s_per_gpu": round(cb * 15 / (msp / 1000)),
                                       "algorithmic_bytes_per_frame": cpb,
                                       "achieved_gbs_per_gpu": round(cpb / (msp / 1000) / 1e9, 1),
                                       "persistent_equals_fifteen_launches": bool(cp_same)}

    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        c = cpu_baseline_sample(1, args.cpu_seconds)
        cpu = {"value": round(c["rows"] / c["p50_s"], 1), "unit": "tokens/s", "cores": c["threads"],
               "kind": "port",
               "sample": f"config 1 full batch ({c['rows']} rows) x {c['steps']} steps of the CPU oracle "
                         f"(torch-CPU restatement of the reference sampler chain), p50 step "
                         f"{c['p50_s'] * 1e3:.2f} ms, {os.cpu_count()} host cores visible"}

    # ---- the oracle on the whole (gathered) batch, after all timing -------
    check = None
    if rank == 0:
        full = workloads.make_batch(1, total_rows=total)
        rows, mism, bnd, bad = oracle_icdf_check(full, ids_all.cpu().numpy(), flags_all.cpu().numpy())
        check = {"rows": rows, "mismatches": mism, "boundary_rows": bnd, "unexplained_mismatches": bad}

    peak, peak_kind = peaks()
    achieved = bytes_step / (ms_step / 1000) / 1e9
    traffic = profile_traffic("sample_smem_cfg1_ncu.txt")
    clk = clocks.summary(t0, t1)
    # every rank checks its own launches; rank 0 also holds the oracle's
    # verdict on the gathered batch; all ranks agree on the outcome (MIN)
    ok = bool(same and e2e_ok and err_word == 0 and
              (rank != 0 or (check is not None and check["unexplained_mismatches"] == 0)))
    if world > 1:
        okt = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(okt, op=dist.ReduceOp.MIN)
        ok = bool(okt.item())
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(total / (ms_step / 1000), 1), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(ms_step, 6),
            "p50_step_us": round(1000 * p50_ms, 3), "event_pair_p50_step_us": round(1000 * ev_p50_ms, 3),
            "cold_isolated_p50_step_us": round(1000 * iso_p50_ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: seeded config-1 inputs (bf16 logits N(0,1)*3 +8 spikes, ragged histories, "
                    "per-row params, Philox uniforms)",
            "config": headline_config(world),
            "timing": {
                "value": f"{K} launches back to back from a CUDA graph captured before timing, rotating over "
                         f"{len(copies)} input copies ({len(copies) * bytes_step / 2**20:.0f} MiB > 3x L2); ahead "
                         "of the first event, inside the barrier + synchronize bracket, the warm-up replays and an "
                         "untimed rotation over every copy, so each timed launch reads inputs that left L2 long "
                         "before and no host latency lands in the timed region; CUDA events on the launching "
                         "stream, max over ranks",
                "p50": f"median over {PASSES} timed passes of the same {K} launches (the first is the pass "
                       "`value` reports), each behind the same lead-in; per pass the max over ranks",
                "event_pair_p50": f"{n_per} launches again (copies 0..{n_per - 1}, after the same lead-in), each "
                                  "a single-launch graph replay between its own event pair; median, max over "
                                  "ranks -- an upper bound: the pair adds the event records and a graph launch "
                                  "to every step",
                "cold_isolated_p50": f"{K} launches each after its own L2 flush (outside the event pair): the "
                                     "launch meets cold L2, TLBs and caches; median, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": bytes_step,
                         "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": round(total * E / e2e_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 8 * (r1 - r0), "steps": E,
                    "us_per_step": round(1e6 * e2e_s / E, 2),
                    "api": "q3s.SamplePlan.launch on persistent device buffers; one packed pinned H2D copy "
                           "and one pinned D2H copy of the ids per step, stream synchronised every step",
                    "per_call_api": {"api": "torch.ops.q3s.sample_codebook0_packed (one H2D copy per input "
                                            "tensor, ids via .cpu())",
                                     "us_per_step": round(1e6 * pc_s / E, 2),
                                     "value": round(total * E / pc_s, 1)}},
            "gpu_launches": K,
            "clocks": clk,
            "verified": {"ids_identical_across_launches": bool(same), "e2e_matches_device": bool(e2e_ok),
                         "device_error_word": err_word, "oracle": check, "passed": ok},
            "extra": extra,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    if not ok:
        print(f"bench verification failed on rank {rank}: identical={same} e2e={e2e_ok} "
              f"oracle={check} error_word={err_word}", file=sys.stderr, flush=True)
        sys.exit(1)


# ---------------------------------------------------------------------------
# reference arm: the CPU restatement of the reference sampler
# ---------------------------------------------------------------------------

def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import torch

    # torchrun sets OMP_NUM_THREADS=1: the CPU arm uses every host thread
    torch.set_num_threads(os.cpu_count() or 1)
    K, W = max(1, args.steps), max(3, args.warmup)
    sys.path.insert(0, str(ROOT / "oracle"))
    import q3s_oracle as O
    from q3s import workloads

    total = ROWS_PER_GPU * world
    b = workloads.make_batch(1, total_rows=total)
    a = dict(uniforms=b.uniforms.numpy(), temperature=b.temperature.numpy(), top_k=b.top_k.numpy(),
             top_p=b.top_p.numpy(), penalty=b.penalty.numpy(), history=b.history.numpy(),
             offsets=b.offsets.numpy(), min_new_tokens=b.min_new_tokens.numpy(),
             suppress=b.suppress.numpy(), eos_id=b.eos_id)
    for _ in range(min(W, 3)):
        O.sample_icdf(b.logits, **a)
    budget = 90.0
    times = []
    t_end = time.perf_counter() + budget
    for _ in range(K):
        t0 = time.perf_counter()
        O.sample_icdf(b.logits, **a)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end:
            break
    mean = sum(times) / len(times)
    val = b.B / mean
    threads = torch.get_num_threads()
    line = {"impl": "reference", "metric": METRIC, "value": round(val, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": K, "steps_timed": len(times), "warmup": W, "ms_per_step": round(1000 * mean, 4),
            "p50_step_us": round(1e6 * statistics.median(times), 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: seeded config-1 inputs", "config": headline_config(world),
            "cpu_baseline": {"value": round(val, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"config 1, the whole {b.B}-row batch per step (the oracle: torch-CPU "
                                       f"restatement of the reference sampler chain), {len(times)} steps timed, "
                                       f"{threads} torch threads of {os.cpu_count()} host cores, rank 0 only"},
            "e2e": {"value": round(val, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_profile(args):
    """W + K eager launches of one configuration over 4 input copies (ncu target)."""
    import torch

    import q3s
    from q3s import workloads

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    q3s.load_library()
    cfg = args.profile_config
    if args.profile_step:
        import numpy as np

        b = workloads.make_batch(cfg).to(dev)
        rng = np.random.default_rng(4242 + cfg)
        ids = torch.from_numpy(rng.integers(0, 2048, b.B)).to(dev)
        if args.profile_packed:
            guard = q3s.StepGuard(b.B, device=dev)
            plans = [_StepPlan(guard, ids, b.history if i == 0 else b.history.clone(), b.offsets)
                     for i in range(4)]
        else:
            lens = b.offsets[1:].cpu().long() - b.offsets[:-1].cpu().long()
            plans = []
            for _ in range(4):
                rows = q3s.RowHistory.from_packed(b.history, b.offsets.cpu(), (lens + 256).tolist(), device=dev)
                plans.append(_InPlacePlan(q3s.StepGuard(b.B, device=dev), ids, rows))
    elif args.profile_head:
        b = workloads.make_batch(cfg)
        g = torch.Generator().manual_seed(2024)
        hidden = torch.randn(b.B, HEAD_H, generator=g).to(torch.bfloat16).to(dev)
        weight = (torch.randn(b.V, HEAD_H, generator=g) * (3.0 / HEAD_H ** 0.5)).to(torch.bfloat16).to(dev)
        plans = [q3s.HeadPlan(hidden, weight.clone() if i else weight) for i in range(4)]
    elif cfg == 2:
        f = workloads.make_cp_frame().to(dev)
        plans = [q3s.CpFramePlan(f.base if i == 0 else f.base.clone(), mode="gumbel", topk=50,
                                 ids_init=f.ids_init, rotate=True, temperature=f.temperature,
                                 gumbel_noise=f.gumbel_noise) for i in range(4)]
    elif args.profile_gumbel:
        b = workloads.make_batch(cfg).to(dev)
        counts = b.token_counts()
        plans = [gumbel_plan_for(g, counts.clone()) for g in [b] + [clone_batch(b) for _ in range(3)]]
    else:
        b = workloads.make_batch(cfg).to(dev)
        plans = [plan_for(g) for g in [b] + [clone_batch(b) for _ in range(3)]]
    stream = torch.cuda.current_stream()
    n = max(3, args.warmup) + max(1, args.steps)
    for i in range(n):
        plans[i % len(plans)].launch(stream)
    torch.cuda.synchronize()
    print(json.dumps({"profile": True, "config": cfg, "step_update": bool(args.profile_step),
                      "head": bool(args.profile_head),
                      "gumbel": bool(args.profile_gumbel), "launches": n}), flush=True)


def main():
    args = parse_args()
    if args.profile_config is not None:
        run_profile(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_q3s(args)


if __name__ == "__main__":
    main()
