"""Seeded synthetic inputs for the sampler benchmark configurations.

The reference publishes no dataset or benchmark for this path, so these
generators stand in for it with the shapes, sizes and value distributions of
the five benchmark configurations:

  0  B=1    fp32 [1,3072]   N(0,1)*3, +8 on 5 ids in [0,2048), ids 2048..3071
            = -inf except EOS 2150; history 256 ids; T=0.9 k=50 p=1 pen=1.05
  1  B=128  bf16 [128,3072] same distribution; T~U[0.6,1], k in {20,50,100},
            p~U[0.8,1], pen~U[1,1.2], history lengths U[16,2048],
            min_new_tokens U[0,64]
  2  code-predictor frame: 15 x bf16 [128,2048] N(0,1)*2.5, T=0.9 k=50 p=1,
            no penalty; stage j reads base_j rotated by stage j-1's ids
  3  B=1024 bf16 [1024,3072] as 1 with lengths U[16,4096], 10% greedy rows
  4  B=4096 fp32 [4096,3072] N(0,1)*1.5, top-k off, p=0.95, pen=1.1,
            lengths U[512,4096] (T=1, the suppress mask applies)

Every row is generated from its own generator keyed by (seed, config, global
row index), so any contiguous shard of rows can be produced on its own and
the union of the shards equals the single-GPU batch.  Uniforms and Gumbel
noise come from Philox4x32-10 keyed the same way.
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Optional

import numpy as np
import torch

from .philox import gumbel_from_uniforms, row_uniforms

VOCAB = 3072
CP_VOCAB = 2048
EOS = 2150
CP_STAGES = 15
TOPK = 50


def default_seed(cfg: int) -> int:
    return 1000 + int(cfg)


def suppress_mask_np(vocab: int = VOCAB, eos: int = EOS) -> np.ndarray:
    m = np.zeros(vocab, dtype=bool)
    m[max(0, vocab - 1024):] = True
    if 0 <= eos < vocab:
        m[eos] = False
    return m


@dataclass
class Batch:
    """One codebook-0 sampling step (CPU tensors until ``.to(device)``)."""

    cfg: int
    row0: int
    logits: torch.Tensor          # [B,V] bf16 or fp32
    history: torch.Tensor         # int32 packed ids
    offsets: torch.Tensor         # int32 [B+1]
    temperature: torch.Tensor     # fp32 [B] (0 = greedy)
    top_k: torch.Tensor           # int32 [B] (0 = off)
    top_p: torch.Tensor           # fp32 [B]
    penalty: torch.Tensor         # fp32 [B]
    min_new_tokens: torch.Tensor  # int32 [B]
    uniforms: torch.Tensor        # fp32 [B]
    gumbel_noise: torch.Tensor    # fp32 [B,K] (reference noise transform of Philox uniforms)
    suppress: torch.Tensor        # bool [V]
    eos_id: int = EOS

    @property
    def B(self) -> int:
        return self.logits.shape[0]

    @property
    def V(self) -> int:
        return self.logits.shape[1]

    def to(self, device) -> "Batch":
        kw = {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in self.__dict__.items()}
        return Batch(**kw)

    def token_counts(self) -> torch.Tensor:
        """The same histories in the reference's dense int64 [B,V] count layout."""
        B, V = self.B, self.V
        h = self.history.cpu().long()
        o = self.offsets.cpu().long()
        row = torch.repeat_interleave(torch.arange(B), o[1:] - o[:-1])
        tc = torch.zeros(B, V, dtype=torch.int64)
        tc.index_put_((row, h), torch.ones_like(h), accumulate=True)
        return tc.to(self.logits.device)

    def algorithmic_bytes(self, ids_bytes: int = 8) -> int:
        """Bytes one step must move: logits + packed history + offsets + the
        per-row parameters actually present + uniforms + output ids (+ the
        suppress mask once)."""
        B, V = self.B, self.V
        return (B * V * self.logits.element_size() + 4 * int(self.history.numel()) + 4 * (B + 1)
                + 20 * B + 4 * B + ids_bytes * B + V)


def _row_logits(rng: np.random.Generator, V: int, scale: float, spikes: bool, mask_high: bool) -> np.ndarray:
    x = (rng.standard_normal(V) * scale).astype(np.float32)
    if spikes:
        x[rng.choice(min(V, 2048), size=5, replace=False)] += 8.0
    if mask_high:
        hi = np.arange(max(0, V - 1024), V)
        x[hi[hi != EOS]] = -np.inf
    return x


def make_batch(cfg: int, rows: Optional[tuple[int, int]] = None, seed: Optional[int] = None,
               total_rows: Optional[int] = None) -> Batch:
    """Rows ``[r0, r1)`` of configuration ``cfg`` (default: all its rows)."""
    if cfg not in (0, 1, 3, 4):
        raise ValueError("codebook-0 configs are 0, 1, 3, 4 (config 2 is make_cp_frame)")
    seed = default_seed(cfg) if seed is None else int(seed)
    B_total = {0: 1, 1: 128, 3: 1024, 4: 4096}[cfg] if total_rows is None else int(total_rows)
    r0, r1 = (0, B_total) if rows is None else (int(rows[0]), int(rows[1]))
    V = VOCAB
    n = r1 - r0
    logits = np.empty((n, V), np.float32)
    hists = []
    T = np.empty(n, np.float32)
    K = np.empty(n, np.int32)
    P = np.empty(n, np.float32)
    PEN = np.empty(n, np.float32)
    MN = np.zeros(n, np.int32)
    for i, r in enumerate(range(r0, r1)):
        rng = np.random.default_rng([seed, cfg, r])
        if cfg == 4:
            logits[i] = _row_logits(rng, V, 1.5, spikes=False, mask_high=False)
            L = int(rng.integers(512, 4097))
            hists.append(rng.integers(0, 2048, L, dtype=np.int32))
            T[i], K[i], P[i], PEN[i] = 1.0, 0, 0.95, 1.1
            continue
        logits[i] = _row_logits(rng, V, 3.0, spikes=True, mask_high=True)
        if cfg == 0:
            hists.append(rng.integers(0, 2048, 256, dtype=np.int32))
            T[i], K[i], P[i], PEN[i] = 0.9, 50, 1.0, 1.05
            continue
        hi = 2049 if cfg == 1 else 4097
        L = int(rng.integers(16, hi))
        hists.append(rng.integers(0, 2048, L, dtype=np.int32))
        T[i] = np.float32(rng.uniform(0.6, 1.0))
        K[i] = int(rng.choice([20, 50, 100]))
        P[i] = np.float32(rng.uniform(0.8, 1.0))
        PEN[i] = np.float32(rng.uniform(1.0, 1.2))
        MN[i] = int(rng.integers(0, 65))
        if cfg == 3 and rng.random() < 0.1:
            T[i] = 0.0
    offsets = np.zeros(n + 1, np.int64)
    offsets[1:] = np.cumsum([len(h) for h in hists])
    history = np.concatenate(hists) if hists else np.zeros(0, np.int32)
    lt = torch.from_numpy(logits)
    if cfg in (1, 3):
        lt = lt.to(torch.bfloat16)
    u = row_uniforms(seed, np.arange(r0, r1), cols=1).reshape(-1)
    gu = row_uniforms(seed + 7777, np.arange(r0, r1), cols=TOPK)
    return Batch(cfg=cfg, row0=r0, logits=lt, history=torch.from_numpy(history.astype(np.int32)),
                 offsets=torch.from_numpy(offsets.astype(np.int32)), temperature=torch.from_numpy(T),
                 top_k=torch.from_numpy(K), top_p=torch.from_numpy(P), penalty=torch.from_numpy(PEN),
                 min_new_tokens=torch.from_numpy(MN), uniforms=torch.from_numpy(u),
                 gumbel_noise=torch.from_numpy(gumbel_from_uniforms(gu)),
                 suppress=torch.from_numpy(suppress_mask_np(V, EOS)))


@dataclass
class CpFrame:
    """One code-predictor frame: base stage logits and the stage inputs."""

    base: torch.Tensor          # bf16 [S,B,V]
    ids_init: torch.Tensor      # int64 [B] (id_{-1} of the rotation producer)
    temperature: torch.Tensor   # fp32 [B]
    uniforms: torch.Tensor      # fp32 [B,S]
    gumbel_noise: torch.Tensor  # fp32 [B,S,K]
    topk: int = TOPK
    top_p: float = 1.0

    @property
    def S(self) -> int:
        return self.base.shape[0]

    @property
    def B(self) -> int:
        return self.base.shape[1]

    @property
    def V(self) -> int:
        return self.base.shape[2]

    def to(self, device) -> "CpFrame":
        kw = {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in self.__dict__.items()}
        return CpFrame(**kw)

    def algorithmic_bytes(self) -> int:
        S, B, V = self.S, self.B, self.V
        return S * B * V * self.base.element_size() + 8 * B + 4 * B + 8 * B * S + 4 * B * S


def make_cp_frame(rows: Optional[tuple[int, int]] = None, seed: Optional[int] = None,
                  total_rows: int = 128, stages: int = CP_STAGES, vocab: int = CP_VOCAB) -> CpFrame:
    """Configuration 2: ``base[j,b,:]`` ~ N(0,1)*2.5 (bf16), T=0.9, k=50, p=1."""
    seed = default_seed(2) if seed is None else int(seed)
    r0, r1 = (0, total_rows) if rows is None else (int(rows[0]), int(rows[1]))
    n = r1 - r0
    base = np.empty((stages, n, vocab), np.float32)
    init = np.empty(n, np.int64)
    for i, r in enumerate(range(r0, r1)):
        rng = np.random.default_rng([seed, 2, r])
        base[:, i, :] = rng.standard_normal((stages, vocab)).astype(np.float32) * np.float32(2.5)
        init[i] = int(rng.integers(0, vocab))
    u = row_uniforms(seed, np.arange(r0, r1), cols=stages)
    gu = row_uniforms(seed + 7777, np.arange(r0, r1), cols=stages * TOPK).reshape(n, stages, TOPK)
    return CpFrame(base=torch.from_numpy(base).to(torch.bfloat16), ids_init=torch.from_numpy(init),
                   temperature=torch.full((n,), 0.9, dtype=torch.float32), uniforms=torch.from_numpy(u),
                   gumbel_noise=torch.from_numpy(gumbel_from_uniforms(gu)))
