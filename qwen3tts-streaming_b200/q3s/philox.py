"""Host-side Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw,
"Parallel Random Numbers: As Easy as 1, 2, 3", SC'11), written from the paper.

The sampler kernels never generate randomness themselves: the caller supplies
one fp32 uniform per row (inverse-CDF draw) or a ``[B, K]`` block of Gumbel
noise, exactly as the reference engine hands ``gumbel_noise`` /
``cp_gumbel_noise`` to its fused graph (engine/backend/executor.py:3256-3295).
This module produces those arrays reproducibly from ``(seed, stream, index)``
so the kernel and the CPU oracle see the same numbers.

Round function (paper, section 5): with multipliers M0, M1 and the 2x32-bit
key (k0, k1),

    (hi0, lo0) = M0 * x0          (hi1, lo1) = M1 * x2
    x' = (hi1 ^ x1 ^ k0,  lo1,  hi0 ^ x3 ^ k1,  lo0)

and the key is bumped by the Weyl constants (W0, W1) between rounds.
Ten rounds give Philox4x32-10.
"""
from __future__ import annotations

import numpy as np

_M0 = np.uint64(0xD2511F53)
_M1 = np.uint64(0xCD9E8D57)
_W0 = np.uint32(0x9E3779B9)
_W1 = np.uint32(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(counter: np.ndarray, key: np.ndarray) -> np.ndarray:
    """Apply Philox4x32-10 to ``counter`` (uint32 [..., 4]) under ``key``
    (uint32 [..., 2], broadcastable).  Returns uint32 [..., 4]."""
    c = np.asarray(counter, dtype=np.uint32)
    k = np.asarray(key, dtype=np.uint32)
    x0, x1, x2, x3 = (c[..., i].astype(np.uint64) for i in range(4))
    k0 = np.broadcast_to(k[..., 0], c.shape[:-1]).astype(np.uint64)
    k1 = np.broadcast_to(k[..., 1], c.shape[:-1]).astype(np.uint64)
    for rnd in range(10):
        if rnd:
            k0 = (k0 + np.uint64(_W0)) & _MASK32
            k1 = (k1 + np.uint64(_W1)) & _MASK32
        p0 = _M0 * x0
        p1 = _M1 * x2
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK32
        x0, x1, x2, x3 = (hi1 ^ x1 ^ k0, lo1, hi0 ^ x3 ^ k1, lo0)
    return np.stack([x0, x1, x2, x3], axis=-1).astype(np.uint32)


def uint32_to_unit_float(bits: np.ndarray) -> np.ndarray:
    """Map uint32 to fp32 in [0, 1) keeping the top 24 bits: ``(x >> 8) * 2^-24``.
    Every output is exactly representable in fp32 and strictly below 1."""
    b = np.asarray(bits, dtype=np.uint32)
    return ((b >> np.uint32(8)).astype(np.float64) * (1.0 / 16777216.0)).astype(np.float32)


def philox_uniforms(seed: int, stream: int, n: int) -> np.ndarray:
    """``n`` fp32 uniforms in [0,1) for ``(seed, stream)``.

    Key = (seed low 32, seed high 32); counter = (i, stream low 32,
    stream high 32, 0) for block i, each block yielding 4 uniforms."""
    seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    stream = int(stream) & 0xFFFFFFFFFFFFFFFF
    nblk = (int(n) + 3) // 4
    ctr = np.zeros((nblk, 4), dtype=np.uint32)
    ctr[:, 0] = np.arange(nblk, dtype=np.uint64).astype(np.uint32)
    ctr[:, 1] = stream & 0xFFFFFFFF
    ctr[:, 2] = stream >> 32
    key = np.array([seed & 0xFFFFFFFF, seed >> 32], dtype=np.uint32)
    out = philox4x32_10(ctr, key).reshape(-1)[:n]
    return uint32_to_unit_float(out)


def row_uniforms(seed: int, rows: np.ndarray | int, cols: int = 1, step: int = 0) -> np.ndarray:
    """Per-row uniforms keyed by the row's global index, so a row's numbers do
    not depend on which batch (or which rank's shard) it sits in -- the same
    per-lane independence the reference pins for its per-slot generators
    (tests/unit/engine_core/test_executor_trt_engine.py:250-267).

    Returns fp32 ``[len(rows), cols]``; block j of row key r (any 64-bit
    value) uses counter ``(j, r mod 2^32, step, 0xA5A5 ^ (r >> 32))`` under
    key ``seed`` -- for r < 2^32 that is ``(j, r, step, 0xA5A5)``."""
    r = np.arange(rows) if np.isscalar(rows) else np.asarray(rows)
    r = r.astype(np.uint64)
    nblk = (int(cols) + 3) // 4
    ctr = np.zeros((r.shape[0], nblk, 4), dtype=np.uint32)
    ctr[:, :, 0] = np.arange(nblk, dtype=np.uint32)[None, :]
    ctr[:, :, 1] = (r & np.uint64(0xFFFFFFFF)).astype(np.uint32)[:, None]
    ctr[:, :, 2] = np.uint32(int(step) & 0xFFFFFFFF)
    ctr[:, :, 3] = (np.uint64(0xA5A5) ^ (r >> np.uint64(32))).astype(np.uint32)[:, None]
    seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    key = np.array([seed & 0xFFFFFFFF, seed >> 32], dtype=np.uint32)
    bits = philox4x32_10(ctr, key).reshape(r.shape[0], nblk * 4)[:, :cols]
    return uint32_to_unit_float(bits)


def seeded_uniforms(seeds, cols: int, step: int = 0, stage: int = 0) -> np.ndarray:
    """Per-row uniforms from one 64-bit seed per row (the row's Philox key):
    block j of a row with seed q at (step, stage) uses counter
    ``(j, step, stage, 0x5EED)`` under key ``(q mod 2^32, q >> 32)``.  The
    reference seeds one generator per slot with a 63-bit blake2b digest of
    (base seed, request identity, segment[, retry])
    (engine/backend/executor.py:79-86, 3216-3254); with that digest as the
    row's seed, a slot's numbers are its seed's alone, whatever batch or
    shard it sits in.  Returns fp32 ``[len(seeds), cols]``."""
    # element by element as Python ints: a list mixing values past 2^63 with
    # small ones would otherwise become float64 and lose bits
    it = seeds.tolist() if hasattr(seeds, "tolist") else (seeds if isinstance(seeds, (list, tuple)) else [seeds])
    q = np.fromiter((int(x) & 0xFFFFFFFFFFFFFFFF for x in it), dtype=np.uint64)
    nblk = (int(cols) + 3) // 4
    ctr = np.zeros((q.shape[0], nblk, 4), dtype=np.uint32)
    ctr[:, :, 0] = np.arange(nblk, dtype=np.uint32)[None, :]
    ctr[:, :, 1] = np.uint32(int(step) & 0xFFFFFFFF)
    ctr[:, :, 2] = np.uint32(int(stage) & 0xFFFFFFFF)
    ctr[:, :, 3] = np.uint32(0x5EED)
    key = np.stack([(q & np.uint64(0xFFFFFFFF)).astype(np.uint32), (q >> np.uint64(32)).astype(np.uint32)], -1)
    bits = philox4x32_10(ctr, key[:, None, :]).reshape(q.shape[0], nblk * 4)[:, :cols]
    return uint32_to_unit_float(bits)


def gumbel_from_uniforms(u: np.ndarray) -> np.ndarray:
    """The reference's noise transform ``-log(-log(clamp(u, 1e-8, 1)))``
    (engine/backend/executor.py:3293-3295), evaluated in fp32 like torch."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(u, dtype=np.float32)).clamp(1e-8, 1.0)
    return (-torch.log(-torch.log(t))).numpy()
