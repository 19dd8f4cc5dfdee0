"""Torch-facing sampler API, mirroring the reference's sampler interfaces.

Each function validates its tensors, fills a C descriptor and calls the CUDA
library through the C ABI on the current CUDA stream; nothing here computes
on the CPU.  The mirrored reference interfaces:

* ``sample_codebook0``  -- the sampler sub-graph of
  ``TalkerUnifiedFusedONNX.forward`` (scripts/export/talker_unified_modules.py:
  407-422): ``(logits, token_counts, gumbel_noise, temperature, penalty) ->
  (codec_token_0, updated_token_counts)``.
* ``select_token``      -- ``CodePredictorUnrolled._select_token``
  (scripts/export/utils.py:1178-1193).
* ``sample_token``      -- ``_sample_token`` (tools/validation/
  prefill_compare.py:383-399) with the ``torch.multinomial`` draw replaced by
  an inverse-CDF draw from caller-supplied uniforms.
* ``sample_packed``     -- the batched form used by the engine step: packed
  ragged histories and per-row temperature / top-k / top-p / penalty /
  min-new-tokens.
* ``sample_cp_frame``   -- the 15-stage loop of ``CodePredictorUnrolled.forward``
  (scripts/export/utils.py:1218-1237) as one persistent kernel.

Errors follow the reference's executor: bad inputs raise ``RuntimeError`` /
``ValueError`` (engine/backend/executor.py:355-365, 395-410).
"""
from __future__ import annotations

import contextlib
import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence, Union

import torch

from . import _lib
from ._lib import CpFrameDesc, SampleDesc

Scalar = Union[float, int]
TensorOrScalar = Union[torch.Tensor, float, int, None]

DEFAULT_VOCAB = 3072       # engine/backend/kv_cache_pool.py:44 (codec_vocab_size)
DEFAULT_EOS = 2150         # talker_unified_modules.py:378 (codec_eos_token_id)
DEFAULT_TOPK = 50          # talker_unified_modules.py:22 (LOGITS_TOPK)
CP_STAGES = 15             # engine/backend/kv_cache_pool.py:46 (cp_num_stages)


def suppress_mask(vocab_size: int = DEFAULT_VOCAB, eos_id: int = DEFAULT_EOS,
                  device: Union[str, torch.device] = "cuda") -> torch.Tensor:
    """bool[V], true for ids in [V-1024, V) except EOS
    (talker_unified_modules.py:384-389)."""
    m = torch.zeros(vocab_size, dtype=torch.bool)
    m[max(0, vocab_size - 1024):] = True
    if 0 <= eos_id < vocab_size:
        m[eos_id] = False
    return m.to(device)


# ---------------------------------------------------------------------------
# validation helpers
# ---------------------------------------------------------------------------

def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need_cuda(t: torch.Tensor, name: str, device: torch.device) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")


def _rows_2d(logits: torch.Tensor, name: str = "logits") -> torch.Tensor:
    """Accept [B,V], or [B,S,V] (last position, as ``logits[:, -1, :]``)."""
    if logits.dim() == 3:
        logits = logits[:, -1, :]
    if logits.dim() != 2:
        raise ValueError(f"{name} must be [B,V] or [B,S,V], got {tuple(logits.shape)}")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    return logits


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.DTYPE_BF16
    if t.dtype == torch.float32:
        return _lib.DTYPE_F32
    raise ValueError(f"logits dtype {t.dtype} unsupported (bf16 or fp32)")


def _row_param(x: TensorOrScalar, B: int, dtype: torch.dtype, device: torch.device,
               name: str) -> tuple[Optional[torch.Tensor], float]:
    """Per-row tensor ([B] or [B,1]) -> (contiguous tensor, 0); scalar -> (None, value)."""
    if x is None:
        return None, 0
    if isinstance(x, torch.Tensor):
        if x.numel() == 1 and B != 1:
            return None, x.item()
        _need_cuda(x, name, device)
        if x.numel() != B:
            raise ValueError(f"{name} has {x.numel()} values for {B} rows")
        return x.reshape(B).to(dtype).contiguous(), 0
    return None, x


def _stream_handle(stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


# ---------------------------------------------------------------------------
# plans: a filled descriptor plus the tensors it points at
# ---------------------------------------------------------------------------

def philox_rows(seed: int, rows: int, cols: int, *, step: int = 0, row0: int = 0,
                row_keys: Optional[torch.Tensor] = None, kind: str = "uniform",
                device: Optional[torch.device] = None, out: Optional[torch.Tensor] = None,
                stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Per-row randomness generated on the GPU in one launch: fp32 ``[rows, cols]``
    uniforms in [0, 1) (``kind="uniform"``) or Gumbel noise
    ``-log(-log(max(u, 1e-8)))`` (``kind="gumbel"``), the same bits as
    ``q3s.philox.row_uniforms(seed, keys, cols, step)`` for the row keys
    ``row_keys`` (int64, on the device) or ``row0 .. row0+rows-1``.  Replaces
    the reference's per-slot ``torch.rand`` + noise transform
    (engine/backend/executor.py:3216-3295)."""
    lib = _lib.load()
    if kind not in ("uniform", "gumbel"):
        raise ValueError(f"kind must be 'uniform' or 'gumbel', got {kind!r}")
    if row_keys is not None:
        dev = row_keys.device
        if dev.type != "cuda":
            raise RuntimeError("row_keys must be a CUDA tensor (no CPU fallback)")
        row_keys = row_keys.reshape(-1).to(torch.int64).contiguous()
        if row_keys.numel() != rows:
            raise ValueError(f"row_keys has {row_keys.numel()} entries for {rows} rows")
    else:
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if out is None:
        out = torch.empty(rows, cols, dtype=torch.float32, device=dev)
    elif out.dtype != torch.float32 or out.dim() != 2 or out.shape != (rows, cols) or out.stride(1) != 1:
        raise ValueError("out must be fp32 [rows, cols] with unit column stride")
    kcode = _lib.PHILOX_UNIFORM if kind == "uniform" else _lib.PHILOX_GUMBEL
    _lib.check(lib.q3s_philox_rows(int(seed) & 0xFFFFFFFFFFFFFFFF, int(step) & 0xFFFFFFFF,
                                   row_keys.data_ptr() if row_keys is not None else None, int(row0), int(rows),
                                   int(cols), kcode, out.data_ptr() if out.numel() else None,
                                   out.stride(0) if out.numel() else cols, _stream_handle(stream)),
               "q3s_philox_rows")
    return out


def philox_seeds(row_seeds: torch.Tensor, cols: int, *, step: int = 0, stage: int = 0, kind: str = "uniform",
                 out: Optional[torch.Tensor] = None, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Per-row randomness from one 64-bit seed per row (``row_seeds``: int64
    [B] on the device, read as unsigned) in one launch: fp32 ``[B, cols]``
    uniforms or Gumbel noise, the same bits as
    ``q3s.philox.seeded_uniforms(seeds, cols, step, stage)``.  The row's seed
    is its Philox key, so the reference's per-slot seeds
    (engine/backend/executor.py:79-86, a retry's salted seed included) map
    one to one; ``stage`` separates codebook 0 from the code-predictor
    stages."""
    lib = _lib.load()
    if kind not in ("uniform", "gumbel"):
        raise ValueError(f"kind must be 'uniform' or 'gumbel', got {kind!r}")
    if row_seeds.device.type != "cuda":
        raise RuntimeError("row_seeds must be a CUDA tensor (no CPU fallback)")
    seeds = row_seeds.reshape(-1).to(torch.int64).contiguous()
    rows = seeds.numel()
    if out is None:
        out = torch.empty(rows, cols, dtype=torch.float32, device=seeds.device)
    elif out.dtype != torch.float32 or out.dim() != 2 or out.shape != (rows, cols) or out.stride(1) != 1:
        raise ValueError("out must be fp32 [rows, cols] with unit column stride")
    kcode = _lib.PHILOX_UNIFORM if kind == "uniform" else _lib.PHILOX_GUMBEL
    _lib.check(lib.q3s_philox_seeds(seeds.data_ptr() if rows else None, int(step) & 0xFFFFFFFF,
                                    int(stage) & 0xFFFFFFFF, rows, int(cols), kcode,
                                    out.data_ptr() if out.numel() else None, out.stride(0) if out.numel() else cols,
                                    _stream_handle(stream)), "q3s_philox_seeds")
    return out


def set_kernel_policy(policy: str) -> str:
    """Choose the kernel family for icdf steps (process-wide): "auto", "cta"
    (register-resident CTA per row), "warp" (shared-memory row kernel, warps
    per row from the batch size) or "w1" / "w2" / "w4" / "w8" / "wmax" (that
    kernel with the warps per row forced; wmax = 12 for V > 2048, 16 below) or "lean" (register-resident row
    kernel, 128 threads a row).  Returns the previous policy.  All return the same ids away from flagged boundary
    rows."""
    codes = {"auto": _lib.POLICY_AUTO, "cta": _lib.POLICY_CTA, "warp": _lib.POLICY_WARP,
             **{f"w{w}": c for w, c in _lib.POLICY_ROW_W.items()}, "lean": _lib.POLICY_LEAN}
    if policy not in codes:
        raise ValueError(f"unknown kernel policy {policy!r}")
    prev = _lib.load().q3s_set_kernel_policy(codes[policy])
    return {v: k for k, v in codes.items()}[prev]


@contextlib.contextmanager
def kernel_policy(policy: str):
    """Run a block under a kernel policy, restoring the previous one."""
    prev = set_kernel_policy(policy)
    try:
        yield
    finally:
        set_kernel_policy(prev)


class SamplePlan:
    """A ready-to-launch ``q3s_sample`` call.

    Holds references to every tensor the descriptor points at, so the plan can
    be launched repeatedly (e.g. inside CUDA-graph capture) with one C call.
    All tensors must live on the same CUDA device; outputs are allocated here
    unless given."""

    def __init__(self, logits: torch.Tensor, *, mode: str = "icdf", topk: int = DEFAULT_TOPK,
                 token_counts: Optional[torch.Tensor] = None,
                 history: Optional[torch.Tensor] = None, offsets: Optional[torch.Tensor] = None,
                 history_lengths: Optional[torch.Tensor] = None,
                 temperature: TensorOrScalar = 1.0, top_k: Optional[torch.Tensor] = None,
                 top_p: TensorOrScalar = 1.0, penalty: TensorOrScalar = 1.0,
                 min_new_tokens: TensorOrScalar = 0, cur_len: Optional[torch.Tensor] = None,
                 gumbel_noise: Optional[torch.Tensor] = None, uniforms: Optional[torch.Tensor] = None,
                 suppress_mask: Optional[torch.Tensor] = None, eos_id: int = -1,
                 col_shift: Optional[torch.Tensor] = None,
                 ids: Optional[torch.Tensor] = None, ids_i32: Optional[torch.Tensor] = None,
                 counts_out: Optional[torch.Tensor] = None,
                 processed: Optional[torch.Tensor] = None, row_flags: Optional[torch.Tensor] = None,
                 error_word: Optional[torch.Tensor] = None, want_ids_i64: bool = True):
        lib = _lib.load()
        self._lib = lib
        logits = _rows_2d(logits)
        dev = logits.device
        if dev.type != "cuda":
            raise RuntimeError("q3s sampler runs on CUDA tensors only (no CPU fallback)")
        B, V = logits.shape
        if mode not in ("icdf", "gumbel"):
            raise ValueError(f"mode must be 'icdf' or 'gumbel', got {mode!r}")
        keep = [logits]
        d = SampleDesc()
        d.struct_size = C.sizeof(SampleDesc)
        d.mode = _lib.DRAW_ICDF if mode == "icdf" else _lib.DRAW_GUMBEL
        d.batch = B
        d.vocab = V
        d.topk = int(topk)
        d.logits_dtype = _dtype_code(logits)
        d.logits_row_stride = logits.stride(0)
        d.logits = logits.data_ptr()
        if col_shift is not None:
            _need_cuda(col_shift, "col_shift", dev)
            col_shift = col_shift.reshape(B).to(torch.int64).contiguous()
            keep.append(col_shift)
            d.col_shift = col_shift.data_ptr()
        if token_counts is not None:
            _need_cuda(token_counts, "token_counts", dev)
            if token_counts.dtype != torch.int64 or token_counts.dim() != 2 or \
                    token_counts.shape != (B, V) or token_counts.stride(1) != 1:
                raise ValueError("token_counts must be int64 [B,V] with unit column stride")
            keep.append(token_counts)
            d.token_counts = token_counts.data_ptr()
            d.token_counts_row_stride = token_counts.stride(0)
        if history is not None:
            if offsets is None:
                raise ValueError("packed history needs offsets [B+1]")
            _need_cuda(history, "history", dev)
            _need_cuda(offsets, "offsets", dev)
            history = history.reshape(-1).to(torch.int32).contiguous()
            offsets = offsets.reshape(-1).to(torch.int32).contiguous()
            if offsets.numel() != B + 1:
                raise ValueError(f"offsets has {offsets.numel()} entries for {B} rows (need B+1)")
            keep += [history, offsets]
            d.history = history.data_ptr() if history.numel() else offsets.data_ptr()
            d.offsets = offsets.data_ptr()
            d.history_len = history.numel()
            if history_lengths is not None:
                # capacity layout: row b = history[offsets[b] : offsets[b] + history_lengths[b]]
                _need_cuda(history_lengths, "history_lengths", dev)
                if history_lengths.dtype != torch.int32 or history_lengths.numel() != B or \
                        not history_lengths.is_contiguous():
                    raise ValueError("history_lengths must be a contiguous int32 [B] tensor")
                keep.append(history_lengths)
                d.history_lengths = history_lengths.data_ptr()
        elif history_lengths is not None:
            raise ValueError("history_lengths needs history and offsets")
        t, tv = _row_param(temperature, B, torch.float32, dev, "temperature")
        d.temperature, d.temperature_default = _ptr(t), float(tv if t is None else 0.0)
        p, pv = _row_param(top_p, B, torch.float32, dev, "top_p")
        d.top_p, d.top_p_default = _ptr(p), float(pv if p is None else 1.0)
        pe, pev = _row_param(penalty, B, torch.float32, dev, "penalty")
        d.penalty, d.penalty_default = _ptr(pe), float(pev if pe is None else 1.0)
        mn, mnv = _row_param(min_new_tokens, B, torch.int32, dev, "min_new_tokens")
        d.min_new_tokens, d.min_new_tokens_default = _ptr(mn), int(mnv if mn is None else 0)
        keep += [x for x in (t, p, pe, mn) if x is not None]
        if top_k is not None:
            if isinstance(top_k, torch.Tensor):
                tk, _ = _row_param(top_k, B, torch.int32, dev, "top_k")
                if tk is None:
                    d.topk = int(top_k.item())
                else:
                    keep.append(tk)
                    d.top_k = tk.data_ptr()
            else:
                d.topk = int(top_k)
        if cur_len is not None:
            cl, clv = _row_param(cur_len, B, torch.int32, dev, "cur_len")
            if cl is None:
                cl = torch.full((B,), int(clv), dtype=torch.int32, device=dev)
            keep.append(cl)
            d.cur_len = cl.data_ptr()
        if gumbel_noise is not None:
            _need_cuda(gumbel_noise, "gumbel_noise", dev)
            g = gumbel_noise.reshape(B, -1)
            if g.dtype != torch.float32 or g.stride(1) != 1:
                g = g.float().contiguous()
            keep.append(g)
            d.gumbel_noise = g.data_ptr()
            d.gumbel_row_stride = g.stride(0)
            if mode == "gumbel" and g.shape[1] < min(int(topk), V):
                raise ValueError(f"gumbel_noise has {g.shape[1]} columns, need {min(int(topk), V)}")
        if uniforms is not None:
            _need_cuda(uniforms, "uniforms", dev)
            u = uniforms.reshape(B).to(torch.float32).contiguous()
            keep.append(u)
            d.uniforms = u.data_ptr()
        if suppress_mask is not None:
            _need_cuda(suppress_mask, "suppress_mask", dev)
            sm = suppress_mask.reshape(-1)
            if sm.numel() != V:
                raise ValueError(f"suppress_mask has {sm.numel()} entries for vocab {V}")
            sm = sm.to(torch.bool).contiguous()
            keep.append(sm)
            d.suppress_mask = sm.data_ptr()
        d.eos_id = int(eos_id) if eos_id is not None else -1
        if ids is None and want_ids_i64:
            ids = torch.empty(B, dtype=torch.int64, device=dev)
        if ids is not None:
            _need_cuda(ids, "ids", dev)
            d.ids_i64 = ids.data_ptr()
        if ids_i32 is not None:
            _need_cuda(ids_i32, "ids_i32", dev)
            d.ids_i32 = ids_i32.data_ptr()
        if counts_out is not None:
            _need_cuda(counts_out, "counts_out", dev)
            if counts_out.dtype != torch.int64 or counts_out.shape != (B, V) or counts_out.stride(1) != 1:
                raise ValueError("counts_out must be int64 [B,V] with unit column stride")
            d.counts_out = counts_out.data_ptr()
            d.counts_out_row_stride = counts_out.stride(0)
        if processed is not None:
            _need_cuda(processed, "processed", dev)
            if processed.dtype != torch.float32 or processed.shape != (B, V) or processed.stride(1) != 1:
                raise ValueError("processed must be fp32 [B,V] with unit column stride")
            d.processed_logits = processed.data_ptr()
            d.processed_row_stride = processed.stride(0)
        if row_flags is not None:
            _need_cuda(row_flags, "row_flags", dev)
            d.row_flags = row_flags.data_ptr()
        if error_word is not None:
            _need_cuda(error_word, "error_word", dev)
            d.error_word = error_word.data_ptr()
        self.desc = d
        self._ref = C.byref(d)
        self._keep = keep
        self.ids, self.ids_i32, self.counts_out = ids, ids_i32, counts_out
        self.processed, self.row_flags, self.error_word = processed, row_flags, error_word
        self.device = dev

    def launch(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        _lib.check(self._lib.q3s_sample(self._ref, _stream_handle(stream)), "q3s_sample")


class HeadPlan:
    """A ready-to-launch ``q3s_head_sample`` call: ``logits = hidden @ weight^T``
    on the tensor cores (the codec head, talker_unified_modules.py:345, or a
    code predictor's lm_heads[stage], utils.py:1223), then, with ``sample``
    (a ``SamplePlan`` bound to the same ``logits`` tensor), that sampling step
    launched behind the head so that it starts while the GEMM runs and reads
    the logits from L2.

    ``hidden`` bf16 [B, H] (or [B, S, H]: the last position), ``weight`` bf16
    [V, H] (``nn.Linear.weight``), ``logits`` bf16 [B, V] (allocated if not
    given).  H must be a multiple of 256 and V of 64."""

    def __init__(self, hidden: torch.Tensor, weight: torch.Tensor, logits: Optional[torch.Tensor] = None, *,
                 sample: Optional["SamplePlan"] = None, error_word: Optional[torch.Tensor] = None):
        lib = _lib.load()
        self._lib = lib
        if hidden.dim() == 3:
            hidden = hidden[:, -1, :]
        if hidden.dim() != 2 or weight.dim() != 2:
            raise ValueError("hidden must be [B,H] (or [B,S,H]) and weight [V,H]")
        dev = hidden.device
        if dev.type != "cuda":
            raise RuntimeError("q3s head runs on CUDA tensors only (no CPU fallback)")
        _need_cuda(weight, "weight", dev)
        if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
            raise ValueError("hidden and weight must be bf16")
        if hidden.stride(1) != 1:
            hidden = hidden.contiguous()
        if weight.stride(1) != 1:
            weight = weight.contiguous()
        B, H = hidden.shape
        V, H2 = weight.shape
        if H2 != H:
            raise ValueError(f"weight is [{V},{H2}] for hidden size {H}")
        if logits is None:
            logits = torch.empty(B, V, dtype=torch.bfloat16, device=dev)
        _need_cuda(logits, "logits", dev)
        if logits.dtype != torch.bfloat16 or logits.shape != (B, V) or logits.stride(1) != 1:
            raise ValueError("logits must be bf16 [B,V] with unit column stride")
        d = _lib.HeadDesc()
        d.struct_size = C.sizeof(_lib.HeadDesc)
        d.batch, d.hidden_size, d.vocab = B, H, V
        d.hidden, d.hidden_row_stride = hidden.data_ptr(), hidden.stride(0) if B > 1 else H
        d.weight, d.weight_row_stride = weight.data_ptr(), weight.stride(0) if V > 1 else H
        d.logits, d.logits_row_stride = logits.data_ptr(), logits.stride(0) if B > 1 else V
        if sample is not None:
            if sample.desc.logits != logits.data_ptr():
                raise ValueError("the sample plan must be bound to the head's logits tensor")
            d.sample = C.addressof(sample.desc)
        if error_word is not None:
            _need_cuda(error_word, "error_word", dev)
            d.error_word = error_word.data_ptr()
        self.desc = d
        self._ref = C.byref(d)
        self._keep = [hidden, weight, logits, sample]
        self.logits, self.sample, self.error_word = logits, sample, error_word
        self.ids = sample.ids if sample is not None else None
        self.device = dev

    def launch(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        _lib.check(self._lib.q3s_head_sample(self._ref, _stream_handle(stream)), "q3s_head_sample")


def head_sample(hidden: torch.Tensor, weight: torch.Tensor, **sample_kwargs) -> tuple[torch.Tensor, torch.Tensor]:
    """``codec_head(hidden)`` and one sampling step over its logits in one call:
    returns (ids int64 [B], logits bf16 [B, V]).  ``sample_kwargs`` are
    ``SamplePlan``'s (mode, history / offsets, temperature, top_k, top_p,
    penalty, uniforms or gumbel_noise, suppress_mask, eos_id, ...)."""
    h = hidden[:, -1, :] if hidden.dim() == 3 else hidden
    logits = torch.empty(h.shape[0], weight.shape[0], dtype=torch.bfloat16, device=hidden.device)
    plan = HeadPlan(hidden, weight, logits, sample=SamplePlan(logits, **sample_kwargs))
    plan.launch()
    return plan.ids, logits


class CpFramePlan:
    """A ready-to-launch ``q3s_sample_cp_frame`` call (see ``sample_cp_frame``)."""

    def __init__(self, logits: torch.Tensor, *, mode: str = "gumbel", topk: int = DEFAULT_TOPK,
                 ids_init: Optional[torch.Tensor] = None, rotate: bool = False,
                 temperature: TensorOrScalar = 1.0, top_p: TensorOrScalar = 1.0,
                 gumbel_noise: Optional[torch.Tensor] = None, uniforms: Optional[torch.Tensor] = None,
                 ids_out: Optional[torch.Tensor] = None, row_flags: Optional[torch.Tensor] = None,
                 error_word: Optional[torch.Tensor] = None):
        lib = _lib.load()
        self._lib = lib
        if logits.dim() != 3 or logits.stride(2) != 1:
            raise ValueError("logits must be [S,B,V] with unit column stride")
        dev = logits.device
        if dev.type != "cuda":
            raise RuntimeError("q3s sampler runs on CUDA tensors only (no CPU fallback)")
        S, B, V = logits.shape
        keep = [logits]
        d = CpFrameDesc()
        d.struct_size = C.sizeof(CpFrameDesc)
        d.mode = _lib.DRAW_ICDF if mode == "icdf" else _lib.DRAW_GUMBEL
        if mode not in ("icdf", "gumbel"):
            raise ValueError(f"mode must be 'icdf' or 'gumbel', got {mode!r}")
        d.batch, d.vocab, d.stages, d.topk = B, V, S, int(topk)
        d.logits_dtype = _dtype_code(logits)
        d.producer = _lib.CP_ROTATE if rotate else _lib.CP_DIRECT
        d.logits = logits.data_ptr()
        d.logits_row_stride = logits.stride(1)
        d.logits_stage_stride = logits.stride(0)
        if rotate:
            if ids_init is None:
                raise ValueError("rotate=True needs ids_init [B]")
            _need_cuda(ids_init, "ids_init", dev)
            ids_init = ids_init.reshape(B).to(torch.int64).contiguous()
            keep.append(ids_init)
            d.ids_init = ids_init.data_ptr()
        t, tv = _row_param(temperature, B, torch.float32, dev, "temperature")
        d.temperature, d.temperature_default = _ptr(t), float(tv if t is None else 0.0)
        p, pv = _row_param(top_p, B, torch.float32, dev, "top_p")
        d.top_p, d.top_p_default = _ptr(p), float(pv if p is None else 1.0)
        keep += [x for x in (t, p) if x is not None]
        if gumbel_noise is not None:
            _need_cuda(gumbel_noise, "gumbel_noise", dev)
            g = gumbel_noise
            if g.dim() != 3 or g.shape[0] != B or g.shape[1] != S:
                raise ValueError("gumbel_noise must be [B,S,K] (cp_gumbel_noise layout)")
            if g.dtype != torch.float32 or g.stride(2) != 1:
                g = g.float().contiguous()
            keep.append(g)
            d.gumbel_noise = g.data_ptr()
            d.gumbel_row_stride = g.stride(0)
            d.gumbel_stage_stride = g.stride(1)
        if uniforms is not None:
            _need_cuda(uniforms, "uniforms", dev)
            u = uniforms.reshape(B, S).to(torch.float32).contiguous()
            keep.append(u)
            d.uniforms = u.data_ptr()
        if ids_out is None:
            ids_out = torch.empty(B, S, dtype=torch.int64, device=dev)
        _need_cuda(ids_out, "ids_out", dev)
        if ids_out.dtype != torch.int64 or ids_out.shape != (B, S) or not ids_out.is_contiguous():
            raise ValueError("ids_out must be contiguous int64 [B,S]")
        d.ids_out = ids_out.data_ptr()
        if row_flags is not None:
            d.row_flags = row_flags.data_ptr()
        if error_word is not None:
            d.error_word = error_word.data_ptr()
        self.desc = d
        self._ref = C.byref(d)
        self._keep = keep
        self.ids = ids_out
        self.row_flags, self.error_word = row_flags, error_word
        self.device = dev

    def launch(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        _lib.check(self._lib.q3s_sample_cp_frame(self._ref, _stream_handle(stream)), "q3s_sample_cp_frame")


# ---------------------------------------------------------------------------
# reference-shaped functions
# ---------------------------------------------------------------------------

def _torch_ops():
    from . import torch_ops

    return torch_ops.load()


def _as_rows(x: TensorOrScalar, device: torch.device) -> torch.Tensor:
    """A per-row parameter as a tensor (a scalar as one value the operator
    broadcasts to every row)."""
    if isinstance(x, torch.Tensor):
        return x
    return torch.full((1,), float(1.0 if x is None else x), dtype=torch.float32, device=device)


def sample_codebook0(logits: torch.Tensor, token_counts: torch.Tensor, gumbel_noise: torch.Tensor,
                     temperature: TensorOrScalar, penalty: TensorOrScalar, *,
                     suppress: Optional[torch.Tensor] = None, topk: int = DEFAULT_TOPK,
                     inplace: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """Drop-in for the codebook-0 sampler of ``TalkerUnifiedFusedONNX.forward``
    (talker_unified_modules.py:407-422).

    ``logits`` [B,V] or [B,S,V] (bf16/fp32; the last position is used),
    ``token_counts`` int64 [B,V], ``gumbel_noise`` fp32 [B,>=K],
    ``temperature`` / ``penalty`` fp32 [B,1] (or scalars), ``suppress`` bool
    [V] (the module's ``suppress_mask`` buffer).  Returns ``codec_token_0``
    int64 [B] and ``updated_token_counts`` = token_counts + one_hot(id): a new
    tensor, or ``token_counts`` itself updated when ``inplace``.  Runs the
    registered operator ``torch.ops.q3s.sample_codebook0`` (``_`` in place)."""
    ops = _torch_ops()
    dev = logits.device
    T = _as_rows(temperature, dev)
    P = _as_rows(penalty, dev)
    if inplace:
        return ops.sample_codebook0_(logits, token_counts, gumbel_noise, T, P, suppress, int(topk)), token_counts
    return ops.sample_codebook0(logits, token_counts, gumbel_noise, T, P, suppress, int(topk))


def select_token(logits: torch.Tensor, *, temperature: TensorOrScalar = None,
                 gumbel_noise: Optional[torch.Tensor] = None, topk: int = DEFAULT_TOPK) -> torch.Tensor:
    """Drop-in for ``CodePredictorUnrolled._select_token`` (utils.py:1178-1193):
    ``logits`` [B,1,V] or [B,V]; no noise -> argmax over the full row; else
    top-min(K,V) -> /T -> +noise -> argmax -> gather.  Returns int64 [B].
    Runs the registered operator ``torch.ops.q3s.sample_cp_stage``."""
    if logits.dim() == 3:
        logits = logits.squeeze(1)
    T = None if temperature is None else _as_rows(temperature, logits.device)
    return _torch_ops().sample_cp_stage(logits, T, gumbel_noise, int(topk))


def _packed_from_hist(hist: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[B,L] id matrix (HF ``input_ids``) -> packed int32 ids + offsets."""
    B, L = hist.shape
    packed = hist.reshape(-1).to(torch.int32).contiguous()
    offsets = torch.arange(0, (B + 1) * L, L, dtype=torch.int32, device=hist.device)
    return packed, offsets


def sample_token(logits: torch.Tensor, hist: torch.Tensor, *, top_k: int, temperature: float,
                 rep_pen: float, suppress: Optional[Sequence[int]], uniforms: torch.Tensor,
                 top_p: float = 1.0, min_new_tokens: int = 0, eos_id: int = DEFAULT_EOS) -> torch.Tensor:
    """``_sample_token`` (prefill_compare.py:383-399) with the multinomial draw
    taken by inverse CDF on ``uniforms`` [B]: suppress ids -> -1e9,
    RepetitionPenalty(rep_pen) over ``hist`` [B,L], (EOS gate), Temperature,
    TopK(top_k), (TopP), softmax, draw.  Returns int64 [B]."""
    logits = _rows_2d(logits)
    B, V = logits.shape
    dev = logits.device
    sm = None
    if suppress:
        sm = torch.zeros(V, dtype=torch.bool, device=dev)
        sm[torch.as_tensor(list(suppress), dtype=torch.long, device=dev)] = True
    if hist.dim() == 1:
        hist = hist.reshape(1, -1).expand(B, -1)
    packed, offsets = _packed_from_hist(hist.to(dev))
    plan = SamplePlan(logits, mode="icdf", topk=int(top_k) if top_k > 0 else 0,
                      history=packed, offsets=offsets, temperature=float(temperature),
                      top_p=float(top_p), penalty=float(rep_pen), min_new_tokens=int(min_new_tokens),
                      uniforms=uniforms, suppress_mask=sm, eos_id=eos_id)
    plan.launch()
    return plan.ids


def sample_packed(logits: torch.Tensor, history: Optional[torch.Tensor], offsets: Optional[torch.Tensor], *,
                  uniforms: Optional[torch.Tensor] = None, temperature: TensorOrScalar = 1.0,
                  top_k: Union[torch.Tensor, int, None] = DEFAULT_TOPK, top_p: TensorOrScalar = 1.0,
                  penalty: TensorOrScalar = 1.0, min_new_tokens: TensorOrScalar = 0,
                  suppress: Optional[torch.Tensor] = None, eos_id: int = DEFAULT_EOS,
                  mode: str = "icdf", gumbel_noise: Optional[torch.Tensor] = None,
                  topk: int = DEFAULT_TOPK, processed: Optional[torch.Tensor] = None,
                  row_flags: Optional[torch.Tensor] = None, error_word: Optional[torch.Tensor] = None,
                  ids: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One batched codebook-0 step over packed ragged histories (int32 ids +
    int32 offsets [B+1]) with per-row parameters.  ``icdf``: temperature <= 0
    marks a greedy row; ``top_k`` <= 0 disables top-k; ``top_p`` >= 1 disables
    top-p.  ``gumbel``: exactly-``topk`` candidates paired with
    ``gumbel_noise`` by rank.  Returns int64 ids [B]."""
    k_arg = top_k if isinstance(top_k, torch.Tensor) else None
    plan = SamplePlan(logits, mode=mode, topk=int(top_k) if isinstance(top_k, int) else topk,
                      history=history, offsets=offsets, temperature=temperature, top_k=k_arg,
                      top_p=top_p, penalty=penalty, min_new_tokens=min_new_tokens, uniforms=uniforms,
                      gumbel_noise=gumbel_noise, suppress_mask=suppress, eos_id=eos_id,
                      processed=processed, row_flags=row_flags, error_word=error_word, ids=ids)
    plan.launch()
    return plan.ids


def sample_cp_frame(logits: torch.Tensor, *, mode: str = "gumbel", ids_init: Optional[torch.Tensor] = None,
                    rotate: bool = False, temperature: TensorOrScalar = 1.0, topk: int = DEFAULT_TOPK,
                    top_p: TensorOrScalar = 1.0, gumbel_noise: Optional[torch.Tensor] = None,
                    uniforms: Optional[torch.Tensor] = None, row_flags: Optional[torch.Tensor] = None,
                    error_word: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All code-predictor stages of a frame in one persistent launch
    (utils.py:1218-1237 sampling loop).  ``logits`` [S,B,V]; with ``rotate``
    stage j reads ``logits[j][b][(v + id_{j-1}[b]) mod V]`` (``id_{-1}`` =
    ``ids_init``), the synthetic stage producer of the benchmark.  ``gumbel``
    takes ``gumbel_noise`` [B,S,K] (``cp_gumbel_noise``; None = greedy);
    ``icdf`` takes ``uniforms`` [B,S].  Returns int64 [B,S]."""
    plan = CpFramePlan(logits, mode=mode, topk=topk, ids_init=ids_init, rotate=rotate,
                       temperature=temperature, top_p=top_p, gumbel_noise=gumbel_noise,
                       uniforms=uniforms, row_flags=row_flags, error_word=error_word)
    plan.launch()
    return plan.ids


@dataclass
class CodecSampler:
    """The sampling half of ``TalkerUnifiedFusedONNX`` (talker_unified_modules.py:
    358-440): owns the static suppress mask built from ``vocab_size`` and
    ``codec_eos_token_id`` and samples codebook 0 plus the code-predictor
    stages with the reference's fixed K."""

    vocab_size: int = DEFAULT_VOCAB
    codec_eos_token_id: int = DEFAULT_EOS
    logits_topk: int = DEFAULT_TOPK
    device: Union[str, torch.device] = "cuda"

    def __post_init__(self):
        self.suppress_mask = suppress_mask(self.vocab_size, self.codec_eos_token_id, self.device)

    def codebook0(self, logits, token_counts, gumbel_noise, temperature, penalty, *, inplace=False):
        return sample_codebook0(logits, token_counts, gumbel_noise, temperature, penalty,
                                suppress=self.suppress_mask, topk=self.logits_topk, inplace=inplace)

    def cp_stage(self, logits, *, temperature=None, gumbel_noise=None):
        return select_token(logits, temperature=temperature, gumbel_noise=gumbel_noise, topk=self.logits_topk)

    def cp_frame(self, logits, *, temperature=None, cp_gumbel_noise=None):
        return sample_cp_frame(logits, mode="gumbel", temperature=1.0 if temperature is None else temperature,
                               topk=self.logits_topk, gumbel_noise=cp_gumbel_noise)
