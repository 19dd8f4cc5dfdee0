"""``torch.ops.q3s``: the sampler registered as PyTorch operators.

The reference's sampler is a sub-graph of its fused decode graph, so its
torch-side callers (the export and validation code, an eager decode step)
call it as tensor operations.  ``libq3s_torch_ops.so`` (csrc/q3s_torch_ops.cpp)
registers the same call shapes as operators with schemas, CUDA kernels that
call the C ABI of libq3s_sampler.so on the current stream, and Meta kernels
(shapes only) so that tracing and fake-tensor passes see them:

* ``torch.ops.q3s.sample_codebook0(logits, token_counts, gumbel_noise,
  temperature, penalty, suppress_mask=None, topk=50) -> (codec_token_0,
  updated_token_counts)`` -- talker_unified_modules.py:407-422;
* ``torch.ops.q3s.sample_codebook0_(...)`` -- the same with ``token_counts``
  updated in place (the engine's count write-back);
* ``torch.ops.q3s.sample_codebook0_packed(logits, history, offsets, uniforms,
  temperature, top_k, top_p, penalty, min_new_tokens, suppress_mask=None,
  eos_id=2150) -> ids`` -- the batched step over packed ragged histories;
* ``torch.ops.q3s.sample_cp_stage(logits, temperature=None, gumbel_noise=None,
  topk=50) -> ids`` -- CodePredictorUnrolled._select_token (utils.py:1178-1193);
* ``torch.ops.q3s.sample_cp_frame(logits[S,B,V], temperature,
  cp_gumbel_noise=None, topk=50) -> ids[B,S]`` -- the stage loop of
  utils.py:1218-1237 over given stage logits, one persistent launch.

There is no CPU kernel: a CPU tensor raises.
"""
from __future__ import annotations

import threading

import torch

from . import _lib
from .build import TORCH_OPS_PATH

_lock = threading.Lock()
_loaded = False


def load():
    """Register the operators (once) and return ``torch.ops.q3s``."""
    global _loaded
    with _lock:
        if not _loaded:
            _lib.load()  # the C-ABI library the operators call (same file the ops library links)
            if not TORCH_OPS_PATH.exists():
                raise RuntimeError(f"q3s operator library not found at {TORCH_OPS_PATH}; build it with "
                                   "__graft_entry__.build()")
            torch.ops.load_library(str(TORCH_OPS_PATH))
            _loaded = True
    return torch.ops.q3s
