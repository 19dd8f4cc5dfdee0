"""q3s -- B200-native codec-token sampler for Qwen3TTS-Streaming's decode step.

Python host side over the C ABI of ``include/q3s_sampler.h``; the sampling
itself runs only in the sm_100a kernels of ``libq3s_sampler.so``.
"""
from . import _lib
from .step import RowHistory, StepGuard, step_update
from .ops import (
    CodecSampler,
    CpFramePlan,
    HeadPlan,
    SamplePlan,
    head_sample,
    kernel_policy,
    philox_rows,
    philox_seeds,
    sample_codebook0,
    sample_cp_frame,
    sample_packed,
    sample_token,
    select_token,
    set_kernel_policy,
    suppress_mask,
)

__all__ = [
    "CodecSampler",
    "CpFramePlan",
    "HeadPlan",
    "head_sample",
    "SamplePlan",
    "RowHistory",
    "StepGuard",
    "step_update",
    "kernel_policy",
    "philox_rows",
    "philox_seeds",
    "sample_codebook0",
    "sample_cp_frame",
    "sample_packed",
    "sample_token",
    "select_token",
    "set_kernel_policy",
    "suppress_mask",
    "load_library",
    "load_torch_ops",
]


def load_library():
    """Load the CUDA library (raises if it has not been built)."""
    return _lib.load()


def load_torch_ops():
    """Register ``torch.ops.q3s.*`` (raises if the operator library has not
    been built) and return the namespace."""
    from . import torch_ops

    return torch_ops.load()
