"""ctypes binding of the C ABI in ``include/q3s_sampler.h``.

The structures below mirror the C descriptors field for field; ``load()``
checks their sizes against ``q3s_desc_size`` so a stale library or a layout
drift fails at import instead of corrupting a launch.  There is no CPU
fallback: if the library is missing, ``load()`` raises.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

from .build import LIB_PATH

Q3S_ABI_VERSION = 2
MAX_VOCAB = 8192
MAX_TOPK = 512
MAX_CP_STAGES = 64

OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3
DRAW_GUMBEL, DRAW_ICDF = 0, 1
DTYPE_F32, DTYPE_BF16 = 0, 1
CP_DIRECT, CP_ROTATE = 0, 1
POLICY_AUTO, POLICY_CTA, POLICY_WARP = 0, 1, 2
POLICY_ROW_W = {1: 3, 2: 4, 4: 5, 8: 6, "max": 7}
POLICY_LEAN = 8
PHILOX_UNIFORM, PHILOX_GUMBEL = 0, 1

ROW_DRAW_BOUNDARY, ROW_TOPP_BOUNDARY, ROW_GREEDY, ROW_FALLBACK, ROW_EXACT_CORE = 1, 2, 4, 8, 16
DEVERR_HISTORY_ID, DEVERR_OFFSETS, DEVERR_NO_MASS, DEVERR_WAIT_TIMEOUT, DEVERR_CANDIDATES = 1, 2, 4, 8, 16
DEVERR_HISTORY_FULL = 32

_p = C.c_void_p


class SampleDesc(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("mode", C.c_int32),
        ("batch", C.c_int32),
        ("vocab", C.c_int32),
        ("topk", C.c_int32),
        ("logits_dtype", C.c_int32),
        ("logits_row_stride", C.c_int64),
        ("logits", _p),
        ("col_shift", _p),
        ("token_counts", _p),
        ("token_counts_row_stride", C.c_int64),
        ("history", _p),
        ("offsets", _p),
        ("history_len", C.c_int64),
        ("temperature", _p),
        ("temperature_default", C.c_float),
        ("top_k", _p),
        ("top_p", _p),
        ("top_p_default", C.c_float),
        ("penalty", _p),
        ("penalty_default", C.c_float),
        ("min_new_tokens", _p),
        ("min_new_tokens_default", C.c_int32),
        ("cur_len", _p),
        ("gumbel_noise", _p),
        ("gumbel_row_stride", C.c_int64),
        ("uniforms", _p),
        ("suppress_mask", _p),
        ("eos_id", C.c_int32),
        ("reserved0", C.c_int32),
        ("ids_i64", _p),
        ("ids_i32", _p),
        ("counts_out", _p),
        ("counts_out_row_stride", C.c_int64),
        ("processed_logits", _p),
        ("processed_row_stride", C.c_int64),
        ("row_flags", _p),
        ("error_word", _p),
        ("history_lengths", _p),
    ]


class CpFrameDesc(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("mode", C.c_int32),
        ("batch", C.c_int32),
        ("vocab", C.c_int32),
        ("stages", C.c_int32),
        ("topk", C.c_int32),
        ("logits_dtype", C.c_int32),
        ("producer", C.c_int32),
        ("logits", _p),
        ("logits_row_stride", C.c_int64),
        ("logits_stage_stride", C.c_int64),
        ("ids_init", _p),
        ("temperature", _p),
        ("temperature_default", C.c_float),
        ("top_p", _p),
        ("top_p_default", C.c_float),
        ("gumbel_noise", _p),
        ("gumbel_row_stride", C.c_int64),
        ("gumbel_stage_stride", C.c_int64),
        ("uniforms", _p),
        ("ids_out", _p),
        ("row_flags", _p),
        ("error_word", _p),
    ]


EVT_EOS, EVT_SUSPECT, EVT_RECOVERED, EVT_DEFERRED, EVT_ABORT_PROGRESS, EVT_ABORT_EMERGENCY = 1, 2, 4, 8, 16, 32


class StepDesc(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("batch", C.c_int32),
        ("ids_i64", _p),
        ("ids_i32", _p),
        ("eos_id", C.c_int32),
        ("reserved0", C.c_int32),
        ("history", _p),
        ("offsets", _p),
        ("history_len", C.c_int64),
        ("history_out", _p),
        ("offsets_out", _p),
        ("history_out_capacity", C.c_int64),
        ("suspect_frames", C.c_int32),
        ("abort_frames", C.c_int32),
        ("emergency_frames", C.c_int32),
        ("reserved1", C.c_int32),
        ("min_audio_text_ratio", C.c_double),
        ("loop_token", _p),
        ("loop_run", _p),
        ("loop_max_run", _p),
        ("loop_suspect_count", _p),
        ("loop_recovery_count", _p),
        ("frame_idx", _p),
        ("decode_start_frame", _p),
        ("text_tokens_consumed", _p),
        ("input_complete", _p),
        ("events", _p),
        ("event_run", _p),
        ("event_list", _p),
        ("event_count", _p),
        ("error_word", _p),
        ("history_lengths", _p),
    ]


class HeadDesc(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("batch", C.c_int32),
        ("hidden_size", C.c_int32),
        ("vocab", C.c_int32),
        ("hidden", _p),
        ("hidden_row_stride", C.c_int64),
        ("weight", _p),
        ("weight_row_stride", C.c_int64),
        ("logits", _p),
        ("logits_row_stride", C.c_int64),
        ("sample", _p),
        ("error_word", _p),
        ("reserved0", C.c_int32),
    ]


# every symbol include/q3s_sampler.h declares
EXPORTS = (
    "q3s_sample",
    "q3s_sample_cp_frame",
    "q3s_last_error_string",
    "q3s_abi_version",
    "q3s_desc_size",
    "q3s_set_kernel_policy",
    "q3s_philox_rows",
    "q3s_philox_seeds",
    "q3s_step_update",
    "q3s_head_sample",
)

_lock = threading.Lock()
_lib = None


def load(path: str | Path | None = None) -> C.CDLL:
    """Load (once) and type the library.  Raises if it is missing or stale."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"q3s CUDA library not found at {p}; build it with __graft_entry__.build() "
                "(there is no CPU fallback for the sampler)")
        lib = C.CDLL(str(p))
        lib.q3s_sample.argtypes = [C.POINTER(SampleDesc), _p]
        lib.q3s_sample.restype = C.c_int
        lib.q3s_sample_cp_frame.argtypes = [C.POINTER(CpFrameDesc), _p]
        lib.q3s_sample_cp_frame.restype = C.c_int
        lib.q3s_last_error_string.argtypes = []
        lib.q3s_last_error_string.restype = C.c_char_p
        lib.q3s_abi_version.argtypes = []
        lib.q3s_abi_version.restype = C.c_int32
        lib.q3s_desc_size.argtypes = [C.c_int32]
        lib.q3s_desc_size.restype = C.c_uint32
        lib.q3s_set_kernel_policy.argtypes = [C.c_int32]
        lib.q3s_set_kernel_policy.restype = C.c_int32
        lib.q3s_philox_rows.argtypes = [C.c_uint64, C.c_uint32, _p, C.c_int64, C.c_int32, C.c_int32, C.c_int32,
                                        _p, C.c_int64, _p]
        lib.q3s_philox_rows.restype = C.c_int
        lib.q3s_philox_seeds.argtypes = [_p, C.c_uint32, C.c_uint32, C.c_int32, C.c_int32, C.c_int32, _p, C.c_int64,
                                         _p]
        lib.q3s_philox_seeds.restype = C.c_int
        lib.q3s_step_update.argtypes = [C.POINTER(StepDesc), _p]
        lib.q3s_step_update.restype = C.c_int
        lib.q3s_head_sample.argtypes = [C.POINTER(HeadDesc), _p]
        lib.q3s_head_sample.restype = C.c_int
        if lib.q3s_abi_version() != Q3S_ABI_VERSION:
            raise RuntimeError(f"q3s ABI {lib.q3s_abi_version()} != binding {Q3S_ABI_VERSION}; rebuild")
        for which, st in ((0, SampleDesc), (1, CpFrameDesc), (2, StepDesc), (3, HeadDesc)):
            if lib.q3s_desc_size(which) != C.sizeof(st):
                raise RuntimeError(f"q3s descriptor {st.__name__} size {C.sizeof(st)} != library "
                                   f"{lib.q3s_desc_size(which)}; rebuild")
        if path is None:
            _lib = lib
        return lib


def last_error() -> str:
    return load().q3s_last_error_string().decode("utf-8", "replace")


def check(status: int, what: str) -> None:
    if status != OK:
        raise RuntimeError(f"{what} failed (status {status}): {last_error()}")
