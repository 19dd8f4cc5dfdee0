"""Host-side logic on CPU: Philox known answers, workload sharding, the C ABI
(library loads, exports every declared symbol, validates arguments before any
CUDA call), and the multi-rank gather over gloo."""
import ctypes as C
import os
import re
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import q3s_oracle as O
from q3s import _lib, build, shard, workloads
from q3s.philox import philox4x32_10, row_uniforms, uint32_to_unit_float

REPO = Path(__file__).resolve().parents[1]


# ---- Philox4x32-10 (Salmon et al. SC'11 known-answer vectors) -------------

@pytest.mark.parametrize("ctr,key,want", [
    ([0, 0, 0, 0], [0, 0], [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]),
    ([0xffffffff] * 4, [0xffffffff] * 2, [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]),
    ([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], [0xa4093822, 0x299f31d0],
     [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]),
])
def test_philox_known_answers(ctr, key, want):
    out = philox4x32_10(np.array(ctr, np.uint32), np.array(key, np.uint32))
    assert [int(x) for x in out] == want


def test_uniform_mapping_range():
    u = uint32_to_unit_float(np.array([0, 255, 256, 0xffffffff], np.uint32))
    assert u[0] == 0.0 and u[1] == 0.0 and u[2] == np.float32(2**-24)
    assert u[3] == np.float32(1 - 2**-24) and u[3] < 1.0


def test_row_uniforms_are_per_row_independent():
    full = row_uniforms(5, np.arange(10), cols=3)
    part = row_uniforms(5, np.arange(4, 7), cols=3)
    np.testing.assert_array_equal(full[4:7], part)


# ---- workloads -------------------------------------------------------------

def test_shards_union_equals_full_batch():
    full = workloads.make_batch(1)
    parts = [workloads.make_batch(1, rows=shard.row_range(r, 3, 128)) for r in range(3)]
    assert torch.equal(torch.cat([p.logits for p in parts]).view(torch.int16), full.logits.view(torch.int16))
    assert torch.equal(torch.cat([p.history for p in parts]), full.history)
    for name in ("temperature", "top_k", "top_p", "penalty", "min_new_tokens", "uniforms"):
        assert torch.equal(torch.cat([getattr(p, name) for p in parts]), getattr(full, name))


def test_config_shapes_and_distributions():
    b = workloads.make_batch(1)
    assert b.logits.dtype == torch.bfloat16 and b.logits.shape == (128, 3072)
    lens = np.diff(b.offsets.numpy())
    assert lens.min() >= 16 and lens.max() <= 2048
    assert set(b.top_k.tolist()) <= {20, 50, 100}
    assert float(b.top_p.min()) >= 0.8 and float(b.penalty.max()) <= 1.2
    hi = b.logits[:, 2048:].float()
    assert torch.isinf(hi[:, torch.arange(1024) != 102]).all()  # -inf except EOS 2150
    b0 = workloads.make_batch(0)
    assert b0.logits.dtype == torch.float32 and b0.history.numel() == 256
    b3 = workloads.make_batch(3, rows=(0, 200))
    assert (b3.temperature == 0).any() and np.diff(b3.offsets.numpy()).max() <= 4096
    cp = workloads.make_cp_frame(rows=(0, 4))
    assert cp.base.shape == (15, 4, 2048) and cp.gumbel_noise.shape == (4, 15, 50)


def test_algorithmic_bytes_formula():
    b = workloads.make_batch(1)
    want = 128 * 3072 * 2 + 4 * b.history.numel() + 4 * 129 + 20 * 128 + 4 * 128 + 8 * 128 + 3072
    assert b.algorithmic_bytes() == want


def test_row_range_partitions():
    for total in (1, 7, 128, 4096):
        for world in (1, 2, 3, 8):
            rs = [shard.row_range(r, world, total) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))


# ---- the C ABI without a GPU ----------------------------------------------

@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    header = (REPO / "include" / "q3s_sampler.h").read_text()
    declared = set(re.findall(r"^\s*[\w\s\*]+?\b(q3s_\w+)\s*\(", header, re.M))
    assert declared == set(_lib.EXPORTS)
    for name in declared:
        assert hasattr(lib, name)
    assert lib.q3s_abi_version() == _lib.Q3S_ABI_VERSION
    assert lib.q3s_desc_size(0) == C.sizeof(_lib.SampleDesc)
    assert lib.q3s_desc_size(1) == C.sizeof(_lib.CpFrameDesc)
    assert lib.q3s_desc_size(2) == C.sizeof(_lib.StepDesc)


def _desc(**kw):
    d = _lib.SampleDesc()
    d.struct_size = C.sizeof(_lib.SampleDesc)
    d.mode, d.batch, d.vocab, d.topk = _lib.DRAW_ICDF, 4, 3072, 50
    d.logits_dtype, d.logits_row_stride = _lib.DTYPE_BF16, 3072
    d.logits = 0x1000
    d.uniforms = 0x2000
    d.ids_i64 = 0x3000
    d.temperature_default, d.top_p_default, d.penalty_default = 1.0, 1.0, 1.0
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw,msg", [
    (dict(struct_size=8), "struct_size"),
    (dict(mode=7), "mode"),
    (dict(vocab=0), "vocab"),
    (dict(vocab=9000), "vocab"),
    (dict(logits=None), "logits"),
    (dict(logits_row_stride=100), "stride"),
    (dict(ids_i64=None), "ids"),
    (dict(uniforms=None), "uniforms"),
    (dict(token_counts=0x10, history=0x20, token_counts_row_stride=3072), "not both"),
    (dict(history=0x20, offsets=None), "offsets"),
    (dict(counts_out=0x40, counts_out_row_stride=3072), "token_counts"),
    (dict(penalty_default=0.0), "penalty"),
    (dict(mode=_lib.DRAW_GUMBEL, gumbel_noise=0x50, gumbel_row_stride=50, topk=0), "topk"),
    (dict(mode=_lib.DRAW_GUMBEL, gumbel_noise=0x50, gumbel_row_stride=10, topk=50), "gumbel_row_stride"),
    (dict(logits_dtype=5), "dtype"),
])
def test_sample_rejects_bad_arguments_on_host(lib, kw, msg):
    d = _desc(**kw)
    st = lib.q3s_sample(C.byref(d), None)
    assert st == _lib.ERR_INVALID_ARGUMENT
    assert msg in lib.q3s_last_error_string().decode()


def test_sample_null_desc_and_empty_batch(lib):
    assert lib.q3s_sample(None, None) == _lib.ERR_INVALID_ARGUMENT
    d = _desc(batch=0)
    assert lib.q3s_sample(C.byref(d), None) == _lib.OK  # no-op, no CUDA call


def test_all_greedy_icdf_needs_no_uniforms(lib):
    d = _desc(uniforms=None, temperature_default=0.0, batch=0)
    assert lib.q3s_sample(C.byref(d), None) == _lib.OK


def test_cp_frame_rejects_bad_arguments(lib):
    d = _lib.CpFrameDesc()
    d.struct_size = C.sizeof(_lib.CpFrameDesc)
    d.mode, d.batch, d.vocab, d.stages, d.topk = _lib.DRAW_GUMBEL, 4, 2048, 15, 50
    d.logits_dtype, d.producer = _lib.DTYPE_BF16, _lib.CP_ROTATE
    d.logits, d.ids_out = 0x1000, 0x2000
    d.logits_row_stride, d.logits_stage_stride = 2048, 4 * 2048
    st = lib.q3s_sample_cp_frame(C.byref(d), None)
    assert st == _lib.ERR_INVALID_ARGUMENT and "ids_init" in lib.q3s_last_error_string().decode()
    d.ids_init = 0x3000
    d.stages = 0
    assert lib.q3s_sample_cp_frame(C.byref(d), None) == _lib.ERR_INVALID_ARGUMENT
    d.stages = 15
    d.logits_stage_stride = 100
    assert lib.q3s_sample_cp_frame(C.byref(d), None) == _lib.ERR_INVALID_ARGUMENT


def _step_desc(**kw):
    d = _lib.StepDesc()
    d.struct_size = C.sizeof(_lib.StepDesc)
    d.batch, d.eos_id, d.ids_i64 = 4, 2150, 0x1000
    d.suspect_frames, d.abort_frames, d.emergency_frames, d.min_audio_text_ratio = 4, 10, 20, 2.0
    d.loop_token, d.loop_run, d.loop_max_run = 0x2000, 0x2100, 0x2200
    d.loop_suspect_count, d.loop_recovery_count, d.frame_idx = 0x2300, 0x2400, 0x2500
    d.decode_start_frame, d.text_tokens_consumed, d.input_complete = 0x2600, 0x2700, 0x2800
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw,msg", [
    (dict(struct_size=8), "struct_size"),
    (dict(batch=-1), "batch"),
    (dict(batch=1 << 23), "batch"),
    (dict(ids_i64=None), "exactly one"),
    (dict(ids_i32=0x1100), "exactly one"),
    (dict(loop_run=None), "guard state"),
    (dict(input_complete=None), "progress gate"),
    (dict(min_audio_text_ratio=float("nan")), "NaN"),
    (dict(event_list=0x3000), "event_count"),
    (dict(event_list=0x3000, event_count=0x3100), "compacted from events"),
    (dict(history_out=0x4000), "needs history"),
    (dict(history_out=0x4000, history=0x5000, offsets=0x6000, offsets_out=0x7000, history_len=100,
          history_out_capacity=103), "capacity"),
    (dict(history_out=0x5010, history=0x5000, offsets=0x6000, offsets_out=0x7000, history_len=100,
          history_out_capacity=104), "overlaps history"),
    (dict(history_out=0x9000, history=0x5000, offsets=0x6000, offsets_out=0x6008, history_len=100,
          history_out_capacity=104), "overlaps offsets"),
    # capacity layout: the append is in place, into the same buffer
    (dict(history_lengths=0x8000, history=0x5000, history_out=0x9000, offsets=0x6000,
          history_out_capacity=64), "history_out == history"),
    (dict(history_lengths=0x8000, history=0x5000, history_out=0x5000, history_out_capacity=64),
     "history_out == history"),
    (dict(history_lengths=0x8000, history=0x5000, history_out=0x5000, offsets=0x6000,
          history_out_capacity=-1), "outside"),
])
def test_step_update_rejects_bad_arguments_on_host(lib, kw, msg):
    d = _step_desc(**kw)
    assert lib.q3s_step_update(C.byref(d), None) == _lib.ERR_INVALID_ARGUMENT
    assert msg in lib.q3s_last_error_string().decode()


def test_step_update_guard_off_and_empty_batch(lib):
    assert lib.q3s_step_update(None, None) == _lib.ERR_INVALID_ARGUMENT
    # guard off (abort <= 0): the state arrays are not needed; batch 0 is a no-op
    d = _step_desc(batch=0, abort_frames=0, loop_run=None, input_complete=None)
    assert lib.q3s_step_update(C.byref(d), None) == _lib.OK


def test_sample_rejects_history_lengths_without_history(lib):
    d = _desc(history_lengths=0x8000)
    assert lib.q3s_sample(C.byref(d), None) == _lib.ERR_INVALID_ARGUMENT
    assert "history_lengths" in lib.q3s_last_error_string().decode()


def test_row_history_round_trips_a_packed_history():
    """RowHistory.from_packed places each row at the start of its region and
    packed() gives the packed rows back (host tensors, no GPU)."""
    import numpy as np

    import q3s

    rng = np.random.default_rng(5)
    lens = rng.integers(0, 9, 6)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    hist = rng.integers(0, 3072, int(offs[-1])).astype(np.int32)
    caps = (lens + rng.integers(0, 4, 6)).tolist()
    rh = q3s.RowHistory.from_packed(torch.from_numpy(hist), torch.from_numpy(offs), caps, device="cpu")
    assert rh.offsets.tolist() == np.concatenate([[0], np.cumsum(caps)]).tolist()
    assert rh.lengths.tolist() == lens.tolist()
    ph, po = rh.packed()
    assert ph.tolist() == hist.tolist() and po.tolist() == offs.tolist()
    for b in range(6):
        assert rh.ids[rh.offsets[b]:rh.offsets[b] + lens[b]].tolist() == hist[offs[b]:offs[b + 1]].tolist()
    with pytest.raises(ValueError, match="longer than its capacity"):
        q3s.RowHistory.from_packed(torch.from_numpy(hist), torch.from_numpy(offs), 0, device="cpu")
    rh.reset_rows([1, 3])
    assert rh.lengths.tolist()[1] == 0 and rh.lengths.tolist()[3] == 0


def test_python_api_refuses_cpu_tensors():
    import q3s

    with pytest.raises(RuntimeError, match="CUDA"):
        q3s.SamplePlan(torch.zeros(2, 64), uniforms=torch.zeros(2))


# ---- multi-rank host path over gloo ---------------------------------------

def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, cfg, total, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r0, r1 = shard.row_range(rank, world, total)
        b = workloads.make_batch(cfg, rows=(r0, r1), total_rows=total)
        out = O.sample_icdf(b.logits, uniforms=b.uniforms, temperature=b.temperature, top_k=b.top_k,
                            top_p=b.top_p, penalty=b.penalty, history=b.history.numpy(),
                            offsets=b.offsets.numpy(), min_new_tokens=b.min_new_tokens,
                            suppress=b.suppress.numpy(), eos_id=b.eos_id)
        ids = shard.gather_ids(torch.from_numpy(out["ids"]), total)
        mx = shard.max_over_ranks(float(rank + 1), torch.device("cpu"))
        if rank == 0:
            q.put((ids.numpy(), mx))
    finally:
        dist.destroy_process_group()


def test_sharded_step_over_gloo_equals_single_process():
    total, world = 24, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, 1, total, q)) for r in range(world)]
    for p in procs:
        p.start()
    ids, mx = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    b = workloads.make_batch(1, total_rows=total)
    ref = O.sample_icdf(b.logits, uniforms=b.uniforms, temperature=b.temperature, top_k=b.top_k,
                        top_p=b.top_p, penalty=b.penalty, history=b.history.numpy(), offsets=b.offsets.numpy(),
                        min_new_tokens=b.min_new_tokens, suppress=b.suppress.numpy(), eos_id=b.eos_id)
    np.testing.assert_array_equal(ids, ref["ids"])
    assert mx == 2.0


def _failing_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            raise RuntimeError("rank 1 fails before its step")
        shard.gather_ids(torch.zeros(2, dtype=torch.int64), 4)
        q.put("no-error")
    except RuntimeError as e:  # the survivor sees the collective fail instead of hanging
        q.put(f"error: {type(e).__name__}")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_rank_failure_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msgs = [q.get(timeout=120)]
    for p in procs:
        p.join(timeout=60)
    assert msgs[0].startswith("error")


# ---------------------------------------------------------------------------
# torch.ops.q3s registration (schemas and Meta kernels need no GPU)
# ---------------------------------------------------------------------------

def test_torch_ops_register_schemas_and_meta_kernels():
    import torch

    import q3s

    ops = q3s.load_torch_ops()
    B, V = 4, 3072
    meta = dict(device="meta")
    lg = torch.empty(B, 2, V, dtype=torch.bfloat16, **meta)
    tc = torch.empty(B, V, dtype=torch.int64, **meta)
    col = torch.empty(B, 1, **meta)
    ids, upd = ops.sample_codebook0(lg, tc, torch.empty(B, 50, **meta), col, col, None, 50)
    assert ids.shape == (B,) and ids.dtype == torch.int64 and upd.shape == (B, V) and upd.dtype == torch.int64
    assert ops.sample_codebook0_(lg, tc, torch.empty(B, 50, **meta), col, col, None, 50).shape == (B,)
    i32 = torch.empty(B + 1, dtype=torch.int32, **meta)
    assert ops.sample_codebook0_packed(lg, i32, i32, *([torch.empty(B, **meta)] * 6), None, 2150).shape == (B,)
    assert ops.sample_cp_stage(torch.empty(B, 1, 2048, **meta), None, None, 50).shape == (B,)
    assert ops.sample_cp_frame(torch.empty(15, B, 2048, **meta), col, None, 50).shape == (B, 15)
    schema = str(ops.sample_codebook0_.default._schema)
    assert "Tensor(a!) token_counts" in schema
    for name in ("sample_codebook0", "sample_codebook0_", "sample_codebook0_packed", "sample_cp_stage",
                 "sample_cp_frame"):
        assert hasattr(ops, name)


def test_torch_ops_have_no_cpu_kernel():
    import torch

    import q3s

    ops = q3s.load_torch_ops()
    with pytest.raises(NotImplementedError):
        ops.sample_cp_stage(torch.zeros(2, 2048), None, None, 50)


def test_torch_ops_library_defines_no_libstdcxx_internals():
    """The operator library must use the process's libstdc++ (a private copy
    of its locale machinery crashes when an error message is formatted)."""
    from q3s import build as qbuild

    assert qbuild.TORCH_OPS_PATH.exists()
    assert qbuild.defined_libstdcxx_internals(qbuild.TORCH_OPS_PATH) == []


def test_row_keys_use_all_64_bits():
    """Keys r and r + 2^32 give different streams; keys below 2^32 keep the
    counter (j, r, step, 0xA5A5)."""
    import numpy as np

    from q3s import philox as P

    r = np.array([5, 5 + 2**32, 2**40 + 3], dtype=np.int64)
    u = P.row_uniforms(11, r, cols=8, step=2)
    assert not np.array_equal(u[0], u[1])
    ctr = np.zeros((2, 4), np.uint32)
    ctr[:, 0] = [0, 1]
    ctr[:, 1], ctr[:, 2], ctr[:, 3] = 5, 2, 0xA5A5
    old = P.uint32_to_unit_float(P.philox4x32_10(ctr, np.array([11, 0], np.uint32)).reshape(-1))
    np.testing.assert_array_equal(u[0], old)


def test_seeded_uniforms_depend_only_on_the_row_seed():
    import numpy as np

    from q3s import philox as P

    seeds = [2**63 + 7, 12345, 2**62, 12345 + 2**32]
    a = P.seeded_uniforms(seeds, cols=50, step=3, stage=0)
    b = P.seeded_uniforms(seeds[::-1], cols=50, step=3, stage=0)
    np.testing.assert_array_equal(a, b[::-1])            # batch position does not matter
    assert not np.array_equal(a[1], a[3])                 # all 64 bits of the seed
    assert not np.array_equal(a, P.seeded_uniforms(seeds, cols=50, step=3, stage=1))  # stages differ
    assert not np.array_equal(a, P.seeded_uniforms(seeds, cols=50, step=4, stage=0))  # steps differ
    assert a.min() >= 0.0 and a.max() < 1.0


def test_seeded_uniforms_keep_every_bit_of_large_seeds():
    """Seeds past 2^63 mixed with small ones (a list numpy would turn into
    float64) and int64 tensors (negative = past 2^63) give the same rows."""
    import numpy as np

    from q3s import philox as P

    a = P.seeded_uniforms([3, 2**64 - 1, 2**63 + 1], cols=8)
    b = P.seeded_uniforms(torch.tensor([3, -1, -(2**63) + 1], dtype=torch.int64), cols=8)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(a[1], P.seeded_uniforms([2**64 - 1], cols=8)[0])
    assert not np.array_equal(a[1], P.seeded_uniforms([2**64 - 2], cols=8)[0])


def _head_desc(**kw):
    d = _lib.HeadDesc()
    d.struct_size = C.sizeof(_lib.HeadDesc)
    d.batch, d.hidden_size, d.vocab = 4, 2048, 3072
    d.hidden, d.hidden_row_stride = 0x10000, 2048
    d.weight, d.weight_row_stride = 0x20000, 2048
    d.logits, d.logits_row_stride = 0x30000, 3072
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw,msg", [
    (dict(struct_size=8), "struct_size"),
    (dict(batch=-1), "batch"),
    (dict(hidden_size=1000), "hidden_size"),
    (dict(hidden_size=384), "hidden_size"),
    (dict(vocab=3000), "vocab"),
    (dict(vocab=3040), "vocab"),
    (dict(vocab=16384), "vocab"),
    (dict(logits=None), "required"),
    (dict(weight=0x20008), "aligned"),
    (dict(hidden_row_stride=2047), "row strides"),
    (dict(logits_row_stride=3068), "row strides"),
])
def test_head_rejects_bad_arguments_on_host(lib, kw, msg):
    d = _head_desc(**kw)
    assert lib.q3s_head_sample(C.byref(d), None) == _lib.ERR_INVALID_ARGUMENT
    assert msg in lib.q3s_last_error_string().decode()


def test_head_empty_batch_is_a_no_op(lib):
    assert lib.q3s_head_sample(None, None) == _lib.ERR_INVALID_ARGUMENT
    d = _head_desc(batch=0)
    assert lib.q3s_head_sample(C.byref(d), None) == _lib.OK
