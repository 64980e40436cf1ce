"""CPU oracle for the cid-engine display-refinement path — TEST INFRASTRUCTURE.

Python entry points over ``libcid_oracle.so`` (a plain-C restatement of the
reference CPU backend, ``oracle/cid_oracle.c``).  Signatures and error
behaviour follow the reference's ``torch.ops.cid_engine`` operators
(fwerkor/cid-engine v1.1.0, ``csrc/registration.cpp:5-49``): inputs are torch
tensors (any device; they are copied to the host), outputs are CPU tensors.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg use this module, and only as the checker.  The product never imports it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import torch

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "libcid_oracle.so"
_lib: ctypes.CDLL | None = None

DT = {
    torch.float32: 0,
    torch.float64: 1,
    torch.float16: 2,
    torch.bfloat16: 3,
    torch.bool: 4,
    torch.int64: 5,
    torch.int32: 6,
    torch.uint8: 7,
    torch.int8: 8,
    torch.int16: 9,
}


def build() -> Path:
    """Compile the C restatement (``make -C oracle``) if it is missing or stale."""
    src = [_HERE / "cid_oracle.c", _HERE / "cid_oracle.h"]
    if not _LIB_PATH.exists() or any(
        p.stat().st_mtime > _LIB_PATH.stat().st_mtime for p in src
    ):
        subprocess.run(
            ["make", "-C", str(_HERE), "libcid_oracle.so"],
            check=True,
            stdout=subprocess.DEVNULL,
        )
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(str(_LIB_PATH))
    return _lib


def _host(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu").contiguous()


def _p(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _i(x: int) -> ctypes.c_int64:
    return ctypes.c_int64(int(x))


def _d(x: float) -> ctypes.c_double:
    return ctypes.c_double(float(x))


def _check(rc: int, message: str) -> None:
    if rc == -2:
        raise IndexError(message)
    if rc != 0:
        raise RuntimeError(message)


def display_token_statistics(token_ids: torch.Tensor, logits: torch.Tensor):
    """csrc/cpu/display_stats.cpp:54-126 (f32/f16/bf16) and csrc/ops.cpp:446-474.

    Confidences are the exactly rounded values: the sum of exp(x - max) is
    taken in double and rounded to float32 once."""
    return _stats(token_ids, logits, "cid_oracle_display_stats")


def display_token_statistics_reference_order(token_ids: torch.Tensor, logits: torch.Tensor):
    """csrc/cpu/display_stats.cpp:14-50 evaluated in the reference's own
    float32 order (8 lanes of ATen's generic Vectorized<float>, libm expf,
    serial horizontal sum), so the confidences carry the reference's own
    rounding; argmax is identical to ``display_token_statistics``."""
    return _stats(token_ids, logits, "cid_oracle_display_stats_reference_order")


def _stats(token_ids: torch.Tensor, logits: torch.Tensor, entry: str):
    ids = _host(token_ids)
    lg = _host(logits)
    if ids.dtype != torch.int64:
        raise RuntimeError("token_ids must use torch.int64")
    conf = torch.empty(ids.shape, dtype=torch.float32)
    cur = torch.empty(ids.shape, dtype=torch.float32)
    pred = torch.empty(ids.shape, dtype=torch.int64)
    rows = ids.numel()
    if rows == 0:
        return conf, pred, cur
    rc = getattr(lib(), entry)(
        DT[lg.dtype], _p(lg), _p(ids), _i(rows), _i(lg.shape[-1]),
        _p(conf), _p(pred), _p(cur),
    )
    _check(rc, "token id is outside vocabulary size")
    return conf, pred, cur


def display_token_statistics_with_repetition(
    token_ids, logits, mask_token_id, eos_token_id, repetition_score_multiplier=0.7
):
    """csrc/ops.cpp:477-552."""
    ids = _host(token_ids)
    lg = _host(logits)
    conf = torch.empty(ids.shape, dtype=torch.float32)
    cur = torch.empty(ids.shape, dtype=torch.float32)
    pred = torch.empty(ids.shape, dtype=torch.int64)
    if ids.numel() == 0:
        return conf, pred, cur
    rc = lib().cid_oracle_display_stats_repetition(
        DT[lg.dtype], _p(lg), _p(ids), _i(ids.shape[0]), _i(ids.shape[1]),
        _i(lg.shape[-1]), _i(mask_token_id), ctypes.c_int(eos_token_id is not None),
        _i(eos_token_id if eos_token_id is not None else -1),
        _d(repetition_score_multiplier), _p(conf), _p(pred), _p(cur),
    )
    _check(rc, "repetition_score_multiplier must be in (0, 1] / token id out of range")
    return conf, pred, cur


def refine_display_from_statistics(
    token_ids, confidence, predicted, current_confidence, mask_token_id,
    eos_token_id, reveal_fraction, revision_fraction, revision_margin,
):
    """csrc/refine.cpp:222-429."""
    ids = _host(token_ids)
    conf = _host(confidence).float()
    pred = _host(predicted)
    cur = _host(current_confidence).float()
    out = torch.empty_like(ids)
    if ids.numel() == 0:
        return out
    rc = lib().cid_oracle_refine(
        _p(ids), _p(conf), _p(pred), _p(cur), _i(ids.shape[0]), _i(ids.shape[1]),
        _i(mask_token_id), ctypes.c_int(eos_token_id is not None),
        _i(eos_token_id if eos_token_id is not None else -1),
        _d(reveal_fraction), _d(revision_fraction), _d(revision_margin), _p(out),
    )
    _check(rc, "refine fractions must be in [0, 1] and margin non-negative")
    return out


def prefix_allocation_mask(occupancy, allocation_logits, threshold, max_allocations):
    """csrc/ops.cpp:41-65."""
    occ = _host(occupancy)
    if occ.dim() == 3:
        occ = occ.squeeze(-1).contiguous()
    lg = _host(allocation_logits)
    out = torch.empty(occ.shape, dtype=torch.bool)
    rc = lib().cid_oracle_prefix_allocation(
        DT[occ.dtype], _p(occ), DT[lg.dtype], _p(lg), _i(occ.shape[0]),
        _i(occ.shape[1]), _d(threshold), _i(max_allocations), _p(out),
    )
    _check(rc, "threshold must be in [0, 1] and max_allocations positive")
    return out


def rollout_slot_transition(
    occupancy, allocation_logits, lifecycle_logits, revision_logits, input_lifecycle,
    threshold, max_allocations, retired_index,
):
    """csrc/ops.cpp:184-256."""
    occ = _host(occupancy)
    if occ.dim() == 3:
        occ = occ.squeeze(-1).contiguous()
    al = _host(allocation_logits)
    dtype = al.dtype
    lc = _host(lifecycle_logits).to(dtype)
    rv = _host(revision_logits).to(dtype)
    il = _host(input_lifecycle).to(dtype)
    b, s = occ.shape
    outs = (
        torch.empty((b, s), dtype=torch.bool),
        torch.empty((b, s), dtype=torch.int64),
        torch.empty((b, s), dtype=torch.int64),
        torch.empty((b, s), dtype=torch.int64),
        torch.empty((b, s), dtype=torch.bool),
        torch.empty((b, s), dtype=torch.bool),
    )
    rc = lib().cid_oracle_rollout(
        DT[occ.dtype], _p(occ), DT[dtype], _p(al), _p(lc), _p(rv), _p(il),
        _i(b), _i(s), _i(lc.shape[-1]), _i(rv.shape[-1]), _d(threshold),
        _i(max_allocations), _i(retired_index), *[_p(o) for o in outs],
    )
    _check(rc, "invalid rollout arguments")
    return outs


def live_slot_occupancy(slot_occupancy, lifecycle_features, retired_index):
    """csrc/ops.cpp:12-39 (same-dtype inputs)."""
    occ = _host(slot_occupancy)
    out = torch.empty_like(occ)
    lc = None if lifecycle_features is None else _host(lifecycle_features).to(occ.dtype)
    feats = 0 if lc is None else lc.shape[-1]
    rc = lib().cid_oracle_live_occupancy(
        DT[occ.dtype], _p(occ), _p(lc), _i(occ.numel()), _i(feats),
        _i(retired_index), _p(out),
    )
    _check(rc, "retired_index is outside lifecycle_features")
    return out


def materialize_cell_snapshot(
    thought_semantic, role_logits, uncertainty, noise_delta, lifecycle_logits,
    selected, semantic_indices,
):
    """csrc/ops.cpp:556-615."""
    sem = _host(thought_semantic)
    roles = _host(role_logits)
    unc = _host(uncertainty)
    noise = _host(noise_delta)
    life = _host(lifecycle_logits)
    sel = _host(selected)
    idx = _host(semantic_indices)
    b, s, h = sem.shape
    out = torch.empty((b, s, 4 + roles.shape[-1] + idx.numel()), dtype=torch.float32)
    rc = lib().cid_oracle_snapshot(
        DT[sem.dtype], _p(sem), _i(h), DT[roles.dtype], _p(roles), _i(roles.shape[-1]),
        DT[unc.dtype], _p(unc), DT[noise.dtype], _p(noise), DT[life.dtype], _p(life),
        _i(life.shape[-1]), _p(sel), _p(idx), _i(idx.numel()), _i(b * s), _p(out),
    )
    _check(rc, "semantic_indices contain values outside semantic width")
    return out


def masked_diffusion_corrupt_from_random(
    clean_ids, ratio_random, mask_random, mask_token_id, min_mask_ratio, max_mask_ratio
):
    """csrc/ops.cpp:394-444."""
    clean = _host(clean_ids)
    rr = _host(ratio_random)
    mr = _host(mask_random)
    b, t = clean.shape
    corrupted = torch.empty_like(clean)
    masked = torch.empty((b, t), dtype=torch.bool)
    ratio = torch.empty((b, 1), dtype=torch.float32)
    metrics = torch.empty(2, dtype=torch.float32)
    rc = lib().cid_oracle_masked_diffusion(
        _p(clean), DT[rr.dtype], _p(rr), DT[mr.dtype], _p(mr), _i(b), _i(t),
        _i(mask_token_id), _d(min_mask_ratio), _d(max_mask_ratio),
        _p(corrupted), _p(masked), _p(ratio), _p(metrics),
    )
    _check(rc, "mask ratio range must satisfy 0 < min <= max <= 1")
    return corrupted, masked, ratio, metrics


def thought_corrupt_from_epsilon(semantic, timesteps, occupancy, epsilon):
    """csrc/ops.cpp:258-290."""
    sem = _host(semantic)
    ts = _host(timesteps)
    occ = _host(occupancy)
    eps = _host(epsilon)
    b, s, h = sem.shape
    corrupted = torch.empty_like(sem)
    local = torch.empty((b, s, 1), dtype=sem.dtype)
    masked_eps = torch.empty_like(sem)
    rc = lib().cid_oracle_thought(
        DT[sem.dtype], _p(sem), DT[ts.dtype], _p(ts), DT[occ.dtype], _p(occ),
        _p(eps), _i(b * s), _i(h), _p(corrupted), _p(local), _p(masked_eps),
    )
    _check(rc, "invalid thought corruption arguments")
    return corrupted, local, masked_eps


def display_corrupt_from_random(
    token_ids, timesteps, eligible_mask, corruption_random, replacement_random,
    replacement_offsets, mask_token_id, eos_token_id, vocab_size, replacement_fraction,
):
    """csrc/ops.cpp:292-391."""
    ids = _host(token_ids)
    ts = _host(timesteps)
    el = _host(eligible_mask)
    cr = _host(corruption_random)
    rr = None if replacement_random is None else _host(replacement_random)
    ro = None if replacement_offsets is None else _host(replacement_offsets)
    b, t = ids.shape
    if replacement_fraction > 0.0 and (rr is None or ro is None):
        raise RuntimeError("replacement random tensors are required when "
                           "replacement_fraction > 0")  # csrc/ops.cpp:347-349
    corrupted = torch.empty_like(ids)
    labels = torch.empty_like(ids)
    masked = torch.empty((b, t), dtype=torch.bool)
    replaced = torch.empty((b, t), dtype=torch.bool)
    rc = lib().cid_oracle_display_corrupt(
        _p(ids), DT[ts.dtype], _p(ts), DT[el.dtype], _p(el), DT[cr.dtype], _p(cr),
        DT[rr.dtype] if rr is not None else 0, _p(rr), _p(ro), _i(b), _i(t),
        _i(mask_token_id), ctypes.c_int(eos_token_id is not None),
        _i(eos_token_id if eos_token_id is not None else -1), _i(vocab_size),
        _d(replacement_fraction), _p(corrupted), _p(labels), _p(masked), _p(replaced),
    )
    _check(rc, "invalid display corruption arguments")
    return corrupted, labels, masked, replaced


def set_num_threads(n: int) -> None:
    """OpenMP thread count used by the C restatement."""
    os.environ["OMP_NUM_THREADS"] = str(n)


def display_shard_records(token_ids, logits_shard, vocab_offset, total_vocab):
    """Per-row (max, sum exp(x - max), first argmax | NaN flag, current logit)
    record of one contiguous vocabulary shard, as int32 [rows, 4]."""
    ids = _host(token_ids)
    lg = _host(logits_shard)
    rows = ids.numel()
    out = torch.empty((rows, 4), dtype=torch.int32)
    if rows:
        rc = lib().cid_oracle_shard_records(
            DT[lg.dtype], _p(lg), _p(ids), _i(rows), _i(lg.shape[-1]), _i(vocab_offset), _p(out)
        )
        _check(rc, "invalid shard")
    return out


def display_combine_records(records, token_ids, shard_offsets):
    """Merge [world, rows, 4] records into the unsharded statistics."""
    rec = _host(records)
    ids = _host(token_ids)
    offs = torch.tensor(list(shard_offsets), dtype=torch.int64)
    conf = torch.empty(ids.shape, dtype=torch.float32)
    cur = torch.empty(ids.shape, dtype=torch.float32)
    pred = torch.empty(ids.shape, dtype=torch.int64)
    if ids.numel():
        lib().cid_oracle_combine_records(
            _p(rec), ctypes.c_int(rec.shape[0]), _p(offs), _p(ids), _i(ids.numel()),
            _p(conf), _p(pred), _p(cur),
        )
    return conf, pred, cur


def batched_linear_assignment(costs, row_counts):
    """csrc/ops.cpp:68-175."""
    c = _host(costs)
    rc_ = _host(row_counts)
    b, r, m = c.shape
    out = torch.empty((b, r), dtype=torch.int64)
    rc = lib().cid_oracle_linear_assignment(
        DT[c.dtype], _p(c), _p(rc_), _i(b), _i(r), _i(m), _p(out)
    )
    _check(rc, "row_counts values must be in [0, rows]")
    return out
