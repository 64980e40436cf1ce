"""Host logic without a GPU: schemas, validation messages, meta shapes and
the no-CPU-fallback rule."""

from __future__ import annotations

import pytest
import torch

import cid_engine

# The reference's operator ABI, csrc/registration.cpp:5-49 (fwerkor/cid-engine
# v1.1.0), as torch prints the registered schemas.
REFERENCE_SCHEMAS = {
    "live_slot_occupancy": "cid_engine::live_slot_occupancy(Tensor slot_occupancy, Tensor? lifecycle_features, int retired_index) -> Tensor",
    "prefix_allocation_mask": "cid_engine::prefix_allocation_mask(Tensor occupancy, Tensor allocation_logits, float threshold, int max_allocations) -> Tensor",
    "batched_linear_assignment": "cid_engine::batched_linear_assignment(Tensor costs, Tensor row_counts) -> Tensor",
    "rollout_slot_transition": "cid_engine::rollout_slot_transition(Tensor occupancy, Tensor allocation_logits, Tensor lifecycle_logits, Tensor revision_logits, Tensor input_lifecycle, float threshold, int max_allocations, int retired_index) -> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)",
    "thought_corrupt_from_epsilon": "cid_engine::thought_corrupt_from_epsilon(Tensor semantic, Tensor timesteps, Tensor occupancy, Tensor epsilon) -> (Tensor, Tensor, Tensor)",
    "display_corrupt_from_random": "cid_engine::display_corrupt_from_random(Tensor token_ids, Tensor timesteps, Tensor eligible_mask, Tensor corruption_random, Tensor? replacement_random, Tensor? replacement_offsets, int mask_token_id, int? eos_token_id, int vocab_size, float replacement_fraction) -> (Tensor, Tensor, Tensor, Tensor)",
    "masked_diffusion_corrupt_from_random": "cid_engine::masked_diffusion_corrupt_from_random(Tensor clean_ids, Tensor ratio_random, Tensor mask_random, int mask_token_id, float min_mask_ratio, float max_mask_ratio) -> (Tensor, Tensor, Tensor, Tensor)",
    "display_token_statistics": "cid_engine::display_token_statistics(Tensor token_ids, Tensor logits) -> (Tensor, Tensor, Tensor)",
    "display_token_statistics_with_repetition": "cid_engine::display_token_statistics_with_repetition(Tensor token_ids, Tensor logits, int mask_token_id, int? eos_token_id, float repetition_score_multiplier) -> (Tensor, Tensor, Tensor)",
    "refine_display_from_statistics": "cid_engine::refine_display_from_statistics(Tensor token_ids, Tensor confidence, Tensor predicted, Tensor current_confidence, int mask_token_id, int? eos_token_id, float reveal_fraction, float revision_fraction, float revision_margin) -> Tensor",
    "materialize_cell_snapshot": "cid_engine::materialize_cell_snapshot(Tensor thought_semantic, Tensor role_logits, Tensor uncertainty, Tensor noise_delta, Tensor lifecycle_logits, Tensor selected, Tensor semantic_indices) -> Tensor",
}


@pytest.mark.parametrize("name", sorted(REFERENCE_SCHEMAS))
def test_schema_is_the_reference_schema(name: str) -> None:
    assert str(getattr(torch.ops.cid_engine, name).default._schema) == REFERENCE_SCHEMAS[name]


def test_backend_build_flags_are_boolean() -> None:
    assert cid_engine.CUDA_BACKEND_BUILT is True
    assert cid_engine.ROCM_BACKEND_BUILT is False
    assert cid_engine.CANN_BACKEND_BUILT is False


def test_cpu_tensors_are_rejected_after_validation() -> None:
    ids = torch.zeros(2, 3, dtype=torch.long)
    lg = torch.randn(2, 3, 11)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        cid_engine.display_token_statistics(ids, lg)


def test_non_int64_display_ids_are_rejected() -> None:
    # reference tests/test_engine.py:304-313
    with pytest.raises(RuntimeError, match="torch.int64"):
        cid_engine.display_token_statistics(torch.tensor([[0, 1]], dtype=torch.int32),
                                            torch.zeros(1, 2, 3))


def test_snapshot_rejects_non_bool_selection() -> None:
    # reference tests/test_engine.py:486-504
    with pytest.raises(RuntimeError, match="selected must use torch.bool"):
        cid_engine.materialize_cell_snapshot(
            torch.randn(1, 2, 4), torch.randn(1, 2, 3), torch.rand(1, 2, 1),
            torch.randn(1, 2, 1), torch.randn(1, 2, 4), torch.ones(1, 2),
            torch.tensor([0, 3]))


def test_snapshot_rejects_host_indices_outside_width() -> None:
    with pytest.raises(RuntimeError, match="outside semantic width"):
        cid_engine.materialize_cell_snapshot(
            torch.randn(1, 2, 4), torch.randn(1, 2, 3), torch.rand(1, 2, 1),
            torch.randn(1, 2, 1), torch.randn(1, 2, 4), torch.ones(1, 2, dtype=torch.bool),
            torch.tensor([0, 4]))


@pytest.mark.parametrize("threshold", [-1e-9, 1.000000001, float("nan")])
def test_invalid_allocation_threshold_is_rejected(threshold: float) -> None:
    # reference tests/test_fuzz.py:330-351
    with pytest.raises(RuntimeError, match="threshold"):
        cid_engine.prefix_allocation_mask(torch.zeros(1, 4), torch.zeros(1, 4),
                                          threshold=threshold, max_allocations=2)


@pytest.mark.parametrize(
    "kwargs,match",
    [
        (dict(reveal_fraction=1.5, revision_fraction=0.1, revision_margin=0.0), "reveal_fraction"),
        (dict(reveal_fraction=0.5, revision_fraction=-0.1, revision_margin=0.0), "revision_fraction"),
        (dict(reveal_fraction=0.5, revision_fraction=0.1, revision_margin=-1.0), "revision_margin"),
    ],
)
def test_refine_validation(kwargs, match) -> None:
    ids = torch.zeros(1, 4, dtype=torch.long)
    with pytest.raises(RuntimeError, match=match):
        cid_engine.refine_display_from_statistics(
            ids, torch.zeros(1, 4), ids, torch.zeros(1, 4), mask_token_id=0, eos_token_id=None,
            **kwargs)


def test_masked_diffusion_validation() -> None:
    with pytest.raises(RuntimeError, match="0 < min <= max <= 1"):
        cid_engine.masked_diffusion_corrupt_from_random(
            torch.zeros(2, 4, dtype=torch.long), torch.zeros(2, 1), torch.zeros(2, 4),
            mask_token_id=9, min_mask_ratio=0.0, max_mask_ratio=1.0)
    with pytest.raises(RuntimeError, match="non-empty"):
        cid_engine.masked_diffusion_corrupt_from_random(
            torch.zeros(0, 4, dtype=torch.long), torch.zeros(0, 1), torch.zeros(0, 4),
            mask_token_id=9, min_mask_ratio=0.1, max_mask_ratio=1.0)


def test_repetition_multiplier_validation() -> None:
    with pytest.raises(RuntimeError, match=r"\(0, 1\]"):
        cid_engine.display_token_statistics_with_repetition(
            torch.zeros(1, 3, dtype=torch.long), torch.zeros(1, 3, 8), mask_token_id=0,
            eos_token_id=None, repetition_score_multiplier=1.5)


def _meta(*ts):
    return [t.to("meta") if isinstance(t, torch.Tensor) else t for t in ts]


def test_meta_shapes() -> None:
    ops = torch.ops.cid_engine
    ids = torch.zeros(3, 5, dtype=torch.long)
    c, p, u = ops.display_token_statistics(*_meta(ids, torch.zeros(3, 5, 7)))
    assert c.shape == (3, 5) and c.dtype == torch.float32 and p.dtype == torch.int64
    out = ops.refine_display_from_statistics(*_meta(ids, c, p, u), 0, 1, 0.5, 0.1, 0.0)
    assert out.shape == (3, 5) and out.dtype == torch.int64
    m = ops.prefix_allocation_mask(*_meta(torch.zeros(3, 9, 1), torch.zeros(3, 9)), 0.5, 2)
    assert m.shape == (3, 9) and m.dtype == torch.bool
    r = ops.rollout_slot_transition(*_meta(torch.zeros(3, 9), torch.zeros(3, 9),
                                           torch.zeros(3, 9, 4), torch.zeros(3, 9, 3),
                                           torch.zeros(3, 9, 4)), 0.5, 2, 3)
    assert [t.dtype for t in r] == [torch.bool, torch.int64, torch.int64, torch.int64,
                                    torch.bool, torch.bool]
    s = ops.materialize_cell_snapshot(*_meta(torch.zeros(2, 4, 16), torch.zeros(2, 4, 6),
                                             torch.zeros(2, 4, 1), torch.zeros(2, 4, 1),
                                             torch.zeros(2, 4, 4),
                                             torch.zeros(2, 4, dtype=torch.bool),
                                             torch.zeros(12, dtype=torch.long)))
    assert s.shape == (2, 4, 4 + 6 + 12) and s.dtype == torch.float32
    md = ops.masked_diffusion_corrupt_from_random(
        *_meta(torch.zeros(4, 8, dtype=torch.long), torch.zeros(4, 1), torch.zeros(4, 8)),
        9, 0.1, 1.0)
    assert [tuple(t.shape) for t in md] == [(4, 8), (4, 8), (4, 1), (2,)]
    th = ops.thought_corrupt_from_epsilon(*_meta(torch.zeros(2, 3, 5, dtype=torch.bfloat16),
                                                 torch.zeros(2, 3), torch.zeros(2, 3, 1),
                                                 torch.zeros(2, 3, 5, dtype=torch.bfloat16)))
    assert th[0].dtype == torch.bfloat16 and th[1].shape == (2, 3, 1)
    rec = ops.display_shard_records(*_meta(ids, torch.zeros(3, 5, 7)), 7, 21)
    assert rec.shape == (15, 4) and rec.dtype == torch.int32
    hid = torch.zeros(3, 5, 64, dtype=torch.bfloat16)
    wgt = torch.zeros(100, 64, dtype=torch.bfloat16)
    lc, lp, lu = ops.lm_head_display_statistics(*_meta(ids, hid, wgt))
    assert lc.shape == (3, 5) and lp.dtype == torch.int64 and lu.dtype == torch.float32
    lr = ops.lm_head_shard_records(*_meta(ids, hid, wgt), 50, 150)
    assert lr.shape == (15, 4) and lr.dtype == torch.int32


def test_lm_head_validation_on_host() -> None:
    ops = torch.ops.cid_engine
    ids = torch.zeros(3, 5, dtype=torch.long)
    hid = torch.zeros(3, 5, 64, dtype=torch.bfloat16)
    wgt = torch.zeros(100, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.lm_head_display_statistics(ids, hid, wgt)
    with pytest.raises(RuntimeError, match="bfloat16"):
        ops.lm_head_display_statistics(ids, hid.float(), wgt)
    with pytest.raises(RuntimeError, match="inside"):
        ops.lm_head_shard_records(ids, hid, wgt, 60, 150)
