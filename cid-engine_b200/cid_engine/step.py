"""One display-refinement decode step as a single device-resident launch chain.

The reference leaves the per-step sequencing to the external CID scheduler
(``benchmarks/README.md:29-43`` of fwerkor/cid-engine v1.1.0): statistics, the
refinement policy (a host round trip there), slot transition, live occupancy
and the materialisation snapshot.  ``refine_step`` enqueues the same chain of
operators on the current stream with no host synchronisation anywhere (four
kernels: statistics, refinement, slot rollout with live occupancy,
snapshot), so a caller can run many steps back to back or capture them in a
CUDA graph.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor


@dataclass
class SlotInputs:
    """Thought-slot inputs of one step (shapes as the reference operators)."""

    occupancy: Tensor  # [B, S] or [B, S, 1]
    allocation_logits: Tensor  # [B, S]
    lifecycle_logits: Tensor  # [B, S, F]
    revision_logits: Tensor  # [B, S, Rv]
    input_lifecycle: Tensor  # [B, S, F]
    semantic: Tensor  # [B, S, H]
    role_logits: Tensor  # [B, S, R]
    uncertainty: Tensor  # [B, S, 1]
    noise_delta: Tensor  # [B, S, 1]
    semantic_indices: Tensor  # [K] int64
    threshold: float = 0.5
    max_allocations: int = 8
    retired_index: int = 3


@dataclass
class StepOutputs:
    token_ids: Tensor  # refined display ids [B, L]
    confidence: Tensor
    predicted: Tensor
    current_confidence: Tensor
    next_occupancy: Tensor | None = None
    live_occupancy: Tensor | None = None
    snapshot: Tensor | None = None
    rollout: tuple[Tensor, ...] | None = None


def refine_step(
    token_ids: Tensor,
    logits: Tensor,
    *,
    mask_token_id: int,
    eos_token_id: int | None,
    reveal_fraction: float,
    revision_fraction: float,
    revision_margin: float,
    slots: SlotInputs | None = None,
) -> StepOutputs:
    """stats -> refine (-> rollout -> live occupancy -> snapshot), enqueued
    on the current stream without any host synchronisation."""
    conf, pred, cur = torch.ops.cid_engine.display_token_statistics(token_ids, logits)
    return step_from_statistics(token_ids, conf, pred, cur, mask_token_id=mask_token_id,
                                eos_token_id=eos_token_id, reveal_fraction=reveal_fraction,
                                revision_fraction=revision_fraction,
                                revision_margin=revision_margin, slots=slots)


def refine_step_from_hidden(
    token_ids: Tensor,
    hidden: Tensor,
    lm_head_weight: Tensor,
    *,
    mask_token_id: int,
    eos_token_id: int | None,
    reveal_fraction: float,
    revision_fraction: float,
    revision_margin: float,
    slots: SlotInputs | None = None,
    round_bf16: bool = True,
) -> StepOutputs:
    """The same step from the display positions' hidden states: the LM head
    and the statistics in one kernel (``lm_head_display_statistics``), so no
    ``[B, L, V]`` logits are written, then the chain of ``refine_step``."""
    conf, pred, cur = torch.ops.cid_engine.lm_head_display_statistics(
        token_ids, hidden, lm_head_weight, round_bf16)
    return step_from_statistics(token_ids, conf, pred, cur, mask_token_id=mask_token_id,
                                eos_token_id=eos_token_id, reveal_fraction=reveal_fraction,
                                revision_fraction=revision_fraction,
                                revision_margin=revision_margin, slots=slots)


def step_from_statistics(
    token_ids: Tensor,
    conf: Tensor,
    pred: Tensor,
    cur: Tensor,
    *,
    mask_token_id: int,
    eos_token_id: int | None,
    reveal_fraction: float,
    revision_fraction: float,
    revision_margin: float,
    slots: SlotInputs | None = None,
) -> StepOutputs:
    """refine (-> rollout -> live occupancy -> snapshot) from the step's
    display statistics."""
    ops = torch.ops.cid_engine
    refined = ops.refine_display_from_statistics(
        token_ids, conf, pred, cur, mask_token_id, eos_token_id,
        reveal_fraction, revision_fraction, revision_margin,
    )
    out = StepOutputs(refined, conf, pred, cur)
    if slots is None:
        return out
    # slot rollout and the live occupancy of its next state (retired slots
    # masked out) from one kernel
    *roll, live = ops.rollout_slot_transition_with_live(
        slots.occupancy, slots.allocation_logits, slots.lifecycle_logits,
        slots.revision_logits, slots.input_lifecycle, slots.threshold,
        slots.max_allocations, slots.retired_index,
    )
    roll = tuple(roll)
    next_occ = roll[0]
    live_slots = roll[5]
    snap = ops.materialize_cell_snapshot(
        slots.semantic, slots.role_logits, slots.uncertainty, slots.noise_delta,
        slots.lifecycle_logits, live_slots, slots.semantic_indices,
    )
    out.next_occupancy = next_occ
    out.live_occupancy = live
    out.snapshot = snap
    out.rollout = roll
    return out
