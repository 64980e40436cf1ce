"""cid-engine, B200 (sm_100a) build of the display-refinement path.

Drop-in for the reference package's operator API (fwerkor/cid-engine v1.1.0,
``src/cid_engine/__init__.py:41-225``): the same keyword-only wrappers over the
same ``torch.ops.cid_engine`` operators with byte-identical schemas.  Here the
operators are registered on the CUDA dispatch key by the C++20 host in
``_C`` and run as hand-written sm_100a kernels behind the C ABI of
``libcid_engine_b200.so``.  There is no CPU backend: CPU tensors are
validated and then rejected with a clear error, and importing this package
fails loudly when the native library is missing.

Added here (no reference counterpart): vocabulary-parallel statistics
(``display_shard_records`` / ``display_combine_records`` and
``cid_engine.parallel``), the fused decode step ``refine_step`` and the device
status word (``device_status``).
"""

from __future__ import annotations

import torch
from torch import Tensor

from cid_engine import _C  # noqa: F401  (registers torch.ops.cid_engine)

__version__ = "1.1.0+b200"
CUDA_BACKEND_BUILT = bool(_C.cuda_backend_built)
ROCM_BACKEND_BUILT = bool(_C.rocm_backend_built)
CANN_BACKEND_BUILT = bool(_C.cann_backend_built)

# Bits of the device status word (include/cid_engine_b200.h).
STATUS_TOKEN_ID_OUT_OF_RANGE = 0x1
STATUS_SEMANTIC_INDEX_OUT_OF_RANGE = 0x2
STATUS_REPETITION_ID_OUT_OF_RANGE = 0x4
STATUS_ASSIGNMENT_INVALID = 0x8
STATUS_LM_HEAD_TIMEOUT = 0x10
STATUS_PEER_TIMEOUT = 0x20
STATUS_PEER_OUT_OF_STEP = 0x40


def device_status(device: int | torch.device = 0, *, reset: bool = False) -> int:
    """Status bits raised by the kernels on ``device`` since the last reset.

    Conditions the reference CPU backend raises on (out-of-range token ids,
    snapshot indices outside the semantic width) cannot raise from a device
    kernel without a host sync; the kernels write NaN for the affected
    outputs and set a bit here instead.  Reading synchronises the device.
    """
    index = torch.device(device).index if not isinstance(device, int) else device
    return int(_C.device_status(index or 0, reset))


def live_slot_occupancy(
    slot_occupancy: Tensor,
    lifecycle_features: Tensor | None,
    *,
    retired_index: int,
) -> Tensor:
    return torch.ops.cid_engine.live_slot_occupancy(
        slot_occupancy,
        lifecycle_features,
        retired_index,
    )


def prefix_allocation_mask(
    occupancy: Tensor,
    allocation_logits: Tensor,
    *,
    threshold: float,
    max_allocations: int,
) -> Tensor:
    return torch.ops.cid_engine.prefix_allocation_mask(
        occupancy,
        allocation_logits,
        threshold,
        max_allocations,
    )


def thought_corrupt_from_epsilon(
    semantic: Tensor,
    timesteps: Tensor,
    occupancy: Tensor,
    epsilon: Tensor,
) -> tuple[Tensor, Tensor, Tensor]:
    return torch.ops.cid_engine.thought_corrupt_from_epsilon(
        semantic,
        timesteps,
        occupancy,
        epsilon,
    )


def display_corrupt_from_random(
    token_ids: Tensor,
    timesteps: Tensor,
    eligible_mask: Tensor,
    corruption_random: Tensor,
    replacement_random: Tensor | None,
    replacement_offsets: Tensor | None,
    *,
    mask_token_id: int,
    eos_token_id: int | None,
    vocab_size: int,
    replacement_fraction: float,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    return torch.ops.cid_engine.display_corrupt_from_random(
        token_ids,
        timesteps,
        eligible_mask,
        corruption_random,
        replacement_random,
        replacement_offsets,
        mask_token_id,
        eos_token_id,
        vocab_size,
        replacement_fraction,
    )


def masked_diffusion_corrupt_from_random(
    clean_ids: Tensor,
    ratio_random: Tensor,
    mask_random: Tensor,
    *,
    mask_token_id: int,
    min_mask_ratio: float,
    max_mask_ratio: float,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    return torch.ops.cid_engine.masked_diffusion_corrupt_from_random(
        clean_ids,
        ratio_random,
        mask_random,
        mask_token_id,
        min_mask_ratio,
        max_mask_ratio,
    )


def display_token_statistics(
    token_ids: Tensor,
    logits: Tensor,
) -> tuple[Tensor, Tensor, Tensor]:
    return torch.ops.cid_engine.display_token_statistics(token_ids, logits)


def display_token_statistics_with_repetition(
    token_ids: Tensor,
    logits: Tensor,
    *,
    mask_token_id: int,
    eos_token_id: int | None,
    repetition_score_multiplier: float = 0.7,
) -> tuple[Tensor, Tensor, Tensor]:
    return torch.ops.cid_engine.display_token_statistics_with_repetition(
        token_ids,
        logits,
        mask_token_id,
        eos_token_id,
        repetition_score_multiplier,
    )


def batched_linear_assignment(
    costs: Tensor,
    row_counts: Tensor,
) -> Tensor:
    return torch.ops.cid_engine.batched_linear_assignment(costs, row_counts)


def rollout_slot_transition(
    occupancy: Tensor,
    allocation_logits: Tensor,
    lifecycle_logits: Tensor,
    revision_logits: Tensor,
    input_lifecycle: Tensor,
    *,
    threshold: float,
    max_allocations: int,
    retired_index: int,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    return torch.ops.cid_engine.rollout_slot_transition(
        occupancy,
        allocation_logits,
        lifecycle_logits,
        revision_logits,
        input_lifecycle,
        threshold,
        max_allocations,
        retired_index,
    )


def rollout_slot_transition_with_live(
    occupancy: Tensor,
    allocation_logits: Tensor,
    lifecycle_logits: Tensor,
    revision_logits: Tensor,
    input_lifecycle: Tensor,
    *,
    threshold: float,
    max_allocations: int,
    retired_index: int,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """``rollout_slot_transition`` and, from the same kernel, the live
    occupancy of its next state: ``live_slot_occupancy(next_occupancy
    .unsqueeze(-1).to(lifecycle_logits.dtype), lifecycle_logits,
    retired_index)`` as a seventh output ([B, S, 1], lifecycle dtype)."""
    return torch.ops.cid_engine.rollout_slot_transition_with_live(
        occupancy,
        allocation_logits,
        lifecycle_logits,
        revision_logits,
        input_lifecycle,
        threshold,
        max_allocations,
        retired_index,
    )


def materialize_cell_snapshot(
    thought_semantic: Tensor,
    role_logits: Tensor,
    uncertainty: Tensor,
    noise_delta: Tensor,
    lifecycle_logits: Tensor,
    selected: Tensor,
    semantic_indices: Tensor,
) -> Tensor:
    return torch.ops.cid_engine.materialize_cell_snapshot(
        thought_semantic,
        role_logits,
        uncertainty,
        noise_delta,
        lifecycle_logits,
        selected,
        semantic_indices,
    )


def refine_display_from_statistics(
    token_ids: Tensor,
    confidence: Tensor,
    predicted: Tensor,
    current_confidence: Tensor,
    *,
    mask_token_id: int,
    eos_token_id: int | None,
    reveal_fraction: float,
    revision_fraction: float,
    revision_margin: float,
) -> Tensor:
    return torch.ops.cid_engine.refine_display_from_statistics(
        token_ids,
        confidence,
        predicted,
        current_confidence,
        mask_token_id,
        eos_token_id,
        reveal_fraction,
        revision_fraction,
        revision_margin,
    )


def display_shard_records(
    token_ids: Tensor,
    logits_shard: Tensor,
    *,
    vocab_offset: int,
    total_vocab: int,
) -> Tensor:
    """Per-row ``(max, sum exp(x - max), first argmax, current logit)`` record
    of one contiguous vocabulary shard, as an int32 ``[rows, 4]`` tensor (16
    bytes per row; see ``cid_shard_record_t``)."""
    return torch.ops.cid_engine.display_shard_records(
        token_ids, logits_shard, vocab_offset, total_vocab
    )


def display_combine_records(
    records: Tensor,
    token_ids: Tensor,
    shard_offsets: list[int],
) -> tuple[Tensor, Tensor, Tensor]:
    """Merge ``[world, rows, 4]`` shard records (rank order, ascending
    contiguous column ranges ``shard_offsets``) into the unsharded
    ``display_token_statistics`` outputs."""
    return torch.ops.cid_engine.display_combine_records(records, token_ids, list(shard_offsets))



def lm_head_display_statistics(
    token_ids: Tensor,
    hidden: Tensor,
    weight: Tensor,
    *,
    round_bf16: bool = True,
) -> tuple[Tensor, Tensor, Tensor]:
    """``display_token_statistics(token_ids, hidden @ weight.T)`` without
    writing the ``[*, vocab]`` logits: bf16 ``hidden [*token_ids.shape, H]``
    and ``weight [vocab, H]`` (H % 8 == 0) multiplied on the tcgen05 tensor
    cores with f32 accumulation, each logit rounded to bf16 first when
    ``round_bf16`` (the statistics of a bf16 LM head's stored output)."""
    return torch.ops.cid_engine.lm_head_display_statistics(token_ids, hidden, weight, round_bf16)



def lm_head_shard_records(
    token_ids: Tensor,
    hidden: Tensor,
    weight_shard: Tensor,
    *,
    vocab_offset: int,
    total_vocab: int,
    round_bf16: bool = True,
) -> Tensor:
    """The per-rank half of a vocabulary-parallel LM head: the 16-byte shard
    record of every row (as ``display_shard_records``) over
    ``hidden @ weight_shard.T``, whose columns are the global vocabulary ids
    ``[vocab_offset, vocab_offset + weight_shard.shape[0])``, without writing
    those logits."""
    return torch.ops.cid_engine.lm_head_shard_records(token_ids, hidden, weight_shard,
                                                      vocab_offset, total_vocab, round_bf16)


from cid_engine.step import refine_step, refine_step_from_hidden  # noqa: E402
from cid_engine.loop import DisplayRefineLoop  # noqa: E402

__all__ = [
    "CANN_BACKEND_BUILT",
    "CUDA_BACKEND_BUILT",
    "DisplayRefineLoop",
    "ROCM_BACKEND_BUILT",
    "batched_linear_assignment",
    "device_status",
    "display_combine_records",
    "display_corrupt_from_random",
    "display_shard_records",
    "display_token_statistics",
    "display_token_statistics_with_repetition",
    "live_slot_occupancy",
    "lm_head_display_statistics",
    "lm_head_shard_records",
    "materialize_cell_snapshot",
    "masked_diffusion_corrupt_from_random",
    "prefix_allocation_mask",
    "refine_display_from_statistics",
    "refine_step",
    "refine_step_from_hidden",
    "rollout_slot_transition",
    "rollout_slot_transition_with_live",
    "thought_corrupt_from_epsilon",
]
