"""The graph-replayed decode loop (``cid_engine.loop.DisplayRefineLoop``).

Checks that replaying the captured chain gives bit-identical state and
snapshots to issuing the operators eagerly step by step, that every stage of
every step matches the oracle applied to that step's inputs, that a captured
logits producer sees the current ids, and the host-ring bookkeeping.
"""

from __future__ import annotations

import pytest
import torch

import compare
from oracle import oracle

pytestmark = pytest.mark.gpu

MASK, EOS = 0, 1
PARAMS = dict(mask_token_id=MASK, eos_token_id=EOS, reveal_fraction=0.25,
              revision_fraction=0.1, revision_margin=0.05)


@pytest.fixture(scope="module", autouse=True)
def _engine():
    import cid_engine  # noqa: F401

    assert torch.cuda.is_available()
    yield
    torch.cuda.empty_cache()


def _inputs(B=4, L=96, V=1000, S=16, ring=3, seed=11, dtype=torch.bfloat16):
    from cid_engine.step import SlotInputs

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(seed)
    logits = [(torch.randn(B, L, V, generator=g) * 3).to(dtype).to(dev) for _ in range(ring)]
    ids = torch.randint(2, V, (B, L), generator=g)
    ids[torch.rand(B, L, generator=g) < 0.6] = MASK
    ids[:, L - 5] = EOS
    ids[:, L - 4:] = MASK
    slots = SlotInputs(
        occupancy=(torch.rand(B, S, 1, generator=g) < 0.4).float().to(dev),
        allocation_logits=torch.randn(B, S, generator=g).to(dev),
        lifecycle_logits=torch.randn(B, S, 4, generator=g).to(dev),
        revision_logits=torch.randn(B, S, 3, generator=g).to(dev),
        input_lifecycle=torch.randn(B, S, 4, generator=g).to(dev),
        semantic=torch.randn(B, S, 64, generator=g).to(dev),
        role_logits=torch.randn(B, S, 6, generator=g).to(dev),
        uncertainty=torch.rand(B, S, 1, generator=g).to(dev),
        noise_delta=torch.randn(B, S, 1, generator=g).to(dev),
        semantic_indices=torch.randint(0, 64, (12,), generator=g).to(dev),
        threshold=0.5, max_allocations=3, retired_index=3,
    )
    return ids.to(dev), logits, slots


def _eager_chain(ids, logits, slots, steps):
    """The same steps issued operator by operator."""
    import dataclasses

    from cid_engine.step import refine_step

    occ = slots.occupancy.reshape(slots.allocation_logits.shape) != 0
    states, snaps = [], []
    for s in range(steps):
        out = refine_step(ids, logits[s % len(logits)], slots=dataclasses.replace(slots, occupancy=occ),
                          **PARAMS)
        ids, occ = out.token_ids, out.next_occupancy
        states.append((ids.cpu(), occ.cpu()))
        snaps.append(out.snapshot.cpu())
    return states, snaps


@pytest.mark.parametrize("use_graphs", [True, False])
def test_loop_matches_eager_chain(use_graphs) -> None:
    from cid_engine.loop import DisplayRefineLoop

    ids, logits, slots = _inputs()
    steps = 9
    states, snaps = _eager_chain(ids, logits, slots, steps)
    loop = DisplayRefineLoop(ids, logits, slots=slots, host_snapshots=3, use_graphs=use_graphs,
                             **PARAMS)
    assert loop.period == 6  # lcm(ring 3, 2 snapshot buffers)
    got = []
    loop.run(steps, on_snapshot=lambda s, h: got.append((s, h.clone())))
    torch.cuda.synchronize()
    assert [s for s, _ in got] == list(range(steps))
    for s, h in got:
        assert torch.equal(h, snaps[s]), f"snapshot of step {s}"
    assert torch.equal(loop.token_ids.cpu(), states[-1][0])
    assert torch.equal(loop.occupancy.cpu(), states[-1][1])
    # inputs untouched
    assert torch.equal(loop.logits[0], logits[0])
    loop.close()


def test_loop_stages_match_oracle() -> None:
    """Every stage of every step against the oracle on that step's inputs."""
    from cid_engine.loop import DisplayRefineLoop

    ids, logits, slots = _inputs(B=3, L=80, V=700, S=12, seed=5)
    loop = DisplayRefineLoop(ids, logits, slots=slots, host_snapshots=2, **PARAMS)
    ids_prev = ids.cpu()
    occ_prev = (slots.occupancy.reshape(3, 12) != 0).cpu()
    for s in range(5):
        loop.step()
        torch.cuda.synchronize()
        out = loop.last_outputs
        lg = logits[s % len(logits)].cpu()
        stats = oracle.display_token_statistics(ids_prev, lg)
        compare.assert_matches("display_token_statistics",
                               (out.confidence, out.predicted, out.current_confidence), stats,
                               f"step {s} stats")
        # the policy on the device's own statistics is exact
        exp_ids = oracle.refine_display_from_statistics(
            ids_prev, out.confidence.cpu(), out.predicted.cpu(), out.current_confidence.cpu(),
            MASK, EOS, 0.25, 0.1, 0.05)
        assert torch.equal(out.token_ids.cpu(), exp_ids), f"step {s} refine"
        roll = oracle.rollout_slot_transition(
            occ_prev, slots.allocation_logits, slots.lifecycle_logits, slots.revision_logits,
            slots.input_lifecycle, slots.threshold, slots.max_allocations, slots.retired_index)
        if not bool(compare.sigmoid_ambiguous(slots.allocation_logits, slots.threshold).any()):
            for a, e in zip(out.rollout, roll):
                assert torch.equal(a.cpu(), e), f"step {s} rollout"
        live = oracle.live_slot_occupancy(out.next_occupancy.cpu().unsqueeze(-1).float(),
                                          slots.lifecycle_logits, slots.retired_index)
        assert torch.equal(out.live_occupancy.cpu(), live), f"step {s} live"
        snap = oracle.materialize_cell_snapshot(
            slots.semantic, slots.role_logits, slots.uncertainty, slots.noise_delta,
            slots.lifecycle_logits, out.rollout[5].cpu(), slots.semantic_indices)
        compare.assert_matches("materialize_cell_snapshot", out.snapshot, snap, f"step {s} snapshot")
        assert torch.equal(loop.snapshot(s), out.snapshot.cpu())
        ids_prev = loop.token_ids.cpu()
        occ_prev = loop.occupancy.cpu()
        assert torch.equal(ids_prev, exp_ids)
    with pytest.raises(IndexError):
        loop.snapshot(0)  # overwritten: the host ring holds two steps
    loop.close()


def test_loop_captured_producer_sees_current_ids() -> None:
    """A producer captured in the graph computes logits from the ids of the
    step it feeds: here a bias that favours each position's current id."""
    from cid_engine.loop import DisplayRefineLoop

    ids, base, slots = _inputs(B=2, L=64, V=512, S=8, ring=2, seed=9)

    def producer(k, cur_ids, out):
        out.copy_(base[k])
        out.scatter_add_(-1, cur_ids.unsqueeze(-1),
                         torch.full(cur_ids.shape + (1,), 4.0, device=out.device, dtype=out.dtype))

    bufs = [torch.empty_like(b) for b in base]
    loop = DisplayRefineLoop(ids, bufs, slots=slots, producer=producer, **PARAMS)
    ref = DisplayRefineLoop(ids, [torch.empty_like(b) for b in base], slots=slots,
                            producer=producer, use_graphs=False, **PARAMS)
    for _ in range(7):
        loop.step()
        ref.step()
    torch.cuda.synchronize()
    assert torch.equal(loop.token_ids, ref.token_ids)
    assert torch.equal(loop.occupancy, ref.occupancy)
    loop.close()
    ref.close()


def test_loop_reset_and_display_only() -> None:
    """Without slots the loop refines display ids only; reset restarts it."""
    from cid_engine.loop import DisplayRefineLoop
    from cid_engine.step import refine_step

    ids, logits, _ = _inputs(B=2, L=48, V=300, seed=3)
    loop = DisplayRefineLoop(ids, logits, **PARAMS)
    assert loop.period == 3 and loop.occupancy is None
    first = loop.run(4).clone()
    loop.reset(ids)
    again = loop.run(4)
    assert torch.equal(first, again)
    cur = ids
    for s in range(4):
        cur = refine_step(cur, logits[s % 3], **PARAMS).token_ids
    assert torch.equal(cur, again)
    with pytest.raises(RuntimeError):
        loop.snapshot(0)
    loop.close()


def test_loop_from_hidden_states_matches_eager() -> None:
    """The loop over hidden-state buffers (LM head fused with the statistics)
    equals the eager chain of refine_step_from_hidden, and each step's
    statistics are the fused LM head's."""
    import dataclasses

    import cid_engine
    from cid_engine.loop import DisplayRefineLoop
    from cid_engine.step import refine_step_from_hidden

    ids, _, slots = _inputs(B=3, L=64, V=512, S=8, ring=2, seed=21)
    dev = ids.device
    g = torch.Generator(device=dev).manual_seed(3)
    H, V = 64, 3000
    hidden = [(torch.randn(3, 64, H, generator=g, device=dev) * 0.5).to(torch.bfloat16)
              for _ in range(2)]
    weight = (torch.randn(V, H, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    ids = ids.clamp(max=V - 1)
    loop = DisplayRefineLoop(ids, hidden, slots=slots, lm_head_weight=weight, **PARAMS)
    occ = slots.occupancy.reshape(3, 8) != 0
    cur = ids
    for s in range(5):
        loop.step()
        out = refine_step_from_hidden(cur, hidden[s % 2], weight,
                                      slots=dataclasses.replace(slots, occupancy=occ), **PARAMS)
        torch.cuda.synchronize()
        c, p, u = cid_engine.lm_head_display_statistics(cur, hidden[s % 2], weight)
        assert torch.equal(out.predicted, p) and torch.equal(out.confidence, c)
        assert torch.equal(loop.last_outputs.token_ids, out.token_ids), f"step {s}"
        assert torch.equal(loop.last_outputs.snapshot, out.snapshot)
        cur, occ = out.token_ids, out.next_occupancy
    loop.close()
