"""Property-based differential fuzzing of the CUDA path against the oracle.

The generators follow the reference's fuzz suite (tests/test_fuzz.py of
fwerkor/cid-engine v1.1.0): random shapes including empty ones, all logit
dtypes, scales from 0 to 100, strided views, random fractions/margins and EOS
layouts for the refinement policy, structural insert/delete proposals.  The
budget is ``CID_ENGINE_FUZZ_EXAMPLES`` (default 60 per test).
"""

from __future__ import annotations

import os

import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

import cases
import compare
from oracle import oracle

pytestmark = [pytest.mark.gpu, pytest.mark.fuzz]

EXAMPLES = int(os.environ.get("CID_ENGINE_FUZZ_EXAMPLES", "60"))
SETTINGS = settings(max_examples=EXAMPLES, deadline=None, print_blob=True, derandomize=True,
                    suppress_health_check=[HealthCheck.too_slow])
DTYPES = st.sampled_from([torch.float16, torch.bfloat16, torch.float32, torch.float64])
SCALES = st.sampled_from([0.0, 1.0e-4, 0.1, 1.0, 20.0, 100.0])
UNIT = st.one_of(st.sampled_from([0.0, 1.0, 0.5, 1.0e-7, 1.0 - 1.0e-7]),
                 st.floats(min_value=0.0, max_value=1.0, allow_nan=False))


@pytest.fixture(scope="module", autouse=True)
def _engine():
    import cid_engine  # noqa: F401

    assert torch.cuda.is_available()


def _cuda(t: torch.Tensor) -> torch.Tensor:
    if t.is_contiguous():
        return t.cuda()
    out = torch.empty_strided(t.size(), t.stride(), dtype=t.dtype, device="cuda")
    out.copy_(t)
    return out


@SETTINGS
@given(batch=st.integers(0, 4), tokens=st.integers(0, 40), vocab=st.integers(1, 3000),
       seed=st.integers(0, 2**31 - 1), dtype=DTYPES, scale=SCALES, strided=st.booleans())
def test_fuzz_display_statistics(batch, tokens, vocab, seed, dtype, scale, strided) -> None:
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(vocab, (batch, tokens), generator=g)
    lg = (torch.randn(batch, tokens, vocab, generator=g) * scale).to(dtype)
    if strided:
        lg = cases._strided_last_dim(lg)
    out = torch.ops.cid_engine.display_token_statistics(ids.cuda(), _cuda(lg))
    compare.assert_matches("display_token_statistics", out,
                           oracle.display_token_statistics(ids, lg), "fuzz stats")


@SETTINGS
@given(batch=st.integers(1, 3), tokens=st.integers(2, 70), vocab=st.integers(4, 300),
       seed=st.integers(0, 2**31 - 1), dtype=DTYPES, mult=st.floats(0.05, 1.0),
       with_eos=st.booleans())
def test_fuzz_repetition(batch, tokens, vocab, seed, dtype, mult, with_eos) -> None:
    g = torch.Generator().manual_seed(seed)
    alphabet = torch.tensor([0, 1, 2, 3, vocab - 1])
    ids = alphabet[torch.randint(len(alphabet), (batch, tokens), generator=g)]
    lg = (torch.randn(batch, tokens, vocab, generator=g) * 3).to(dtype)
    eos = 1 if with_eos else None
    out = torch.ops.cid_engine.display_token_statistics_with_repetition(ids.cuda(), lg.cuda(), 0,
                                                                        eos, mult)
    compare.assert_matches("display_token_statistics_with_repetition", out,
                           oracle.display_token_statistics_with_repetition(ids, lg, 0, eos, mult),
                           "fuzz repetition")


@SETTINGS
@given(seed=st.integers(0, 2**31 - 1), reveal=UNIT, revision=UNIT,
       margin=st.one_of(st.sampled_from([0.0, 1.0e-7, 0.01, 0.1, 1.0]),
                        st.floats(0.0, 1.0, allow_nan=False)),
       tokens=st.integers(1, 600), batch=st.integers(1, 6), with_eos=st.booleans())
def test_fuzz_refinement(seed, reveal, revision, margin, tokens, batch, with_eos) -> None:
    ids, (conf, pred, cur) = cases.refine_inputs_large(seed, batch, tokens)
    eos = 1 if with_eos else None
    got = torch.ops.cid_engine.refine_display_from_statistics(
        ids.cuda(), conf.cuda(), pred.cuda(), cur.cuda(), 0, eos, reveal, revision, margin)
    exp = oracle.refine_display_from_statistics(ids, conf, pred, cur, 0, eos, reveal, revision,
                                                margin)
    assert torch.equal(got.cpu(), exp)


@pytest.mark.parametrize("tokens", [1, 31, 32, 33, 127, 128, 129, 160, 5535, 5536])
@pytest.mark.parametrize("with_eos", [False, True])
def test_refinement_at_the_kernel_limits(tokens, with_eos) -> None:
    """Rows of up to 128 positions are refined by one warp each, longer rows by
    a CTA each, staged in shared memory up to 5535 positions (37 bytes a
    position) and read from global memory beyond: both sides of each limit,
    with structural-heavy rows (shifted predictions), many rows per launch,
    against the oracle."""
    ids, (conf, pred, cur) = cases.refine_inputs_large(tokens, 37 if tokens < 1000 else 3, tokens,
                                                       structural=0.5)
    eos = 1 if with_eos else None
    for reveal, revision, margin in ((0.25, 0.1, 0.05), (1.0, 1.0, 0.0), (0.5, 0.0, 0.1)):
        got = torch.ops.cid_engine.refine_display_from_statistics(
            ids.cuda(), conf.cuda(), pred.cuda(), cur.cuda(), 0, eos, reveal, revision, margin)
        exp = oracle.refine_display_from_statistics(ids, conf, pred, cur, 0, eos, reveal,
                                                    revision, margin)
        assert torch.equal(got.cpu(), exp)


@SETTINGS
@given(seed=st.integers(0, 2**31 - 1), mode=st.sampled_from(["insert", "delete"]))
def test_fuzz_structural_refinement(seed, mode) -> None:
    ids, (conf, pred, cur) = cases.refine_inputs_structural(seed, mode)
    got = torch.ops.cid_engine.refine_display_from_statistics(
        ids.cuda(), conf.cuda(), pred.cuda(), cur.cuda(), 0, 1, 1.0, 1.0, 0.1)
    assert torch.equal(got.cpu(), oracle.refine_display_from_statistics(ids, conf, pred, cur, 0,
                                                                        1, 1.0, 1.0, 0.1))


@SETTINGS
@given(batch=st.integers(0, 6), slots=st.integers(0, 200), seed=st.integers(0, 2**31 - 1),
       threshold=UNIT, max_extra=st.integers(1, 8), scale=SCALES, rank3=st.booleans(),
       strided=st.booleans(), dtype=DTYPES)
def test_fuzz_prefix_allocation(batch, slots, seed, threshold, max_extra, scale, rank3, strided,
                                dtype) -> None:
    g = torch.Generator().manual_seed(seed)
    occ = torch.randint(-1, 2, (batch, slots), generator=g).float()
    lg = (torch.randn(batch, slots, generator=g) * scale).to(dtype)
    if rank3:
        occ = occ.unsqueeze(-1)
    if strided and slots:
        lg = cases._strided_last_dim(lg)
    max_alloc = 1 + (seed % max(1, slots + max_extra))
    got = torch.ops.cid_engine.prefix_allocation_mask(_cuda(occ), _cuda(lg), threshold, max_alloc)
    exp = oracle.prefix_allocation_mask(occ, lg, threshold, max_alloc)
    compare.assert_matches("prefix_allocation_mask", got, exp, "fuzz prefix",
                           compare.sigmoid_ambiguous(lg, threshold))


@SETTINGS
@given(batch=st.integers(1, 5), slots=st.integers(1, 150), F=st.integers(1, 6),
       Rv=st.integers(1, 5), seed=st.integers(0, 2**31 - 1), dtype=DTYPES,
       threshold=UNIT, max_alloc=st.integers(1, 10))
def test_fuzz_rollout(batch, slots, F, Rv, seed, dtype, threshold, max_alloc) -> None:
    g = torch.Generator().manual_seed(seed)
    occ = torch.randint(0, 2, (batch, slots), generator=g).bool()
    al = torch.randn(batch, slots, generator=g).to(dtype)
    lc = torch.randint(-2, 3, (batch, slots, F), generator=g).to(dtype)  # ties
    rv = torch.randn(batch, slots, Rv, generator=g).to(dtype)
    il = torch.randint(-1, 2, (batch, slots, F), generator=g).to(dtype)
    r = seed % F
    got = torch.ops.cid_engine.rollout_slot_transition(occ.cuda(), al.cuda(), lc.cuda(), rv.cuda(),
                                                       il.cuda(), threshold, max_alloc, r)
    exp = oracle.rollout_slot_transition(occ, al, lc, rv, il, threshold, max_alloc, r)
    amb = compare.sigmoid_ambiguous(al, threshold)
    if bool(amb.any()):
        return  # the reference's own decision is position-dependent there
    for a, e in zip(got, exp):
        assert torch.equal(a.cpu(), e)


@SETTINGS
@given(batch=st.integers(1, 5), slots=st.integers(1, 150), F=st.integers(1, 6),
       Rv=st.integers(1, 5), seed=st.integers(0, 2**31 - 1), dtype=DTYPES,
       threshold=UNIT, max_alloc=st.integers(1, 10), special=st.booleans())
def test_fuzz_rollout_with_live(batch, slots, F, Rv, seed, dtype, threshold, max_alloc,
                                special) -> None:
    """The fused rollout + live occupancy equals rollout_slot_transition
    followed by live_slot_occupancy of its next occupancy (csrc/ops.cpp:184-256
    then :12-39); lifecycle values outside [0, 1] and NaN exercise the clamps."""
    g = torch.Generator().manual_seed(seed)
    occ = torch.randint(0, 2, (batch, slots), generator=g).bool()
    al = torch.randn(batch, slots, generator=g).to(dtype)
    lc = (torch.rand(batch, slots, F, generator=g) * 3 - 1).to(dtype)
    if special:
        lc.view(-1)[:: 7] = float("nan")
    rv = torch.randn(batch, slots, Rv, generator=g).to(dtype)
    il = torch.randint(-1, 2, (batch, slots, F), generator=g).to(dtype)
    r = seed % F
    got = torch.ops.cid_engine.rollout_slot_transition_with_live(
        occ.cuda(), al.cuda(), lc.cuda(), rv.cuda(), il.cuda(), threshold, max_alloc, r)
    exp = oracle.rollout_slot_transition(occ, al, lc, rv, il, threshold, max_alloc, r)
    if bool(compare.sigmoid_ambiguous(al, threshold).any()):
        return  # the reference's own decision is position-dependent there
    for a, e in zip(got[:6], exp):
        assert torch.equal(a.cpu(), e)
    live = oracle.live_slot_occupancy(exp[0].unsqueeze(-1).to(dtype), lc, r)
    assert got[6].dtype == dtype and got[6].shape == (batch, slots, 1)
    torch.testing.assert_close(got[6].cpu(), live, rtol=0, atol=0, equal_nan=True)


@SETTINGS
@given(batch=st.integers(1, 12), tokens=st.integers(1, 3000), seed=st.integers(0, 2**31 - 1),
       lo=st.floats(1e-6, 1.0), span=st.floats(0.0, 1.0), zero_rows=st.booleans())
def test_fuzz_masked_diffusion(batch, tokens, seed, lo, span, zero_rows) -> None:
    hi = min(1.0, lo + span)
    g = torch.Generator().manual_seed(seed)
    clean = torch.randint(0, 1000, (batch, tokens), generator=g)
    rr = torch.rand(batch, 1, generator=g)
    if zero_rows:
        rr[::2] = 0.0
    mr = torch.rand(batch, tokens, generator=g)
    got = torch.ops.cid_engine.masked_diffusion_corrupt_from_random(clean.cuda(), rr.cuda(),
                                                                    mr.cuda(), 999, lo, hi)
    exp = oracle.masked_diffusion_corrupt_from_random(clean, rr, mr, 999, lo, hi)
    compare.assert_matches("masked_diffusion_corrupt_from_random", got, exp, "fuzz md")


@SETTINGS
@given(batch=st.integers(0, 4), slots=st.integers(0, 40), hidden=st.integers(1, 300),
       seed=st.integers(0, 2**31 - 1), dtype=st.sampled_from([torch.float32, torch.float64,
                                                               torch.bfloat16, torch.float16]),
       tdtype=st.sampled_from([torch.float32, torch.float64, torch.bfloat16]))
def test_fuzz_thought_corruption(batch, slots, hidden, seed, dtype, tdtype) -> None:
    g = torch.Generator().manual_seed(seed)
    sem = torch.randn(batch, slots, hidden, generator=g).to(dtype)
    eps = torch.randn(batch, slots, hidden, generator=g).to(dtype)
    ts = (torch.rand(batch, slots, generator=g) * 1.5 - 0.25).to(tdtype)
    occ = torch.randint(0, 2, (batch, slots, 1), generator=g).to(dtype)
    got = torch.ops.cid_engine.thought_corrupt_from_epsilon(sem.cuda(), ts.cuda(), occ.cuda(),
                                                            eps.cuda())
    compare.assert_matches("thought_corrupt_from_epsilon", got,
                           oracle.thought_corrupt_from_epsilon(sem, ts, occ, eps), "fuzz thought")


@SETTINGS
@given(batch=st.integers(1, 40), columns=st.integers(1, 16), seed=st.integers(0, 2**31 - 1),
       integer_costs=st.booleans())
def test_fuzz_linear_assignment(batch, columns, seed, integer_costs) -> None:
    g = torch.Generator().manual_seed(seed)
    rows = 1 + seed % columns
    costs = torch.randn(batch, rows, columns, generator=g)
    if integer_costs:
        costs = (costs * 2).round()
    counts = torch.randint(0, rows + 1, (batch,), generator=g)
    got = torch.ops.cid_engine.batched_linear_assignment(costs.cuda(), counts.cuda())
    assert torch.equal(got.cpu(), oracle.batched_linear_assignment(costs, counts))


@SETTINGS
@given(batch=st.integers(0, 5), slots=st.integers(0, 48), features=st.integers(1, 8),
       seed=st.integers(0, 2**31 - 1), dtype=DTYPES, with_lifecycle=st.booleans(),
       special=st.booleans())
def test_fuzz_live_slot_occupancy(batch, slots, features, seed, dtype, with_lifecycle,
                                  special) -> None:
    """tests/test_fuzz.py:50-81 of the reference: occupancy and lifecycle
    drawn as N(0, 1.5^2) so both clamps of csrc/ops.cpp:12-39 are hit, the
    retired index from the seed; ``special`` adds NaN and infinities."""
    g = torch.Generator().manual_seed(seed)
    occ = (torch.randn(batch, slots, 1, generator=g) * 1.5).to(dtype)
    lc = None
    r = 0
    if with_lifecycle:
        lc = (torch.randn(batch, slots, features, generator=g) * 1.5).to(dtype)
        r = seed % features
        if special and lc.numel():
            lc.view(-1)[::5] = float("nan")
            lc.view(-1)[1::7] = float("inf")
            occ.view(-1)[::3] = float("-inf")
    got = torch.ops.cid_engine.live_slot_occupancy(occ.cuda(), None if lc is None else lc.cuda(),
                                                   r)
    exp = oracle.live_slot_occupancy(occ, lc, r)
    assert got.dtype == dtype and got.shape == occ.shape
    torch.testing.assert_close(got.cpu(), exp, rtol=0, atol=0, equal_nan=True)


@SETTINGS
@given(batch=st.integers(0, 4), slots=st.integers(0, 40), hidden=st.integers(1, 300),
       roles=st.integers(0, 8), lifecycles=st.integers(1, 6), picks=st.integers(0, 24),
       seed=st.integers(0, 2**31 - 1), dtypes=st.lists(DTYPES, min_size=5, max_size=5),
       ties=st.booleans(), host_indices=st.booleans())
def test_fuzz_materialize_cell_snapshot(batch, slots, hidden, roles, lifecycles, picks, seed,
                                        dtypes, ties, host_indices) -> None:
    """csrc/ops.cpp:556-615 of the reference with every input in its own
    dtype, repeated semantic indices, role counts down to zero, and (with
    ``ties``) integer-valued lifecycle logits with NaN so the argmax meets
    ties and NaN; indices resident on the host or on the device."""
    g = torch.Generator().manual_seed(seed)
    sem = torch.randn(batch, slots, hidden, generator=g).to(dtypes[0])
    rl = (torch.randn(batch, slots, roles, generator=g) * 8).to(dtypes[1])
    unc = torch.rand(batch, slots, 1, generator=g).to(dtypes[2])
    noise = torch.randn(batch, slots, 1, generator=g).to(dtypes[3])
    life = torch.randn(batch, slots, lifecycles, generator=g)
    if ties:
        life = (life * 1.5).round()
        if life.numel():
            life.view(-1)[::9] = float("nan")
    life = life.to(dtypes[4])
    sel = torch.rand(batch, slots, generator=g) > 0.5
    idx = torch.randint(0, hidden, (picks,), generator=g)
    got = torch.ops.cid_engine.materialize_cell_snapshot(
        sem.cuda(), rl.cuda(), unc.cuda(), noise.cuda(), life.cuda(), sel.cuda(),
        idx if host_indices else idx.cuda())
    exp = oracle.materialize_cell_snapshot(sem, rl, unc, noise, life, sel, idx)
    assert got.shape == (batch, slots, 4 + roles + picks)
    compare.assert_matches("materialize_cell_snapshot", got, exp, "fuzz snapshot")


@SETTINGS
@given(batch=st.integers(0, 6), tokens=st.integers(0, 3000),
       vocab=st.sampled_from([3, 4, 7, 50, 32000, 50257, (1 << 32) + 5]),
       seed=st.integers(0, 2**31 - 1), fraction=UNIT, density=UNIT,
       eos=st.sampled_from([None, 0, 1, 2]), mask_at_end=st.booleans(),
       el_dtype=st.sampled_from([torch.bool, torch.uint8, torch.int64, torch.float32]),
       r_dtype=DTYPES, t_dtype=DTYPES)
def test_fuzz_display_corruption(batch, tokens, vocab, seed, fraction, density, eos,
                                 mask_at_end, el_dtype, r_dtype, t_dtype) -> None:
    """csrc/ops.cpp:292-391 of the reference (the CUDA differential test of
    tests/test_cuda.py:155-195 over random shapes): timesteps at 0 and 1
    included, eligibility masks of every density in several dtypes, random
    dtypes for the uniform draws, offsets that wrap the vocabulary, EOS and
    mask ids that collide with the replacement candidates."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, min(vocab, 1 << 40), (batch, tokens), generator=g)
    ts = torch.rand(batch, generator=g)
    if batch:
        ts[torch.rand(batch, generator=g) < 0.25] = 0.0
        ts[torch.rand(batch, generator=g) < 0.15] = 1.0
    ts = ts.to(t_dtype)
    el = (torch.rand(batch, tokens, generator=g) < density).to(el_dtype)
    cr = torch.rand(batch, tokens, generator=g).to(r_dtype)
    rr = torch.rand(batch, tokens, generator=g).to(r_dtype)
    ro = torch.randint(-3 * min(vocab, 1 << 40), 3 * min(vocab, 1 << 40), (batch, tokens),
                       generator=g)
    mask_id = vocab - 1 if mask_at_end else 0
    got = torch.ops.cid_engine.display_corrupt_from_random(
        ids.cuda(), ts.cuda(), el.cuda(), cr.cuda(), rr.cuda(), ro.cuda(), mask_id, eos, vocab,
        fraction)
    exp = oracle.display_corrupt_from_random(ids, ts, el, cr, rr, ro, mask_id, eos, vocab,
                                             fraction)
    compare.assert_matches("display_corrupt_from_random", got, exp, "fuzz display corruption")
