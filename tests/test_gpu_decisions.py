"""End-to-end decision parity: logits -> statistics -> refined display ids.

Two paths over the same seeded logits:

* reference: the reference CPU kernel's own arithmetic for the statistics
  (``oracle.display_token_statistics_reference_order``, which reproduces the
  reference's golden confidences bit for bit for f32/f16/bf16 logits,
  csrc/cpu/display_stats.cpp:14-126) followed by the refinement policy of
  csrc/refine.cpp:222-429 (``oracle.refine_display_from_statistics``);
* device: ``display_token_statistics`` then
  ``refine_display_from_statistics`` on the GPU, with no host step between.

The refined ids must be identical.  Two further checks isolate the cause of
any difference: the argmax must match exactly, and the device policy fed
with the device's own statistics must equal the oracle policy on those same
statistics (so a remaining difference could only come from a confidence
that rounds differently, never from the policy).  The chain pattern follows
tests/test_cuda.py:103-123 of the reference.

Workloads: fp32 [4, 256, 32000] in full; the decode loop's 256 sequences of
512 positions over 32000 bf16 logits for one step and for 8 chained steps
(each step's refined ids feed the next; logits of step s from seed 4 + s);
the bf16 [32, 1024, 128256] display step in full.
"""

from __future__ import annotations

import pytest
import torch

import cases
import compare
from oracle import oracle

pytestmark = pytest.mark.gpu

MASK, EOS = 0, 1
POLICIES = ((0.25, 0.1, 0.05), (1.0, 1.0, 0.0))


@pytest.fixture(scope="module", autouse=True)
def _engine():
    import cid_engine  # noqa: F401

    assert torch.cuda.is_available()
    yield
    torch.cuda.empty_cache()


def _device(ids, logits, policy):
    ops = torch.ops.cid_engine
    stats = ops.display_token_statistics(ids, logits)
    refined = ops.refine_display_from_statistics(ids, *stats, MASK, EOS, *policy)
    return [t.cpu() for t in stats], refined.cpu()


def _reference(ids_h, logits_h, policy):
    stats = oracle.display_token_statistics_reference_order(ids_h, logits_h)
    refined = oracle.refine_display_from_statistics(ids_h, *stats, MASK, EOS, *policy)
    return stats, refined


def _compare(name, ids_h, dev, ref, policy, exact=None) -> int:
    """Rows whose refined ids differ between the two paths (asserted 0 by the
    callers), after checking argmax, the confidences and the policy on the
    device's own statistics.  With ``exact`` (the exactly rounded
    statistics) the confidences are held to 1e-5 of the reference's values
    widened by the reference's own drift; without it (the multi-GB cases) to
    2e-5 of the reference's values, the 1e-5 plus the largest drift of the
    reference's float32 sums measured on the golden cases (1.3e-5)."""
    (d_stats, d_ids), (r_stats, r_ids) = dev, ref
    assert torch.equal(d_stats[1], r_stats[1]), f"{name}: argmax differs"
    for k in (0, 2):
        if exact is not None:
            compare.assert_stats_close(d_stats[k], exact[k], f"{name}: stats[{k}] vs exact")
            compare.assert_stats_vs_reference(d_stats[k], r_stats[k], exact[k],
                                              f"{name}: stats[{k}] vs reference")
        else:
            torch.testing.assert_close(d_stats[k], r_stats[k], rtol=2e-5,
                                       atol=compare.STATS_ATOL, equal_nan=True,
                                       msg=f"{name}: stats[{k}] vs reference")
    policy_on_device_stats = oracle.refine_display_from_statistics(
        ids_h, *d_stats, MASK, EOS, *policy)
    assert torch.equal(policy_on_device_stats, d_ids), f"{name}: device policy differs"
    rows = (d_ids != r_ids).any(dim=1)
    return int(rows.sum())


@pytest.mark.parametrize("policy", POLICIES, ids=["bench-policy", "reveal-all"])
def test_fp32_4x256x32000_decisions(policy) -> None:
    ids, logits = cases.display_f32_4x256x32000()
    dev = _device(ids.cuda(), logits.cuda(), policy)
    ref = _reference(ids, logits, policy)
    exact = oracle.display_token_statistics(ids, logits)
    assert _compare("fp32 [4,256,32000]", ids, dev, ref, policy, exact) == 0


def _loop_logits(step: int, dev) -> torch.Tensor:
    import bench

    return bench.loop_logits(step, dev)


def test_decode_loop_256x512x32000_one_step() -> None:
    import bench

    dev = torch.device("cuda", 0)
    ids = bench.loop_initial_ids(dev)
    logits = _loop_logits(0, dev)
    policy = POLICIES[0]
    d = _device(ids, logits, policy)
    r = _reference(ids.cpu(), logits.cpu(), policy)
    assert _compare("decode loop step 0", ids.cpu(), d, r, policy) == 0


def test_decode_loop_256x512x32000_eight_chained_steps() -> None:
    """Each path carries its own ids from step to step; a row that diverged
    once would stay diverged, so the final count covers every step."""
    import bench

    dev = torch.device("cuda", 0)
    policy = POLICIES[0]
    d_ids = bench.loop_initial_ids(dev)
    r_ids = d_ids.cpu()
    changed = 0
    for s in range(8):
        logits = _loop_logits(s, dev)
        ids_before = d_ids.cpu()
        d = _device(d_ids, logits, policy)
        r = _reference(r_ids, logits.cpu(), policy)
        if torch.equal(ids_before, r_ids):
            assert _compare(f"decode loop step {s}", r_ids, d, r, policy) == 0
        assert torch.equal(d[1], r[1]), f"step {s}: refined ids diverged"
        changed += int((d[1] != ids_before).sum())
        d_ids = d[1].to(dev)
        r_ids = r[1]
        del logits
    assert changed > 0  # the chain did refine something


def test_display_step_32x1024x128256_decisions() -> None:
    import bench

    dev = torch.device("cuda", 0)
    ids, logits = bench.display_inputs(32, 1024, 128256, seed=1, device=dev)
    policy = POLICIES[0]
    d = _device(ids, logits, policy)
    r = _reference(ids.cpu(), logits.cpu(), policy)
    assert _compare("display step [32,1024,128256]", ids.cpu(), d, r, policy) == 0
