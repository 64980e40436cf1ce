"""Pin the CPU oracle against the reference's own outputs.

``tests/golden/golden.pt`` holds the outputs of the reference CPU backend
(fwerkor/cid-engine v1.1.0 built from its sources by ``oracle/Makefile``) on
every case of ``tests/golden/cases.py``; ``tests/golden/make_golden.py``
produced it.  Here the oracle (``oracle/cid_oracle.c``) is run on the same
rebuilt inputs and must agree: exactly for decisions, ids, masks and argmax,
within the documented tolerances for floating outputs.
"""

from __future__ import annotations

import pytest
import torch

import cases
import compare
from oracle import oracle

GOLDEN = torch.load(compare.__file__.replace("compare.py", "golden.pt"))
CASES = list(cases.all_cases())


def _ambiguous(case: cases.Case):
    if case.op == "prefix_allocation_mask":
        lg = case.args[1]
        return compare.sigmoid_ambiguous(lg, case.args[2])
    return None


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_matches_reference(case: cases.Case) -> None:
    entry = GOLDEN[case.name]
    assert cases.digest(case.args) == entry["digest"], "input generator drifted"
    fn = getattr(oracle, case.op)
    if "error" in entry:
        with pytest.raises((RuntimeError, IndexError, ValueError)):
            fn(*case.args, **case.kwargs)
        return
    out = fn(*case.args, **case.kwargs)
    compare.assert_matches(case.op, out, entry["out"], case.name, _ambiguous(case))


def test_every_case_has_a_golden_entry() -> None:
    names = {c.name for c in CASES}
    assert names == set(GOLDEN), "regenerate tests/golden/golden.pt"


def test_sigmoid_band_is_narrow() -> None:
    """Outside a +-4 ulp band around the float32 threshold the allocation
    decision is exact.  The band is vanishingly thin for realistic logits:
    among 2**20 N(0, 3^2) logits at each threshold at most a couple fall in
    it."""
    g = torch.Generator().manual_seed(11)
    lg = torch.randn(1 << 20, generator=g) * 3.0
    for thr in (0.01, 0.3, 0.45, 0.5, 0.7, 0.99):
        assert int(compare.sigmoid_ambiguous(lg, thr).sum()) <= 2
