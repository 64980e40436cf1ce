"""GPU parity: every golden case through the CUDA path versus the oracle.

For each case of ``tests/golden/cases.py`` the inputs are rebuilt, placed on
``cuda:0`` with their strides preserved, and run through
``torch.ops.cid_engine``; the outputs must match the CPU oracle on the same
inputs with the tolerances of ``compare.py`` (exact for decisions, ids, masks
and argmax; float32 statistics within a pure relative 1e-5 of the exactly
rounded value).  Where the input digest matches the stored one, the
reference's own golden outputs are checked too (statistics: within 1e-5 of
the reference's value widened by the reference's own float32 summation drift
at that element).
"""

from __future__ import annotations

import pytest
import torch

import cases
import compare
from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = torch.load(compare.__file__.replace("compare.py", "golden.pt"))
CASES = list(cases.all_cases())


def to_cuda(x):
    """Copy to cuda:0 keeping the exact strides (non-contiguous views stay
    non-contiguous)."""
    if not isinstance(x, torch.Tensor):
        return x
    if x.is_contiguous():
        return x.to("cuda")
    out = torch.empty_strided(x.size(), x.stride(), dtype=x.dtype, device="cuda")
    out.copy_(x)
    return out


@pytest.fixture(scope="module", autouse=True)
def _engine():
    import cid_engine  # noqa: F401

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    yield


def _ambiguous(case: cases.Case):
    if case.op == "prefix_allocation_mask":
        return compare.sigmoid_ambiguous(case.args[1], case.args[2])
    return None


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_cuda_matches_oracle(case: cases.Case) -> None:
    entry = GOLDEN[case.name]
    fn = getattr(torch.ops.cid_engine, case.op)
    args = [to_cuda(a) for a in case.args]
    if "error" in entry:
        with pytest.raises((RuntimeError, IndexError, ValueError)):
            fn(*args)
        return
    out = fn(*args)
    torch.cuda.synchronize()
    if isinstance(out, torch.Tensor):
        out = (out,)
    for o in out:
        assert o.device.type == "cuda"
    expected = getattr(oracle, case.op)(*case.args)
    if isinstance(expected, torch.Tensor):
        expected = (expected,)
    compare.assert_matches(case.op, out, expected, case.name, _ambiguous(case))
    if cases.digest(case.args) != entry["digest"]:
        return
    if case.op in compare.STATS_OPS:
        # argmax exactly; confidences within 1e-5 of the reference's own
        # values, widened by the reference's drift from the exact value
        compare.assert_matches(case.op, (out[0], out[1], out[2]),
                               (expected[0], entry["out"][1], expected[2]),
                               case.name + "/golden argmax")
        for k in (0, 2):
            enc = entry["out"][k]
            a, r, e = out[k].cpu().flatten(), None, expected[k].flatten()
            if "full" in enc:
                r = enc["full"].flatten()
            else:
                a, e, r = a[:: enc["step"]], e[:: enc["step"]], enc["sample"].flatten()
            compare.assert_stats_vs_reference(a, r, e, f"{case.name}/golden[{k}]")
        return
    compare.assert_matches(case.op, out, entry["out"], case.name + "/golden", _ambiguous(case))
