"""Deterministic input builders for the golden parity fixtures.

Every case is rebuilt from a seeded CPU ``torch.Generator`` on whichever
machine runs the tests, so the fixture file stores only expected outputs (and a
digest of the inputs, to detect generator drift).  Shapes and recipes follow
the reference's own tests (fwerkor/cid-engine v1.1.0, ``tests/``) and the
synthetic workloads of the benchmark configurations; the cited test lines are
given per case.

A case is ``Case(name, op, args, kwargs)`` where ``op`` names the reference
operator (``torch.ops.cid_engine.<op>``) and ``args`` are positional operator
arguments in schema order.
"""

from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass, field
from typing import Any, Callable, Iterator

import torch

MASK, EOS = 0, 1


@dataclass
class Case:
    name: str
    op: str
    args: list[Any]
    kwargs: dict[str, Any] = field(default_factory=dict)


def _g(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def digest(values: list[Any]) -> str:
    h = hashlib.sha256()
    for v in values:
        if isinstance(v, torch.Tensor):
            t = v.detach().contiguous()
            h.update(str((t.dtype, tuple(t.shape))).encode())
            h.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
        else:
            h.update(repr(v).encode())
    return h.hexdigest()


def _strided_last_dim(t: torch.Tensor) -> torch.Tensor:
    """Non-contiguous view with the same values (tests/test_fuzz.py:38-47)."""
    if t.shape[-1] == 0:
        return t
    storage = torch.zeros((*t.shape[:-1], t.shape[-1] * 2), dtype=t.dtype)
    storage[..., ::2] = t
    return storage[..., ::2]


# --------------------------------------------------------------------------
# display_token_statistics
# --------------------------------------------------------------------------


def adversarial_logits(vocab: int, dtype: torch.dtype, pattern: str):
    """tests/test_precision.py:43-68."""
    g = _g(0xC1D + vocab)
    shape = (2, 3, vocab)
    if pattern == "random":
        logits = torch.randn(shape, generator=g) * 7.0
    elif pattern == "wide":
        row = torch.linspace(-80.0, 80.0, vocab)
        logits = row.expand(shape).clone()
        logits[1] = logits[1].flip(-1)
    elif pattern == "near_tie":
        logits = torch.randn(shape, generator=g) * 1.0e-3
        logits[..., 0] = 1.0
        if vocab > 1:
            logits[..., 1] = 1.0 - 2.0e-6
    elif pattern == "offset":
        logits = torch.randn(shape, generator=g) * 0.25 + 10000.0
    else:
        raise AssertionError(pattern)
    logits = logits.to(dtype)
    ids = torch.randint(vocab, shape[:2], generator=g)
    return ids, logits


def display_f32_4x256x32000(seed: int = 0):
    """Display logits fp32 [4,256,32000] = 3*N(0,1); ids uniform; display mask
    Bernoulli(0.5) (inactive positions hold the mask id); an EOS planted per
    row with the tail masked, as tests/test_fuzz.py:232-237 does."""
    g = _g(seed)
    b, l, v = 4, 256, 32000
    logits = torch.randn((b, l, v), generator=g) * 3.0
    ids = torch.randint(2, v, (b, l), generator=g)
    active = torch.rand((b, l), generator=g) < 0.5
    ids[~active] = MASK
    for row in range(b):
        pos = int(torch.randint(l // 2, l, (), generator=g))
        ids[row, pos] = EOS
        ids[row, pos + 1 :] = MASK
    return ids, logits


def peaked_display_rows(rows: int, seed: int = 1, vocab: int = 128256):
    """Rows of the [32, 1024, 128256] bench distribution: bf16(2*N(0,1)) with
    a +8 peak in 10% of rows and an exact two-way tie at rowmax+1 in 1% of
    rows (lowest index wins)."""
    g = _g(seed)
    logits = (torch.randn((rows, vocab), generator=g) * 2.0).to(torch.bfloat16)
    peak = torch.rand(rows, generator=g) < 0.10
    where = torch.randint(vocab, (rows,), generator=g)
    for r in torch.nonzero(peak).flatten().tolist():
        c = int(where[r])
        logits[r, c] = (logits[r, c].float() + 8.0).to(torch.bfloat16)
    tie = torch.rand(rows, generator=g) < 0.01
    tie[0] = True
    for r in torch.nonzero(tie).flatten().tolist():
        j = torch.randperm(vocab, generator=g)[:2]
        top = logits[r].float().max() + 1.0
        logits[r, j] = top.to(torch.bfloat16)
    ids = torch.randint(vocab, (rows,), generator=g)
    return ids.view(1, rows), logits.view(1, rows, vocab)


def special_rows(dtype: torch.dtype):
    """NaN / +inf / all -inf rows (ATen max: first NaN wins; a non-finite
    max makes the normaliser NaN)."""
    v = 37
    logits = torch.randn((1, 8, v), generator=_g(5))
    logits[0, 0, 5] = float("nan")
    logits[0, 0, 9] = float("nan")
    logits[0, 1, 3] = float("inf")
    logits[0, 1, 30] = float("inf")
    logits[0, 2, :] = float("-inf")
    logits[0, 3, ::2] = float("-inf")
    logits[0, 4, 0] = float("nan")
    logits[0, 5, 36] = float("nan")
    logits[0, 6, :] = 0.0
    logits[0, 7, 36] = float("inf")
    logits[0, 7, 2] = float("nan")
    ids = torch.tensor([[1, 3, 0, 1, 2, 36, 4, 2]])
    return ids, logits.to(dtype)


def stats_cases() -> Iterator[Case]:
    op = "display_token_statistics"
    g = _g(7)  # tests/test_engine.py:16-26
    ids = torch.randint(257, (2, 13), generator=g)
    yield Case("stats/engine_seed7", op, [ids, torch.randn(2, 13, 257, generator=g)])
    for dt in (torch.float32, torch.bfloat16):  # tests/test_cuda.py:17-40 shapes
        g = _g(123)
        ids = torch.randint(4096, (2, 64), generator=g)
        lg = torch.randn(2, 64, 4096, generator=g).to(dt)
        yield Case(f"stats/cuda_shape_{str(dt)[6:]}", op, [ids, lg])
    yield Case(  # tests/test_cuda.py:94-100
        "stats/first_tie", op, [torch.tensor([[2]]), torch.tensor([[[1.0, 5.0, 5.0, 2.0]]])]
    )
    yield Case(  # tests/test_precision.py:25-40
        "stats/argmax_before_softmax", op,
        [torch.tensor([[0]]), torch.tensor([[[0.0, 1.0e-8]]])],
    )
    for dt in (torch.float32, torch.float64, torch.float16, torch.bfloat16):
        for vocab in (1, 2, 31, 32, 33, 255, 1023, 1024, 1025, 4097, 32000, 65536, 65537):
            for pattern in ("random", "wide", "near_tie", "offset"):
                ids, lg = adversarial_logits(vocab, dt, pattern)
                yield Case(f"stats/precision_{str(dt)[6:]}_{vocab}_{pattern}", op, [ids, lg])
        yield Case(f"stats/special_{str(dt)[6:]}", op, list(special_rows(dt)))
    # tests/test_fuzz.py:166-196 recipe
    for k in range(80):
        g = _g(1000 + k)
        batch = int(torch.randint(0, 5, (), generator=g))
        tokens = int(torch.randint(0, 33, (), generator=g))
        vocab = int(torch.randint(1, 1025, (), generator=g))
        dt = [torch.float16, torch.bfloat16, torch.float32, torch.float64][k % 4]
        scale = [0.0, 1.0e-4, 0.1, 1.0, 20.0, 100.0][k % 6]
        ids = torch.randint(vocab, (batch, tokens), generator=g)
        lg = (torch.randn(batch, tokens, vocab, generator=g) * scale).to(dt)
        if k % 3 == 0:
            lg = _strided_last_dim(lg)
        yield Case(f"stats/fuzz_{k}", op, [ids, lg])
    yield Case("stats/f32_4x256x32000", op, list(display_f32_4x256x32000()))
    yield Case("stats/peaked_rows256", op, list(peaked_display_rows(256)))
    g = _g(4)
    lg = (torch.randn(2, 512, 32000, generator=g) * 3.0).to(torch.bfloat16)
    yield Case("stats/bf16_2x512x32000", op, [torch.randint(32000, (2, 512), generator=g), lg])


# --------------------------------------------------------------------------
# display_token_statistics_with_repetition
# --------------------------------------------------------------------------


def repetition_cases() -> Iterator[Case]:
    op = "display_token_statistics_with_repetition"
    lg = torch.zeros(1, 5, 16)  # tests/test_engine.py:29-52
    lg[..., 9] = 3.0
    lg[..., 7] = 4.0
    yield Case("rep/engine", op, [torch.tensor([[7, 7, 7, 8, 7]]), lg, 5, 2, 0.7])
    lg = torch.zeros(1, 3, 16)  # tests/test_engine.py:55-71
    lg[0, 0, 7], lg[0, 0, 8], lg[0, 1, 7], lg[0, 2, 7] = 4.0, 3.0, 20.0, 20.0
    yield Case("rep/right_run", op, [torch.tensor([[7, 7, 7]]), lg, 5, 2, 0.5])
    for dt in (torch.float32, torch.bfloat16):  # tests/test_cuda.py:43-72
        lg = torch.zeros(1, 8, 32, dtype=dt)
        lg[..., 7] = 4.0
        lg[..., 9] = 3.0
        yield Case(
            f"rep/cuda_{str(dt)[6:]}", op,
            [torch.tensor([[7, 7, 7, 8, 7, 7, 5, 2]]), lg, 5, 2, 0.7],
        )
    for k in range(40):
        g = _g(2000 + k)
        b = 1 + k % 3
        t = [1, 2, 3, 7, 24, 33][k % 6]
        v = [16, 64, 300][k % 3]
        dt = [torch.float32, torch.bfloat16, torch.float16, torch.float64][k % 4]
        alphabet = torch.tensor([0, 1, 2, 3, 5, 7, v - 1])
        ids = alphabet[torch.randint(len(alphabet), (b, t), generator=g)]
        lg = (torch.randn(b, t, v, generator=g) * [0.5, 2.0, 8.0][k % 3]).to(dt)
        mult = [0.7, 0.5, 0.9, 1.0, 0.25][k % 5]
        eos = None if k % 4 == 3 else 1
        yield Case(f"rep/random_{k}", op, [ids, lg, 0, eos, mult])
    g = _g(2100)
    ids = torch.randint(2, 6, (2, 64), generator=g)
    lg = (torch.randn(2, 64, 4096, generator=g) * 2.0).to(torch.bfloat16)
    yield Case("rep/bf16_4096", op, [ids, lg, 0, 1, 0.7])


# --------------------------------------------------------------------------
# refine_display_from_statistics
# --------------------------------------------------------------------------


def softmax_stats(ids: torch.Tensor, logits: torch.Tensor):
    """The statistics the reference tests feed to refine
    (src/cid_engine/reference.py:293-308)."""
    lf = logits.float()
    prob = torch.softmax(lf, dim=-1)
    pred = lf.argmax(dim=-1)
    conf = prob.gather(-1, pred.unsqueeze(-1)).squeeze(-1)
    cur = prob.gather(-1, ids.unsqueeze(-1)).squeeze(-1)
    return conf, pred, cur


def _refine(name, ids, stats, mask, eos, reveal, revision, margin) -> Case:
    conf, pred, cur = stats
    return Case(
        name,
        "refine_display_from_statistics",
        [ids, conf, pred, cur, mask, eos, float(reveal), float(revision), float(margin)],
    )


def refine_inputs_fuzz(seed: int):
    """tests/test_fuzz.py:214-264 recipe, driven by one seed."""
    g = _g(seed)
    batch = int(torch.randint(1, 4, (), generator=g))
    tokens = int(torch.randint(1, 33, (), generator=g))
    vocab = int(torch.randint(4, 97, (), generator=g))
    units = [0.0, 1.0, 0.5, 1.0e-7, 1.0 - 1.0e-7]
    pick = lambda: (  # noqa: E731
        units[int(torch.randint(len(units), (), generator=g))]
        if torch.rand((), generator=g) < 0.4
        else float(torch.rand((), generator=g, dtype=torch.float64))
    )
    reveal, revision = pick(), pick()
    margins = [0.0, 1.0e-7, 0.01, 0.1, 1.0]
    margin = (
        margins[int(torch.randint(len(margins), (), generator=g))]
        if torch.rand((), generator=g) < 0.5
        else float(torch.rand((), generator=g, dtype=torch.float64))
    )
    with_eos = bool(torch.randint(0, 2, (), generator=g))
    scale = [0.0, 1.0e-4, 0.1, 1.0, 20.0, 100.0][int(torch.randint(6, (), generator=g))]
    eos = EOS if with_eos else None
    ids = torch.randint(2, vocab, (batch, tokens), generator=g)
    ids[torch.rand(batch, tokens, generator=g) < 0.3] = MASK
    if eos is not None:
        for row in range(batch):
            pos = (seed + row * 17) % tokens
            ids[row, pos] = eos
            if pos + 1 < tokens:
                ids[row, pos + 1 :] = MASK
    lg = torch.randn(batch, tokens, vocab, generator=g) * scale
    return ids, softmax_stats(ids, lg), eos, reveal, revision, margin


def refine_inputs_structural(seed: int, mode: str):
    """tests/test_fuzz.py:274-327 recipe."""
    g = _g(seed)
    active_tokens = int(torch.randint(4, 25, (), generator=g))
    capacity_extra = int(torch.randint(0, 9, (), generator=g))
    capacity = active_tokens + capacity_extra
    content = torch.arange(2, active_tokens + 1, dtype=torch.long)
    ids = torch.full((1, capacity), MASK, dtype=torch.long)
    ids[0, : active_tokens - 1] = content[: active_tokens - 1]
    ids[0, active_tokens - 1] = EOS
    pred = ids.clone()
    start = 1 + seed % max(1, active_tokens - 3)
    if mode == "insert" and capacity_extra > 0:
        inserted = int(torch.randint(64, 128, (), generator=g))
        shifted = ids[0, start : active_tokens - 1].clone()
        pred[0, start] = inserted
        n = min(len(shifted), capacity - start - 1)
        pred[0, start + 1 : start + 1 + n] = shifted[:n]
    elif mode == "delete" and start + 2 < active_tokens - 1:
        pred[0, start : active_tokens - 2] = ids[0, start + 1 : active_tokens - 1]
    conf = torch.full((1, capacity), 0.6)
    cur = torch.full((1, capacity), 0.6)
    conf[0, start] = 0.95
    cur[0, start] = 0.05
    return ids, (conf, pred, cur)


def refine_inputs_large(seed: int, batch: int, tokens: int, structural: float = 0.3):
    """Large refine workload built directly in statistics space: display ids
    with masked positions and an EOS per row, predictions that mostly agree
    with the ids, plus rows whose prediction is a shifted copy (so that the
    structural insert/delete search finds anchors)."""
    g = _g(seed)
    vocab = 97
    ids = torch.randint(2, vocab, (batch, tokens), generator=g)
    ids[torch.rand(batch, tokens, generator=g) < 0.35] = MASK
    eos_at = torch.randint(tokens // 4, tokens, (batch,), generator=g)
    has_eos = torch.rand(batch, generator=g) < 0.8
    for r in range(batch):
        if has_eos[r]:
            ids[r, eos_at[r]] = EOS
            ids[r, eos_at[r] + 1 :] = MASK
    pred = torch.where(
        torch.rand(batch, tokens, generator=g) < 0.7,
        ids,
        torch.randint(0, vocab, (batch, tokens), generator=g),
    )
    pred[ids == MASK] = torch.randint(2, vocab, (int((ids == MASK).sum()),), generator=g)
    shift_rows = torch.rand(batch, generator=g) < structural
    for r in torch.nonzero(shift_rows).flatten().tolist():
        s = int(torch.randint(0, max(1, tokens - 4), (), generator=g))
        if torch.rand((), generator=g) < 0.5:
            pred[r, s + 1 :] = ids[r, s:-1].clone()  # insertion proposal
            pred[r, s] = int(torch.randint(2, vocab, (), generator=g))
        else:
            d = int(torch.randint(1, 4, (), generator=g))
            pred[r, s : tokens - d] = ids[r, s + d :].clone()  # deletion proposal
    conf = torch.rand(batch, tokens, generator=g)
    # quantised keys produce many exact ties (stable order matters)
    conf = torch.where(torch.rand(batch, tokens, generator=g) < 0.3, (conf * 8).floor() / 8, conf)
    cur = torch.where(pred == ids, conf, conf * torch.rand(batch, tokens, generator=g))
    return ids, (conf, pred, cur)


def refine_cases() -> Iterator[Case]:
    # tests/test_engine.py:337-359
    ids = torch.tensor([[5, 9, 10, 11]])
    lg = torch.zeros(1, 4, 16)
    lg[0, 0, 5], lg[0, 0, 7], lg[0, 1, 12], lg[0, 2, 10], lg[0, 3, 13] = 20, 10, 10, 10, 9
    yield _refine("refine/reveal_revise", ids, softmax_stats(ids, lg), 5, None, 1.0, 0.5, 0.1)
    # tests/test_engine.py:362-381
    yield _refine(
        "refine/margin_quantization", torch.tensor([[2]]),
        (torch.tensor([[0.25]]), torch.tensor([[0]]), torch.tensor([[0.25]])),
        0, None, 0.0, 1.0, float.fromhex("0x0.0000000000001p-1022"),
    )
    # tests/test_engine.py:384-405
    ids = torch.tensor([[9, 2, 5, 5]])
    lg = torch.zeros(1, 4, 16)
    lg[0, 0, 9], lg[0, 1, 7], lg[0, 2, 8], lg[0, 3, 2] = 30, 30, 30, 30
    yield _refine("refine/eos_expansion", ids, softmax_stats(ids, lg), 5, 2, 1.0, 1.0, 0.0)
    # tests/test_engine.py:408-451
    for name, toks, proposal in (
        ("insertion", [9, 10, 11, 12, 13, 14, 2, 5, 5], [9, 10, 7, 11, 12, 13, 0, 0, 0]),
        ("deletion", [9, 10, 7, 11, 12, 13, 14, 2, 5], [9, 10, 11, 12, 13, 0, 0, 0, 0]),
    ):
        ids = torch.tensor([toks])
        lg = torch.full((1, 9, 16), -20.0)
        for p, t in enumerate(proposal):
            lg[0, p, t] = 20.0
        yield _refine(f"refine/{name}", ids, softmax_stats(ids, lg), 5, 2, 1.0, 1.0, 0.0)
    for k in range(400):
        ids, stats, eos, reveal, revision, margin = refine_inputs_fuzz(3000 + k)
        yield _refine(f"refine/fuzz_{k}", ids, stats, MASK, eos, reveal, revision, margin)
    for k in range(160):
        mode = "insert" if k % 2 == 0 else "delete"
        ids, stats = refine_inputs_structural(5000 + k, mode)
        yield _refine(f"refine/structural_{mode}_{k}", ids, stats, MASK, EOS, 1.0, 1.0, 0.1)
    for k, (b, t) in enumerate(((64, 40), (32, 96), (16, 257), (8, 512))):
        ids, stats = refine_inputs_large(6000 + k, b, t)
        for j, (rv, rf, mg) in enumerate(((0.25, 0.1, 0.05), (1.0, 1.0, 0.0), (0.5, 0.3, 0.2))):
            yield _refine(f"refine/large_{b}x{t}_{j}", ids, stats, MASK, EOS, rv, rf, mg)
        yield _refine(f"refine/large_{b}x{t}_noeos", ids, stats, MASK, None, 0.3, 0.2, 0.01)


# --------------------------------------------------------------------------
# slot operators
# --------------------------------------------------------------------------


def sigmoid_boundary_logits(threshold: float, ulps: int) -> torch.Tensor:
    """float32 logits within +-ulps of the float32 sigmoid boundary."""
    boundary = math.log(threshold / (1.0 - threshold))
    centre = torch.tensor([boundary], dtype=torch.float32).view(torch.int32)
    offs = torch.arange(-ulps, ulps + 1, dtype=torch.int32)
    if boundary < 0:
        offs = -offs
    bits = centre + offs
    return bits.view(torch.float32)


def prefix_cases() -> Iterator[Case]:
    op = "prefix_allocation_mask"
    occ = torch.tensor([[[1.0], [0.0], [0.0], [0.0], [0.0]], [[0.0], [1.0], [0.0], [0.0], [0.0]]])
    lg = torch.tensor([[10.0, 10.0, 10.0, -10.0, 10.0], [10.0, -10.0, 10.0, 10.0, 10.0]])
    yield Case("prefix/engine", op, [occ, lg, 0.5, 2])  # tests/test_engine.py:74-95
    yield Case(  # tests/cpp/test_ops.cpp:10-29
        "prefix/cpp_kat", op,
        [torch.tensor([1.0, 0.0, 0.0, 0.0]).reshape(1, 4, 1),
         torch.tensor([10.0, 10.0, 10.0, -10.0]).reshape(1, 4), 0.5, 2],
    )
    for dt in (torch.float16, torch.bfloat16, torch.float32, torch.float64):
        for batch in (1, 8):  # tests/test_cuda.py:289-334 recipe
            for rank3 in (False, True):
                g = _g(812)
                occ = torch.randint(-1, 2, (batch, 128), generator=g).float()
                if rank3:
                    occ = occ.unsqueeze(-1)
                storage = torch.randn(batch, 256, generator=g).to(dt)
                yield Case(
                    f"prefix/cuda_{str(dt)[6:]}_{batch}_{int(rank3)}", op,
                    [occ, storage[:, ::2], 0.45, 4],
                )
    for thr in (1.0e-6, 0.01, 0.5, 0.99, 1.0 - 1.0e-6):  # tests/test_precision.py:157-183
        boundary = math.log(thr / (1.0 - thr))
        lg = torch.tensor(
            [[math.nextafter(boundary, -math.inf), boundary,
              math.nextafter(boundary, math.inf), 80.0, -80.0]],
            dtype=torch.float64,
        )
        yield Case(f"prefix/boundary_{thr}", op, [torch.zeros(1, 5), lg, thr, 5])
    # dense ulp sweep around the boundary: one slot per row so every logit is
    # an independent decision
    for thr in (1.0e-6, 0.01, 0.3, 0.45, 0.5, 0.7, 0.99, 1.0 - 1.0e-6):
        lg = sigmoid_boundary_logits(thr, 256).view(-1, 1)
        yield Case(f"prefix/sweep_{thr}", op, [torch.zeros_like(lg), lg, thr, 1])
    for k in range(120):  # tests/test_fuzz.py:84-126 recipe
        g = _g(7000 + k)
        batch = int(torch.randint(0, 6, (), generator=g))
        slots = int(torch.randint(0, 65, (), generator=g))
        thr = [0.0, 1.0, 0.5, 1.0e-7, 1.0 - 1.0e-7, float(torch.rand((), generator=g))][k % 6]
        scale = [0.0, 1.0e-4, 0.1, 1.0, 20.0, 100.0][(k // 6) % 6]
        occ = torch.randint(-1, 2, (batch, slots), generator=g).float()
        lg = torch.randn(batch, slots, generator=g) * scale
        if k % 2:
            occ = occ.unsqueeze(-1)
        if k % 3 == 0 and slots:
            lg = _strided_last_dim(lg)
        max_alloc = 1 + (k % max(1, slots + 1 + k % 8))
        yield Case(f"prefix/fuzz_{k}", op, [occ, lg, thr, max_alloc])
    for dt in (torch.bool, torch.int64, torch.uint8, torch.float64):
        g = _g(7500)
        occ = torch.randint(0, 2, (3, 40), generator=g).to(dt)
        yield Case(f"prefix/occ_{str(dt)[6:]}", op, [occ, torch.randn(3, 40, generator=g), 0.4, 6])


def rollout_cases() -> Iterator[Case]:
    op = "rollout_slot_transition"
    g = _g(433)  # tests/test_engine.py:98-128
    occ = torch.randint(0, 2, (3, 17, 1), generator=g).bool()
    al = torch.randn(3, 17, generator=g)
    lc = torch.randn(3, 17, 4, generator=g)
    rv = torch.randn(3, 17, 3, generator=g)
    il = torch.randn(3, 17, 4, generator=g)
    il[:, ::5] = 0
    yield Case("rollout/engine", op, [occ, al, lc, rv, il, 0.45, 3, 3])
    for dt in (torch.float16, torch.bfloat16, torch.float32):  # tests/test_cuda.py:453-492
        g = _g(744)
        occ = torch.randint(0, 2, (8, 128), generator=g).bool()
        al = torch.randn(8, 128, generator=g).to(dt)
        lc = torch.randn(8, 128, 4, generator=g).to(dt)
        rv = torch.randn(8, 128, 3, generator=g).to(dt)
        il = torch.randn(8, 128, 4, generator=g).to(dt)
        il[:, ::7] = 0
        yield Case(f"rollout/cuda_{str(dt)[6:]}", op, [occ, al, lc, rv, il, 0.45, 4, 3])
    g = _g(745)  # ties and NaN in the argmax inputs
    lc = torch.randint(-1, 2, (4, 33, 4), generator=g).float()
    rv = torch.randint(-1, 2, (4, 33, 3), generator=g).float()
    il = torch.randint(-1, 2, (4, 33, 4), generator=g).float()
    lc[0, 0, 2] = float("nan")
    il[1, 3, 1] = float("nan")
    occ = torch.randint(0, 2, (4, 33, 1), generator=g).float()
    yield Case("rollout/ties_nan", op, [occ, torch.randn(4, 33, generator=g), lc, rv, il, 0.5, 5, 1])
    g = _g(4)  # decode-loop slot state: B=256, S=128, F=4, Rv=3, retired index 3
    occ = (torch.rand(256, 128, generator=g) < 0.4).float().unsqueeze(-1)
    yield Case(
        "rollout/256x128", op,
        [occ, torch.randn(256, 128, generator=g), torch.randn(256, 128, 4, generator=g),
         torch.randn(256, 128, 3, generator=g), torch.randn(256, 128, 4, generator=g),
         0.5, 8, 3],
    )


def live_cases() -> Iterator[Case]:
    op = "live_slot_occupancy"
    occ = torch.tensor([[[1.0], [0.7], [0.0], [1.2]]])  # tests/test_engine.py:131-154
    lc = torch.zeros(1, 4, 3)
    lc[0, 1, 2] = 1.0
    lc[0, 3, 2] = 0.25
    yield Case("live/engine", op, [occ, lc, 2])
    yield Case("live/no_lifecycle", op, [torch.tensor([[[1.2], [-0.1], [0.5]]]), None, 0])
    for k in range(30):  # tests/test_fuzz.py:50-81 recipe
        g = _g(8000 + k)
        b, s, f = 1 + k % 5, [0, 1, 17, 48][k % 4], 1 + k % 8
        dt = [torch.float32, torch.float64, torch.bfloat16, torch.float16][k % 4]
        occ = (torch.randn(b, s, 1, generator=g) * 1.5).to(dt)
        lc = None if k % 5 == 4 else (torch.randn(b, s, f, generator=g) * 1.5).to(dt)
        yield Case(f"live/fuzz_{k}", op, [occ, lc, (k * 7) % f if lc is not None else 0])


def snapshot_cases() -> Iterator[Case]:
    op = "materialize_cell_snapshot"
    g = _g(31)  # tests/test_engine.py:454-483
    yield Case(
        "snapshot/engine", op,
        [torch.randn(2, 5, 17, generator=g), torch.randn(2, 5, 6, generator=g),
         torch.rand(2, 5, 1, generator=g), torch.randn(2, 5, 1, generator=g),
         torch.randn(2, 5, 4, generator=g), torch.rand(2, 5, generator=g) > 0.5,
         torch.tensor([0, 3, 8, 16])],
    )
    idx = torch.tensor([0, 23, 47, 70, 93, 117, 140, 163, 187, 210, 233, 256])
    for dt in (torch.float16, torch.bfloat16, torch.float32):  # tests/test_cuda.py:392-424
        g = _g(902)
        yield Case(
            f"snapshot/cuda_{str(dt)[6:]}", op,
            [torch.randn(2, 128, 257, generator=g).to(dt), torch.randn(2, 128, 6, generator=g).to(dt),
             torch.rand(2, 128, 1, generator=g).to(dt), torch.randn(2, 128, 1, generator=g).to(dt),
             torch.randn(2, 128, 4, generator=g).to(dt), torch.rand(2, 128, generator=g) > 0.5, idx],
        )
    g = _g(903)
    yield Case(
        "snapshot/8x128x512", op,
        [torch.randn(8, 128, 512, generator=g).to(torch.bfloat16),
         torch.randn(8, 128, 6, generator=g).to(torch.bfloat16),
         torch.rand(8, 128, 1, generator=g).to(torch.bfloat16),
         torch.randn(8, 128, 1, generator=g).to(torch.bfloat16),
         torch.randn(8, 128, 4, generator=g).to(torch.bfloat16),
         torch.rand(8, 128, generator=g) > 0.5,
         torch.randint(0, 512, (12,), generator=g)],
    )
    g = _g(904)
    yield Case(
        "snapshot/empty_indices", op,
        [torch.randn(1, 3, 8, generator=g), torch.randn(1, 3, 2, generator=g),
         torch.rand(1, 3, 1, generator=g), torch.randn(1, 3, 1, generator=g),
         torch.randn(1, 3, 5, generator=g), torch.tensor([[True, False, True]]),
         torch.zeros(0, dtype=torch.long)],
    )


def masked_diffusion_cases() -> Iterator[Case]:
    op = "masked_diffusion_corrupt_from_random"
    g = _g(71)  # tests/test_engine.py:247-273
    yield Case(
        "md/engine", op,
        [torch.randint(0, 97, (4, 33), generator=g), torch.rand(4, 1, generator=g),
         torch.rand(4, 33, generator=g), 96, 0.001, 0.9],
    )
    yield Case(  # tests/test_engine.py:276-301
        "md/forced_fallback", op,
        [torch.tensor([[1, 2, 3, 4], [5, 6, 7, 8]]), torch.zeros(2, 1),
         torch.tensor([[0.9, 0.7, 0.8, 0.6], [0.5, 0.4, 0.3, 0.2]]), 99, 1.0e-6, 1.0e-6],
    )
    g = _g(211)  # tests/test_cuda.py:126-152 shapes
    yield Case(
        "md/cuda_shape", op,
        [torch.randint(0, 32000, (8, 2048), generator=g), torch.rand(8, 1, generator=g),
         torch.rand(8, 2048, generator=g), 31999, 0.001, 1.0],
    )
    yield Case("md/64x2048", op, list(masked_diffusion_64x2048()))
    for k in range(30):
        g = _g(9000 + k)
        b, t = 1 + k % 7, [1, 2, 5, 64, 333][k % 5]
        lo = [1.0e-6, 0.001, 0.3][k % 3]
        hi = [lo, 0.9, 1.0][k % 3]
        rr = torch.rand(b, 1, generator=g)
        rr[torch.rand(b, 1, generator=g) < 0.3] = 0.0
        mr = torch.rand(b, t, generator=g)
        if k % 4 == 0:
            mr = (mr * 4).floor() / 4  # ties for the argmin fallback
        yield Case(f"md/random_{k}", op, [torch.randint(0, 500, (b, t), generator=g), rr, mr, 499, lo, hi])
    # long rows (one to three batches of loads per thread at each block size);
    # ratio-0 rows take the argmin fallback, quantised uniforms make it a tie
    for k, (b, t) in enumerate(((3, 1025), (5, 4097), (2, 9000))):
        g = _g(9050 + k)
        rr = torch.rand(b, 1, generator=g)
        rr[0] = 0.0
        mr = torch.rand(b, t, generator=g)
        mr[0] = (mr[0] * 64).floor() / 64
        yield Case(f"md/long_{k}", op, [torch.randint(0, 50257, (b, t), generator=g), rr, mr, 50256, 1.0e-6, 1.0])


def masked_diffusion_64x2048(seed: int = 2):
    """Masked diffusion: ids [64,2048] uniform in [0,50257); ratio U(0,1) with 3 of
    64 rows forced to 0; uniforms fp32; mask id 50256; min 1e-6, max 1."""
    g = _g(seed)
    clean = torch.randint(0, 50257, (64, 2048), generator=g)
    ratio = torch.rand(64, 1, generator=g)
    ratio[torch.randperm(64, generator=g)[:3]] = 0.0
    mask_random = torch.rand(64, 2048, generator=g)
    return clean, ratio, mask_random, 50256, 1.0e-6, 1.0


def thought_cases() -> Iterator[Case]:
    op = "thought_corrupt_from_epsilon"
    g = _g(9)  # tests/test_engine.py:157-182
    sem = torch.randn(2, 5, 16, generator=g)
    eps = torch.randn(2, 5, 16, generator=g)
    ts = torch.rand(2, 5, generator=g)
    occ = torch.tensor([[[1.0], [1.0], [0.0], [1.0], [0.0]], [[1.0], [0.0], [1.0], [1.0], [1.0]]])
    yield Case("thought/engine", op, [sem, ts, occ, eps])
    for dt in (torch.float16, torch.bfloat16, torch.float32):  # tests/test_cuda.py:198-226
        g = _g(194)
        yield Case(
            f"thought/cuda_{str(dt)[6:]}", op,
            [torch.randn(4, 128, 257, generator=g).to(dt), torch.rand(4, 128, generator=g),
             torch.rand(4, 128, 1, generator=g) > 0.3, torch.randn(4, 128, 257, generator=g).to(dt)],
        )
    for dt in (torch.bfloat16, torch.float32, torch.float64):  # tests/test_precision.py:102-154
        for t in (0.0, 1.0e-7, 0.25, 0.5, 0.75, 1.0 - 1.0e-7, 1.0):
            g = _g(1701)
            sem = (torch.randn(2, 5, 17, generator=g) * 3.0).to(dt)
            eps = (torch.randn(2, 5, 17, generator=g) * 3.0).to(dt)
            occ = torch.randint(0, 2, (2, 5, 1), generator=g).to(dt)
            yield Case(f"thought/precision_{str(dt)[6:]}_{t}", op, [sem, torch.full((2, 5), t, dtype=dt), occ, eps])
    for k in range(24):  # tests/test_fuzz.py:129-163 recipe
        g = _g(9500 + k)
        b, s, h = k % 4, [0, 1, 24][k % 3], [1, 17, 96][k % 3]
        dt = [torch.float32, torch.float64, torch.bfloat16][k % 3]
        yield Case(
            f"thought/fuzz_{k}", op,
            [torch.randn(b, s, h, generator=g).to(dt),
             (torch.rand(b, s, generator=g) * 1.5 - 0.25).to(dt),
             torch.randint(0, 2, (b, s, 1), generator=g).to(dt),
             torch.randn(b, s, h, generator=g).to(dt)],
        )
    yield Case("thought/4x32x512", op, list(thought_4x32x512()))


def thought_4x32x512(seed: int = 0):
    """Thought state fp32 [4,32,512] N(0,1), eps N(0,1), t = 0.3,
    occupancy Bernoulli(0.4)."""
    g = _g(seed + 100)
    sem = torch.randn(4, 32, 512, generator=g)
    eps = torch.randn(4, 32, 512, generator=g)
    occ = (torch.rand(4, 32, 1, generator=g) < 0.4).float()
    return sem, torch.full((4, 32), 0.3), occ, eps


def display_corrupt_cases() -> Iterator[Case]:
    op = "display_corrupt_from_random"
    g = _g(177)  # tests/test_engine.py:185-219
    yield Case(
        "dc/engine", op,
        [torch.randint(0, 257, (4, 41), generator=g), torch.rand(4, generator=g),
         torch.rand(4, 41, generator=g) > 0.2, torch.rand(4, 41, generator=g),
         torch.rand(4, 41, generator=g), torch.randint(1, 257, (4, 41), generator=g),
         256, 2, 257, 0.25],
    )
    yield Case(  # tests/test_engine.py:222-244
        "dc/first_eligible_fallback", op,
        [torch.tensor([[10, 11, 12, 13]]), torch.tensor([1.0e-6]),
         torch.tensor([[False, False, True, True]]), torch.ones(1, 4), None, None,
         99, None, 100, 0.0],
    )
    g = _g(913)  # tests/test_cuda.py:155-195 shapes
    yield Case(
        "dc/cuda_shape", op,
        [torch.randint(0, 32000, (8, 1536), generator=g), torch.rand(8, generator=g),
         torch.rand(8, 1536, generator=g) > 0.15, torch.rand(8, 1536, generator=g),
         torch.rand(8, 1536, generator=g), torch.randint(1, 32000, (8, 1536), generator=g),
         31999, 2, 32000, 0.25],
    )
    for k in range(30):
        g = _g(9700 + k)
        b, t, v = 1 + k % 4, [1, 3, 50, 300][k % 4], [3, 5, 50][k % 3]
        ids = torch.randint(0, v, (b, t), generator=g)
        ts = torch.rand(b, generator=g)
        ts[torch.rand(b, generator=g) < 0.3] = 0.0
        el = torch.rand(b, t, generator=g) > [0.0, 0.5, 0.95][k % 3]
        frac = [0.0, 0.25, 1.0][k % 3]
        rr = torch.rand(b, t, generator=g) if frac > 0 else None
        ro = torch.randint(-5, 2 * v, (b, t), generator=g) if frac > 0 else None
        eos = None if k % 5 == 0 else 1
        yield Case(f"dc/random_{k}", op, [ids, ts, el, torch.rand(b, t, generator=g), rr, ro, 0, eos, v, frac])
    # long rows (one, two and three batches of loads per thread at each block
    # size), vocabularies at and past 2^32, offsets at the int64 limits (the
    # id + offset sum wraps as ATen's int64 add does)
    top = torch.iinfo(torch.int64).max
    shapes = ((3, 1025, 50257, 0.25), (2, 2049, 7, 1.0), (4, 5000, (1 << 33) + 7, 0.25),
              (2, 9000, 1 << 32, 1.0), (2, 4097, (1 << 32) - 1, 0.5))
    for k, (b, t, v, frac) in enumerate(shapes):
        g = _g(9800 + k)
        ids = torch.randint(0, min(v, 1 << 40), (b, t), generator=g)
        ts = torch.rand(b, generator=g)
        ts[0] = 0.0
        el = torch.rand(b, t, generator=g) > 0.15
        ro = torch.randint(-(1 << 62), 1 << 62, (b, t), generator=g)
        ro[0, :64] = top - torch.arange(64)
        ro[1, :64] = -top - 1 + torch.arange(64)
        ro[1, 64:128] = torch.randint(-5, 2 * min(v, 1 << 40), (64,), generator=g)
        yield Case(
            f"dc/long_{k}", op,
            [ids, ts, el, torch.rand(b, t, generator=g), torch.rand(b, t, generator=g), ro,
             v - 1, None if k == 1 else 1, v, frac],
        )


def assignment_cases() -> Iterator[Case]:
    op = "batched_linear_assignment"
    costs = torch.tensor(  # tests/test_engine.py:507-530
        [[[4.0, 1.0, 3.0, 8.0], [2.0, 0.0, 5.0, 7.0], [3.0, 2.0, 2.0, 6.0], [9.0, 9.0, 9.0, 9.0]],
         [[1.0, 1.0, 2.0, 3.0], [1.0, 1.0, 2.0, 3.0], [2.0, 2.0, 0.0, 0.0], [4.0, 3.0, 2.0, 1.0]]])
    yield Case("assign/engine", op, [costs, torch.tensor([3, 4])])
    yield Case("assign/cpp_kat", op, [costs[:1], torch.tensor([3])])  # tests/cpp/test_ops.cpp:33-53
    yield Case("assign/first_tie", op, [torch.zeros(2, 8, 8), torch.tensor([4, 8])])  # test_cuda.py:495-502
    for columns in (4, 8):  # tests/test_cuda.py:427-450 recipe
        g = _g(1417 + columns)
        yield Case(
            f"assign/cuda_{columns}", op,
            [torch.randn(128, columns, columns, generator=g),
             torch.randint(0, columns + 1, (128,), generator=g)],
        )
    for k in range(24):
        g = _g(9900 + k)
        columns = [1, 2, 5, 9, 16, 16][k % 6]
        rows = max(1, columns - (k % 3))
        b = 1 + k % 5
        c = torch.randn(b, rows, columns, generator=g)
        if k % 4 == 0:
            c = (c * 2).round()  # many equal costs: tie order matters
        if k % 4 == 1:
            c = c.to(torch.float64)
        yield Case(f"assign/random_{k}", op, [c, torch.randint(0, rows + 1, (b,), generator=g)])


ALL: dict[str, Callable[[], Iterator[Case]]] = {
    "stats": stats_cases,
    "repetition": repetition_cases,
    "refine": refine_cases,
    "prefix": prefix_cases,
    "rollout": rollout_cases,
    "live": live_cases,
    "snapshot": snapshot_cases,
    "masked_diffusion": masked_diffusion_cases,
    "thought": thought_cases,
    "display_corrupt": display_corrupt_cases,
    "assignment": assignment_cases,
}


def all_cases(groups: list[str] | None = None) -> Iterator[Case]:
    for name, fn in ALL.items():
        if groups is None or name in groups:
            yield from fn()
