"""The LM head fused with the display statistics
(``cid_engine.lm_head_display_statistics``) against the statistics of the
materialised logits.

References: logits = hidden.float() @ weight.float().T from torch in f32
(no TF32), then the (separately oracle-checked) statistics kernel on those
logits — as f32 for ``round_bf16=False``, rounded to bf16 for
``round_bf16=True``.  The tensor-core accumulation order differs from the
reference GEMM's, so: confidences within rtol 1e-4 (f32) / 1e-2 (bf16: a
logit can round to the neighbouring bf16 value); the predicted column must
hold the row maximum of the reference logits within the accumulation error
(f32: 1e-3 absolute; bf16: one bf16 ulp of the maximum), and must equal the
reference argmax exactly on every row whose maximum is unique by more than
that band.  Exact structure
is checked exactly: duplicated weight rows give bit-identical columns, and
the lower column must win.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _engine():
    import cid_engine  # noqa: F401

    assert torch.cuda.is_available()
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.cuda.empty_cache()


def _inputs(rows, vocab, hidden, seed, scale=0.5):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(seed)
    h = (torch.randn(rows, hidden, generator=g, device=dev) * scale).to(torch.bfloat16)
    w = (torch.randn(vocab, hidden, generator=g, device=dev) * scale).to(torch.bfloat16)
    ids = torch.randint(0, vocab, (rows,), generator=g, device=dev)
    return ids, h, w


def _check(ids, h, w, round_bf16):
    import cid_engine

    conf, pred, cur = cid_engine.lm_head_display_statistics(ids, h, w, round_bf16=round_bf16)
    logits = h.float() @ w.float().T
    if round_bf16:
        logits = logits.to(torch.bfloat16)
    e_conf, e_pred, e_cur = cid_engine.display_token_statistics(ids.view(1, -1),
                                                                logits.unsqueeze(0))
    e_conf, e_pred, e_cur = e_conf[0], e_pred[0], e_cur[0]
    rtol = 1e-2 if round_bf16 else 1e-4
    torch.testing.assert_close(conf, e_conf, rtol=rtol, atol=1e-7)
    torch.testing.assert_close(cur, e_cur, rtol=rtol, atol=1e-7)
    lf = logits.float()
    rowmax = lf.max(dim=1).values
    got = lf.gather(1, pred.view(-1, 1)).view(-1)
    tol = (rowmax.abs() * 2.0**-7 + 1e-6) if round_bf16 else torch.full_like(rowmax, 1e-3)
    assert bool(((rowmax - got) <= tol).all()), "predicted column does not hold the row maximum"
    # exact argmax wherever the reference logits' maximum is unique by more
    # than the accumulation-order band (bf16: one ulp of the maximum; f32:
    # 1e-3): only there can the tensor-core sum not reorder the top two
    second = lf.topk(2, dim=1).values[:, 1]
    clear = (rowmax - second) > tol
    assert bool(clear.any())
    assert torch.equal(pred[clear], e_pred[clear]), "argmax differs on a clear maximum"
    return conf, pred, cur


@pytest.mark.parametrize("round_bf16", [False, True])
@pytest.mark.parametrize("rows,vocab,hidden", [
    (5, 300, 64),        # one row block, two tiles, the last partial
    (300, 1000, 128),    # partial row block, 4 tiles
    (256, 5000, 72),     # hidden not a multiple of 64 (zero-filled K tail)
    (1000, 32000, 256),  # many work units and vocabulary groups
    (130, 70001, 64),    # groups of more than 4 tiles, odd vocabulary
    # launches of 1024 rows and more run the wide (256-row) tiles when the
    # logits are rounded to bf16
    (1024, 4096, 128),   # whole 256-row blocks
    (1100, 32000, 256),  # partial 256-row block
    (2300, 32000, 72),   # partial 256-row block, K tail
    (4100, 70001, 64),   # many raster groups, odd vocabulary
])
def test_lm_head_matches_materialised_logits(rows, vocab, hidden, round_bf16) -> None:
    import cid_engine

    cid_engine.device_status(0, reset=True)
    ids, h, w = _inputs(rows, vocab, hidden, seed=rows + vocab)
    _check(ids, h, w, round_bf16)
    assert cid_engine.device_status(0) == 0


def test_lm_head_wide_and_128_row_tiles_agree_bitwise() -> None:
    """The wide-tile kernel (launches of 1024 rows and more, bf16-rounded
    logits) accumulates every logit over K in the order of the 128-row
    kernel and rounds it the same way, so the statistics of a row are
    bit-identical whichever kernel served the launch: the first 1023 rows
    (128-row tiles) against the same rows of a 1100-row launch (wide tiles,
    a partial last block; both launches group the vocabulary alike)."""
    import cid_engine

    ids, h, w = _inputs(1100, 50001, 200, seed=11)
    cid_engine.device_status(0, reset=True)
    big = cid_engine.lm_head_display_statistics(ids, h, w)
    small = cid_engine.lm_head_display_statistics(ids[:1023], h[:1023].contiguous(), w)
    for a, b in zip(big, small):
        assert torch.equal(a[:1023], b)
    assert cid_engine.device_status(0) == 0


def test_lm_head_exact_ties_take_the_lower_column() -> None:
    import cid_engine

    ids, h, w = _inputs(200, 3000, 128, seed=4)
    # rows of the weight duplicated across tiles and groups: identical columns
    w[2900] = w[17]
    w[1500] = w[17]
    w[600] = w[599]
    conf, pred, cur = cid_engine.lm_head_display_statistics(ids, h, w, round_bf16=False)
    logits = h.float() @ w.float().T
    top = logits.argmax(dim=1)
    for dup, base in ((2900, 17), (1500, 17), (600, 599)):
        rows_dup = (pred == dup).nonzero().flatten()
        assert rows_dup.numel() == 0, f"column {dup} chosen over its duplicate {base}"
    # rows whose maximum sits on a duplicated column report the lower one
    hits = (top == 17) | (top == 1500) | (top == 2900)
    assert bool((pred[hits] == 17).all())


def test_lm_head_peaks_and_batch_shape() -> None:
    import cid_engine

    B, L, V, H = 3, 50, 4096, 64
    ids, h, w = _inputs(B * L, V, H, seed=9)
    # a planted dominant logit per row: hidden aligned with one weight row
    cols = torch.randint(0, V, (B * L,), device=h.device)
    h = (w[cols].float() * 4).to(torch.bfloat16)
    conf, pred, cur = cid_engine.lm_head_display_statistics(ids.view(B, L), h.view(B, L, H), w)
    assert conf.shape == (B, L) and pred.dtype == torch.int64
    logits = (h.float() @ w.float().T).to(torch.bfloat16).float()
    assert bool((logits.gather(1, pred.view(-1, 1)).view(-1) >= logits.max(1).values).all())


def test_lm_head_out_of_range_id_sets_status() -> None:
    import cid_engine

    ids, h, w = _inputs(64, 512, 64, seed=2)
    ids[3] = 512
    ids[5] = -1
    cid_engine.device_status(0, reset=True)
    conf, pred, cur = cid_engine.lm_head_display_statistics(ids, h, w)
    assert bool(cur[3].isnan()) and bool(cur[5].isnan())
    assert cid_engine.device_status(0) & cid_engine.STATUS_TOKEN_ID_OUT_OF_RANGE


def test_lm_head_validation() -> None:
    import cid_engine

    ids, h, w = _inputs(8, 256, 64, seed=1)
    with pytest.raises(RuntimeError, match="bfloat16"):
        cid_engine.lm_head_display_statistics(ids, h.float(), w)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        cid_engine.lm_head_display_statistics(ids, h[:, :60].contiguous(), w[:, :60].contiguous())
    with pytest.raises(RuntimeError, match="shape"):
        cid_engine.lm_head_display_statistics(ids[:4], h, w)


@pytest.mark.parametrize("rows,V", [(300, 20011), (1100, 20011), (200, 70001)])
@pytest.mark.parametrize("world", [2, 3])
def test_lm_head_shard_records_combine_to_unsharded(world, rows, V) -> None:
    """Vocabulary shards of the weight (as a vocabulary-parallel LM head holds
    them), reduced to records and combined, give the unsharded statistics:
    every column's logit is accumulated in the same order, so the argmax is
    exact; the sums are regrouped (rtol 1e-5).  1100 rows run the wide-tile
    kernel, whose records carry the shard's column offset too; 70001 columns
    make more than 32 groups a shard, merged by a warp per row."""
    import cid_engine
    from cid_engine import parallel

    H = 128
    ids, h, w = _inputs(rows, V, H, seed=world)
    conf, pred, cur = cid_engine.lm_head_display_statistics(ids, h, w)
    offs = parallel.shard_offsets(V, world)
    recs = torch.stack([
        cid_engine.lm_head_shard_records(ids, h, w[offs[r]:offs[r + 1]].contiguous(),
                                         vocab_offset=offs[r], total_vocab=V)
        for r in range(world)])
    c, p, u = cid_engine.display_combine_records(recs, ids.view(1, -1), offs)
    assert torch.equal(p.view(-1), pred)
    torch.testing.assert_close(c.view(-1), conf, rtol=1e-5, atol=1e-30)
    torch.testing.assert_close(u.view(-1), cur, rtol=1e-5, atol=1e-30)


def test_lm_head_shard_records_validation() -> None:
    import cid_engine

    ids, h, w = _inputs(8, 256, 64, seed=1)
    with pytest.raises(RuntimeError, match="inside"):
        cid_engine.lm_head_shard_records(ids, h, w, vocab_offset=10, total_vocab=256)
