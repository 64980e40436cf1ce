"""GPU parity at the benchmark configurations' sizes, and device behaviours.

Full-size inputs are generated on the device; rows small enough for the
oracle are copied back and checked exactly (argmax, ids, decisions) or within
the statistics tolerance; the rest is checked through size-independent
properties (planted-tie rows must report the lower column, every argmax must
hold the row maximum, sharded == unsharded, repeated calls are identical).
"""

from __future__ import annotations

import pytest
import torch

import cases
import compare
from oracle import oracle

pytestmark = pytest.mark.gpu

STATS = "display_token_statistics"


@pytest.fixture(scope="module", autouse=True)
def _engine():
    import cid_engine  # noqa: F401

    assert torch.cuda.is_available()
    yield
    torch.cuda.empty_cache()


def _check_stats(out, ids, logits, name):
    expected = oracle.display_token_statistics(ids, logits)
    compare.assert_matches(STATS, out, expected, name)


def test_full_size_32x1024x128256_rows_match_oracle() -> None:
    """The bench step's logits, bf16 [32, 1024, 128256], with planted peaks and exact ties."""
    import bench

    dev = torch.device("cuda", 0)
    ids, logits = bench.display_inputs(32, 1024, 128256, seed=1, device=dev)
    conf, pred, cur = torch.ops.cid_engine.display_token_statistics(ids, logits)
    torch.cuda.synchronize()
    flat = logits.view(-1, 128256)
    # every argmax holds the row maximum (size-independent property)
    row_max = flat.amax(dim=1)  # exact in bf16
    got = flat.gather(1, pred.view(-1, 1)).view(-1)
    assert torch.equal(got, row_max)
    # rows with two equal maxima report the lower column (first maximum)
    first = torch.max((flat == row_max[:, None]).to(torch.uint8), dim=1).indices
    assert torch.equal(pred.view(-1), first)
    del first
    # 512 rows spread over the tensor against the oracle
    sel = torch.linspace(0, 32 * 1024 - 1, 512, device=dev).long()
    sub_ids = ids.view(-1)[sel].view(1, -1).cpu()
    sub_lg = flat[sel].view(1, -1, 128256).cpu()
    out = (conf.view(-1)[sel].view(1, -1), pred.view(-1)[sel].view(1, -1), cur.view(-1)[sel].view(1, -1))
    _check_stats(out, sub_ids, sub_lg, "32x1024x128256 rows")
    assert bool(torch.isfinite(conf).all()) and bool(((conf > 0) & (conf <= 1)).all())
    assert bool((cur <= conf * (1 + 1e-6)).all())


@pytest.mark.parametrize("rows", [1, 3, 8, 16, 32, 64, 128, 256, 512])
@pytest.mark.parametrize("dtype,vocab", [(torch.bfloat16, 155136), (torch.float32, 32000),
                                         (torch.float16, 50021)])
def test_decode_rows_match_oracle(rows: int, dtype: torch.dtype, vocab: int) -> None:
    """Few-row (decode) launches, which split each row over a cluster of up
    to 16 CTAs, on the published decode widths; a planted peak and an exact
    tie in a few rows."""
    g = torch.Generator().manual_seed(rows * 7 + vocab)
    logits = (torch.randn(1, rows, vocab, generator=g) * 2).to(dtype)
    ids = torch.randint(vocab, (1, rows), generator=g)
    logits[0, 0, vocab - 1] = 30.0
    if rows > 2:
        logits[0, 2, [5, vocab // 2]] = 40.0
    out = torch.ops.cid_engine.display_token_statistics(ids.cuda(), logits.cuda())
    torch.cuda.synchronize()
    _check_stats(out, ids, logits, f"decode [1,{rows},{vocab}] {dtype}")


def test_chain_4x256x32000_matches_oracle() -> None:
    """fp32 [4, 256, 32000] stats -> refine, S=32 slots, thought t=0.3."""
    ids, logits = cases.display_f32_4x256x32000()
    conf, pred, cur = torch.ops.cid_engine.display_token_statistics(ids.cuda(), logits.cuda())
    _check_stats((conf, pred, cur), ids, logits, "4x256x32000 stats")
    refined = torch.ops.cid_engine.refine_display_from_statistics(
        ids.cuda(), conf, pred, cur, 0, 1, 0.25, 0.1, 0.05)
    expected = oracle.refine_display_from_statistics(ids, conf.cpu(), pred.cpu(), cur.cpu(),
                                                     0, 1, 0.25, 0.1, 0.05)
    assert torch.equal(refined.cpu(), expected)
    g = torch.Generator().manual_seed(10)
    occ = (torch.rand(4, 32, 1, generator=g) < 0.4).float()
    life = torch.zeros(4, 32, 4)
    life[..., 3] = (torch.rand(4, 32, generator=g) < 0.1).float()
    live = torch.ops.cid_engine.live_slot_occupancy(occ.cuda(), life.cuda(), 3)
    assert torch.equal(live.cpu(), oracle.live_slot_occupancy(occ, life, 3))
    th = cases.thought_4x32x512()
    got = torch.ops.cid_engine.thought_corrupt_from_epsilon(*[t.cuda() for t in th])
    compare.assert_matches("thought_corrupt_from_epsilon", got,
                           oracle.thought_corrupt_from_epsilon(*th), "4x32x512 thought")


def test_masked_diffusion_64x2048_deterministic() -> None:
    args = list(cases.masked_diffusion_64x2048())
    dev_args = [a.cuda() if isinstance(a, torch.Tensor) else a for a in args]
    out1 = torch.ops.cid_engine.masked_diffusion_corrupt_from_random(*dev_args)
    out2 = torch.ops.cid_engine.masked_diffusion_corrupt_from_random(*dev_args)
    for a, b in zip(out1, out2):
        assert torch.equal(a, b)  # fixed-order metrics: bit-identical
    compare.assert_matches("masked_diffusion_corrupt_from_random", out1,
                           oracle.masked_diffusion_corrupt_from_random(*args), "64x2048")
    assert bool(out1[1].any(dim=1).all())  # zero-ratio rows took the fallback


@pytest.mark.parametrize("batch,tokens", [(3000, 100), (1, 9000), (7, 33)])
def test_masked_diffusion_row_shapes_match_oracle(batch: int, tokens: int) -> None:
    """Masked diffusion with many short rows (3000 rows: more CTAs than the
    device holds at once, and the metrics kernel's loop over rows), one long
    row (several loads batches per thread) and rows shorter than a CTA; a
    third of the rows take the empty-row fallback."""
    g = torch.Generator().manual_seed(batch + tokens)
    clean = torch.randint(0, 50257, (batch, tokens), generator=g)
    rr = torch.rand(batch, 1, generator=g)
    rr[::3] = 0.0
    mr = torch.rand(batch, tokens, generator=g)
    args = (clean, rr, mr, 50256, 1e-6, 1.0)
    dev = [a.cuda() if isinstance(a, torch.Tensor) else a for a in args]
    out1 = torch.ops.cid_engine.masked_diffusion_corrupt_from_random(*dev)
    out2 = torch.ops.cid_engine.masked_diffusion_corrupt_from_random(*dev)
    for a, b in zip(out1, out2):
        assert torch.equal(a, b)
    compare.assert_matches("masked_diffusion_corrupt_from_random", out1,
                           oracle.masked_diffusion_corrupt_from_random(*args),
                           f"masked diffusion [{batch},{tokens}]")


def _graph_kernel_nodes(graph) -> int:
    """Kernel nodes of a captured torch.cuda.CUDAGraph(keep_graph=True)."""
    import ctypes

    cu = ctypes.CDLL("libcuda.so.1")
    handle = ctypes.c_void_p(graph.raw_cuda_graph())
    n = ctypes.c_size_t(0)
    assert cu.cuGraphGetNodes(handle, None, ctypes.byref(n)) == 0
    nodes = (ctypes.c_void_p * n.value)()
    assert cu.cuGraphGetNodes(handle, nodes, ctypes.byref(n)) == 0
    kinds = []
    for node in nodes:
        kind = ctypes.c_int(-1)
        assert cu.cuGraphNodeGetType(ctypes.c_void_p(node), ctypes.byref(kind)) == 0
        kinds.append(kind.value)
    assert all(k == 0 for k in kinds), kinds  # CU_GRAPH_NODE_TYPE_KERNEL only
    return len(kinds)


def test_masked_diffusion_in_a_graph_is_one_kernel_and_matches_eager() -> None:
    """Captured into a CUDA graph, each masked-diffusion call is one kernel
    whose last row writes the metrics; its slot is cleared after each run,
    so replays over new inputs must equal eager calls (two kernels) bit for
    bit and the oracle.  Shapes: ratios summed by every row (64 rows of 2048),
    by the last row alone (300 rows), 512-thread rows (8 rows of 9000), and
    a single short row; a third of the rows take the empty-row fallback."""
    shapes = [(64, 2048), (300, 100), (8, 9000), (1, 33)]
    gen = torch.Generator().manual_seed(11)

    def fresh(batch, tokens):
        clean = torch.randint(0, 50257, (batch, tokens), generator=gen)
        rr = torch.rand(batch, 1, generator=gen)
        rr[::3] = 0.0
        return clean, rr, torch.rand(batch, tokens, generator=gen)

    static = [[t.cuda() for t in fresh(b, t)] for b, t in shapes]
    md = torch.ops.cid_engine.masked_diffusion_corrupt_from_random
    for clean, rr, mr in static:  # eager first: the one-kernel form needs it
        md(clean, rr, mr, 50256, 1e-6, 1.0)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph(keep_graph=True)
    with torch.cuda.graph(graph):
        outs = [md(clean, rr, mr, 50256, 1e-6, 1.0) for clean, rr, mr in static]
    assert _graph_kernel_nodes(graph) == len(shapes)
    for rep in range(3):
        if rep:
            for (b, t), dst in zip(shapes, static):
                for d, s in zip(dst, fresh(b, t)):
                    d.copy_(s)
        graph.replay()
        torch.cuda.synchronize()
        for (b, t), (clean, rr, mr), got in zip(shapes, static, outs):
            want = md(clean, rr, mr, 50256, 1e-6, 1.0)
            for x, y in zip(got, want):
                assert torch.equal(x, y), (rep, b, t)
            args = (clean.cpu(), rr.cpu(), mr.cpu(), 50256, 1e-6, 1.0)
            compare.assert_matches("masked_diffusion_corrupt_from_random", got,
                                   oracle.masked_diffusion_corrupt_from_random(*args),
                                   f"graph masked diffusion [{b},{t}] replay {rep}")
    del graph


@pytest.mark.parametrize("tokens", [512, 4096, 8192])
def test_refine_large_rows_match_oracle(tokens: int) -> None:
    """Decode-loop refine shape (B=256, L=512) plus long rows that exceed the
    shared-memory staging (global-memory path)."""
    batch = 256 if tokens == 512 else 4
    ids, (conf, pred, cur) = cases.refine_inputs_large(77 + tokens, batch, tokens)
    for reveal, revision, margin in ((0.25, 0.1, 0.05), (1.0, 1.0, 0.0)):
        got = torch.ops.cid_engine.refine_display_from_statistics(
            ids.cuda(), conf.cuda(), pred.cuda(), cur.cuda(), 0, 1, reveal, revision, margin)
        exp = oracle.refine_display_from_statistics(ids, conf, pred, cur, 0, 1, reveal,
                                                    revision, margin)
        assert torch.equal(got.cpu(), exp)


@pytest.mark.parametrize("world", [2, 3, 4, 8, 40, 200])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_vocab_sharded_records_equal_unsharded(world: int, dtype: torch.dtype) -> None:
    """Vocabulary sharding emulated on one GPU: records of each shard,
    combined, equal the unsharded statistics (past 32 shards the combine
    takes a warp per row)."""
    from cid_engine import parallel

    g = torch.Generator().manual_seed(world)
    V = 152064 if world in (2, 8) else 4099
    ids = torch.randint(V, (2, 40), generator=g)
    lg = (torch.randn(2, 40, V, generator=g) * 2).to(dtype)
    lg[0, 3, V - 1] = 40.0  # peak in the last shard
    lg[1, 7, [5, V // 2 + 3]] = 50.0  # exact cross-shard tie: lowest column wins
    lg[1, 9, 17] = float("nan")
    lg[0, 11, :] = float("-inf")
    lgd, idd = lg.cuda(), ids.cuda()
    offs = parallel.shard_offsets(V, world)
    recs = torch.stack([
        torch.ops.cid_engine.display_shard_records(idd, lgd[..., offs[r]:offs[r + 1]], offs[r], V)
        for r in range(world)
    ])
    got = torch.ops.cid_engine.display_combine_records(recs, idd, offs)
    unsharded = torch.ops.cid_engine.display_token_statistics(idd, lgd)
    assert torch.equal(got[1], unsharded[1])
    torch.testing.assert_close(got[0], unsharded[0], rtol=compare.STATS_RTOL, atol=compare.STATS_ATOL, equal_nan=True)
    torch.testing.assert_close(got[2], unsharded[2], rtol=compare.STATS_RTOL, atol=compare.STATS_ATOL, equal_nan=True)
    compare.assert_matches(STATS, got, oracle.display_token_statistics(ids, lg), "sharded")
    # the device records agree with the oracle's records
    orc = torch.stack([oracle.display_shard_records(ids, lg[..., offs[r]:offs[r + 1]], offs[r], V)
                       for r in range(world)])
    assert torch.equal(recs[..., 2].cpu(), orc[..., 2])  # argmax / NaN flag exact


def test_out_of_range_ids_set_status_and_nan() -> None:
    import cid_engine

    cid_engine.device_status(0, reset=True)
    ids = torch.tensor([[3, 99, -1]], device="cuda")
    lg = torch.randn(1, 3, 16, device="cuda")
    conf, pred, cur = cid_engine.display_token_statistics(ids, lg)
    assert bool(torch.isnan(cur[0, 1:]).all()) and bool(torch.isfinite(cur[0, 0]))
    assert cid_engine.device_status(0) & cid_engine.STATUS_TOKEN_ID_OUT_OF_RANGE
    idx = torch.tensor([0, 40], device="cuda")
    snap = cid_engine.materialize_cell_snapshot(
        torch.randn(1, 2, 8, device="cuda"), torch.randn(1, 2, 3, device="cuda"),
        torch.rand(1, 2, 1, device="cuda"), torch.randn(1, 2, 1, device="cuda"),
        torch.randn(1, 2, 4, device="cuda"), torch.ones(1, 2, dtype=torch.bool, device="cuda"), idx)
    assert bool(torch.isnan(snap[..., -1]).all())
    assert cid_engine.device_status(0, reset=True) & cid_engine.STATUS_SEMANTIC_INDEX_OUT_OF_RANGE
    assert cid_engine.device_status(0) == 0


@pytest.mark.parametrize("kind", ["repetition", "records"])
@pytest.mark.parametrize("shape,dtype", [
    ((4, 256, 32000), torch.float32),     # 1024 rows: 128-thread CTAs (one wave)
    ((1, 256, 155136), torch.bfloat16),   # 310 KB a CTA: 512-thread CTAs
    ((1, 128, 155136), torch.float32),    # cluster of 2, 310 KB a CTA: 512 threads
    ((1, 32, 155136), torch.bfloat16),    # cluster of 8, 39 KB a CTA: 128 threads
])
def test_stats_block_sizes_match_oracle(kind, shape, dtype) -> None:
    """The repetition and vocabulary-shard record variants of the CTA kernel
    at the shapes whose launch picks 128- and 512-thread CTAs (with and
    without clusters), against the oracle; repeated ids make patches."""
    B, L, V = shape
    g = torch.Generator().manual_seed(B * L + V)
    lg = (torch.randn(B, L, V, generator=g) * 2).to(dtype)
    ids = torch.randint(V, (B, L), generator=g)
    ids[:, 1::4] = ids[:, 0::4]  # adjacent repeats
    lg[0, 2, V - 1] = 30.0
    ids[0, 3] = 0  # mask id
    if kind == "repetition":
        got = torch.ops.cid_engine.display_token_statistics_with_repetition(
            ids.cuda(), lg.cuda(), 0, 1, 0.7)
        exp = oracle.display_token_statistics_with_repetition(ids, lg, 0, 1, 0.7)
        compare.assert_matches("display_token_statistics_with_repetition", got, exp,
                               f"repetition {shape} {dtype}")
    else:
        half = V // 2
        got = torch.ops.cid_engine.display_shard_records(ids.cuda(), lg[..., half:].cuda(), half, V)
        exp = oracle.display_shard_records(ids, lg[..., half:], half, V)
        got = got.cpu().reshape(exp.shape)
        # int32 records: max, argmax | NaN flag and the current logit exactly,
        # the sum of exponentials (float32 bits) within the statistics tolerance
        assert torch.equal(got[:, [0, 2, 3]], exp[:, [0, 2, 3]])
        torch.testing.assert_close(got[:, 1].contiguous().view(torch.float32),
                                   exp[:, 1].contiguous().view(torch.float32),
                                   rtol=compare.STATS_RTOL, atol=compare.STATS_ATOL)


def test_repetition_long_runs() -> None:
    """Runs longer than a warp (the ballot scan loops) and runs touching the
    sequence ends."""
    ids = torch.full((2, 200), 7)
    ids[0, 100:] = 9
    ids[1, ::50] = 4
    g = torch.Generator().manual_seed(3)
    lg = torch.randn(2, 200, 64, generator=g) * 2
    lg[..., 7] += 6
    got = torch.ops.cid_engine.display_token_statistics_with_repetition(ids.cuda(), lg.cuda(), 0, 1, 0.9)
    exp = oracle.display_token_statistics_with_repetition(ids, lg, 0, 1, 0.9)
    compare.assert_matches("display_token_statistics_with_repetition", got, exp, "long runs")


@pytest.mark.parametrize("rows_per_seq,seqs,V", [(64, 2, 4099), (1000, 12, 4099), (8, 2, 152063)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_repetition_patch_moves_row_maximum(rows_per_seq, seqs, V, dtype) -> None:
    """Every position's right neighbour holds that position's argmax column,
    so the patch lowers the row maximum (the argmax moves, or ties with the
    runner-up: the planted runner-up equals the patched maximum); 128 rows
    run one CTA per row, 12000 rows one warp per row, 16 rows of 152063 a
    cluster of CTAs per row (each CTA streams a slice of the row).  Odd
    vocabularies: unaligned row starts, head and tail columns."""
    g = torch.Generator().manual_seed(41)
    lg = (torch.randn(seqs, rows_per_seq, V, generator=g) * 2).to(dtype).float()
    top = lg.argmax(-1)
    ids = torch.roll(top, 1, dims=1)  # ids[p + 1] = argmax of row p
    ids[:, ::7] = 0  # mask ids (no patch from these)
    mult = 0.5
    # runner-up at a later column equal to the patched maximum on every third row
    flat = lg.view(-1, V)
    right = torch.roll(ids, -1, dims=1).view(-1)  # the right neighbour's id of each row
    patched_max = flat.gather(1, top.view(-1, 1)).squeeze(1) + torch.log(torch.tensor(mult))
    for r in range(0, flat.shape[0], 3):
        if int(right[r]) == int(top.view(-1)[r]) and int(right[r]) > 1:
            c = (int(top.view(-1)[r]) + 1 + r) % V
            flat[r, c] = patched_max[r]
    lg = lg.to(dtype)
    got = torch.ops.cid_engine.display_token_statistics_with_repetition(ids.cuda(), lg.cuda(), 0, 1, mult)
    exp = oracle.display_token_statistics_with_repetition(ids, lg, 0, 1, mult)
    compare.assert_matches("display_token_statistics_with_repetition", got, exp,
                           f"patch at maximum {rows_per_seq}x{seqs} {dtype}")


def test_unaligned_and_strided_rows() -> None:
    """Row strides that break 16-byte alignment (odd vocab, sliced views)."""
    g = torch.Generator().manual_seed(5)
    base = torch.randn(3, 50, 4099, generator=g).to(torch.bfloat16)
    view = base[:, :, 1:4098]  # unaligned start, row stride 4099
    ids = torch.randint(4097, (3, 50), generator=g)
    got = torch.ops.cid_engine.display_token_statistics(ids.cuda(), base.cuda()[:, :, 1:4098])
    _check_stats(got, ids, view, "strided")


def test_fused_step_chain_runs_without_host_sync() -> None:
    from cid_engine.step import SlotInputs, refine_step

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1)
    B, L, V, S = 4, 64, 1000, 16
    ids = torch.randint(2, V, (B, L), generator=g, device=dev)
    lg = torch.randn(B, L, V, generator=g, device=dev)
    slots = SlotInputs(
        occupancy=(torch.rand(B, S, 1, generator=g, device=dev) < 0.4).float(),
        allocation_logits=torch.randn(B, S, generator=g, device=dev),
        lifecycle_logits=torch.randn(B, S, 4, generator=g, device=dev),
        revision_logits=torch.randn(B, S, 3, generator=g, device=dev),
        input_lifecycle=torch.randn(B, S, 4, generator=g, device=dev),
        semantic=torch.randn(B, S, 32, generator=g, device=dev),
        role_logits=torch.randn(B, S, 6, generator=g, device=dev),
        uncertainty=torch.rand(B, S, 1, generator=g, device=dev),
        noise_delta=torch.randn(B, S, 1, generator=g, device=dev),
        semantic_indices=torch.tensor([0, 5, 31], device=dev),
    )
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        out = refine_step(ids, lg, mask_token_id=0, eos_token_id=1, reveal_fraction=0.5,
                          revision_fraction=0.2, revision_margin=0.0, slots=slots)
    stream.synchronize()
    c, p, u = oracle.display_token_statistics(ids, lg)
    assert torch.equal(out.token_ids.cpu(),
                       oracle.refine_display_from_statistics(ids, c, p, u, 0, 1, 0.5, 0.2, 0.0))
    roll = oracle.rollout_slot_transition(slots.occupancy, slots.allocation_logits,
                                          slots.lifecycle_logits, slots.revision_logits,
                                          slots.input_lifecycle, 0.5, 8, 3)
    for a, b in zip(out.rollout, roll):
        assert torch.equal(a.cpu(), b)
    snap = oracle.materialize_cell_snapshot(slots.semantic, slots.role_logits, slots.uncertainty,
                                            slots.noise_delta, slots.lifecycle_logits, roll[5],
                                            slots.semantic_indices)
    torch.testing.assert_close(out.snapshot.cpu(), snap, rtol=2.5e-7, atol=1e-12)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible CUDA devices")
def test_tensor_device_not_current_device() -> None:
    """reference tests/test_cuda.py:371-389: ops run on the tensors' device."""
    import cid_engine

    cur = torch.cuda.current_device()
    dev = torch.device("cuda", 1 if cur == 0 else 0)
    occ = torch.tensor([[0.0, 0.0, 1.0, 0.0]], device=dev)
    lg = torch.tensor([[8.0, 7.0, -5.0, 6.0]], device=dev)
    out = cid_engine.prefix_allocation_mask(occ, lg, threshold=0.5, max_allocations=2)
    assert out.device == dev and torch.cuda.current_device() == cur
    assert torch.equal(out.cpu(), oracle.prefix_allocation_mask(occ, lg, 0.5, 2))


def test_assignment_invalid_rows_and_nonfinite_costs_do_not_hang() -> None:
    """Row counts outside [0, rows] and NaN costs (on which a sequential
    Hungarian search never ends) leave -1 and set the status bit."""
    import cid_engine

    cid_engine.device_status(0, reset=True)
    out = cid_engine.batched_linear_assignment(torch.rand(2, 3, 4, device="cuda"),
                                               torch.tensor([5, 2], device="cuda"))
    assert bool((out[0] == -1).all()) and bool((out[1, :2] >= 0).all())
    assert cid_engine.device_status(0, reset=True) & cid_engine.STATUS_ASSIGNMENT_INVALID
    nan_costs = torch.full((1, 2, 2), float("nan"), device="cuda")
    out = cid_engine.batched_linear_assignment(nan_costs, torch.tensor([2], device="cuda"))
    assert bool((out == -1).all())
    assert cid_engine.device_status(0, reset=True) & cid_engine.STATUS_ASSIGNMENT_INVALID


def test_c_abi_known_answers(tmp_path) -> None:
    """The reference's C++ KATs, a peer-exchange round and an exact LM-head
    case through the C ABI from plain C."""
    import subprocess
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    lib_dir = root / "cid-engine_b200" / "cid_engine"
    exe = tmp_path / "capi_kats"
    subprocess.run(
        ["gcc", "-O1", "-o", str(exe), str(root / "tests" / "cpp" / "capi_kats.c"),
         f"-I{root / 'include'}", "-I/usr/local/cuda/include", f"-L{lib_dir}",
         "-l:libcid_engine_b200.so", f"-Wl,-rpath,{lib_dir}", "-L/usr/local/cuda/lib64",
         "-lcudart", "-Wl,-rpath,/usr/local/cuda/lib64", "-lm"],
        check=True,
    )
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr
    assert "passed" in res.stdout
