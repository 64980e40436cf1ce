"""Vocabulary-parallel statistics over NCCL on 2+ GPUs of one node.

Each rank holds one contiguous vocabulary shard of the same seeded logits;
``cid_engine.parallel.vocab_parallel_statistics`` (device records -> NCCL
all-gather -> device combine) must equal the unsharded statistics computed
on one GPU: argmax exactly, confidences within the statistics tolerance.
Ranks run as spawned child processes with NVLS off and a short process-group
timeout.
"""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, result_dir: str) -> None:
    for p in (ROOT, ROOT / "tests" / "golden", ROOT / "cid-engine_b200"):
        sys.path.insert(0, str(p))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    import cid_engine
    import compare
    from cid_engine import parallel

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        for V, dtype in ((50021, torch.bfloat16), (152064, torch.bfloat16), (9001, torch.float32)):
            g = torch.Generator(device=dev).manual_seed(V)
            logits = (torch.randn(2, 96, V, generator=g, device=dev) * 2).to(dtype)
            logits[0, 5, V - 3] = 30.0
            logits[1, 9, [1, V - 2]] = 40.0  # cross-shard tie: lowest column wins
            logits[1, 10, V // 2] = float("nan")
            ids = torch.randint(V, (2, 96), generator=g, device=dev)
            offs = parallel.shard_offsets(V, world)
            shard = logits[..., offs[rank]:offs[rank + 1]].contiguous()
            conf, pred, cur = parallel.vocab_parallel_statistics(ids, shard, total_vocab=V)
            e_conf, e_pred, e_cur = cid_engine.display_token_statistics(ids, logits)
            assert torch.equal(pred, e_pred)
            torch.testing.assert_close(conf, e_conf, rtol=compare.STATS_RTOL, atol=compare.STATS_ATOL, equal_nan=True)
            torch.testing.assert_close(cur, e_cur, rtol=compare.STATS_RTOL, atol=compare.STATS_ATOL, equal_nan=True)
        # the vocabulary-parallel workload's row width, 4096 rows: records
        # through the peer exchange == the unsharded statistics, and rank 0's
        # rows against the oracle
        V = 152064
        g = torch.Generator(device=dev).manual_seed(3)
        logits = (torch.randn(4, 1024, V, generator=g, device=dev) * 2).to(torch.bfloat16)
        flat = logits.view(-1, V)
        peak = torch.nonzero(torch.rand(4096, generator=g, device=dev) < 0.05).flatten()
        col = torch.randint(V, (peak.numel(),), generator=g, device=dev)
        flat[peak, col] = (flat[peak, col].float() + 8.0).to(torch.bfloat16)
        ids = torch.randint(V, (4, 1024), generator=g, device=dev)
        offs = parallel.shard_offsets(V, world)
        shard = logits[..., offs[rank]:offs[rank + 1]].contiguous()
        ex = parallel.PeerRecordExchange(4 * 1024)
        try:
            conf, pred, cur = ex.statistics(ids, shard, vocab_offset=offs[rank], total_vocab=V,
                                            shard_offsets=offs)
        finally:
            ex.close()
        e_conf, e_pred, e_cur = cid_engine.display_token_statistics(ids, logits)
        assert torch.equal(pred, e_pred)
        compare.assert_stats_close(conf, e_conf, "sharded [4,1024,152064] conf")
        compare.assert_stats_close(cur, e_cur, "sharded [4,1024,152064] cur")
        if rank == 0:
            from oracle import oracle

            sel = torch.arange(0, 4096, 64, device=dev)
            o_conf, o_pred, o_cur = oracle.display_token_statistics(
                ids.view(-1)[sel].view(1, -1), flat[sel].view(1, -1, V))
            assert torch.equal(pred.view(-1)[sel].cpu(), o_pred.view(-1))
            compare.assert_stats_close(conf.view(-1)[sel], o_conf.view(-1), "vs oracle conf")
            compare.assert_stats_close(cur.view(-1)[sel], o_cur.view(-1), "vs oracle cur")
        del logits, flat, shard
        torch.cuda.empty_cache()
        # the fused vocabulary-parallel step == statistics then refinement
        V = 50021
        g = torch.Generator(device=dev).manual_seed(7)
        logits = (torch.randn(5, 64, V, generator=g, device=dev) * 3).to(torch.bfloat16)
        ids = torch.randint(2, V, (5, 64), generator=g, device=dev)
        ids[torch.rand((5, 64), generator=g, device=dev) < 0.6] = 0
        ids[:, 40] = 1
        offs = parallel.shard_offsets(V, world)
        shard = logits[..., offs[rank]:offs[rank + 1]].contiguous()
        kw = dict(mask_token_id=0, eos_token_id=1, reveal_fraction=0.25, revision_fraction=0.1,
                  revision_margin=0.05)
        c, p, u = parallel.vocab_parallel_statistics(ids, shard, total_vocab=V)
        expected = cid_engine.refine_display_from_statistics(ids, c, p, u, **kw)
        got = parallel.vocab_parallel_refine(ids, shard, total_vocab=V, **kw)
        assert torch.equal(got, expected)
        # records stored into every rank's inbox by the statistics kernel (no
        # collective) == the NCCL all-gather path, bit for bit, over steps of
        # both epoch parities
        ex = parallel.PeerRecordExchange(2 * 96, wait_seconds=10.0)
        try:
            for step in range(3):
                V = 60013
                g = torch.Generator(device=dev).manual_seed(100 + step)
                logits = (torch.randn(2, 96, V, generator=g, device=dev) * 2).to(torch.bfloat16)
                logits[1, 9, [1, V - 2]] = 40.0
                ids = torch.randint(V, (2, 96), generator=g, device=dev)
                offs = parallel.shard_offsets(V, world)
                shard = logits[..., offs[rank]:offs[rank + 1]].contiguous()
                got = ex.statistics(ids, shard, vocab_offset=offs[rank], total_vocab=V,
                                    shard_offsets=offs)
                exp = parallel.vocab_parallel_statistics(ids, shard, total_vocab=V)
                for a, e in zip(got, exp):
                    torch.testing.assert_close(a, e, rtol=0, atol=0, equal_nan=True)
            torch.cuda.synchronize()
            assert cid_engine.device_status(rank) == 0
        finally:
            ex.close()
        # failure detection without a fault: the other ranks leave between steps
        # (nothing of theirs in flight) and skip step 2; rank 0's combine waits
        # out its limit, reports STATUS_PEER_TIMEOUT and leaves NaN statistics;
        # the ranks then meet on the host and close
        ex = parallel.PeerRecordExchange(2 * 96, wait_seconds=0.5)
        try:
            V = 60013
            g = torch.Generator(device=dev).manual_seed(200)
            logits = (torch.randn(2, 96, V, generator=g, device=dev) * 2).to(torch.bfloat16)
            ids = torch.randint(V, (2, 96), generator=g, device=dev)
            offs = parallel.shard_offsets(V, world)
            shard = logits[..., offs[rank]:offs[rank + 1]].contiguous()
            kw2 = dict(vocab_offset=offs[rank], total_vocab=V, shard_offsets=offs)
            ok = ex.statistics(ids, shard, **kw2)
            torch.cuda.synchronize()
            assert cid_engine.device_status(rank, reset=True) == 0
            assert not bool(ok[0].isnan().all())
            if rank == 0:
                lost = ex.statistics(ids, shard, **kw2)
                torch.cuda.synchronize()
                assert cid_engine.device_status(rank, reset=True) & cid_engine.STATUS_PEER_TIMEOUT
                assert bool(lost[0].isnan().all()) and bool((lost[1] == 0).all())
        finally:
            ex.close()  # host barrier: every rank is between steps
        # vocabulary-parallel LM head: weight rows sharded, logits never written
        V, H = 32003, 128
        g = torch.Generator(device=dev).manual_seed(11)
        hid = (torch.randn(3, 40, H, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        wgt = (torch.randn(V, H, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        lids = torch.randint(0, V, (3, 40), generator=g, device=dev)
        offs = parallel.shard_offsets(V, world)
        w_shard = wgt[offs[rank]:offs[rank + 1]].contiguous()
        c, p, u = parallel.vocab_parallel_lm_head_statistics(lids, hid, w_shard, total_vocab=V)
        e_c, e_p, e_u = cid_engine.lm_head_display_statistics(lids, hid, wgt)
        assert torch.equal(p, e_p)
        torch.testing.assert_close(c, e_c, rtol=1e-5, atol=1e-30)
        torch.testing.assert_close(u, e_u, rtol=1e-5, atol=1e-30)
        # the same through the peer exchange: bit for bit the NCCL result
        ex = parallel.PeerRecordExchange(3 * 40, wait_seconds=10.0)
        try:
            for _ in range(2):
                pc, pp, pu = parallel.vocab_parallel_lm_head_statistics(
                    lids, hid, w_shard, total_vocab=V, exchange=ex)
                for x, y in ((pc, c), (pp, p), (pu, u)):
                    torch.testing.assert_close(x, y, rtol=0, atol=0, equal_nan=True)
        finally:
            ex.close()
        torch.cuda.synchronize()
        Path(result_dir, f"ok{rank}").write_text("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible CUDA devices")
def test_vocab_parallel_statistics_over_nccl(tmp_path) -> None:
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    assert sorted(p.name for p in tmp_path.iterdir()) == [f"ok{r}" for r in range(world)]
