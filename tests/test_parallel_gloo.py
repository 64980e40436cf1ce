"""Vocabulary-parallel statistics on CPU ranks (gloo, world size 2 and 3).

Each rank holds one contiguous vocabulary shard, reduces it to 16-byte row
records (here with the oracle, since the product kernels need a GPU), the
records are all-gathered by ``cid_engine.parallel.gather_records`` — the same
orchestration code the NCCL path runs — and merged; the result must equal the
unsharded statistics (argmax exactly).  Failure handling is exercised on the
host: a rank that raises before the collective makes the surviving rank's
collective fail within the process group's timeout instead of hanging.
"""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup_paths() -> None:
    for p in (ROOT, ROOT / "tests" / "golden", ROOT / "cid-engine_b200"):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))


def _worker(rank: int, world: int, port: int, dtype_name: str, result_dir: str) -> None:
    _setup_paths()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        import cases
        import compare
        from cid_engine import parallel
        from oracle import oracle

        dtype = getattr(torch, dtype_name)
        ids, logits = cases.special_rows(dtype)
        g = torch.Generator().manual_seed(3)
        extra = (torch.randn(2, 16, 301, generator=g) * 3).to(dtype)
        extra[0, 3, 150] = 50.0  # a peak in one shard
        extra[1, 5, [7, 290]] = 60.0  # an exact cross-shard tie: lowest column wins
        for lg, tid in ((logits, ids), (extra, torch.randint(301, (2, 16), generator=g))):
            V = lg.shape[-1]
            offs = parallel.shard_offsets(V, world)
            shard = lg[..., offs[rank]:offs[rank + 1]]
            rec = oracle.display_shard_records(tid, shard, offs[rank], V)
            gathered = parallel.gather_records(rec)
            assert gathered.shape == (world, tid.numel(), 4)
            c, p, u = oracle.display_combine_records(gathered, tid, offs)
            e = oracle.display_token_statistics(tid, lg)
            assert torch.equal(p, e[1])
            torch.testing.assert_close(c, e[0], rtol=compare.STATS_RTOL, atol=compare.STATS_ATOL, equal_nan=True)
            torch.testing.assert_close(u, e[2], rtol=compare.STATS_RTOL, atol=compare.STATS_ATOL, equal_nan=True)
        Path(result_dir, f"ok{rank}").write_text("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
def test_vocab_parallel_combine_on_gloo(world: int, dtype_name: str, tmp_path) -> None:
    mp.start_processes(_worker, args=(world, _free_port(), dtype_name, str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    assert sorted(p.name for p in tmp_path.iterdir()) == [f"ok{r}" for r in range(world)]


def _failing_worker(rank: int, world: int, port: int, result_dir: str) -> None:
    _setup_paths()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    from cid_engine import parallel

    if rank == 1:
        # this rank fails on the host before it joins the collective
        Path(result_dir, "rank1_failed").write_text("x")
        os._exit(3)
    try:
        parallel.gather_records(torch.zeros(4, 4, dtype=torch.int32))
    except Exception as exc:  # the survivor sees an error, not a hang
        Path(result_dir, "rank0_error").write_text(type(exc).__name__)
    os._exit(0)


def test_rank_failure_surfaces_as_error(tmp_path) -> None:
    ctx = mp.start_processes(_failing_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                             join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    names = sorted(p.name for p in tmp_path.iterdir())
    assert "rank1_failed" in names
    assert "rank0_error" in names
