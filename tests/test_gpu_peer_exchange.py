"""The peer record exchange (``cid_engine.parallel.PeerRecordExchange``) on
one GPU: a one-rank exchange equals the record + combine path bit for bit
over consecutive steps (both epoch parities), and a combine whose epoch no
rank publishes gives up after its wait limit with a status bit and NaN
statistics instead of hanging; from then on the exchange is poisoned (NaN at
once, no wait) until the status word is cleared, and a flag two epochs ahead
(a peer that moved on) is refused with its own bit.  The multi-rank exchange
over NVLink is checked in ``test_multi_gpu.py``."""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _engine():
    import cid_engine  # noqa: F401

    assert torch.cuda.is_available()
    torch.cuda.set_device(0)
    yield
    torch.cuda.empty_cache()


def _same(a, b):
    torch.testing.assert_close(a, b, rtol=0, atol=0, equal_nan=True)


def test_one_rank_exchange_equals_records_and_combine() -> None:
    import cid_engine
    from cid_engine import parallel

    dev = torch.device("cuda", 0)
    B, L, V = 3, 70, 5003
    ex = parallel.PeerRecordExchange(B * L + 7)
    try:
        for step in range(3):
            g = torch.Generator(device=dev).manual_seed(step)
            logits = (torch.randn(B, L, V, generator=g, device=dev) * 3).to(torch.bfloat16)
            logits[1, 4, [3, V - 1]] = 30.0  # tie: the lower column
            logits[2, 9, 100] = float("nan")
            ids = torch.randint(V, (B, L), generator=g, device=dev)
            ids[0, 0] = V + 3  # outside the vocabulary
            got = ex.statistics(ids, logits, vocab_offset=0, total_vocab=V, shard_offsets=[0, V])
            rec = cid_engine.display_shard_records(ids, logits, vocab_offset=0, total_vocab=V)
            exp = cid_engine.display_combine_records(rec.view(1, B * L, 4), ids, [0, V])
            for a, e in zip(got, exp):
                _same(a, e)
        assert ex.epoch == 3
    finally:
        ex.close()


def test_unpublished_epoch_times_out_with_status() -> None:
    """A flag that nothing sets: the combine waits 0.2 s, then reports."""
    import cid_engine
    from cid_engine import parallel

    dev = torch.device("cuda", 0)
    B, L, V = 2, 40, 997
    ex = parallel.PeerRecordExchange(B * L)
    try:
        g = torch.Generator(device=dev).manual_seed(5)
        logits = torch.randn(B, L, V, generator=g, device=dev)
        ids = torch.randint(V, (B, L), generator=g, device=dev)
        ex.statistics(ids, logits, vocab_offset=0, total_vocab=V, shard_offsets=[0, V])
        torch.cuda.synchronize()
        cid_engine.device_status(0, reset=True)
        conf = torch.empty(B, L, device=dev)
        pred = torch.empty(B, L, dtype=torch.int64, device=dev)
        cur = torch.empty(B, L, device=dev)
        offs = (ctypes.c_int64 * 2)(0, V)
        rc = ex.lib.cid_display_combine_inbox(
            ex.own, 1, offs, ids.data_ptr(), B * L, B * L, ex.epoch + 2, 0.2, conf.data_ptr(),
            pred.data_ptr(), cur.data_ptr(), cid_engine._C.status_word_ptr(0),
            torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert cid_engine.device_status(0) & cid_engine.STATUS_PEER_TIMEOUT
        assert bool(conf.isnan().all()) and bool(cur.isnan().all()) and bool((pred == 0).all())
        # while the bit is set the exchange is poisoned: the next step
        # writes NaN at once, without waiting
        assert not ex.healthy()
        got = ex.statistics(ids, logits, vocab_offset=0, total_vocab=V, shard_offsets=[0, V])
        torch.cuda.synchronize()
        assert bool(got[0].isnan().all()) and bool((got[1] == 0).all())
        cid_engine.device_status(0, reset=True)
        # with the word cleared (one rank: no peer can be out of step) the
        # exchange serves again
        assert ex.healthy()
        got = ex.statistics(ids, logits, vocab_offset=0, total_vocab=V, shard_offsets=[0, V])
        exp = cid_engine.display_token_statistics(ids, logits)
        assert torch.equal(got[1], exp[1])
        torch.cuda.synchronize()
        assert cid_engine.device_status(0) == 0
    finally:
        ex.close()


def test_peer_out_of_step_sets_its_bit() -> None:
    """A flag two epochs ahead of the combine's epoch (a peer that gave up
    waiting and moved on) is refused at once: NaN statistics and
    STATUS_PEER_OUT_OF_STEP, no wait."""
    import ctypes

    import cid_engine
    from cid_engine import parallel

    dev = torch.device("cuda", 0)
    B, L, V = 1, 64, 512
    ex = parallel.PeerRecordExchange(B * L)
    try:
        g = torch.Generator(device=dev).manual_seed(6)
        logits = torch.randn(B, L, V, generator=g, device=dev)
        ids = torch.randint(V, (B, L), generator=g, device=dev)
        for _ in range(3):
            ex.statistics(ids, logits, vocab_offset=0, total_vocab=V, shard_offsets=[0, V])
        torch.cuda.synchronize()
        cid_engine.device_status(0, reset=True)
        conf = torch.empty(B, L, device=dev)
        pred = torch.empty(B, L, dtype=torch.int64, device=dev)
        cur = torch.empty(B, L, device=dev)
        offs = (ctypes.c_int64 * 2)(0, V)
        rc = ex.lib.cid_display_combine_inbox(
            ex.own, 1, offs, ids.data_ptr(), B * L, B * L, ex.epoch - 2, 1.0, conf.data_ptr(),
            pred.data_ptr(), cur.data_ptr(), cid_engine._C.status_word_ptr(0),
            torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        st = cid_engine.device_status(0, reset=True)
        assert st & cid_engine.STATUS_PEER_OUT_OF_STEP
        assert not st & cid_engine.STATUS_PEER_TIMEOUT
        assert bool(conf.isnan().all()) and bool((pred == 0).all())
        with pytest.raises(ValueError, match="wait_seconds"):
            parallel.PeerRecordExchange(4, wait_seconds=120.0)
    finally:
        ex.close()


def test_exchange_validation() -> None:
    from cid_engine import parallel

    dev = torch.device("cuda", 0)
    ex = parallel.PeerRecordExchange(10)
    try:
        ids = torch.zeros(2, 8, dtype=torch.int64, device=dev)
        lg = torch.zeros(2, 8, 16, device=dev)
        with pytest.raises(ValueError, match="capacity"):
            ex.statistics(ids, lg, vocab_offset=0, total_vocab=16, shard_offsets=[0, 16])
    finally:
        ex.close()


def test_one_rank_exchange_from_lm_head_records() -> None:
    """Records from the fused LM head through the exchange equal the fused
    LM head's statistics (argmax exact; sums regrouped, rtol 1e-5)."""
    import cid_engine
    from cid_engine import parallel

    dev = torch.device("cuda", 0)
    R, V, H = 200, 9001, 128
    g = torch.Generator(device=dev).manual_seed(8)
    hid = (torch.randn(R, H, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    wgt = (torch.randn(V, H, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    ids = torch.randint(V, (R,), generator=g, device=dev)
    ex = parallel.PeerRecordExchange(R)
    try:
        rec = cid_engine.lm_head_shard_records(ids, hid, wgt, vocab_offset=0, total_vocab=V)
        c, p, u = ex.from_records(rec, ids, shard_offsets=[0, V])
        e_c, e_p, e_u = cid_engine.lm_head_display_statistics(ids, hid, wgt)
        assert torch.equal(p, e_p)
        torch.testing.assert_close(c, e_c, rtol=1e-5, atol=1e-30)
        torch.testing.assert_close(u, e_u, rtol=1e-5, atol=1e-30)
    finally:
        ex.close()


@pytest.mark.parametrize("world", [2, 3, 8])
def test_emulated_ranks_store_records_into_every_inbox(world: int) -> None:
    """``world`` ranks emulated on one GPU: one inbox each, every rank's
    record launch (``cid_display_shard_records_to_peers``) stores each record
    into every inbox as it finishes the row, then publishes; every rank's
    combine must equal the records + combine path bit for bit, over three
    steps (both epoch parities).  All launches go to one stream in rank
    order, so every flag is published before any combine reads it (no kernel
    waits on another that runs at the same time)."""
    import cid_engine
    from cid_engine import parallel

    lib = parallel._capi()
    dev = torch.device("cuda", 0)
    B, L, V = 2, 150, 20011
    rows = B * L
    offs = parallel.shard_offsets(V, world)
    stream = torch.cuda.current_stream().cuda_stream
    status = cid_engine._C.status_word_ptr(0)
    cid_engine.device_status(0, reset=True)
    nbytes = lib.cid_peer_inbox_bytes(world, rows)
    inboxes = []
    try:
        for _ in range(world):
            p = ctypes.c_void_p()
            assert lib.cid_peer_inbox_alloc(nbytes, ctypes.byref(p)) == 0
            inboxes.append(p.value)
        table = (ctypes.c_void_p * world)(*inboxes)
        c_offs = (ctypes.c_int64 * (world + 1))(*offs)
        for epoch in (1, 2, 3):
            g = torch.Generator(device=dev).manual_seed(40 + epoch)
            logits = (torch.randn(B, L, V, generator=g, device=dev) * 3).to(torch.bfloat16)
            logits[0, 7, [offs[1] - 1, offs[1]]] = 40.0  # tie across a shard edge: the lower
            logits[1, 3, offs[-2] + 5] = float("nan")
            ids = torch.randint(V, (B, L), generator=g, device=dev)
            shards = [logits[..., offs[r]:offs[r + 1]].contiguous() for r in range(world)]
            for r in range(world):
                rc = lib.cid_display_shard_records_to_peers(
                    3, shards[r].data_ptr(), offs[r + 1] - offs[r], ids.data_ptr(), rows,
                    offs[r + 1] - offs[r], offs[r], V, r, world, table, rows, epoch, status,
                    stream)
                assert rc == 0
            rec = torch.stack([cid_engine.display_shard_records(ids, shards[r], vocab_offset=offs[r],
                                                               total_vocab=V)
                               for r in range(world)])
            exp = cid_engine.display_combine_records(rec, ids, offs)
            for r in range(world):
                got = [torch.empty(B, L, device=dev), torch.empty(B, L, dtype=torch.int64, device=dev),
                       torch.empty(B, L, device=dev)]
                rc = lib.cid_display_combine_inbox(
                    inboxes[r], world, c_offs, ids.data_ptr(), rows, rows, epoch, 1.0,
                    got[0].data_ptr(), got[1].data_ptr(), got[2].data_ptr(), status, stream)
                assert rc == 0
                for a, e in zip(got, exp):
                    _same(a, e)
            assert int(exp[1][0, 7]) == offs[1] - 1 and int(exp[1][1, 3]) == offs[-2] + 5
        torch.cuda.synchronize()
        assert cid_engine.device_status(0) == 0
    finally:
        torch.cuda.synchronize()
        for p in inboxes:
            lib.cid_peer_inbox_free(p)
