"""Vocabulary-parallel display statistics over several GPUs of one node.

The display logits of a row are split by contiguous vocabulary ranges, one
range per rank (rank r owns columns [offsets[r], offsets[r+1])).  Each rank
reduces its shard to one 16-byte record per row — (max, sum exp(x - max),
global first argmax, current-token logit) — the records of all ranks are
all-gathered over NCCL (16 bytes x rows x world: a few MB, against GBs of
logits streamed per rank), and every rank merges them with the combine kernel
into the unsharded statistics: M = max_r m_r (lowest rank on ties, which
holds the lowest columns), S = sum_r s_r exp(m_r - M), confidence = 1/S,
current = exp(x_id - M)/S.  Every rank then holds identical statistics and
can run the refinement policy without a further collective.

NCCL has no user-defined reduction operator, so the "packed reduction" is
an all-gather of records followed by a deterministic device-side merge.
"""

from __future__ import annotations


import torch
import torch.distributed as dist
from torch import Tensor


def shard_offsets(total_vocab: int, world: int) -> list[int]:
    """Contiguous, balanced column ranges: rank r owns [o[r], o[r+1])."""
    return [r * total_vocab // world for r in range(world + 1)]


def gather_records(records: Tensor, group=None) -> Tensor:
    """All-gather ``[rows, 4]`` int32 records of every rank into a
    ``[world, rows, 4]`` tensor in rank order (NCCL on CUDA tensors, any
    backend on host tensors)."""
    world = dist.get_world_size(group)
    rows = records.shape[0]
    out = torch.empty((world * rows, *records.shape[1:]), dtype=records.dtype,
                      device=records.device)
    dist.all_gather_into_tensor(out, records.contiguous(), group=group)
    return out.view(world, rows, *records.shape[1:])


def vocab_parallel_statistics(token_ids: Tensor, logits_shard: Tensor, *, total_vocab: int,
                              group=None) -> tuple[Tensor, Tensor, Tensor]:
    """``display_token_statistics`` of logits sharded by vocabulary over the
    ranks of ``group`` (this rank's shard: ``logits_shard`` [B, L, V_r], the
    columns given by ``shard_offsets(total_vocab, world)[rank]``).  Returns
    the unsharded (confidence, predicted, current_confidence) on every rank."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    offs = shard_offsets(total_vocab, world)
    assert logits_shard.shape[-1] == offs[rank + 1] - offs[rank], "shard width mismatch"
    ops = torch.ops.cid_engine
    records = ops.display_shard_records(token_ids, logits_shard, offs[rank], total_vocab)
    gathered = gather_records(records, group)
    return ops.display_combine_records(gathered, token_ids, offs)


_DTYPE_CODES = {torch.float32: 0, torch.float64: 1, torch.float16: 2, torch.bfloat16: 3}


def _capi():
    """The C ABI library (loaded already by the torch extension), with the
    signatures of the peer-exchange entry points."""
    import ctypes
    from pathlib import Path

    lib = ctypes.CDLL(str(Path(__file__).resolve().parent / "libcid_engine_b200.so"))
    if not getattr(lib, "_peer_signatures", False):
        P, I64, I, U32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint32
        lib.cid_peer_inbox_bytes.restype = ctypes.c_size_t
        lib.cid_peer_inbox_bytes.argtypes = [I, I64]
        lib.cid_peer_inbox_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(P)]
        lib.cid_peer_inbox_free.argtypes = [P]
        lib.cid_peer_inbox_export.argtypes = [P, ctypes.c_char_p]
        lib.cid_peer_inbox_import.argtypes = [ctypes.c_char_p, ctypes.POINTER(P)]
        lib.cid_peer_inbox_release.argtypes = [P]
        lib.cid_display_shard_records_to_peers.argtypes = [
            I, P, I64, P, I64, I64, I64, I64, I, I, ctypes.POINTER(P), I64, U32, P, P]
        lib.cid_peer_push_records.argtypes = [P, I64, I, I, ctypes.POINTER(P), I64, U32, P]
        lib.cid_display_combine_inbox.argtypes = [
            P, I, ctypes.POINTER(I64), P, I64, I64, U32, ctypes.c_double, P, P, P, P, P]
        lib.cid_result_string.restype = ctypes.c_char_p
        lib.cid_last_cuda_error.restype = ctypes.c_char_p
        lib._peer_signatures = True
    return lib


def _check(lib, rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"cid_engine.{what}: {lib.cid_result_string(rc).decode()} "
                           f"({lib.cid_last_cuda_error().decode()})")


class PeerRecordExchange:
    """Vocabulary-parallel statistics whose record exchange is fused into the
    statistics kernel over peer memory: no collective in the step.

    At set-up every rank allocates one inbox (``rows_capacity`` rows, two
    epoch parities), exports its CUDA IPC handle, receives the others' (one
    ``all_gather_object`` on the process group) and maps them (peer access
    over NVLink).  A step is two launches on the current stream: the record
    kernel stores each row's 16-byte record into every rank's inbox and
    publishes the step's epoch in every rank's flag word, and the combine
    kernel waits (bounded by ``wait_seconds``) until every rank has published
    the epoch in this rank's inbox, then merges.  Two parities make reuse
    safe: a rank starts step k+2 only after every rank's step-k combine.  A
    wait that runs out sets ``cid_engine.STATUS_PEER_TIMEOUT`` in the device
    status word and leaves NaN statistics.  That breaks the two-parity
    argument (the rank that gave up may overwrite a slower rank's slot), so
    from then on the exchange is poisoned on the device: a combine that finds
    a peer two epochs ahead sets ``STATUS_PEER_OUT_OF_STEP``, and every
    combine on a device whose status word holds either bit writes NaN without
    waiting.  ``healthy()`` reads the word (a host sync); after a failure the
    caller resets the word (``cid_engine.device_status(reset=True)``) and
    builds a new exchange on every rank.  Every rank must call ``statistics``
    the same number of times.  ``wait_seconds`` (at most 60) bounds each
    combine's wait."""

    def __init__(self, rows_capacity: int, *, group=None, wait_seconds: float = 2.0) -> None:
        import ctypes

        self.lib = _capi()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.capacity = int(rows_capacity)
        if not 0.0 < wait_seconds <= 60.0:
            raise ValueError("wait_seconds must be in (0, 60]")
        self.wait_seconds = float(wait_seconds)
        self.device = torch.device("cuda", torch.cuda.current_device())
        nbytes = self.lib.cid_peer_inbox_bytes(self.world, self.capacity)
        if nbytes == 0:
            raise ValueError("a peer exchange spans 1..8 ranks and a non-negative capacity")
        own = ctypes.c_void_p()
        _check(self.lib, self.lib.cid_peer_inbox_alloc(nbytes, ctypes.byref(own)), "peer_inbox")
        self.own = own.value
        handle = ctypes.create_string_buffer(64)
        _check(self.lib, self.lib.cid_peer_inbox_export(self.own, handle), "peer_inbox")
        handles = [handle.raw]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
        self.mapped = []
        ptrs = []
        for q in range(self.world):
            if q == self.rank:
                ptrs.append(self.own)
                continue
            peer = ctypes.c_void_p()
            _check(self.lib, self.lib.cid_peer_inbox_import(handles[q], ctypes.byref(peer)),
                   "peer_inbox")
            self.mapped.append(peer.value)
            ptrs.append(peer.value)
        self.inboxes = (ctypes.c_void_p * self.world)(*ptrs)
        self.epoch = 0
        if self.world > 1:
            dist.barrier(group=group)  # every inbox zeroed and mapped before any store

    def statistics(self, token_ids: Tensor, logits_shard: Tensor, *, vocab_offset: int,
                   total_vocab: int, shard_offsets: list[int], timing: tuple | None = None):
        """(confidence, predicted, current) of ``display_token_statistics`` on
        the unsharded logits, from this rank's shard ``logits_shard`` [B, L, V_r]
        (columns from ``vocab_offset``) and the ranks' ``shard_offsets``.
        ``timing`` = (start, end[, combined]) CUDA events recorded before the
        record kernel, after it (its stores into the peers' inboxes and the
        epoch's publication included) and, with a third event, after the
        combine (its wait included)."""
        import ctypes

        import cid_engine

        ids = token_ids.contiguous()
        lg = logits_shard.contiguous()
        rows = ids.numel()
        if rows > self.capacity:
            raise ValueError(f"{rows} rows exceed the exchange's capacity {self.capacity}")
        conf = torch.empty(ids.shape, dtype=torch.float32, device=ids.device)
        pred = torch.empty(ids.shape, dtype=torch.int64, device=ids.device)
        cur = torch.empty(ids.shape, dtype=torch.float32, device=ids.device)
        if rows == 0:
            return conf, pred, cur
        self.epoch += 1
        cur_stream = torch.cuda.current_stream(ids.device)
        stream = cur_stream.cuda_stream
        status = cid_engine._C.status_word_ptr(ids.device.index)
        if timing is not None:
            timing[0].record(cur_stream)
        _check(self.lib, self.lib.cid_display_shard_records_to_peers(
            _DTYPE_CODES[lg.dtype], lg.data_ptr(), lg.shape[-1], ids.data_ptr(), rows,
            lg.shape[-1], vocab_offset, total_vocab, self.rank, self.world, self.inboxes,
            self.capacity, self.epoch & 0xffffffff, status, stream), "shard_records_to_peers")
        if timing is not None:
            timing[1].record(cur_stream)
        self._combine(ids, shard_offsets, conf, pred, cur, status, stream)
        if timing is not None and len(timing) > 2:
            timing[2].record(cur_stream)
        return conf, pred, cur

    def from_records(self, records: Tensor, token_ids: Tensor, *, shard_offsets: list[int]):
        """The unsharded statistics from this rank's shard records [rows, 4]
        (int32, e.g. ``lm_head_shard_records``): pushed into every rank's
        inbox, then combined as in ``statistics``."""
        ids = token_ids.contiguous()
        rows = ids.numel()
        if rows > self.capacity:
            raise ValueError(f"{rows} rows exceed the exchange's capacity {self.capacity}")
        assert records.shape == (rows, 4) and records.dtype == torch.int32, "records [rows, 4]"
        conf = torch.empty(ids.shape, dtype=torch.float32, device=ids.device)
        pred = torch.empty(ids.shape, dtype=torch.int64, device=ids.device)
        cur = torch.empty(ids.shape, dtype=torch.float32, device=ids.device)
        if rows == 0:
            return conf, pred, cur
        import cid_engine

        self.epoch += 1
        stream = torch.cuda.current_stream(ids.device).cuda_stream
        rec = records.contiguous()
        _check(self.lib, self.lib.cid_peer_push_records(
            rec.data_ptr(), rows, self.rank, self.world, self.inboxes, self.capacity,
            self.epoch & 0xffffffff, stream), "peer_push_records")
        self._combine(ids, shard_offsets, conf, pred, cur,
                      cid_engine._C.status_word_ptr(ids.device.index), stream)
        return conf, pred, cur

    def _combine(self, ids, shard_offsets, conf, pred, cur, status, stream) -> None:
        import ctypes

        offs = (ctypes.c_int64 * (self.world + 1))(*shard_offsets)
        _check(self.lib, self.lib.cid_display_combine_inbox(
            self.own, self.world, offs, ids.data_ptr(), ids.numel(), self.capacity,
            self.epoch & 0xffffffff, self.wait_seconds, conf.data_ptr(), pred.data_ptr(),
            cur.data_ptr(), status, stream), "combine_inbox")

    def healthy(self) -> bool:
        """False once a combine on this device has timed out or met a peer out
        of step (reads the device status word: synchronises the device)."""
        import cid_engine

        bad = cid_engine.STATUS_PEER_TIMEOUT | cid_engine.STATUS_PEER_OUT_OF_STEP
        return not (cid_engine.device_status(self.device) & bad)

    def close(self) -> None:
        """Unmaps the peers' inboxes and frees this rank's (after every rank
        has finished its steps)."""
        if self.own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        for ptr in self.mapped:
            self.lib.cid_peer_inbox_release(ptr)
        self.mapped = []
        self.lib.cid_peer_inbox_free(self.own)
        self.own = None


def vocab_parallel_lm_head_statistics(token_ids: Tensor, hidden: Tensor, weight_shard: Tensor, *,
                                      total_vocab: int, round_bf16: bool = True, group=None,
                                      exchange: PeerRecordExchange | None = None
                                      ) -> tuple[Tensor, Tensor, Tensor]:
    """``display_token_statistics`` of the logits of a vocabulary-parallel LM
    head: this rank holds ``weight_shard`` = the rows
    ``shard_offsets(total_vocab, world)[rank:rank+2]`` of the output
    embedding and the full ``hidden`` states.  Each rank reduces its logits
    to 16-byte row records inside the GEMM (the logits never reach memory),
    the records are all-gathered over NCCL (or, with ``exchange``, pushed into
    every rank's inbox over peer memory) and combined; every rank returns the
    unsharded statistics."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    offs = shard_offsets(total_vocab, world)
    assert weight_shard.shape[0] == offs[rank + 1] - offs[rank], "shard height mismatch"
    ops = torch.ops.cid_engine
    records = ops.lm_head_shard_records(token_ids, hidden, weight_shard, offs[rank], total_vocab,
                                        round_bf16)
    if exchange is not None:
        return exchange.from_records(records, token_ids, shard_offsets=offs)
    ids = token_ids.reshape(1, -1)
    c, p, u = ops.display_combine_records(gather_records(records, group), ids, offs)
    return c.view(token_ids.shape), p.view(token_ids.shape), u.view(token_ids.shape)


def vocab_parallel_refine(token_ids: Tensor, logits_shard: Tensor, *, total_vocab: int,
                          mask_token_id: int, eos_token_id: int | None, reveal_fraction: float,
                          revision_fraction: float, revision_margin: float, group=None,
                          timing: tuple | None = None) -> Tensor:
    """One vocabulary-parallel decode step: this rank's shard records, the
    NCCL all-gather, the combine and the refinement, enqueued on the current
    stream without host synchronisation.  Every rank returns the same refined
    ids [B, L].  ``timing`` = (start, end) CUDA events recorded around the
    record kernel.  (Splitting the step into chunks of sequences so that the
    exchange of one chunk overlaps the streaming of the next measured slower
    on B200: the step's exposed exchange is ~2% of it.)"""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    offs = shard_offsets(total_vocab, world)
    assert logits_shard.shape[-1] == offs[rank + 1] - offs[rank], "shard width mismatch"
    ops = torch.ops.cid_engine
    stream = torch.cuda.current_stream(logits_shard.device)
    if timing is not None:
        timing[0].record(stream)
    rec = ops.display_shard_records(token_ids, logits_shard, offs[rank], total_vocab)
    if timing is not None:
        timing[1].record(stream)
    c, p, u = ops.display_combine_records(gather_records(rec, group), token_ids, offs)
    return ops.refine_display_from_statistics(token_ids, c, p, u, mask_token_id, eos_token_id,
                                              reveal_fraction, revision_fraction, revision_margin)
