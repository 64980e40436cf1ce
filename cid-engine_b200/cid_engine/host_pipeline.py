"""Display statistics and refinement for logits that live in host memory.

When the display logits sit in (pinned) host memory, the step is bound by the
host->device link, not by HBM.  ``display_token_statistics_from_host`` streams
the logits to the device in chunks of sequences on a copy stream while the
statistics kernel consumes the previous chunk on the compute stream (double
buffering with CUDA events), so the kernel time hides under the transfer.
"""

from __future__ import annotations

import time

import torch
from torch import Tensor


class HostStatisticsPipeline:
    """Reusable device buffers + copy stream for host-resident logits of a
    fixed shape [B, L, V] (any float dtype).

    ``reduce(ids_chunk, logits_chunk)`` is the per-chunk operator, by default
    ``display_token_statistics``; ``display_shard_records`` of a vocabulary
    shard fits the same slot.  Its outputs are concatenated along dim 0."""

    def __init__(self, batch: int, tokens: int, vocab: int, dtype: torch.dtype,
                 device: torch.device | int = 0, chunk: int | None = None, buffers: int = 2,
                 reduce=None):
        self.reduce = reduce or torch.ops.cid_engine.display_token_statistics
        self.device = torch.device("cuda", device) if isinstance(device, int) else device
        self.shape = (batch, tokens, vocab)
        row_bytes = tokens * vocab * torch.empty((), dtype=dtype).element_size()
        # ~256 MB per chunk: long enough to amortise launch/event overheads
        self.chunk = chunk or max(1, min(batch, (256 << 20) // max(1, row_bytes)))
        self.bufs = [torch.empty((self.chunk, tokens, vocab), dtype=dtype, device=self.device)
                     for _ in range(buffers)]
        self.copy_stream = torch.cuda.Stream(self.device)
        self.free = [None] * buffers

    def statistics(self, token_ids: Tensor, logits: Tensor):
        """display_token_statistics of host `logits` (pinned for overlap);
        `token_ids` may be on the host or the device.  Returns device tensors."""
        B, L, V = self.shape
        assert tuple(logits.shape) == self.shape, "logits shape differs from the pipeline's"
        compute = torch.cuda.current_stream(self.device)
        ids = token_ids.to(self.device, non_blocking=True)
        outs = []
        start = torch.cuda.Event()
        start.record(compute)
        self.copy_stream.wait_event(start)
        for i, b0 in enumerate(range(0, B, self.chunk)):
            b1 = min(B, b0 + self.chunk)
            k = i % len(self.bufs)
            buf = self.bufs[k][: b1 - b0]
            if self.free[k] is not None:
                self.copy_stream.wait_event(self.free[k])
            with torch.cuda.stream(self.copy_stream):
                buf.copy_(logits[b0:b1], non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(self.copy_stream)
            compute.wait_event(ready)
            out = self.reduce(ids[b0:b1], buf)
            outs.append(out if isinstance(out, tuple) else (out,))
            done = torch.cuda.Event()
            done.record(compute)
            self.free[k] = done
        if len(outs) == 1:
            res = outs[0]
        else:
            res = tuple(torch.cat([o[j] for o in outs]) for j in range(len(outs[0])))
        return res if len(res) > 1 else res[0]


def display_token_statistics_from_host(token_ids: Tensor, logits: Tensor, *,
                                       device: torch.device | int = 0, chunk: int | None = None):
    pipe = HostStatisticsPipeline(*logits.shape, dtype=logits.dtype, device=device, chunk=chunk)
    return pipe.statistics(token_ids, logits)


def bench_e2e(ids_dev: Tensor, logits_dev: Tensor, *, steps: int, warmup: int, mask_id: int,
              eos_id: int, reveal: float, revision: float, margin: float) -> dict:
    """End-to-end step through the public API from pinned host buffers: per
    step the host->device copy of the logits and ids, statistics, refinement
    and the device->host read of the refined ids, timed on the device."""
    dev = logits_dev.device
    logits_h = torch.empty(logits_dev.shape, dtype=logits_dev.dtype, pin_memory=True)
    logits_h.copy_(logits_dev)
    ids_h = torch.empty(ids_dev.shape, dtype=ids_dev.dtype, pin_memory=True)
    ids_h.copy_(ids_dev)
    out_h = torch.empty(ids_dev.shape, dtype=ids_dev.dtype, pin_memory=True)
    pipe = HostStatisticsPipeline(*logits_dev.shape, dtype=logits_dev.dtype, device=dev)
    ops = torch.ops.cid_engine

    def step():
        ids = ids_h.to(dev, non_blocking=True)
        conf, pred, cur = pipe.statistics(ids, logits_h)
        refined = ops.refine_display_from_statistics(ids, conf, pred, cur, mask_id, eos_id,
                                                     reveal, revision, margin)
        out_h.copy_(refined, non_blocking=True)
        return refined

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    a.record()
    for _ in range(steps):
        step()
    b.record()
    torch.cuda.synchronize(dev)
    wall = (time.perf_counter() - w0) / steps
    ms = a.elapsed_time(b) / steps
    nbytes = logits_dev.numel() * logits_dev.element_size()
    h2d = nbytes + ids_dev.numel() * ids_dev.element_size()
    d2h = ids_dev.numel() * ids_dev.element_size()
    del pipe, logits_h
    return {"value": round(nbytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": round(ms, 3), "wall_ms_per_step": round(wall * 1e3, 3),
            "steps": steps, "api": "cid_engine.host_pipeline + refine_display_from_statistics"}
