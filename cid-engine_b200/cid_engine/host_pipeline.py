"""Display statistics and refinement for logits that live in host memory.

When the display logits sit in (pinned) host memory, the step is bound by the
host->device link, not by HBM.  ``display_token_statistics_from_host`` streams
the logits to the device in chunks of sequences on a copy stream while the
statistics kernel consumes the previous chunk on the compute stream (double
buffering with CUDA events), so the kernel time hides under the transfer.
"""

from __future__ import annotations

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
