"""Multi-step display-refinement decode loop replayed from CUDA graphs.

The reference's caller, the CID scheduler's ``refine_display`` loop
(``benchmarks/README.md:29-43`` of fwerkor/cid-engine v1.1.0; the scheduler
itself is not part of that repository), runs one refinement step per model
step and copies the compact materialisation snapshot to the host once per
step (``benchmarks/README.md:62-66``).  ``DisplayRefineLoop`` is that driver
for the device-resident chain:

* the chain of one step (statistics -> refinement -> slot rollout -> live
  occupancy -> snapshot, ``cid_engine.step.refine_step``) is captured once per
  ring position in a CUDA graph; a step is one graph replay;
* the display ids and the slot occupancy are device state carried from one
  step to the next (two small device copies per step inside the graph; in
  eager mode the step's outputs simply become the state); nothing is read
  back to decide the next step;
* every step's snapshot is copied into a ring of pinned host buffers on a
  separate copy stream while the following steps compute; the compute stream
  waits for that copy only before the graph that rewrites the same snapshot
  buffer replays again (``period`` steps later);
* an optional ``producer(position, token_ids, logits_out)`` callable (the
  model's LM head, say) is captured into the same graph ahead of the
  statistics and fills the ring position's logits buffer from the current ids.

Without a producer the caller owns the logits ring: step ``s`` reads
``logits_buffers[s % len(logits_buffers)]``.  With ``lm_head_weight`` the ring
holds the display positions' hidden states ``[B, L, H]`` instead, and each
step runs the LM head fused with the statistics
(``refine_step_from_hidden``): no ``[B, L, V]`` logits are written at all.
"""

from __future__ import annotations

import dataclasses
import math
from collections.abc import Callable, Sequence

import torch
from torch import Tensor

from cid_engine.step import SlotInputs, StepOutputs, refine_step, refine_step_from_hidden

Producer = Callable[[int, Tensor, Tensor], None]


class DisplayRefineLoop:
    """Graph-replayed decode loop over a ring of display-logits buffers.

    ``token_ids`` [B, L] int64 and ``slots.occupancy`` ([B, S] or [B, S, 1],
    any dtype; non-zero = occupied) are the initial state; they are copied,
    not modified.  ``host_snapshots`` pinned host buffers receive the
    snapshots (0 disables the copies).  The snapshot of step ``s`` stays
    valid in its host buffer until step ``s + host_snapshots`` is issued.
    Steps run on the stream that is current when the loop is built.
    """

    def __init__(
        self,
        token_ids: Tensor,
        logits_buffers: Sequence[Tensor],
        *,
        mask_token_id: int,
        eos_token_id: int | None,
        reveal_fraction: float,
        revision_fraction: float,
        revision_margin: float,
        slots: SlotInputs | None = None,
        producer: Producer | None = None,
        host_snapshots: int = 4,
        use_graphs: bool = True,
        lm_head_weight: Tensor | None = None,
    ) -> None:
        if token_ids.device.type != "cuda":
            raise RuntimeError("DisplayRefineLoop runs on CUDA devices only")
        if not logits_buffers:
            raise ValueError("logits_buffers must hold at least one buffer")
        for lg in logits_buffers:
            if lg.device != token_ids.device or tuple(lg.shape[:2]) != tuple(token_ids.shape):
                raise ValueError("every buffer must be [B, L, V] logits (or [B, L, H] hidden "
                                 "states with lm_head_weight) on the ids' device")
        if host_snapshots < 0:
            raise ValueError("host_snapshots must be >= 0")
        self.device = token_ids.device
        self.logits = list(logits_buffers)
        self.lm_head_weight = lm_head_weight
        self.params = dict(mask_token_id=mask_token_id, eos_token_id=eos_token_id,
                           reveal_fraction=reveal_fraction, revision_fraction=revision_fraction,
                           revision_margin=revision_margin)
        self.slots = slots
        self.producer = producer
        self.use_graphs = use_graphs
        self.ids = token_ids.detach().clone()
        self.occ = None
        if slots is not None:
            B, S = slots.allocation_logits.shape
            self.occ = slots.occupancy.detach().reshape(B, S) != 0
        # a snapshot buffer is rewritten every `period` steps; two device
        # buffers at least so that a copy overlaps the next step
        n = len(self.logits)
        self.period = math.lcm(n, 2) if (slots is not None and host_snapshots) else n
        self.compute = torch.cuda.current_stream(self.device)
        self.copy_stream = torch.cuda.Stream(self.device)
        self.depth = host_snapshots if slots is not None else 0
        self.host: list[Tensor] = []
        self.copied: dict[int, torch.cuda.Event] = {}
        self.issued = 0
        self.graphs: list[torch.cuda.CUDAGraph] = []
        self.outs: list[StepOutputs | None] = [None] * self.period
        if use_graphs:
            self._capture()

    # -- one step of the chain (eager, or recorded into a graph) ---------------
    def _chain(self, j: int) -> StepOutputs:
        lg = self.logits[j % len(self.logits)]
        if self.producer is not None:
            self.producer(j % len(self.logits), self.ids, lg)
        slots = None
        if self.slots is not None:
            slots = dataclasses.replace(self.slots, occupancy=self.occ)
        if self.lm_head_weight is not None:
            out = refine_step_from_hidden(self.ids, lg, self.lm_head_weight, slots=slots,
                                          **self.params)
        else:
            out = refine_step(self.ids, lg, slots=slots, **self.params)
        if self.use_graphs:
            # a graph replays on fixed addresses: carry the state in place
            self.ids.copy_(out.token_ids)
            if slots is not None:
                self.occ.copy_(out.next_occupancy)
        else:
            # eager: the step's outputs become the state (no copy kernels)
            self.ids = out.token_ids
            if slots is not None:
                self.occ = out.next_occupancy
        return out

    def _capture(self) -> None:
        ids0 = self.ids.clone()
        occ0 = None if self.occ is None else self.occ.clone()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(self.compute)
        with torch.cuda.stream(side):  # warm-up outside capture (lazy init)
            self._chain(0)
        self.compute.wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.ids.copy_(ids0)
        if occ0 is not None:
            self.occ.copy_(occ0)
        for j in range(self.period):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.outs[j] = self._chain(j)
            self.graphs.append(g)
        torch.cuda.synchronize(self.device)

    # -- public API ------------------------------------------------------------
    @property
    def token_ids(self) -> Tensor:
        """Current display ids (device state)."""
        return self.ids

    @property
    def occupancy(self) -> Tensor | None:
        """Current slot occupancy, bool [B, S] (device state)."""
        return self.occ

    @property
    def last_outputs(self) -> StepOutputs | None:
        """Device outputs of the most recent step (graph mode: valid until the
        same ring position replays again)."""
        if self.issued == 0:
            return None
        return self.outs[(self.issued - 1) % self.period]

    def reset(self, token_ids: Tensor, occupancy: Tensor | None = None) -> None:
        """Start a new sequence from ``token_ids`` (and ``occupancy``)."""
        self.drain()
        self.ids.copy_(token_ids)
        if occupancy is not None:
            self.occ.copy_(occupancy.reshape(self.occ.shape) != 0)
        self.issued = 0
        self.copied.clear()

    def step(self) -> int:
        """Enqueue one step; returns its index.  No host synchronisation
        unless the compute stream must first wait for an old snapshot copy
        (that wait is on the device, not the host)."""
        s = self.issued
        j = s % self.period
        old = self.copied.get(s - self.period)
        with torch.cuda.stream(self.compute):
            if old is not None:
                self.compute.wait_event(old)
            if self.use_graphs:
                self.graphs[j].replay()
            else:
                self.outs[j] = self._chain(j)
        self.issued += 1
        if self.depth:
            self._copy_snapshot(s, self.outs[j].snapshot)
            keep = max(self.period, self.depth)
            for k in [k for k in self.copied if k < s - keep]:
                del self.copied[k]
        return s

    def _copy_snapshot(self, s: int, snap: Tensor) -> None:
        if not self.host:
            self.host = [torch.empty(snap.shape, dtype=snap.dtype, pin_memory=True)
                         for _ in range(self.depth)]
        ready = torch.cuda.Event()
        ready.record(self.compute)
        self.copy_stream.wait_event(ready)
        with torch.cuda.stream(self.copy_stream):
            self.host[s % self.depth].copy_(snap, non_blocking=True)
            if not self.use_graphs:
                snap.record_stream(self.copy_stream)
        done = torch.cuda.Event()
        done.record(self.copy_stream)
        self.copied[s] = done

    def snapshot(self, s: int) -> Tensor:
        """Host snapshot of step ``s`` (waits for its copy only)."""
        if not self.depth:
            raise RuntimeError("host snapshots are disabled (no slots or host_snapshots=0)")
        if not (self.issued - self.depth <= s < self.issued):
            raise IndexError(f"snapshot of step {s} is no longer (or not yet) in the host ring")
        ev = self.copied.get(s)
        if ev is not None:
            ev.synchronize()
        return self.host[s % self.depth]

    def run(self, steps: int, on_snapshot: Callable[[int, Tensor], None] | None = None) -> Tensor:
        """Issue ``steps`` steps.  With ``on_snapshot``, each step's host
        snapshot is handed over in order as soon as its copy completes (the
        host blocks only when it falls ``host_snapshots`` steps behind).
        Returns the device ids after the last step (not synchronised)."""
        pending = []
        for _ in range(steps):
            if on_snapshot is not None and self.depth and len(pending) == self.depth:
                s0 = pending.pop(0)
                on_snapshot(s0, self.snapshot(s0))
            s = self.step()
            if on_snapshot is not None and self.depth:
                pending.append(s)
                while pending and self.copied[pending[0]].query():
                    s0 = pending.pop(0)
                    on_snapshot(s0, self.snapshot(s0))
        for s0 in pending:
            on_snapshot(s0, self.snapshot(s0))
        return self.ids

    def drain(self) -> None:
        """Wait for the outstanding snapshot copies."""
        for ev in self.copied.values():
            ev.synchronize()

    def close(self) -> None:
        """Release the graphs and host buffers."""
        self.drain()
        self.graphs.clear()
        self.outs = [None] * self.period
        self.host.clear()
