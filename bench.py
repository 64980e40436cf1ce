#!/usr/bin/env python
"""Display-refinement step throughput on B200.

One step = ``display_token_statistics`` over display logits [B, L, V] followed
by ``refine_display_from_statistics`` on the same rows, all on the device with
no host sync (the "fused display-stats + refine step").

* N=1 workload: logits bf16 [32, 1024, 128256] = bf16(2 N(0,1)), 10% of rows
  with a +8 peak, 1% with an exact two-way max tie, display positions masked
  with probability 0.6 and one EOS per row (synthetic data, seeded).
* ``value`` = logits bytes of all ranks / device time of the timed steps
  (GB/s, inputs resident in HBM; 8.4 GB of logits per step, far above the
  126 MB L2, so no flush is needed between steps).
* ``e2e`` = the same metric through the public API from pinned host buffers,
  host->device copies of every step's logits and ids and the device->host
  read of the refined ids inside the timed region (copies overlapped with the
  statistics kernel in row chunks by ``cid_engine.host_pipeline``).
* ``roofline`` = the statistics kernel's algorithmic bytes per launch / its
  CUDA-event duration, against the measured HBM copy bandwidth.
* ``cpu_baseline`` = the reference's own CPU backend (built from its sources
  into oracle/_ref) on a bounded sample, in a separate process.
* ``refine_loop`` = decode loop: B=256, L=512, V=32000 bf16, 128
  slots, stats -> refine -> rollout -> live occupancy -> snapshot per step,
  64 steps, steps/s.

``--impl reference`` times the reference CPU backend on the host cores with
the same workload, metric and unit.  Multi-GPU (torchrun, N>1): vocabulary-
parallel statistics of [64, 4096, 152064] bf16 sharded over the ranks' GPUs
(records all-gathered over NCCL, combined on every rank), then refinement.
"""

from __future__ import annotations

import argparse
import json
import os
import signal
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "cid-engine_b200"))
sys.path.insert(0, str(ROOT))

MASK_ID, EOS_ID = 0, 1
REVEAL, REVISION, MARGIN = 0.25, 0.1, 0.05
# the headline metric, the same in every arm (B200 at N=1 and N>1, reference)
METRIC = "display logits GB/s (display_token_statistics + refine_display_from_statistics step)"
# display step at N=1: logits bf16 [32, 1024, 128256]
STEP = dict(B=32, L=1024, V=128256)
# vocabulary-parallel step at N>1: logits bf16 [64, 4096, 152064] sharded by columns
SHARDED = dict(B=64, L=4096, V=152064)
# decode loop: 256 sequences of 512 over 32000 tokens, 128 thought slots, 64 steps
LOOP = dict(B=256, L=512, V=32000, S=128, F=4, Rv=3, Rr=6, H=512, K=12, steps=64)
# DRAM bytes (read + write) per row of the statistics kernel that serves the
# [32, 1024, 128256] step (warp per row), measured by ncu (dram__bytes_read.sum +
# dram__bytes_write.sum) on a [1, 10240, 128256] bf16 launch and divided by
# its 10240 rows; traffic grows in proportion to rows.
NCU_TRAFFIC_PER_ROW = (2_632_891_000 + 4_414_848) / 10240
# The same for the record kernel on a rank's shard rows at N ranks of the
# [64, 4096, 152064] workload (152064 / N columns), from ncu captures of
# `bench.py --profile-case shard<N>` (8192 N rows each, 2.5 GB), per row.
NCU_SHARD_TRAFFIC_PER_ROW: dict[int, float] = {
    2: (2_499_850_240 + 3_524_608) / 16384,
    4: (2_504_554_496 + 3_683_072) / 32768,
    8: (2_505_670_912 + 4_321_280) / 65536,
}


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# synthetic inputs
# ---------------------------------------------------------------------------


def loop_logits(step: int, device, batch: int | None = None):
    """Decode-loop logits of step ``step``: bf16 [256, 512, 32000] =
    bf16(3 N(0,1)) from seed 4 + step (the first ``batch`` sequences)."""
    import torch

    B, L, V = LOOP["B"], LOOP["L"], LOOP["V"]
    g = torch.Generator(device=device).manual_seed(4 + step)
    lg = torch.randn((B, L, V), generator=g, device=device, dtype=torch.bfloat16)
    lg.mul_(3.0)
    return lg if batch is None else lg[:batch].contiguous()


def loop_state(device):
    """Decode-loop start state (seed 4): display ids [256, 512] over 32000
    tokens with positions masked with probability 0.6, and the 128-slot
    thought state with occupancy Bernoulli(0.4)."""
    import torch

    from cid_engine.step import SlotInputs

    c = LOOP
    B, L, V, S = c["B"], c["L"], c["V"], c["S"]
    dev = device
    g = torch.Generator(device=dev).manual_seed(4)
    ids0 = torch.randint(2, V, (B, L), generator=g, device=dev)
    ids0[torch.rand((B, L), generator=g, device=dev) < 0.6] = MASK_ID
    occ = (torch.rand((B, S, 1), generator=g, device=dev) < 0.4).float()
    slot = SlotInputs(
        occupancy=occ,
        allocation_logits=torch.randn((B, S), generator=g, device=dev),
        lifecycle_logits=torch.randn((B, S, c["F"]), generator=g, device=dev),
        revision_logits=torch.randn((B, S, c["Rv"]), generator=g, device=dev),
        input_lifecycle=torch.randn((B, S, c["F"]), generator=g, device=dev),
        semantic=torch.randn((B, S, c["H"]), generator=g, device=dev),
        role_logits=torch.randn((B, S, c["Rr"]), generator=g, device=dev),
        uncertainty=torch.rand((B, S, 1), generator=g, device=dev),
        noise_delta=torch.randn((B, S, 1), generator=g, device=dev),
        semantic_indices=torch.randint(0, c["H"], (c["K"],), generator=g, device=dev),
        threshold=0.5, max_allocations=8, retired_index=3,
    )
    return ids0, slot


def loop_initial_ids(device):
    """Display ids the decode loop starts from."""
    return loop_state(device)[0]


def display_inputs(B, L, V, seed, device, dtype=None):
    """bf16(2 N(0,1)) logits with planted peaks/ties, display ids with masked
    positions (p=0.6) and one EOS per row."""
    import torch

    dtype = dtype or torch.bfloat16
    g = torch.Generator(device=device).manual_seed(seed)
    logits = torch.randn((B, L, V), generator=g, device=device, dtype=dtype)
    logits.mul_(2.0)
    rows = B * L
    flat = logits.view(rows, V)
    peak_rows = torch.nonzero(torch.rand(rows, generator=g, device=device) < 0.10).flatten()
    peak_cols = torch.randint(V, (peak_rows.numel(),), generator=g, device=device)
    flat[peak_rows, peak_cols] = (flat[peak_rows, peak_cols].float() + 8.0).to(dtype)
    tie_rows = torch.nonzero(torch.rand(rows, generator=g, device=device) < 0.01).flatten()
    if tie_rows.numel():
        top = flat[tie_rows].float().amax(dim=1) + 1.0
        c1 = torch.randint(V, (tie_rows.numel(),), generator=g, device=device)
        c2 = (c1 + 1 + torch.randint(V - 1, (tie_rows.numel(),), generator=g, device=device)) % V
        flat[tie_rows, c1] = top.to(dtype)
        flat[tie_rows, c2] = top.to(dtype)
    ids = torch.randint(2, V, (B, L), generator=g, device=device)
    ids[torch.rand((B, L), generator=g, device=device) < 0.6] = MASK_ID
    eos_at = torch.randint(L // 2, L, (B,), generator=g, device=device)
    pos = torch.arange(L, device=device).expand(B, L)
    ids[pos == eos_at[:, None]] = EOS_ID
    ids[pos > eos_at[:, None]] = MASK_ID
    return ids, logits


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------


class ClockSampler:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.window = None  # (start, end) wall-clock seconds of the timed region

    def mark_start(self) -> None:
        self.t0 = time.time()

    def mark_end(self) -> None:
        self.window = (self.t0, time.time())

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except OSError:
            self.proc = None
        time.sleep(0.5)  # let nvidia-smi start sampling before the timed region
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.send_signal(signal.SIGTERM)
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        else:
            self.lines = []

    def summary(self) -> dict:
        import datetime

        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 10:
                continue
            if self.window is not None:
                try:
                    ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    ts = None
                if ts is not None and not (self.window[0] - 0.1 <= ts <= self.window[1] + 0.1):
                    continue
            try:
                sm.append(float(f[2]))
                mx = max(mx, float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[6:10]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# reference CPU backend (separate process: it registers torch.ops.cid_engine)
# ---------------------------------------------------------------------------


def _reference_inputs(args):
    """The CPU sample's inputs: rows of the B200 arm's own workload.  With
    ``--sample-gen cuda`` they are generated on the GPU by the same
    generators as the B200 arm (so the values are identical) and copied to
    the host; otherwise on the host.  Only plain torch runs here: this
    process must not load this repository's extension."""
    import torch

    dev = "cuda" if args.sample_gen == "cuda" and torch.cuda.is_available() else "cpu"
    B, L, V = args.sample_b, args.sample_l, args.sample_v
    if dev == "cpu" and B * L * V > (1 << 28):
        # host generation runs at ~25 M values/s: without a GPU, keep the
        # sample to one sequence's first 1024 rows
        B, L = 1, min(L, 1024)
    if args.sample_world:  # vocabulary-parallel workload: its shards side by side
        W = args.sample_world
        parts, ids = [], None
        for r in range(W):
            i, lg, _ = sharded_display_inputs(SHARDED["B"], SHARDED["L"], V, r, W, 3, dev)
            parts.append(lg[:B, :L].cpu())
            ids = i[:B, :L].cpu()
            del lg
        return ids, torch.cat(parts, dim=-1), dev
    ids, logits = display_inputs(B, L, V, seed=1, device=dev)
    return ids.cpu(), logits.cpu(), dev


def cpu_reference_worker(args) -> None:
    import torch

    lib = ROOT / "oracle" / "_ref" / "libcid_engine_ref.so"
    ids, logits, gen = _reference_inputs(args)
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    B, L, V = logits.shape
    if lib.exists():
        torch.ops.load_library(str(lib))
        kind = "reference"

        def step():
            c, p, u = torch.ops.cid_engine.display_token_statistics(ids, logits)
            torch.ops.cid_engine.refine_display_from_statistics(
                ids, c, p, u, MASK_ID, EOS_ID, REVEAL, REVISION, MARGIN)
    else:
        from oracle import oracle

        kind = "port"

        def step():
            c, p, u = oracle.display_token_statistics(ids, logits)
            oracle.refine_display_from_statistics(ids, c, p, u, MASK_ID, EOS_ID, REVEAL,
                                                  REVISION, MARGIN)

    step()  # warm-up
    times = []
    t_end = time.perf_counter() + args.cpu_seconds
    while time.perf_counter() < t_end or len(times) < args.cpu_min_reps:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    per = statistics.median(times)
    nbytes = logits.numel() * logits.element_size()
    print(json.dumps({
        "value": nbytes / per / 1e9, "unit": "GB/s", "cores": cores, "kind": kind,
        "ms_per_step": per * 1e3, "reps": len(times),
        "sample": f"stats+refine on logits bf16 [{B},{L},{V}] ({nbytes / 1e9:.3f} GB) per step, "
                  f"median of {len(times)} reps (inputs generated on {gen})",
    }))


def run_cpu_baseline(sample=(1, 1024, 128256), seconds=10.0, *, gen="cpu", world=0,
                     min_reps=3) -> dict | None:
    cmd = [sys.executable, str(ROOT / "bench.py"), "--cpu-worker", "--sample-b", str(sample[0]),
           "--sample-l", str(sample[1]), "--sample-v", str(sample[2]),
           "--cpu-seconds", str(seconds), "--cpu-min-reps", str(min_reps),
           "--sample-gen", gen, "--sample-world", str(world)]
    env = dict(os.environ)
    if gen == "cpu":
        env["CUDA_VISIBLE_DEVICES"] = ""
    try:
        res = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=900)
        return json.loads(res.stdout.strip().splitlines()[-1])
    except Exception as exc:  # the baseline is reported, never fatal
        return {"error": f"{type(exc).__name__}: {exc}"[:300]}


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------


def time_device_steps(step, K, W, stream, clock=None):
    import torch

    for _ in range(W):
        step(None)
    torch.cuda.synchronize()
    if clock is not None:
        clock.mark_start()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    pairs = []
    start.record(stream)
    for _ in range(K):
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        pairs.append(ev)
        step(ev)
    end.record(stream)
    torch.cuda.synchronize()
    if clock is not None:
        clock.mark_end()
    total_ms = start.elapsed_time(end)
    kern = [a.elapsed_time(b) for a, b in pairs]
    return total_ms, kern


def bench_single(args) -> dict:
    import torch

    import cid_engine  # noqa: F401  (loads the extension)

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, L, V = STEP["B"], STEP["L"], STEP["V"]
    ids, logits = display_inputs(B, L, V, seed=1, device=dev)
    stream = torch.cuda.current_stream()
    ops = torch.ops.cid_engine

    def step(ev):
        if ev is not None:
            ev[0].record(stream)
        c, p, u = ops.display_token_statistics(ids, logits)
        if ev is not None:
            ev[1].record(stream)
        ops.refine_display_from_statistics(ids, c, p, u, MASK_ID, EOS_ID, REVEAL, REVISION, MARGIN)

    K, W = args.steps, args.warmup
    with ClockSampler(0) as clk:
        total_ms, kern = time_device_steps(step, K, W, stream, clk)
    clocks = clk.summary()
    nbytes = logits.numel() * logits.element_size()
    ms = total_ms / K
    value = nbytes / (ms * 1e-3) / 1e9
    rows = B * L
    alg_bytes = nbytes + rows * (8 + 4 + 8 + 4)  # logits + ids in, conf/pred/cur out
    kern_ms = statistics.mean(kern)
    peak, peak_kind = _peaks()
    achieved = alg_bytes / (kern_ms * 1e-3) / 1e9
    traffic = None if NCU_TRAFFIC_PER_ROW is None else round(NCU_TRAFFIC_PER_ROW * rows)

    # end-to-end through the public API from pinned host memory
    e2e = None
    if not args.no_e2e:
        e2e = bench_e2e(ids, logits, steps=max(3, min(K, args.e2e_steps)),
                                      warmup=2, mask_id=MASK_ID, eos_id=EOS_ID,
                                      reveal=REVEAL, revision=REVISION, margin=MARGIN)
    del logits
    torch.cuda.empty_cache()

    vp1 = None if args.no_loop else bench_vocab_parallel_n1(dev)
    loop = None if args.no_loop else bench_refine_loop(dev)
    small = None if args.no_loop else bench_small_workloads(dev)
    lm_head = None if args.no_loop else bench_lm_head(dev)
    decode = None if args.no_loop else bench_decode_and_reference_cuda(dev)
    cpu = None if args.no_cpu_baseline else run_cpu_baseline(seconds=args.cpu_seconds)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded bf16 2*N(0,1) logits, 10% planted peaks, 1% exact ties)",
        "config": {"workload": "display stats + refine, logits bf16 [32,1024,128256]",
                   "batch": B, "tokens": L, "vocab": V, "parallelism": "single GPU",
                   "l2": "inputs 8.4 GB per step >> 126 MB L2; no flush needed"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "frac_of_8TBps_nominal": round(achieved / 8000.0, 4), "traffic": traffic,
                     "kernel": "display_stats_rows_kernel<bf16> (warp per row)", "peak_kind": peak_kind,
                     "kernel_ms": round(kern_ms, 4),
                     "algorithmic_bytes_per_launch": alg_bytes},
        "e2e": e2e,
        "gpu_launches": 2 * K,
        "clocks": clocks,
        "cpu_baseline": cpu,
        "refine_loop": loop,
        "vocab_parallel_n1": vp1,
        "small_workloads": small,
        "lm_head": lm_head,
        "decode_rows": None if decode is None else decode["decode_rows"],
        "reference_cuda": None if decode is None else decode["reference_cuda"],
    }
    return line


def bench_vocab_parallel_n1(dev, steps: int = 20) -> dict:
    """The vocabulary-parallel workload, logits bf16 [64, 4096, 152064]
    (79.7 GB), on one GPU: statistics + refinement of the whole tensor, the
    one-GPU anchor of the multi-GPU lines (same problem, same generator as
    rank 0 of one)."""
    import torch

    B, L, V = SHARDED["B"], SHARDED["L"], SHARDED["V"]
    ids, logits, _ = sharded_display_inputs(B, L, V, 0, 1, 3, dev)
    ops = torch.ops.cid_engine
    stream = torch.cuda.current_stream()

    def step(ev):
        if ev is not None:
            ev[0].record(stream)
        c, p, u = ops.display_token_statistics(ids, logits)
        if ev is not None:
            ev[1].record(stream)
        ops.refine_display_from_statistics(ids, c, p, u, MASK_ID, EOS_ID, REVEAL, REVISION, MARGIN)

    total_ms, kern = time_device_steps(step, steps, 3, stream)
    ms = total_ms / steps
    kern_ms = statistics.mean(kern)
    nbytes = logits.numel() * logits.element_size()
    peak, peak_kind = _peaks()
    alg = nbytes + B * L * (8 + 4 + 8 + 4)
    del logits
    torch.cuda.empty_cache()
    return {"workload": "display stats + refine, logits bf16 [64,4096,152064] on one GPU",
            "value": round(nbytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(ms, 4), "steps": steps, "kernel_ms": round(kern_ms, 4),
            "kernel_frac": round(alg / (kern_ms * 1e-3) / 1e9 / peak, 4), "peak_kind": peak_kind}


def bench_e2e(ids_dev: Tensor, logits_dev: Tensor, *, steps: int, warmup: int, mask_id: int,
              eos_id: int, reveal: float, revision: float, margin: float) -> dict:
    """End-to-end step through the public API from pinned host buffers: per
    step the host->device copy of the logits and ids, statistics, refinement
    and the device->host read of the refined ids, timed on the device."""
    import time
    import torch
    from cid_engine.host_pipeline import HostStatisticsPipeline

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


def bench_refine_loop(dev) -> dict:
    """Decode loop (B=256, L=512, V=32000, 128 slots): 64 consecutive steps
    of the fused chain, no host sync."""
    import torch

    from cid_engine.loop import DisplayRefineLoop

    c = LOOP
    B, L, V, S = c["B"], c["L"], c["V"], c["S"]
    # ring of pre-generated logits (each 8.4 GB > L2)
    ring = [loop_logits(k, dev) for k in range(3)]
    ids0, slot = loop_state(dev)
    params = dict(mask_token_id=MASK_ID, eos_token_id=EOS_ID, reveal_fraction=REVEAL,
                  revision_fraction=REVISION, revision_margin=MARGIN)
    steps = c["steps"]
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    result = {}
    # eager: every step's operators issued from Python; graph: one replay per
    # step of the captured chain, with each step's snapshot copied to pinned
    # host memory on a copy stream (overlapping the next step)
    for mode, graphs in (("eager", False), ("graph", True)):
        loop = DisplayRefineLoop(ids0, ring, slots=slot, host_snapshots=4, use_graphs=graphs,
                                 **params)
        loop.run(3)
        loop.drain()
        loop.reset(ids0, slot.occupancy)
        torch.cuda.synchronize()
        a.record()
        loop.run(steps)
        b.record()
        torch.cuda.synchronize()
        loop.drain()
        result[mode] = a.elapsed_time(b) / steps
        snap_bytes = loop.host[0].numel() * 4
        loop.close()
    ms, ms_graph = result["eager"], result["graph"]
    logits_bytes = B * L * V * 2
    peak, _ = _peaks()
    del ring
    torch.cuda.empty_cache()
    return {"workload": "refine loop B=256 L=512 V=32000 bf16, S=128, 64 steps",
            "api": "cid_engine.DisplayRefineLoop",
            "steps_per_s": round(1e3 / ms, 2), "ms_per_step": round(ms, 4),
            "graph_steps_per_s": round(1e3 / ms_graph, 2), "graph_ms_per_step": round(ms_graph, 4),
            "logits_GBps": round(logits_bytes / (ms * 1e-3) / 1e9, 1),
            "roofline_steps_per_s": round(peak * 1e9 / logits_bytes, 1),
            "snapshot_d2h_bytes_per_step": snap_bytes,
            "launches_per_step": 4,
            "device_copies_per_step": {"graph": 2, "eager": 0}}


def _graph_time_ms(fn, reps: int) -> float:
    """Per-call device time of `fn` replayed `reps` times inside one CUDA graph."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    torch.cuda.synchronize()
    del graph
    return a.elapsed_time(b) / reps


def bench_small_workloads(dev) -> dict:
    """The small workloads: the fp32 [4,256,32000] chain (statistics,
    refinement, rollout and live occupancy of 32 slots, thought corruption
    [4,32,512]), masked diffusion [64,2048], repetition statistics, display
    corruption and linear assignment; all launch-bound, so each is timed as
    CUDA-graph replays (the [4,256,32000] logits rotate over 8 copies,
    1 GB > L2)."""
    import torch

    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import cases

    ops = torch.ops.cid_engine
    ids, logits = cases.display_f32_4x256x32000()
    ids, logits = ids.to(dev), logits.to(dev)
    copies = [logits] + [logits.clone() for _ in range(7)]
    g = torch.Generator().manual_seed(10)
    occ = (torch.rand(4, 32, 1, generator=g) < 0.4).float().to(dev)
    life = torch.zeros(4, 32, 4)
    life[..., 3] = (torch.rand(4, 32, generator=g) < 0.1).float()
    life = life.to(dev)
    al = torch.randn(4, 32, generator=g).to(dev)
    rv = torch.randn(4, 32, 3, generator=g).to(dev)
    th = [t.to(dev) for t in cases.thought_4x32x512()]
    state = {"k": 0}

    def chain_step():
        lg = copies[state["k"] % len(copies)]
        state["k"] += 1
        c, p, u = ops.display_token_statistics(ids, lg)
        ops.refine_display_from_statistics(ids, c, p, u, MASK_ID, EOS_ID, REVEAL, REVISION, MARGIN)
        # slot rollout with the live occupancy of its next state, one kernel
        ops.rollout_slot_transition_with_live(occ, al, life, rv, life, 0.5, 8, 3)
        ops.thought_corrupt_from_epsilon(*th)

    ms1 = _graph_time_ms(chain_step, 64)
    md = [a.to(dev) if isinstance(a, torch.Tensor) else a for a in cases.masked_diffusion_64x2048()]

    def md_call():
        ops.masked_diffusion_corrupt_from_random(*md)

    ms3 = _graph_time_ms(md_call, 1000)

    def rep_step():
        lg = copies[state["k"] % len(copies)]
        state["k"] += 1
        ops.display_token_statistics_with_repetition(ids, lg, MASK_ID, EOS_ID, 0.7)

    ms_rep = _graph_time_ms(rep_step, 64)

    # display-token corruption at the masked-diffusion shape: ids [64,2048] over
    # a 50257-token vocabulary, 85 % eligible, a quarter of the corrupted
    # positions replaced by random tokens
    gd = torch.Generator().manual_seed(11)
    B3, T3, V3 = 64, 2048, 50257
    dc = [torch.randint(0, V3, (B3, T3), generator=gd), torch.rand(B3, generator=gd),
          torch.rand(B3, T3, generator=gd) > 0.15, torch.rand(B3, T3, generator=gd),
          torch.rand(B3, T3, generator=gd), torch.randint(1, V3, (B3, T3), generator=gd)]
    dc = [t.to(dev) for t in dc]

    def dc_call():
        ops.display_corrupt_from_random(*dc, V3 - 1, EOS_ID, V3, 0.25)

    ms_dc = _graph_time_ms(dc_call, 1000)

    # linear assignment: 4096 problems of 16 x 16 costs (the largest column
    # count the warp solver takes), full rows
    costs = torch.randn(4096, 16, 16, generator=gd).to(dev)
    counts = torch.full((4096,), 16, dtype=torch.int64).to(dev)

    def la_call():
        ops.batched_linear_assignment(costs, counts)

    ms_la = _graph_time_ms(la_call, 200)
    del copies
    torch.cuda.empty_cache()
    return {
        "chain_f32_4x256x32000": {"workload": "fp32 [4,256,32000] stats+refine, 32 slots rollout+live, "
                                   "thought [4,32,512]", "us_per_step": round(ms1 * 1e3, 2),
                       "logits_GBps": round(131_072_000 / (ms1 * 1e-3) / 1e9, 1),
                       "launches_per_step": 4, "timing": "CUDA graph, 64 steps"},
        "masked_diffusion_64x2048": {"workload": "ids [64,2048], mask id 50256",
                                  "us_per_call": round(ms3 * 1e3, 3),
                                  "GBps": round(2_753_032 / (ms3 * 1e-3) / 1e9, 1),
                                  "launches_per_call": 1,
                                  "timing": "CUDA graph, 1000 calls (captured: one kernel a call; "
                                            "eager: two)"},
        "repetition_stats_f32_4x256x32000": {"workload": "fp32 [4,256,32000], mask 0, eos 1, multiplier 0.7",
                                  "us_per_call": round(ms_rep * 1e3, 2),
                                  "logits_GBps": round(131_072_000 / (ms_rep * 1e-3) / 1e9, 1),
                                  "timing": "CUDA graph, 64 calls, 8 rotating inputs"},
        "display_corruption": {"workload": "ids [64,2048], vocab 50257, replacement 0.25",
                               "us_per_call": round(ms_dc * 1e3, 3),
                               # 25 B in + 18 B out per token, 4 B timestep per row
                               "GBps": round((B3 * T3 * 43 + B3 * 4) / (ms_dc * 1e-3) / 1e9, 1),
                               "timing": "CUDA graph, 1000 calls"},
        "linear_assignment": {"workload": "4096 problems, 16 x 16 f32 costs",
                              "us_per_call": round(ms_la * 1e3, 2),
                              "problems_per_s": round(4096 / (ms_la * 1e-3)),
                              "timing": "CUDA graph, 200 calls"},
    }


# ---------------------------------------------------------------------------
# decode shapes and the reference's own CUDA kernels (secondary GPU bar)
# ---------------------------------------------------------------------------

# the reference's published microbenchmark shapes: display rows x 155136-token
# vocabulary, bf16 logits, one sequence; refinement at 64 display rows in
# four scenarios (all masked / EOS at 16 or 48, revision off or on)
DECODE = dict(V=155136, rows=(32, 64, 128, 256), refine_rows=64)
DECODE_SCENARIOS = (("all masked, no revision", None, 0.0),
                    ("EOS at 16, no revision", 16, 0.0),
                    ("EOS at 16, revision=1", 16, 1.0),
                    ("EOS at 48, revision=1", 48, 1.0))
L2_BYTES = 126 * 1024 * 1024


def _ring(make, nbytes: int) -> list:
    """Enough copies of an input that one pass over them is twice the L2."""
    n = max(2, -(-2 * L2_BYTES // max(1, nbytes)))
    return [make(k) for k in range(n)]


def _events_time_ms(fn, reps: int) -> float:
    """Per-call device time of `fn` issued eagerly `reps` times (for calls
    that synchronise inside and cannot be captured)."""
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def decode_logits(rows: int, k: int, dev):
    import torch

    g = torch.Generator(device=dev).manual_seed(20 + 1000 * rows + k)
    lg = torch.randn((1, rows, DECODE["V"]), generator=g, device=dev, dtype=torch.bfloat16)
    return lg.mul_(2.0)


def decode_ids(rows: int, eos_at, dev):
    import torch

    g = torch.Generator(device=dev).manual_seed(30 + rows)
    ids = torch.randint(2, DECODE["V"], (1, rows), generator=g, device=dev)
    if eos_at is None:
        ids.fill_(MASK_ID)
    else:
        ids[torch.rand((1, rows), generator=g, device=dev) < 0.5] = MASK_ID
        ids[0, eos_at] = EOS_ID
        ids[0, eos_at + 1:] = MASK_ID
    return ids


def decode_suite(dev, graphs: bool) -> dict:
    """Statistics of [1, rows, 155136] bf16 logits for the published row
    counts, and statistics + refinement at 64 rows, through whichever
    ``torch.ops.cid_engine`` this process has loaded.  Inputs rotate over
    copies totalling twice the L2.  ``graphs``: time as CUDA-graph replays
    (statistics + refinement then runs without a host round trip)."""
    import torch

    ops = torch.ops.cid_engine
    timer = _graph_time_ms if graphs else _events_time_ms
    out = {"stats": {}, "stats_refine": {}}
    for rows in DECODE["rows"]:
        nbytes = rows * DECODE["V"] * 2
        ring = _ring(lambda k: decode_logits(rows, k, dev), nbytes)
        ids = decode_ids(rows, 16, dev)
        st = {"k": 0}

        def call():
            lg = ring[st["k"] % len(ring)]
            st["k"] += 1
            ops.display_token_statistics(ids, lg)

        out["stats"][rows] = timer(call, 20 * len(ring)) * 1e3
        del ring
    rows = DECODE["refine_rows"]
    ring = _ring(lambda k: decode_logits(rows, k, dev), rows * DECODE["V"] * 2)
    for name, eos_at, revision in DECODE_SCENARIOS:
        ids = decode_ids(rows, eos_at, dev)
        st = {"k": 0}

        def step():
            lg = ring[st["k"] % len(ring)]
            st["k"] += 1
            c, p, u = ops.display_token_statistics(ids, lg)
            ops.refine_display_from_statistics(ids, c, p, u, MASK_ID, EOS_ID, REVEAL, revision,
                                               MARGIN)

        out["stats_refine"][name] = timer(step, 10 * len(ring)) * 1e3
    del ring
    torch.cuda.empty_cache()
    return out


def _time_into(res: dict, key: str, measure) -> None:
    """res[key] = measure(), or None when the operator fails in this process
    (an operator the loaded implementation does not support)."""
    try:
        res[key] = measure()
    except Exception:  # noqa: BLE001 - recorded as a missing measurement
        res[key] = None


def secondary_suite(dev, graphs: bool) -> dict:
    """Per-call device time (us) of the operators the reference also ships as
    CUDA kernels, on the benchmark shapes, through whichever
    ``torch.ops.cid_engine`` this process has loaded."""
    import torch

    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import cases

    ops = torch.ops.cid_engine
    timer = _graph_time_ms if graphs else _events_time_ms
    res = {}
    # statistics of the [32, 1024, 128256] display step (8.4 GB > L2)
    ids, logits = display_inputs(STEP["B"], STEP["L"], STEP["V"], seed=1, device=dev)
    res["stats_32x1024x128256_ms"] = _events_time_ms(
        lambda: ops.display_token_statistics(ids, logits), 10)
    del logits
    torch.cuda.empty_cache()
    md = [a.to(dev) if isinstance(a, torch.Tensor) else a for a in cases.masked_diffusion_64x2048()]
    res["masked_diffusion_64x2048_us"] = timer(
        lambda: ops.masked_diffusion_corrupt_from_random(*md), 1000) * 1e3
    th = [t.to(dev) for t in cases.thought_4x32x512()]
    res["thought_corruption_4x32x512_us"] = timer(
        lambda: ops.thought_corrupt_from_epsilon(*th), 1000) * 1e3
    # slot kernels at the decode loop's 256 x 128 slots
    g = torch.Generator().manual_seed(40)
    B, S = LOOP["B"], LOOP["S"]
    occ = (torch.rand(B, S, 1, generator=g) < 0.4).float().to(dev)
    al = torch.randn(B, S, generator=g).to(dev)
    lc = torch.randn(B, S, LOOP["F"], generator=g).to(dev)
    rv = torch.randn(B, S, LOOP["Rv"], generator=g).to(dev)
    il = torch.randn(B, S, LOOP["F"], generator=g).to(dev)
    res["rollout_256x128_us"] = timer(
        lambda: ops.rollout_slot_transition(occ, al, lc, rv, il, 0.5, 8, 3), 1000) * 1e3
    # prefix allocation over 128 slots, the reference's published cases
    for dt in (torch.float32, torch.bfloat16):
        for b in (1, 8):
            o = (torch.rand(b, 128, generator=g) < 0.4).to(dt).to(dev)
            lg = torch.randn(b, 128, generator=g).to(dt).to(dev)
            res[f"prefix_allocation_{str(dt)[6:]}_b{b}_us"] = timer(
                lambda o=o, lg=lg: ops.prefix_allocation_mask(o, lg, 0.5, 8), 1000) * 1e3
    # snapshot of 128 slots x 4096 semantic dims, bf16 (published case)
    sem = torch.randn(1, 128, 4096, generator=g).to(torch.bfloat16).to(dev)
    roles = torch.randn(1, 128, 6, generator=g).to(torch.bfloat16).to(dev)
    unc = torch.rand(1, 128, 1, generator=g).to(torch.bfloat16).to(dev)
    noise = torch.randn(1, 128, 1, generator=g).to(torch.bfloat16).to(dev)
    life = torch.randn(1, 128, 4, generator=g).to(torch.bfloat16).to(dev)
    sel = (torch.rand(1, 128, generator=g) < 0.5).to(dev)
    idx = torch.randint(0, 4096, (12,), generator=g).to(dev)
    res["snapshot_128x4096_bf16_us"] = timer(
        lambda: ops.materialize_cell_snapshot(sem, roles, unc, noise, life, sel, idx), 1000) * 1e3
    # repetition statistics on the fp32 [4, 256, 32000] logits, two copies
    # rotating (262 MB > L2)
    rids, rlg = cases.display_f32_4x256x32000()
    rids = rids.to(dev)
    rcopies = [rlg.to(dev), rlg.to(dev)]
    state = {"k": 0}

    def rep_call():
        lg = rcopies[state["k"] % 2]
        state["k"] += 1
        ops.display_token_statistics_with_repetition(rids, lg, MASK_ID, EOS_ID, 0.7)

    _time_into(res, "repetition_stats_f32_4x256x32000_us", lambda: timer(rep_call, 64) * 1e3)
    del rcopies
    # display corruption at [64, 2048] over 50257 tokens (bench_small_workloads' inputs)
    gd = torch.Generator().manual_seed(11)
    B3, T3, V3 = 64, 2048, 50257
    dc = [torch.randint(0, V3, (B3, T3), generator=gd), torch.rand(B3, generator=gd),
          torch.rand(B3, T3, generator=gd) > 0.15, torch.rand(B3, T3, generator=gd),
          torch.rand(B3, T3, generator=gd), torch.randint(1, V3, (B3, T3), generator=gd)]
    dc = [t.to(dev) for t in dc]
    _time_into(res, "display_corruption_64x2048_us", lambda: timer(
        lambda: ops.display_corrupt_from_random(*dc, V3 - 1, EOS_ID, V3, 0.25), 1000) * 1e3)
    # linear assignment: 4096 problems of 16 x 16 costs
    costs = torch.randn(4096, 16, 16, generator=gd).to(dev)
    counts = torch.full((4096,), 16, dtype=torch.int64).to(dev)
    _time_into(res, "linear_assignment_4096x16x16_us", lambda: timer(
        lambda: ops.batched_linear_assignment(costs, counts), 200) * 1e3)
    torch.cuda.empty_cache()
    return res


def ref_cuda_worker(args) -> None:
    """The reference's own CUDA kernels (compiled unchanged for sm_100a by
    ``make -C oracle ref-cuda``), in a process that never loads this
    repository's extension."""
    import torch

    lib = ROOT / "oracle" / "_ref" / "libcid_engine_ref_cuda.so"
    if not lib.exists():
        print(json.dumps({"error": "oracle/_ref/libcid_engine_ref_cuda.so not built"}))
        return
    torch.ops.load_library(str(lib))
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    out = {"decode": decode_suite(dev, graphs=False), "secondary": secondary_suite(dev, graphs=False)}
    print(json.dumps(out))


def run_ref_cuda() -> dict:
    cmd = [sys.executable, str(ROOT / "bench.py"), "--ref-cuda-worker"]
    try:
        res = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
        return json.loads(res.stdout.strip().splitlines()[-1])
    except Exception as exc:  # a secondary bar is reported, never fatal
        return {"error": f"{type(exc).__name__}: {exc}"[:300]}


def bench_decode_and_reference_cuda(dev) -> dict:
    """Decode shapes and the secondary GPU bar: this repository's kernels
    (CUDA-graph replays; statistics + refinement without a host round trip,
    and eagerly) against the reference's own CUDA kernels on the same box,
    shapes and inputs (eager: its refinement is a host round trip, and CUDA
    graphs would only flatter its launch-bound kernels)."""
    ours = decode_suite(dev, graphs=True)
    ours_eager = decode_suite(dev, graphs=False)
    sec = secondary_suite(dev, graphs=True)
    ref = run_ref_cuda()
    peak, _ = _peaks()
    rdec = ref.get("decode", {}) if isinstance(ref, dict) else {}
    rsec = ref.get("secondary", {}) if isinstance(ref, dict) else {}

    def ratio(r, o):
        return None if r is None or not o else round(r / o, 2)

    stats = []
    for rows in DECODE["rows"]:
        us = ours["stats"][rows]
        r = rdec.get("stats", {}).get(str(rows))
        nbytes = rows * DECODE["V"] * 2 + rows * 32
        gbps = nbytes / (us * 1e-6) / 1e9
        stats.append({"rows": rows, "us": round(us, 2), "us_eager": round(ours_eager["stats"][rows], 2),
                      "GBps": round(gbps, 1), "frac": round(gbps / peak, 4),
                      "reference_cuda_us": None if r is None else round(r, 2),
                      "speedup_vs_reference_cuda": ratio(r, us)})
    refine = []
    for name, _, _ in DECODE_SCENARIOS:
        us = ours["stats_refine"][name]
        r = rdec.get("stats_refine", {}).get(name)
        refine.append({"scenario": name, "us": round(us, 2),
                       "us_eager": round(ours_eager["stats_refine"][name], 2),
                       "reference_cuda_us": None if r is None else round(r, 2),
                       "speedup_vs_reference_cuda": ratio(r, us)})
    secondary = {}
    for k, v in sec.items():
        r = rsec.get(k)
        secondary[k] = {"ours": None if v is None else round(v, 3),
                        "reference_cuda": None if r is None else round(r, 3),
                        "speedup": ratio(r, v)}
    return {"decode_rows": {"workload": "display statistics, logits bf16 [1, rows, 155136]; "
                                        "statistics + refinement at 64 rows",
                            "timing": "ours: CUDA-graph replays (us), and eager (us_eager); "
                                      "reference: eager, separate process; inputs rotate over "
                                      "copies totalling 2x L2",
                            "stats": stats, "stats_refine_64": refine},
            "reference_cuda": {"what": "the reference's csrc/cuda kernels compiled unchanged for "
                                       "sm_100a (oracle/Makefile ref-cuda), same box, same inputs",
                               "timing": "ours: CUDA-graph replays (eager for the 8.4 GB "
                                         "statistics); reference: eager",
                               "ops": secondary,
                               "error": ref.get("error") if isinstance(ref, dict) else None}}


def bench_lm_head(dev) -> dict:
    """LM head fused with the display statistics on the display step's rows:
    hidden bf16 [32*1024, 4096] x weight bf16 [128256, 4096] (the
    [32, 1024, 128256] display logits produced by a 4096-wide LM head),
    statistics of the
    bf16-rounded logits; against cuBLAS writing the bf16 logits and the
    statistics kernel reading them back, timed in the same run."""
    import torch

    import cid_engine

    R, H, V = STEP["B"] * STEP["L"], 4096, STEP["V"]
    g = torch.Generator(device=dev).manual_seed(5)
    h = (torch.randn(R, H, generator=g, device=dev) * 0.05).to(torch.bfloat16)
    w = (torch.randn(V, H, generator=g, device=dev) * 0.05).to(torch.bfloat16)
    ids = torch.randint(0, V, (R,), generator=g, device=dev)
    flop = 2.0 * R * V * H

    def timed(fn, reps=4):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    def unfused():
        logits = h @ w.T
        return cid_engine.display_token_statistics(ids.view(1, -1), logits.view(1, R, V))

    ms_fused = timed(lambda: cid_engine.lm_head_display_statistics(ids, h, w))
    ms_gemm = timed(lambda: h @ w.T)
    ms_unfused = timed(unfused)
    c, p, u = cid_engine.lm_head_display_statistics(ids, h, w)
    e_c, e_p, e_u = unfused()
    agree = float((p == e_p[0]).float().mean())
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak_burst = float(peaks.get("bf16_tflops", 1590.0))
    peak_sust = float(peaks.get("bf16_tflops_sustained", 1400.0))
    tflops = flop / (ms_fused * 1e-3) / 1e12
    del h, w
    torch.cuda.empty_cache()
    return {"workload": f"LM head + display statistics, hidden bf16 [{R},{H}] x weight bf16 [{V},{H}]",
            "api": "cid_engine.lm_head_display_statistics",
            "fused_ms": round(ms_fused, 3), "fused_tflops": round(tflops, 1),
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "unit": "TFLOP/s",
                         "peak_burst": peak_burst, "frac_burst": round(tflops / peak_burst, 4),
                         "peak_sustained": peak_sust, "frac_sustained": round(tflops / peak_sust, 4),
                         "peak_kind": "measured" if peaks else "fallback"},
            "cublas_gemm_ms": round(ms_gemm, 3),
            "cublas_gemm_tflops": round(flop / (ms_gemm * 1e-3) / 1e12, 1),
            "unfused_ms": round(ms_unfused, 3),
            "logits_bytes_not_written": R * V * 2,
            "argmax_agreement_with_unfused": agree,
            "launches_per_call": 2}


def bench_reference(args, world: int = 1) -> dict:
    """Reference CPU backend on the host cores, on the B200 arm's workload,
    metric and unit: logits [32, 1024, 128256] at N=1, the vocabulary-parallel
    [64, 4096, 152064] under
    torchrun (rank 0 only; a CPU sample of one sequence's rows over the full
    vocabulary stands for it)."""
    if world > 1:
        B, L, V = SHARDED["B"], SHARDED["L"], SHARDED["V"]
        # 8 of the 64 sequences (10 GB), every rank's shard side by side
        res = run_cpu_baseline(sample=(8, L, V), seconds=1.0, gen="cuda", world=world)
        workload = "vocab-parallel display stats + refine, logits bf16 [64,4096,152064]"
        scaling = "strong"
    else:
        B, L, V = STEP["B"], STEP["L"], STEP["V"]
        # the whole [32, 1024, 128256] step (8.4 GB), three timed reps
        res = run_cpu_baseline(sample=(B, L, V), seconds=1.0, gen="cuda")
        workload = "display stats + refine, logits bf16 [32,1024,128256]"
        scaling = "weak"
    val = res.get("value") if res else None
    return {
        "metric": METRIC,
        "value": None if val is None else round(val, 3),
        "unit": "GB/s",
        "impl": "reference",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": None if not res or "ms_per_step" not in res else round(res["ms_per_step"], 2),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded)",
        "config": {"workload": workload, "batch": B, "tokens": L, "vocab": V,
                   "parallelism": "host CPU", "sample": res.get("sample") if res else None},
        "cpu_baseline": res,
        "e2e": {"value": None if val is None else round(val, 3), "unit": "GB/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# multi-GPU arm (torchrun, N>1): vocabulary-parallel [64, 4096, 152064]
# ---------------------------------------------------------------------------


def sharded_display_inputs(B, L, V, rank, world, seed, device):
    """This rank's vocabulary shard of the [64, 4096, 152064] logits: bf16(2 N(0,1))
    with a +8 peak in 5% of rows at a column drawn once for all ranks."""
    import torch

    offs = [r * V // world for r in range(world + 1)]  # cid_engine.parallel.shard_offsets
    lo, hi = offs[rank], offs[rank + 1]
    g = torch.Generator(device=device).manual_seed(seed * 1000 + rank)
    logits = torch.randn((B, L, hi - lo), generator=g, device=device, dtype=torch.bfloat16)
    logits.mul_(2.0)
    gs = torch.Generator(device=device).manual_seed(seed)  # shared by all ranks
    rows = B * L
    peak = torch.rand(rows, generator=gs, device=device) < 0.05
    col = torch.randint(V, (rows,), generator=gs, device=device)
    mine = torch.nonzero(peak & (col >= lo) & (col < hi)).flatten()
    flat = logits.view(rows, hi - lo)
    flat[mine, col[mine] - lo] = (flat[mine, col[mine] - lo].float() + 8.0).to(torch.bfloat16)
    # display ids (identical on every rank): masked with p=0.6, one EOS per row
    ids = torch.randint(2, V, (B, L), generator=gs, device=device)
    ids[torch.rand((B, L), generator=gs, device=device) < 0.6] = 0
    eos_at = torch.randint(L // 2, L, (B,), generator=gs, device=device)
    pos = torch.arange(L, device=device).expand(B, L)
    ids[pos == eos_at[:, None]] = 1
    ids[pos > eos_at[:, None]] = 0
    return ids, logits, offs


def e2e_vocab_parallel(ids: Tensor, logits: Tensor, offs: list[int], rank: int, *, batch: int,
                       steps: int, warmup: int) -> dict:
    """End-to-end vocabulary-parallel step through the public API from pinned
    host memory on every rank, on the headline path: per step the ids and
    this rank's logits shard (the first ``batch`` sequences) go host->device,
    overlapped in chunks with the record kernel (``HostStatisticsPipeline``
    over ``display_shard_records``), the records go into every rank's inbox
    through the ``PeerRecordExchange`` and are combined there, the rows are
    refined and the refined ids read back.  Device time, max over ranks."""
    import torch
    import torch.distributed as dist
    from cid_engine.host_pipeline import HostStatisticsPipeline
    from cid_engine.parallel import PeerRecordExchange

    dev = logits.device
    V, lo = offs[-1], offs[rank]
    world = dist.get_world_size()
    sub = logits[:batch]
    logits_h = torch.empty(sub.shape, dtype=sub.dtype, pin_memory=True)
    logits_h.copy_(sub)
    ids_h = torch.empty(ids[:batch].shape, dtype=ids.dtype, pin_memory=True)
    ids_h.copy_(ids[:batch])
    out_h = torch.empty_like(ids_h, pin_memory=True)
    ops = torch.ops.cid_engine
    pipe = HostStatisticsPipeline(*sub.shape, dtype=sub.dtype, device=dev,
                                  reduce=lambda i, x: ops.display_shard_records(i, x, lo, V))
    ex = PeerRecordExchange(ids_h.numel())

    def step():
        i = ids_h.to(dev, non_blocking=True)
        rec = pipe.statistics(i, logits_h)
        c, p, u = ex.from_records(rec.view(-1, 4), i, shard_offsets=offs)
        refined = ops.refine_display_from_statistics(i, c, p, u, MASK_ID, EOS_ID, REVEAL,
                                                     REVISION, MARGIN)
        out_h.copy_(refined, non_blocking=True)

    try:
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            step()
        b.record()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / steps], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    finally:
        ex.close()
    total = batch * ids.shape[1] * V * logits.element_size()
    ids_bytes = ids_h.numel() * ids_h.element_size()
    del pipe, logits_h
    return {"value": round(total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": total + world * ids_bytes,
            "d2h_bytes_per_step": world * ids_bytes,
            "ms_per_step": round(ms, 3), "steps": steps,
            "sample": f"first {batch} of {ids.shape[0]} sequences on every rank (bytes: all ranks)",
            "api": "cid_engine.host_pipeline (display_shard_records) + "
                   "parallel.PeerRecordExchange.from_records + refine_display_from_statistics"}


def sharded_parity(ids: Tensor, logits: Tensor, offs: list[int], stats, rows: int = 256) -> dict:
    """Outside the timed region: the shard slices of ``rows`` rows spread
    over the tensor are gathered to every rank, reassembled into full
    vocabulary rows, and the unsharded single-GPU statistics of those rows
    are compared with the combined ones (argmax exactly; confidences within
    a pure relative 1e-5)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size()
    dev = logits.device
    n = ids.numel()
    sel = torch.linspace(0, n - 1, rows, device=dev).long()
    width = max(offs[r + 1] - offs[r] for r in range(world))
    mine = torch.zeros((rows, width), dtype=logits.dtype, device=dev)
    flat = logits.reshape(n, -1)
    mine[:, : flat.shape[1]] = flat[sel]
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine)
    full = torch.cat([parts[r][:, : offs[r + 1] - offs[r]] for r in range(world)], dim=1)
    sub_ids = ids.reshape(-1)[sel].view(1, rows)
    e_c, e_p, e_u = torch.ops.cid_engine.display_token_statistics(sub_ids, full.view(1, rows, -1))
    c, p, u = (t.reshape(-1)[sel] for t in stats)
    argmax_ok = bool(torch.equal(p, e_p.view(-1)))
    rel = max(float(((c - e_c.view(-1)).abs() / e_c.view(-1).abs()).max()),
              float(((u - e_u.view(-1)).abs() / e_u.view(-1).abs().clamp_min(1e-30)).max()))
    return {"rows": rows, "ok": argmax_ok and rel <= 1e-5, "argmax_exact": argmax_ok,
            "max_rel_diff": rel,
            "against": "display_token_statistics of the reassembled unsharded rows on one GPU"}


def bench_sharded_loop(rank: int, world: int, dev) -> dict:
    """Decode loop batch-sharded over the ranks: 256 / N sequences of 512
    positions over 32000 tokens per rank, 128 slots, 64 graph-replayed
    steps, no collective; steps/s of the whole job (max over ranks)."""
    import dataclasses

    import torch
    import torch.distributed as dist
    from cid_engine.loop import DisplayRefineLoop

    B = LOOP["B"]
    per = B // world
    lo, hi = rank * per, (rank + 1) * per
    ring = [loop_logits(k, dev)[lo:hi].contiguous() for k in range(3)]
    torch.cuda.empty_cache()
    ids0, slot = loop_state(dev)
    fields = {f.name: getattr(slot, f.name) for f in dataclasses.fields(slot)}
    for name, val in fields.items():
        if isinstance(val, torch.Tensor) and name != "semantic_indices":
            fields[name] = val[lo:hi].contiguous()
    slot = type(slot)(**fields)
    ids0 = ids0[lo:hi].contiguous()
    loop = DisplayRefineLoop(ids0, ring, slots=slot, host_snapshots=4, use_graphs=True,
                             mask_token_id=MASK_ID, eos_token_id=EOS_ID, reveal_fraction=REVEAL,
                             revision_fraction=REVISION, revision_margin=MARGIN)
    try:
        loop.run(3)
        loop.drain()
        loop.reset(ids0, slot.occupancy)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        steps = LOOP["steps"]
        a.record()
        loop.run(steps)
        b.record()
        torch.cuda.synchronize()
        loop.drain()
    finally:
        loop.close()
    t = torch.tensor([a.elapsed_time(b) / steps], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    peak, _ = _peaks()
    logits_bytes = B * LOOP["L"] * LOOP["V"] * 2
    del ring
    torch.cuda.empty_cache()
    return {"workload": f"refine loop B=256 L=512 V=32000 bf16, S=128, 64 steps, "
                        f"{per} sequences per rank",
            "api": "cid_engine.DisplayRefineLoop (CUDA-graph replay)",
            "graph_steps_per_s": round(1e3 / ms, 2), "graph_ms_per_step": round(ms, 4),
            "logits_GBps": round(logits_bytes / (ms * 1e-3) / 1e9, 1),
            "roofline_steps_per_s": round(world * peak * 1e9 / logits_bytes, 1),
            "scaling": "strong (256 sequences in total), no collective", "timing": "max over ranks"}


def bench_vocab_parallel(args, display_inputs, ClockSampler, peaks, run_cpu_baseline) -> dict:
    import statistics as pystats
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    from cid_engine.parallel import PeerRecordExchange, vocab_parallel_refine

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        B, L, V = SHARDED["B"], SHARDED["L"], SHARDED["V"]
        ids, logits, offs = sharded_display_inputs(B, L, V, rank, world, 3, dev)
        peers = getattr(args, "exchange", "peers") == "peers"
        ex = PeerRecordExchange(B * L) if peers else None
        ops = torch.ops.cid_engine

        def step(ev):
            if ex is None:
                vocab_parallel_refine(ids, logits, total_vocab=V, mask_token_id=MASK_ID,
                                      eos_token_id=EOS_ID, reveal_fraction=REVEAL,
                                      revision_fraction=REVISION, revision_margin=MARGIN,
                                      timing=ev)
                return None
            c, p, u = ex.statistics(ids, logits, vocab_offset=offs[rank], total_vocab=V,
                                    shard_offsets=offs, timing=ev)
            ops.refine_display_from_statistics(ids, c, p, u, MASK_ID, EOS_ID, REVEAL, REVISION,
                                               MARGIN)
            if ev is not None and len(ev) > 3:
                ev[3].record()
            return c, p, u

        K, W = args.steps, args.warmup
        for _ in range(W):
            step(None)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        nev = 4 if peers else 2
        evs = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(nev)) for _ in range(K)]
        with ClockSampler(local) as clk:
            clk.mark_start()
            a.record()
            for k in range(K):
                step(evs[k])
            b.record()
            torch.cuda.synchronize()
            clk.mark_end()
        dist.barrier()
        torch.cuda.synchronize()
        ms_local = a.elapsed_time(b) / K
        kern_local = pystats.mean(e[0].elapsed_time(e[1]) for e in evs)
        stage = [kern_local]
        if peers:
            stage += [pystats.mean(e[1].elapsed_time(e[2]) for e in evs),
                      pystats.mean(e[2].elapsed_time(e[3]) for e in evs)]
        t = torch.tensor([ms_local, kern_local], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, kern_ms = float(t[0]), float(t[1])
        st = torch.tensor([ms_local, *stage], device=dev, dtype=torch.float64)
        st_all = [torch.empty_like(st) for _ in range(world)]
        dist.all_gather(st_all, st)
        stages = [{"rank": r, "step_ms": round(float(x[0]), 4), "records_ms": round(float(x[1]), 4),
                   **({"combine_ms": round(float(x[2]), 4), "refine_ms": round(float(x[3]), 4)}
                      if peers else {})} for r, x in enumerate(st_all)]
        # correctness outside the timed region: one more step's statistics
        # against the unsharded statistics of 256 reassembled rows
        if peers:
            stats = step(None)
        else:
            from cid_engine.parallel import vocab_parallel_statistics

            stats = vocab_parallel_statistics(ids, logits, total_vocab=V)
        torch.cuda.synchronize()
        parity = sharded_parity(ids, logits, offs, stats)
        if ex is not None:
            ex.close()
        e2e = None
        if not args.no_e2e:
            e2e = e2e_vocab_parallel(ids, logits, offs, rank, batch=16,
                                     steps=max(20, args.e2e_steps), warmup=2)
        total_bytes = B * L * V * 2
        shard_bytes = logits.numel() * 2
        del logits, stats
        torch.cuda.empty_cache()
        loop = None if args.no_loop else bench_sharded_loop(rank, world, dev)
        peak, peak_kind = peaks()
        rows = B * L
        alg = shard_bytes + rows * (8 + 16)
        achieved = alg / (kern_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC,
            "value": round(total_bytes / (ms * 1e-3) / 1e9, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": K,
            "warmup": W,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded bf16 2*N(0,1) logits, 5% planted peaks)",
            "config": {"workload": "vocab-parallel display stats + refine, logits bf16 [64,4096,152064]",
                       "batch": B, "tokens": L, "vocab": V,
                       "parallelism": f"vocab-sharded x{world} " + (
                           "(16 B row records stored into every rank's inbox by the statistics "
                           "kernel over NVLink; no collective in the step)" if peers else
                           "(NCCL all-gather of 16 B row records)"),
                       "l2": f"{shard_bytes / 1e9:.1f} GB per rank per step >> 126 MB L2"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "frac_of_8TBps_nominal": round(achieved / 8000.0, 4),
                         "traffic": (round(NCU_SHARD_TRAFFIC_PER_ROW[world] * rows)
                                     if world in NCU_SHARD_TRAFFIC_PER_ROW else None),
                         "kernel": "display_stats_rows_kernel<bf16, records> (per rank, max over ranks"
                                   + ("; records stored into every rank's inbox)" if peers else ")"),
                         "peak_kind": peak_kind, "kernel_ms": round(kern_ms, 4),
                         "algorithmic_bytes_per_launch": alg},
            "parity": parity,
            "stages": stages,
            "e2e": e2e,
            # records (storing into every inbox), publish, flag wait, merge,
            # refine (peers); records, combine, refine (NCCL; its all-gather
            # kernel is NCCL's)
            "gpu_launches": (5 if peers else 3) * K,
            "clocks": clk.summary(),
            "refine_loop": loop,
        }
        if rank == 0 and not args.no_cpu_baseline:
            line["cpu_baseline"] = run_cpu_baseline(sample=(1, 512, V), seconds=args.cpu_seconds)
        dist.barrier()
        return line
    finally:
        dist.destroy_process_group()


def profile_case(name: str) -> None:
    """Small launches for ncu: three statistics launches on rows of 128256, large enough to leave L2 (CTA-per-row kernel: [1, 4096, 128256]
    bf16, 1.05 GB; warp-per-row kernel: [1, 10240, 128256] bf16, 2.6 GB)."""
    import torch

    import cid_engine

    if name == "refine":  # refinement alone: warp rows [1, 64], [64, 128]; CTA rows [32, 1024], [64, 4096]
        g = torch.Generator(device="cuda").manual_seed(1)
        for B, L in ((1, 64), (64, 128), (32, 1024), (64, 4096)):
            ids = torch.randint(2, 32000, (B, L), generator=g, device="cuda")
            ids[torch.rand((B, L), generator=g, device="cuda") < 0.6] = MASK_ID
            ids[:, L // 2 + 7] = EOS_ID
            conf = torch.rand((B, L), generator=g, device="cuda")
            cur = torch.rand((B, L), generator=g, device="cuda") * conf
            pred = torch.randint(2, 32000, (B, L), generator=g, device="cuda")
            for _ in range(3):
                out = cid_engine.refine_display_from_statistics(
                    ids, conf, pred, cur, mask_token_id=MASK_ID, eos_token_id=EOS_ID,
                    reveal_fraction=REVEAL, revision_fraction=REVISION, revision_margin=MARGIN)
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": name, "checksum": int(out.sum())}))
        return
    if name == "lm_head":  # fused LM head + statistics: rows 8192, vocab 128256, hidden 4096
        g = torch.Generator(device="cuda").manual_seed(1)
        h = (torch.randn(8192, 4096, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
        w = (torch.randn(128256, 4096, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
        ids = torch.randint(0, 128256, (8192,), generator=g, device="cuda")
        for _ in range(3):
            c, p, u = cid_engine.lm_head_display_statistics(ids, h, w)
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": name, "mean_conf": float(c.mean())}))
        return
    if name == "corruption":  # training corruption, two launches of each kernel (eager),
        # then masked diffusion captured in a CUDA graph (one kernel) and replayed twice
        sys.path.insert(0, str(ROOT / "tests" / "golden"))
        import cases

        ops = torch.ops.cid_engine
        md = [a.cuda() if isinstance(a, torch.Tensor) else a for a in cases.masked_diffusion_64x2048()]
        gd = torch.Generator().manual_seed(11)
        B3, T3, V3 = 64, 2048, 50257
        dc = [torch.randint(0, V3, (B3, T3), generator=gd), torch.rand(B3, generator=gd),
              torch.rand(B3, T3, generator=gd) > 0.15, torch.rand(B3, T3, generator=gd),
              torch.rand(B3, T3, generator=gd), torch.randint(1, V3, (B3, T3), generator=gd)]
        dc = [t.cuda() for t in dc]
        th = [t.cuda() for t in cases.thought_4x32x512()]
        for _ in range(2):
            m = ops.masked_diffusion_corrupt_from_random(*md)
            d = ops.display_corrupt_from_random(*dc, V3 - 1, EOS_ID, V3, 0.25)
            t = ops.thought_corrupt_from_epsilon(*th)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            mg = ops.masked_diffusion_corrupt_from_random(*md)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        same = all(torch.equal(a, b) for a, b in zip(m, mg))
        del graph
        print(json.dumps({"profile_case": name, "masked": int(m[1].sum()),
                          "replaced": int(d[3].sum()), "thought": float(t[0].sum()),
                          "graph_equals_eager": same}))
        return
    if name == "decode64":  # decode shape: [1, 64, 155136] bf16, three launches over 16 copies
        ids = decode_ids(64, 16, "cuda")
        ring = [decode_logits(64, k, "cuda") for k in range(16)]
        for k in range(3):
            c, p, u = cid_engine.display_token_statistics(ids, ring[k * 5])
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": name, "mean_conf": float(c.mean())}))
        return
    if name.startswith("shard"):  # a rank's record kernel at N ranks: rows of 152064 / N, 2.5 GB
        world = int(name[5:])
        V = SHARDED["V"] // world
        n = 8192 * world
        g = torch.Generator(device="cuda").manual_seed(world)
        lg = torch.randn((1, n, V), generator=g, device="cuda", dtype=torch.bfloat16) * 2
        ids = torch.randint(0, SHARDED["V"], (1, n), device="cuda")
        for _ in range(3):
            r = cid_engine.display_shard_records(ids, lg, vocab_offset=0, total_vocab=SHARDED["V"])
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": name, "checksum": int(r[:, 2].sum())}))
        return
    shape = {"cta": (1, 4096, 128256), "rows": (1, 10240, 128256),
             "rows_records": (1, 10240, 128256)}[name]
    g = torch.Generator(device="cuda").manual_seed(1)
    lg = torch.randn(shape, generator=g, device="cuda", dtype=torch.bfloat16) * 2
    ids = torch.randint(0, shape[2], shape[:2], device="cuda")
    for _ in range(3):
        if name == "rows_records":  # the same rows reduced to shard records
            r = cid_engine.display_shard_records(ids, lg, vocab_offset=0, total_vocab=shape[2])
            c = r[:, 0].view(torch.float32)
        else:
            c, p, u = cid_engine.display_token_statistics(ids, lg)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": name, "shape": shape, "mean_conf": float(c.mean())}))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-loop", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--exchange", choices=("peers", "nccl"), default="peers",
                    help="N>1: record exchange inside the statistics kernel (peers) or NCCL all-gather")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--cpu-min-reps", type=int, default=3)
    ap.add_argument("--cpu-worker", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--ref-cuda-worker", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--profile-case", choices=("cta", "rows", "rows_records", "lm_head", "refine", "corruption",
                             "decode64", "shard2", "shard4", "shard8"), default=None,
                    help="run a small statistics case for ncu and exit")
    ap.add_argument("--sample-b", type=int, default=1)
    ap.add_argument("--sample-l", type=int, default=1024)
    ap.add_argument("--sample-v", type=int, default=128256)
    ap.add_argument("--sample-gen", choices=("cpu", "cuda"), default="cpu")
    ap.add_argument("--sample-world", type=int, default=0)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.cpu_worker:
        cpu_reference_worker(args)
        return
    if args.ref_cuda_worker:
        ref_cuda_worker(args)
        return
    if args.profile_case:
        profile_case(args.profile_case)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    line_out = sys.stdout
    if world > 1:
        # Libraries write to file descriptor 1 during set-up (NCCL's version
        # banner at communicator creation): send that to stderr and keep the
        # original stdout for the one JSON line.
        sys.stdout.flush()
        line_out = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(bench_reference(args, world)), file=line_out, flush=True)
        return
    if world > 1:
        line = bench_vocab_parallel(args, display_inputs, ClockSampler, _peaks,
                                             run_cpu_baseline)
        if rank == 0:
            print(json.dumps(line), file=line_out, flush=True)
        return
    print(json.dumps(bench_single(args)))


if __name__ == "__main__":
    main()
