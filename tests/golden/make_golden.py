"""Generate tests/golden/golden.pt from the reference's own CPU backend.

Run in the development container, where the reference checkout exists:

    make -C oracle ref            # builds oracle/_ref/libcid_engine_ref.so
    python tests/golden/make_golden.py

The reference library registers ``torch.ops.cid_engine`` itself, so this
script must run in a process that has not loaded this repository's
extension; it is a standalone script for that reason.  For every case in
``cases.py`` it stores a digest of the inputs and the reference's outputs
(small tensors in full; large integer outputs as a SHA-256 plus a strided
sample; large float outputs as a strided sample of 16384 values).
"""

from __future__ import annotations

import sys
import time
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(HERE))

import cases  # noqa: E402

def encode(t: torch.Tensor):
    t = t.detach().contiguous()
    limit = (1 << 14) if t.is_floating_point() else (1 << 12)
    if t.numel() <= limit:
        return {"full": t.clone()}
    step = -(-t.numel() // (limit // 4 if not t.is_floating_point() else limit))
    return {
        "sha256": cases.digest([t]),
        "shape": tuple(t.shape),
        "dtype": str(t.dtype),
        "step": step,
        "sample": t.flatten()[::step].clone(),
    }


def main() -> None:
    lib = REPO / "oracle" / "_ref" / "libcid_engine_ref.so"
    if not lib.exists():
        raise SystemExit("build the reference first: make -C oracle ref")
    torch.ops.load_library(str(lib))
    torch.set_num_threads(8)
    out: dict[str, dict] = {}
    t0 = time.time()
    for case in cases.all_cases():
        fn = getattr(torch.ops.cid_engine, case.op)
        entry: dict = {"op": case.op, "digest": cases.digest(case.args)}
        try:
            result = fn(*case.args, **case.kwargs)
        except Exception as exc:  # the reference raised: record the class
            entry["error"] = type(exc).__name__
        else:
            if isinstance(result, torch.Tensor):
                result = (result,)
            entry["out"] = [encode(r) for r in result]
        out[case.name] = entry
    torch.save(out, HERE / "golden.pt")
    print(f"{len(out)} cases in {time.time() - t0:.1f}s -> {HERE / 'golden.pt'}")


if __name__ == "__main__":
    main()
