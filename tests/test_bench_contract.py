"""The bench's reference arm on the host cores: one JSON line with the keys
the benchmark contract names, on the B200 arm's metric, unit and workload.

The reference arm times the reference's CPU backend (built from its sources
into oracle/_ref); the test is skipped where that build is absent.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
REF_LIB = ROOT / "oracle" / "_ref" / "libcid_engine_ref.so"


@pytest.mark.skipif(not REF_LIB.exists(), reason="reference CPU backend not built")
def test_reference_arm_prints_one_contract_line() -> None:
    sys.path.insert(0, str(ROOT))
    import bench

    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "3",
         "--warmup", "3", "--cpu-seconds", "1"],
        capture_output=True, text=True, timeout=600, cwd=ROOT,
    )
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e", "impl"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "GB/s"
    assert d["higher_is_better"] is True
    assert (d["n_gpus"], d["steps"], d["warmup"]) == (1, 3, 3)
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"].startswith("display stats + refine, logits bf16 [32,1024,128256]")
    cpu = d["cpu_baseline"]
    assert cpu["kind"] == "reference" and cpu["cores"] >= 1 and cpu["sample"]
    assert cpu["value"] == pytest.approx(d["value"], rel=1e-3)
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
