"""Sanitizer-checked fuzzing of the C ABI's host-side validation (no GPU).

The counterpart of the reference's libFuzzer target over its C++ core
(tests/fuzz/fuzz_engine.cpp:279-307 of fwerkor/cid-engine v1.1.0, built with
``-fsanitize=address,undefined`` by CMakeLists.txt:31-52).  The kernels'
host code (every entry point of ``include/cid_engine_b200.h``) is compiled
with AddressSanitizer and UndefinedBehaviorSanitizer, linked with the
byte-driven harness ``tests/cpp/capi_fuzz.c`` and run over seeded random
inputs with no GPU visible: arguments outside the header's contract must be
rejected before any CUDA call, valid ones accepted, and no host read or
arithmetic may leave its bounds.  ``CID_ENGINE_CAPI_FUZZ_INPUTS`` sets the
number of inputs (default 300000).
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
KERNELS = ROOT / "cid-engine_b200" / "csrc" / "kernels"
HARNESS = ROOT / "tests" / "cpp" / "capi_fuzz.c"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = CUDA_HOME / "bin" / "nvcc"
SANITIZE = "-fsanitize=address,undefined"
INPUTS = int(os.environ.get("CID_ENGINE_CAPI_FUZZ_INPUTS", "300000"))


def _run(cmd: list[str], cwd: Path) -> None:
    out = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    assert out.returncode == 0, f"{' '.join(cmd)}\n{out.stdout}\n{out.stderr}"


@pytest.fixture(scope="module")
def harness(tmp_path_factory) -> Path:
    if not NVCC.exists() or shutil.which("gcc") is None:
        pytest.skip("nvcc and gcc are needed to build the sanitizer harness")
    work = tmp_path_factory.mktemp("capi_fuzz")
    # one -Xcompiler per flag: nvcc splits a -Xcompiler value at commas
    host_flags = [x for f in ("-fsanitize=address", "-fsanitize=undefined",
                              "-fno-sanitize-recover=all", "-fno-omit-frame-pointer")
                  for x in ("-Xcompiler", f)]
    sources = sorted(KERNELS.glob("*.cu"))
    cmds = [
        [str(NVCC), "-gencode", "arch=compute_100a,code=sm_100a", "-O1", "-std=c++17",
         "--extended-lambda", *host_flags, f"-I{ROOT / 'include'}", f"-I{KERNELS}",
         "-c", str(src), "-o", f"{src.stem}.o"]
        for src in sources
    ]
    cmds.append(["gcc", "-std=c11", "-O1", "-g", SANITIZE, "-fno-sanitize-recover=all",
                 "-fno-omit-frame-pointer", f"-I{ROOT / 'include'}", "-c", str(HARNESS),
                 "-o", "capi_fuzz.o"])
    with cf.ThreadPoolExecutor(max_workers=len(cmds)) as pool:
        list(pool.map(lambda c: _run(c, work), cmds))
    objects = [f"{src.stem}.o" for src in sources] + ["capi_fuzz.o"]
    _run(["g++", SANITIZE, *objects, f"-L{CUDA_HOME / 'lib64'}", "-lcudart_static", "-ldl",
          "-lpthread", "-lrt", "-o", "capi_fuzz"], work)
    return work / "capi_fuzz"


def test_c_abi_validation_under_sanitizers(harness: Path) -> None:
    env = dict(os.environ)
    env.update(CUDA_VISIBLE_DEVICES="", ASAN_OPTIONS="detect_leaks=0:abort_on_error=1",
               UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1")
    for seed in (1, 2):
        out = subprocess.run([str(harness), str(INPUTS // 2), str(seed)], env=env,
                             capture_output=True, text=True, timeout=900)
        assert out.returncode == 0, out.stdout + out.stderr[-6000:]
        assert "every result within the contract" in out.stdout
