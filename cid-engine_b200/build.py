"""In-tree build of the B200 extension.

Produces, inside ``cid-engine_b200/cid_engine/``:

* ``libcid_engine_b200.so`` — the sm_100a kernels behind the C ABI of
  ``include/cid_engine_b200.h`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``,
  static CUDA runtime, no torch dependency);
* ``_C.<abi>.so`` — the C++20 torch host (operator registration, validation,
  launches), linked against the library above with ``$ORIGIN`` rpath.

Usage: ``python cid-engine_b200/build.py [--force] [-j N]``.  Objects go to
``cid-engine_b200/_build/``; only stale outputs are rebuilt.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
KERNELS = CSRC / "kernels"
OUT_DIR = PKG_ROOT / "cid_engine"
BUILD = PKG_ROOT / "_build"
INCLUDE = REPO / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = CUDA_HOME / "bin" / "nvcc"
CXX = os.environ.get("CID_CXX", "/usr/bin/g++")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH, "-O3", "-lineinfo", "-std=c++17", "--extended-lambda", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}", f"-I{KERNELS}",
]

LIB_NAME = "libcid_engine_b200.so"
EXT_SUFFIX = sysconfig.get_config_var("EXT_SUFFIX") or ".so"


def _torch_dirs() -> tuple[Path, Path]:
    import torch

    root = Path(torch.__file__).resolve().parent
    return root / "include", root / "lib"


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(" ".join(map(str, cmd)) + "\n" + res.stdout + res.stderr)
        raise SystemExit(f"build failed: {cmd[0]}")


def _headers() -> list[Path]:
    return [*KERNELS.glob("*.cuh"), *INCLUDE.glob("*.h"), *(CSRC / "include").rglob("*.hpp")]


def build(force: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    jobs = jobs or min(8, os.cpu_count() or 4)

    # 1. kernels -> C-ABI shared library
    cu_sources = sorted(KERNELS.glob("*.cu"))
    cu_objs = [BUILD / (s.stem + ".cu.o") for s in cu_sources]
    todo = [
        (s, o) for s, o in zip(cu_sources, cu_objs) if force or _stale(o, [s, *headers])
    ]
    lib = OUT_DIR / LIB_NAME

    # 2. torch host translation units
    tinc, tlib = _torch_dirs()
    py_inc = sysconfig.get_paths()["include"]
    cxx_flags = [
        "-std=c++20", "-O2", "-fPIC", "-fvisibility=hidden", "-D_GLIBCXX_USE_CXX11_ABI=1",
        "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_C",
        f"-I{CSRC / 'include'}", f"-I{INCLUDE}", f"-I{tinc}",
        f"-I{tinc / 'torch' / 'csrc' / 'api' / 'include'}", f"-I{CUDA_HOME / 'include'}",
        f"-I{py_inc}",
    ]
    cpp_sources = [CSRC / n for n in ("ops.cpp", "refine.cpp", "registration.cpp", "bindings.cpp")]
    cpp_objs = [BUILD / (s.stem + ".cpp.o") for s in cpp_sources]
    todo_cpp = [
        (s, o) for s, o in zip(cpp_sources, cpp_objs) if force or _stale(o, [s, *headers])
    ]

    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        futs = [ex.submit(_run, [str(NVCC), *NVCC_FLAGS, "-c", str(s), "-o", str(o)]) for s, o in todo]
        futs += [ex.submit(_run, [CXX, *cxx_flags, "-c", str(s), "-o", str(o)]) for s, o in todo_cpp]
        for f in futs:
            f.result()

    if force or _stale(lib, cu_objs):
        _run([str(NVCC), *ARCH, "-shared", "-cudart", "static", "-o", str(lib), *map(str, cu_objs),
              "-Xlinker", "-z,defs", "-lrt", "-lpthread", "-ldl"])

    ext = OUT_DIR / ("_C" + EXT_SUFFIX)
    if force or _stale(ext, [*cpp_objs, lib]):
        _run([
            CXX, "-shared", "-o", str(ext), *map(str, cpp_objs),
            f"-L{OUT_DIR}", "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN",
            f"-L{tlib}", f"-Wl,-rpath,{tlib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
            "-ltorch_cuda", "-ltorch_python",
        ])
    return ext


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.j))


if __name__ == "__main__":
    main()
