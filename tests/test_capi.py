"""The C-ABI library loads without a GPU and exports every declared symbol.

``include/cid_engine_b200.h`` is the drop-in boundary; every ``CID_API``
declaration there must be exported by ``libcid_engine_b200.so``.  Argument
validation happens on the host before any CUDA call, so invalid arguments are
rejected here without a device.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "cid_engine_b200.h"
LIB = ROOT / "cid-engine_b200" / "cid_engine" / "libcid_engine_b200.so"

CID_OK, CID_ERR_INVALID_ARGUMENT, CID_ERR_UNSUPPORTED_DTYPE = 0, 1, 2


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^CID_API\s+[\w\s\*]+?\b(cid_\w+)\s*\(", text, flags=re.M)


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    assert LIB.exists(), "build first: python cid-engine_b200/build.py"
    return ctypes.CDLL(str(LIB))


def test_header_declares_the_boundary() -> None:
    names = declared_symbols()
    assert len(names) == len(set(names))
    for op in (
        "cid_display_token_statistics",
        "cid_display_token_statistics_with_repetition",
        "cid_refine_display",
        "cid_prefix_allocation_mask",
        "cid_rollout_slot_transition",
        "cid_live_slot_occupancy",
        "cid_materialize_cell_snapshot",
        "cid_masked_diffusion_corrupt",
        "cid_thought_corrupt",
        "cid_display_corrupt",
        "cid_display_shard_records",
        "cid_display_combine_records",
    ):
        assert op in names


def test_every_declared_symbol_is_exported(lib: ctypes.CDLL) -> None:
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_only_the_c_abi_is_exported() -> None:
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True)
    exported = {ln.split()[-1] for ln in out.stdout.splitlines() if " T " in ln}
    assert exported == set(declared_symbols())


def test_version_and_strings(lib: ctypes.CDLL) -> None:
    assert lib.cid_abi_version() == 1
    lib.cid_result_string.restype = ctypes.c_char_p
    assert lib.cid_result_string(0) == b"ok"
    assert lib.cid_result_string(1) == b"invalid argument"


def test_host_validation_rejects_without_a_device(lib: ctypes.CDLL) -> None:
    null = ctypes.c_void_p(0)
    i64, dbl = ctypes.c_int64, ctypes.c_double
    # threshold outside [0, 1] (csrc/ops.cpp:50)
    rc = lib.cid_prefix_allocation_mask(0, null, i64(1), i64(1), 0, null, i64(1), i64(1),
                                        i64(1), i64(4), dbl(1.5), i64(1), null, null)
    assert rc == CID_ERR_INVALID_ARGUMENT
    # max_allocations <= 0 (csrc/ops.cpp:51)
    rc = lib.cid_prefix_allocation_mask(0, null, i64(1), i64(1), 0, null, i64(1), i64(1),
                                        i64(1), i64(4), dbl(0.5), i64(0), null, null)
    assert rc == CID_ERR_INVALID_ARGUMENT
    # refine fractions (csrc/refine.cpp:240-244)
    rc = lib.cid_refine_display(null, null, null, null, i64(1), i64(4), i64(0), 0, i64(-1),
                                dbl(1.5), dbl(0.1), dbl(0.0), null, null)
    assert rc == CID_ERR_INVALID_ARGUMENT
    rc = lib.cid_refine_display(null, null, null, null, i64(1), i64(4), i64(0), 0, i64(-1),
                                dbl(0.5), dbl(0.1), dbl(-1.0), null, null)
    assert rc == CID_ERR_INVALID_ARGUMENT
    # masked diffusion ratio range (csrc/ops.cpp:416-420)
    rc = lib.cid_masked_diffusion_corrupt(null, null, null, i64(2), i64(4), i64(9), dbl(0.0),
                                          dbl(1.0), null, null, null, null, null, null)
    assert rc == CID_ERR_INVALID_ARGUMENT
    # repetition multiplier in (0, 1] (csrc/ops.cpp:484-486)
    rc = lib.cid_display_token_statistics_with_repetition(
        3, null, i64(8), null, i64(1), i64(2), i64(8), i64(0), 0, i64(-1), dbl(1.5),
        null, null, null, null, null)
    assert rc == CID_ERR_INVALID_ARGUMENT
    # integer logits are not a statistics dtype
    rc = lib.cid_display_token_statistics(5, null, i64(8), null, i64(1), i64(8), null, null,
                                          null, null, null)
    assert rc == CID_ERR_UNSUPPORTED_DTYPE
    # empty inputs are a no-op (no launch)
    rc = lib.cid_display_token_statistics(3, null, i64(8), null, i64(0), i64(8), null, null,
                                          null, null, null)
    assert rc == CID_OK
    lib.cid_masked_diffusion_workspace_bytes.restype = ctypes.c_size_t
    assert lib.cid_masked_diffusion_workspace_bytes(i64(64)) == 64 * 8


def test_peer_inbox_layout_sizes() -> None:
    """Inbox bytes: records [2][world][capacity] x 16 B + a 256-byte tail."""
    import ctypes

    lib = ctypes.CDLL(str(LIB))
    lib.cid_peer_inbox_bytes.restype = ctypes.c_size_t
    lib.cid_peer_inbox_bytes.argtypes = [ctypes.c_int, ctypes.c_int64]
    assert lib.cid_peer_inbox_bytes(2, 100) == 2 * 2 * 100 * 16 + 256
    assert lib.cid_peer_inbox_bytes(8, 262144) == 2 * 8 * 262144 * 16 + 256
    assert lib.cid_peer_inbox_bytes(9, 10) == 0 and lib.cid_peer_inbox_bytes(0, 10) == 0
