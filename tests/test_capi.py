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


def test_host_validation_of_the_other_entry_points(lib: ctypes.CDLL) -> None:
    """Display corruption, linear assignment, thought corruption and the LM
    head reject invalid arguments before any CUDA call.  The LM-head checks
    never dereference their pointers, so 16-byte-aligned stand-in addresses
    are enough here."""
    null = ctypes.c_void_p(0)
    i64, dbl, c_int = ctypes.c_int64, ctypes.c_double, ctypes.c_int
    F32, I64 = 0, 5

    def display_corrupt(t_dtype, vocab, frac, rr=null, ro=null):
        return lib.cid_display_corrupt(null, t_dtype, null, 4, null, F32, null, F32, rr, ro,
                                       i64(2), i64(8), i64(0), c_int(1), i64(1), i64(vocab),
                                       dbl(frac), null, null, null, null, null)

    # replacement_fraction outside [0, 1] (csrc/ops.cpp:320-322)
    assert display_corrupt(F32, 100, 1.5) == CID_ERR_INVALID_ARGUMENT
    # replacement needs vocab >= 3 and both random tensors (csrc/ops.cpp:343-348)
    assert display_corrupt(F32, 2, 0.25, ctypes.c_void_p(16), ctypes.c_void_p(16)) == CID_ERR_INVALID_ARGUMENT
    assert display_corrupt(F32, 100, 0.25) == CID_ERR_INVALID_ARGUMENT
    # integer timesteps are not a floating dtype (csrc/ops.cpp:317-319)
    assert display_corrupt(I64, 100, 0.0) == CID_ERR_UNSUPPORTED_DTYPE

    # linear assignment: at most 16 columns, rows <= columns (csrc/ops.cpp:71-86)
    def assign(dtype, rows, cols):
        return lib.cid_batched_linear_assignment(dtype, null, null, i64(1), i64(rows),
                                                 i64(cols), null, null, null)

    assert assign(F32, 4, 17) == CID_ERR_INVALID_ARGUMENT
    assert assign(F32, 5, 4) == CID_ERR_INVALID_ARGUMENT
    assert assign(I64, 4, 4) == CID_ERR_UNSUPPORTED_DTYPE
    assert assign(F32, 0, 4) == CID_OK  # nothing to assign: no launch

    # thought corruption: semantic and timesteps must be floating
    rc = lib.cid_thought_corrupt(I64, null, F32, null, F32, null, null, i64(1), i64(8),
                                 null, null, null, null)
    assert rc == CID_ERR_UNSUPPORTED_DTYPE
    rc = lib.cid_thought_corrupt(F32, null, F32, null, F32, null, null, i64(-1), i64(8),
                                 null, null, null, null)
    assert rc == CID_ERR_INVALID_ARGUMENT

    # LM head: hidden width a multiple of 8 (16-byte TMA rows), 16-byte-aligned
    # operands, a workspace of cid_lm_head_workspace_bytes
    lib.cid_lm_head_workspace_bytes.restype = ctypes.c_size_t
    ws_need = lib.cid_lm_head_workspace_bytes(i64(4), i64(300))
    assert ws_need > 0

    def lm_head(hidden_dim, hidden_addr, ws_bytes):
        p = ctypes.c_void_p
        return lib.cid_lm_head_display_statistics(
            p(hidden_addr), i64(4), i64(hidden_dim), p(0x2000), i64(300), p(0x3000), c_int(1),
            p(0x4000), p(0x5000), p(0x6000), p(0x7000), ctypes.c_size_t(ws_bytes), null, null)

    assert lm_head(12, 0x1000, ws_need) == CID_ERR_INVALID_ARGUMENT
    assert lm_head(64, 0x1008, ws_need) == 4  # CID_ERR_MISALIGNED
    assert lm_head(64, 0x1000, ws_need - 1) == 6  # CID_ERR_SCRATCH_LIMIT


def test_peer_inbox_layout_sizes() -> None:
    """Inbox bytes: records [2][world][capacity] x 16 B + a 256-byte tail."""
    import ctypes

    lib = ctypes.CDLL(str(LIB))
    lib.cid_peer_inbox_bytes.restype = ctypes.c_size_t
    lib.cid_peer_inbox_bytes.argtypes = [ctypes.c_int, ctypes.c_int64]
    assert lib.cid_peer_inbox_bytes(2, 100) == 2 * 2 * 100 * 16 + 256
    assert lib.cid_peer_inbox_bytes(8, 262144) == 2 * 8 * 262144 * 16 + 256
    assert lib.cid_peer_inbox_bytes(9, 10) == 0 and lib.cid_peer_inbox_bytes(0, 10) == 0
