"""The allocation-free masked-diffusion entry point agrees with the regular one.

``cid_masked_diffusion_corrupt_no_alloc`` serves callers that cannot give the
library device memory for a workspace (a host program that owns all device
memory through its own pool, a serving loop that must not call cudaMalloc on
its request path, an FFI binding with no device allocator): its scratch is a
fixed array inside the library.  Both entry points are called here through
the C ABI with the same inputs, twice in a row with different inputs, and
must produce identical outputs (the kernels are deterministic, so the
tolerance is zero), on device 0 and, when a second GPU is visible, on device
1 too (the array's address is looked up per device).  This file is collected
last on purpose.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parent.parent / "cid-engine_b200" / "cid_engine" / "libcid_engine_b200.so"


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _inputs(seed: int, batch: int, tokens: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    clean = torch.randint(0, 50257, (batch, tokens), generator=g, device="cuda")
    ratio = torch.rand(batch, 1, generator=g, device="cuda")
    ratio[::7] = 0.0  # rows that take the empty-row fallback
    mask_random = torch.rand(batch, tokens, generator=g, device="cuda")
    return clean, ratio, mask_random


def _outputs(batch: int, tokens: int):
    return (
        torch.empty(batch, tokens, dtype=torch.int64, device="cuda"),
        torch.empty(batch, tokens, dtype=torch.bool, device="cuda"),
        torch.empty(batch, 1, dtype=torch.float32, device="cuda"),
        torch.empty(2, dtype=torch.float32, device="cuda"),
    )


def _call(lib, fn_name: str, inputs, outputs, lo: float, hi: float, workspace=None) -> int:
    clean, ratio, mask_random = inputs
    corrupted, masked, ratio_out, metrics = outputs
    batch, tokens = clean.shape
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [
        _ptr(clean), _ptr(ratio), _ptr(mask_random), ctypes.c_int64(batch),
        ctypes.c_int64(tokens), ctypes.c_int64(50256), ctypes.c_double(lo), ctypes.c_double(hi),
        _ptr(corrupted), _ptr(masked), _ptr(ratio_out), _ptr(metrics),
    ]
    if workspace is not None:
        args.append(_ptr(workspace))
    return getattr(lib, fn_name)(*args, stream)


def _devices() -> list[int]:
    """Device 0, and device 1 when a second GPU is visible (the scratch
    address is looked up and cached per device)."""
    return [0, 1] if torch.cuda.device_count() > 1 else [0]


@pytest.mark.parametrize("device", _devices())
def test_no_alloc_entry_point_matches_workspace_entry_point(device: int) -> None:
    assert torch.cuda.is_available()
    torch.cuda.set_device(device)
    lib = ctypes.CDLL(str(LIB))
    lib.cid_masked_diffusion_workspace_bytes.restype = ctypes.c_size_t
    for k, (batch, tokens) in enumerate(((64, 2048), (37, 333))):
        inputs = _inputs(100 + k, batch, tokens)
        ref_out = _outputs(batch, tokens)
        ws_bytes = lib.cid_masked_diffusion_workspace_bytes(ctypes.c_int64(batch))
        workspace = torch.empty(max(1, ws_bytes // 8), dtype=torch.int64, device="cuda")
        assert _call(lib, "cid_masked_diffusion_corrupt", inputs, ref_out, 1e-6, 1.0,
                     workspace) == 0
        no_alloc_out = _outputs(batch, tokens)
        assert _call(lib, "cid_masked_diffusion_corrupt_no_alloc", inputs, no_alloc_out,
                     1e-6, 1.0) == 0
        torch.cuda.synchronize()
        for a, b in zip(no_alloc_out, ref_out):
            torch.testing.assert_close(a, b, rtol=0, atol=0)
        assert bool(no_alloc_out[1].any(dim=1).all())  # fallback rows got one mask
    torch.cuda.set_device(0)


def test_no_alloc_entry_point_rejects_batches_beyond_its_scratch() -> None:
    lib = ctypes.CDLL(str(LIB))
    null = ctypes.c_void_p(0)
    rc = lib.cid_masked_diffusion_corrupt_no_alloc(
        null, null, null, ctypes.c_int64(65537), ctypes.c_int64(4), ctypes.c_int64(9),
        ctypes.c_double(0.1), ctypes.c_double(1.0), null, null, null, null, null)
    assert rc == 6  # CID_ERR_SCRATCH_LIMIT
    lib.cid_result_string.restype = ctypes.c_char_p
    assert b"CID_NO_ALLOC_MAX_BATCH" in lib.cid_result_string(6)
