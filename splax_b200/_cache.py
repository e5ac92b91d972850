"""Persistent scratch cache of the CUDA path (splax/_cache.py:1-164).

The storage itself lives in libsplax_b200, per device: grow-only sort keys and values with
1.25x headroom, tile bins, depth ranges and packed blend records, keyed on the (B, n, tiles)
signature and dropped when it changes. ``clear_cache`` keeps the reference's signature.
"""

from __future__ import annotations

import ctypes

import torch

from splax_b200 import _lib


def clear_cache() -> None:
    """Release the persistent sort and bin scratch buffers on all devices."""
    _lib.load().splax_clear_cache()


def scratch_info(device: int | torch.device | None = None) -> dict:
    """The current device's scratch entry: capacity, key dtype, bytes held and signature."""
    lib = _lib.load()
    out = (ctypes.c_int64 * 6)()
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        k = lib.splax_scratch_info(out, 6)
    if k < 0:
        _lib.check(-k)
    cap, kb, nbytes, B, n, T = list(out)
    return {
        "isect_cap": cap,
        "isect_dtype": {32: torch.int32, 64: torch.int64}.get(kb),
        "bytes": nbytes,
        "sig": (B, n, T) if B >= 0 else None,
    }
