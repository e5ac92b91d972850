"""ctypes binding of libsplax_b200.so, the C ABI declared in include/splax_b200.h.

There is no fallback: if the library is missing, or no CUDA device is present, every entry
point raises. Arrays cross the boundary as raw device pointers plus their leading lengths,
exactly as the XLA FFI bridge of the reference hands Warp the collapsed vmap batches.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libsplax_b200.so"

SPLAX_OK = 0
SPLAX_ERR_INVALID_ARGUMENT = 1
SPLAX_ERR_KEY_OVERFLOW = 2
SPLAX_ERR_OUT_OF_MEMORY = 3
SPLAX_ERR_CUDA = 4
SPLAX_ERR_DEVICE = 5
SPLAX_ERR_COUNT_OVERFLOW = 6

P, I64, I32, F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float

# name -> argument types, in the order of include/splax_b200.h
SIGNATURES: dict[str, list] = {
    "splax_project": [P, I64, P, I64, P, I64, P, I64, P, I64, P, I64, P, I32, I32, I32, I32, I32,
                      F32, F32, F32, F32, F32, F32, I64, P, P, P, P, P, P, P],
    "splax_project_noalloc": [P, I64, P, I64, P, I64, P, I64, P, I64, P, I64, P, I32, I32, I32,
                              I32, I32, F32, F32, F32, F32, F32, F32, I64, P, P, P, P, P, P, P],
    "splax_project_bwd": [P, I64, P, I64, P, I64, P, I64, P, I64, P, I64, P, I64, P, I64, P, I64,
                          P, I64, P, I32, I32, I32, F32, F32, F32, I64, P, P, P, P, P, P],
    "splax_project_ex": [P, I64, P, I64, P, I64, P, I64, P, I64, P, I64, P, I32, I32, I32, I32,
                         I32, F32, F32, F32, F32, F32, F32, I64, P, P, P, P, P, P, I32, F32, F32,
                         P, P],
    "splax_project_bwd_ex": [P, I64, P, I64, P, I64, P, I64, P, I64, P, I64, P, I64, P, I64, P,
                             I64, P, I64, F32, F32, P, I64, P, I32, I32, I32, F32, F32, F32, I64,
                             I32, I32, P, P, P, P, P, P],
    "splax_rasterize": [P, I64, P, I64, P, I64, P, I64, P, P, P, P, P, I64, I32, I32, I32, I64,
                        I32, P, P, P, P],
    "splax_rasterize_depth": [P, I64, P, I64, P, I64, P, I64, P, P, P, P, P, I64, I32, I32, I32,
                              I64, I32, P, P, P, P, P],
    "splax_rasterize_bwd": [P, I64, P, I64, P, I64, P, I64, P, P, P, P, P, I64, P, P, P, I64, I32,
                            I32, I32, I64, I32, P, P, P, P, P],
    "splax_rasterize_bwd_depth": [P, I64, P, I64, P, I64, P, I64, P, P, P, P, P, I64, P, P, P,
                                  I64, P, I64, I32, I32, I32, I64, I32, P, P, P, P, P, P],
    "splax_rasterize_bwd_ex": [P, I64, P, I64, P, I64, P, I64, P, P, P, P, P, I64, P, P, P, I64,
                               P, I64, I32, I32, I32, I64, I32, I32, I32, P, P, P, P, P, P],
    "splax_sort_and_bin": [P, P, P, P, P, I64, P, I32, I32, I32, I32, I32, P, I64, P, P, P, P, P],
    "splax_clear_cache": [],
    "splax_scratch_info": [P, I32],
    "splax_check_device_errors": [P],
    "splax_debug_fail_alloc_after": [I64],
    "splax_last_sort_token": [],
    "splax_reuse_sort": [I64],
    "splax_profile_enable": [I32, I32],
    "splax_profile_stages": [ctypes.c_uint32],
    "splax_profile_reset": [],
    "splax_profile_report": [P, I32],
    "splax_mse_loss": [P, P, I64, F32, P, P],
    "splax_l1_dssim_loss": [P, P, I32, I32, I32, I32, F32, P, P],
    "splax_l1_dssim_loss_bwd": [P, P, I32, I32, I32, I32, F32, P, P, P],
    "splax_l1_dssim_loss_and_grad": [P, P, I32, I32, I32, I32, F32, P, P, P],
    "splax_adam_step": [I32, P, P, P, P, P, P, I32, F32, F32, F32, P],
    "splax_nvls_allreduce_f32": [P, P, I32, I32, I64, ctypes.c_uint64, P, P],
    "splax_nvls_adam_step": [P, P, P, P, P, I64, I32, P, P, I32, F32, F32, F32, P, I32, I32,
                             ctypes.c_uint64, P, P],
    "splax_nvls_adam_shard_len": [I64, I32, I32, P],
    "splax_ply_info": [ctypes.c_char_p, P],
    "splax_ply_load": [ctypes.c_char_p, I64, P, P, P, P, P, P],
    "splax_mse_loss_bwd": [P, P, I64, F32, P, P, P],
    "splax_last_error": [],
    "splax_version": [],
}

_lib: ctypes.CDLL | None = None


class SplaxDeviceError(RuntimeError):
    """A device-side check of the CUDA path failed (see the message)."""


def load() -> ctypes.CDLL:
    """Load the in-tree library; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH.name} is not built: run `python -c 'import __graft_entry__ as g; g.build()'`"
            " (there is no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    lib.splax_last_error.restype = ctypes.c_char_p
    lib.splax_version.restype = ctypes.c_char_p
    lib.splax_clear_cache.restype = None
    lib.splax_debug_fail_alloc_after.restype = None
    lib.splax_profile_enable.restype = None
    lib.splax_profile_stages.restype = None
    lib.splax_last_sort_token.restype = ctypes.c_int64
    lib.splax_reuse_sort.restype = None
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc == SPLAX_OK:
        return
    msg = load().splax_last_error().decode()
    if rc in (SPLAX_ERR_INVALID_ARGUMENT, SPLAX_ERR_KEY_OVERFLOW):
        raise ValueError(msg)
    if rc == SPLAX_ERR_OUT_OF_MEMORY:
        raise torch.cuda.OutOfMemoryError(msg)
    if rc in (SPLAX_ERR_DEVICE, SPLAX_ERR_COUNT_OVERFLOW):
        raise SplaxDeviceError(msg)
    raise RuntimeError(msg)


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def stream_of(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("splax_b200 runs on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all operands must live on the same CUDA device")
    if dev is None:
        raise ValueError("no CUDA operand given")
    return dev


def profile_enable(timing: bool = True, count_work: bool = False) -> None:
    """Switch on per-launch CUDA-event timing and / or the instrumented work counters."""
    load().splax_profile_enable(int(timing), int(count_work))


STAGES = ("project_fwd", "project_bwd", "depth_minmax", "pair_keys", "pair_sort", "pair_scan",
          "emit_keys", "radix_sort", "tile_bins", "raster_fwd", "raster_bwd", "loss", "optim",
          "allreduce")


def profile_stages(names=None) -> None:
    """Time only the named stages (all when None); the others add no events to the streams."""
    mask = 0xFFFFFFFF if names is None else sum(1 << STAGES.index(n) for n in names)
    load().splax_profile_stages(mask)


def profile_reset() -> None:
    check(load().splax_profile_reset())


def profile_report() -> dict:
    """Per-kernel launches / ms and the work units since the last reset (current device)."""
    import json

    buf = ctypes.create_string_buffer(1 << 14)
    k = load().splax_profile_report(buf, len(buf))
    if k < 0:
        check(-k)
    return json.loads(buf.value.decode())
