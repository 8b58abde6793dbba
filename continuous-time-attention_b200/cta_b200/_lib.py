"""ctypes binding of libcta_stencil.so (the C ABI in include/cta_stencil.h).

Every entry point takes raw device pointers, sizes and element strides plus the
caller's CUDA stream; this module turns torch tensors into those arguments and
maps the library's status codes onto the exceptions the reference raises
(``ValueError`` for invalid arguments, ``RuntimeError`` otherwise).

There is no fallback: if the shared library is missing or fails to load, every
operator raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_float, c_int, c_int64, c_void_p
from pathlib import Path

import torch

import os

# CTA_STENCIL_LIB selects another build of the library (e.g. a tuning variant)
LIB_PATH = Path(os.environ.get("CTA_STENCIL_LIB") or Path(__file__).resolve().with_name("libcta_stencil.so"))

CTA_OK, CTA_EINVAL, CTA_EUNSUPPORTED, CTA_ECUDA = 0, 1, 2, 3
SHARD_INTERIOR, SHARD_LO_EDGE, SHARD_HI_EDGE = 0, 1, 2
PDE_ADVECTION, PDE_REACTION = 0, 1
MAX_STEPS = 8
PDE_STACK_MAX_STEPS = 4
ARITH_EXACT, ARITH_CONTRACTED = 0, 1
_ARITH_CODES = {"exact": ARITH_EXACT, "contracted": ARITH_CONTRACTED}

_DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
_MASK_CODES = {
    torch.bool: 0,
    torch.uint8: 0,
    torch.int8: 0,
    torch.int32: 1,
    torch.int64: 2,
    torch.float32: 3,
    torch.bfloat16: 4,
    torch.float16: 5,
}

# name -> (restype, argtypes); mirrors include/cta_stencil.h
_SIGNATURES = {
    "cta_abi_version": (c_int, []),
    "cta_last_error": (ctypes.c_char_p, []),
    "cta_device_error": (c_int, [c_int]),
    "cta_set_tuning": (c_int, [c_int, c_int]),
    "cta_set_arithmetic": (c_int, [c_int]),
    "cta_set_thread_arithmetic": (c_int, [c_int]),
    "cta_diffusion_fwd_bdl": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_int, c_float,
                                      c_void_p]),
    "cta_diffusion_bwd_bdl": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_int, c_float,
                                      c_void_p]),
    "cta_diffusion_bdl_ex": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
                                     c_int, c_int, POINTER(c_float), POINTER(c_void_p), c_int, c_void_p, c_int,
                                     c_int64, c_int64, c_void_p]),
    "cta_diffusion_fwd_bld": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
                                      c_int64, c_int, c_int, c_int, POINTER(c_float), POINTER(c_void_p), c_int,
                                      c_void_p, c_int, c_int64, c_int64, c_void_p]),
    "cta_diffusion_bwd_bld_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64, c_int, c_int, c_int]),
    "cta_diffusion_bwd_bld": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                      c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
                                      c_int, POINTER(c_float), POINTER(c_void_p), c_int, c_void_p, c_int, c_int64,
                                      c_int64, c_void_p]),
    "cta_diffusion_fwd_varlen": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_int64,
                                         c_int64, c_int, c_int, c_int, c_float, c_void_p]),
    "cta_diffusion_bwd_bld_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                              c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
                                              c_int, POINTER(c_float), POINTER(c_void_p), c_int, c_void_p, c_int,
                                              c_int64, c_int64, c_void_p]),
    "cta_diffusion_fwd_varlen_residual": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                                                  c_int64, c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_float,
                                                  c_void_p]),
    "cta_diffusion_fwd_bld_residual": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                                               c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
                                               POINTER(c_float), c_void_p, c_int, c_int64, c_int64, c_void_p]),
    "cta_pde_step_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "cta_pde_stack_bld": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
                                  c_int64, c_int, c_int, c_int, c_int, POINTER(c_void_p), POINTER(c_void_p), c_int,
                                  c_void_p, c_int, c_int64, c_int64, c_void_p]),
    "cta_pde_step_bld": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                                 c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int, c_int, c_int,
                                 c_void_p, c_void_p, c_int, c_void_p, c_int, c_int64, c_int64, c_void_p]),
    "cta_diffusion_fwd_bld_pool_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "cta_diffusion_fwd_bld_pool": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
                                           c_int64, c_int, c_int, POINTER(c_float), POINTER(c_void_p), c_int,
                                           c_void_p, c_int, c_int64, c_int64, c_void_p]),
    "cta_diffusion_shard_bld_dalpha": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                                               c_int64, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p,
                                               c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int, c_int, c_int,
                                               c_int, POINTER(c_float), c_void_p]),
    "cta_diffusion_shard_bld": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p,
                                        c_int64, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int, c_float,
                                        c_void_p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load (once) and return the shared library; raise if it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built (expected at {LIB_PATH}); run `python -m cta_b200.build`"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.cta_abi_version() != 1:
                raise RuntimeError(f"{LIB_PATH.name}: unexpected ABI version {lib.cta_abi_version()}")
            _lib = lib
    return _lib


def check(rc: int) -> None:
    """Raise the reference's exception type for a non-zero status."""
    if rc == CTA_OK:
        return
    msg = load().cta_last_error().decode(errors="replace")
    if rc == CTA_EINVAL:
        raise ValueError(msg)
    raise RuntimeError(msg)


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}; expected float32, bfloat16 or float16") from None


def mask_code(dt: torch.dtype) -> int:
    try:
        return _MASK_CODES[dt]
    except KeyError:
        raise ValueError(f"unsupported attention_mask dtype {dt}") from None


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(t: torch.Tensor) -> int:
    """The caller's current CUDA stream on t's device, as a raw cudaStream_t."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t: torch.Tensor | None) -> int:
    return t.data_ptr() if t is not None else 0


_float_arrays: dict = {}


def float_array(vals) -> ctypes.Array:
    """ctypes float[8] of the given host coefficients (cached, treat as read-only)."""
    key = tuple(float(v) for v in vals)
    arr = _float_arrays.get(key)
    if arr is None:
        arr = (c_float * MAX_STEPS)()
        for i, v in enumerate(key):
            arr[i] = v
        if len(_float_arrays) < 4096:
            _float_arrays[key] = arr
    return arr


class on_device:
    """Make t's device current for the call (no-op when it already is)."""

    __slots__ = ("idx", "prev")

    def __init__(self, t: torch.Tensor):
        self.idx = t.device.index
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


def ptr_array(tensors) -> ctypes.Array:
    arr = (c_void_p * MAX_STEPS)()
    for i, t in enumerate(tensors):
        arr[i] = t.data_ptr()
    return arr


def device_error(clear: bool = True) -> int:
    """Device-side error word (0 = ok, 1 = a bounded in-kernel wait timed out)."""
    return int(load().cta_device_error(1 if clear else 0))


def set_tuning(key: int, value: int) -> int:
    return int(load().cta_set_tuning(int(key), int(value)))


def arith_code(mode) -> int:
    """'exact' / 'contracted' (or the integer code) -> the C ABI's code."""
    if isinstance(mode, int) and mode in (ARITH_EXACT, ARITH_CONTRACTED):
        return mode
    try:
        return _ARITH_CODES[mode]
    except KeyError:
        raise ValueError(f"arithmetic must be 'exact' or 'contracted', got {mode!r}") from None


class thread_arithmetic:
    """Run the enclosed calls of this thread with the given forward arithmetic
    (None: leave the current setting), restoring the previous override after."""

    __slots__ = ("code", "prev")

    def __init__(self, mode):
        self.code = None if mode is None else arith_code(mode)
        self.prev = None

    def __enter__(self):
        if self.code is not None:
            self.prev = load().cta_set_thread_arithmetic(self.code)
        return self

    def __exit__(self, *exc):
        if self.code is not None:
            load().cta_set_thread_arithmetic(self.prev)
        return False
