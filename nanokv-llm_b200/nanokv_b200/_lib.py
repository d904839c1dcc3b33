"""ctypes binding of libnkv.so, the C ABI declared in include/nkv.h.

This is the only module that talks to the shared library. It loads the
in-tree build (never a fallback implementation): if the library is missing or
lacks a symbol, loading fails loudly.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_size_t, c_uint32, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libnkv.so"

NKV_OK = 0
STATUS_NAMES = {
    0: "NKV_OK",
    1: "NKV_ERR_INVALID_ARGUMENT",
    2: "NKV_ERR_UNSUPPORTED",
    3: "NKV_ERR_WORKSPACE",
    4: "NKV_ERR_ALIGNMENT",
    5: "NKV_ERR_CUDA",
}

DEVERR_STORE_SLOT = 0x1
DEVERR_DECODE_BLOCK = 0x2
DEVERR_WAIT_TIMEOUT = 0x4
DEVERR_COMPRESS_RANGE = 0x8
DEVERR_RING_RANGE = 0x10
DEVERR_PREFILL_RANGE = 0x20
DEVERR_ROPE_POSITION = 0x40
DEVERR_LAUNCH_SHAPE = 0x80

# Size of the library's fixed decode scratch (NKV_STATIC_SCRATCH_BYTES, nkv.h).
STATIC_SCRATCH_BYTES = 16 << 20

_P = c_void_p
_I32P = c_void_p  # device int32 pointers are passed as raw addresses

# name -> (restype, argtypes); mirrors include/nkv.h one to one.
SIGNATURES: dict[str, tuple] = {
    "nkv_status_string": (ctypes.c_char_p, [c_int]),
    "nkv_abi_version": (c_int, []),
    "nkv_last_cuda_error": (c_int, []),
    "nkv_read_device_error": (c_int, [POINTER(c_uint32), c_int]),
    "nkv_store_kvcache": (
        c_int,
        [_P, c_int64, _P, c_int64, _P, _P, c_int64, _I32P, c_int32, c_int32, c_int32, _P],
    ),
    "nkv_paged_decode_workspace_size": (
        c_size_t,
        [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32],
    ),
    "nkv_paged_decode": (
        c_int,
        [_P, c_int64, c_int64, _P, _P, c_int64, _I32P, c_int32, _I32P, _P, c_int64,
         c_int32, c_int32, c_int32, c_int32, c_int32, c_float, _P, c_size_t, _P],
    ),
    "nkv_decode_step": (
        c_int,
        [_P, c_int64, c_int64, _P, c_int64, _P, c_int64, _I32P, _P, _P, c_int64, _I32P, c_int32,
         _I32P, _P, c_int32, c_int32, c_int32, c_int32, _I32P, _I32P, _P, c_int64,
         c_int32, c_int32, c_int32, c_int32, c_int32, c_float, c_int32, _P, c_size_t, _P],
    ),
    "nkv_qk_norm_rope_store": (
        c_int,
        [_P, c_int64, c_int32, _P, _P, c_int64, _P, _P, c_float, _P, c_int64, _P, c_int64,
         _P, _P, c_int64, _I32P, c_int32, c_int32, c_int32, _P],
    ),
    "nkv_oproj_allreduce": (
        c_int,
        [_P, c_int64, _P, c_int64, c_int32, c_int32, c_int32, _P, _P, _P, _P, _P, _P, _P,
         c_int32, c_int32, c_uint64, _P, c_int64, _P, c_int64, _P],
    ),
    "nkv_oproj_allreduce_p2p": (
        c_int,
        [_P, c_int64, _P, c_int64, c_int32, c_int32, c_int32, _P, c_int64, _P, _P, _P,
         c_int32, c_int32, c_uint64, _P, c_int64, _P, c_int64, _P],
    ),
    "nkv_paged_prefill": (
        c_int,
        [_P, c_int64, c_int64, c_int64, _P, c_int64, _P, c_int64, c_int64, _I32P, c_int32,
         c_int32, _I32P, _I32P, c_int32, c_int32, c_int32, _P, c_int64, c_int32, c_int32,
         c_int32, c_float, _P],
    ),
    "nkv_window_compress": (
        c_int,
        [_P, c_int64, _P, _P, c_int64, _I32P, c_int32, _I32P, _I32P, _I32P, c_int32,
         c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_float,
         _I32P, _I32P, _P, _P],
    ),
    "nkv_window_select": (
        c_int,
        [_I32P, _I32P, c_int32, c_int32, c_int32, c_int32, _I32P, _I32P, _I32P, _P],
    ),
    "nkv_query_window_append": (
        c_int,
        [_P, c_int64, _P, c_int32, c_int32, c_int32, c_int32, _I32P, _I32P, _I32P,
         c_int32, c_int32, c_int32, _P],
    ),
    "nkv_paged_decode_static_scratch": (
        c_int,
        [_P, c_int64, c_int64, _P, _P, c_int64, _I32P, c_int32, _I32P, _P, c_int64,
         c_int32, c_int32, c_int32, c_int32, c_int32, c_float, _P],
    ),
    "nkv_threshold_compress": (
        c_int,
        [_P, c_int32, c_int32, c_int32, c_int32, _I32P, _P, _P, c_int64, _I32P, c_int32,
         _I32P, _I32P, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
         c_float, _I32P, _P, _P],
    ),
}

_lib = None


class NkvError(RuntimeError):
    """A non-zero nkv_status from the C ABI."""

    def __init__(self, fn: str, status: int, cuda_err: int = 0):
        name = STATUS_NAMES.get(status, f"status {status}")
        msg = f"{fn} failed: {name}"
        if cuda_err:
            msg += f" (cudaError {cuda_err})"
        super().__init__(msg)
        self.status = status
        self.cuda_error = cuda_err


def load(path: Path | str | None = None):
    """Loads libnkv.so once and binds every entry point of include/nkv.h."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"libnkv.so not found at {p}; build it with `python -m nanokv_b200.build` "
            "(the attention path has no fallback implementation)"
        )
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError here means a missing export
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(fn_name: str, status: int) -> None:
    if status != NKV_OK:
        raise NkvError(fn_name, status, load().nkv_last_cuda_error())


def read_device_error(clear: bool = True) -> int:
    """Sticky device error bits (NKV_DEVERR_*); synchronises the device."""
    bits = c_uint32(0)
    check("nkv_read_device_error", load().nkv_read_device_error(ctypes.byref(bits), int(clear)))
    return int(bits.value)
