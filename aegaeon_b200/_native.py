"""ctypes binding of ``libaegaeon_b200.so`` (the C ABI declared in ``include/aegaeon_b200.h``).

The library is loaded from the package directory. If it is missing the import of this module
fails loudly; there is no fallback implementation of any operation.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libaegaeon_b200.so")

AEG_OK = 0
AEG_ERR_INVALID_ARGUMENT = 1
AEG_ERR_CUDA = 2
AEG_ERR_UNSUPPORTED = 3

AEG_DTYPE_FP16 = 0
AEG_DTYPE_BF16 = 1

AEG_DEVERR_BLOCK_ID_RANGE = 0x1
AEG_DEVERR_SLOT_RANGE = 0x2
AEG_DEVERR_SEQ_LEN_RANGE = 0x4
AEG_DEVERR_WAIT_TIMEOUT = 0x8
AEG_DEVERR_PLAN_MISMATCH = 0x10

AEG_DECODE_PREFETCH = 0x1
AEG_DECODE_PREFETCH_AFTER_DECODE_WRITE = 0x2

AEG_IPC_HANDLE_BYTES = 96

AEG_COPY_ENGINE_DMA = 0
AEG_COPY_ENGINE_SM = 1

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/aegaeon_b200.h one to one.
SIGNATURES = {
    "aeg_version": (_i32, []),
    "aeg_last_error": (ctypes.c_char_p, []),
    "aeg_read_device_errors": (_i32, [_c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "aeg_swap": (_i32, [_c_void_p, _c_void_p, _sz, _i64, _i64, _c_void_p, _c_void_p, _i64, _i32, _c_void_p]),
    "aeg_swap_sm": (_i32, [_c_void_p, _c_void_p, _sz, _i64, _i64, _c_void_p, _c_void_p, _i64, _i32, _c_void_p]),
    "aeg_copy_blocks": (_i32, [_c_void_p, _sz, _i64, _c_void_p, _c_void_p, _i64, _c_void_p]),
    "aeg_ipc_export": (_i32, [_c_void_p, _c_void_p]),
    "aeg_ipc_open": (_i32, [_c_void_p, ctypes.POINTER(_c_void_p), ctypes.POINTER(_i64)]),
    "aeg_ipc_close": (_i32, [_c_void_p]),
    "aeg_migrate_blocks": (_i32, [_c_void_p, _i64, _c_void_p, _i64, _sz, _c_void_p, _c_void_p, _i64, _c_void_p]),
    "aeg_migrate_blocks_dma": (_i32, [_c_void_p, _i64, _c_void_p, _i64, _sz, _c_void_p, _c_void_p, _i64, _c_void_p]),
    "aeg_prefill_attention": (_i32, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64,
                                     _i32, _i32, _i32, _i32, _i32, ctypes.c_float, _i32, _c_void_p]),
    "aeg_copy_segments_workspace_size": (_sz, [_i64]),
    "aeg_copy_segments": (_i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i32, _c_void_p, _sz,
                                 _c_void_p]),
    "aeg_prepare_step_inputs": (_i32, [_c_void_p, _i32, _c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p, _i64,
                                       _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "aeg_update_block_tables": (_i32, [_c_void_p, _i32, _i32, _c_void_p, _i64, _c_void_p]),
    "aeg_reshape_and_cache": (_i32, [_c_void_p, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64, _i64,
                                     _c_void_p, _i64, _i32, _i32, _c_void_p]),
    "aeg_decode_workspace_size": (_sz, [_i32, _i32, _i32, _i32]),
    "aeg_decode_plan": (_i32, [_c_void_p, _sz, _c_void_p, _i32, _c_void_p, _i32, _i32, _i32, _i32, _c_void_p]),
    "aeg_paged_attn_decode": (_i32, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i64,
                                     _c_void_p, _i32, _c_void_p, _i32, _i32, _i32, _i32, ctypes.c_float, _i32,
                                     _c_void_p, _sz, _i32, _c_void_p]),
    "aeg_decode_layer": (_i32, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _c_void_p,
                                _c_void_p, _i64, _i64, _c_void_p, _i32, _c_void_p, _i32, _i32, _i32, _i32,
                                ctypes.c_float, _i32, _c_void_p, _sz, _i32, _c_void_p]),
    "aeg_paged_attn_decode_noalloc": (_i32, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i64,
                                             _c_void_p, _i32, _c_void_p, _i32, _i32, _i32, _i32, ctypes.c_float,
                                             _i32, _c_void_p]),
}


class AegaeonError(RuntimeError):
    """A CUDA-side failure reported by the library (status AEG_ERR_CUDA)."""


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"aegaeon_b200 native library not found at {LIB_PATH}; build it with "
            "`python -m aegaeon_b200.build` (there is no non-CUDA fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error() -> str:
    msg = lib.aeg_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    """Raises the Python exception matching a non-zero aeg_status."""
    if status == AEG_OK:
        return
    msg = f"{what}: {last_error()}"
    if status == AEG_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if status == AEG_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise AegaeonError(msg)
