"""ctypes binding of libpad_b200.so (declared in include/pad_b200.h).

This is the whole native boundary: plain pointers, sizes and strides go in, a
status code comes out. The library must have been built (``pad_b200.build``);
there is no fallback implementation -- if the library is missing the import
fails loudly.
"""

from __future__ import annotations

import ctypes
import os

from .build import LIB_PATH, OPS_PATH

_c_i64 = ctypes.c_int64
_c_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p

PAD_OK = 0
PAD_ERR_INVALID_ARGUMENT = 1
PAD_ERR_UNSUPPORTED = 2
PAD_ERR_WORKSPACE = 3
PAD_ERR_CUDA = 4

PAD_FLAG_BAD_PAGE_ID = 0x1
PAD_FLAG_SEQ_LEN_RANGE = 0x2
PAD_FLAG_WAIT_TIMEOUT = 0x100

# (name, restype, argtypes) for every symbol the header declares
SIGNATURES = {
    "pad_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "pad_last_error": (ctypes.c_char_p, []),
    "pad_version": (ctypes.c_int, []),
    "pad_device_info": (ctypes.c_int, [ctypes.c_int, _c_i64, _c_i64, ctypes.POINTER(ctypes.c_int),
                                       ctypes.POINTER(ctypes.c_int)]),
    "pad_decode_partitions": (ctypes.c_int, [ctypes.c_int] + [_c_i64] * 7 + [_c_i64p]),
    "pad_decode_workspace_bytes": (ctypes.c_int, [ctypes.c_int] + [_c_i64] * 7 + [ctypes.POINTER(ctypes.c_size_t)]),
    "pad_paged_attention_decode": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp] + [_c_i64] * 7
                                   + [_c_i64p, _c_i64p, _c_i64p, _c_i64, _c_i64p, ctypes.c_float, _c_i64,
                                      _vp, ctypes.c_size_t, _vp, _vp]),
    "pad_decode_csr_workspace_bytes": (ctypes.c_int, [ctypes.c_int] + [_c_i64] * 7 + [ctypes.POINTER(ctypes.c_size_t)]),
    "pad_paged_attention_decode_csr": (ctypes.c_int, [_vp] * 7 + [_c_i64] * 7
                                       + [_c_i64p, _c_i64p, _c_i64p, _c_i64p, ctypes.c_float, _c_i64, _vp,
                                          ctypes.c_size_t, _vp, _vp]),
    "pad_paged_kv_append": (ctypes.c_int, [_vp] * 6 + [_c_i64] * 6 + [_c_i64p] * 4 + [_c_i64, _vp, _vp]),
    "pad_paged_attention_decode_noalloc": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp] + [_c_i64] * 7
                                           + [_c_i64p, _c_i64p, _c_i64p, _c_i64, _c_i64p, ctypes.c_float,
                                              _c_i64, _vp, _vp]),
}

# Bytes of the library's built-in scratch used by pad_paged_attention_decode_noalloc.
PAD_STATIC_SCRATCH_BYTES = 16 << 20

_lib = None
_ops = None


class PadError(RuntimeError):
    """A status code other than PAD_OK from libpad_b200."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python paged-attention-decode_b200/pad_b200/build.py` "
                              "(there is no non-CUDA fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def ops():
    """torch.ops.pad_b200 -- the torch operator library over the C ABI
    (_pad_torch_ops.so, which links libpad_b200.so). Fails loudly if it has
    not been built."""
    global _ops
    if _ops is None:
        load()
        if not os.path.exists(OPS_PATH):
            raise ImportError(f"{OPS_PATH} is missing: build it with `python paged-attention-decode_b200/pad_b200/build.py`")
        import torch

        torch.ops.load_library(OPS_PATH)
        _ops = torch.ops.pad_b200
    return _ops


def check(status: int) -> None:
    if status != PAD_OK:
        lib = load()
        msg = lib.pad_last_error().decode(errors="replace")
        kind = lib.pad_status_string(status).decode()
        raise PadError(status, f"libpad_b200: {kind}: {msg}")


def i64_array(values) -> ctypes.Array:
    return (ctypes.c_int64 * len(values))(*[int(v) for v in values])
