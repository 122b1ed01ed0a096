"""CPU oracle for paged-attention decode -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this package; the shipped decode path never does.

* ``pa_oracle.paged_attention_decode_reference`` -- numpy restatement of the
  reference's fp32 oracle (src/reference.py:8-54).
* ``decode_c`` -- the same algorithm in C + pthreads (``pa_oracle.c``), used as
  the timed CPU baseline and for the larger parity cases.
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

from .pa_oracle import paged_attention_decode_reference, sdpa_style_oracle, validate_inputs  # noqa: F401

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libpa_oracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile ``libpa_oracle.so`` with the committed Makefile."""
    src = os.path.join(_HERE, "pa_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "all"], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(_LIB_PATH)
        argt = [ctypes.c_void_p] * 6 + [ctypes.c_int64] * 7 + [ctypes.c_float, ctypes.c_int]
        for name in ("pa_oracle_decode_f16", "pa_oracle_decode_f32"):
            fn = getattr(lib, name)
            fn.argtypes = argt
            fn.restype = ctypes.c_int
        lib.pa_oracle_max_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def max_threads() -> int:
    return int(_load().pa_oracle_max_threads())


def decode_c(q, k_cache, v_cache, block_table, seq_lens, scale=None, nthreads: int = 0):
    """Run the C oracle on numpy arrays (fp16 or fp32, contiguous). Returns fp32 [B,Hq,D]."""
    lib = _load()
    q = np.ascontiguousarray(q)
    k_cache = np.ascontiguousarray(k_cache)
    v_cache = np.ascontiguousarray(v_cache)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    if not (q.dtype == k_cache.dtype == v_cache.dtype) or q.dtype not in (np.float16, np.float32):
        raise TypeError("q, k_cache and v_cache must share dtype float16 or float32")
    batch, hq, d = q.shape
    num_pages, ps, hkv, _ = k_cache.shape
    out = np.empty((batch, hq, d), dtype=np.float32)
    s = (1.0 / math.sqrt(d)) if scale is None else float(scale)
    fn = lib.pa_oracle_decode_f16 if q.dtype == np.float16 else lib.pa_oracle_decode_f32
    rc = fn(q.ctypes.data, k_cache.ctypes.data, v_cache.ctypes.data, bt.ctypes.data, sl.ctypes.data,
            out.ctypes.data, batch, hq, hkv, d, num_pages, ps, bt.shape[1], s, nthreads)
    if rc == -1:
        raise ValueError("block_table contains an invalid physical page id")
    if rc == -3:
        raise ValueError("seq_lens contains values larger than block_table can address")
    if rc != 0:
        raise ValueError(f"oracle rejected the arguments (status {rc})")
    return out
