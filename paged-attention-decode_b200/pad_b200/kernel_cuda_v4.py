"""Drop-in replacement for the reference's ``src/kernel_cuda_v4.py``.

``paged_attention_decode_cuda_v4(q, k_cache, v_cache, block_table, seq_lens,
num_splits=None, scale=None)`` keeps the reference signature and contract
(src/kernel_cuda_v4.py:19-65): fp16 CUDA tensors in, a new fp16 ``out``
shaped like ``q`` back, ``scale=None`` meaning ``1/sqrt(head_dim)``, Python
``assert`` for the caller-contract checks the reference asserts
(src/kernel_cuda_v4.py:37-48), ``block_table``/``seq_lens`` cast to int32
(src/kernel_cuda_v4.py:58-59).

Differences, by design:
  * ``num_splits=None`` selects the B200 heuristic (one persistent partition
    per resident CTA slot, stream-K balanced) instead of the reference's
    fixed 64; an explicit ``num_splits=S`` launches ``S * batch * Hkv``
    partitions, i.e. S splits per (sequence, KV head) pair for uniform
    batches, exactly as the reference's grid.z = S did.
  * The call goes through the torch operator ``torch.ops.pad_b200.decode``
    (csrc/pad_torch_op.cpp, host C++ over the C ABI of libpad_b200.so), which
    launches on the current torch stream of ``q``'s device and keeps one
    reusable workspace per (device, stream).
  * Argument errors the native library detects raise RuntimeError (the
    operator's TORCH_CHECK, like the reference's, cuda/kernel_v4_split_k.cu:216-223).
  * With ``PAD_B200_CHECK=1`` in the environment the call synchronises and
    raises ValueError for invalid block-table page ids or out-of-range
    seq_lens -- the value checks of the reference oracle
    (src/reference.py:40-41,107-112); off by default because it syncs.
"""

from __future__ import annotations

import math
import os

import torch

from . import _lib

_SUPPORTED_HEAD_DIMS = (16, 32, 64, 128)
_OPS = _lib.ops()
_CHECK_VALUES = os.environ.get("PAD_B200_CHECK", "0") not in ("", "0")


_WS_CACHE: dict[tuple, int] = {}


def workspace_bytes(device_index: int, batch: int, num_kv_heads: int, gqa_ratio: int, head_dim: int,
                    page_size: int, max_pages: int, num_splits: int) -> int:
    key = (device_index, batch, num_kv_heads, gqa_ratio, head_dim, page_size, max_pages, num_splits)
    n = _WS_CACHE.get(key)
    if n is None:
        lib = _lib.load()
        out = _lib.ctypes.c_size_t(0)
        _lib.check(lib.pad_decode_workspace_bytes(device_index, batch, num_kv_heads, gqa_ratio, head_dim,
                                                  page_size, max_pages, num_splits, _lib.ctypes.byref(out)))
        n = _WS_CACHE[key] = int(out.value)
    return n


def partitions(device_index: int, batch: int, num_kv_heads: int, gqa_ratio: int, head_dim: int,
               page_size: int, max_pages: int, num_splits: int | None = None) -> int:
    """Number of persistent partitions (CTAs) a call with these sizes launches."""
    lib = _lib.load()
    out = _lib.ctypes.c_int64(0)
    _lib.check(lib.pad_decode_partitions(device_index, batch, num_kv_heads, gqa_ratio, head_dim, page_size,
                                         max_pages, 0 if num_splits is None else num_splits,
                                         _lib.ctypes.byref(out)))
    return int(out.value)


def _raise_for_flags(flags: int) -> None:
    if flags & _lib.PAD_FLAG_BAD_PAGE_ID:
        raise ValueError("block_table contains an invalid physical page id")
    if flags & _lib.PAD_FLAG_SEQ_LEN_RANGE:
        raise ValueError("seq_lens contains negative values or values larger than block_table can address")
    if flags & _lib.PAD_FLAG_WAIT_TIMEOUT:
        raise RuntimeError("libpad_b200: an in-kernel wait timed out")


def paged_attention_decode_cuda_v4(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    num_splits: int | None = None,
    scale: float | None = None,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Decode attention over a paged fp16 KV cache with GQA on a B200.

    q [B, Hq, D] fp16, k_cache/v_cache [num_pages, page_size, Hkv, D] fp16,
    block_table [B, max_pages] int, seq_lens [B] int -> out [B, Hq, D] fp16.
    """
    assert q.is_cuda and k_cache.is_cuda and v_cache.is_cuda, "pad_b200 requires CUDA tensors"
    assert q.dtype == torch.float16 and k_cache.dtype == torch.float16 and v_cache.dtype == torch.float16, (
        "pad_b200 expects fp16 q/k_cache/v_cache"
    )
    assert q.dim() == 3 and k_cache.dim() == 4, "q must be [B, Hq, D] and k_cache [num_pages, page_size, Hkv, D]"
    assert v_cache.shape == k_cache.shape, "v_cache must have k_cache's shape"
    batch, num_q_heads, head_dim = q.shape
    num_pages, page_size, num_kv_heads, cache_head_dim = k_cache.shape
    assert cache_head_dim == head_dim, "q head_dim must match the KV cache head_dim"
    assert num_q_heads % num_kv_heads == 0, "num_q_heads must be divisible by num_kv_heads (GQA)"
    assert head_dim in _SUPPORTED_HEAD_DIMS, f"head_dim must be one of {_SUPPORTED_HEAD_DIMS}"
    assert block_table.dim() == 2 and block_table.shape[0] == batch, "block_table must be [B, max_pages]"
    assert seq_lens.dim() == 1 and seq_lens.shape[0] == batch, "seq_lens must be [B]"
    assert num_splits is None or num_splits >= 1, "num_splits must be >= 1"
    assert out is None or (out.shape == q.shape and out.dtype == torch.float16), "bad out tensor"
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    if _CHECK_VALUES:
        read_error_flags(q.device)
    out = _OPS.decode(q, k_cache, v_cache, block_table, seq_lens, 0 if num_splits is None else int(num_splits),
                      float(scale), out)
    if _CHECK_VALUES:
        _raise_for_flags(read_error_flags(q.device))
    return out


def read_error_flags(device: torch.device | None = None, reset: bool = True) -> int:
    """PAD_FLAG_* bits the kernels raised on ``device``'s current stream since the last reset (syncs)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    flags = _OPS.error_flags(dev.index)
    v = int(flags.item())
    if reset:
        flags.zero_()
    return v


def paged_kv_indices(block_table: torch.Tensor, seq_lens: torch.Tensor, page_size: int):
    """Dense block table + seq_lens -> CSR (indptr, indices, last_page_len).

    The conversion of the reference's FlashInfer adapter
    (src/flashinfer_adapter.py:40-65): sequence b uses its first
    ceil(seq_len/page_size) block-table entries; last_page_len lies in
    [1, page_size] (page_size for an empty sequence, which has no pages)."""
    sl = seq_lens.to(torch.int64)
    pages = (sl + page_size - 1) // page_size
    mask = torch.arange(block_table.shape[1], device=block_table.device)[None, :] < pages[:, None]
    indices = block_table[mask].to(torch.int32)
    indptr = torch.zeros(block_table.shape[0] + 1, dtype=torch.int32, device=block_table.device)
    indptr[1:] = torch.cumsum(pages, 0).to(torch.int32)
    last = (sl - (pages - 1) * page_size).to(torch.int32)
    return indptr, indices, last


def paged_attention_decode_csr(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    kv_indptr: torch.Tensor,
    kv_indices: torch.Tensor,
    kv_last_page_len: torch.Tensor,
    num_splits: int | None = None,
    scale: float | None = None,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Decode over a paged fp16 KV cache addressed by a CSR page index
    (kv_indptr [B+1], kv_indices [nnz], kv_last_page_len [B], int32) --
    the format of the reference's FlashInfer comparison path -- on the same
    B200 kernel as paged_attention_decode_cuda_v4."""
    assert q.is_cuda and k_cache.is_cuda and v_cache.is_cuda, "pad_b200 requires CUDA tensors"
    assert q.dtype == torch.float16 and k_cache.dtype == torch.float16 and v_cache.dtype == torch.float16, (
        "pad_b200 expects fp16 q/k_cache/v_cache"
    )
    batch, num_q_heads, head_dim = q.shape
    num_pages, page_size, num_kv_heads, _ = k_cache.shape
    assert v_cache.shape == k_cache.shape and k_cache.shape[3] == head_dim
    assert num_q_heads % num_kv_heads == 0, "num_q_heads must be divisible by num_kv_heads (GQA)"
    assert head_dim in _SUPPORTED_HEAD_DIMS, f"head_dim must be one of {_SUPPORTED_HEAD_DIMS}"
    assert kv_indptr.shape == (batch + 1,) and kv_last_page_len.shape == (batch,), "bad CSR shapes"
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    out = _OPS.decode_csr(q, k_cache, v_cache, kv_indptr, kv_indices, kv_last_page_len,
                          0 if num_splits is None else int(num_splits), float(scale), out)
    if _CHECK_VALUES:
        _raise_for_flags(read_error_flags(q.device))
    return out


def paged_kv_append(k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_table: torch.Tensor, positions: torch.Tensor) -> None:
    """Write token positions[b] (k_new/v_new [B, Hkv, D] fp16) of every
    sequence into the paged caches in place; positions[b] < 0 skips b."""
    assert k_new.is_cuda and k_cache.is_cuda and k_new.dtype == torch.float16 and k_cache.dtype == torch.float16
    assert v_new.shape == k_new.shape and v_cache.shape == k_cache.shape
    batch, hkv, d = k_new.shape
    num_pages, page_size, cache_hkv, cache_d = k_cache.shape
    assert (cache_hkv, cache_d) == (hkv, d), "k_new must be [B, Hkv, D] matching the cache"
    _OPS.kv_append(k_new, v_new, k_cache, v_cache, block_table, positions)
    if _CHECK_VALUES:
        _raise_for_flags(read_error_flags(k_cache.device))
