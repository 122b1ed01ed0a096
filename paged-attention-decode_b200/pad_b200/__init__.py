"""pad_b200 -- paged-attention decode for NVIDIA B200 (sm_100a).

The public call is the reference project's wrapper signature
(src/kernel_cuda_v4.py:19-27)::

    from pad_b200 import paged_attention_decode_cuda_v4
    out = paged_attention_decode_cuda_v4(q, k_cache, v_cache, block_table, seq_lens,
                                         num_splits=None, scale=None)

backed by the C-ABI library libpad_b200.so (include/pad_b200.h).
"""

from .kernel_cuda_v4 import (paged_attention_decode_csr, paged_attention_decode_cuda_v4, paged_kv_append, paged_kv_indices,  # noqa: F401
                             partitions, read_error_flags, workspace_bytes)
from ._lib import PadError  # noqa: F401


def paged_attention_decode_v4(q, k_cache, v_cache, block_table, seq_lens, num_splits=16, scale=None, block_n=128):
    """The reference's Triton-v4 call surface (src/kernel_v4_split_k.py:213-222)
    on the B200 kernel.

    Same defaults (``num_splits=16``, ``scale=None`` meaning 1/sqrt(D)) and the
    same caller-contract asserts (src/kernel_v4_split_k.py:245-259): power-of-two
    head_dim and page_size, ``block_n`` a power of two >= 16. ``block_n`` is the
    Triton kernel's token tile; the B200 kernel chooses its own tile (128
    (token, KV head) rows: 128 / HG tokens for HG KV heads per tile), so the
    value is validated and then has no effect on the result or the launch.
    """
    assert q.is_cuda and k_cache.is_cuda and v_cache.is_cuda, "kernel_v4_split_k requires CUDA tensors"
    assert num_splits >= 1, "num_splits must be >= 1"
    head_dim, page_size = q.shape[-1], k_cache.shape[1]
    assert head_dim & (head_dim - 1) == 0, "head_dim must be a power of 2"
    assert page_size & (page_size - 1) == 0, "page_size must be a power of 2"
    assert block_n & (block_n - 1) == 0 and block_n >= 16, "block_n must be a power of 2 and >= 16"
    return paged_attention_decode_cuda_v4(q, k_cache, v_cache, block_table, seq_lens, num_splits, scale)


__all__ = ["paged_attention_decode_cuda_v4", "paged_attention_decode_v4", "paged_attention_decode_csr",
           "paged_kv_indices", "paged_kv_append", "partitions", "workspace_bytes",
           "read_error_flags", "PadError"]
