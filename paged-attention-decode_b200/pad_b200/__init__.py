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
    """The reference's Triton-v4 signature (src/kernel_v4_split_k.py:213-222)
    routed to the same B200 kernel; ``block_n`` is accepted for call
    compatibility (the B200 kernel's token tile is fixed at 64)."""
    assert block_n & (block_n - 1) == 0 and block_n >= 16, "block_n must be a power of 2 and >= 16"
    return paged_attention_decode_cuda_v4(q, k_cache, v_cache, block_table, seq_lens, num_splits, scale)


__all__ = ["paged_attention_decode_cuda_v4", "paged_attention_decode_v4", "paged_attention_decode_csr",
           "paged_kv_indices", "paged_kv_append", "partitions", "workspace_bytes",
           "read_error_flags", "PadError"]
