"""Paged KV append (the cache writer the decode path reads from): a numpy
restatement of the write on CPU, GPU parity with it, and decode after append
against the oracle."""

import numpy as np
import pytest
import torch

import oracle
import pad_b200
from pad_b200.cases import explicit_case


def append_reference(k_new, v_new, k_cache, v_cache, block_table, positions):
    """Token positions[b] of sequence b -> page block_table[b, pos // ps], row pos % ps."""
    k, v = k_cache.copy(), v_cache.copy()
    ps = k.shape[1]
    for b, pos in enumerate(positions):
        if pos < 0:
            continue
        page = block_table[b, pos // ps]
        k[page, pos % ps] = k_new[b]
        v[page, pos % ps] = v_new[b]
    return k, v


@pytest.mark.gpu
@pytest.mark.parametrize("head_dim,page_size", [(128, 16), (64, 4), (32, 1), (16, 32)])
def test_append_then_decode(head_dim, page_size):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from gpu_utils import assert_parity

    seqs = [0, 15, 16, 99, 300]
    c = explicit_case([s + 1 for s in seqs], num_kv_heads=2, gqa_ratio=4, head_dim=head_dim, page_size=page_size,
                      seed=head_dim + page_size)
    rng = np.random.default_rng(5)
    k_new = rng.standard_normal((len(seqs), 2, head_dim), dtype=np.float32).astype(np.float16)
    v_new = rng.standard_normal((len(seqs), 2, head_dim), dtype=np.float32).astype(np.float16)
    positions = np.array(seqs, dtype=np.int32)
    positions[2] = -1  # skipped
    k_ref, v_ref = append_reference(k_new.astype(np.float32), v_new.astype(np.float32), c.k_cache, c.v_cache,
                                    c.block_table, positions)
    kc = torch.from_numpy(c.k_cache).half().cuda()
    vc = torch.from_numpy(c.v_cache).half().cuda()
    pad_b200.paged_kv_append(torch.from_numpy(k_new).cuda(), torch.from_numpy(v_new).cuda(), kc, vc,
                             torch.from_numpy(c.block_table).cuda(), torch.from_numpy(positions).cuda())
    np.testing.assert_array_equal(kc.float().cpu().numpy(), k_ref)
    np.testing.assert_array_equal(vc.float().cpu().numpy(), v_ref)
    # decode over the appended cache (seq_len = position + 1)
    sl = torch.from_numpy(c.seq_lens).cuda()
    out = pad_b200.paged_attention_decode_cuda_v4(torch.from_numpy(c.q).half().cuda(), kc, vc,
                                                  torch.from_numpy(c.block_table).cuda(), sl)
    ref = oracle.decode_c(c.q, k_ref, v_ref, c.block_table, c.seq_lens)
    assert_parity(out.float().cpu().numpy(), ref)
