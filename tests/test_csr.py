"""The CSR page-index entry point (the (indptr, indices, last_page_len) layout
of the reference's FlashInfer adapter, src/flashinfer_adapter.py:40-65):
conversion on CPU, and GPU parity with the oracle and the dense path."""

import numpy as np
import pytest
import torch

import oracle
import pad_b200
from pad_b200.cases import config_case, explicit_case, random_case


def test_paged_kv_indices_layout():
    bt = torch.tensor([[7, 2, 9, 5], [1, 0, 0, 0], [3, 4, 6, 8]], dtype=torch.int32)
    sl = torch.tensor([40, 0, 64], dtype=torch.int32)
    indptr, indices, last = pad_b200.paged_kv_indices(bt, sl, 16)
    assert indptr.tolist() == [0, 3, 3, 7]
    assert indices.tolist() == [7, 2, 9, 3, 4, 6, 8]
    assert last.tolist() == [8, 16, 16]


def _gpu(case):
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dt)  # noqa: E731
    return (t(case.q, torch.float16), t(case.k_cache, torch.float16), t(case.v_cache, torch.float16),
            t(case.block_table, torch.int32), t(case.seq_lens, torch.int32))


CASES = [("ragged", lambda: explicit_case([1, 17, 300, 4000, 0, 65], num_kv_heads=2, gqa_ratio=6, head_dim=128,
                                         page_size=16, seed=3)),
         ("small_pages", lambda: explicit_case([5, 70, 333], num_kv_heads=4, gqa_ratio=4, head_dim=64, page_size=4,
                                               seed=4)),
         ("c4_slice", lambda: config_case("c4", batch=32)),
         ("fuzz_1", lambda: random_case(11, min_seq_len=0, max_seq_len=500)),
         ("fuzz_2", lambda: random_case(12, min_seq_len=0, max_seq_len=500))]


@pytest.mark.gpu
@pytest.mark.parametrize("name,make", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("num_splits", [None, 1, 3])
def test_csr_matches_oracle_and_dense(name, make, num_splits):
    from gpu_utils import assert_parity

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    c = make()
    q, k, v, bt, sl = _gpu(c)
    indptr, indices, last = pad_b200.paged_kv_indices(bt, sl, c.page_size)
    got = pad_b200.paged_attention_decode_csr(q, k, v, indptr, indices, last, num_splits=num_splits)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    assert_parity(got.float().cpu().numpy(), ref, f"{name} S={num_splits}")
    dense = pad_b200.paged_attention_decode_cuda_v4(q, k, v, bt, sl, num_splits=num_splits)
    torch.testing.assert_close(got.float(), dense.float(), rtol=1e-2, atol=2e-3)
