"""Oracle edge cases and input validation, mirroring the reference's
tests/test_reference_validation.py:29-134 and
tests/test_reference_edge_cases.py:99-160."""

import numpy as np
import pytest

import oracle
from pad_b200.cases import explicit_case


def _valid():
    rng = np.random.default_rng(0)
    return dict(
        q=rng.standard_normal((2, 8, 32), dtype=np.float32),
        k_cache=rng.standard_normal((4, 16, 2, 32), dtype=np.float32),
        v_cache=rng.standard_normal((4, 16, 2, 32), dtype=np.float32),
        block_table=np.array([[0, 1], [2, 3]], dtype=np.int32),
        seq_lens=np.array([20, 20], dtype=np.int32),
    )


def _call(**over):
    kw = _valid()
    kw.update(over)
    return oracle.paged_attention_decode_reference(**kw)


def test_valid_inputs_do_not_raise():
    _call()


F32, F16, I32 = np.float32, np.float16, np.int32
INVALID = [
    ("q_wrong_ndim", dict(q=np.zeros((2, 8, 32, 1), F32)), ValueError),
    ("k_cache_wrong_ndim", dict(k_cache=np.zeros((4, 16, 2), F32)), ValueError),
    ("v_cache_shape_mismatch", dict(v_cache=np.zeros((4, 16, 2, 16), F32)), ValueError),
    ("block_table_wrong_ndim", dict(block_table=np.zeros((2, 2, 1), I32)), ValueError),
    ("seq_lens_wrong_ndim", dict(seq_lens=np.zeros((2, 1), I32)), ValueError),
    ("q_wrong_dtype", dict(q=np.zeros((2, 8, 32), F16)), TypeError),
    ("k_cache_wrong_dtype", dict(k_cache=np.zeros((4, 16, 2, 32), F16)), TypeError),
    ("v_cache_wrong_dtype", dict(v_cache=np.zeros((4, 16, 2, 32), F16)), TypeError),
    ("block_table_wrong_dtype", dict(block_table=np.zeros((2, 2), F32)), TypeError),
    ("seq_lens_wrong_dtype", dict(seq_lens=np.zeros(2, F32)), TypeError),
    ("block_table_batch_mismatch", dict(block_table=np.zeros((3, 2), I32)), ValueError),
    ("seq_lens_batch_mismatch", dict(seq_lens=np.zeros(3, I32)), ValueError),
    ("head_dim_mismatch", dict(q=np.zeros((2, 8, 16), F32)), ValueError),
    ("page_size_zero", dict(k_cache=np.zeros((4, 0, 2, 32), F32), v_cache=np.zeros((4, 0, 2, 32), F32)), ValueError),
    ("num_kv_heads_zero", dict(k_cache=np.zeros((4, 16, 0, 32), F32), v_cache=np.zeros((4, 16, 0, 32), F32)),
     ValueError),
    ("gqa_not_divisible", dict(q=np.zeros((2, 5, 32), F32)), ValueError),
    ("negative_seq_len", dict(seq_lens=np.array([-1, 20], I32)), ValueError),
    ("seq_len_exceeds_capacity", dict(seq_lens=np.array([999, 20], I32)), ValueError),
    ("negative_page_id", dict(block_table=np.array([[-1, 1], [2, 3]], I32)), ValueError),
    ("page_id_out_of_range", dict(block_table=np.array([[99, 1], [2, 3]], I32)), ValueError),
]


@pytest.mark.parametrize("name,over,exc", INVALID, ids=[x[0] for x in INVALID])
def test_invalid_inputs_raise(name, over, exc):
    with pytest.raises(exc):
        _call(**over)


def test_c_oracle_rejects_bad_page_and_capacity():
    kw = _valid()
    with pytest.raises(ValueError):
        oracle.decode_c(kw["q"], kw["k_cache"], kw["v_cache"], np.array([[99, 1], [2, 3]], I32), kw["seq_lens"])
    with pytest.raises(ValueError):
        oracle.decode_c(kw["q"], kw["k_cache"], kw["v_cache"], kw["block_table"], np.array([999, 20], I32))


def test_ragged_rows_are_independent():
    c = explicit_case([3, 8, 17, 64], num_kv_heads=2, gqa_ratio=6, head_dim=32, page_size=8, seed=42)
    batched = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    for b in range(4):
        solo = oracle.decode_c(c.q[b:b + 1], c.k_cache, c.v_cache, c.block_table[b:b + 1], c.seq_lens[b:b + 1])
        np.testing.assert_array_equal(batched[b:b + 1], solo)


def test_zero_length_sequence_gives_zeros():
    c = explicit_case([0, 20], num_kv_heads=2, gqa_ratio=4, head_dim=32, page_size=16, seed=7)
    for fn in (oracle.paged_attention_decode_reference, oracle.decode_c):
        out = fn(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
        assert np.all(out[0] == 0.0)


def test_long_sequence_32768():
    c = explicit_case([32768], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=9, identity=True)
    a = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    b = oracle.paged_attention_decode_reference(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-5)
