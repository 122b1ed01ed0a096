"""Parity of the decode's shortcuts for uniform batches with the oracle.

The decode kernel starts fast when every seq_len is equal: with full block-
table rows (seq_len == max_pages * page_size) the page ids guessed from the
parameters are used as loaded; with equal but shorter lengths the cursor has a
closed form; anything else (ragged lengths, an empty sequence, more than 256
sequences, a CSR index) takes the scan hand-off. The merge kernel guesses its
split descriptors for full rows and folds again when the descriptor differs.
Each case here lands on one of those paths, with the heuristic split count and
an explicit one, and is checked against the C oracle.
"""

import numpy as np
import pytest
import torch

import oracle
from gpu_utils import assert_parity, run, to_gpu
from pad_b200 import paged_attention_decode_cuda_v4
from pad_b200.cases import explicit_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


UNIFORM = [
    # batch, seq_len, page_size, spare block-table columns, KV heads, head_dim
    (1, 4096, 16, 0, 2, 128),    # full rows, one long sequence: deep merge, guessed descriptors
    (5, 2048, 32, 0, 2, 128),    # full rows, a few pairs
    (64, 512, 16, 0, 2, 128),    # full rows, batch 64: narrow merge
    (3, 4001, 16, 0, 2, 128),    # equal lengths, last page partly used: closed-form cursor, guess misses
    (4, 1000, 16, 7, 2, 128),    # equal lengths, block table wider than needed
    (2, 960, 24, 0, 2, 128),     # full rows, page size not a power of two
    (2, 950, 24, 3, 2, 128),     # page size not a power of two, wider table
    (6, 768, 16, 0, 8, 128),     # full rows, 8 KV heads in one head group
    (3, 640, 32, 0, 1, 64),      # full rows, one KV head, D = 64
    (257, 128, 16, 0, 2, 128),   # more sequences than the fast start checks
    (300, 64, 8, 2, 2, 64),
]


@pytest.mark.parametrize("batch,seq,page_size,spare,hkv,head_dim", UNIFORM,
                         ids=[f"B{b}-s{s}-ps{p}-x{x}-h{h}-d{d}" for b, s, p, x, h, d in UNIFORM])
def test_uniform_batches(batch, seq, page_size, spare, hkv, head_dim):
    need = -(-seq // page_size)
    c = explicit_case([seq] * batch, num_kv_heads=hkv, gqa_ratio=6 if hkv < 8 else 4, head_dim=head_dim,
                      page_size=page_size, seed=batch * 7919 + seq, max_pages=need + spare)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    what = f"B={batch} seq={seq} ps={page_size} spare={spare} Hkv={hkv} D={head_dim}"
    assert_parity(run(c), ref, what)
    assert_parity(run(c, num_splits=3), ref, what + " S=3")


def test_uniform_but_one_empty_sequence():
    c = explicit_case([512, 512, 0, 512], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=31)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    out = run(c)
    assert_parity(out, ref, "one empty sequence")
    assert np.all(out[2] == 0.0)


def test_guess_miss_after_guess_hit_on_one_workspace():
    """A full-row call, then a same-shaped call whose rows are not full: the
    merge's guessed slots are stale for the second call and must be refolded
    from the descriptors (both calls share the cached workspace)."""
    full = explicit_case([1024] * 2, num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=41)
    short = explicit_case([1000, 1000], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=42,
                          max_pages=64)
    assert full.block_table.shape == short.block_table.shape
    for c in (full, short, full, short):
        ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
        out = paged_attention_decode_cuda_v4(*to_gpu(c)).float().cpu().numpy()
        assert_parity(out, ref, f"seq={int(c.seq_lens[0])}")
