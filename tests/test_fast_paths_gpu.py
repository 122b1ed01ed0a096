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


def _abi_decode(c, ws, num_splits=0):
    """One decode through the C ABI with a caller-owned workspace."""
    from pad_b200 import _lib

    q, k, v, bt, sl = to_gpu(c)
    out = torch.empty_like(q)
    _lib.check(_lib.load().pad_paged_attention_decode(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), bt.data_ptr(), sl.data_ptr(), out.data_ptr(), q.shape[0],
        q.shape[1], k.shape[2], q.shape[2], k.shape[0], k.shape[1], bt.shape[1], _lib.i64_array(q.stride()),
        _lib.i64_array(k.stride()), _lib.i64_array(v.stride()), bt.stride(0), _lib.i64_array(out.stride()),
        1.0 / q.shape[2] ** 0.5, num_splits, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream,
        0))
    return out


def test_one_workspace_shared_by_calls_of_different_shapes():
    """One caller-owned workspace (never initialised) reused by calls of
    different shapes through the C ABI: long context, oversplit with empty
    partitions, ragged with an empty sequence, many pairs, 8 KV heads with an
    explicit split count. Every result matches the oracle, whatever the
    previous call left in the workspace."""
    cases = [
        (explicit_case([20000], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=32, seed=51), 0),
        (explicit_case([5], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=52), 64),
        (explicit_case([3000, 17, 0, 9000], num_kv_heads=4, gqa_ratio=4, head_dim=64, page_size=16, seed=53), 0),
        (explicit_case([300] * 40, num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=54), 0),
        (explicit_case([2500, 7000], num_kv_heads=8, gqa_ratio=8, head_dim=128, page_size=16, seed=55), 5),
        (explicit_case([20000], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=32, seed=51), 0),
    ]
    ws = torch.full((64 << 20,), 0xA5, dtype=torch.uint8, device="cuda")
    for i, (c, s) in enumerate(cases):
        ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
        out = _abi_decode(c, ws, s)
        torch.cuda.synchronize()
        assert_parity(out.float().cpu().numpy(), ref, f"case {i} S={s}")


def test_block_table_rewritten_in_place_between_calls():
    """The kernel warms L2 from page ids it reads before its dependency wait
    (they may be stale); only prefetches follow from them. Rewriting the block
    table and the KV pages in place between consecutive calls on the same
    buffers must still give each call's own exact result."""
    a = explicit_case([2048] * 8, num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=61)
    b = explicit_case([2048] * 8, num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=62)
    assert a.k_cache.shape == b.k_cache.shape and a.block_table.shape == b.block_table.shape
    ga, gb = to_gpu(a), to_gpu(b)
    q, k, v, bt, sl = (t.clone() for t in ga)
    out = torch.empty_like(q)
    for c, g in ((a, ga), (b, gb), (a, ga), (b, gb)):
        for dst, src in zip((q, k, v, bt, sl), g):
            dst.copy_(src)
        paged_attention_decode_cuda_v4(q, k, v, bt, sl, out=out)
        ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
        assert_parity(out.float().cpu().numpy(), ref, "rewritten in place")
