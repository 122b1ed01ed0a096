"""Host logic of the batch-sharded multi-GPU launcher, run as world-size-2
(and 3) gloo process groups on CPU: shard ranges, local page pools with a
remapped block table, and the ordered gather of outputs to rank 0. The decode
itself is the CPU oracle here (the CUDA path needs a GPU); the GPU runs of the
same launcher are in test_sharded_gpu.py."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from pad_b200.cases import explicit_case, random_case
from pad_b200.sharded import gather_to_rank0, localize, shard_range


def test_shard_ranges_cover_batch_evenly():
    for batch in (1, 5, 64, 1024, 1023):
        for world in (1, 2, 3, 4, 8):
            rs = [shard_range(batch, world, r) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            sizes = [h - l for l, h in rs]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("world", [1, 2, 3])
def test_local_pool_reproduces_global_rows(seed, world):
    c = random_case(seed, max_batch=7, min_seq_len=0, max_seq_len=300)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    for rank in range(world):
        sh = localize(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens, world, rank, shuffle_seed=rank)
        assert sh.k_cache.shape[0] >= 1
        got = oracle.decode_c(sh.q.numpy(), sh.k_cache.numpy(), sh.v_cache.numpy(), sh.block_table.numpy(),
                              sh.seq_lens.numpy())
        np.testing.assert_array_equal(got, ref[sh.lo:sh.hi])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = explicit_case([40, 0, 333, 17, 128, 600, 5], num_kv_heads=2, gqa_ratio=4, head_dim=32, page_size=8,
                          seed=3)
        sh = localize(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens, world, rank, shuffle_seed=10 + rank)
        out = torch.from_numpy(oracle.decode_c(sh.q.numpy(), sh.k_cache.numpy(), sh.v_cache.numpy(),
                                               sh.block_table.numpy(), sh.seq_lens.numpy()))
        full = gather_to_rank0(out, c.q.shape[0], world)
        if rank == 0:
            ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
            q.put(float(np.abs(full.numpy() - ref).max()))
        else:
            assert full is None
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_gather_to_rank0_in_sequence_order(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_worker, args=(world, _free_port(), q), nprocs=world, join=True, start_method="spawn")
    assert q.get(timeout=60) == 0.0


def test_local_pool_holds_only_the_shards_pages():
    """A rank's pool holds exactly the distinct pages its own sequences use
    (a page shared by two sequences is copied once), and the remapped block
    table addresses the same rows as the global one."""
    c = explicit_case([40, 0, 333, 17, 128, 600, 5], num_kv_heads=2, gqa_ratio=4, head_dim=32, page_size=8, seed=3)
    bt = c.block_table.copy()
    bt[1, 0] = bt[0, 0]  # sequence 1 is empty: its entries are never used
    bt[3, 1] = bt[2, 3]  # sequences 2 and 3 share a page
    for world in (1, 2, 4):
        for rank in range(world):
            sh = localize(c.q, c.k_cache, c.v_cache, bt, c.seq_lens, world, rank, shuffle_seed=rank)
            used = set()
            for b in range(sh.lo, sh.hi):
                used |= set(bt[b, : (int(c.seq_lens[b]) + 7) // 8].tolist())
            assert sh.k_cache.shape[0] == max(len(used), 1)
            assert set(sh.page_map.tolist()) == used
            for i, b in enumerate(range(sh.lo, sh.hi)):
                n = (int(c.seq_lens[b]) + 7) // 8
                glob = bt[b, :n]
                loc = sh.block_table[i, :n].numpy()
                assert np.array_equal(sh.page_map.numpy()[loc], glob)
                np.testing.assert_array_equal(sh.k_cache.numpy()[loc], c.k_cache[glob])


def test_sharded_decoder_rejects_another_ranks_shard():
    from pad_b200.sharded import ShardedDecoder

    c = explicit_case([40, 7, 333], num_kv_heads=2, gqa_ratio=4, head_dim=32, page_size=8, seed=3)
    sh = localize(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens, 2, 1)
    with pytest.raises(ValueError, match="owns sequences"):
        ShardedDecoder(3, 2, 0, "cpu").decode(sh)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_balanced_ranges_cover_contiguously_with_near_equal_tokens(world):
    from pad_b200.cases import config_seq_lens
    from pad_b200.sharded import balanced_ranges

    for sl in (config_seq_lens("c5"), config_seq_lens("c4"), np.array([5, 0, 0, 100, 7, 7000, 3]),
               np.zeros(9, dtype=np.int64), np.array([3, 1])):
        r = balanced_ranges(sl, world)
        assert len(r) == world and r[0][0] == 0 and r[-1][1] == len(sl)
        assert all(a[1] == b[0] and a[0] <= a[1] for a, b in zip(r, r[1:]))
        if len(sl) >= world:
            assert all(h > l for l, h in r)  # every rank gets a sequence when there are enough
        tok = [int(np.asarray(sl)[l:h].sum()) for l, h in r]
        # each rank within one (longest) sequence of the mean
        assert max(tok) - sum(tok) / world <= int(np.max(sl)) + 1 if len(sl) else True


def _worker_ranges(rank, world, port, q):
    from pad_b200.sharded import ShardedDecoder, balanced_ranges

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = explicit_case([40, 0, 333, 17, 128, 600, 5, 2000], num_kv_heads=2, gqa_ratio=4, head_dim=32,
                          page_size=8, seed=4)
        ranges = balanced_ranges(c.seq_lens, world)
        sh = localize(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens, world, rank, ranges=ranges)
        assert (sh.lo, sh.hi) == ranges[rank]
        out = torch.from_numpy(oracle.decode_c(sh.q.numpy(), sh.k_cache.numpy(), sh.v_cache.numpy(),
                                               sh.block_table.numpy(), sh.seq_lens.numpy()))
        full = ShardedDecoder(c.q.shape[0], world, rank, "cpu", ranges=ranges).gather(out)
        if rank == 0:
            ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
            q.put(float(np.abs(full.numpy() - ref).max()))
    finally:
        dist.destroy_process_group()


def test_gloo_gather_with_token_balanced_ranges():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_worker_ranges, args=(3, _free_port(), q), nprocs=3, join=True, start_method="spawn")
    assert q.get(timeout=60) == 0.0
