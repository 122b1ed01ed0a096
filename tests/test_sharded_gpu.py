"""The batch-sharded launcher on real GPUs: every rank decodes its own
sequences from its own local page pool with the CUDA kernel, outputs are
gathered to rank 0 over NCCL and checked against the CPU oracle. Uses as many
GPUs as the box has (up to 4); on a one-GPU box it runs the single-rank path."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from gpu_utils import assert_parity
from pad_b200.cases import explicit_case
from pad_b200.sharded import decode_sharded

pytestmark = pytest.mark.gpu


def _case():
    rng = np.random.default_rng(2)
    seqs = rng.integers(1024, 4097, size=24).tolist()  # C5-like spread at test size
    seqs[3] = 0
    return explicit_case(seqs, num_kv_heads=8, gqa_ratio=8, head_dim=128, page_size=16, seed=21)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        c = _case()
        qh, kh, vh = (torch.from_numpy(a).half() for a in (c.q, c.k_cache, c.v_cache))
        _, full = decode_sharded(qh, kh, vh, torch.from_numpy(c.block_table), torch.from_numpy(c.seq_lens),
                                 world=world, rank=rank, device=torch.device("cuda", rank), shuffle_seed=rank)
        if rank == 0:
            # send back only scalars: a large object in the queue would block
            # this child's exit while the parent waits in join()
            ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
            got = full.float().cpu().numpy()
            err = np.abs(got - ref)
            q.put((bool(np.all(err <= 2e-3 + 1e-2 * np.abs(ref))), float(err.max())))
    finally:
        dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.timeout(240)
def test_sharded_decode_matches_oracle():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    c = _case()
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    world = min(4, torch.cuda.device_count())
    if world == 1:
        from pad_b200.sharded import localize
        import pad_b200

        sh = localize(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens, 1, 0, shuffle_seed=0)
        out = pad_b200.paged_attention_decode_cuda_v4(sh.q.half().cuda(), sh.k_cache.half().cuda(),
                                                      sh.v_cache.half().cuda(), sh.block_table.cuda(),
                                                      sh.seq_lens.cuda())
        assert_parity(out.float().cpu().numpy(), ref)
        return
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    mp.start_processes(_worker, args=(world, _port(), qq), nprocs=world, join=True, start_method="spawn")
    ok, max_err = qq.get(timeout=60)
    assert ok and max_err <= 2e-3, f"world={world}: max abs err {max_err:.3e}"


@pytest.mark.timeout(600)
def test_c5_shape_shard_built_with_localize():
    """BASELINE config 5 at its own shape on one GPU: Llama-3-70B heads
    (64 Q / 8 KV, head_dim 128, page 16), seq_lens U{1024..16384} with seed 2.
    A 256-sequence global problem (its first 256 lengths) lives on the GPU;
    rank 1 of 2 takes its 128 sequences with ``localize`` (only its pages are
    copied, into a permuted local pool) and decodes them through the
    launcher. 32 sampled sequences plus the longest and shortest are checked
    against the CPU oracle."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from pad_b200.cases import config_case, config_seq_lens
    from pad_b200.sharded import ShardedDecoder, localize

    sl = config_seq_lens("c5")[:256]
    g = config_case("c5", seq_lens=sl, device="cuda", seed=5)
    sh = localize(g.q, g.k_cache, g.v_cache, g.block_table, g.seq_lens, 2, 1, shuffle_seed=1)
    assert sh.k_cache.shape[0] == int(((sl[128:] + 15) // 16).sum())
    del g
    torch.cuda.empty_cache()
    dec = ShardedDecoder(256, 2, 1, "cuda")
    out = dec.decode(sh).float().cpu().numpy()
    lens = sh.seq_lens.cpu().numpy()
    idx = np.random.default_rng(0).choice(len(lens), 32, replace=False)
    idx = np.unique(np.concatenate([idx, [int(np.argmax(lens)), int(np.argmin(lens))]]))
    ti = torch.from_numpy(idx).cuda()
    sub = localize(sh.q[ti], sh.k_cache, sh.v_cache, sh.block_table[ti], sh.seq_lens[ti], 1, 0, device="cpu")
    ref = oracle.decode_c(sub.q.numpy(), sub.k_cache.numpy(), sub.v_cache.numpy(), sub.block_table.numpy(),
                          sub.seq_lens.numpy())
    assert_parity(out[idx], ref, "C5 shard (sampled)")
