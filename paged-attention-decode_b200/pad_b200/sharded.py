"""Batch-sharded decode over several GPUs (one process per GPU).

Sequences are independent, so the batch is split into contiguous shards of
sequences, one per rank; each rank owns the KV pages of its own sequences in a
local page pool and runs the single-GPU decode on them. Nothing crosses
NVLink on the hot path; the only collective is an optional gather of the
outputs to rank 0 (for checking), done outside the decode.

The reference has no multi-GPU code; this module adds the launcher the
decode path needs to scale out (batch sharding, local page pools, output
gather), written against ``torch.distributed`` so that the same logic runs on
NCCL over NVLink and, for tests, on gloo over CPU processes.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


def shard_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) sequence range of `rank`; sizes differ by at most one."""
    base, extra = divmod(batch, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


@dataclass
class LocalShard:
    lo: int
    hi: int
    q: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    block_table: torch.Tensor
    seq_lens: torch.Tensor
    page_map: torch.Tensor  # global page id of each local page


def localize(q, k_cache, v_cache, block_table, seq_lens, world: int, rank: int, device=None,
             shuffle_seed: int | None = None) -> LocalShard:
    """Cut rank `rank`'s sequences out of a global problem.

    The pages its sequences reference (block_table[b, :ceil(seq_b / page_size)])
    are copied into a compact local pool -- in a random order when
    ``shuffle_seed`` is given, so the local pool is a permuted layout like the
    global one -- and the block table is rewritten to local page ids. Unused
    trailing block-table entries become 0. Works for numpy or torch inputs.
    """
    t = lambda a: a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    q, k_cache, v_cache, block_table, seq_lens = map(t, (q, k_cache, v_cache, block_table, seq_lens))
    lo, hi = shard_range(q.shape[0], world, rank)
    page_size = k_cache.shape[1]
    sl = seq_lens[lo:hi].to(torch.int64).clamp(min=0)
    bt = block_table[lo:hi].to(torch.int64)
    need = (sl + page_size - 1) // page_size
    width = max(int(need.max().item()) if len(need) else 0, 1)
    used = [bt[i, : int(need[i])] for i in range(hi - lo)]
    glob = torch.cat(used) if used else torch.zeros(0, dtype=torch.int64)
    # distinct pages in first-use order (a page shared by sequences is copied once)
    uniq, first = np.unique(glob.cpu().numpy(), return_index=True)
    order = uniq[np.argsort(first)]
    if shuffle_seed is not None and len(order):
        order = order[np.random.default_rng(shuffle_seed).permutation(len(order))]
    page_map = torch.from_numpy(order.astype(np.int64))
    lookup = {int(g): i for i, g in enumerate(order)}
    local_bt = torch.zeros((hi - lo, width), dtype=torch.int32)
    for i, row in enumerate(used):
        if len(row):
            local_bt[i, : len(row)] = torch.tensor([lookup[int(g)] for g in row], dtype=torch.int32)
    idx = page_map.to(k_cache.device)
    if len(page_map):
        k_loc, v_loc = k_cache.index_select(0, idx), v_cache.index_select(0, idx)
    else:
        k_loc = k_cache[:1].clone()
        v_loc = v_cache[:1].clone()
    dev = device if device is not None else k_cache.device
    return LocalShard(lo, hi, q[lo:hi].to(dev), k_loc.to(dev), v_loc.to(dev), local_bt.to(dev),
                      seq_lens[lo:hi].to(torch.int32).to(dev), page_map)


def gather_to_rank0(out_local: torch.Tensor, batch: int, world: int, group=None):
    """Gather every rank's output rows to rank 0 in sequence order.

    Shards may differ in size by one sequence, so each rank pads to the
    largest shard; rank 0 returns the [batch, Hq, D] tensor, others None."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    sizes = [shard_range(batch, world, r) for r in range(world)]
    rows = max(h - l for l, h in sizes)
    pad = torch.zeros((rows,) + tuple(out_local.shape[1:]), dtype=out_local.dtype, device=out_local.device)
    pad[: out_local.shape[0]] = out_local
    bucket = [torch.empty_like(pad) for _ in range(world)] if rank == 0 else None
    dist.gather(pad, bucket, dst=0, group=group)
    if rank != 0:
        return None
    return torch.cat([bucket[r][: h - l] for r, (l, h) in enumerate(sizes)], dim=0)


def decode_sharded(q, k_cache, v_cache, block_table, seq_lens, *, world: int, rank: int, device,
                   num_splits=None, scale=None, gather: bool = True, shuffle_seed: int | None = None):
    """Localize this rank's shard, decode it on `device` and (optionally)
    gather the outputs to rank 0. Returns (local output, gathered or None)."""
    from .kernel_cuda_v4 import paged_attention_decode_cuda_v4

    shard = localize(q, k_cache, v_cache, block_table, seq_lens, world, rank, device=device,
                     shuffle_seed=shuffle_seed)
    out = paged_attention_decode_cuda_v4(shard.q, shard.k_cache, shard.v_cache, shard.block_table,
                                         shard.seq_lens, num_splits=num_splits, scale=scale)
    full = gather_to_rank0(out, q.shape[0], world) if gather else None
    return out, full
