"""Batch-sharded decode over several GPUs (one process per GPU).

Sequences are independent, so the batch is split into contiguous shards of
sequences, one per rank; each rank owns the KV pages of its own sequences in a
local page pool and runs the single-GPU decode on them. Nothing crosses
NVLink on the hot path; the only collective is an optional gather of the
outputs to rank 0 (for checking), done after the decode.

The reference has no multi-GPU code; this module adds the launcher the
decode path needs to scale out, written against ``torch.distributed`` so that
the same logic runs on NCCL over NVLink and, for tests, on gloo over CPU
processes:

* ``shard_range``     -- which sequences a rank owns (equal counts);
* ``balanced_ranges`` -- contiguous ranges with near-equal KV tokens instead
                         (ragged batches: the slowest rank sets the step time);
* ``LocalShard``      -- a rank's own problem: its q rows, its local page pool
                         and its block table in local page ids;
* ``localize``        -- cut a rank's shard out of a global problem (only that
                         rank's pages are copied to its device);
* ``ShardedDecoder``  -- the launcher: decode a rank's local shard on its GPU
                         (the same call on every rank, no collective) and,
                         optionally, gather the outputs to rank 0;
* ``decode_sharded``  -- ``localize`` + ``ShardedDecoder`` for a global problem.

A serving engine already holds each rank's pool on that rank; it builds a
``LocalShard`` from its own tensors and calls ``ShardedDecoder.decode``.
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


def balanced_ranges(seq_lens, world: int) -> list[tuple[int, int]]:
    """Contiguous [lo, hi) sequence ranges, one per rank, cut where the running
    token count crosses k * total / world: each rank's KV bytes are within
    one sequence of the mean (equal-count ranges can differ by the spread of
    the lengths). Every rank gets at least one sequence while there are
    enough; empty ranges only when batch < world."""
    sl = np.clip(np.asarray(seq_lens, dtype=np.int64), 0, None)
    batch = len(sl)
    cum = np.concatenate([[0], np.cumsum(sl)])
    total = int(cum[-1])
    cuts = [0]
    for k in range(1, world):
        target = total * k / world
        c = int(np.searchsorted(cum, target, side="left"))
        # the closer of the two boundaries around the target, kept monotone
        if c > 0 and abs(cum[c - 1] - target) <= abs(cum[min(c, batch)] - target):
            c -= 1
        lo_bound = cuts[-1] + (1 if batch - cuts[-1] >= world - k + 1 else 0)
        hi_bound = batch - (world - k) if batch >= world else batch
        cuts.append(int(min(max(c, lo_bound), max(hi_bound, lo_bound))))
    cuts.append(batch)
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


@dataclass
class LocalShard:
    """One rank's decode problem: sequences [lo, hi) of the global batch,
    their KV pages in a local pool, block_table in local page ids."""

    lo: int
    hi: int
    q: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    block_table: torch.Tensor
    seq_lens: torch.Tensor
    page_map: torch.Tensor | None = None  # global page id of each local page (None: built locally)


def _as_tensor(a):
    return a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a))


def localize(q, k_cache, v_cache, block_table, seq_lens, world: int, rank: int, device=None,
             shuffle_seed: int | None = None, ranges: list[tuple[int, int]] | None = None) -> LocalShard:
    """Cut rank `rank`'s sequences out of a global problem.

    The distinct pages its sequences reference (block_table[b, :ceil(seq_b /
    page_size)]) are gathered, on the device the global caches live on, into
    a compact local pool -- in ascending global page order, or in a random
    order when ``shuffle_seed`` is given so that the local pool is a permuted
    layout like the global one -- and the block table is rewritten to local
    page ids by one ``torch.unique(..., return_inverse=True)``. Unused
    trailing block-table entries become 0. Only the shard moves to ``device``.
    ``ranges`` (one [lo, hi) per rank, e.g. from ``balanced_ranges``) replaces
    the equal-count split. Works for numpy or torch inputs.
    """
    q, k_cache, v_cache, block_table, seq_lens = map(_as_tensor, (q, k_cache, v_cache, block_table, seq_lens))
    lo, hi = ranges[rank] if ranges is not None else shard_range(q.shape[0], world, rank)
    page_size = k_cache.shape[1]
    src = k_cache.device
    sl = seq_lens[lo:hi].to(device=src, dtype=torch.int64).clamp(min=0)
    need = (sl + page_size - 1) // page_size
    width = max(int(need.max().item()) if need.numel() else 0, 1)
    bt = block_table[lo:hi, :width].to(device=src, dtype=torch.int64)
    if bt.shape[1] < width:
        raise ValueError("seq_lens address more pages than block_table holds")
    mask = torch.arange(width, device=src)[None, :] < need[:, None]
    glob = bt[mask]
    uniq, inv = torch.unique(glob, return_inverse=True)
    if shuffle_seed is not None and uniq.numel():
        gen = torch.Generator().manual_seed(shuffle_seed)
        perm = torch.randperm(uniq.numel(), generator=gen).to(src)  # local page i holds uniq[perm[i]]
        where = torch.empty_like(perm)
        where[perm] = torch.arange(perm.numel(), device=src)
        page_map, local_ids = uniq[perm], where[inv]
    else:
        page_map, local_ids = uniq, inv
    local_bt = torch.zeros((hi - lo, width), dtype=torch.int32, device=src)
    local_bt[mask] = local_ids.to(torch.int32)
    if page_map.numel():
        k_loc, v_loc = k_cache.index_select(0, page_map), v_cache.index_select(0, page_map)
    else:  # an all-empty shard still gets a one-page pool (never read)
        k_loc, v_loc = k_cache[:1].clone(), v_cache[:1].clone()
    dev = device if device is not None else src
    return LocalShard(lo, hi, q[lo:hi].to(dev), k_loc.to(dev), v_loc.to(dev), local_bt.to(dev),
                      seq_lens[lo:hi].to(torch.int32).to(dev), page_map.cpu())


def gather_to_rank0(out_local: torch.Tensor, batch: int, world: int, group=None,
                    ranges: list[tuple[int, int]] | None = None):
    """Gather every rank's output rows to rank 0 in sequence order.

    Shards may differ in size, so each rank pads to the largest shard; rank 0
    returns the [batch, Hq, D] tensor, others None. ``ranges`` as for
    ``localize`` (default: the equal-count split)."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    sizes = ranges if ranges is not None else [shard_range(batch, world, r) for r in range(world)]
    rows = max(h - l for l, h in sizes)
    if out_local.shape[0] == rows:
        pad = out_local.contiguous()
    else:
        pad = torch.zeros((rows,) + tuple(out_local.shape[1:]), dtype=out_local.dtype, device=out_local.device)
        pad[: out_local.shape[0]] = out_local
    bucket = [torch.empty_like(pad) for _ in range(world)] if rank == 0 else None
    dist.gather(pad, bucket, dst=0, group=group)
    if rank != 0:
        return None
    return torch.cat([bucket[r][: h - l] for r, (l, h) in enumerate(sizes)], dim=0)


class ShardedDecoder:
    """The batch-sharded launcher of one rank.

    ``decode(shard)`` runs the single-GPU B200 decode on this rank's local
    shard, on the current stream of ``device`` -- the same call on every rank,
    with no collective and no host synchronisation -- into a reused output
    buffer. ``gather()`` collects the last outputs on rank 0 in global
    sequence order (one NCCL gather; call it only when rank 0 needs them)."""

    def __init__(self, batch_total: int, world: int, rank: int, device, group=None,
                 ranges: list[tuple[int, int]] | None = None):
        self.batch_total, self.world, self.rank = batch_total, world, rank
        self.device = torch.device(device)
        self.group = group
        self.ranges = ranges
        self.lo, self.hi = ranges[rank] if ranges is not None else shard_range(batch_total, world, rank)
        self._out: torch.Tensor | None = None

    def decode(self, shard: LocalShard, num_splits=None, scale=None) -> torch.Tensor:
        from .kernel_cuda_v4 import paged_attention_decode_cuda_v4

        if (shard.lo, shard.hi) != (self.lo, self.hi):
            raise ValueError(f"rank {self.rank} owns sequences [{self.lo}, {self.hi}), "
                             f"the shard holds [{shard.lo}, {shard.hi})")
        if self._out is None or self._out.shape != shard.q.shape:
            self._out = torch.empty(shard.q.shape, dtype=torch.float16, device=self.device)
        return paged_attention_decode_cuda_v4(shard.q, shard.k_cache, shard.v_cache, shard.block_table,
                                              shard.seq_lens, num_splits=num_splits, scale=scale, out=self._out)

    def gather(self, out_local: torch.Tensor | None = None):
        out = self._out if out_local is None else out_local
        return gather_to_rank0(out, self.batch_total, self.world, self.group, self.ranges)


def decode_sharded(q, k_cache, v_cache, block_table, seq_lens, *, world: int, rank: int, device,
                   num_splits=None, scale=None, gather: bool = True, shuffle_seed: int | None = None,
                   balance_tokens: bool = False):
    """Localize this rank's shard of a global problem (only its pages go to
    `device`), decode it and (optionally) gather the outputs to rank 0.
    ``balance_tokens`` splits by KV tokens instead of sequence counts.
    Returns (local output, gathered or None)."""
    ranges = balanced_ranges(_as_tensor(seq_lens).cpu().numpy(), world) if balance_tokens else None
    shard = localize(q, k_cache, v_cache, block_table, seq_lens, world, rank, device=device,
                     shuffle_seed=shuffle_seed, ranges=ranges)
    dec = ShardedDecoder(q.shape[0], world, rank, device, ranges=ranges)
    out = dec.decode(shard, num_splits=num_splits, scale=scale)
    full = dec.gather(out) if gather else None
    return out, full
