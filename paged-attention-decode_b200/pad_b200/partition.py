"""Host mirror of the decode kernel's stream-K work partition.

The kernel flattens the batch into one list of tiles ordered (sequence, KV
head group, tile) -- a tile is ``128 / HG`` tokens of ``HG`` KV heads, HG the
largest of 8, 4, 2, 1 dividing the KV head count (at most 4 when a head has
more than 8 query rows) -- and gives partition ``w`` of ``W`` the tiles
``[floor(w*T/W), floor((w+1)*T/W))``. A (sequence, head group) pair whose tiles
fall in one partition is finished there; a pair spread over several
partitions gets one fp32 partial per partition, in slots
``pair + w`` for ``w`` in ``[owner(first tile), owner(last tile)]``, which the
merge kernel combines. This module computes the same plan on the host (for
tests, diagnostics and workspace sizing); it never runs on the decode path.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

TILE_ROWS = 128


def head_group(num_kv_heads: int, gqa_ratio: int) -> int:
    cap = 8 if gqa_ratio <= 8 else 4
    hg = cap
    while hg > 1 and num_kv_heads % hg:
        hg //= 2
    return hg


def tiles_of(seq: int, tt: int = 64) -> int:
    return (max(int(seq), 0) + tt - 1) // tt


def part_begin(w: int, total: int, parts: int) -> int:
    return (w * total) // parts


def part_owner(t: int, total: int, parts: int) -> int:
    return ((t + 1) * parts - 1) // total


@dataclass
class PairPlan:
    pair: int
    first_tile: int
    n_tiles: int
    first_part: int
    last_part: int

    @property
    def split(self) -> bool:
        return self.last_part > self.first_part

    @property
    def slots(self) -> range:
        return range(self.pair + self.first_part, self.pair + self.last_part + 1)


def plan(seq_lens, num_groups: int, parts: int, cap: int | None = None, tt: int = 64
         ) -> tuple[int, list[PairPlan]]:
    """Return (total tiles, per-pair plan) for ``parts`` partitions over
    ``num_groups`` head groups per sequence and ``tt``-token tiles."""
    seq = np.asarray(seq_lens, dtype=np.int64)
    if cap is not None:
        seq = np.clip(seq, 0, cap)
    total = int(sum(tiles_of(s, tt) for s in seq) * num_groups)
    pairs: list[PairPlan] = []
    start = 0
    for b, s in enumerate(seq):
        n = tiles_of(s, tt)
        for h in range(num_groups):
            if n > 0:
                pairs.append(PairPlan(b * num_groups + h, start, n, part_owner(start, total, parts),
                                      part_owner(start + n - 1, total, parts)))
            start += n
    return total, pairs


FEW_PAIRS = 16


def heuristic_partitions(num_sms: int, ctas_per_sm: int, batch: int, num_kv_heads: int, gqa_ratio: int,
                         max_pages: int, page_size: int) -> int:
    """The num_splits=None choice: one partition per resident CTA slot --
    rounded down to a power of two when there are at most FEW_PAIRS
    (sequence, head group) pairs -- capped by the number of tiles the batch
    can hold."""
    hg = head_group(num_kv_heads, gqa_ratio)
    groups = num_kv_heads // hg
    cap_tiles = batch * groups * tiles_of(max_pages * page_size, TILE_ROWS // hg)
    parts = num_sms * ctas_per_sm
    if batch * groups <= FEW_PAIRS:
        parts = 1 << (parts.bit_length() - 1)
    return max(1, min(parts, cap_tiles))
