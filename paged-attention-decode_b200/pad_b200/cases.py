"""Seeded synthetic decode workloads: paged KV caches, block tables and seq_lens.

The reference project has no datasets; its tests and benches build random
paged caches (tests/case_generators.py:19-70, bench/bench_decode.py:71-83).
This module builds the same kinds of cases with its own generators:

* ``random_case`` -- a ragged batch over a shuffled physical page pool with
  spare pages and unused "hole" columns in the block table (the semantics of
  tests/case_generators.py:19-70), drawn from numpy's PCG64 so the bytes are
  identical on every machine (the golden fixtures depend on that).
* ``config_case`` -- the five BASELINE configurations (C1..C5), generated
  either with numpy (small, host) or with torch directly on a CUDA device
  (large; C5 is tens of GB).

Layout everywhere (README.md:38-44 of the reference):
``q [B, Hq, D]``, ``k_cache/v_cache [num_pages, page_size, Hkv, D]``,
``block_table [B, max_pages] int32``, ``seq_lens [B] int32``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np


@dataclass
class PagedCase:
    """One decode problem. Arrays are numpy (host) or torch tensors."""

    q: object
    k_cache: object
    v_cache: object
    block_table: object
    seq_lens: object
    page_size: int
    scale: float | None = None
    meta: dict = field(default_factory=dict)

    @property
    def shape_tuple(self):
        b, hq, d = self.q.shape
        p, ps, hkv, _ = self.k_cache.shape
        return b, hq, hkv, d, p, ps, self.block_table.shape[1]


def pages_for(seq_lens: Sequence[int], page_size: int) -> list[int]:
    return [(int(s) + page_size - 1) // page_size if s > 0 else 0 for s in seq_lens]


def permuted_block_table(seq_lens: Sequence[int], page_size: int, num_pages: int,
                         rng: np.random.Generator, max_pages: int | None = None,
                         hole_fill: str = "zero") -> np.ndarray:
    """Assign every logical page a distinct physical page from a random
    permutation of ``range(num_pages)``.

    ``hole_fill`` decides what the unused trailing columns hold: ``"zero"``
    (page 0, as BASELINE config 1 specifies) or ``"spare"`` (a page holding
    other data, so reading past the sequence would change the answer, as in
    tests/case_generators.py:62-63).
    """
    need = pages_for(seq_lens, page_size)
    width = max(max(need) if need else 0, 1) if max_pages is None else max_pages
    total = sum(need)
    if total > num_pages:
        raise ValueError(f"pool of {num_pages} pages cannot hold {total} pages")
    perm = rng.permutation(num_pages).astype(np.int32)
    bt = np.zeros((len(need), width), dtype=np.int32)
    cur = 0
    for b, n in enumerate(need):
        bt[b, :n] = perm[cur:cur + n]
        cur += n
        if hole_fill == "spare" and width > n:
            bt[b, n:] = perm[(cur + np.arange(width - n)) % num_pages]
    return bt


def _normal_fp16_as_fp32(rng: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    """N(0, std) values rounded through fp16 and returned as fp32, so that the
    fp32 oracle and the fp16 kernel see exactly the same numbers
    (tests/kernel_test_utils.py:47-51 of the reference rounds the same way)."""
    x = rng.standard_normal(size=shape, dtype=np.float32) * np.float32(std)
    return x.astype(np.float16).astype(np.float32)


def random_case(seed: int, *, kv_heads_choices=(1, 2, 4), gqa_ratio_choices=(1, 2, 4, 6, 8),
                head_dim_choices=(16, 32, 64, 128), page_size_choices=(1, 4, 8, 16, 32),
                max_batch: int = 4, min_seq_len: int = 0, max_seq_len: int = 200) -> PagedCase:
    """Ragged batch, shuffled physical layout, spare pages and hole columns
    (the case family of tests/case_generators.py:19-70), numpy-seeded."""
    rng = np.random.default_rng(seed)
    hkv = int(rng.choice(kv_heads_choices))
    g = int(rng.choice(gqa_ratio_choices))
    d = int(rng.choice(head_dim_choices))
    ps = int(rng.choice(page_size_choices))
    batch = int(rng.integers(1, max_batch + 1))
    seq = [int(rng.integers(min_seq_len, max_seq_len + 1)) for _ in range(batch)]
    need = pages_for(seq, ps)
    width = max(max(need), 1) + int(rng.integers(0, 3))
    num_pages = sum(need) + int(rng.integers(2, 6))
    bt = permuted_block_table(seq, ps, num_pages, rng, max_pages=width, hole_fill="spare")
    k = _normal_fp16_as_fp32(rng, (num_pages, ps, hkv, d))
    v = _normal_fp16_as_fp32(rng, (num_pages, ps, hkv, d))
    q = _normal_fp16_as_fp32(rng, (batch, hkv * g, d))
    return PagedCase(q, k, v, bt, np.asarray(seq, dtype=np.int32), ps,
                     meta={"seed": seed, "gqa": g, "hkv": hkv, "d": d})


def explicit_case(seq_lens: Sequence[int], *, num_kv_heads: int, gqa_ratio: int, head_dim: int,
                  page_size: int, seed: int, spare_pages: int = 3, std: float = 1.0,
                  identity: bool = False, hole_fill: str = "spare",
                  max_pages: int | None = None) -> PagedCase:
    """A hand-specified case (the named edge cases of the reference tests)."""
    rng = np.random.default_rng(seed)
    need = pages_for(seq_lens, page_size)
    num_pages = max(sum(need) + spare_pages, 1)
    if identity:
        width = max(max(need), 1) if max_pages is None else max_pages
        bt = np.zeros((len(seq_lens), width), dtype=np.int32)
        cur = 0
        for b, n in enumerate(need):
            bt[b, :n] = np.arange(cur, cur + n, dtype=np.int32)
            cur += n
            if hole_fill == "spare" and width > n:
                bt[b, n:] = (cur + np.arange(width - n)) % num_pages
    else:
        bt = permuted_block_table(seq_lens, page_size, num_pages, rng, max_pages=max_pages,
                                  hole_fill=hole_fill)
    hq = num_kv_heads * gqa_ratio
    k = _normal_fp16_as_fp32(rng, (num_pages, page_size, num_kv_heads, head_dim), std)
    v = _normal_fp16_as_fp32(rng, (num_pages, page_size, num_kv_heads, head_dim), std)
    q = _normal_fp16_as_fp32(rng, (len(seq_lens), hq, head_dim), std)
    return PagedCase(q, k, v, bt, np.asarray(seq_lens, dtype=np.int32), page_size)


# --------------------------------------------------------------------------------------
# BASELINE configurations
# --------------------------------------------------------------------------------------

CONFIGS = {
    # name: (Hq, Hkv, D, page_size, std)
    "c1": (12, 2, 128, 16, 1.0),   # Qwen2.5-1.5B shape, CPU oracle case
    "c2": (12, 2, 128, 16, 1.0),   # Qwen2.5-1.5B batch sweep, seq 4096
    "c3": (12, 2, 128, 32, 0.5),   # long-context split-K stress
    "c4": (32, 8, 128, 16, 1.0),   # Llama-3-8B ragged B=256
    "c5": (64, 8, 128, 16, 1.0),   # Llama-3-70B batch-sharded B=1024
}


def config_seq_lens(name: str, batch: int | None = None, seq_len: int | None = None) -> np.ndarray:
    """The seq_lens each BASELINE config prescribes (seeded where random)."""
    if name == "c1":
        rng = np.random.default_rng(0)
        return rng.integers(1, 513, size=batch or 4).astype(np.int32)
    if name == "c2":
        return np.full(batch or 64, seq_len or 4096, dtype=np.int32)
    if name == "c3":
        return np.full(batch or 1, seq_len or 32768, dtype=np.int32)
    if name == "c4":
        rng = np.random.default_rng(1)
        u = rng.uniform(math.log(128), math.log(8192), size=batch or 256)
        return np.clip(np.exp(u).round(), 128, 8192).astype(np.int32)
    if name == "c5":
        rng = np.random.default_rng(2)
        return rng.integers(1024, 16385, size=batch or 1024).astype(np.int32)
    raise KeyError(name)


def config_pool_pages(name: str, seq_lens: np.ndarray, page_size: int) -> int:
    need = sum(pages_for(seq_lens, page_size))
    if name == "c1":
        return need + 16
    if name == "c4":
        return need + max(1, int(math.ceil(0.05 * need)))
    return need


def config_case(name: str, *, batch: int | None = None, seq_len: int | None = None,
                seq_lens: np.ndarray | None = None, seed: int = 0, device=None,
                dtype: str = "fp16", table_width: int | None = None) -> PagedCase:
    """Build config ``name`` (c1..c5).

    ``device=None`` returns numpy fp32 arrays holding fp16-rounded values;
    a torch device returns torch tensors generated on that device in fp16
    (``dtype="fp16"``) -- this is how the multi-GB configs are made without
    a host copy. ``seq_lens`` overrides the config's own lengths (used by the
    sharded launcher, which hands each rank its slice). ``table_width`` makes
    the block table that many columns wide (a serving engine's table is wider
    than the current lengths); the extra columns hold page 0.
    """
    hq, hkv, d, ps, std = CONFIGS[name]
    if seq_lens is None:
        seq_lens = config_seq_lens(name, batch, seq_len)
    seq_lens = np.asarray(seq_lens, dtype=np.int32)
    num_pages = max(config_pool_pages(name, seq_lens, ps), 1)
    rng = np.random.default_rng(1000 + seed)
    bt = permuted_block_table(seq_lens, ps, num_pages, rng, hole_fill="zero", max_pages=table_width)
    b = len(seq_lens)
    if device is None:
        k = _normal_fp16_as_fp32(rng, (num_pages, ps, hkv, d), std)
        v = _normal_fp16_as_fp32(rng, (num_pages, ps, hkv, d), std)
        q = _normal_fp16_as_fp32(rng, (b, hq, d), std)
        return PagedCase(q, k, v, bt, seq_lens, ps, meta={"config": name})
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(1000 + seed)
    tdt = torch.float16 if dtype == "fp16" else torch.float32
    k = torch.empty((num_pages, ps, hkv, d), dtype=tdt, device=device)
    v = torch.empty_like(k)
    k.normal_(0.0, std, generator=gen)
    v.normal_(0.0, std, generator=gen)
    q = torch.empty((b, hq, d), dtype=tdt, device=device).normal_(0.0, std, generator=gen)
    return PagedCase(q, k, v, torch.from_numpy(bt).to(device), torch.from_numpy(seq_lens).to(device),
                     ps, meta={"config": name})


def kv_bytes(seq_lens, num_kv_heads: int, head_dim: int, elem_bytes: int = 2) -> int:
    """Algorithmic KV bytes one call must read: sum_b seq_b * Hkv * D * 2 (K,V) * 2 B.

    The reference's roofline formula (bench/roofline.py:55-59) generalised to
    ragged batches."""
    total = int(np.asarray(seq_lens, dtype=np.int64).clip(min=0).sum())
    return total * num_kv_heads * head_dim * 2 * elem_bytes
