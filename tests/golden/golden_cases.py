"""The seeded cases whose reference outputs are stored in decode_golden.npz.

Inputs are regenerated from seeds by ``pad_b200.cases`` (numpy PCG64, so the
bytes are identical on every machine); the fixture stores a sha256 of the
input bytes beside each output so a drift in the generator is caught rather
than silently compared against stale outputs.

The list mirrors the reference's own test inventory for this path:
tests/test_reference_edge_cases.py (partial page, seq 1, one full page,
shuffled holes, GQA 1/4/6/8, ragged, zero-length), tests/test_kernel_cuda_v4.py
(primary shape, split-invariance shape, oversplit, ragged), the fuzz matrix of
tests/case_generators.py, and BASELINE config 1.
"""

from __future__ import annotations

import hashlib

import numpy as np

from pad_b200.cases import PagedCase, config_case, explicit_case, random_case


def golden_cases():
    cases: list[tuple[str, PagedCase]] = []
    cases.append(("c1_seed0", config_case("c1")))
    cases.append(("partial_last_page", explicit_case([100], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=1)))
    cases.append(("seq_len_one", explicit_case([1], num_kv_heads=2, gqa_ratio=4, head_dim=32, page_size=16, seed=2)))
    cases.append(("one_full_page", explicit_case([16], num_kv_heads=2, gqa_ratio=6, head_dim=32, page_size=16, seed=3)))
    cases.append(("shuffled_holes", explicit_case([48], num_kv_heads=2, gqa_ratio=6, head_dim=32, page_size=16, seed=4,
                                                  spare_pages=7, max_pages=6, hole_fill="spare")))
    for g in (1, 4, 6, 8):
        cases.append((f"gqa_{g}", explicit_case([200], num_kv_heads=2, gqa_ratio=g, head_dim=128, page_size=16, seed=100 + g)))
    cases.append(("ragged_3_17_100_512", explicit_case([3, 17, 100, 512], num_kv_heads=2, gqa_ratio=6, head_dim=128,
                                                       page_size=16, seed=43)))
    cases.append(("zero_length_row", explicit_case([0, 20], num_kv_heads=2, gqa_ratio=4, head_dim=32, page_size=16, seed=7)))
    cases.append(("primary_1_17_256_4000", explicit_case([1, 17, 256, 4000], num_kv_heads=2, gqa_ratio=6, head_dim=128,
                                                         page_size=16, seed=0)))
    cases.append(("split_shape_2000", explicit_case([2000], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16,
                                                    seed=600, identity=True)))
    cases.append(("oversplit_5", explicit_case([5], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=700)))
    for d in (16, 32, 64):
        cases.append((f"head_dim_{d}", explicit_case([77, 300], num_kv_heads=2, gqa_ratio=4, head_dim=d, page_size=16, seed=800 + d)))
    for ps in (1, 2, 4, 8, 12, 32, 64):
        cases.append((f"page_size_{ps}", explicit_case([1, 70, 333], num_kv_heads=2, gqa_ratio=6, head_dim=128,
                                                       page_size=ps, seed=900 + ps)))
    cases.append(("gqa_16", explicit_case([150], num_kv_heads=1, gqa_ratio=16, head_dim=128, page_size=16, seed=950)))
    cases.append(("std_half_long", explicit_case([3000], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=32,
                                                 seed=960, std=0.5)))
    for seed in range(24):
        cases.append((f"fuzz_{seed}", random_case(seed, min_seq_len=1)))
    for seed in range(100, 108):
        cases.append((f"fuzz_kernel_{seed}", random_case(seed, gqa_ratio_choices=(1, 4, 6, 8), head_dim_choices=(32, 128),
                                                         page_size_choices=(16, 32), min_seq_len=1)))
    return cases


def input_digest(case: PagedCase) -> str:
    h = hashlib.sha256()
    for a in (case.q, case.k_cache, case.v_cache, case.block_table, case.seq_lens):
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()
