"""Shared helpers of the GPU parity tests.

Tolerance (on fp16 outputs vs the fp32 reference oracle
run on the same fp16-rounded inputs): elementwise
    |out - ref| <= ATOL + RTOL * |ref|,  ATOL = 2e-3, RTOL = 1e-2,
plus max |out - ref| <= ATOL over all elements, plus max-rel
max(|out - ref| / |ref|) <= RTOL over the elements with |ref| >= REL_FLOOR
(1e-2; relative error is meaningless near zero, where the absolute bound
governs). All three are asserted.
"""

from __future__ import annotations

import numpy as np
import torch

import pad_b200

ATOL, RTOL = 2e-3, 1e-2
REL_FLOOR = 1e-2


def to_gpu(case, device="cuda"):
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dt)  # noqa: E731
    return (t(case.q, torch.float16), t(case.k_cache, torch.float16), t(case.v_cache, torch.float16),
            t(case.block_table, torch.int32), t(case.seq_lens, torch.int32))


def run(case, num_splits=None, scale=None, device="cuda"):
    out = pad_b200.paged_attention_decode_cuda_v4(*to_gpu(case, device), num_splits=num_splits, scale=scale)
    return out.float().cpu().numpy()


def assert_parity(actual, expected, what=""):
    actual = np.asarray(actual, dtype=np.float32)
    expected = np.asarray(expected, dtype=np.float32)
    assert actual.shape == expected.shape
    assert np.all(np.isfinite(actual)), f"{what}: non-finite output"
    err = np.abs(actual - expected)
    bound = ATOL + RTOL * np.abs(expected)
    bad = err > bound
    big = np.abs(expected) >= REL_FLOOR
    rel = float((err[big] / np.abs(expected[big])).max()) if big.any() else 0.0
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements out of tolerance; max abs {err.max():.3e}, "
                           f"max rel {rel:.3e}")
    assert err.max() <= ATOL, f"{what}: max abs error {err.max():.3e} > {ATOL}"
    assert rel <= RTOL, f"{what}: max rel error {rel:.3e} > {RTOL} (over |ref| >= {REL_FLOOR})"
    return float(err.max()), rel
