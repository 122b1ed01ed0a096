"""The oracle against the reference's own outputs (tests/golden/decode_golden.npz,
made by tests/golden/make_golden.py from src/reference.py:8-54 and
tests/oracle_sdpa.py:17-58 of the reference)."""

import os

import numpy as np
import pytest

import oracle
from golden.golden_cases import golden_cases, input_digest

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "decode_golden.npz"))
CASES = golden_cases()


def test_every_case_has_a_fixture():
    names = {k.split("__")[0] for k in GOLDEN.files}
    assert names == {n for n, _ in CASES}


@pytest.mark.parametrize("name,case", CASES, ids=[n for n, _ in CASES])
def test_inputs_regenerate_bit_exactly(name, case):
    assert bytes(GOLDEN[f"{name}__digest"]).hex() == input_digest(case)


@pytest.mark.parametrize("name,case", CASES, ids=[n for n, _ in CASES])
def test_numpy_oracle_matches_reference(name, case):
    out = oracle.paged_attention_decode_reference(case.q, case.k_cache, case.v_cache, case.block_table,
                                                  case.seq_lens)
    np.testing.assert_allclose(out, GOLDEN[f"{name}__out"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name,case", CASES, ids=[n for n, _ in CASES])
def test_c_oracle_matches_reference(name, case):
    out = oracle.decode_c(case.q, case.k_cache, case.v_cache, case.block_table, case.seq_lens)
    np.testing.assert_allclose(out, GOLDEN[f"{name}__out"], rtol=1e-5, atol=1e-5)
    # fp16 inputs carry the same values (they were fp16-rounded at generation)
    out16 = oracle.decode_c(case.q.astype(np.float16), case.k_cache.astype(np.float16),
                            case.v_cache.astype(np.float16), case.block_table, case.seq_lens)
    np.testing.assert_array_equal(out16, out)


@pytest.mark.parametrize("name,case", CASES[::5], ids=[n for n, _ in CASES[::5]])
def test_independent_oracle_matches_reference_sdpa(name, case):
    out = oracle.sdpa_style_oracle(case.q, case.k_cache, case.v_cache, case.block_table, case.seq_lens,
                                   case.page_size)
    np.testing.assert_allclose(out, GOLDEN[f"{name}__sdpa"], rtol=1e-4, atol=1e-4)
