"""The allocation-free decode entry point, pad_paged_attention_decode_noalloc.

Some callers cannot allocate device memory at the moment they decode: code
running inside someone else's CUDA stream capture (where cudaMalloc is not
allowed), engines that hand all device memory to their own arena, and latency
paths that must never block in an allocator. For them the library carries its
own fixed scratch array (16 MiB per GPU) and this entry point uses it instead
of a caller-provided workspace. These tests call both entry points through
the C ABI on the same inputs, twice in a row (the scratch keeps the previous
call's contents, which must not matter), and require the same results within
the parity tolerance of the other GPU tests. This file is collected last so
that a run stopping at the first failure has already run everything else.
"""

import numpy as np
import pytest
import torch

import oracle
import pad_b200
from gpu_utils import assert_parity, to_gpu
from pad_b200 import _lib
from pad_b200.cases import config_case, explicit_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _noalloc(q, k, v, bt, sl, out, num_splits=0):
    lib = _lib.load()
    b, hq, d = q.shape
    p, ps, hkv, _ = k.shape
    stream = torch.cuda.current_stream().cuda_stream
    return lib.pad_paged_attention_decode_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), bt.data_ptr(), sl.data_ptr(), out.data_ptr(), b, hq, hkv, d, p,
        ps, bt.shape[1], _lib.i64_array(q.stride()), _lib.i64_array(k.stride()), _lib.i64_array(v.stride()),
        bt.stride(0), _lib.i64_array(out.stride()), 1.0 / d ** 0.5, num_splits, stream, 0)


CASES = [
    ("ragged_gqa6", lambda: explicit_case([1, 17, 300, 4000], num_kv_heads=2, gqa_ratio=6, head_dim=128,
                                          page_size=16, seed=5)),
    ("long_context_many_partials", lambda: config_case("c3", batch=1, seq_len=32768, seed=4)),
    ("c2_batch8", lambda: config_case("c2", batch=8)),
    ("small_pages_8_heads", lambda: explicit_case([228, 183, 376], num_kv_heads=8, gqa_ratio=4, head_dim=64,
                                                  page_size=4, seed=6)),
]


@pytest.mark.parametrize("name,make", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("num_splits", [None, 3])
def test_noalloc_matches_workspace_entry_two_calls(name, make, num_splits):
    c = make()
    q, k, v, bt, sl = to_gpu(c)
    ref = pad_b200.paged_attention_decode_cuda_v4(q, k, v, bt, sl, num_splits=num_splits).float().cpu().numpy()
    cpu = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        _lib.check(_noalloc(q, k, v, bt, sl, out, 0 if num_splits is None else num_splits))
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert_parity(got, ref, f"{name} S={num_splits} vs workspace entry")
        assert_parity(got, cpu, f"{name} S={num_splits} vs CPU oracle")


def test_noalloc_rejects_problems_larger_than_its_scratch():
    c = explicit_case([64] * 4, num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=7)
    q, k, v, bt, sl = to_gpu(c)
    out = torch.empty_like(q)
    # 2^15 splits per pair need far more than 16 MiB of partials
    rc = _noalloc(q, k, v, bt, sl, out, num_splits=1 << 15)
    assert rc == _lib.PAD_ERR_WORKSPACE
    assert b"static scratch" in _lib.load().pad_last_error()
    # and the entry point still works afterwards
    _lib.check(_noalloc(q, k, v, bt, sl, out))
    ref = pad_b200.paged_attention_decode_cuda_v4(q, k, v, bt, sl)
    assert_parity(out.float().cpu().numpy(), ref.float().cpu().numpy())


def test_noalloc_and_workspace_entries_agree_on_invalid_arguments():
    """Bad arguments get the same status from both entry points (the scratch
    size is checked only after the shared argument checks)."""
    c = explicit_case([64] * 2, num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=8)
    q, k, v, bt, sl = to_gpu(c)
    out = torch.empty_like(q)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")

    def both(**over):
        a = dict(b=q.shape[0], hq=q.shape[1], hkv=k.shape[2], d=q.shape[2], p=k.shape[0], ps=k.shape[1],
                 maxp=bt.shape[1], scale=1.0 / 128 ** 0.5, bts=bt.stride(0), qs=list(q.stride()))
        a.update(over)
        common = (q.data_ptr(), k.data_ptr(), v.data_ptr(), bt.data_ptr(), sl.data_ptr(), out.data_ptr(), a["b"],
                  a["hq"], a["hkv"], a["d"], a["p"], a["ps"], a["maxp"], _lib.i64_array(a["qs"]),
                  _lib.i64_array(k.stride()), _lib.i64_array(v.stride()), a["bts"], _lib.i64_array(out.stride()),
                  a["scale"], 0)
        r1 = lib.pad_paged_attention_decode(*common, ws.data_ptr(), ws.numel(), stream, 0)
        r2 = lib.pad_paged_attention_decode_noalloc(*common, stream, 0)
        return r1, r2

    for over in (dict(d=0), dict(d=96), dict(hq=9), dict(ps=0), dict(scale=float("inf")), dict(bts=1),
                 dict(qs=[1536, 128, 2])):
        r1, r2 = both(**over)
        assert r1 == r2 != _lib.PAD_OK, (over, r1, r2)
    assert both() == (_lib.PAD_OK, _lib.PAD_OK)
    torch.cuda.synchronize()
