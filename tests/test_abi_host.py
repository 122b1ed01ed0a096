"""C-ABI library load / symbol export, argument checks that need no GPU, the
Python wrapper's contract asserts, and the host mirror of the stream-K
partition (pad_b200.partition)."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

import pad_b200
from pad_b200 import _lib, partition

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "pad_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pad_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    syms = declared_symbols()
    assert "pad_paged_attention_decode" in syms
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in pad_b200.h but not exported"
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.pad_status_string(0) == b"ok"
    assert lib.pad_status_string(3).startswith(b"workspace")
    assert lib.pad_version() >= 100


def _decode(**over):
    lib = _lib.load()
    kw = dict(q=0, k=0, v=0, bt=0, sl=0, out=0, batch=2, hq=12, hkv=2, d=128, pages=10, ps=16, maxp=4,
              qs=[1536, 128, 1], ks=[4096, 256, 128, 1], vs=[4096, 256, 128, 1], bts=4, os=[1536, 128, 1],
              scale=0.088, splits=0, ws=0, wsb=0, stream=0, flags=0)
    kw.update(over)
    arr = lambda x: None if x is None else _lib.i64_array(x)  # noqa: E731
    return lib.pad_paged_attention_decode(kw["q"], kw["k"], kw["v"], kw["bt"], kw["sl"], kw["out"], kw["batch"],
                                          kw["hq"], kw["hkv"], kw["d"], kw["pages"], kw["ps"], kw["maxp"],
                                          arr(kw["qs"]), arr(kw["ks"]), arr(kw["vs"]), kw["bts"], arr(kw["os"]),
                                          kw["scale"], kw["splits"], kw["ws"], kw["wsb"], kw["stream"], kw["flags"])


def test_abi_rejects_bad_shapes_without_touching_a_device():
    assert _decode(batch=-1) == _lib.PAD_ERR_INVALID_ARGUMENT
    assert _decode(hq=10, hkv=4) == _lib.PAD_ERR_INVALID_ARGUMENT
    assert b"divisible" in _lib.load().pad_last_error()
    assert _decode(ps=0) == _lib.PAD_ERR_INVALID_ARGUMENT
    assert _decode(qs=None) == _lib.PAD_ERR_INVALID_ARGUMENT
    assert _decode(scale=float("nan")) == _lib.PAD_ERR_INVALID_ARGUMENT
    # batch 0 is a no-op
    assert _decode(batch=0) == _lib.PAD_OK
    # null tensors
    assert _decode() == _lib.PAD_ERR_INVALID_ARGUMENT
    # layout requirements (fake, never dereferenced, 16-byte aligned addresses)
    p = 1 << 20
    base = dict(q=p, k=p, v=p, bt=p, sl=p, out=p)
    assert _decode(**base, ks=[4096, 256, 128, 2]) == _lib.PAD_ERR_UNSUPPORTED
    assert _decode(**base, ks=[4096, 256, 129, 1]) == _lib.PAD_ERR_UNSUPPORTED
    assert _decode(**base, qs=[1536, 129, 1]) == _lib.PAD_ERR_UNSUPPORTED
    assert _decode(**dict(base, q=p + 2)) == _lib.PAD_ERR_UNSUPPORTED
    assert _decode(**base, bts=2) == _lib.PAD_ERR_INVALID_ARGUMENT


def _append(**over):
    lib = _lib.load()
    kw = dict(kn=0, vn=0, k=0, v=0, bt=0, pos=0, batch=2, hkv=2, d=128, pages=10, ps=16, maxp=4,
              kns=[256, 128, 1], vns=[256, 128, 1], ks=[4096, 256, 128, 1], vs=[4096, 256, 128, 1], bts=4)
    kw.update(over)
    arr = lambda x: None if x is None else _lib.i64_array(x)  # noqa: E731
    return lib.pad_paged_kv_append(kw["kn"], kw["vn"], kw["k"], kw["v"], kw["bt"], kw["pos"], kw["batch"], kw["hkv"],
                                   kw["d"], kw["pages"], kw["ps"], kw["maxp"], arr(kw["kns"]), arr(kw["vns"]),
                                   arr(kw["ks"]), arr(kw["vs"]), kw["bts"], 0, 0)


def test_kv_append_errors_set_the_last_error_text():
    """Every non-OK status of pad_paged_kv_append comes with its own message
    (never a stale one from an earlier call)."""
    lib = _lib.load()
    assert _decode(hq=10, hkv=4) == _lib.PAD_ERR_INVALID_ARGUMENT  # leaves a decode message behind
    assert _append(batch=-1) == _lib.PAD_ERR_INVALID_ARGUMENT
    assert b"kv_append" in lib.pad_last_error() and b"size" in lib.pad_last_error()
    assert _append() == _lib.PAD_ERR_INVALID_ARGUMENT
    assert b"null" in lib.pad_last_error()
    p = 1 << 20
    base = dict(kn=p, vn=p, k=p, v=p, bt=p, pos=p)
    assert _append(**base, bts=2) == _lib.PAD_ERR_INVALID_ARGUMENT
    assert b"stride" in lib.pad_last_error()
    assert _append(**base, ks=[4096, 256, 128, 2]) == _lib.PAD_ERR_UNSUPPORTED
    assert b"contiguous" in lib.pad_last_error()
    assert _append(batch=0) == _lib.PAD_OK


def test_wrapper_contract_asserts_on_cpu_tensors():
    q = torch.zeros(1, 12, 128, dtype=torch.float16)
    k = torch.zeros(4, 16, 2, 128, dtype=torch.float16)
    bt = torch.zeros(1, 4, dtype=torch.int32)
    sl = torch.ones(1, dtype=torch.int32)
    with pytest.raises(AssertionError):
        pad_b200.paged_attention_decode_cuda_v4(q, k, k, bt, sl)
    with pytest.raises(AssertionError):  # the Triton-v4 twin asserts the same contract
        pad_b200.paged_attention_decode_v4(q, k, k, bt, sl)


@pytest.mark.parametrize("seed", range(12))
@pytest.mark.parametrize("parts", [1, 3, 7, 148, 296, 1000])
def test_partition_covers_every_tile_once_with_disjoint_slots(seed, parts):
    rng = np.random.default_rng(seed)
    batch = int(rng.integers(1, 40))
    hkv = int(rng.choice([1, 2, 8]))
    seq = rng.integers(0, 3000, size=batch)
    seq[rng.random(batch) < 0.2] = 0
    total, pairs = partition.plan(seq, hkv, parts)
    if total == 0:
        return
    covered = np.zeros(total, dtype=np.int64)
    for w in range(parts):
        covered[partition.part_begin(w, total, parts):partition.part_begin(w + 1, total, parts)] += 1
    assert np.all(covered == 1)
    used = set()
    for pp in pairs:
        # the owner of every tile of the pair lies in [first_part, last_part]
        for t in (pp.first_tile, pp.first_tile + pp.n_tiles - 1):
            w = partition.part_owner(t, total, parts)
            assert partition.part_begin(w, total, parts) <= t < partition.part_begin(w + 1, total, parts)
        s = set(pp.slots)
        assert not (s & used)
        used |= s
        assert max(s) < parts + batch * hkv
    # pairs fully inside one partition are exactly the unsplit ones
    for pp in pairs:
        assert pp.split == (pp.first_part != pp.last_part)


def test_heuristic_partitions():
    assert partition.heuristic_partitions(148, 1, 64, 2, 6, 256, 16) == 148
    assert partition.heuristic_partitions(148, 1, 1, 2, 6, 1, 16) == 1  # tiny batch: one per tile
    # at most 16 (sequence, head group) pairs: a power-of-two partition count
    assert partition.heuristic_partitions(148, 1, 1, 2, 6, 1024, 32) == 128   # C3 batch 1, 32k
    assert partition.heuristic_partitions(148, 1, 16, 2, 6, 256, 16) == 128   # C2 batch 16
    assert partition.heuristic_partitions(148, 1, 17, 2, 6, 256, 16) == 148   # 17 pairs: all CTAs
    assert partition.heuristic_partitions(148, 1, 4, 8, 4, 512, 16) == 128    # 4 seqs x 1 group of 8 heads
    assert partition.heuristic_partitions(148, 1, 2, 2, 6, 64, 16) == 32      # capped by tiles (2 x 16)
    assert partition.head_group(8, 4) == 8 and partition.head_group(2, 6) == 2 and partition.head_group(6, 1) == 2
    assert partition.head_group(8, 16) == 4 and partition.head_group(3, 2) == 1


def test_build_entry_does_not_import_the_package(tmp_path):
    """__graft_entry__.build() must run on a fresh checkout, before any library
    exists: the build step is loaded by file path, never through pad_b200."""
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import importlib.util, os, sys; p = os.path.join(%r, 'paged-attention-decode_b200', 'pad_b200', 'build.py');"
            "s = importlib.util.spec_from_file_location('b', p); m = importlib.util.module_from_spec(s);"
            "s.loader.exec_module(m); assert 'pad_b200' not in sys.modules; print(m.LIB_PATH)") % root
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    import __graft_entry__

    assert "spec_from_file_location" in open(__graft_entry__.__file__).read()
