"""Parity of the B200 decode kernel (through the C ABI) with the reference
oracle. Mirrors tests/test_kernel_cuda_v4.py of the reference: primary shape,
split invariance, oversplit, page boundary, GQA ratios, ragged batches, fuzz;
plus the golden fixtures, every BASELINE config, and size-independent
properties at full size."""

import functools
import os

import numpy as np
import pytest
import torch

import oracle
import pad_b200
from golden.golden_cases import golden_cases
from gpu_utils import assert_parity, run, to_gpu
from pad_b200.cases import config_case, explicit_case, random_case

pytestmark = pytest.mark.gpu

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "decode_golden.npz"))
CASES = golden_cases()
FUZZ_ITERS = int(os.environ.get("PAD_KERNEL_FUZZ_ITERS", "40"))


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


@pytest.mark.parametrize("name,case", CASES, ids=[n for n, _ in CASES])
def test_golden_heuristic_splits(name, case):
    assert_parity(run(case), GOLDEN[f"{name}__out"], name)


@pytest.mark.parametrize("name,case", CASES, ids=[n for n, _ in CASES])
@pytest.mark.parametrize("num_splits", [1, 3, 8])
def test_golden_explicit_splits(name, case, num_splits):
    assert_parity(run(case, num_splits=num_splits), GOLDEN[f"{name}__out"], f"{name}/S={num_splits}")


@pytest.mark.parametrize("num_splits", [1, 2, 4, 8, 16, 32, 64])
def test_split_invariance_seq_2000(num_splits):
    c = explicit_case([2000], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=600 + num_splits,
                      identity=True)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    assert_parity(run(c, num_splits=num_splits), ref, f"S={num_splits}")


@functools.lru_cache(maxsize=8)
def _c3_case(batch, seq_len):
    c = config_case("c3", batch=batch, seq_len=seq_len, seed=seq_len + batch)
    return c, oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)


C3_SPLITS = [1, 2, 4, 8, 16, 32, 64, None]


@pytest.mark.parametrize("batch,seq_len", [(1, 8192), (1, 32768), (4, 8192), (4, 32768), (1, 131072)])
@pytest.mark.parametrize("num_splits", C3_SPLITS)
def test_split_invariance_long_context_c3(batch, seq_len, num_splits):
    """page 32, N(0, 0.5) inputs, batch 1 and 4, every
    num_splits of the sweep (tests/test_kernel_cuda_v4.py:62-76 of the
    reference checks split invariance the same way)."""
    c, ref = _c3_case(batch, seq_len)
    assert_parity(run(c, num_splits=num_splits), ref, f"B={batch} seq={seq_len} S={num_splits}")


def test_c3_131072_batch4():
    c = config_case("c3", batch=4, seq_len=131072, seed=3)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    for s in (None, 64):
        assert_parity(run(c, num_splits=s), ref, f"131072 S={s}")


def test_num_splits_one_close_to_heuristic():
    c = explicit_case([1, 17, 4000], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=42)
    a, b = run(c, num_splits=1), run(c)
    np.testing.assert_allclose(a, b, rtol=1e-2, atol=1e-3)


def test_oversplit_more_splits_than_tokens():
    c = explicit_case([5], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=700)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    for s in (8, 64, 512):
        assert_parity(run(c, num_splits=s), ref, f"S={s}")


@pytest.mark.parametrize("gqa", [1, 2, 4, 6, 8, 12, 16])
def test_gqa_ratios(gqa):
    c = explicit_case([200, 777], num_kv_heads=2, gqa_ratio=gqa, head_dim=128, page_size=16, seed=100 + gqa)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    assert_parity(run(c), ref, f"G={gqa}")


@pytest.mark.parametrize("page_size", [1, 2, 4, 8, 12, 16, 24, 32, 64, 128, 256])
@pytest.mark.parametrize("head_dim", [16, 32, 64, 128])
def test_page_size_head_dim_matrix(page_size, head_dim):
    c = explicit_case([1, 63, 64, 65, 700], num_kv_heads=2, gqa_ratio=4, head_dim=head_dim, page_size=page_size,
                      seed=page_size * 1000 + head_dim)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    assert_parity(run(c), ref, f"ps={page_size} D={head_dim}")
    assert_parity(run(c, num_splits=5), ref, f"ps={page_size} D={head_dim} S=5")


def test_zero_length_rows_are_zero():
    c = explicit_case([0, 20, 0, 300], num_kv_heads=2, gqa_ratio=4, head_dim=128, page_size=16, seed=7)
    out = run(c)
    assert np.all(out[0] == 0) and np.all(out[2] == 0)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    assert_parity(out, ref)


def test_all_rows_empty():
    c = explicit_case([0, 0], num_kv_heads=2, gqa_ratio=4, head_dim=64, page_size=16, seed=8)
    assert np.all(run(c) == 0)


@pytest.mark.parametrize("seed", range(FUZZ_ITERS))
def test_fuzz_reference_matrix(seed):
    c = random_case(10_000 + seed, min_seq_len=0, max_seq_len=600)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    assert_parity(run(c), ref, f"seed={seed}")
    assert_parity(run(c, num_splits=4), ref, f"seed={seed} S=4")


def test_garbage_past_seq_len_is_never_used():
    """Slots past seq_len in the last page and unused pages hold NaN/Inf; the
    reference never reads them (src/reference.py:43-44) and neither may we."""
    c = explicit_case([5, 70, 129], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=11,
                      hole_fill="spare")
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    q, k, v, bt, sl = to_gpu(c)
    used = np.zeros(k.shape[:2], dtype=bool)
    for b, s in enumerate(c.seq_lens):
        for t in range(int(s)):
            used[c.block_table[b, t // 16], t % 16] = True
    mask = torch.from_numpy(~used).cuda()
    k[mask] = float("nan")
    v[mask] = float("inf")
    out = pad_b200.paged_attention_decode_cuda_v4(q, k, v, bt, sl).float().cpu().numpy()
    assert_parity(out, ref)


def test_bad_page_id_and_seq_len_are_flagged_not_faulted():
    c = explicit_case([40, 20], num_kv_heads=2, gqa_ratio=4, head_dim=64, page_size=16, seed=5)
    q, k, v, bt, sl = to_gpu(c)
    pad_b200.read_error_flags()
    bt[0, 1] = 10_000
    pad_b200.paged_attention_decode_cuda_v4(q, k, v, bt, sl)
    assert pad_b200.read_error_flags() & 0x1
    sl2 = sl.clone()
    sl2[1] = 10_000
    pad_b200.paged_attention_decode_cuda_v4(q, k, v, bt, sl2)
    assert pad_b200.read_error_flags() & 0x2


def test_non_contiguous_q_and_out_views():
    c = explicit_case([100, 900], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=12)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    q, k, v, bt, sl = to_gpu(c)
    big = torch.zeros(q.shape[0], q.shape[1] * 2, 128, dtype=torch.float16, device="cuda")
    big[:, ::2] = q
    qv = big[:, ::2]  # head stride 256 elements
    out_big = torch.zeros_like(big)
    ov = out_big[:, 1::2]
    pad_b200.paged_attention_decode_cuda_v4(qv, k, v, bt, sl, out=ov)
    assert_parity(ov.float().cpu().numpy(), ref)
    assert torch.all(out_big[:, ::2] == 0)


def test_side_stream_and_cuda_graph_replay():
    c = explicit_case([300, 4000, 17], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=13)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    q, k, v, bt, sl = to_gpu(c)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = pad_b200.paged_attention_decode_cuda_v4(q, k, v, bt, sl)
    s.synchronize()
    assert_parity(out.float().cpu().numpy(), ref)
    # capture (workspace sizing happens on the warm-up call above on this stream)
    g = torch.cuda.CUDAGraph()
    out_g = torch.empty_like(q)
    with torch.cuda.stream(s):
        pad_b200.paged_attention_decode_cuda_v4(q, k, v, bt, sl, out=out_g)
    s.synchronize()
    with torch.cuda.graph(g, stream=s):
        pad_b200.paged_attention_decode_cuda_v4(q, k, v, bt, sl, out=out_g)
    out_g.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert_parity(out_g.float().cpu().numpy(), ref)


@pytest.mark.parametrize("batch", [1, 2, 8, 32, 64])
def test_c2_batch_sweep_full_size(batch):
    c = config_case("c2", batch=batch)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    assert_parity(run(c), ref, f"C2 B={batch}")


def test_c1_config():
    c = config_case("c1")
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    assert_parity(run(c), ref)


def test_c4_ragged_llama8b_sampled():
    c = config_case("c4")
    out = run(c)
    idx = np.random.default_rng(0).choice(len(c.seq_lens), 32, replace=False)
    idx = np.concatenate([idx, [int(np.argmax(c.seq_lens)), int(np.argmin(c.seq_lens))]])
    ref = oracle.decode_c(c.q[idx], c.k_cache, c.v_cache, c.block_table[idx], c.seq_lens[idx])
    assert_parity(out[idx], ref, "C4 sampled")


def test_full_size_properties_c2_b64_on_device():
    """Size-independent properties at the full bench size: determinism,
    invariance to a relabelling of physical pages, and row independence."""
    c = config_case("c2", batch=64, device="cuda")
    q, k, v, bt, sl = c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens
    o1 = pad_b200.paged_attention_decode_cuda_v4(q, k, v, bt, sl)
    o2 = pad_b200.paged_attention_decode_cuda_v4(q, k, v, bt, sl)
    assert torch.equal(o1, o2)
    perm = torch.randperm(k.shape[0], device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel(), device="cuda")
    k2, v2 = k[perm], v[perm]          # physical page i of k2 holds old page perm[i]
    bt2 = inv[bt.long()].int()         # so logical page -> inv[old page]
    o3 = pad_b200.paged_attention_decode_cuda_v4(q, k2, v2, bt2, sl)
    assert torch.equal(o1, o3)
    for b in (0, 31, 63):
        solo = pad_b200.paged_attention_decode_cuda_v4(q[b:b + 1], k, v, bt[b:b + 1], sl[b:b + 1])
        torch.testing.assert_close(solo.float(), o1[b:b + 1].float(), rtol=1e-2, atol=2e-3)


@pytest.mark.parametrize("hkv", [1, 2, 4, 8])
@pytest.mark.parametrize("head_dim", [32, 64, 128])
@pytest.mark.parametrize("page_size", [1, 4, 16])
def test_head_group_page_split_matrix(hkv, head_dim, page_size):
    """Every head-group width (8/4/2/1 KV heads per tile) on the swizzled and
    unswizzled paths, with split counts that make partitions start on the last
    (partial) tile of one sequence and continue into the next -- the pattern
    that exercises the single-slot query ring."""
    seqs = [228, 183, 376, 95, 160]
    c = explicit_case(seqs, num_kv_heads=hkv, gqa_ratio=4, head_dim=head_dim, page_size=page_size,
                      seed=hkv * 100 + head_dim + page_size)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    for s in (None, 1, 2, 3, 4, 5, 6, 7, 9):
        assert_parity(run(c, num_splits=s), ref, f"hkv={hkv} D={head_dim} ps={page_size} S={s}")


def test_reused_workspace_split_then_empty_pair():
    """Merge descriptors live in the reused workspace: a pair split in one call
    and empty (seq_len 0) in the next must not be merged from stale partials."""
    a = explicit_case([8000, 9000], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=31)
    run(a)  # both pairs split across many partitions
    b = explicit_case([0, 9000], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=32)
    out = run(b)
    assert np.all(out[0] == 0)
    ref = oracle.decode_c(b.q, b.k_cache, b.v_cache, b.block_table, b.seq_lens)
    assert_parity(out, ref)


@pytest.mark.parametrize("block_n", [16, 64, 128, 256])
def test_triton_twin_signature(block_n):
    """The reference's Triton-v4 call surface (src/kernel_v4_split_k.py:213-222):
    num_splits defaults to 16, block_n is validated like the reference's and
    otherwise only accepted -- the B200 kernel picks its own token tile."""
    c = explicit_case([1, 300, 2500], num_kv_heads=2, gqa_ratio=6, head_dim=128, page_size=16, seed=77)
    ref = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    q, k, v, bt, sl = to_gpu(c)
    out = pad_b200.paged_attention_decode_v4(q, k, v, bt, sl, block_n=block_n)
    assert_parity(out.float().cpu().numpy(), ref, f"block_n={block_n}")
    out = pad_b200.paged_attention_decode_v4(q, k, v, bt, sl, num_splits=3, scale=0.05, block_n=block_n)
    ref2 = oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens, scale=0.05)
    assert_parity(out.float().cpu().numpy(), ref2, f"block_n={block_n} S=3 scale=0.05")
