"""Benchmark of the B200 paged-attention decode path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c2|c3|c4|c5]

Prints ONE JSON line on rank 0.

Workload (default ``c2``): BASELINE config 2, the Qwen2.5-1.5B-shaped decode
(12 Q / 2 KV heads, head_dim 128, page 16, seq 4096, random page permutation)
at batch 64 -- the largest point of the batch-1..64 sweep the metric is quoted
on. A step is one decode call over the whole batch. ``value`` is achieved
KV-read bandwidth in TB/s: algorithmic bytes (sum_b seq_b * Hkv * D * 2 (K,V)
* 2 B, the reference's bench/roofline.py:55-59 formula) / device time, summed
over ranks (each rank decodes its own batch: weak scaling, no collective).

Extra keys (all printed by this script; the design notes cite them by name):
  sweep_c2_seq4096        C2 batch 1..64
  c2_b64_wide_table       C2 batch 64 with a block table twice as wide as the
                          sequences need (a serving engine's table)
  long_context_c3_batch1  C3 batch 1 at seq 8k / 32k / 128k (heuristic splits)
  num_splits_sweep_c3     C3 seq 32k, batch 1 and 4, num_splits 1..64 and the
                          heuristic (bench/bench_cuda_v4_num_splits.py:78-149
                          of the reference sweeps the same way)
  c4_llama8b_b256         C4, the ragged Llama-3-8B batch of 256
  c5_strong               C5 (1024 Llama-3-70B sequences) split over the N
                          ranks (equal sequence counts, as the config states)
                          through pad_b200.sharded.ShardedDecoder: strong
                          scaling, max-rank device time, gather time, sampled
                          oracle check
  c5_strong_token_balanced  the same with contiguous ranges of near-equal KV
                          tokens (balanced_ranges), N > 1 only
  host_us_per_call        CPU time of one paged_attention_decode_cuda_v4 call
                          (resident inputs, no copies, no sync inside)
  e2e / e2e_kv_resident   through the public API with host buffers
  e2e_kv_resident_pipelined  the same with the next step's upload overlapping
                          this step's decode (two staging buffers, a copy stream)
  cpu_baseline / cpu_port the reference's CPU path (src/reference.py as
                          shipped) / the C restatement, on the host cores
  same_box_*              the reference's Triton v4 and FlashInfer, timed the
                          same way (comparators, never on our path)

Timing: inputs are rotated over independent KV pools whose total exceeds L2
(126 MB), so every step reads HBM; steps are recorded once into a CUDA graph
(the per-call host overhead is measured separately) and replayed; CUDA events
on the launching stream bracket exactly K steps, with a barrier and device
synchronisation on both sides; multi-GPU takes the max over ranks.
``nvidia-smi`` samples clocks during the timed region.

``--impl reference`` times the reference's own CPU implementation of the
path -- ``paged_attention_decode_reference`` of src/reference.py, imported
unmodified from the offline install in baseline/_ref, on fp32 CPU tensors
with all host threads -- on a bounded sample of the same workload. Without
that install it falls back to the C restatement in oracle/ (kind "port").
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
for _p in (REPO, os.path.join(REPO, "paged-attention-decode_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)
REF_DIR = os.path.join(REPO, "baseline", "_ref")

import numpy as np  # noqa: E402

L2_BYTES = 126 * 2**20
GRAPH_STEPS = 100  # steps recorded per CUDA graph; the graph is replayed to reach K
C5_BATCH = 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c2", "c3", "c4", "c5"])
    ap.add_argument("--no-sweep", action="store_true", help="skip the sweeps and the same-box comparators")
    ap.add_argument("--no-extras", action="store_true",
                    help="time the workload only (no e2e, CPU baseline, C5 or sweeps); used for ncu captures")
    return ap.parse_args()


def workload_spec(name: str, n_gpus: int, rank: int):
    """(config name, batch, seq_len, seq_lens override) for this rank."""
    from pad_b200.cases import config_seq_lens
    from pad_b200.sharded import shard_range

    if name == "c2":
        return "c2", 64, 4096, None
    if name == "c3":
        return "c3", 1, 32768, None
    if name == "c4":
        return "c4", 256, None, None
    if name == "c5":  # batch 1024 split evenly by sequence across the GPUs
        lo, hi = shard_range(C5_BATCH, n_gpus, rank)
        return "c5", hi - lo, None, config_seq_lens("c5")[lo:hi]
    raise KeyError(name)


def metric_name(workload: str) -> str:
    if workload == "c2":
        return "decode-attn achieved KV HBM TB/s (Qwen2.5-1.5B shape, seq 4096, batch 64)"
    return f"decode-attn achieved KV HBM TB/s ({workload})"


def workload_config(workload: str, world: int) -> dict:
    """The `config` object, identical in both arms for the same workload."""
    from pad_b200.cases import CONFIGS

    cfg, batch, seq_len, _ = workload_spec(workload, world, 0)
    hq, hkv, d, ps, std = CONFIGS[cfg]
    wl = {"c2": "c2 batch=64 per GPU seq=4096", "c3": "c3 batch=1 per GPU seq=32768",
          "c4": "c4 batch=256 per GPU, ragged", "c5": f"c5 batch={C5_BATCH} split over {world} GPUs"}[workload]
    return {"workload": wl, "heads_q_kv": [hq, hkv], "head_dim": d, "page_size": ps,
            "inputs": f"fp16 N(0,{std}) q/K/V, random page permutation",
            "l2": "GPU arm: inputs rotated over independent KV pools totalling > 2.5x L2; CPU arm: host memory",
            "parallelism": f"batch-sharded x{world}, no collective on the decode path"}


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic():
    """DRAM bytes per launch of the decode kernel at C2 batch 64, from the
    committed ncu summary (measured once with ncu, not in this run)."""
    path = os.path.join(REPO, "profiles", "decode_stream_kernel_c2_b64.md")
    if not os.path.exists(path):
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", open(path).read())
    return float(m.group(1)) if m else None


def rate(nbytes, ms, peak_gbs):
    return {"us_per_call": round(ms * 1e3, 3), "TB_s": round(nbytes / (ms * 1e-3) / 1e12, 4),
            "frac_of_measured_hbm": round(nbytes / (ms * 1e-3) / 1e9 / peak_gbs, 4)}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.15)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            try:
                mhz.append(float(f[1]))
                mx = float(f[2])
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz)}


# ------------------------------------------------------------------ our arm
def make_pools(cfg, batch, seq_len, seq_lens, device, min_bytes, table_width=None):
    from pad_b200.cases import config_case, kv_bytes

    kw = dict(batch=batch, seq_len=seq_len, seq_lens=seq_lens, device=device, table_width=table_width)
    first = config_case(cfg, seed=0, **kw)
    per = kv_bytes(first.seq_lens.cpu().numpy(), first.k_cache.shape[2], first.k_cache.shape[3])
    # one pool is enough once a single step streams well past L2 (C5: ~36 GB)
    n = 1 if per >= min_bytes else max(2, min(64, math.ceil(min_bytes / max(per, 1))))
    pools = [first] + [config_case(cfg, seed=i, **kw) for i in range(1, n)]
    return pools, per


def time_device(pools, steps, warmup, torch, barrier, fn=None, num_splits=None):
    """Device time of `steps` decode calls rotated over `pools` (ms). `fn(case)`
    replaces the call of this package (used for the launcher and the
    same-box comparators)."""
    import pad_b200

    stream = torch.cuda.Stream()
    outs = [torch.empty_like(c.q) for c in pools]

    def call(i):
        c = pools[i % len(pools)]
        if fn is not None:
            fn(c)
            return
        pad_b200.paged_attention_decode_cuda_v4(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens,
                                                num_splits=num_splits, out=outs[i % len(pools)])

    with torch.cuda.stream(stream):
        for i in range(max(warmup, len(pools))):
            call(i)
    stream.synchronize()
    g_steps = min(GRAPH_STEPS, steps)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(g_steps):
            call(i)
    reps, tail = divmod(steps, g_steps)
    g_tail = None
    if tail:
        g_tail = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_tail, stream=stream):
            for i in range(tail):
                call(i)
    with torch.cuda.stream(stream):
        g.replay()
    stream.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(reps):
            g.replay()
        if g_tail is not None:
            g_tail.replay()
        end.record(stream)
    torch.cuda.synchronize()
    barrier()
    return start.elapsed_time(end)


def time_e2e(pool, steps, torch, barrier):
    """Through the public API with host buffers: per step H2D of every input
    (q, k_cache, v_cache, block_table, seq_lens) from pinned memory, the
    decode, and D2H of the output. Returns (ms per step, h2d bytes, d2h bytes)."""
    import pad_b200

    host = [t.cpu().pin_memory() for t in (pool.q, pool.k_cache, pool.v_cache, pool.block_table, pool.seq_lens)]
    dev = [torch.empty_like(t, device="cuda") for t in host]
    out_h = torch.empty(pool.q.shape, dtype=torch.float16).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = out_h.numel() * out_h.element_size()

    def step():
        for d, h in zip(dev, host):
            d.copy_(h, non_blocking=True)
        o = pad_b200.paged_attention_decode_cuda_v4(*dev)
        out_h.copy_(o, non_blocking=True)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    s.record()
    for _ in range(steps):
        step()
    e.record()
    torch.cuda.synchronize()
    barrier()
    return s.elapsed_time(e) / steps, h2d, d2h


def time_e2e_resident(pool, steps, torch):
    """KV cache resident in HBM (as in a serving engine); per step one H2D copy
    of the step's packed inputs (q, block_table and seq_lens staged together
    in one pinned buffer, the way a serving loop ships them), the decode
    through the public API (Python wrapper, torch operator, C ABI; no graph)
    and the D2H copy of the output."""
    import pad_b200

    parts = [pool.q.cpu(), pool.block_table.cpu().to(torch.int32), pool.seq_lens.cpu().to(torch.int32)]
    sizes = [t.numel() * t.element_size() for t in parts]
    offs = [0]
    for n in sizes:
        offs.append(offs[-1] + (n + 255) // 256 * 256)
    host = torch.empty(offs[-1], dtype=torch.uint8).pin_memory()
    for t, o, n in zip(parts, offs, sizes):
        host[o:o + n].copy_(t.contiguous().view(-1).view(torch.uint8))
    dev = torch.empty_like(host, device="cuda")
    q = dev[offs[0]:offs[0] + sizes[0]].view(torch.float16).view(pool.q.shape)
    bt = dev[offs[1]:offs[1] + sizes[1]].view(torch.int32).view(pool.block_table.shape)
    sl = dev[offs[2]:offs[2] + sizes[2]].view(torch.int32)
    out_h = torch.empty(pool.q.shape, dtype=torch.float16).pin_memory()
    out_d = torch.empty_like(pool.q)

    def step():
        dev.copy_(host, non_blocking=True)
        pad_b200.paged_attention_decode_cuda_v4(q, pool.k_cache, pool.v_cache, bt, sl, out=out_d)
        out_h.copy_(out_d, non_blocking=True)

    for _ in range(5):
        step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        step()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / steps, sum(sizes), out_h.numel() * out_h.element_size()


def time_e2e_resident_pipelined(pool, steps, torch):
    """As time_e2e_resident, but the way a serving loop overlaps transfers:
    two staging buffers, the next step's inputs uploaded on a copy stream
    while this step decodes, the output copied back on the copy stream once
    the decode is done. Every step still moves its own inputs H2D and its
    output D2H; ms per step is the steady-state period."""
    import pad_b200

    parts = [pool.q.cpu(), pool.block_table.cpu().to(torch.int32), pool.seq_lens.cpu().to(torch.int32)]
    sizes = [t.numel() * t.element_size() for t in parts]
    offs = [0]
    for n in sizes:
        offs.append(offs[-1] + (n + 255) // 256 * 256)
    host = torch.empty(offs[-1], dtype=torch.uint8).pin_memory()
    for t, o, n in zip(parts, offs, sizes):
        host[o:o + n].copy_(t.contiguous().view(-1).view(torch.uint8))
    bufs = [torch.empty_like(host, device="cuda") for _ in range(2)]
    views = [(b[offs[0]:offs[0] + sizes[0]].view(torch.float16).view(pool.q.shape),
              b[offs[1]:offs[1] + sizes[1]].view(torch.int32).view(pool.block_table.shape),
              b[offs[2]:offs[2] + sizes[2]].view(torch.int32)) for b in bufs]
    outs = [torch.empty_like(pool.q) for _ in range(2)]
    out_h = [torch.empty(pool.q.shape, dtype=torch.float16).pin_memory() for _ in range(2)]
    comp, copy = torch.cuda.current_stream(), torch.cuda.Stream()
    up = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    back = [torch.cuda.Event() for _ in range(2)]

    def run(n):
        with torch.cuda.stream(copy):
            bufs[0].copy_(host, non_blocking=True)
            up[0].record(copy)
        for i in range(n):
            cur, nxt = i % 2, (i + 1) % 2
            if i + 1 < n:
                with torch.cuda.stream(copy):
                    copy.wait_event(done[nxt]) if i >= 1 else None  # buffer nxt's last decode finished
                    bufs[nxt].copy_(host, non_blocking=True)
                    up[nxt].record(copy)
            comp.wait_event(up[cur])
            if i >= 2:
                comp.wait_event(back[cur])  # outs[cur] copied out two steps ago
            q, bt, sl = views[cur]
            pad_b200.paged_attention_decode_cuda_v4(q, pool.k_cache, pool.v_cache, bt, sl, out=outs[cur])
            done[cur].record(comp)
            with torch.cuda.stream(copy):
                copy.wait_event(done[cur])
                out_h[cur].copy_(outs[cur], non_blocking=True)
                back[cur].record(copy)
        comp.wait_stream(copy)

    run(6)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(comp)
    run(steps)
    e.record(comp)
    torch.cuda.synchronize()
    return s.elapsed_time(e) / steps, sum(sizes), out_h[0].numel() * out_h[0].element_size()


def host_us_per_call(pool, torch, calls=200):
    """CPU wall time of one paged_attention_decode_cuda_v4 call on resident
    inputs (no copies, no synchronisation inside the loop; the launches only
    queue, so this is the host cost of the wrapper and the C-ABI call)."""
    import pad_b200

    out = torch.empty_like(pool.q)
    args = (pool.q, pool.k_cache, pool.v_cache, pool.block_table, pool.seq_lens)
    for _ in range(10):
        pad_b200.paged_attention_decode_cuda_v4(*args, out=out)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(5):
        t0 = time.perf_counter()
        for _ in range(calls):
            pad_b200.paged_attention_decode_cuda_v4(*args, out=out)
        best = min(best, (time.perf_counter() - t0) / calls * 1e6)
        torch.cuda.synchronize()
    return round(best, 2)


def reference_gpu_comparator(torch, barrier, peak_gbs):
    """The reference's own GPU kernel timed on this box the same way (CUDA-graph
    replay over KV pools rotated past L2): its Triton v4 split-K kernel
    (src/kernel_v4_split_k.py:213, num_splits=16), imported from the offline
    install of the reference in baseline/_ref. Recorded beside our numbers,
    not a target. Its CUDA v4 kernel is not in that install (the package
    carries no .cu sources), so it cannot be built here."""
    if not os.path.isfile(os.path.join(REF_DIR, "kernel_v4_split_k.py")):
        return {"unavailable": "baseline/_ref (offline install of the reference) is absent"}
    sys.path.insert(0, REF_DIR)
    try:
        import kernel_v4_split_k as ref_tv4
    except Exception as e:  # noqa: BLE001 -- report, do not fail the bench
        return {"unavailable": f"importing the reference Triton v4 failed: {e!r}"[:200]}
    finally:
        sys.path.remove(REF_DIR)
    import pad_b200

    def fn(c):
        return ref_tv4.paged_attention_decode_v4(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens, num_splits=16)

    res = {"impl": "reference Triton v4 (src/kernel_v4_split_k.py, num_splits=16), same box and timing method"}
    for cfg, b, sl in (("c2", 1, 4096), ("c2", 64, 4096), ("c3", 1, 32768)):
        pl, nb = make_pools(cfg, b, sl, None, "cuda", 2.5 * L2_BYTES)
        c = pl[0]
        ours = pad_b200.paged_attention_decode_cuda_v4(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
        diff = (fn(c).float() - ours.float()).abs().max().item()
        m = time_device(pl, 200, 5, torch, barrier, fn=fn) / 200
        res[f"{cfg}_batch{b}_seq{sl}"] = dict(rate(nb, m, peak_gbs), max_abs_diff_vs_ours=diff)
        del pl
    return res


def flashinfer_comparator(torch, barrier, peak_gbs):
    """FlashInfer's paged decode (BatchDecodeWithPagedKVCacheWrapper, tensor
    cores, the configuration the reference's own adapter uses,
    src/flashinfer_adapter.py:92-107) on this box: planned once per KV pool
    with CUDA-graph buffers, then timed exactly like our kernel. A library
    comparator, recorded beside our numbers; never on our path."""
    try:
        import flashinfer
    except Exception as e:  # noqa: BLE001 -- report, do not fail the bench
        return {"unavailable": f"import flashinfer failed: {e!r}"[:200]}
    import pad_b200
    from pad_b200 import paged_kv_indices

    res = {"impl": f"flashinfer {getattr(flashinfer, '__version__', '?')} BatchDecodeWithPagedKVCacheWrapper "
                   "(NHD, use_tensor_cores=True, CUDA-graph buffers), same box and timing method"}
    try:
        for cfg, b, sl in (("c2", 1, 4096), ("c2", 64, 4096), ("c3", 1, 32768)):
            pl, nb = make_pools(cfg, b, sl, None, "cuda", 2.5 * L2_BYTES)
            c = pl[0]
            _, hq, d = c.q.shape
            _, ps, hkv, _ = c.k_cache.shape
            wraps = {}
            for cc in pl:
                ip, ix, lp = paged_kv_indices(cc.block_table, cc.seq_lens, ps)
                ws = torch.zeros(128 << 20, dtype=torch.uint8, device="cuda")
                wr = flashinfer.BatchDecodeWithPagedKVCacheWrapper(
                    ws, "NHD", use_cuda_graph=True, use_tensor_cores=True, paged_kv_indptr_buffer=ip.clone(),
                    paged_kv_indices_buffer=ix.clone(), paged_kv_last_page_len_buffer=lp.clone())
                wr.plan(ip, ix, lp, hq, hkv, d, ps, q_data_type=torch.float16, sm_scale=d ** -0.5)
                wraps[id(cc)] = (wr, torch.empty_like(cc.q))

            def fn(cc):
                wr, o = wraps[id(cc)]
                return wr.run(cc.q, (cc.k_cache, cc.v_cache), out=o)

            ours = pad_b200.paged_attention_decode_cuda_v4(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
            diff = (fn(c).float() - ours.float()).abs().max().item()
            m = time_device(pl, 200, 5, torch, barrier, fn=fn) / 200
            res[f"{cfg}_batch{b}_seq{sl}"] = dict(rate(nb, m, peak_gbs), max_abs_diff_vs_ours=diff)
            del pl, wraps
    except Exception as e:  # noqa: BLE001
        res["unavailable"] = f"flashinfer run failed: {e!r}"[:200]
    return res


# ------------------------------------------------------------------ CPU legs
def _reference_fn():
    """paged_attention_decode_reference of the reference's src/reference.py,
    imported unmodified from the offline install (baseline/_ref), or None."""
    if not os.path.isfile(os.path.join(REF_DIR, "reference.py")):
        return None
    sys.path.insert(0, REF_DIR)
    try:
        import reference
    except Exception:  # noqa: BLE001 -- the caller falls back to the port
        return None
    finally:
        sys.path.remove(REF_DIR)
    return reference.paged_attention_decode_reference


def cpu_sample(cfg, batch, seq_len, seq_lens, seconds: float, port: bool = False, steps_cap: int = 50,
               warmup: int = 1):
    """Time the reference's CPU path on a bounded sample of the workload: the
    first `take` sequences of the config, sized so one step takes about
    seconds / 4. Returns (TB/s of KV read, description, steps, step ms, kind, threads)."""
    import torch

    from pad_b200.cases import config_case, config_seq_lens, kv_bytes

    sl_all = np.asarray(seq_lens if seq_lens is not None else config_seq_lens(cfg, batch, seq_len))
    ref = None if port else _reference_fn()
    threads = os.cpu_count() or 1
    if ref is not None:
        torch.set_num_threads(threads)
        kind, what = "reference", "src/reference.py paged_attention_decode_reference (unmodified, baseline/_ref)"

        def run(c):
            t = [torch.from_numpy(np.ascontiguousarray(a)) for a in (c.q, c.k_cache, c.v_cache, c.block_table,
                                                                     c.seq_lens)]
            ref(*t)
    else:
        import oracle

        threads = oracle.max_threads()
        kind, what = "port", "C restatement of src/reference.py (oracle/pa_oracle.c)"

        def run(c):
            oracle.decode_c(c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens, nthreads=threads)

    # size the sample from a one-sequence probe; at most 64 sequences are built
    probe = config_case(cfg, seq_lens=sl_all[:1])
    run(probe)
    t0 = time.perf_counter()
    run(probe)
    dt = max(time.perf_counter() - t0, 1e-4)
    take = max(1, min(len(sl_all), 64, int((seconds / 4) / dt)))
    c = config_case(cfg, seq_lens=sl_all[:take])
    for _ in range(max(1, warmup)):
        run(c)
    calls, t0 = 0, time.perf_counter()
    while calls < steps_cap and (calls < 2 or time.perf_counter() - t0 < seconds):
        run(c)
        calls += 1
    el = time.perf_counter() - t0
    nb = kv_bytes(sl_all[:take], c.k_cache.shape[2], c.k_cache.shape[3])
    desc = (f"{take} of {len(sl_all)} sequences per step x {calls} steps ({el:.1f} s), {what}, fp32 on "
            f"{threads} host threads")
    return nb * calls / el / 1e12, desc, calls, el / calls * 1e3, kind, threads


def cpu_baselines(cfg, batch, seq_len, seq_lens):
    v, desc, _, _, kind, thr = cpu_sample(cfg, batch, seq_len, seq_lens, 10.0)
    res = {"cpu_baseline": {"value": v, "unit": "TB/s", "cores": thr, "kind": kind, "sample": desc}}
    if kind == "reference":
        v2, desc2, _, _, _, thr2 = cpu_sample(cfg, batch, seq_len, seq_lens, 5.0, port=True)
        res["cpu_port"] = {"value": v2, "unit": "TB/s", "cores": thr2, "kind": "port", "sample": desc2}
    return res


# ------------------------------------------------------------------ C5 strong scaling
def c5_strong(world, rank, local, torch, barrier, peak_gbs, steps=20, balanced=False):
    """C5 (1024 Llama-3-70B sequences) split over the ranks: each rank builds
    only its own sequences' KV pages, in a permuted local pool on its GPU,
    and decodes them through the launcher (ShardedDecoder). Device time is
    the max over ranks; the aggregate is all ranks' KV bytes over it. Then
    the outputs are gathered to rank 0 (timed separately) and every rank
    checks sampled sequences against the CPU oracle."""
    import oracle
    from pad_b200.cases import config_case, kv_bytes
    from pad_b200.sharded import LocalShard, ShardedDecoder, localize

    from pad_b200.cases import config_seq_lens
    from pad_b200.sharded import balanced_ranges

    ranges = balanced_ranges(config_seq_lens("c5"), world) if balanced else None
    if balanced:
        lo, hi = ranges[rank]
        sl = config_seq_lens("c5")[lo:hi]
    else:
        _, _, _, sl = workload_spec("c5", world, rank)
    c = config_case("c5", seq_lens=sl, device="cuda", seed=100 + rank)
    dec = ShardedDecoder(C5_BATCH, world, rank, torch.device("cuda", local), ranges=ranges)
    shard = LocalShard(dec.lo, dec.hi, c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)
    nb = kv_bytes(sl, c.k_cache.shape[2], c.k_cache.shape[3])
    ms = time_device([c], steps, 3, torch, barrier, fn=lambda _c: dec.decode(shard)) / steps
    t = torch.tensor([ms, nb, nb, nb], device="cuda", dtype=torch.float64)
    out = dec.decode(shard)
    # sampled oracle check of this rank's shard
    lens = sl
    idx = np.random.default_rng(rank).choice(len(lens), min(4, len(lens)), replace=False)
    idx = np.unique(np.concatenate([idx, [int(np.argmax(lens))]]))
    ti = torch.from_numpy(idx).cuda()
    sub = localize(c.q[ti], c.k_cache, c.v_cache, c.block_table[ti], c.seq_lens[ti], 1, 0, device="cpu")
    ref = oracle.decode_c(sub.q.numpy(), sub.k_cache.numpy(), sub.v_cache.numpy(), sub.block_table.numpy(),
                          sub.seq_lens.numpy())
    got = out[ti].float().cpu().numpy()
    err = np.abs(got - ref)
    ok = bool(np.all(err <= 2e-3 + 1e-2 * np.abs(ref)))
    e = torch.tensor([float(err.max()), 0.0 if ok else 1.0], device="cuda", dtype=torch.float64)
    gather_ms = None
    if world > 1:
        import torch.distributed as dist

        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        mn = t.clone()
        dist.all_reduce(mn, op=dist.ReduceOp.MIN)
        sm = t.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        dist.all_reduce(e, op=dist.ReduceOp.MAX)
        ms_max, bytes_total, bytes_max, bytes_min = mx[0].item(), sm[1].item(), mx[2].item(), mn[3].item()
        ms_min = mn[0].item()
        dec.gather(out)  # warm the collective
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        full = dec.gather(out)
        torch.cuda.synchronize()
        gather_ms = (time.perf_counter() - t0) * 1e3
        if rank == 0:
            assert full.shape[0] == C5_BATCH
    else:
        ms_max = ms_min = ms
        bytes_total = bytes_max = bytes_min = nb
    rows = torch.tensor([dec.hi - dec.lo], device="cuda", dtype=torch.int64)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(rows, op=dist.ReduceOp.MAX)
    return {"n_gpus": world, "sequences": C5_BATCH, "sequences_per_gpu_max": int(rows.item()),
            "split": "contiguous, near-equal KV tokens per rank" if balanced else "contiguous, equal sequence counts",
            "steps": steps,
            "us_per_call_max_rank": round(ms_max * 1e3, 2), "us_per_call_min_rank": round(ms_min * 1e3, 2),
            "TB_s_aggregate": round(bytes_total / (ms_max * 1e-3) / 1e12, 4),
            "frac_of_measured_hbm_per_gpu": round(bytes_total / world / (ms_max * 1e-3) / 1e9 / peak_gbs, 4),
            "kv_bytes_total": int(bytes_total), "kv_bytes_rank_max_over_min": round(bytes_max / bytes_min, 4),
            "gather_to_rank0_ms": None if gather_ms is None else round(gather_ms, 3),
            "launcher": "pad_b200.sharded.ShardedDecoder.decode (CUDA-graph replay), local permuted pools",
            "check": {"sampled_sequences_per_rank": int(len(idx)), "max_abs_err_vs_oracle": e[0].item(),
                      "within_tolerance": e[1].item() == 0.0, "tolerance": "2e-3 + 1e-2*|ref|"}}


# ------------------------------------------------------------------ our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        barrier = lambda: dist.barrier()  # noqa: E731
    else:
        barrier = lambda: None  # noqa: E731
    assert args.warmup >= 3, "at least 3 warm-up steps"
    import pad_b200
    from pad_b200.cases import CONFIGS

    cfg, batch, seq_len, seq_lens = workload_spec(args.workload, world, rank)
    hq, hkv, d, ps, _ = CONFIGS[cfg]
    pools, per_step_bytes = make_pools(cfg, batch, seq_len, seq_lens, "cuda", 2.5 * L2_BYTES)
    npools = len(pools)
    parts = pad_b200.partitions(local, batch, hkv, hq // hkv, d, ps, pools[0].block_table.shape[1])

    with ClockSampler(local) as clk:
        ms = time_device(pools, args.steps, args.warmup, torch, barrier)
    t = torch.tensor([ms, per_step_bytes], device="cuda", dtype=torch.float64)
    if world > 1:
        tb = t.clone()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(tb, op=dist.ReduceOp.SUM)
        total_bytes = tb[1].item()
    else:
        total_bytes = per_step_bytes
    ms = float(t[0].item())
    ms_per_step = ms / args.steps
    value = total_bytes * args.steps / (ms * 1e-3) / 1e12
    clocks = clk.summary()
    peak_gbs, peak_kind = peaks()
    achieved_gbs = per_step_bytes / (ms_per_step * 1e-3) / 1e9
    traffic = committed_traffic() if cfg == "c2" and batch == 64 else None

    extra = {}
    if args.no_extras:
        args.no_sweep = True
    else:
        e2e_ms, h2d, d2h = time_e2e(pools[0], 10 if per_step_bytes < 4e9 else 3, torch, barrier)
        te = torch.tensor([e2e_ms], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        extra["e2e"] = {"value": total_bytes / (te.item() * 1e-3) / 1e12, "unit": "TB/s",
                        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": te.item(),
                        "path": "pinned host -> device copies of q, k_cache, v_cache, block_table, seq_lens; "
                                "pad_b200.paged_attention_decode_cuda_v4; device -> host copy of out"}
        if rank == 0:
            res_ms, rh2d, rd2h = time_e2e_resident(pools[0], 200, torch)
            extra["e2e_kv_resident"] = {"value": per_step_bytes / (res_ms * 1e-3) / 1e12, "unit": "TB/s",
                                        "h2d_bytes_per_step": rh2d, "d2h_bytes_per_step": rd2h,
                                        "us_per_call": res_ms * 1e3}
            pp_ms, ph2d, pd2h = time_e2e_resident_pipelined(pools[0], 200, torch)
            extra["e2e_kv_resident_pipelined"] = {"value": per_step_bytes / (pp_ms * 1e-3) / 1e12, "unit": "TB/s",
                                                  "h2d_bytes_per_step": ph2d, "d2h_bytes_per_step": pd2h,
                                                  "us_per_call": pp_ms * 1e3}
            extra["host_us_per_call"] = host_us_per_call(pools[0], torch)
        del pools
        torch.cuda.empty_cache()
        extra["c5_strong"] = c5_strong(world, rank, local, torch, barrier, peak_gbs)
        torch.cuda.empty_cache()
        if world > 1:
            extra["c5_strong_token_balanced"] = c5_strong(world, rank, local, torch, barrier, peak_gbs, balanced=True)
            torch.cuda.empty_cache()
        if rank == 0 and world == 1:
            extra.update(cpu_baselines(cfg, batch, seq_len, seq_lens))
    if not args.no_sweep and world == 1 and args.workload == "c2":
        sweep = {}
        for b in (1, 2, 4, 8, 16, 32, 64):
            pl, nb = make_pools("c2", b, 4096, None, "cuda", 2.5 * L2_BYTES)
            sweep[str(b)] = rate(nb, time_device(pl, 1000, 10, torch, barrier) / 1000, peak_gbs)
            del pl
        extra["sweep_c2_seq4096"] = sweep
        pl, nb = make_pools("c2", 64, 4096, None, "cuda", 2.5 * L2_BYTES, table_width=512)
        extra["c2_b64_wide_table"] = dict(rate(nb, time_device(pl, 1000, 10, torch, barrier) / 1000, peak_gbs),
                                          block_table_width=512, pages_used_per_sequence=256)
        del pl
        lc = {}
        for sl_ in (8192, 32768, 131072):
            pl, nb = make_pools("c3", 1, sl_, None, "cuda", 2.5 * L2_BYTES)
            lc[str(sl_)] = rate(nb, time_device(pl, 1000, 10, torch, barrier) / 1000, peak_gbs)
            del pl
        extra["long_context_c3_batch1"] = lc
        sw = {}
        for b in (1, 4):
            pl, nb = make_pools("c3", b, 32768, None, "cuda", 2.5 * L2_BYTES)
            row = {}
            for s in (1, 2, 4, 8, 16, 32, 64, None):
                m = time_device(pl, 500, 10, torch, barrier, num_splits=s) / 500
                row["heuristic" if s is None else str(s)] = dict(
                    rate(nb, m, peak_gbs), partitions=pad_b200.partitions(local, b, 2, 6, 128, 32, 1024, s))
            sw[f"batch{b}"] = row
            del pl
        extra["num_splits_sweep_c3"] = dict(sw, seq_len=32768)
        pl, nb = make_pools("c4", 256, None, None, "cuda", 2.5 * L2_BYTES)
        extra["c4_llama8b_b256"] = dict(rate(nb, time_device(pl, 200, 10, torch, barrier) / 200, peak_gbs),
                                        kv_bytes=nb)
        del pl
        torch.cuda.empty_cache()
        extra["same_box_reference_gpu"] = reference_gpu_comparator(torch, barrier, peak_gbs)
        extra["same_box_flashinfer"] = flashinfer_comparator(torch, barrier, peak_gbs)

    if rank == 0:
        line = {
            "metric": metric_name(args.workload),
            "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "us_per_call": ms_per_step * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 in / f32 accumulate", "data": "synthetic",
            "config": workload_config(args.workload, world),
            "setup": {"partitions_per_gpu": parts, "kv_pools_rotated": npools,
                      "batch_per_gpu": batch},
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peak_gbs, "unit": "GB/s",
                         "frac": achieved_gbs / peak_gbs, "traffic": traffic,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6650 GB/s",
                         "kernel_time": "whole step (decode_stream_kernel + merge_kernel) per call",
                         "traffic_source": "ncu dram bytes per decode launch, profiles/decode_stream_kernel_c2_b64.md"},
            "clocks": clocks,
            "gpu_launches": args.steps * (2 if parts > 1 else 1),
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg, batch, seq_len, seq_lens = workload_spec(args.workload, world, 0)
    if cfg == "c5":  # the reference arm samples the whole 1024-sequence batch
        from pad_b200.cases import config_seq_lens

        seq_lens = config_seq_lens("c5")
    steps_cap = max(1, min(args.steps, 20))
    value, desc, steps, step_ms, kind, threads = cpu_sample(cfg, batch, seq_len, seq_lens, 20.0,
                                                            steps_cap=steps_cap, warmup=min(args.warmup, 3))
    print(json.dumps({
        "impl": "reference", "metric": metric_name(args.workload),
        "value": value, "unit": "TB/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.workload, world),
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": threads, "kind": kind, "sample": desc},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
