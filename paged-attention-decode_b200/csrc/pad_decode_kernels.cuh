// pad_decode_kernels.cuh -- the two decode kernels (see pad_decode_kernel.cuh
// for the design summary and the shared definitions).
#pragma once

#include <climits>

#include "pad_b200.h"
#include "pad_decode_kernel.cuh"

namespace pad {

__device__ __forceinline__ void raise_flag(const DecodeParams& p, int bits) {
  if (p.error_flags != nullptr) atomicOr(p.error_flags, bits);
}

#ifdef PAD_TRACE
// Development-only timeline: per-CTA %globaltimer stamps (compile with -DPAD_TRACE;
// read back with pad_debug_trace_read). Decode slots: 0 start, 10 dependency
// wait done, 13 seq_lens reduced (fast start), 7 producer ready, 5 first page
// ids ready, 14 first expect_tx, 15 first K/V TMA instruction, 2 first tile
// issued, 1 consumer scan done, 3 first tile ready, 4 last tile ready, 8 last
// tile computed, 11 / 12 epilogue barrier / add tree done, 9 consumer exit;
// 16-20 sums per CTA: producer wait and busy time, tiles, consumer (warp 0)
// wait and compute time. Merge slots: 0 start, 1 wait done, 3 folded, 2 end.
// Decode CTAs own 32 slots each; merge CTAs own 4 slots each after them.
__device__ uint64_t g_pad_trace[1024 * 32 + 4096 * 4];
#define PAD_STAMP(i) (g_pad_trace[blockIdx.x * 32 + (i)] = globaltimer_ns())
#define PAD_MSTAMP(i)                                                                                  \
  (g_pad_trace[1024 * 32 + ((blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) * 4 + (i)] = \
       globaltimer_ns())
#else
#define PAD_STAMP(i) ((void)0)
#define PAD_MSTAMP(i) ((void)0)
#endif

template <class TR>
__device__ __forceinline__ int tiles_of(int seq) {
  return (seq + TR::TT - 1) / TR::TT;
}

// seq_len of sequence b as given (dense: seq_lens[b]; CSR: from the page
// count and the last page's fill).
__device__ __forceinline__ int raw_seq(const DecodeParams& p, int b) {
  if (p.csr_indptr == nullptr) return __ldg(p.seq_lens + b);
  const int pages = __ldg(p.csr_indptr + b + 1) - __ldg(p.csr_indptr + b);
  return pages > 0 ? (pages - 1) * p.page_size + __ldg(p.csr_last + b) : 0;
}

// Offset of sequence b's row of page ids.
__device__ __forceinline__ int64_t row_base(const DecodeParams& p, int b) {
  return p.csr_indptr == nullptr ? (int64_t)b * p.bt_stride : (int64_t)__ldg(p.csr_indptr + b);
}

// seq_len of sequence b, clamped: from the shared-memory copy made by the
// prologue scan when the batch fits in it, else from global memory.
__device__ __forceinline__ int seq_of(const DecodeParams& p, const int* sseq, int b, int cap) {
  return b < kSeqCache ? sseq[b] : clamp_seq(raw_seq(p, b), cap);
}

// Step a cursor to the next tile of the flattened (sequence, head group,
// tile) list; past the end it reports n = 0. useq >= 0: every sequence has
// seq_len useq (no seq_lens lookup).
template <class TR>
__device__ __forceinline__ void cursor_next(Cursor& c, const DecodeParams& p, int cap, int ngroups, const int* sseq,
                                            int useq) {
  if (++c.i < c.n) return;
  c.i = 0;
  c.pair_start += c.n;
  if (++c.hg < ngroups) return;
  c.hg = 0;
  do {
    if (++c.b >= p.batch) {
      c.n = 0;
      return;
    }
    c.seq = useq >= 0 ? useq : seq_of(p, sseq, c.b, cap);
    c.n = tiles_of<TR>(c.seq);
    c.base = row_base(p, c.b);
  } while (c.n == 0);
}

// Cursor at global tile t of a dense batch whose sequences all have seq_len
// seq > 0 (the tile list is then a plain 3-level index).
template <class TR>
__device__ __forceinline__ Cursor uniform_cursor(int t, int seq, int ngroups, int64_t bt_stride) {
  const int n = tiles_of<TR>(seq), per = ngroups * n;
  const int b = t / per, r = t - b * per, hg = r / n, i = r - hg * n;
  return Cursor{b, hg, i, n, seq, t - i, (int64_t)b * bt_stride};
}

// Page holding token `tok` of a sequence, and the token's row in it (shift
// and mask for power-of-two page sizes).
__device__ __forceinline__ int page_of(const DecodeParams& p, int tok) {
  return p.page_shift >= 0 ? tok >> p.page_shift : tok / p.page_size;
}
__device__ __forceinline__ int row_in_page(const DecodeParams& p, int tok) {
  return p.page_shift >= 0 ? tok & (p.page_size - 1) : tok % p.page_size;
}

// Addresses of the page ids of the TMA boxes of the tile at cursor `c`: lane
// l takes boxes l, l + 32, ... Boxes past seq_len get no address (id 0, never
// issued).
template <class TR>
__device__ __forceinline__ void page_id_ptrs(const DecodeParams& p, const Cursor& c, int lane,
                                             const int32_t* (&dst)[TR::NB_PER_LANE]) {
  const int R = p.box_rows;
#pragma unroll
  for (int u = 0; u < TR::NB_PER_LANE; ++u) {
    const int j = lane + 32 * u;
    const int tok = c.i * TR::TT + j * R;
    dst[u] = (j * R < TR::TT && tok < c.seq) ? p.block_table + c.base + page_of(p, tok) : nullptr;
  }
}

// Page ids of the tile at cursor `c` (see page_id_ptrs). The loads are
// pinned in program order so that they start as early as written.
template <class TR>
__device__ __forceinline__ void load_page_ids(const DecodeParams& p, const Cursor& c, int lane,
                                              int (&dst)[TR::NB_PER_LANE]) {
  const int32_t* a[TR::NB_PER_LANE];
  page_id_ptrs<TR>(p, c, lane, a);
#pragma unroll
  for (int u = 0; u < TR::NB_PER_LANE; ++u) dst[u] = a[u] != nullptr ? ld_nc_early(a[u]) : 0;
}

template <class TR>
__device__ __forceinline__ void store_page_ids(int* slot_ids, int lane, const int (&v)[TR::NB_PER_LANE]) {
#pragma unroll
  for (int u = 0; u < TR::NB_PER_LANE; ++u)
    if (lane + 32 * u < TR::NB_MAX) slot_ids[lane + 32 * u] = v[u];
}

// Named barriers of the consumer warps (ids 1 and 2; 0 is __syncthreads).
// Safe from deadlock because consumer warps only ever leave the tile loop
// together: every exit decision goes through consumer_vote first.
constexpr uint32_t kConsumerThreads = 32 * kConsumerWarps;
__device__ __forceinline__ void consumer_sync() { named_barrier(1, kConsumerThreads); }
__device__ __forceinline__ bool consumer_vote(bool ok) { return named_barrier_and(2, kConsumerThreads, ok); }

template <class TR>
__global__ void __launch_bounds__(kThreads, 1) decode_stream_kernel(const __grid_constant__ DecodeParams p) {
  constexpr int D = TR::D, NT = TR::NT, HG = TR::HG, S = TR::STAGES, KSTEPS = TR::KSTEPS;
  constexpr int TT = TR::TT, WPH = TR::WPH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* qtiles = smem + S * TR::STAGE_BYTES;                        // [TR::QSLOTS][Q_BYTES]
  float* epi = reinterpret_cast<float*>(qtiles + TR::QSLOTS * TR::Q_BYTES);  // [HG][8*NT][D]
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(epi) + TR::EPI_BYTES);
  uint64_t* empty = full + S;
  uint64_t* qfull = empty + S;
  uint64_t* qempty = qfull + TR::QSLOTS;
  uint64_t* ebar = qempty + TR::QSLOTS;
  TileDesc* descs = reinterpret_cast<TileDesc*>(ebar + 2);
  int* ids = reinterpret_cast<int*>(descs + S);                      // [S][NB_MAX]
  float2* sml = reinterpret_cast<float2*>(ids + S * TR::NB_MAX);     // [warps][8*NT]
  float2* sML = sml + kConsumerWarps * 8 * NT;                       // [HG][8*NT]
  int* scan = reinterpret_cast<int*>(sML + HG * 8 * NT);             // [kThreads/32]
  volatile int* abort_flag = scan + 12;
  int* cur_smem = scan + 16;                                         // Cursor as 6 ints
  int* range_smem = scan + 40;                                       // t0, t1, total
  int* sink = scan + 24;                                             // [consumer warps] scratch
  int* sseq = scan + 64;                                             // [kSeqCache] clamped seq_lens

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cap = p.max_pages * p.page_size;
  const int64_t W = gridDim.x;
  const int w = blockIdx.x;
  const int G = p.gqa;
  const int ngroups = p.hkv / HG;
  if (tid == 0) PAD_STAMP(0);
  if (tid == 32 * kConsumerWarps) {  // producer lane 0: descriptors of the three tensor maps
    prefetch_tmap(&p.tm_k);
    prefetch_tmap(&p.tm_v);
    prefetch_tmap(&p.tm_q);
  }

  // ---- set-up, on this CTA's shared memory only (so before the wait on the
  // previous kernel): zero the query tiles (rows past HG*G stay zero), init
  // the barriers, make both visible to the async proxy and to every warp.
  for (int x = tid; x < TR::QSLOTS * TR::Q_BYTES / 16; x += kThreads)
    reinterpret_cast<uint4*>(qtiles)[x] = make_uint4(0, 0, 0, 0);
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int s = 0; s < TR::QSLOTS; ++s) {
      mbar_init(&qfull[s], 1);
      mbar_init(&qempty[s], kConsumerWarps);
    }
    mbar_init(&ebar[0], kConsumerWarps);
    *abort_flag = 0;
    cur_smem[0] = -1;
    fence_mbar_init();
  }
  fence_proxy_async_smem();  // zeroed query tiles before any TMA write to them
  __syncthreads();

  // A dense batch of at most kFastBatch sequences whose rows are all full
  // (seq_len == cap) has a tile list known from the parameters alone, so the
  // producer can fetch its first page ids in the same round trip as seq_lens.
  const int ncap = tiles_of<TR>(cap);
  const int tg_total = (p.csr_indptr == nullptr && p.batch <= kFastBatch) ? p.batch * ngroups * ncap : 0;
  const int tg0 = tg_total > 0 ? part_begin(w, tg_total, W) : 0;
  const int tg1 = tg_total > 0 ? part_begin(w + 1, tg_total, W) : 0;
  // the producer's guessed first cursor, the cursor S tiles on, and the
  // addresses of the guessed tiles' page ids
  Cursor gc{-1, 0, 0, 0, 0, 0, 0}, gla = gc;
  const int32_t* gptr[S][TR::NB_PER_LANE];
#pragma unroll
  for (int k = 0; k < S; ++k)
#pragma unroll
    for (int u = 0; u < TR::NB_PER_LANE; ++u) gptr[k][u] = nullptr;
  if (warp == kConsumerWarps && tg_total > 0) {
    gc = uniform_cursor<TR>(tg0, cap, ngroups, p.bt_stride);
    gla = gc;
#pragma unroll
    for (int k = 0; k < S; ++k) {
      if (tg0 + k < tg1) {
        page_id_ptrs<TR>(p, gla, lane, gptr[k]);
        cursor_next<TR>(gla, p, cap, ngroups, sseq, cap);
      }
    }
  }

  // Warm L2 with the first l2_warm guessed tiles while the previous kernel
  // runs -- the last consumer warp does it, so the producer's path to its
  // first TMA never waits on it, and the consumers wait for tile 0 anyway:
  // K/V boxes at the page ids read now (possibly stale -- they only steer
  // prefetches; the loads after the wait read the ids again), the query rows,
  // and the seq_lens lines. Reads go through L2 only, so no L1 line can feed
  // a later non-coherent load a stale value. Only for CTAs with at least 3
  // tiles: with 1-2 the warming warp is late for its own short run (measured
  // +0.4-0.7 us at C2 batch 2 and 4).
  if (warp == kConsumerWarps - 1 && tg_total > 0 && p.l2_warm > 0 && tg1 - tg0 >= 3) {
    Cursor pc = uniform_cursor<TR>(tg0, cap, ngroups, p.bt_stride);
    for (int b = 32 * lane; b < p.batch; b += 32 * 32) prefetch_l2(p.seq_lens + b);
    int pg[S][TR::NB_PER_LANE];
    {
      Cursor lc = pc;
#pragma unroll
      for (int k = 0; k < S; ++k) {
        const int32_t* a[TR::NB_PER_LANE];
        page_id_ptrs<TR>(p, lc, lane, a);
#pragma unroll
        for (int u = 0; u < TR::NB_PER_LANE; ++u)
          pg[k][u] = (k < p.l2_warm && tg0 + k < tg1 && a[u] != nullptr) ? ld_cg_i32(a[u]) : -1;
        if (tg0 + k < tg1) cursor_next<TR>(lc, p, cap, ngroups, sseq, cap);
      }
    }
    const uint64_t pol = l2_evict_normal_policy();
    const int R = p.box_rows;
#pragma unroll
    for (int k = 0; k < S; ++k) {
      if (k < p.l2_warm && tg0 + k < tg1) {
#pragma unroll
        for (int u = 0; u < TR::NB_PER_LANE; ++u) {
          const int page = pg[k][u];
          if ((unsigned)page >= (unsigned)p.num_pages) continue;
          const int row = row_in_page(p, pc.i * TT + (lane + 32 * u) * R);
#pragma unroll
          for (int sg = 0; sg < TR::NSEG; ++sg) {
            tma_prefetch_l2_4d(&p.tm_k, sg * (TR::SEGW / 2), row, pc.hg * HG, page, pol);
            tma_prefetch_l2_4d(&p.tm_v, sg * (TR::SEGW / 2), row, pc.hg * HG, page, pol);
          }
        }
        if (lane == 0 && (k == 0 || pc.i == 0))
#pragma unroll
          for (int sg = 0; sg < TR::NSEG; ++sg) tma_prefetch_l2_3d(&p.tm_q, sg * (TR::SEGW / 2), pc.hg * HG * G, pc.b);
        cursor_next<TR>(pc, p, cap, ngroups, sseq, cap);
      }
    }
  }

  // Launched as a programmatic dependent of the previous kernel in the
  // stream: everything above touches only this CTA's shared memory; wait for
  // the previous kernel's results (and for it to finish with the workspace)
  // before reading any input or writing any global memory.
  pdl_wait_primary();
  if (tid == 0) PAD_STAMP(10);

  if (warp == kConsumerWarps) {
    // =============================== producer warp ===============================
    // Fast start: when every seq_len is the same value L the partition's
    // range and first cursor have a closed form, so the producer needs no
    // block-wide scan. L == cap also validates the page ids loaded on the
    // guess above; otherwise they are loaded once L is known. Any other batch
    // takes the range and cursor from the consumer warps' scan.
    int t0 = 0, t1 = 0, total = 0, useq = -1;
    bool have_ids = false;
    Cursor c{-1, 0, 0, 0, 0, 0, 0};
    int pid[S][TR::NB_PER_LANE];
    if (tg_total > 0) {
#pragma unroll
      for (int k = 0; k < S; ++k)
#pragma unroll
        for (int u = 0; u < TR::NB_PER_LANE; ++u) pid[k][u] = gptr[k][u] != nullptr ? ld_nc_early(gptr[k][u]) : 0;
      int mn = INT_MAX, mx = INT_MIN;
#pragma unroll
      for (int u = 0; u < kFastBatch / 32; ++u) {
        const int b = lane + 32 * u;
        if (b < p.batch) {
          const int v = ld_nc_early(p.seq_lens + b);
          mn = min(mn, v);
          mx = max(mx, v);
        }
      }
      mn = __reduce_min_sync(0xffffffffu, mn);
      mx = __reduce_max_sync(0xffffffffu, mx);
      if (lane == 0) PAD_STAMP(13);
      if (mn == mx && mn > 0 && mn <= cap) {
        useq = mn;
        if (mn == cap) {
          t0 = tg0;
          t1 = tg1;
          total = tg_total;
          have_ids = true;
          c = gc;
        } else {
          total = p.batch * ngroups * tiles_of<TR>(mn);
          t0 = part_begin(w, total, W);
          t1 = part_begin(w + 1, total, W);
          if (t0 < total) c = uniform_cursor<TR>(t0, useq, ngroups, p.bt_stride);
        }
      }
    }
    if (useq >= 0) {
      named_barrier_arrive(3, kThreads);  // the consumers' hand-off is not needed
    } else {
      named_barrier(3, kThreads);
      t0 = range_smem[0];
      t1 = range_smem[1];
      total = range_smem[2];
      c = Cursor{cur_smem[0], cur_smem[1], cur_smem[2], cur_smem[3], cur_smem[4], cur_smem[5], 0};
      if (c.b >= 0) c.base = row_base(p, c.b);
    }
    const int ntiles = t1 - t0;
    if (lane == 0 && !p.meta_by_pair) p.ws_meta[w] = make_int4(-1, 0, 0, 0);
    if (lane == 0) PAD_STAMP(7);
    if (ntiles <= 0) {
      // An empty partition (more partitions than tiles) can sit between the
      // first and last partition of a split pair; it owns a partial slot of
      // that pair, which it marks empty (m = -inf, l = 0) for every head.
      if (c.b >= 0 && c.pair_start < t0) {
        const int slot = c.b * ngroups + c.hg + w;
        for (int x = lane; x < HG * G; x += 32) p.ws_ml[(int64_t)slot * HG * G + x] = make_float2(-INFINITY, 0.f);
      }
      return;
    }
    const int R = p.box_rows;
    const uint64_t kv_policy = l2_evict_first_policy();
    Cursor la = have_ids ? gla : c;
    if (!have_ids) {
#pragma unroll
      for (int k = 0; k < S; ++k) {
        if (k < ntiles) {
          load_page_ids<TR>(p, la, lane, pid[k]);
          cursor_next<TR>(la, p, cap, ngroups, sseq, useq);
        }
      }
    }
    if (lane == 0) PAD_STAMP(5);
#pragma unroll
    for (int k = 0; k < S; ++k)
      if (k < ntiles) store_page_ids<TR>(ids + k * TR::NB_MAX, lane, pid[k]);
    __syncwarp();
#ifdef PAD_TRACE
    uint64_t tr_pwait = 0, tr_pbusy = 0;
#endif
    int issued = 0, segs = 0;
    bool ok = true;
    const uint32_t qbytes = (uint32_t)(HG * G * TR::ROW_BYTES);
    for (int k = 0; k < ntiles; ++k) {
      const int s = k % S;
#ifdef PAD_TRACE
      const uint64_t tr0 = globaltimer_ns();
#endif
      if (k >= S) ok = mbar_wait_bounded(&empty[s], ((k / S) - 1) & 1, kWaitTimeoutNs);
#ifdef PAD_TRACE
      const uint64_t tr1 = globaltimer_ns();
      tr_pwait += tr1 - tr0;
#endif
      if (!__all_sync(0xffffffffu, ok) || *abort_flag) {
        ok = false;
        break;
      }
      // this tile's page ids: copied into its slot S tiles ago (one copy
      // group per tile; each lane reads only the ids it copied)
      if (k >= S) cp_async_wait_group<S - 1>();
      const int tok0 = c.i * TT;
      const int vt = min(TT, c.seq - tok0);
      const int nvalid = (vt + R - 1) >> p.box_rows_log2;
      const bool first = (k == 0) || (c.i == 0);
      const bool last = (k == ntiles - 1) || (c.i == c.n - 1);
      const int pair = c.b * ngroups + c.hg;
      const bool split = !(c.pair_start >= t0 && c.pair_start + c.n <= t1);
      const int qs = segs % TR::QSLOTS;
      // the query tile of a new segment: wait until its ring slot is free
      if (first && segs >= TR::QSLOTS) {
        ok = mbar_wait_bounded(&qempty[qs], ((segs / TR::QSLOTS) - 1) & 1, kWaitTimeoutNs);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      // K/V boxes first (the latency that matters), then the query tile and
      // the bookkeeping; the tile's phase completes only at the arrive below.
      if (lane == 0) mbar_expect_tx(&full[s], (uint32_t)nvalid * R * HG * TR::ROW_BYTES * 2);
      __syncwarp();
      if (k == 0 && lane == 0) PAD_STAMP(14);
      uint8_t* st = stages + s * TR::STAGE_BYTES;
      for (int j = lane; j < nvalid; j += 32) {
        const int page = ids[s * TR::NB_MAX + j];
        if ((unsigned)page >= (unsigned)p.num_pages) raise_flag(p, PAD_FLAG_BAD_PAGE_ID);
        const int row = row_in_page(p, tok0 + j * R);
#pragma unroll
        for (int sg = 0; sg < TR::NSEG; ++sg) {
          const int off = sg * kTileRows * TR::SEGW + j * (int)TR::box_pitch(R);
          tma_load_4d_hint(st + off, &p.tm_k, &full[s], sg * (TR::SEGW / 2), row, c.hg * HG, page, kv_policy);
          if (k == 0 && j == 0 && sg == 0) PAD_STAMP(15);
          tma_load_4d_hint(st + TR::KT_BYTES + off, &p.tm_v, &full[s], sg * (TR::SEGW / 2), row, c.hg * HG, page,
                           kv_policy);
        }
      }
      if (lane == 0) {
        if (first) {
          mbar_arrive_expect_tx(&qfull[qs], qbytes);
#pragma unroll
          for (int sg = 0; sg < TR::NSEG; ++sg)
            tma_load_3d(qtiles + qs * TR::Q_BYTES + sg * TR::QROWS * TR::SEGW, &p.tm_q, &qfull[qs],
                        sg * (TR::SEGW / 2), c.hg * HG * G, c.b);
        }
        TileDesc dsc;
        dsc.b = c.b;
        dsc.hg = c.hg;
        dsc.i = c.i;
        dsc.seq = c.seq;
        dsc.flags = (first ? kFirst : 0) | (last ? kLast : 0) | (split ? kSplit : 0);
        // Partial slots: pair p uses slots [p + owner(start_p), ...], one per
        // partition touching it; partition w writes slot p + w. These ranges
        // are disjoint across pairs and stay below partitions + pairs.
        dsc.slot = pair + w;
        dsc.qslot = qs;
        dsc.pad = 0;
        descs[s] = dsc;
        mbar_arrive(&full[s]);
        // The partition holding a pair's first tile publishes its merge
        // descriptor (indexed by pair or by partition, see meta_by_pair).
        if (c.i == 0 && (split || p.meta_by_pair)) {
          const int last_owner = part_owner((int64_t)c.pair_start + c.n - 1, total, W);
          p.ws_meta[p.meta_by_pair ? pair : w] =
              split ? make_int4(pair, pair + w, last_owner - w + 1, 1) : make_int4(-1, 0, 0, 0);
        }
      }
      if (k == 0 && lane == 0) PAD_STAMP(2);
      ++issued;
      if (first) ++segs;
      // page ids of tile k + S, straight into the slot this tile just freed
      if (k + S < ntiles) {
        const int32_t* a[TR::NB_PER_LANE];
        page_id_ptrs<TR>(p, la, lane, a);
#pragma unroll
        for (int u = 0; u < TR::NB_PER_LANE; ++u)
          if (lane + 32 * u < TR::NB_MAX)
            cp_async_4(ids + s * TR::NB_MAX + lane + 32 * u, a[u] != nullptr ? a[u] : p.block_table, a[u] != nullptr);
        cursor_next<TR>(la, p, cap, ngroups, sseq, useq);
      }
      cp_async_commit();
      cursor_next<TR>(c, p, cap, ngroups, sseq, useq);
#ifdef PAD_TRACE
      tr_pbusy += globaltimer_ns() - tr1;
#endif
    }
#ifdef PAD_TRACE
    if (lane == 0) {
      g_pad_trace[blockIdx.x * 32 + 16] = tr_pwait;
      g_pad_trace[blockIdx.x * 32 + 17] = tr_pbusy;
      g_pad_trace[blockIdx.x * 32 + 18] = ntiles;
    }
#endif
    cp_async_wait_all();
    if (!ok) {
      // Unwind: record the failure, stop the consumers, and wait (bounded)
      // for this CTA's own copies still in flight before exiting.
      if (lane == 0) {
        raise_flag(p, PAD_FLAG_WAIT_TIMEOUT);
        *abort_flag = 1;
        for (int k = max(0, issued - S); k < issued; ++k)
          (void)mbar_wait_bounded(&full[k % S], (k / S) & 1, kWaitTimeoutNs / 4);
        if (segs > 0)
          (void)mbar_wait_bounded(&qfull[(segs - 1) % TR::QSLOTS], ((segs - 1) / TR::QSLOTS) & 1, kWaitTimeoutNs / 4);
      }
    }
    return;
  }

  // =============================== consumer warps ===============================
  // ---- exclusive scan of tiles per sequence (x head groups) over the
  // consumer threads: this partition's tile range, its first cursor (handed
  // to the producer when it cannot use the fast start) and the seq_lens cache.
  int t0, t1, ntiles;
  {
    const int per = (p.batch + kConsumerThreads - 1) / kConsumerThreads;
    const int b_lo = min(p.batch, tid * per), b_hi = min(p.batch, b_lo + per);
    int local = 0, bad = 0, any_empty = 0;
    for (int b = b_lo; b < b_hi; ++b) {
      const int raw = raw_seq(p, b);
      bad |= (raw < 0 || raw > cap);
      const int sq = clamp_seq(raw, cap);
      if (b < kSeqCache) sseq[b] = sq;
      any_empty |= (sq == 0);
      local += tiles_of<TR>(sq);
    }
    local *= ngroups;
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) scan[warp] = incl;
    any_empty = !named_barrier_and(2, kConsumerThreads, !any_empty);
    int excl = incl - local, total = 0;
#pragma unroll
    for (int x = 0; x < kConsumerWarps; ++x) {
      const int v = scan[x];
      if (x < warp) excl += v;
      total += v;
    }
    if (bad && w == 0) raise_flag(p, PAD_FLAG_SEQ_LEN_RANGE);
    t0 = total > 0 ? part_begin(w, total, W) : 0;
    t1 = total > 0 ? part_begin(w + 1, total, W) : 0;
    if (t0 < total && excl <= t0 && t0 < excl + local) {
      int acc_t = excl;
      for (int b = b_lo; b < b_hi; ++b) {
        const int seq = seq_of(p, sseq, b, cap);
        const int n = tiles_of<TR>(seq);
        const int tb = n * ngroups;
        if (t0 < acc_t + tb) {
          const int o = t0 - acc_t;
          cur_smem[0] = b;
          cur_smem[1] = o / n;
          cur_smem[2] = o % n;
          cur_smem[3] = n;
          cur_smem[4] = seq;
          cur_smem[5] = acc_t + (o / n) * n;
          break;
        }
        acc_t += tb;
      }
    }
    if (tid == 0) {
      range_smem[0] = t0;
      range_smem[1] = t1;
      range_smem[2] = total;
    }
    named_barrier_arrive(3, kThreads);  // range, cursor and seq_lens cache to the producer
    if (tid == 0) PAD_STAMP(1);
    // the merge kernel may be scheduled now; it waits for this grid's results
    if (tid == 0) pdl_launch_dependents();

    // ---- zero output rows of empty sequences (src/reference.py:32-34)
    // (only when the scan saw one: no extra global reads on the common path)
    for (int b = w; any_empty && b < p.batch; b += (int)W) {
      if (seq_of(p, sseq, b, cap) == 0) {
        if (p.meta_by_pair && tid < ngroups) p.ws_meta[b * ngroups + tid] = make_int4(-1, 0, 0, 0);
        const int hq = p.hkv * G;
#pragma unroll 1
        for (int x = tid; x < hq * (D / 2); x += kConsumerThreads) {
          const int hh = x / (D / 2), d = (x % (D / 2)) * 2;
          *reinterpret_cast<__half2*>(p.out + b * p.out_sb + hh * p.out_sh + d) = __floats2half2_rn(0.f, 0.f);
        }
      }
    }
  }
  ntiles = t1 - t0;
  if (ntiles <= 0) return;
  const int hl = warp / WPH;               // local KV head this warp serves
  const uint32_t t_base = (warp % WPH) * 16;  // its 16 tokens within the tile
  const int lr = p.box_rows_log2;
  const int gl = 2 * (lane & 3);
  // this lane's ldmatrix rows: K (A operand of S^T) and V (A operand of O^T)
  uint32_t k_row, k_sw, v_row, v_sw;
  TR::kv_row(t_base + (lane & 7) + ((lane >> 3) & 1) * 8, hl, lr, k_row, k_sw);
  TR::kv_row(t_base + (lane & 7) + ((lane >> 4) & 1) * 8, hl, lr, v_row, v_sw);
  uint32_t qf[KSTEPS][NT][2];
  float acc[KSTEPS][NT][4];
  float m_run[NT][2], l_run[NT][2];
  int segs = 0;

#ifdef PAD_TRACE
  uint64_t tr_cwait = 0, tr_ccomp = 0;
#endif
  for (int k = 0; k < ntiles; ++k) {
    const int s = k % S;
#ifdef PAD_TRACE
    const uint64_t tc0 = globaltimer_ns();
#endif
    bool ok = mbar_wait_bounded(&full[s], (k / S) & 1, kWaitTimeoutNs);
#ifdef PAD_TRACE
    const uint64_t tc1 = globaltimer_ns();
    tr_cwait += tc1 - tc0;
#endif
    const TileDesc dsc = descs[s];
    if (ok && (dsc.flags & kFirst)) {
      const int qs = dsc.qslot;
      ok = mbar_wait_bounded(&qfull[qs], (segs / TR::QSLOTS) & 1, kWaitTimeoutNs);
      const uint32_t qb = smem_u32(qtiles + qs * TR::Q_BYTES);
      const uint32_t qrow0 = hl * G;
      if constexpr (KSTEPS == 1) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          ldsm_x2(TR::q_addr(qb, qrow0 + nt * 8 + (lane & 7), (lane >> 3) & 1), qf[0][nt][0], qf[0][nt][1]);
      } else {
#pragma unroll
        for (int kk = 0; kk < KSTEPS; kk += 2)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            ldsm_x4(TR::q_addr(qb, qrow0 + nt * 8 + (lane & 7), kk * 2 + (lane >> 3)), qf[kk][nt][0],
                    qf[kk][nt][1], qf[kk + 1][nt][0], qf[kk + 1][nt][1]);
      }
      // The slot may be refilled by TMA as soon as it is released, so every
      // lane must have its ldmatrix results in registers first: a store that
      // depends on all fragment registers makes the warp wait for them.
      uint32_t chk = 0;
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) chk ^= qf[kk][nt][0] ^ qf[kk][nt][1];
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(smem_u32(sink + warp)), "r"(chk) : "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&qempty[qs]);
      ++segs;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        m_run[nt][0] = m_run[nt][1] = -INFINITY;
        l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
        for (int mt = 0; mt < KSTEPS; ++mt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.f;
      }
    }
    // collective go/no-go: all consumer warps continue or all leave
    if (!consumer_vote(ok && !*abort_flag)) {
      if (warp == 0 && lane == 0) {
        raise_flag(p, PAD_FLAG_WAIT_TIMEOUT);
        *abort_flag = 1;
      }
      return;
    }
    const uint32_t kb = smem_u32(stages + s * TR::STAGE_BYTES);
    const uint32_t vb = kb + TR::KT_BYTES;
    if (k == 0 && warp == 0 && lane == 0) PAD_STAMP(3);
    if (k == ntiles - 1 && warp == 0 && lane == 0) PAD_STAMP(4);

    const int nv = min(16, dsc.seq - (dsc.i * TT + (int)t_base));
    if (nv > 0) {
      if (nv < 16) {
        // Rows past seq_len hold whatever the page (or an earlier tile) left
        // there -- possibly NaN/Inf. Zero this warp's V rows so 0-probability
        // tokens contribute exactly 0; K rows are masked through the scores.
        for (int x = lane; x < (16 - nv) * (D / 8); x += 32) {
          const uint32_t t = t_base + nv + x / (D / 8), cc = x % (D / 8);
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(TR::kv_addr(vb, t, hl, cc, lr)), "r"(0)
                       : "memory");
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
      // S^T[16 tokens x 8*NT rows] = K[16 x D] . Q^T
      float sc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(TR::kv_at(kb, k_row, k_sw, kk * 2 + (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(sc[nt], a0, a1, a2, a3, qf[kk][nt][0], qf[kk][nt][1]);
      }
      // scale into log2 units, mask tokens past seq_len
      const bool v_lo = (lane >> 2) < nv, v_hi = (lane >> 2) + 8 < nv;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        sc[nt][0] = v_lo ? sc[nt][0] * p.scale_log2 : -INFINITY;
        sc[nt][1] = v_lo ? sc[nt][1] * p.scale_log2 : -INFINITY;
        sc[nt][2] = v_hi ? sc[nt][2] * p.scale_log2 : -INFINITY;
        sc[nt][3] = v_hi ? sc[nt][3] * p.scale_log2 : -INFINITY;
      }
      // online softmax (per query row, over this warp's tokens)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float mx = fmaxf(sc[nt][j], sc[nt][j + 2]);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float mn = fmaxf(m_run[nt][j], mx);
          const float mu = (mn == -INFINITY) ? 0.f : mn;
          const float alpha = ex2(m_run[nt][j] - mu);
          const float p0 = ex2(sc[nt][j] - mu), p1 = ex2(sc[nt][j + 2] - mu);
          sc[nt][j] = p0;
          sc[nt][j + 2] = p1;
          l_run[nt][j] = l_run[nt][j] * alpha + p0 + p1;
          m_run[nt][j] = mn;
#pragma unroll
          for (int mt = 0; mt < KSTEPS; ++mt) {
            acc[mt][nt][j] *= alpha;
            acc[mt][nt][j + 2] *= alpha;
          }
        }
      }
      // P^T as the B operand, split into two fp16 terms P = P_hi + P_lo
      // (P_hi = fp16(P), P_lo = fp16(P - P_hi)), each transposed 8x8-blockwise
      // in registers. Two MMAs per k-step then give O with P at ~22 bits, so
      // O's numerator matches the fp32 l it is divided by; a single fp16 P
      // alone leaves relative errors near 1e-2 on small outputs.
      uint32_t pb[NT][2], pl[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float x0 = sc[nt][2 * h], x1 = sc[nt][2 * h + 1];
          const __half2 hi = __floats2half2_rn(x0, x1);
          const float2 hf = __half22float2(hi);
          pb[nt][h] = movmatrix_trans(*reinterpret_cast<const uint32_t*>(&hi));
          pl[nt][h] = movmatrix_trans(pack_half2(x0 - hf.x, x1 - hf.y));
        }
      // O^T[D x 8*NT] += V^T[D x 16 tokens] . (P_hi^T + P_lo^T)
#pragma unroll
      for (int mt = 0; mt < KSTEPS; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_trans(TR::kv_at(vb, v_row, v_sw, mt * 2 + ((lane >> 3) & 1)), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_16816(acc[mt][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
          mma_16816(acc[mt][nt], a0, a1, a2, a3, pl[nt][0], pl[nt][1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
#ifdef PAD_TRACE
    tr_ccomp += globaltimer_ns() - tc1;
#endif

    if (k == ntiles - 1 && warp == 0 && lane == 0) PAD_STAMP(8);
    if (dsc.flags & kLast) {
      // ------------- segment epilogue: merge the WPH warps of each head, write
      // the fp16 output rows (pair finished here) or the fp32 partial (split pair)
      float lsum[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float l = l_run[nt][j];
          l += __shfl_xor_sync(0xffffffffu, l, 4);
          l += __shfl_xor_sync(0xffffffffu, l, 8);
          l += __shfl_xor_sync(0xffffffffu, l, 16);
          lsum[nt][j] = l;
        }
      const bool split = (dsc.flags & kSplit) != 0;
      const int qrow0 = dsc.hg * HG * G + hl * G;  // first query head of this warp's KV head
      if constexpr (WPH == 1) {
        // one warp per head: write straight from the accumulator fragments
        const int64_t prow = ((int64_t)dsc.slot * HG + hl) * G;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int g = nt * 8 + gl + j;
            if (g >= G) continue;
            const float L = lsum[nt][j];
            const float inv = L > 0.f ? 1.f / L : 0.f;
            if (split && (lane >> 2) == 0) p.ws_ml[prow + g] = make_float2(m_run[nt][j], L);
#pragma unroll
            for (int mt = 0; mt < KSTEPS; ++mt)
#pragma unroll
              for (int hi = 0; hi < 2; ++hi) {
                const int d = mt * 16 + (lane >> 2) + hi * 8;
                const float v = acc[mt][nt][j + 2 * hi];
                if (split) p.ws_o[(prow + g) * D + d] = v;
                else p.out[dsc.b * p.out_sb + (int64_t)(qrow0 + g) * p.out_sh + d] = __float2half_rn(v * inv);
              }
          }
      } else {
        // The WPH warps of a head merge their O^T into EPI_BUFS buffers in a
        // fixed order (deterministic results). Warp tb of the head writes
        // buffer tb % EPI_BUFS at step tb / EPI_BUFS: step 0 stores its
        // accumulator unscaled, beside every warp's (m, l); step 1 rescales
        // that content to the head's running max and adds its own; later
        // steps add. One barrier fewer than exchanging (m, l) first.
        constexpr int NB = TR::EPI_BUFS, LD = TR::EPI_LD, BUF = HG * 8 * NT * LD;
        static_assert(WPH / NB >= 2, "every buffer gets a rescaling add");
        const int tb = (int)(t_base / 16);
        float* buf = epi + (tb % NB) * BUF + hl * (8 * NT * LD);
        if ((lane >> 2) == 0) {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 2; ++j) sml[warp * 8 * NT + nt * 8 + gl + j] = make_float2(m_run[nt][j], lsum[nt][j]);
        }
        if (tb < NB) {
#pragma unroll
          for (int mt = 0; mt < KSTEPS; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e)
                buf[(nt * 8 + gl + (e & 1)) * LD + mt * 16 + (lane >> 2) + (e >= 2 ? 8 : 0)] = acc[mt][nt][e];
        }
        consumer_sync();
        if (k == ntiles - 1 && warp == 0 && lane == 0) PAD_STAMP(11);
        // scale of this warp's rows, and of the warp that stored this buffer
        float scl[NT][2], s0[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int g = nt * 8 + gl + j;
            float M = -INFINITY;
#pragma unroll
            for (int ww = 0; ww < WPH; ++ww) M = fmaxf(M, sml[(hl * WPH + ww) * 8 * NT + g].x);
            const float Mu = (M == -INFINITY) ? 0.f : M;
            scl[nt][j] = ex2(m_run[nt][j] - Mu);
            s0[nt][j] = ex2(sml[(hl * WPH + tb % NB) * 8 * NT + g].x - Mu);
            if (t_base == 0 && (lane >> 2) == 0) {
              float L = 0.f;
#pragma unroll
              for (int ww = 0; ww < WPH; ++ww) {
                const float2 x = sml[(hl * WPH + ww) * 8 * NT + g];
                L += x.y * ex2(x.x - Mu);
              }
              sML[hl * 8 * NT + g] = make_float2(Mu, L);
            }
          }
#pragma unroll 1
        for (int step = 1; step < WPH / NB; ++step) {
          if (tb / NB == step) {
#pragma unroll
            for (int mt = 0; mt < KSTEPS; ++mt)
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int idx = (nt * 8 + gl + (e & 1)) * LD + mt * 16 + (lane >> 2) + (e >= 2 ? 8 : 0);
                  const float v = acc[mt][nt][e] * scl[nt][e & 1];
                  if (step == 1) buf[idx] = buf[idx] * s0[nt][e & 1] + v;
                  else buf[idx] += v;
                }
          }
          consumer_sync();
        }
        if (k == ntiles - 1 && warp == 0 && lane == 0) PAD_STAMP(12);
        const int ctid = warp * 32 + lane;
        if (!split) {
          __half* obase = p.out + dsc.b * p.out_sb + (int64_t)(dsc.hg * HG * G) * p.out_sh;
#pragma unroll 1
          for (int x = ctid; x < HG * G * (D / 2); x += 32 * kConsumerWarps) {
            const int row = x / (D / 2), d = (x % (D / 2)) * 2;
            const int h = row / G, g = row % G;
            const float L = sML[h * 8 * NT + g].y;
            const float inv = L > 0.f ? 1.f / L : 0.f;
            const float* src = epi + h * (8 * NT * LD) + g * LD + d;
            float v0 = src[0], v1 = src[1];
            if constexpr (NB == 2) {
              v0 += src[BUF];
              v1 += src[BUF + 1];
            }
            *reinterpret_cast<__half2*>(obase + row * p.out_sh + d) = __floats2half2_rn(v0 * inv, v1 * inv);
          }
        } else {
          float4* o4 = reinterpret_cast<float4*>(p.ws_o + (int64_t)dsc.slot * HG * G * D);
#pragma unroll 1
          for (int x = ctid; x < HG * G * (D / 4); x += 32 * kConsumerWarps) {
            const int row = x / (D / 4), d = (x % (D / 4)) * 4;
            const int h = row / G, g = row % G;
            float4 v = *reinterpret_cast<const float4*>(epi + h * (8 * NT * LD) + g * LD + d);
            if constexpr (NB == 2) {
              const float4 u = *reinterpret_cast<const float4*>(epi + BUF + h * (8 * NT * LD) + g * LD + d);
              v = make_float4(v.x + u.x, v.y + u.y, v.z + u.z, v.w + u.w);
            }
            o4[x] = v;
          }
          for (int x = ctid; x < HG * G; x += 32 * kConsumerWarps)
            p.ws_ml[(int64_t)dsc.slot * HG * G + x] = sML[(x / G) * 8 * NT + x % G];
        }
        // No trailing sync: the next epilogue's first sync orders these reads
        // before any warp writes the buffer again.
      }
    }
  }
  if (warp == 0 && lane == 0) PAD_STAMP(9);
#ifdef PAD_TRACE
  if (warp == 0 && lane == 0) {
    g_pad_trace[blockIdx.x * 32 + 19] = tr_cwait;
    g_pad_trace[blockIdx.x * 32 + 20] = tr_ccomp;
  }
#endif
}

// Phase 2: merge the partials of one split (sequence, head group) pair for
// one (head, query row). Grid (partitions, HG*G); partition w works only if
// it is the first partition of a split pair (ws_meta[w].w == 1); when there
// are fewer pairs than partitions the grid and descriptors go by pair instead.
//   M = max_s m_s;  L = sum_s l_s 2^(m_s - M);  O = sum_s O_s 2^(m_s - M) / L
// (analysis/split_k_derivation.md:44-65; a partial with m_s = -inf weighs 0
// and its O is not read, the guard of analysis/split_k_derivation.md:67-86).
// Each thread folds a strided subset of the partials with an online LSE
// (loads issued 4 or 8 at a time), then the per-thread states are combined
// through shared memory. Launched as a programmatic dependent of the decode
// kernel: it waits on griddepcontrol before reading the partials.
template <int D, int kMergeThreads, int DS, int UNR>
__global__ void __launch_bounds__(kMergeThreads) merge_kernel(const float* __restrict__ ws_o,
                                                              const float2* __restrict__ ws_ml,
                                                              const int4* __restrict__ ws_meta,
                                                              __half* __restrict__ out, int64_t out_sb,
                                                              int64_t out_sh, int ngroups, int rows,
                                                              int guess_ncap, int guess_parts) {
  constexpr int DC = D / DS;               // columns of D this CTA merges (blockIdx.z picks which)
  constexpr int C4 = DC / 4;               // float4 columns of one partial row slice
  constexpr int PG = kMergeThreads / C4;   // partial groups folded in parallel
  constexpr int NW = kMergeThreads / 32;   // warps
  static_assert(C4 <= 32 && 32 % C4 == 0, "a warp holds whole groups");
  __shared__ float red_o[NW][DC];
  __shared__ float red_m[NW], red_l[NW];
  if (threadIdx.x == 0) PAD_MSTAMP(0);
  pdl_launch_dependents();  // the next decode may start its own set-up
  const int w = blockIdx.x, y = blockIdx.y, tid = threadIdx.x;
  // A dense batch whose rows are all full (guess_ncap > 0, grid by pair) has
  // its split descriptors in closed form: pair w covers tiles
  // [w * ncap, (w + 1) * ncap) of pairs * ncap over guess_parts partitions.
  // (Parameters only: computed before the wait.)
  int gs0 = 0, gns = 0;
  if (guess_ncap > 0) {
    const int64_t total = (int64_t)gridDim.x * guess_ncap, f = (int64_t)w * guess_ncap;
    const int o0 = part_owner(f, total, guess_parts), o1 = part_owner(f + guess_ncap - 1, total, guess_parts);
    gs0 = w + o0;
    gns = o1 - o0 + 1;
  }
  pdl_wait_primary();
  if (tid == 0) PAD_MSTAMP(1);
  const int c = tid % C4 + blockIdx.z * C4, sg = tid / C4;
  float m = -INFINITY, l = 0.f;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  // Fold partial slots [s0, s0 + ns) into (m, l, a). With a guess, the loads
  // (pinned in program order, see ld_nc_*) go out with the descriptor load;
  // a wrong guess folds again from the descriptor (one copy of the loop).
  const int4 meta = ld_nc_i4(ws_meta + w);
  int s0 = gs0, ns = gns;
  if (gns <= 1) {
    if (meta.w != 1) return;
    s0 = meta.y;
    ns = meta.z;
  }
  for (;;) {
    for (int s = sg; s < ns; s += UNR * PG) {
      float2 ml[UNR];
      float4 o[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int su = s + u * PG;
        ml[u] = make_float2(-INFINITY, 0.f);
        if (su < ns) {
          const int64_t row = (int64_t)(s0 + su) * rows + y;
          ml[u] = ld_nc_f2(ws_ml + row);
          o[u] = ld_nc_f4(ws_o + row * D + 4 * c);
        }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        if (ml[u].x == -INFINITY) continue;
        const float mn = fmaxf(m, ml[u].x);
        const float al = ex2(m - mn), be = ex2(ml[u].x - mn);
        l = l * al + ml[u].y * be;
        a.x = a.x * al + o[u].x * be;
        a.y = a.y * al + o[u].y * be;
        a.z = a.z * al + o[u].z * be;
        a.w = a.w * al + o[u].w * be;
        m = mn;
      }
    }
    if (meta.w != 1) return;
    if (meta.y == s0 && meta.z == ns) break;
    m = -INFINITY;
    l = 0.f;
    a = make_float4(0.f, 0.f, 0.f, 0.f);
    s0 = meta.y;
    ns = meta.z;
  }
  const int pair = meta.x;
  if (tid == 0) PAD_MSTAMP(3);
  // Fold the groups of one warp (lanes C4 apart hold the same columns) with
  // shuffles, then the warps' states through shared memory.
#pragma unroll
  for (int o = C4; o < 32; o <<= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), l2 = __shfl_xor_sync(0xffffffffu, l, o);
    float4 a2;
    a2.x = __shfl_xor_sync(0xffffffffu, a.x, o);
    a2.y = __shfl_xor_sync(0xffffffffu, a.y, o);
    a2.z = __shfl_xor_sync(0xffffffffu, a.z, o);
    a2.w = __shfl_xor_sync(0xffffffffu, a.w, o);
    const float mn = fmaxf(m, m2), mu = (mn == -INFINITY) ? 0.f : mn;
    const float al = ex2(m - mu), be = ex2(m2 - mu);
    l = l * al + l2 * be;
    a.x = a.x * al + a2.x * be;
    a.y = a.y * al + a2.y * be;
    a.z = a.z * al + a2.z * be;
    a.w = a.w * al + a2.w * be;
    m = mn;
  }
  const int wid = tid >> 5, lid = tid & 31;
  if (lid < C4) {
    *reinterpret_cast<float4*>(&red_o[wid][lid * 4]) = a;
    if (lid == 0) {
      red_m[wid] = m;
      red_l[wid] = l;
    }
  }
  __syncthreads();
  if (tid < C4) {
    float M = -INFINITY;
#pragma unroll
    for (int x = 0; x < NW; ++x) M = fmaxf(M, red_m[x]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
    float L = 0.f;
#pragma unroll
    for (int x = 0; x < NW; ++x) {
      const float wt = ex2(red_m[x] - Mu);  // 0 for warps that saw no partial
      const float4 v = *reinterpret_cast<const float4*>(&red_o[x][tid * 4]);
      t.x += v.x * wt;
      t.y += v.y * wt;
      t.z += v.z * wt;
      t.w += v.w * wt;
      L += red_l[x] * wt;
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const int b = pair / ngroups, hg = pair % ngroups;
    __half* o = out + b * out_sb + (int64_t)(hg * rows + y) * out_sh + blockIdx.z * DC + tid * 4;
    reinterpret_cast<__half2*>(o)[0] = __floats2half2_rn(t.x * inv, t.y * inv);
    reinterpret_cast<__half2*>(o)[1] = __floats2half2_rn(t.z * inv, t.w * inv);
    if (tid == 0) PAD_MSTAMP(2);
  }
}

}  // namespace pad
