// pad_decode_kernel.cuh -- sm_100a paged-attention decode kernels.
//
// Phase 1 (`decode_stream_kernel`): a persistent, stream-K balanced kernel.
//   The batch is flattened into one list of 64-token tiles ordered
//   (sequence, KV head, tile); every CTA takes an equal contiguous range of
//   that list, so work is balanced to within one tile whatever the mix of
//   sequence lengths. Inside a CTA one producer warp walks its range and
//   gathers each tile's K/V pages from the paged cache with TMA tensor loads
//   (block_table gives the page, the tensor map does the addressing) into a
//   STAGES-deep shared-memory ring guarded by mbarriers; four consumer warps
//   each take 16 tokens of a tile and run all GQA query rows of the KV head
//   together on m16n8k16 tensor-core tiles (S^T = K.Q^T, then O^T += V^T.P^T),
//   with an fp32 online softmax in base 2. When a (sequence, KV head) pair
//   lies entirely inside one CTA's range the CTA writes the fp16 output row
//   directly; otherwise it writes an fp32 partial (O, m, l) -- the split-K
//   partials of the reference's phase 1 (cuda/kernel_v4_split_k.cu:48-150,
//   analysis/split_k_derivation.md:16-35).
// Phase 2 (`merge_kernel`): for the pairs that were split across CTAs, a
//   log-sum-exp merge of the partials (analysis/split_k_derivation.md:44-86),
//   parallel over (pair, query row) and over the partials themselves.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "pad_ptx.cuh"

namespace pad {

constexpr int kTile = 64;           // tokens per pipeline tile
constexpr int kConsumerWarps = 4;   // each owns 16 tokens of a tile
constexpr int kThreads = 32 * (kConsumerWarps + 1);
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s: no legitimate wait comes close
constexpr float kLog2e = 1.4426950408889634f;

struct __align__(64) DecodeParams {
  CUtensorMap tm_k;  // [D, Hkv, page_size, num_pages] fp16, box {SEG, 1, R, 1}
  CUtensorMap tm_v;
  CUtensorMap tm_q;  // [D, Hq, B] fp16, box {SEG, G, 1}
  const int32_t* block_table;
  const int32_t* seq_lens;
  __half* out;
  float* ws_o;      // [slots][G][D] fp32 unnormalised partial outputs
  float2* ws_ml;    // [slots][G] (m, l), m in log2 units
  int4* ws_meta;    // [partitions] merge descriptors {pair, first slot, n slots, valid}
  int32_t* error_flags;
  int64_t bt_stride;
  int64_t out_sb, out_sh;
  int batch, hkv, gqa, page_size, num_pages, max_pages;
  int box_rows;      // R: tokens per TMA box (divides page_size and kTile)
  float scale_log2;  // scale * log2(e)
};

// Compile-time shape of one kernel instance.
template <int D_, int NT_, bool SWZ_, int STAGES_>
struct Traits {
  static constexpr int D = D_;
  static constexpr int NT = NT_;            // n8 tiles of query rows: G <= 8*NT
  static constexpr bool SWZ = SWZ_;         // 128/64/32-byte TMA swizzle (needs R >= 8)
  static constexpr int STAGES = STAGES_;
  static constexpr int QROWS = 8 * NT;
  static constexpr int ROW_BYTES = D * 2;
  static constexpr int SEGW = SWZ ? (ROW_BYTES < 128 ? ROW_BYTES : 128) : ROW_BYTES;  // bytes per row segment
  static constexpr int NSEG = ROW_BYTES / SEGW;
  static constexpr int CPS = SEGW / 16;     // 16-byte chunks per row segment
  // Unswizzled tiles place each TMA box (R rows) at a multiple of 128 bytes
  // (the alignment a tensor copy's shared destination needs), so rows of
  // fewer than 128 bytes with R * ROW_BYTES < 128 leave gaps between boxes.
  static constexpr int KT_BYTES = kTile * (SWZ ? ROW_BYTES : (ROW_BYTES < 128 ? 128 : ROW_BYTES));
  static constexpr int Q_BYTES = QROWS * ROW_BYTES;
  static constexpr int STAGE_BYTES = ((2 * KT_BYTES + Q_BYTES) + 1023) / 1024 * 1024;
  static constexpr int NB_MAX = SWZ ? kTile / 8 : kTile;  // TMA boxes per tile (R >= 8 when swizzled)
  static constexpr int EPI_BYTES = 2 * QROWS * D * 4;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + EPI_BYTES + 4096 /*misc*/;

  // XOR applied to the 16-byte chunk index of a row by the TMA swizzle mode
  // (the chunk bits [4,4+b) of the shared address are XOR-ed with bits [7,7+b)).
  __device__ static __forceinline__ uint32_t swz(uint32_t row) {
    if constexpr (!SWZ) return 0u;
    else if constexpr (SEGW == 128) return row & 7u;
    else if constexpr (SEGW == 64) return (row >> 1) & 3u;
    else return (row >> 2) & 1u;
  }
  // Bytes between consecutive TMA boxes of R rows in a K/V tile.
  __device__ static __forceinline__ uint32_t box_pitch(int R) {
    if constexpr (SWZ) return (uint32_t)(R * SEGW);
    else return (uint32_t)(R * ROW_BYTES < 128 ? 128 : R * ROW_BYTES);
  }
  // Shared address of 16-byte chunk `c` (0 .. D/8-1) of token row `row` of a
  // K/V tile stored from `base` (segment-major when swizzled; box-pitched
  // when not). R = rows per TMA box.
  __device__ static __forceinline__ uint32_t kv_addr(uint32_t base, uint32_t row, uint32_t c, int R) {
    if constexpr (SWZ) {
      const uint32_t seg = c / CPS, cs = c % CPS;
      return base + seg * (uint32_t)(kTile * SEGW) + row * SEGW + ((cs ^ swz(row)) << 4);
    } else {
      return base + (row / R) * box_pitch(R) + (row % R) * ROW_BYTES + (c << 4);
    }
  }
  // Same for the query tile (one box of QROWS rows).
  __device__ static __forceinline__ uint32_t q_addr(uint32_t base, uint32_t row, uint32_t c) {
    const uint32_t seg = c / CPS, cs = c % CPS;
    return base + seg * (uint32_t)(QROWS * SEGW) + row * SEGW + ((cs ^ swz(row)) << 4);
  }
};

// Shared-memory bookkeeping beside the stage ring.
struct TileDesc {
  int b, h, i, seq;   // sequence, KV head, tile index within the pair, clamped seq_len
  int flags;          // kFirst | kLast | kSplit
  int slot;           // partial slot when split
  int pad0, pad1;
};
constexpr int kFirst = 1, kLast = 2, kSplit = 4;

struct Cursor {
  int b, h, i, n, seq;  // n = tiles of sequence b
  int pair_start;       // global index of tile 0 of pair (b, h)
};

__device__ __forceinline__ int clamp_seq(int raw, int cap) { return raw < 0 ? 0 : (raw > cap ? cap : raw); }
__device__ __forceinline__ int tiles_of(int seq) { return (seq + kTile - 1) / kTile; }

// Partition w of W covers global tiles [begin(w), begin(w+1)).
__device__ __forceinline__ int part_begin(int64_t w, int64_t total, int64_t parts) {
  return (int)((w * total) / parts);
}
// The partition owning global tile t: the largest w with begin(w) <= t.
__device__ __forceinline__ int part_owner(int64_t t, int64_t total, int64_t parts) {
  return (int)(((t + 1) * parts - 1) / total);
}

// Step a cursor to the next tile of the flattened (sequence, head, tile) list.
__device__ __forceinline__ void cursor_next(Cursor& c, const DecodeParams& p, int cap) {
  if (++c.i < c.n) return;
  c.i = 0;
  c.pair_start += c.n;
  if (++c.h < p.hkv) return;
  c.h = 0;
  do {
    if (++c.b >= p.batch) {
      c.n = 0;
      return;
    }
    c.seq = clamp_seq(__ldg(p.seq_lens + c.b), cap);
    c.n = tiles_of(c.seq);
  } while (c.n == 0);
}

}  // namespace pad
