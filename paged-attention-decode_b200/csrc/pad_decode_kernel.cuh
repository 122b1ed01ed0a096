// pad_decode_kernel.cuh -- shared definitions of the sm_100a paged-attention
// decode kernels (pad_decode_kernels.cuh holds the kernels themselves).
//
// Phase 1 (`decode_stream_kernel`): a persistent, stream-K balanced kernel.
//   Work unit: a tile of 128 (token, KV head) rows -- TT tokens of a group of
//   HG KV heads of one sequence (HG = 8, 4, 2 or 1 heads, TT = 128 / HG). The
//   batch is flattened into one list of tiles ordered (sequence, head group,
//   tile) and every CTA takes an equal contiguous range of that list, so work
//   is balanced to within one tile whatever the mix of sequence lengths.
//   One producer warp gathers each tile's K/V rows from the paged cache with
//   TMA tensor loads (block_table names the page; one box spans all HG heads
//   of R consecutive tokens, i.e. whole contiguous cache rows) into a
//   STAGES-deep shared-memory ring guarded by mbarriers. Eight consumer
//   warps each own 16 tokens of one head of the tile and run all GQA query
//   rows of that head together on m16n8k16 tensor-core tiles
//   (S^T = K.Q^T, then O^T += V^T.P^T) with an fp32 online softmax in base 2.
//   A (sequence, head group) pair that lies entirely inside one CTA's range is
//   finished there (fp16 output); otherwise the CTA writes an fp32 partial
//   (O, m, l) per head -- the split-K partials of the reference's phase 1
//   (cuda/kernel_v4_split_k.cu:48-150, analysis/split_k_derivation.md:16-35).
// Phase 2 (`merge_kernel`): for pairs split across CTAs, a log-sum-exp merge
//   of the partials (analysis/split_k_derivation.md:44-86), parallel over
//   (pair, head, query row) and over the partials themselves.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "pad_ptx.cuh"

namespace pad {

constexpr int kTileRows = 128;      // (token, head) rows per tile
constexpr int kConsumerWarps = 8;   // each owns 16 tokens of one head
constexpr int kThreads = 32 * (kConsumerWarps + 1);
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s: no legitimate wait comes close
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kSmemBudget = 227 * 1024;
constexpr int kSeqCache = 1024;   // seq_lens kept in shared memory when batch <= this
constexpr int kFastBatch = 256;   // largest batch the producer's fast start checks (8 loads per lane)

struct __align__(64) DecodeParams {
  CUtensorMap tm_k;  // dims {D, page_size, Hkv, num_pages}, box {SEG, R, HG, 1}
  CUtensorMap tm_v;
  CUtensorMap tm_q;  // dims {D, Hq, B}, box {SEG, HG*G, 1}
  const int32_t* block_table;
  const int32_t* seq_lens;
  __half* out;
  float* ws_o;      // [slots][HG][G][D] fp32 unnormalised partial outputs
  float2* ws_ml;    // [slots][HG][G] (m, l), m in log2 units
  int4* ws_meta;    // [partitions] merge descriptors {pair, first slot, n slots, valid}
  int32_t* error_flags;
  int64_t bt_stride;
  // CSR page index (FlashInfer layout): when csr_indptr is set, sequence b's
  // pages are block_table[csr_indptr[b] .. csr_indptr[b+1]) (block_table is the
  // flat `indices` array) and seq_len = (pages - 1) * page_size + csr_last[b].
  const int32_t* csr_indptr;
  const int32_t* csr_last;
  int64_t out_sb, out_sh;
  int batch, hkv, gqa, page_size, num_pages, max_pages;
  int box_rows;      // R: tokens per TMA box (a power of two dividing page_size and TT)
  int box_rows_log2; // log2(R)
  int page_shift;    // log2(page_size) when it is a power of two, else -1
  int meta_by_pair;  // merge descriptors indexed by pair (else by partition)
  int l2_warm;       // guessed first tiles prefetched into L2 before the dependency wait (0: none)
  float scale_log2;  // scale * log2(e)
};

// Compile-time shape of one kernel instance.
template <int D_, int NT_, int HG_, bool SWZ_>
struct Traits {
  static constexpr int D = D_;
  static constexpr int NT = NT_;            // n8 tiles of query rows: G <= 8*NT
  static constexpr int HG = HG_;            // KV heads per tile
  static constexpr bool SWZ = SWZ_;         // 128/64/32-byte TMA swizzle (needs R >= 8)
  static constexpr int WPH = kConsumerWarps / HG;  // consumer warps per head
  static constexpr int TT = 16 * WPH;       // tokens per tile
  static constexpr int KSTEPS = D / 16;
  static constexpr int ROW_BYTES = D * 2;
  static constexpr int SEGW = SWZ ? (ROW_BYTES < 128 ? ROW_BYTES : 128) : ROW_BYTES;  // bytes per row segment
  static constexpr int NSEG = ROW_BYTES / SEGW;
  static constexpr int CPS = SEGW / 16;     // 16-byte chunks per row segment
  // Unswizzled tiles place each TMA box (HG*R rows) at a multiple of 128
  // bytes, the alignment a tensor copy's shared destination needs.
  static constexpr int KT_BYTES = SWZ ? kTileRows * ROW_BYTES
                                      : TT * (HG * ROW_BYTES < 128 ? 128 : HG * ROW_BYTES);
  static constexpr int STAGE_BYTES = (2 * KT_BYTES + 1023) / 1024 * 1024;
  static constexpr int QROWS = HG * 8 * NT;  // query rows held (heads' rows packed, tail zero)
  static constexpr int Q_BYTES = (QROWS * ROW_BYTES + 1023) / 1024 * 1024;
  static constexpr int NB_MAX = SWZ ? TT / 8 : TT;  // TMA boxes per tile
  static constexpr int NB_PER_LANE = (NB_MAX + 31) / 32;
  // Cross-warp merge buffer (only when several warps share a head).
  // Two buffers (a two-level add tree) when 4 or more warps share a head.
  static constexpr int EPI_BUFS = WPH >= 4 ? 2 : 1;
  // Rows padded to D + 4 floats: the accumulator fragments' stores (lanes
  // spread over 4 rows x 8 columns) then hit 32 distinct banks.
  static constexpr int EPI_LD = D + 4;
  static constexpr int EPI_BYTES = WPH > 1 ? EPI_BUFS * HG * 8 * NT * EPI_LD * 4 : 0;
  static constexpr int MISC_BYTES = 4096 + kSeqCache * 4;  // + cached seq_lens
  // Query tiles in flight: two (one segment ahead) unless that costs a stage.
  static constexpr int QSLOTS = (kSmemBudget - (1024 + 2 * Q_BYTES + EPI_BYTES + MISC_BYTES)) / STAGE_BYTES >= 3 ? 2 : 1;
  static constexpr int FIXED_BYTES = 1024 /*align slack*/ + QSLOTS * Q_BYTES + EPI_BYTES + MISC_BYTES;
  static constexpr int STAGES_FIT = (kSmemBudget - FIXED_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 4 ? 4 : STAGES_FIT;
  static_assert(STAGES >= 2, "tile ring does not fit in shared memory");
  static constexpr int SMEM_BYTES = FIXED_BYTES + STAGES * STAGE_BYTES;

  // XOR applied to the 16-byte chunk index of a row by the TMA swizzle mode
  // (chunk bits [4,4+b) of the shared address XOR-ed with bits [7,7+b)).
  __device__ static __forceinline__ uint32_t swz(uint32_t row) {
    if constexpr (!SWZ) return 0u;
    else if constexpr (SEGW == 128) return row & 7u;
    else if constexpr (SEGW == 64) return (row >> 1) & 3u;
    else return (row >> 2) & 1u;
  }
  // Bytes between consecutive TMA boxes (HG heads x R tokens) of a tile segment.
  __device__ static __forceinline__ uint32_t box_pitch(int R) {
    if constexpr (SWZ) return (uint32_t)(HG * R * SEGW);
    else return (uint32_t)(HG * R * ROW_BYTES < 128 ? 128 : HG * R * ROW_BYTES);
  }
  // Where token `t` (0 .. TT-1) of local head `hl` lives in a K/V tile: a
  // box j holds tokens [j*R, j*R + R) of all HG heads, head-major ([hl][r]).
  // Returns the row's byte offset and its swizzle XOR; lr = log2(R).
  __device__ static __forceinline__ void kv_row(uint32_t t, uint32_t hl, int lr, uint32_t& rowoff, uint32_t& sw) {
    const uint32_t R = 1u << lr, j = t >> lr, r = t & (R - 1u);
    if constexpr (SWZ) {
      const uint32_t idx = (j * HG + hl) * R + r;
      rowoff = idx * SEGW;
      sw = swz(idx);
    } else {
      rowoff = j * box_pitch((int)R) + (hl * R + r) * ROW_BYTES;
      sw = 0u;
    }
  }
  // Shared address of 16-byte chunk `c` (0 .. D/8-1) of a row found by kv_row.
  __device__ static __forceinline__ uint32_t kv_at(uint32_t base, uint32_t rowoff, uint32_t sw, uint32_t c) {
    if constexpr (SWZ) {
      return base + (c / CPS) * (uint32_t)(kTileRows * SEGW) + rowoff + (((c % CPS) ^ sw) << 4);
    } else {
      return base + rowoff + (c << 4);
    }
  }
  __device__ static __forceinline__ uint32_t kv_addr(uint32_t base, uint32_t t, uint32_t hl, uint32_t c, int lr) {
    uint32_t rowoff, sw;
    kv_row(t, hl, lr, rowoff, sw);
    return kv_at(base, rowoff, sw, c);
  }
  // Query tile: HG*G rows packed (head hl at rows hl*G ..), segment-major.
  __device__ static __forceinline__ uint32_t q_addr(uint32_t base, uint32_t row, uint32_t c) {
    const uint32_t seg = c / CPS, cs = c % CPS;
    return base + seg * (uint32_t)(QROWS * SEGW) + row * SEGW + ((cs ^ swz(row)) << 4);
  }
};

// Shared-memory bookkeeping beside the stage ring.
struct TileDesc {
  int b, hg, i, seq;  // sequence, head group, tile index within the pair, clamped seq_len
  int flags;          // kFirst | kLast | kSplit
  int slot;           // partial slot when split
  int qslot;          // query-tile ring slot of this segment
  int pad;
};
constexpr int kFirst = 1, kLast = 2, kSplit = 4;

struct Cursor {
  int b, hg, i, n, seq;  // n = tiles of sequence b
  int pair_start;        // global index of tile 0 of pair (b, hg)
  int64_t base;          // offset of sequence b's row in the page index
};

__device__ __forceinline__ int clamp_seq(int raw, int cap) { return raw < 0 ? 0 : (raw > cap ? cap : raw); }

// Partition w of W covers global tiles [begin(w), begin(w+1)).
// floor(a / b) for 0 <= a < 2^52 and 0 < b < 2^31: a double-precision
// quotient corrected to the exact integer result (a 64-bit integer division
// would inline a long instruction sequence at every use).
__device__ __forceinline__ int64_t div_floor(int64_t a, int64_t b) {
  int64_t q = (int64_t)((double)a / (double)b);
  if (q * b > a) --q;
  else if ((q + 1) * b <= a) ++q;
  return q;
}

__device__ __forceinline__ int part_begin(int64_t w, int64_t total, int64_t parts) {
  return (int)div_floor(w * total, parts);
}
// The partition owning global tile t: the largest w with begin(w) <= t.
__device__ __forceinline__ int part_owner(int64_t t, int64_t total, int64_t parts) {
  return (int)div_floor((t + 1) * parts - 1, total);
}

}  // namespace pad
