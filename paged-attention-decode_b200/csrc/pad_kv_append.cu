// pad_kv_append.cu -- write one new token's K and V per sequence into the
// paged cache: the step that precedes decode attention. The reference fixes
// the layout it reads (k_cache/v_cache [num_pages, page_size, Hkv, D],
// block_table [B, max_pages], README.md:38-44) but ships no writer; this is
// the writer for that layout.
//
// Token t of sequence b lives at page block_table[b, t / page_size], row
// t % page_size. positions[b] is the index t of the new token (usually the
// sequence length before the step); positions[b] < 0 skips sequence b.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "pad_b200.h"
#include "pad_error.cuh"

namespace {

// One warp per (sequence, KV head) row; 16-byte vector copies when the row
// and both tensors allow it, 2-byte copies otherwise.
__global__ void kv_append_kernel(const __half* __restrict__ k_new, const __half* __restrict__ v_new,
                                 __half* __restrict__ k_cache, __half* __restrict__ v_cache,
                                 const int32_t* __restrict__ block_table, const int32_t* __restrict__ positions,
                                 int batch, int hkv, int d, int num_pages, int page_size, int max_pages,
                                 int64_t kn_sb, int64_t kn_sh, int64_t vn_sb, int64_t vn_sh, int64_t k_sp,
                                 int64_t k_sr, int64_t k_sh, int64_t v_sp, int64_t v_sr, int64_t v_sh,
                                 int64_t bt_stride, int vec, int32_t* error_flags) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= batch * hkv) return;
  const int b = row / hkv, h = row % hkv;
  const int pos = positions[b];
  if (pos < 0) return;
  const int lp = pos / page_size;
  if (lp >= max_pages) {
    if (lane == 0 && error_flags != nullptr) atomicOr(error_flags, PAD_FLAG_SEQ_LEN_RANGE);
    return;
  }
  const int page = block_table[(int64_t)b * bt_stride + lp];
  if ((unsigned)page >= (unsigned)num_pages) {
    if (lane == 0 && error_flags != nullptr) atomicOr(error_flags, PAD_FLAG_BAD_PAGE_ID);
    return;
  }
  const int r = pos % page_size;
  const __half* ks = k_new + b * kn_sb + h * kn_sh;
  const __half* vs = v_new + b * vn_sb + h * vn_sh;
  __half* kd = k_cache + (int64_t)page * k_sp + (int64_t)r * k_sr + (int64_t)h * k_sh;
  __half* vd = v_cache + (int64_t)page * v_sp + (int64_t)r * v_sr + (int64_t)h * v_sh;
  if (vec) {
    for (int i = lane; i < d / 8; i += 32) {
      reinterpret_cast<uint4*>(kd)[i] = __ldg(reinterpret_cast<const uint4*>(ks) + i);
      reinterpret_cast<uint4*>(vd)[i] = __ldg(reinterpret_cast<const uint4*>(vs) + i);
    }
  } else {
    for (int i = lane; i < d; i += 32) {
      kd[i] = ks[i];
      vd[i] = vs[i];
    }
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int pad_paged_kv_append(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                                   const int32_t* block_table, const int32_t* positions, int64_t batch,
                                   int64_t num_kv_heads, int64_t head_dim, int64_t num_pages, int64_t page_size,
                                   int64_t max_pages_per_seq, const int64_t* k_new_strides,
                                   const int64_t* v_new_strides, const int64_t* k_strides, const int64_t* v_strides,
                                   int64_t block_table_stride, void* stream, int32_t* error_flags) {
  using pad::fail;
  if (batch < 0 || num_kv_heads <= 0 || head_dim <= 0 || num_pages < 0 || page_size <= 0 || max_pages_per_seq < 0)
    return fail(PAD_ERR_INVALID_ARGUMENT, "kv_append: negative or zero size");
  if (batch == 0 || num_pages == 0 || max_pages_per_seq == 0) return PAD_OK;
  if (k_new == nullptr || v_new == nullptr || k_cache == nullptr || v_cache == nullptr || block_table == nullptr ||
      positions == nullptr || k_new_strides == nullptr || v_new_strides == nullptr || k_strides == nullptr ||
      v_strides == nullptr)
    return fail(PAD_ERR_INVALID_ARGUMENT, "kv_append: null pointer argument");
  if (block_table_stride < max_pages_per_seq)
    return fail(PAD_ERR_INVALID_ARGUMENT, "kv_append: block_table row stride smaller than its width");
  if (k_new_strides[2] != 1 || v_new_strides[2] != 1 || k_strides[3] != 1 || v_strides[3] != 1)
    return fail(PAD_ERR_UNSUPPORTED, "kv_append: the head_dim axis of every tensor must be contiguous");
  if (batch * num_kv_heads > INT32_MAX || num_pages > INT32_MAX)
    return fail(PAD_ERR_UNSUPPORTED, "kv_append: batch * num_kv_heads or num_pages exceeds int32");
  const bool vec = head_dim % 8 == 0 && al16(k_new) && al16(v_new) && al16(k_cache) && al16(v_cache) &&
                   k_new_strides[0] % 8 == 0 && k_new_strides[1] % 8 == 0 && v_new_strides[0] % 8 == 0 &&
                   v_new_strides[1] % 8 == 0 && k_strides[0] % 8 == 0 && k_strides[1] % 8 == 0 &&
                   k_strides[2] % 8 == 0 && v_strides[0] % 8 == 0 && v_strides[1] % 8 == 0 && v_strides[2] % 8 == 0;
  const int rows = (int)(batch * num_kv_heads);
  const int warps_per_block = 8;
  kv_append_kernel<<<(rows + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0,
                     static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(k_new), static_cast<const __half*>(v_new), static_cast<__half*>(k_cache),
      static_cast<__half*>(v_cache), block_table, positions, (int)batch, (int)num_kv_heads, (int)head_dim,
      (int)num_pages, (int)page_size, (int)max_pages_per_seq, k_new_strides[0], k_new_strides[1], v_new_strides[0],
      v_new_strides[1], k_strides[0], k_strides[1], k_strides[2], v_strides[0], v_strides[1], v_strides[2],
      block_table_stride, vec ? 1 : 0, error_flags);
  // the launch's own error only: cudaPeekAtLastError would also report (and
  // cudaGetLastError clear) a sticky error left by unrelated earlier work
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PAD_OK : pad::cuda_fail(e, "launching the kv_append kernel");
}
