/*
 * pad_b200.h -- C ABI of the B200 (sm_100a) paged-attention decode library
 * (libpad_b200.so).
 *
 * Every entry point takes plain pointers, sizes and strides (in ELEMENTS),
 * never framework types, and returns a pad_status code. Pointers to tensors
 * are device pointers on the device that is current when the call is made.
 * Calls are asynchronous on the given CUDA stream (a cudaStream_t passed as
 * void*; NULL means the legacy default stream) and never synchronise the
 * device.
 *
 * The decode entry point replaces, as one C call, the reference project's
 * pybind binding ``forward_v4(q, k_cache, v_cache, block_table, seq_lens,
 * scale, gqa_ratio, head_dim, page_size, num_splits)`` (cuda/binding.cpp:13-14,
 * declared at cuda/kernels.h:60-70) and the launcher behind it
 * (cuda/kernel_v4_split_k.cu:205-268). Differences, by design:
 *   - the caller owns `out` and a reusable `workspace` (the reference
 *     allocated both with torch on every call, cuda/kernel_v4_split_k.cu:228-232);
 *   - the stream is explicit (the reference launched on the legacy default
 *     stream, cuda/kernel_v4_split_k.cu:238,257);
 *   - argument errors come back as status codes instead of TORCH_CHECK
 *     exceptions (cuda/kernel_v4_split_k.cu:216-223).
 *
 * Tensor layouts (the reference's, README.md:38-44):
 *   q, out       [batch, num_q_heads, head_dim]            fp16
 *   k/v_cache    [num_pages, page_size, num_kv_heads, head_dim] fp16
 *   block_table  [batch, max_pages_per_seq]                int32
 *   seq_lens     [batch]                                   int32
 * The last dimension of q, out, k_cache and v_cache must be contiguous
 * (stride 1); the other strides of q/k_cache/v_cache must be multiples of
 * 8 elements (16 bytes, a TMA requirement) and the base pointers 16-byte
 * aligned. block_table's inner stride must be 1.
 */
#ifndef PAD_B200_H_
#define PAD_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum pad_status {
  PAD_OK = 0,
  PAD_ERR_INVALID_ARGUMENT = 1, /* a shape, size or pointer is invalid      */
  PAD_ERR_UNSUPPORTED = 2,      /* valid but outside what the kernels cover */
  PAD_ERR_WORKSPACE = 3,        /* workspace missing or too small           */
  PAD_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed        */
} pad_status;

/* Bits OR-ed into *error_flags by the kernels (value checks the reference's
 * oracle performs on the host, src/reference.py:40-41,107-112, done here on
 * the device without a host sync). */
#define PAD_FLAG_BAD_PAGE_ID 0x1     /* a block_table entry outside [0, num_pages) */
#define PAD_FLAG_SEQ_LEN_RANGE 0x2   /* seq_len < 0 or > max_pages_per_seq * page_size */
#define PAD_FLAG_WAIT_TIMEOUT 0x100  /* an in-kernel wait gave up (never expected) */

/* Human-readable text for a status code (static storage). */
const char* pad_status_string(int status);

/* Text of the last error on the calling thread (static thread-local storage). */
const char* pad_last_error(void);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int pad_version(void);

/* Number of SMs of `device` and how many decode CTAs one SM holds for the
 * given head_dim / gqa_ratio (the inputs of the split heuristic). */
int pad_device_info(int device, int64_t head_dim, int64_t gqa_ratio, int* num_sms, int* ctas_per_sm);

/* Number of persistent decode CTAs (work partitions) the decode call will
 * launch for this problem on `device`.
 *   num_splits <= 0 : heuristic -- one partition per resident CTA slot
 *                     (num_sms * ctas_per_sm), capped by the number of
 *                     tiles the batch can hold (a tile is 128 (token,
 *                     KV head) rows: 128 / HG tokens of HG KV heads, HG the
 *                     largest of 8, 4, 2, 1 dividing num_kv_heads, at most
 *                     4 when gqa_ratio > 8);
 *   num_splits >= 1 : num_splits partitions per (sequence, KV head) pair,
 *                     i.e. num_splits * batch * num_kv_heads partitions. */
int pad_decode_partitions(int device, int64_t batch, int64_t num_kv_heads, int64_t gqa_ratio,
                          int64_t head_dim, int64_t page_size, int64_t max_pages_per_seq,
                          int64_t num_splits, int64_t* partitions);

/* Bytes of device workspace pad_paged_attention_decode needs for this
 * problem (same arguments as pad_decode_partitions). The workspace holds the
 * fp32 split partials (O, m, l) and per-partition merge descriptors; it
 * needs no initialisation and may be reused by consecutive calls on one
 * stream (calls that overlap in time must use distinct workspaces). */
int pad_decode_workspace_bytes(int device, int64_t batch, int64_t num_kv_heads, int64_t gqa_ratio,
                               int64_t head_dim, int64_t page_size, int64_t max_pages_per_seq,
                               int64_t num_splits, size_t* bytes);

/* Decode attention over a paged fp16 KV cache with GQA.
 *
 *   out[b, h, :] = softmax(scale * q[b, h, :] . K_b[h / G]^T) @ V_b[h / G]
 *
 * where K_b/V_b are the first seq_lens[b] token rows of the pages
 * block_table[b, 0 .. ceil(seq_lens[b] / page_size) - 1] and
 * G = num_q_heads / num_kv_heads. A sequence with seq_len == 0 yields a zero
 * row (src/reference.py:32-34). Entries of block_table past a sequence's
 * last page are never read.
 *
 * Strides are in elements: q_strides[3], k_strides[4], v_strides[4],
 * out_strides[3]; block_table_stride is the row stride of block_table.
 * error_flags (device int32, optional) receives PAD_FLAG_* bits; it is
 * OR-ed into, never cleared.
 *
 * Invalid values are flagged, never faulted on: a block_table entry outside
 * [0, num_pages) sets PAD_FLAG_BAD_PAGE_ID and the tokens it addresses are
 * read as zero K/V rows (the tensor copy zero-fills out-of-range boxes); a
 * seq_len outside [0, max_pages_per_seq * page_size] sets
 * PAD_FLAG_SEQ_LEN_RANGE and is clamped into that range. When either flag is
 * set the output of the call is undefined (the reference oracle raises
 * ValueError instead, src/reference.py:40-41,107-112).
 *
 * The library caches per-device facts (kernel attributes, occupancy, the
 * no-alloc scratch address) for the life of the process; it must not be used
 * across a cudaDeviceReset of a device it has run on.
 */
int pad_paged_attention_decode(const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* block_table, const int32_t* seq_lens, void* out,
                               int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                               int64_t head_dim, int64_t num_pages, int64_t page_size,
                               int64_t max_pages_per_seq, const int64_t* q_strides,
                               const int64_t* k_strides, const int64_t* v_strides,
                               int64_t block_table_stride, const int64_t* out_strides, float scale,
                               int64_t num_splits, void* workspace, size_t workspace_bytes,
                               void* stream, int32_t* error_flags);

/* Decode with a CSR page index instead of a dense block table -- the
 * (indptr, indices, last_page_len) layout the reference's FlashInfer adapter
 * builds from a block table (src/flashinfer_adapter.py:40-65):
 *   pages of sequence b = kv_indices[kv_indptr[b] .. kv_indptr[b+1])
 *   seq_len of b        = (pages - 1) * page_size + kv_last_page_len[b]
 *                         (0 when the sequence has no pages)
 * nnz_pages is the length of kv_indices. Everything else -- strides, scale,
 * num_splits, workspace (sized by pad_decode_csr_workspace_bytes), stream,
 * error flags -- is as for pad_paged_attention_decode. */
int pad_decode_csr_workspace_bytes(int device, int64_t batch, int64_t num_kv_heads, int64_t gqa_ratio,
                                   int64_t head_dim, int64_t page_size, int64_t nnz_pages,
                                   int64_t num_splits, size_t* bytes);
int pad_paged_attention_decode_csr(const void* q, const void* k_cache, const void* v_cache,
                                   const int32_t* kv_indptr, const int32_t* kv_indices,
                                   const int32_t* kv_last_page_len, void* out, int64_t batch,
                                   int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                   int64_t num_pages, int64_t page_size, int64_t nnz_pages,
                                   const int64_t* q_strides, const int64_t* k_strides,
                                   const int64_t* v_strides, const int64_t* out_strides, float scale,
                                   int64_t num_splits, void* workspace, size_t workspace_bytes,
                                   void* stream, int32_t* error_flags);

/* Write one new token's K and V per sequence into the paged cache (the step
 * before decode; the reference fixes this cache layout, README.md:38-44, but
 * has no writer). Token positions[b] of sequence b goes to page
 * block_table[b, positions[b] / page_size], row positions[b] % page_size,
 * for every KV head; positions[b] < 0 skips sequence b.
 * k_new / v_new are [batch, num_kv_heads, head_dim] fp16 with strides
 * k_new_strides[3] / v_new_strides[3]; caches as for decode. A position past
 * the block table sets PAD_FLAG_SEQ_LEN_RANGE, a bad page id
 * PAD_FLAG_BAD_PAGE_ID (nothing is written for that row). */
int pad_paged_kv_append(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                        const int32_t* block_table, const int32_t* positions, int64_t batch,
                        int64_t num_kv_heads, int64_t head_dim, int64_t num_pages, int64_t page_size,
                        int64_t max_pages_per_seq, const int64_t* k_new_strides,
                        const int64_t* v_new_strides, const int64_t* k_strides, const int64_t* v_strides,
                        int64_t block_table_stride, void* stream, int32_t* error_flags);

/* Decode without any device allocation, for callers that cannot call
 * cudaMalloc: code running inside a CUDA stream capture they do not own,
 * embedders whose memory is owned by a custom allocator or a fixed arena,
 * and real-time paths where an allocation could block. It behaves exactly
 * like pad_paged_attention_decode (same arguments minus the workspace) but
 * keeps the split partials in a scratch array built into the library,
 * PAD_STATIC_SCRATCH_BYTES (16 MiB) per GPU, which every GPU that loads the
 * library holds until the process exits. Problems whose workspace
 * (pad_decode_workspace_bytes) exceeds that size are rejected with
 * PAD_ERR_WORKSPACE. The first call on a device looks up the scratch
 * array's device address (cudaGetSymbolAddress) with that device current,
 * so make that first call before any stream capture. All calls on a device
 * share the one array: calls that overlap on the GPU (different streams, no
 * ordering between them) race and must be avoided. Nothing in the array has
 * to start zeroed; each call rewrites what it reads.
 * No counterpart in the reference. */
#define PAD_STATIC_SCRATCH_BYTES ((size_t)16 << 20)
int pad_paged_attention_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                       const int32_t* block_table, const int32_t* seq_lens, void* out,
                                       int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                                       int64_t head_dim, int64_t num_pages, int64_t page_size,
                                       int64_t max_pages_per_seq, const int64_t* q_strides,
                                       const int64_t* k_strides, const int64_t* v_strides,
                                       int64_t block_table_stride, const int64_t* out_strides,
                                       float scale, int64_t num_splits, void* stream,
                                       int32_t* error_flags);

#ifdef __cplusplus
}
#endif

#endif /* PAD_B200_H_ */
