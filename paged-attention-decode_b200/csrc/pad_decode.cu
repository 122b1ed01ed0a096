// pad_decode.cu -- host side of libpad_b200.so: argument checks, TMA tensor
// map encoding, kernel-instance dispatch and the extern "C" entry points
// declared in include/pad_b200.h.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <map>
#include <cstring>
#include <mutex>
#include <string>

#include "pad_b200.h"
#include "pad_decode_kernels.cuh"
#include "pad_error.cuh"

namespace {

using namespace pad;

// ----------------------------------------------------------------- instances
struct Instance {
  const void* kernel;          // decode_stream_kernel<TR>
  const void* merge_small;     // merge_kernel<D, 128>: few partials per split pair
  const void* merge_mid;       // merge_kernel<D, 256, D/32, 4>: a handful of partials, D split over CTAs
  const void* merge_large;     // merge_kernel<D, 256, D/32, 8>: many partials (long context)
  int merge_dsplit;
  int smem_bytes;
  int segw;                    // bytes per row segment (TMA box inner extent)
  bool swz;
  int hg;                      // KV heads per tile
  int tt;                      // tokens per tile
};

// Columns of D one wide-merge CTA folds (the merge grid splits D by it).
#ifndef PAD_MERGE_COLS
#define PAD_MERGE_COLS 32
#endif
constexpr int kMergeCols = PAD_MERGE_COLS;

template <int D, int NT, int HG, bool SWZ>
Instance make_instance() {
  using TR = Traits<D, NT, HG, SWZ>;
  Instance in;
  in.kernel = reinterpret_cast<const void*>(&decode_stream_kernel<TR>);
  in.merge_small = reinterpret_cast<const void*>(&merge_kernel<D, 128, 1, 4>);
  in.merge_mid = reinterpret_cast<const void*>(&merge_kernel<D, 256, (D >= 2 * kMergeCols ? D / kMergeCols : 1), 4>);
  in.merge_large = reinterpret_cast<const void*>(&merge_kernel<D, 256, (D >= 2 * kMergeCols ? D / kMergeCols : 1), 8>);
  in.merge_dsplit = D >= 2 * kMergeCols ? D / kMergeCols : 1;
  in.smem_bytes = TR::SMEM_BYTES;
  in.segw = TR::SEGW;
  in.swz = SWZ;
  in.hg = HG;
  in.tt = TR::TT;
  return in;
}

template <int D, int NT, int HG>
Instance pick_swz(bool swz) {
  return swz ? make_instance<D, NT, HG, true>() : make_instance<D, NT, HG, false>();
}

template <int D, int NT>
Instance pick_hg(int hg, bool swz) {
  switch (hg) {
    case 8:
      if constexpr (NT == 1) return pick_swz<D, NT, 8>(swz);
      else return pick_swz<D, NT, 4>(swz);  // not reached: G > 8 caps the head group at 4
    case 4: return pick_swz<D, NT, 4>(swz);
    case 2: return pick_swz<D, NT, 2>(swz);
    default: return pick_swz<D, NT, 1>(swz);
  }
}

// KV heads per tile: the largest of 8, 4, 2, 1 dividing num_kv_heads (at
// most 4 when a head has more than 8 query rows, to fit shared memory).
int head_group_for(int64_t hkv, int64_t gqa) {
  const int cap = gqa <= 8 ? 8 : 4;
  for (int hg = cap; hg > 1; hg /= 2)
    if (hkv % hg == 0) return hg;
  return 1;
}

// Merge variant by partials per split pair (partitions / pairs): up to
// kMergeWide the 128-thread kernel (one CTA per query row); above it D is
// split over CTAs, and above kMergeDeep each thread keeps 8 loads in flight.
#ifndef PAD_MERGE_WIDE
#define PAD_MERGE_WIDE 16
#endif
#ifndef PAD_MERGE_DEEP
#define PAD_MERGE_DEEP 32
#endif
constexpr int64_t kMergeWide = PAD_MERGE_WIDE, kMergeDeep = PAD_MERGE_DEEP;
constexpr int64_t kFewPairs = 16;  // the num_splits=None heuristic: see make_plan

bool pick_instance(int64_t head_dim, int64_t gqa, int hg, bool swz, Instance* out) {
  const bool nt1 = gqa <= 8;
  switch (head_dim) {
    case 16: *out = nt1 ? pick_hg<16, 1>(hg, swz) : pick_hg<16, 2>(hg, swz); return true;
    case 32: *out = nt1 ? pick_hg<32, 1>(hg, swz) : pick_hg<32, 2>(hg, swz); return true;
    case 64: *out = nt1 ? pick_hg<64, 1>(hg, swz) : pick_hg<64, 2>(hg, swz); return true;
    case 128: *out = nt1 ? pick_hg<128, 1>(hg, swz) : pick_hg<128, 2>(hg, swz); return true;
    default: return false;
  }
}

// Largest power of two that divides page_size, capped at the tile's token
// count: the token rows of one TMA box. Boxes never straddle a page or a tile.
int box_rows_for(int64_t page_size, int tt) {
  int r = 1;
  while (r < tt && page_size % (2 * r) == 0) r *= 2;
  return r;
}

// Per-device, per-instance cached facts: opt-in shared memory set, occupancy.
constexpr int kMaxDevices = 64;
constexpr int kNumInstanceKeys = 4 * 2 * 4 * 2;
struct DeviceCache {
  int num_sms = 0;
  int occ[kNumInstanceKeys] = {};
  bool smem_set[kNumInstanceKeys] = {};
};
DeviceCache g_dev[kMaxDevices];
std::mutex g_mu;

int instance_key(int64_t head_dim, int64_t gqa, int hg, bool swz) {
  const int di = head_dim == 16 ? 0 : head_dim == 32 ? 1 : head_dim == 64 ? 2 : 3;
  const int hi = hg == 1 ? 0 : hg == 2 ? 1 : hg == 4 ? 2 : 3;
  return ((di * 2 + (gqa <= 8 ? 0 : 1)) * 4 + hi) * 2 + (swz ? 1 : 0);
}

int prepare_device(int device, const Instance& in, int key, int* num_sms, int* occ) {
  if (device < 0 || device >= kMaxDevices) return fail(PAD_ERR_INVALID_ARGUMENT, "device %d out of range", device);
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceCache& dc = g_dev[device];
  if (dc.num_sms == 0) {
    int n = 0;
    cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    dc.num_sms = n;
  }
  if (!dc.smem_set[key]) {
    int cur = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (cur != device && (e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    e = cudaFuncSetAttribute(in.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, in.smem_bytes);
    int o = 0;
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, in.kernel, kThreads, in.smem_bytes);
    if (cur != device) cudaSetDevice(cur);
    if (e != cudaSuccess) return cuda_fail(e, "configuring the decode kernel");
    if (o < 1) return fail(PAD_ERR_UNSUPPORTED, "decode kernel does not fit on an SM (%d B smem)", in.smem_bytes);
    dc.occ[key] = o;
    dc.smem_set[key] = true;
  }
  *num_sms = dc.num_sms;
  *occ = dc.occ[key];
  return PAD_OK;
}

// Integer tuning knob from the environment, read once per name.
int env_int(const char* name, int dflt) {
  static std::mutex mu;
  static std::map<std::string, int> seen;
  std::lock_guard<std::mutex> lk(mu);
  auto it = seen.find(name);
  if (it != seen.end()) return it->second;
  const char* v = std::getenv(name);
  const int x = v != nullptr ? std::atoi(v) : dflt;
  seen[name] = x;
  return x;
}

// ----------------------------------------------------------------- planning
struct Plan {
  Instance inst;
  int key = 0;
  int box_rows = 1;
  int64_t partitions = 0;
  int64_t slots = 0;
  size_t off_meta = 0, off_ml = 0, off_o = 0, bytes = 0;
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// max_pages: block-table width (dense) or total pages of the index (CSR,
// csr = true), which bounds the tiles differently.
int make_plan(int device, int64_t batch, int64_t hkv, int64_t gqa, int64_t head_dim, int64_t page_size,
              int64_t max_pages, int64_t num_splits, Plan* plan, bool csr = false) {
  if (batch < 0 || hkv <= 0 || gqa <= 0 || page_size <= 0 || max_pages < 0)
    return fail(PAD_ERR_INVALID_ARGUMENT,
                "invalid sizes: batch=%lld num_kv_heads=%lld gqa_ratio=%lld page_size=%lld max_pages=%lld",
                (long long)batch, (long long)hkv, (long long)gqa, (long long)page_size, (long long)max_pages);
  if (head_dim != 16 && head_dim != 32 && head_dim != 64 && head_dim != 128)
    return fail(PAD_ERR_UNSUPPORTED, "head_dim %lld not supported (16, 32, 64 or 128)", (long long)head_dim);
  if (gqa > 16) return fail(PAD_ERR_UNSUPPORTED, "gqa_ratio %lld > 16 not supported", (long long)gqa);
  const int64_t cap = max_pages * page_size;
  const int hg = head_group_for(hkv, gqa);
  const int tt = kTileRows / hg;
  const int64_t tiles_max = (cap + tt - 1) / tt;
  const int64_t groups = hkv / hg;
  const int64_t tiles_ub = csr ? groups * (tiles_max + batch) : batch * groups * tiles_max;
  if (cap > INT32_MAX || tiles_ub > INT32_MAX / 2 || batch * groups > INT32_MAX / 4)
    return fail(PAD_ERR_UNSUPPORTED, "problem too large for 32-bit tile indexing (%lld tiles)", (long long)tiles_ub);
  plan->box_rows = box_rows_for(page_size, tt);
  const bool swz = plan->box_rows >= 8;
  if (!pick_instance(head_dim, gqa, hg, swz, &plan->inst))
    return fail(PAD_ERR_UNSUPPORTED, "no kernel instance for head_dim %lld", (long long)head_dim);
  plan->key = instance_key(head_dim, gqa, hg, swz);
  int sms = 0, occ = 0;
  int st = prepare_device(device, plan->inst, plan->key, &sms, &occ);
  if (st != PAD_OK) return st;
  int64_t parts;
  if (num_splits <= 0) {
    parts = (int64_t)sms * occ;
    // Few (sequence, head group) pairs -- long single sequences -- split
    // into a power-of-two count (128 of the 148 resident CTAs on B200): their
    // tile counts are usually powers of two, so every partition gets the same
    // number of tiles, and the merge folds fewer partials. Measured: -0.6 ...
    // -0.8 us at batch 1 / 16k-128k tokens, -0.2 ... -0.3 us at batch 8-16;
    // from 32 pairs up all SMs are needed to keep HBM busy.
    if (batch * groups <= kFewPairs) {
      int64_t pow2 = 1;
      while (pow2 * 2 <= parts) pow2 *= 2;
      parts = pow2;
    }
    if (parts > tiles_ub) parts = tiles_ub;
  } else {
    parts = num_splits * batch * groups;
    if (parts > (int64_t)1 << 30) return fail(PAD_ERR_UNSUPPORTED, "num_splits %lld too large", (long long)num_splits);
  }
  if (parts < 1) parts = 1;
  plan->partitions = parts;
  plan->slots = parts + batch * groups;
  plan->off_meta = 0;
  plan->off_ml = align_up((size_t)std::max<int64_t>(parts, batch * groups) * sizeof(int4), 256);
  plan->off_o = align_up(plan->off_ml + (size_t)plan->slots * hg * gqa * sizeof(float2), 256);
  plan->bytes = align_up(plan->off_o + (size_t)plan->slots * hg * gqa * head_dim * sizeof(float), 256);
  return PAD_OK;
}

// ----------------------------------------------------------------- tensor maps
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

CUtensorMapSwizzle swizzle_mode(const Instance& in) {
  if (!in.swz) return CU_TENSOR_MAP_SWIZZLE_NONE;
  return in.segw == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                        : (in.segw == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

int encode_map(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
               const cuuint32_t* box, CUtensorMapSwizzle swz, const char* what) {
  auto enc = get_encode();
  if (enc == nullptr) return fail(PAD_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PAD_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled(%s) failed (%d)", what, (int)r);
  return PAD_OK;
}

// Encoded maps of recent calls, per thread: a serving loop passes the same
// KV caches (and often the same q buffer) every step, so most calls reuse an
// encoding instead of paying for cuTensorMapEncodeTiled again.
struct MapKey {
  const void* base;
  int rank;
  int swz;
  cuuint64_t dims[5];
  cuuint64_t strides[4];
  cuuint32_t box[5];
};
struct MapCacheEntry {
  MapKey key;
  CUtensorMap map;
  bool valid;
};
constexpr int kMapCacheSize = 16;
thread_local MapCacheEntry t_maps[kMapCacheSize];
thread_local int t_map_next = 0;

int encode_map_cached(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                      const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle swz, const char* what) {
  MapKey k;
  std::memset(&k, 0, sizeof(k));
  k.base = base;
  k.rank = rank;
  k.swz = (int)swz;
  for (int i = 0; i < rank; ++i) {
    k.dims[i] = dims[i];
    k.box[i] = box[i];
    if (i + 1 < rank) k.strides[i] = strides_bytes[i];
  }
  for (int i = 0; i < kMapCacheSize; ++i) {
    if (t_maps[i].valid && std::memcmp(&t_maps[i].key, &k, sizeof(k)) == 0) {
      *map = t_maps[i].map;
      return PAD_OK;
    }
  }
  const int st = encode_map(map, base, rank, dims, strides_bytes, box, swz, what);
  if (st != PAD_OK) return st;
  MapCacheEntry& e = t_maps[t_map_next];
  t_map_next = (t_map_next + 1) % kMapCacheSize;
  e.key = k;
  e.map = *map;
  e.valid = true;
  return PAD_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// =============================================================================
extern "C" {

const char* pad_status_string(int status) {
  switch (status) {
    case PAD_OK: return "ok";
    case PAD_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PAD_ERR_UNSUPPORTED: return "unsupported configuration";
    case PAD_ERR_WORKSPACE: return "workspace missing or too small";
    case PAD_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

const char* pad_last_error(void) { return pad::g_last_error.c_str(); }

int pad_version(void) { return 100; }

int pad_device_info(int device, int64_t head_dim, int64_t gqa_ratio, int* num_sms, int* ctas_per_sm) {
  if (num_sms == nullptr || ctas_per_sm == nullptr) return fail(PAD_ERR_INVALID_ARGUMENT, "null output pointer");
  Instance in;
  if (gqa_ratio < 1 || gqa_ratio > 16 || !pick_instance(head_dim, gqa_ratio, 1, true, &in))
    return fail(PAD_ERR_UNSUPPORTED, "no kernel for head_dim %lld gqa %lld", (long long)head_dim,
                (long long)gqa_ratio);
  return prepare_device(device, in, instance_key(head_dim, gqa_ratio, 1, true), num_sms, ctas_per_sm);
}

int pad_decode_partitions(int device, int64_t batch, int64_t num_kv_heads, int64_t gqa_ratio, int64_t head_dim,
                          int64_t page_size, int64_t max_pages_per_seq, int64_t num_splits, int64_t* partitions) {
  if (partitions == nullptr) return fail(PAD_ERR_INVALID_ARGUMENT, "null output pointer");
  Plan plan;
  int st = make_plan(device, batch, num_kv_heads, gqa_ratio, head_dim, page_size, max_pages_per_seq, num_splits, &plan);
  if (st == PAD_OK) *partitions = plan.partitions;
  return st;
}

int pad_decode_workspace_bytes(int device, int64_t batch, int64_t num_kv_heads, int64_t gqa_ratio, int64_t head_dim,
                               int64_t page_size, int64_t max_pages_per_seq, int64_t num_splits, size_t* bytes) {
  if (bytes == nullptr) return fail(PAD_ERR_INVALID_ARGUMENT, "null output pointer");
  Plan plan;
  int st = make_plan(device, batch, num_kv_heads, gqa_ratio, head_dim, page_size, max_pages_per_seq, num_splits, &plan);
  if (st == PAD_OK) *bytes = plan.bytes;
  return st;
}

}  // extern "C"

namespace {

// Shared body of the dense and the CSR entry points (csr_indptr == nullptr:
// dense block table + seq_lens; else block_table is the CSR `indices` array
// of max_pages_per_seq = nnz entries).
int decode_impl(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                const int32_t* seq_lens, const int32_t* csr_indptr, const int32_t* csr_last, void* out, int64_t batch,
                int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t num_pages, int64_t page_size,
                int64_t max_pages_per_seq, const int64_t* q_strides, const int64_t* k_strides,
                const int64_t* v_strides, int64_t block_table_stride, const int64_t* out_strides, float scale,
                int64_t num_splits, void* workspace, size_t workspace_bytes, void* stream, int32_t* error_flags,
                bool static_scratch = false) {
  const bool csr = csr_indptr != nullptr;
  // ---- shape-only checks (no device access, no sync)
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || num_pages < 0 || page_size <= 0 ||
      max_pages_per_seq < 0)
    return fail(PAD_ERR_INVALID_ARGUMENT, "negative or zero size");
  if (num_q_heads % num_kv_heads != 0)
    return fail(PAD_ERR_INVALID_ARGUMENT, "num_q_heads (%lld) must be divisible by num_kv_heads (%lld)",
                (long long)num_q_heads, (long long)num_kv_heads);
  if (q_strides == nullptr || k_strides == nullptr || v_strides == nullptr || out_strides == nullptr)
    return fail(PAD_ERR_INVALID_ARGUMENT, "null stride array");
  if (!std::isfinite(scale)) return fail(PAD_ERR_INVALID_ARGUMENT, "scale must be finite");
  const int64_t gqa = num_q_heads / num_kv_heads;
  if (batch == 0) return PAD_OK;
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || block_table == nullptr ||
      (!csr && seq_lens == nullptr) || (csr && csr_last == nullptr) || out == nullptr)
    return fail(PAD_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (q_strides[2] != 1 || k_strides[3] != 1 || v_strides[3] != 1 || out_strides[2] != 1)
    return fail(PAD_ERR_UNSUPPORTED, "the head_dim axis of q, k_cache, v_cache and out must be contiguous");
  for (int i = 0; i < 3; ++i)
    if ((k_strides[i] % 8) || (v_strides[i] % 8) || k_strides[i] <= 0 || v_strides[i] <= 0)
      return fail(PAD_ERR_UNSUPPORTED, "k_cache/v_cache strides must be positive multiples of 8 elements");
  if ((q_strides[0] % 8) || (q_strides[1] % 8) || q_strides[0] <= 0 || q_strides[1] <= 0)
    return fail(PAD_ERR_UNSUPPORTED, "q strides must be positive multiples of 8 elements");
  if ((out_strides[0] % 2) || (out_strides[1] % 2))
    return fail(PAD_ERR_UNSUPPORTED, "out strides must be even");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return fail(PAD_ERR_UNSUPPORTED, "q, k_cache, v_cache and out must be 16-byte aligned");
  if (!csr && max_pages_per_seq > 0 && block_table_stride < max_pages_per_seq)
    return fail(PAD_ERR_INVALID_ARGUMENT, "block_table row stride smaller than its width");
  if (num_pages == 0 || max_pages_per_seq == 0) {
    // Nothing addressable: every sequence must be empty. Zero the output.
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int64_t b = 0; b < batch; ++b) {
      cudaError_t e = cudaMemset2DAsync(static_cast<__half*>(out) + b * out_strides[0], out_strides[1] * 2, 0,
                                        head_dim * 2, num_q_heads, s);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemset2DAsync");
    }
    return PAD_OK;
  }
  if (num_pages > INT32_MAX) return fail(PAD_ERR_UNSUPPORTED, "num_pages exceeds int32");

  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  Plan plan;
  int st = make_plan(device, batch, num_kv_heads, gqa, head_dim, page_size, max_pages_per_seq, num_splits, &plan, csr);
  if (st != PAD_OK) return st;
  if (static_scratch && plan.bytes > workspace_bytes)
    return fail(PAD_ERR_WORKSPACE,
                "problem needs %zu bytes of scratch, more than the %zu-byte static scratch of the no-alloc "
                "entry point; use pad_paged_attention_decode with a caller-provided workspace",
                plan.bytes, workspace_bytes);
  if (workspace == nullptr || workspace_bytes < plan.bytes)
    return fail(PAD_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", plan.bytes,
                workspace == nullptr ? (size_t)0 : workspace_bytes);
  if (!aligned16(workspace)) return fail(PAD_ERR_WORKSPACE, "workspace must be 16-byte aligned");

  DecodeParams prm;
  std::memset(&prm, 0, sizeof(prm));
  const Instance& in = plan.inst;
  const CUtensorMapSwizzle swz = swizzle_mode(in);
  {
    // dims ordered {D, token row, KV head, page} so that one box of R tokens x
    // HG heads lands head-major in shared memory
    const cuuint64_t dims[4] = {(cuuint64_t)head_dim, (cuuint64_t)page_size, (cuuint64_t)num_kv_heads,
                                (cuuint64_t)num_pages};
    const cuuint32_t box[4] = {(cuuint32_t)(in.segw / 2), (cuuint32_t)plan.box_rows, (cuuint32_t)in.hg, 1u};
    const cuuint64_t ks[3] = {(cuuint64_t)k_strides[1] * 2, (cuuint64_t)k_strides[2] * 2,
                              (cuuint64_t)k_strides[0] * 2};
    const cuuint64_t vs[3] = {(cuuint64_t)v_strides[1] * 2, (cuuint64_t)v_strides[2] * 2,
                              (cuuint64_t)v_strides[0] * 2};
    if ((st = encode_map_cached(&prm.tm_k, k_cache, 4, dims, ks, box, swz, "k_cache")) != PAD_OK) return st;
    if ((st = encode_map_cached(&prm.tm_v, v_cache, 4, dims, vs, box, swz, "v_cache")) != PAD_OK) return st;
  }
  {
    const cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)num_q_heads, (cuuint64_t)batch};
    const cuuint32_t box[3] = {(cuuint32_t)(in.segw / 2), (cuuint32_t)(gqa * in.hg), 1u};
    const cuuint64_t qs[2] = {(cuuint64_t)q_strides[1] * 2, (cuuint64_t)q_strides[0] * 2};
    if ((st = encode_map_cached(&prm.tm_q, q, 3, dims, qs, box, swz, "q")) != PAD_OK) return st;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  prm.block_table = block_table;
  prm.seq_lens = seq_lens;
  prm.csr_indptr = csr_indptr;
  prm.csr_last = csr_last;
  prm.out = static_cast<__half*>(out);
  prm.ws_meta = reinterpret_cast<int4*>(ws + plan.off_meta);
  prm.ws_ml = reinterpret_cast<float2*>(ws + plan.off_ml);
  prm.ws_o = reinterpret_cast<float*>(ws + plan.off_o);
  prm.error_flags = error_flags;
  prm.bt_stride = block_table_stride;
  prm.out_sb = out_strides[0];
  prm.out_sh = out_strides[1];
  prm.batch = (int)batch;
  prm.hkv = (int)num_kv_heads;
  prm.gqa = (int)gqa;
  prm.page_size = (int)page_size;
  prm.num_pages = (int)num_pages;
  prm.max_pages = (int)max_pages_per_seq;
  prm.box_rows = plan.box_rows;
  prm.box_rows_log2 = __builtin_ctz((unsigned)plan.box_rows);
  prm.page_shift = (page_size & (page_size - 1)) == 0 ? __builtin_ctz((unsigned)page_size) : -1;
  prm.meta_by_pair = batch * (num_kv_heads / in.hg) < plan.partitions ? 1 : 0;
  // guessed first tiles per CTA warmed into L2 before the dependency wait
  // (PAD_B200_L2_WARM overrides, for A/B timing; 0 turns it off)
  prm.l2_warm = env_int("PAD_B200_L2_WARM", 4);
  prm.scale_log2 = scale * kLog2e;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* args[] = {&prm};
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)plan.partitions);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)in.smem_bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    // overlap this launch with the tail of whatever precedes it in the stream
    // (the kernel waits on griddepcontrol before touching global memory)
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelExC(&cfg, in.kernel, args);
  }
  if (e != cudaSuccess) return cuda_fail(e, "launching the decode kernel");
  if (plan.partitions > 1) {
    const float* a0 = prm.ws_o;
    const float2* a1 = prm.ws_ml;
    const int4* a2 = prm.ws_meta;
    __half* a3 = prm.out;
    int ngroups = (int)(num_kv_heads / in.hg), rows = (int)(gqa * in.hg);
    // closed-form split descriptors for a dense batch of full rows (grid by pair)
    int guess_ncap = 0, guess_parts = (int)plan.partitions;
    if (prm.meta_by_pair && !csr) guess_ncap = (int)((max_pages_per_seq * page_size + in.tt - 1) / in.tt);
    void* margs[] = {&a0, &a1, &a2, &a3, &prm.out_sb, &prm.out_sh, &ngroups, &rows, &guess_ncap, &guess_parts};
    cudaLaunchConfig_t cfg = {};
    const bool wide = plan.partitions > kMergeWide * batch * ngroups;
    const int64_t merge_x = prm.meta_by_pair ? batch * ngroups : plan.partitions;
    cfg.gridDim = dim3((unsigned)merge_x, (unsigned)rows, wide ? (unsigned)in.merge_dsplit : 1u);
    // A split pair has about partitions / pairs partials: fold a handful with a
    // small block, long-context splits (hundreds of partials) with a wide one.
    cfg.blockDim = dim3(wide ? 256 : 128);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // overlap its launch with the decode tail
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const bool deep = plan.partitions > kMergeDeep * batch * ngroups;  // 8 loads in flight
    e = cudaLaunchKernelExC(&cfg, wide ? (deep ? in.merge_large : in.merge_mid) : in.merge_small, margs);
    if (e != cudaSuccess) return cuda_fail(e, "launching the merge kernel");
  }
  return PAD_OK;
}

}  // namespace

extern "C" {

int pad_paged_attention_decode(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_table,
                               const int32_t* seq_lens, void* out, int64_t batch, int64_t num_q_heads,
                               int64_t num_kv_heads, int64_t head_dim, int64_t num_pages, int64_t page_size,
                               int64_t max_pages_per_seq, const int64_t* q_strides, const int64_t* k_strides,
                               const int64_t* v_strides, int64_t block_table_stride, const int64_t* out_strides,
                               float scale, int64_t num_splits, void* workspace, size_t workspace_bytes, void* stream,
                               int32_t* error_flags) {
  return decode_impl(q, k_cache, v_cache, block_table, seq_lens, nullptr, nullptr, out, batch, num_q_heads,
                     num_kv_heads, head_dim, num_pages, page_size, max_pages_per_seq, q_strides, k_strides, v_strides,
                     block_table_stride, out_strides, scale, num_splits, workspace, workspace_bytes, stream,
                     error_flags);
}

int pad_decode_csr_workspace_bytes(int device, int64_t batch, int64_t num_kv_heads, int64_t gqa_ratio,
                                   int64_t head_dim, int64_t page_size, int64_t nnz_pages, int64_t num_splits,
                                   size_t* bytes) {
  if (bytes == nullptr) return fail(PAD_ERR_INVALID_ARGUMENT, "null output pointer");
  Plan plan;
  int st = make_plan(device, batch, num_kv_heads, gqa_ratio, head_dim, page_size, nnz_pages, num_splits, &plan, true);
  if (st == PAD_OK) *bytes = plan.bytes;
  return st;
}

int pad_paged_attention_decode_csr(const void* q, const void* k_cache, const void* v_cache, const int32_t* kv_indptr,
                                   const int32_t* kv_indices, const int32_t* kv_last_page_len, void* out,
                                   int64_t batch, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                   int64_t num_pages, int64_t page_size, int64_t nnz_pages,
                                   const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                                   const int64_t* out_strides, float scale, int64_t num_splits, void* workspace,
                                   size_t workspace_bytes, void* stream, int32_t* error_flags) {
  if (kv_indptr == nullptr && batch > 0) return fail(PAD_ERR_INVALID_ARGUMENT, "null kv_indptr");
  return decode_impl(q, k_cache, v_cache, kv_indices, nullptr, kv_indptr, kv_last_page_len, out, batch, num_q_heads,
                     num_kv_heads, head_dim, num_pages, page_size, nnz_pages, q_strides, k_strides, v_strides,
                     nnz_pages, out_strides, scale, num_splits, workspace, workspace_bytes, stream, error_flags);
}

// ----------------------------------------------------------------- no-alloc entry
// Scratch for pad_paged_attention_decode_noalloc, part of the library image:
// the driver reserves it on every GPU the library is loaded on.
static __device__ __align__(256) uint8_t g_pad_static_scratch[PAD_STATIC_SCRATCH_BYTES];

int pad_paged_attention_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                       const int32_t* block_table, const int32_t* seq_lens, void* out,
                                       int64_t batch, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                       int64_t num_pages, int64_t page_size, int64_t max_pages_per_seq,
                                       const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                                       int64_t block_table_stride, const int64_t* out_strides, float scale,
                                       int64_t num_splits, void* stream, int32_t* error_flags) {
  // In host code g_pad_static_scratch names a host-side shadow, not device
  // memory; the device address comes from cudaGetSymbolAddress, looked up
  // once per device with that device current and cached.
  static void* scratch_ptr[kMaxDevices] = {};
  static std::mutex mu;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (device < 0 || device >= kMaxDevices) return fail(PAD_ERR_INVALID_ARGUMENT, "device %d out of range", device);
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (scratch_ptr[device] == nullptr) {
      e = cudaGetSymbolAddress(&scratch_ptr[device], g_pad_static_scratch);
      if (e != cudaSuccess) {
        scratch_ptr[device] = nullptr;
        return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
      }
    }
    ptr = scratch_ptr[device];
  }
  // The size check against the scratch happens inside decode_impl, after the
  // same argument checks as the workspace entry point (same status codes for
  // bad arguments).
  return decode_impl(q, k_cache, v_cache, block_table, seq_lens, nullptr, nullptr, out, batch, num_q_heads,
                     num_kv_heads, head_dim, num_pages, page_size, max_pages_per_seq, q_strides, k_strides, v_strides,
                     block_table_stride, out_strides, scale, num_splits, ptr, PAD_STATIC_SCRATCH_BYTES, stream,
                     error_flags, /*static_scratch=*/true);
}

#ifdef PAD_TRACE
int pad_debug_trace_read(uint64_t* host, size_t n) {
  cudaError_t e = cudaMemcpyFromSymbol(host, g_pad_trace, n * sizeof(uint64_t));
  return e == cudaSuccess ? PAD_OK : cuda_fail(e, "trace read");
}
int pad_debug_trace_reset(void) {
  void* a = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&a, g_pad_trace);
  if (e == cudaSuccess) e = cudaMemset(a, 0, sizeof(g_pad_trace));
  return e == cudaSuccess ? PAD_OK : cuda_fail(e, "trace reset");
}
#endif

}  // extern "C"
