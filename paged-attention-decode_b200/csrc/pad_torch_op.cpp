// pad_torch_op.cpp -- the thin torch operator over the C ABI of
// libpad_b200.so (include/pad_b200.h): torch.ops.pad_b200.*.
//
// It plays the part of the reference's pybind binding `forward_v4`
// (cuda/binding.cpp:13-14, cuda/kernels.h:60-70) and of the launcher glue
// around it (cuda/kernel_v4_split_k.cu:205-268): it takes tensors, makes
// block_table / seq_lens int32 (src/kernel_cuda_v4.py:58-59), allocates `out`,
// keeps one reusable workspace and one error-flag word per (device, stream),
// and calls the C entry point on the current stream of the inputs' device.
// Everything here is host code; the kernels are in libpad_b200.so.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <utility>

#include "pad_b200.h"

namespace {

struct StreamState {
  at::Tensor workspace;  // uint8, grown on demand, never shrunk
  at::Tensor flags;      // int32[1], PAD_FLAG_* bits OR-ed in by the kernels
};

std::mutex g_mu;
std::map<std::pair<int, cudaStream_t>, StreamState> g_state;

StreamState& state_for(const at::Device& dev, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto key = std::make_pair(static_cast<int>(dev.index()), s);
  auto it = g_state.find(key);
  if (it == g_state.end()) {
    StreamState st;
    st.workspace = at::empty({0}, at::TensorOptions().dtype(at::kByte).device(dev));
    st.flags = at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(dev));
    it = g_state.emplace(key, std::move(st)).first;
  }
  return it->second;
}

void check(int status, const char* what) {
  TORCH_CHECK(status == PAD_OK, "libpad_b200 ", what, ": ", pad_status_string(status), ": ", pad_last_error());
}

at::Tensor as_int32_rows(const at::Tensor& t, const at::Device& dev) {
  at::Tensor r = t.device() == dev && t.scalar_type() == at::kInt ? t : t.to(dev, at::kInt);
  return r.dim() >= 1 && r.stride(-1) == 1 ? r : r.contiguous();
}

// q needs a contiguous head_dim axis, 16-byte aligned rows and base.
at::Tensor tma_ready(const at::Tensor& q) {
  const bool ok = q.stride(2) == 1 && q.stride(0) % 8 == 0 && q.stride(1) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0;
  return ok ? q : q.contiguous();
}

at::Tensor prepare_out(const c10::optional<at::Tensor>& out, const at::Tensor& q) {
  if (!out.has_value()) return at::empty(q.sizes(), q.options().dtype(at::kHalf));
  const at::Tensor& o = *out;
  TORCH_CHECK(o.sizes() == q.sizes() && o.scalar_type() == at::kHalf && o.device() == q.device(),
              "out must be an fp16 tensor shaped like q on q's device");
  return o;
}

// Calls `launch(ws_ptr, ws_bytes)`; when the workspace is too small the
// library reports PAD_ERR_WORKSPACE before launching anything, so grow it to
// `need()` and call again.
template <class Launch, class Need>
void with_workspace(StreamState& st, Launch launch, Need need) {
  int rc = launch(st.workspace.data_ptr(), (size_t)st.workspace.numel());
  if (rc == PAD_ERR_WORKSPACE) {
    size_t bytes = 0;
    check(need(&bytes), "workspace size");
    const int64_t grow = std::max<int64_t>((int64_t)bytes, 2 * st.workspace.numel());
    st.workspace = at::empty({grow}, st.workspace.options());
    rc = launch(st.workspace.data_ptr(), (size_t)st.workspace.numel());
  }
  check(rc, "decode");
}

at::Tensor decode(const at::Tensor& q_in, const at::Tensor& k, const at::Tensor& v, const at::Tensor& bt_in,
                  const at::Tensor& sl_in, int64_t num_splits, double scale, const c10::optional<at::Tensor>& out_in) {
  TORCH_CHECK(q_in.dim() == 3 && k.dim() == 4 && v.sizes() == k.sizes(), "bad q / k_cache / v_cache shapes");
  const at::Device dev = q_in.device();
  c10::cuda::CUDAGuard guard(dev);
  const at::Tensor q = tma_ready(q_in);
  const at::Tensor bt = as_int32_rows(bt_in, dev);
  const at::Tensor sl = as_int32_rows(sl_in, dev);
  at::Tensor out = prepare_out(out_in, q_in);
  const int64_t batch = q.size(0);
  if (batch == 0) return out;
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  StreamState& st = state_for(dev, stream);
  const int64_t qs[3] = {q.stride(0), q.stride(1), q.stride(2)};
  const int64_t ks[4] = {k.stride(0), k.stride(1), k.stride(2), k.stride(3)};
  const int64_t vs[4] = {v.stride(0), v.stride(1), v.stride(2), v.stride(3)};
  const int64_t os[3] = {out.stride(0), out.stride(1), out.stride(2)};
  const int64_t hq = q.size(1), d = q.size(2), pages = k.size(0), ps = k.size(1), hkv = k.size(2);
  const int64_t maxp = bt.size(1);
  with_workspace(
      st,
      [&](void* ws, size_t wsb) {
        return pad_paged_attention_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), bt.data_ptr<int32_t>(),
                                          sl.data_ptr<int32_t>(), out.data_ptr(), batch, hq, hkv, d, pages, ps, maxp,
                                          qs, ks, vs, bt.stride(0), os, (float)scale, num_splits, ws, wsb, stream,
                                          st.flags.data_ptr<int32_t>());
      },
      [&](size_t* bytes) {
        return pad_decode_workspace_bytes((int)dev.index(), batch, hkv, hq / hkv, d, ps, maxp, num_splits, bytes);
      });
  return out;
}

at::Tensor decode_csr(const at::Tensor& q_in, const at::Tensor& k, const at::Tensor& v, const at::Tensor& indptr_in,
                      const at::Tensor& indices_in, const at::Tensor& last_in, int64_t num_splits, double scale,
                      const c10::optional<at::Tensor>& out_in) {
  TORCH_CHECK(q_in.dim() == 3 && k.dim() == 4 && v.sizes() == k.sizes(), "bad q / k_cache / v_cache shapes");
  const at::Device dev = q_in.device();
  c10::cuda::CUDAGuard guard(dev);
  const at::Tensor q = tma_ready(q_in);
  const at::Tensor indptr = as_int32_rows(indptr_in, dev);
  at::Tensor indices = as_int32_rows(indices_in, dev);
  const at::Tensor last = as_int32_rows(last_in, dev);
  at::Tensor out = prepare_out(out_in, q_in);
  const int64_t batch = q.size(0);
  if (batch == 0) return out;
  const int64_t nnz = std::max<int64_t>(indices.numel(), 1);
  if (indices.numel() == 0) indices = at::zeros({1}, indices.options());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  StreamState& st = state_for(dev, stream);
  const int64_t qs[3] = {q.stride(0), q.stride(1), q.stride(2)};
  const int64_t ks[4] = {k.stride(0), k.stride(1), k.stride(2), k.stride(3)};
  const int64_t vs[4] = {v.stride(0), v.stride(1), v.stride(2), v.stride(3)};
  const int64_t os[3] = {out.stride(0), out.stride(1), out.stride(2)};
  const int64_t hq = q.size(1), d = q.size(2), pages = k.size(0), ps = k.size(1), hkv = k.size(2);
  with_workspace(
      st,
      [&](void* ws, size_t wsb) {
        return pad_paged_attention_decode_csr(q.data_ptr(), k.data_ptr(), v.data_ptr(), indptr.data_ptr<int32_t>(),
                                              indices.data_ptr<int32_t>(), last.data_ptr<int32_t>(), out.data_ptr(),
                                              batch, hq, hkv, d, pages, ps, nnz, qs, ks, vs, os, (float)scale,
                                              num_splits, ws, wsb, stream, st.flags.data_ptr<int32_t>());
      },
      [&](size_t* bytes) {
        return pad_decode_csr_workspace_bytes((int)dev.index(), batch, hkv, hq / hkv, d, ps, nnz, num_splits, bytes);
      });
  return out;
}

void kv_append(const at::Tensor& k_new_in, const at::Tensor& v_new_in, const at::Tensor& k_cache,
               const at::Tensor& v_cache, const at::Tensor& bt_in, const at::Tensor& pos_in) {
  TORCH_CHECK(k_new_in.dim() == 3 && k_cache.dim() == 4, "k_new must be [B, Hkv, D], the caches 4-D");
  const at::Device dev = k_cache.device();
  c10::cuda::CUDAGuard guard(dev);
  const at::Tensor bt = as_int32_rows(bt_in, dev);
  const at::Tensor pos = as_int32_rows(pos_in, dev);
  const at::Tensor kn = k_new_in.stride(2) == 1 ? k_new_in : k_new_in.contiguous();
  const at::Tensor vn = v_new_in.stride(2) == 1 ? v_new_in : v_new_in.contiguous();
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  StreamState& st = state_for(dev, stream);
  const int64_t kns[3] = {kn.stride(0), kn.stride(1), kn.stride(2)};
  const int64_t vns[3] = {vn.stride(0), vn.stride(1), vn.stride(2)};
  const int64_t ks[4] = {k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), k_cache.stride(3)};
  const int64_t vs[4] = {v_cache.stride(0), v_cache.stride(1), v_cache.stride(2), v_cache.stride(3)};
  check(pad_paged_kv_append(kn.data_ptr(), vn.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                            bt.data_ptr<int32_t>(), pos.data_ptr<int32_t>(), kn.size(0), kn.size(1), kn.size(2),
                            k_cache.size(0), k_cache.size(1), bt.size(1), kns, vns, ks, vs, bt.stride(0), stream,
                            st.flags.data_ptr<int32_t>()),
        "kv_append");
}

// The error-flag word of `device`'s current stream (the kernels OR
// PAD_FLAG_* bits into it; the caller reads and clears it).
at::Tensor error_flags(int64_t device) {
  const at::Device dev(at::kCUDA, (c10::DeviceIndex)device);
  c10::cuda::CUDAGuard guard(dev);
  return state_for(dev, c10::cuda::getCurrentCUDAStream(dev.index()).stream()).flags;
}

}  // namespace

TORCH_LIBRARY(pad_b200, m) {
  m.def("decode(Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_table, Tensor seq_lens, int num_splits, "
        "float scale, Tensor(a!)? out) -> Tensor");
  m.def("decode_csr(Tensor q, Tensor k_cache, Tensor v_cache, Tensor kv_indptr, Tensor kv_indices, "
        "Tensor kv_last_page_len, int num_splits, float scale, Tensor(a!)? out) -> Tensor");
  m.def("kv_append(Tensor k_new, Tensor v_new, Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor block_table, "
        "Tensor positions) -> ()");
  m.def("error_flags(int device) -> Tensor", &error_flags);
}

TORCH_LIBRARY_IMPL(pad_b200, CUDA, m) {
  m.impl("decode", &decode);
  m.impl("decode_csr", &decode_csr);
  m.impl("kv_append", &kv_append);
}
