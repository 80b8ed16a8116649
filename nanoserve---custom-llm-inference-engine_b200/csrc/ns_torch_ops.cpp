// ns_torch_ops.cpp -- registers torch.ops.nanoserve_b200.sample over the C ABI.
//
// A thin adapter: it checks devices/dtypes, turns tensors into raw pointers,
// fills an NsSampleArgs and calls ns_sample() on the current CUDA stream.
// No math happens here; the kernel lives in libnanoserve_sampler.so.
//
// Each (device, stream) gets its own workspace (NsSampleArgs.workspace),
// zeroed once when it is allocated through torch's caching allocator and
// left zero by every call, so calls on different streams never share one.
// Warm a stream up before capturing a graph on it, so that the graph does
// not hold the workspace's first zeroing.
#include <ATen/core/Tensor.h>
#include <ATen/ops/zeros.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <mutex>
#include <unordered_map>

#include "../../include/nanoserve_sampler.h"

namespace {

struct Workspace {
  at::Tensor t;
  bool zero_pending = false;  // made during a stream capture: its zeroing ran only inside the graph
};
std::mutex g_ws_mu;
// never destroyed: the tensors must not be freed after the CUDA context at exit
auto* g_ws = new std::unordered_map<uint64_t, Workspace>();

at::Tensor workspace_for(const at::Device& dev, cudaStream_t stream, int64_t bytes) {
  const uint64_t key = (uint64_t)reinterpret_cast<uintptr_t>(stream) * 64u + (uint64_t)dev.index();
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  TORCH_CHECK(cudaStreamIsCapturing(stream, &cap) == cudaSuccess, "cudaStreamIsCapturing failed");
  const bool capturing = cap != cudaStreamCaptureStatusNone;
  std::lock_guard<std::mutex> lk(g_ws_mu);
  auto it = g_ws->find(key);
  if (it != g_ws->end() && it->second.t.numel() >= bytes) {
    Workspace& w = it->second;
    if (w.zero_pending && !capturing) {
      // a graph made it and may never have been replayed: zero it before this eager call
      TORCH_CHECK(cudaMemsetAsync(w.t.data_ptr(), 0, (size_t)w.t.numel(), stream) == cudaSuccess,
                  "cudaMemsetAsync of the sampler workspace failed");
      w.zero_pending = false;
    }
    return w.t;
  }
  // zeroed on the current stream, the one the kernel is enqueued on (inside a
  // capture the zeroing becomes a node of the graph)
  Workspace w;
  w.t = at::zeros({bytes}, at::TensorOptions().dtype(at::kByte).device(dev));
  w.zero_pending = capturing;
  (*g_ws)[key] = w;
  return w.t;
}

const void* opt_ptr(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr;
}

void check_cuda(const at::Tensor& t, const at::Device& dev, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.device() == dev, name, " must be on ", dev);
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

void check_opt(const c10::optional<at::Tensor>& t, const at::Device& dev, const char* name, at::ScalarType st) {
  if (!t.has_value() || !t->defined()) return;
  check_cuda(*t, dev, name);
  TORCH_CHECK(t->scalar_type() == st, name, " has dtype ", t->scalar_type(), ", expected ", st);
}

// sample(logits, sample_indices, row_params, history_offsets, history_ids,
//        uniforms, philox_seed, philox_offset, row_offset, out,
//        out_penalized, out_filtered, out_probs, status, row_order, kernel) -> ()
void sample_op(const at::Tensor& logits, const c10::optional<at::Tensor>& sample_indices,
               const at::Tensor& row_params, const c10::optional<at::Tensor>& history_offsets,
               const c10::optional<at::Tensor>& history_ids, const c10::optional<at::Tensor>& uniforms,
               int64_t philox_seed, int64_t philox_offset, int64_t row_offset, at::Tensor& out,
               const c10::optional<at::Tensor>& out_penalized, const c10::optional<at::Tensor>& out_filtered,
               const c10::optional<at::Tensor>& out_probs, const c10::optional<at::Tensor>& status,
               const c10::optional<at::Tensor>& row_order, int64_t kernel) {
  TORCH_CHECK(logits.dim() == 2, "logits must be 2-D [rows, vocab]");
  TORCH_CHECK(logits.is_cuda(), "logits must be a CUDA tensor");
  TORCH_CHECK(logits.stride(1) == 1, "logits rows must be contiguous");
  TORCH_CHECK(logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kBFloat16,
              "logits must be float32 or bfloat16");
  const at::Device dev = logits.device();
  c10::cuda::CUDAGuard guard(dev);
  check_cuda(row_params, dev, "row_params");
  TORCH_CHECK(row_params.scalar_type() == at::kByte && row_params.numel() % (int64_t)sizeof(NsRowParams) == 0,
              "row_params must be uint8 with a multiple of ", sizeof(NsRowParams), " bytes");
  const int64_t S = row_params.numel() / (int64_t)sizeof(NsRowParams);
  check_cuda(out, dev, "out");
  TORCH_CHECK(out.numel() == S, "out must have one element per row");
  TORCH_CHECK(out.scalar_type() == at::kLong || out.scalar_type() == at::kInt, "out must be int64 or int32");
  check_opt(sample_indices, dev, "sample_indices", at::kLong);
  check_opt(history_offsets, dev, "history_offsets", at::kLong);
  check_opt(history_ids, dev, "history_ids", at::kInt);
  check_opt(uniforms, dev, "uniforms", at::kFloat);
  check_opt(out_penalized, dev, "out_penalized", at::kFloat);
  check_opt(out_filtered, dev, "out_filtered", at::kFloat);
  check_opt(out_probs, dev, "out_probs", at::kFloat);
  check_opt(status, dev, "status", at::kInt);
  check_opt(row_order, dev, "row_order", at::kInt);
  if (row_order.has_value() && row_order->defined())
    TORCH_CHECK(row_order->numel() == S, "row_order must have one element per row");
  if (sample_indices.has_value() && sample_indices->defined())
    TORCH_CHECK(sample_indices->numel() == S, "sample_indices must have one element per row");
  if (uniforms.has_value() && uniforms->defined())
    TORCH_CHECK(uniforms->numel() == S, "uniforms must have one element per row");
  if (history_offsets.has_value() && history_offsets->defined())
    TORCH_CHECK(history_offsets->numel() == S + 1, "history_offsets must have rows+1 elements");
  const int64_t V = logits.size(1);
  for (const auto* t : {&out_penalized, &out_filtered, &out_probs})
    if (t->has_value() && (*t)->defined())
      TORCH_CHECK((*t)->numel() == S * V, "debug outputs must be [rows, vocab]");

  NsSampleArgs a = {};
  a.logits = logits.data_ptr();
  a.logits_dtype = logits.scalar_type() == at::kFloat ? NS_DTYPE_F32 : NS_DTYPE_BF16;
  a.vocab_size = (int32_t)V;
  a.num_logit_rows = logits.size(0);
  // a single-row tensor may report any stride for its size-1 dimension
  a.logits_row_stride = logits.size(0) == 1 ? V : logits.stride(0);
  a.num_rows = (int32_t)S;
  a.out_dtype = out.scalar_type() == at::kLong ? NS_OUT_I64 : NS_OUT_I32;
  a.sample_indices = static_cast<const int64_t*>(opt_ptr(sample_indices));
  a.row_params = static_cast<const NsRowParams*>(row_params.data_ptr());
  a.history_offsets = static_cast<const int64_t*>(opt_ptr(history_offsets));
  a.history_ids = static_cast<const int32_t*>(opt_ptr(history_ids));
  a.uniforms = static_cast<const float*>(opt_ptr(uniforms));
  a.philox_seed = (uint64_t)philox_seed;
  a.philox_offset = (uint64_t)philox_offset;
  a.row_offset = row_offset;
  a.out_tokens = out.data_ptr();
  a.out_penalized = static_cast<float*>(const_cast<void*>(opt_ptr(out_penalized)));
  a.out_filtered = static_cast<float*>(const_cast<void*>(opt_ptr(out_filtered)));
  a.out_probs = static_cast<float*>(const_cast<void*>(opt_ptr(out_probs)));
  a.status = static_cast<uint32_t*>(const_cast<void*>(opt_ptr(status)));
  a.row_order = static_cast<const int32_t*>(opt_ptr(row_order));
  a.kernel = (int32_t)kernel;
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  const int64_t ws_bytes = ns_workspace_bytes((int32_t)S);
  const at::Tensor ws = workspace_for(dev, stream, ws_bytes);
  a.workspace = ws.data_ptr();
  a.workspace_bytes = ws.numel();
  const int rc = ns_sample(&a, stream);
  TORCH_CHECK(rc == NS_OK, "ns_sample failed (", rc, "): ", ns_last_error());
}

}  // namespace

TORCH_LIBRARY(nanoserve_b200, m) {
  m.def(
      "sample(Tensor logits, Tensor? sample_indices, Tensor row_params, Tensor? history_offsets, "
      "Tensor? history_ids, Tensor? uniforms, int philox_seed, int philox_offset, int row_offset, "
      "Tensor(a!) out, Tensor(b!)? out_penalized, Tensor(c!)? out_filtered, Tensor(d!)? out_probs, "
      "Tensor(e!)? status, Tensor? row_order=None, int kernel=0) -> ()");
}

TORCH_LIBRARY_IMPL(nanoserve_b200, CUDA, m) { m.impl("sample", &sample_op); }
