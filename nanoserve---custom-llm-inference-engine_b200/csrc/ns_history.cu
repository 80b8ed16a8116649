// ns_history.cu -- device-resident prior-token histories for the repetition
// penalty.
//
// The reference rebuilds every request's history as a Python list each step
// (nanoserve/engine.py:242-246: prompt + output token ids) and the sampler
// turns the lists into index tensors (nanoserve/scheduler/sampler.py:34).
// Here the ids live in one append-only device pool (int32), a region per
// request: the prompt is copied in once, and each step appends the sampled
// id of every running request with one launch (ns_history_append).  A step's
// CSR histories -- history_offsets / history_ids of NsSampleArgs -- are
// gathered from the pool on the device (ns_history_gather).  The host only
// handles O(rows) numbers per step: region starts, lengths and offsets.
//
// Both kernels are byte-moving work far below a microsecond of HBM time at
// serving sizes (a config-2 step gathers about 70 k ids); they are sized for
// launch latency, not bandwidth.
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/nanoserve_sampler.h"

namespace ns {
int fail(int code, const std::string& msg);

namespace hist {

constexpr int kThreads = 256;
constexpr int kMaxBlocks = 148 * 8;

// Row r's ids: pool[src[r] + j] -> ids[offsets[r] + j] for j < offsets[r+1] -
// offsets[r].  A row whose source range leaves [0, pool_size) gets ids of -1
// (which ns_sample reports as NS_STATUS_BAD_HISTORY_ID) and sets
// NS_STATUS_BAD_POOL_RANGE.
__global__ void __launch_bounds__(kThreads) gather_kernel(const int32_t* __restrict__ pool, int64_t pool_size,
                                                          const int64_t* __restrict__ src,
                                                          const int64_t* __restrict__ offsets,
                                                          int32_t* __restrict__ ids, int rows, uint32_t* status) {
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t o0 = offsets[r], n = offsets[r + 1] - o0;
    const int64_t s0 = src[r];
    int32_t* d = ids + o0;
    const bool ok = n >= 0 && s0 >= 0 && s0 <= pool_size && n <= pool_size - s0;
    if (!ok) {
      if (threadIdx.x == 0 && status) atomicOr(status, NS_STATUS_BAD_POOL_RANGE);
      for (int64_t j = threadIdx.x; j < n; j += kThreads) d[j] = -1;
      continue;
    }
    const int32_t* s = pool + s0;
    for (int64_t j = threadIdx.x; j < n; j += kThreads) d[j] = __ldg(s + j);
  }
}

// pool[dst[r]] = tokens[r] for every row with dst[r] >= 0 (dst[r] < 0: the
// row's request is not tracked).  A destination at or past pool_size is not
// written and sets NS_STATUS_BAD_POOL_RANGE.
__global__ void __launch_bounds__(kThreads) append_kernel(int32_t* __restrict__ pool, int64_t pool_size,
                                                          const int64_t* __restrict__ dst,
                                                          const void* __restrict__ tokens, int tok_i32, int rows,
                                                          uint32_t* status) {
  const int r = blockIdx.x * kThreads + threadIdx.x;
  if (r >= rows) return;
  const int64_t p = dst[r];
  if (p < 0) return;
  if (p >= pool_size) {
    if (status) atomicOr(status, NS_STATUS_BAD_POOL_RANGE);
    return;
  }
  pool[p] = tok_i32 ? static_cast<const int32_t*>(tokens)[r]
                    : static_cast<int32_t>(static_cast<const int64_t*>(tokens)[r]);
}

}  // namespace hist
}  // namespace ns

extern "C" {

int ns_history_gather(const int32_t* pool, int64_t pool_size, const int64_t* row_src, const int64_t* offsets,
                      int32_t num_rows, int32_t* out_ids, uint32_t* status, void* stream) {
  using namespace ns;
  if (num_rows < 0) return fail(NS_ERR_INVALID_ARG, "ns_history_gather: num_rows < 0");
  if (pool_size < 0) return fail(NS_ERR_INVALID_ARG, "ns_history_gather: pool_size < 0");
  if (num_rows == 0) return NS_OK;
  if (!row_src || !offsets || !out_ids || (!pool && pool_size > 0))
    return fail(NS_ERR_INVALID_ARG, "ns_history_gather: null device pointer");
  const int grid = num_rows < hist::kMaxBlocks ? num_rows : hist::kMaxBlocks;
  hist::gather_kernel<<<grid, hist::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      pool, pool_size, row_src, offsets, out_ids, num_rows, status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NS_ERR_CUDA, std::string("ns_history_gather launch: ") + cudaGetErrorString(e));
  return NS_OK;
}

int ns_history_append(int32_t* pool, int64_t pool_size, const int64_t* row_dst, const void* tokens,
                      int32_t tokens_dtype, int32_t num_rows, uint32_t* status, void* stream) {
  using namespace ns;
  if (num_rows < 0) return fail(NS_ERR_INVALID_ARG, "ns_history_append: num_rows < 0");
  if (pool_size < 0) return fail(NS_ERR_INVALID_ARG, "ns_history_append: pool_size < 0");
  if (tokens_dtype != NS_OUT_I64 && tokens_dtype != NS_OUT_I32)
    return fail(NS_ERR_INVALID_ARG, "ns_history_append: tokens_dtype must be NS_OUT_I64 or NS_OUT_I32");
  if (num_rows == 0) return NS_OK;
  if (!pool || !row_dst || !tokens) return fail(NS_ERR_INVALID_ARG, "ns_history_append: null device pointer");
  const int grid = (num_rows + hist::kThreads - 1) / hist::kThreads;
  hist::append_kernel<<<grid, hist::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      pool, pool_size, row_dst, tokens, tokens_dtype == NS_OUT_I32 ? 1 : 0, num_rows, status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NS_ERR_CUDA, std::string("ns_history_append launch: ") + cudaGetErrorString(e));
  return NS_OK;
}

}  // extern "C"
