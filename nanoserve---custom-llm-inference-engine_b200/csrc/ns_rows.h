// ns_rows.h -- host-side entry points of the one-block-per-row sampling
// kernel (ns_rows.cu), used by ns_sample() in ns_sample.cu.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "../../include/nanoserve_sampler.h"

namespace ns {

// True when the row kernel can serve this call: 16-byte aligned rows whose
// byte length is a multiple of 16 and a vocabulary in the supported range.
bool rows_supported(const NsSampleArgs& a);

// Launches the row kernel; returns NS_OK or an NS_ERR_* code with `err` set.
int rows_launch(const NsSampleArgs& a, cudaStream_t stream, int device, std::string& err);

// Rows the row kernels' static scratch holds (ns_sample_noalloc's limit).
constexpr int kRowsScratchRows = 256;

// Once per device, with that device current: looks up the device address of
// the static pre-pass scratch (cudaGetSymbolAddress) and keeps it.
int rows_noalloc_setup(int device, std::string& err);

// rows_launch whose pre-pass is given that address instead of naming the
// scratch; rows_noalloc_setup must have run on `device`.
int rows_launch_noalloc(const NsSampleArgs& a, cudaStream_t stream, int device, std::string& err);

}  // namespace ns
