// ns_rows.h -- host-side entry points of the row sampling kernel
// (ns_rows.cu), used by ns_sample() in ns_sample.cu.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "../../include/nanoserve_sampler.h"

namespace ns {

// True when the row kernel can serve this call: 16-byte aligned rows
// whose byte length is a multiple of 16 and a vocabulary in the supported
// range.
bool rows_supported(const NsSampleArgs& a);

// Bytes of workspace for calls of up to num_rows rows (ns_workspace_bytes).
int64_t rows_workspace_bytes(int32_t num_rows);

// Launches the row kernel on a.workspace; returns NS_OK or an NS_ERR_*
// code with `err` set.
int rows_launch(const NsSampleArgs& a, cudaStream_t stream, int device, std::string& err);

// The same on the library's static workspace (ns_sample_noalloc): its device
// address is looked up with cudaGetSymbolAddress on the current device.
int rows_launch_noalloc(const NsSampleArgs& a, cudaStream_t stream, int device, std::string& err);

}  // namespace ns
