// Device transform of a float64 feature-major matrix into uint8 bins with a
// fitted BinMapper: the same bin for every value as BinMapper::bin_value
// (binning.mojo:3242-3455 for numeric features, categorical.mojo:298-462 for
// categorical codes), computed on the GPU so that the dense entry point ships
// the raw columns once instead of binning 10^9 values on the host.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "binning.h"

namespace mtb {

// Bins x[f * n_rows + r] (host memory, float64) into d_bins[f * n_rows + r]
// (device memory) on `stream`.  Columns travel through a pinned double buffer
// in chunks of whole features; host copies into the buffer overlap the DMA
// and the kernel of the previous chunk.  Returns when d_bins is complete.
// Throws std::runtime_error on a CUDA error.
void transform_on_device(const BinMapper& m, const double* x, int64_t n_rows, uint8_t* d_bins,
                         cudaStream_t stream);

// Copies `bytes` bytes of host memory (pre-binned columns, labels) to device
// memory on `stream` through page-registered staging buffers; returns when
// the copy is complete.  Throws std::runtime_error on a CUDA error.
void upload_host(const void* src, int64_t bytes, void* dst_dev, cudaStream_t stream);

}  // namespace mtb
