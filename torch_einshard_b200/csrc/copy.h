// Strided gather copy (copy.cu).
#pragma once

#include <cuda_runtime.h>

namespace es {

constexpr int kCopyMaxRank = 8;

// dst (contiguous) = the view of src with the given sizes and element strides.
int strided_gather(const void* src, void* dst, int esize, int rank, const long long* size, const long long* sstride,
                   int num_sms, cudaStream_t stream);

}  // namespace es
