// Strided gather copy (copy.cu).
#pragma once

#include <cuda_runtime.h>

namespace es {

constexpr int kCopyMaxRank = 8;

// dst (contiguous) = the view of src with the given sizes and element strides.
int strided_gather(const void* src, void* dst, int esize, int rank, const long long* size, const long long* sstride,
                   int num_sms, cudaStream_t stream);

// dst (contiguous) = src (contiguous, sizes[rank]) rolled by shift[d] along
// every dim d in one pass (torch.roll semantics: out[i] = src[i - shift]).
int roll_copy(const void* src, void* dst, int esize, int rank, const long long* size, const long long* shift,
              int num_sms, cudaStream_t stream);

// One thread waits (at most timeout_ns) for *flag >= target, the same bounded
// wait the collectives use on peer flags; result[0] = 1 if it arrived, else 0
// and err records the timeout code.  Lets tests exercise the timeout path.
int wait_probe(const int* flag, int target, int* err, long long timeout_ns, int* result, cudaStream_t stream);

}  // namespace es
