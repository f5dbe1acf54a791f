// Elementwise SiLU forward / backward (act.cu).  dtype: 0 bf16, 1 f16.
#pragma once

#include <cuda_runtime.h>

namespace es {

// out = silu(h), n elements.
int silu_forward(const void* h, void* out, long long n, int dtype, int sms, cudaStream_t stream);
// out = grad * silu'(h), n elements.
int silu_backward(const void* grad, const void* h, void* out, long long n, int dtype, int sms, cudaStream_t stream);

}  // namespace es
