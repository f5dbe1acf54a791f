// Elementwise SiLU passes for the activation of a contraction (einshard's
// activation="silu") when it is not fused into the GEMM epilogue, and the
// backward product dH = dA * silu'(H).  16-bit tensors, 16-byte vectors with a
// scalar tail, fp32 arithmetic:
//   silu(x)  = x s,  s = 1 / (1 + e^-x)
//   silu'(x) = s (1 + x (1 - s))
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <stdint.h>

#include "act.h"

namespace es {
namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + __expf(-x)); }

template <typename T, bool kBackward>
__global__ void __launch_bounds__(256) silu_kernel(const T* __restrict__ h, const T* __restrict__ g, T* __restrict__ out,
                                                   long long n) {
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long nth = static_cast<long long>(gridDim.x) * blockDim.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(out) |
                     (kBackward ? reinterpret_cast<uintptr_t>(g) : 0)) & 15) == 0;
  const long long nv = vec ? n / 8 : 0;
  for (long long i = tid; i < nv; i += nth) {
    uint4 hv = reinterpret_cast<const uint4*>(h)[i];
    uint4 gv = kBackward ? reinterpret_cast<const uint4*>(g)[i] : hv;
    const T* hx = reinterpret_cast<const T*>(&hv);
    const T* gx = reinterpret_cast<const T*>(&gv);
    uint4 ov;
    T* ox = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x = to_f(hx[j]);
      const float s = sigmoid_f(x);
      ox[j] = from_f<T>(kBackward ? to_f(gx[j]) * s * (1.0f + x * (1.0f - s)) : x * s);
    }
    reinterpret_cast<uint4*>(out)[i] = ov;
  }
  for (long long i = nv * 8 + tid; i < n; i += nth) {
    const float x = to_f(h[i]);
    const float s = sigmoid_f(x);
    out[i] = from_f<T>(kBackward ? to_f(g[i]) * s * (1.0f + x * (1.0f - s)) : x * s);
  }
}

int grid_for(long long n, int sms) {
  const long long want = (n / 8 + 255) / 256;
  const long long cap = static_cast<long long>(sms) * 8;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

}  // namespace

int silu_forward(const void* h, void* out, long long n, int dtype, int sms, cudaStream_t stream) {
  if (n <= 0) return 0;
  const int grid = grid_for(n, sms);
  if (dtype == 0)
    silu_kernel<__nv_bfloat16, false><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(h), nullptr,
                                                                static_cast<__nv_bfloat16*>(out), n);
  else
    silu_kernel<__half, false><<<grid, 256, 0, stream>>>(static_cast<const __half*>(h), nullptr,
                                                         static_cast<__half*>(out), n);
  return static_cast<int>(cudaGetLastError());
}

int silu_backward(const void* grad, const void* h, void* out, long long n, int dtype, int sms, cudaStream_t stream) {
  if (n <= 0) return 0;
  const int grid = grid_for(n, sms);
  if (dtype == 0)
    silu_kernel<__nv_bfloat16, true><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(h),
                                                               static_cast<const __nv_bfloat16*>(grad),
                                                               static_cast<__nv_bfloat16*>(out), n);
  else
    silu_kernel<__half, true><<<grid, 256, 0, stream>>>(static_cast<const __half*>(h),
                                                        static_cast<const __half*>(grad), static_cast<__half*>(out), n);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace es
