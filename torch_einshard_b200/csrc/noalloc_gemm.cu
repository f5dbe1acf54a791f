// es_gemm_bf16_noalloc: an allocation-free C entry point for the tcgen05 GEMM.
//
// This entry point has no counterpart in the reference implementation; it is
// an addition of this framework.
//
// Who it is for.  Some callers cannot allocate device memory at the point where
// they want a GEMM: code running inside a custom memory pool or arena that
// must not be bypassed, runtimes that forbid cudaMalloc/cudaFree after start-up
// (because those calls synchronise the device or fragment a carefully sized
// pool), plugins hosted by an application that owns all allocations, and
// callers that are not Python/PyTorch at all and so cannot use the torch
// caching allocator.  The regular entry point (torch_einshard_b200._C.gemm)
// allocates its output and, for operands whose row pitch the TMA engine cannot
// address, a padded copy; it also allocates a status word once per device.
// This entry point instead takes the output from the caller and keeps its
// scratch - the padded operand copies and the status word - in one file-scope
// static device array of a fixed size.
//
// Contract.
//   C[M, N] (bf16, row-major, row pitch ldc) = A @ B, bf16 inputs, fp32 accumulate.
//   a_mn = 0: A is stored [M][K] with row pitch lda (elements);
//   a_mn = 1: A is stored [K][M] with row pitch lda.
//   b_mn = 0: B is stored [N][K] with row pitch ldb (the usual nn.Linear weight);
//   b_mn = 1: B is stored [K][N] with row pitch ldb.
//   stream: a cudaStream_t (0 for the legacy default stream).
// An operand whose base address is not 16-byte aligned or whose row pitch is
// not a multiple of 8 elements is first copied into the scratch array with a
// padded pitch.  The scratch holds kNoAllocScratchBytes (16 MiB) for those
// copies; a call whose padded copies need more is rejected with return code
// -2 and a message on stderr, and nothing is launched.  Calls whose operands
// are already aligned use no scratch beyond the 16-byte status word and have
// no size limit.
//
// Return codes: 0 success; -1 invalid arguments; -2 the padded operand copies
// exceed the scratch size; -3 the scratch address could not be obtained;
// -4 a launch of this call failed (the CUDA error is printed);
// -5 a CUDA error from earlier work of the caller was already pending when the
// call began (left pending, nothing launched), so that -4 only ever reports
// this call's own failures.
//
// Status word.  The GEMM's waits are bounded: if one runs out (a stalled
// pipeline), the kernel writes an error code into the status word and exits
// early, leaving C incomplete, while the launch itself succeeded and the call
// returned 0.  es_gemm_bf16_noalloc_status() reports that code: it waits for
// the caller's stream, copies the word to the host and clears it.
//
// Set-up and sharing.  On the first call on each device (with that device
// current), the entry point looks the scratch array up with
// cudaGetSymbolAddress and caches the address; make that first call before
// any stream capture.  Every call on a device shares the one array and it
// keeps the previous call's contents: the padded copies are rewritten in full
// by each call that needs them; the status word starts at zero (static device
// memory is zero-initialised when the library loads), keeps the first error
// code written into it, and is cleared only by es_gemm_bf16_noalloc_status.
// Calls that overlap on the GPU (different streams without ordering between
// them) race on the scratch and must not be issued.
#include <cuda_bf16.h>
#include <stdio.h>

#include "gemm.h"
#include "noalloc_gemm.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;  // padded operand copies
constexpr size_t kStatusBytes = 256;                // status word (kernels set it on a timed-out wait)

// The scratch itself: one array per device that loads this library, held until exit.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kStatusBytes + kNoAllocScratchBytes];

void* g_scratch_addr[64] = {nullptr};  // host-side cache of the device address, per device

// Device address of this device's scratch array (looked up once per device,
// with that device current); nullptr on failure.
unsigned char* scratch_base(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (dev_out) *dev_out = dev;
  if (!g_scratch_addr[dev]) {
    void* addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
    if (e != cudaSuccess || addr == nullptr) {
      fprintf(stderr, "es_gemm_bf16_noalloc: cudaGetSymbolAddress failed: %s\n", cudaGetErrorString(e));
      return nullptr;
    }
    g_scratch_addr[dev] = addr;
  }
  return static_cast<unsigned char*>(g_scratch_addr[dev]);
}

__global__ void pad_rows_kernel(const __nv_bfloat16* src, long long src_pitch, __nv_bfloat16* dst,
                                long long dst_pitch, long long rows, long long cols) {
  const long long total = rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols;
    const long long c = i - r * cols;
    dst[r * dst_pitch + c] = src[r * src_pitch + c];
  }
}

bool needs_padding(const void* p, long long pitch) {
  return (reinterpret_cast<uintptr_t>(p) & 15) != 0 || (pitch * 2) % 16 != 0;
}

long long padded_pitch(long long cols) { return (cols + 7) / 8 * 8; }

}  // namespace

extern "C" int es_gemm_bf16_noalloc(const void* A, long long lda, int a_mn, const void* B, long long ldb, int b_mn,
                                    void* C, long long ldc, int M, int N, int K, void* stream_handle) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || (a_mn != 0 && a_mn != 1) || (b_mn != 0 && b_mn != 1))
    return -1;
  const long long a_rows = a_mn ? K : M, a_cols = a_mn ? M : K;
  const long long b_rows = b_mn ? K : N, b_cols = b_mn ? N : K;
  if (lda < a_cols || ldb < b_cols || ldc < N) return -1;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_handle);

  // an error left pending by the caller's earlier work would be read back (and
  // cleared) by the launch checks below and misreported as this call's failure
  if (cudaPeekAtLastError() != cudaSuccess) return -5;
  int dev = 0;
  unsigned char* scratch = scratch_base(&dev);
  if (!scratch) return -3;
  int* status = reinterpret_cast<int*>(scratch);
  unsigned char* pad_area = scratch + kStatusBytes;

  const bool pad_a = needs_padding(A, lda);
  const bool pad_b = needs_padding(B, ldb);
  const long long a_pitch = pad_a ? padded_pitch(a_cols) : lda;
  const long long b_pitch = pad_b ? padded_pitch(b_cols) : ldb;
  const size_t a_bytes = pad_a ? static_cast<size_t>(a_rows * a_pitch * 2) : 0;
  const size_t b_bytes = pad_b ? static_cast<size_t>(b_rows * b_pitch * 2) : 0;
  const size_t b_offset = (a_bytes + 255) / 256 * 256;
  if (b_offset + b_bytes > kNoAllocScratchBytes) {
    fprintf(stderr,
            "es_gemm_bf16_noalloc: operands need %zu bytes of padded copies, more than the %zu-byte scratch; "
            "pass operands with 16-byte aligned bases and row pitches that are multiples of 8 elements\n",
            b_offset + b_bytes, kNoAllocScratchBytes);
    return -2;
  }

  cudaError_t e = cudaSuccess;
  const void* a_use = A;
  const void* b_use = B;
  if (e == cudaSuccess && pad_a) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(pad_area);
    pad_rows_kernel<<<256, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(A), lda, dst, a_pitch, a_rows, a_cols);
    e = cudaGetLastError();
    a_use = dst;
  }
  if (e == cudaSuccess && pad_b) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(pad_area + b_offset);
    pad_rows_kernel<<<256, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(B), ldb, dst, b_pitch, b_rows, b_cols);
    e = cudaGetLastError();
    b_use = dst;
  }
  if (e != cudaSuccess) {
    fprintf(stderr, "es_gemm_bf16_noalloc: %s\n", cudaGetErrorString(e));
    return -4;
  }

  es::GemmArgs g;
  g.A = a_use;
  g.B = b_use;
  g.C = C;
  g.dtype = es::kDtypeBF16;
  g.out_dtype = es::kDtypeBF16;
  g.batch = 1;
  g.M = M;
  g.N = N;
  g.K = K;
  g.a_mn = a_mn;
  g.lda = a_pitch;
  g.b_mn = b_mn;
  g.ldb = b_pitch;
  g.ldc = ldc;
  g.err = status;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  g.num_sms = sms > 0 ? sms : 148;
  if (es::check_gemm_args(g)) return -1;
  const int rc = es::gemm_launch(g, stream);
  if (rc != 0) {
    fprintf(stderr, "es_gemm_bf16_noalloc: launch failed: %s\n", cudaGetErrorString(static_cast<cudaError_t>(rc)));
    return -4;
  }
  return 0;
}

extern "C" int es_gemm_bf16_noalloc_status(int* code, void* stream_handle) {
  if (!code) return -1;
  unsigned char* scratch = scratch_base(nullptr);
  if (!scratch) return -3;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_handle);
  int value = 0;
  cudaError_t e = cudaMemcpyAsync(&value, scratch, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess && value != 0) e = cudaMemsetAsync(scratch, 0, sizeof(int), stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) {
    fprintf(stderr, "es_gemm_bf16_noalloc_status: %s\n", cudaGetErrorString(e));
    return -4;
  }
  *code = value;
  return 0;
}

namespace es {
// Device address of the status word (the first int of the scratch array), for
// the tests that make a bounded wait run out against it; nullptr on failure.
int* noalloc_status_word() { return reinterpret_cast<int*>(scratch_base(nullptr)); }
}  // namespace es
