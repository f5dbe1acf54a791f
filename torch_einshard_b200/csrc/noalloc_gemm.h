// Allocation-free C entry point for the tcgen05 bf16 GEMM.
//
// This entry point has no counterpart in the reference implementation.  It is
// for callers that cannot allocate device memory where they need a GEMM (a
// memory pool or arena that must not be bypassed, a runtime that forbids
// cudaMalloc/cudaFree after start-up, a host application that owns every
// allocation, code outside Python/PyTorch).  It allocates nothing: the output
// comes from the caller, and the only scratch (padded copies of operands the
// TMA engine cannot address, and a status word) is a 16 MiB + 256 B static
// device array shared by all calls on a device.
//
//   C[M, N] = A @ B  (bf16 in, fp32 accumulate, bf16 out, C row pitch ldc)
//   a_mn = 0: A is [M][K], pitch lda;  a_mn = 1: A is [K][M], pitch lda
//   b_mn = 0: B is [N][K], pitch ldb;  b_mn = 1: B is [K][N], pitch ldb
//   stream: a cudaStream_t (or 0)
//
// Returns 0 on success, -1 for invalid arguments, -2 when the padded copies
// would exceed the 16 MiB scratch (nothing is launched; a message goes to
// stderr), -3 when the scratch address cannot be obtained, -4 when a launch
// of this call fails, -5 when a CUDA error from the caller's earlier work was
// already pending (it is left pending and nothing is launched).
//
// A return of 0 means the work was queued.  If a bounded wait inside the GEMM
// then runs out, the kernel stops early and leaves C incomplete; it records an
// error code in the status word.  Read it with es_gemm_bf16_noalloc_status
// after the call: it waits for `stream`, stores the code in *code (0 = the
// GEMMs since the last read finished normally; nonzero = C may be incomplete)
// and clears the word.  It returns 0, or -1/-3/-4 as above.  The first call on each device looks the scratch address up; make it
// before any stream capture.  Calls that may run concurrently on one device
// (unordered streams) race on the shared scratch and must not be issued.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

int es_gemm_bf16_noalloc(const void* A, long long lda, int a_mn, const void* B, long long ldb, int b_mn, void* C,
                         long long ldc, int M, int N, int K, void* stream_handle);
int es_gemm_bf16_noalloc_status(int* code, void* stream_handle);

#ifdef __cplusplus
}
#endif
