// Plain C++ interface of the native GEMM family (no torch types), shared by the
// torch bindings and the fused compute+collective kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace es {

enum Dtype : int { kDtypeBF16 = 0, kDtypeF16 = 1, kDtypeF32 = 2 };

// C[b] = act(A[b] @ B[b]) with A: [batch, M, K], B: [batch, K, N], C: [batch, M, N] row-major.
// a_mn = 0: A is K-contiguous, lda = elements between consecutive m rows.
// a_mn = 1: A is M-contiguous, lda = elements between consecutive k rows.
// b_mn = 0: B is K-contiguous, ldb = elements between consecutive n columns.
// b_mn = 1: B is N-contiguous, ldb = elements between consecutive k rows.
struct GemmArgs {
  const void* A = nullptr;
  const void* B = nullptr;
  void* C = nullptr;
  int dtype = kDtypeBF16;
  int out_dtype = kDtypeBF16;
  int batch = 1, M = 0, N = 0, K = 0;
  int a_mn = 0;
  long long lda = 0, a_batch_stride = 0;
  int b_mn = 0;
  long long ldb = 0, b_batch_stride = 0;
  long long ldc = 0, c_batch_stride = 0;
  int act = 0;
  int* err = nullptr;
  int num_sms = 148;
  int pair = -1;     // -1: choose; 0: 1-SM kernel; 1: 2-SM (CTA pair) kernel
  int group_m = 0;   // raster group height in M tiles (0: default)
  int split = 0;     // wide kernel cluster split (see GemmShape::split)
  unsigned long long* prof = nullptr;  // optional wait-cycle counters (wide kernel)
  int sleep_ns = 0;  // wide kernel epilogue back-off (tuning)
  int persistent = -1;  // wide kernel: 0 one pair tile per cluster, 1 persistent clusters, -1 by K (persistent for K <= 2048)
  int small_persistent = 1;  // 1-SM kernel: 1 persistent CTAs (default), 0 one tile per CTA (tuning)
};

const char* check_gemm_args(const GemmArgs& g);
void make_operand_maps(const GemmArgs& g, CUtensorMap* ma, CUtensorMap* mb, bool pair = false);
bool use_pair_kernel(const GemmArgs& g);
int gemm_launch(const GemmArgs& g, cudaStream_t stream);
struct GemmShape;
GemmShape make_shape(const GemmArgs& g);
GemmShape make_shape_pair(const GemmArgs& g);
// Output tensor map of the TMA-store epilogues; false (map zeroed) when C does not qualify.
bool make_output_map(const GemmArgs& g, bool trans, CUtensorMap* mc);

// Stream-K on the wide 2-SM kernel (batch 1): every SM pair takes the same
// number of K blocks of the tile-major K-block sequence; partial tiles are
// reduce-added in fp32 into a workspace ws[M][gemm_streamk_ws_ld(g)], which a
// finishing pass converts (with the activation) into C.
// gemm_streamk_iters: K blocks per cluster, or 0 when whole tiles are better
// (mode 1: where the shape allows it; 0 or -1: never, the measured default).
int gemm_streamk_iters(const GemmArgs& g, int mode);
long long gemm_streamk_ws_ld(const GemmArgs& g);
int gemm_launch_streamk(const GemmArgs& g, int sk_iters, float* ws, cudaStream_t stream);

}  // namespace es
