// Plain C++ interface of the native GEMM family (no torch types), shared by the
// torch bindings and the fused compute+collective kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace es {

enum Dtype : int { kDtypeBF16 = 0, kDtypeF16 = 1, kDtypeF32 = 2 };

// Activation applied in the epilogue before the store.  kActSiluDual (TMA-store
// epilogue of the wide kernel only): the pre-activation goes to a second
// output and its SiLU to the output, in one pass over the accumulator.
enum EpiAct : int { kActNone = 0, kActSilu = 1, kActSiluDual = 2 };

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
// C = silu(A @ B) and pre = A @ B (same shape as C, row pitch ld_pre) in one
// launch of the wide kernel; cudaErrorNotSupported when the shapes or layouts
// do not allow it (nothing is launched).
int gemm_launch_silu_dual(const GemmArgs& g, void* pre, long long ld_pre, long long pre_batch_stride,
                          cudaStream_t stream);
struct GemmShape;
GemmShape make_shape(const GemmArgs& g);
GemmShape make_shape_pair(const GemmArgs& g);
// Output tensor map of the TMA-store epilogues; false (map zeroed) when C does not qualify.
bool make_output_map(const GemmArgs& g, bool trans, CUtensorMap* mc);

// Stream-K tail on the wide 2-SM kernel (batch 1): pair tiles [0, sk_first)
// run whole, one per cluster; the K blocks of the other tail_tiles are split
// evenly over the remaining clusters, whose fp32 partials are reduce-added into
// a workspace of gemm_streamk_ws_elems floats and converted (with the
// activation) into C by a finishing pass.
struct StreamKPlan {
  int sk_first = 0;    // whole pair tiles
  int sk_iters = 0;    // K blocks per tail cluster
  int tail_tiles = 0;  // pair tiles split over the tail clusters
  int clusters = 0;    // clusters launched (whole + tail)
};
// mode -1: split only the partial last wave of long-K GEMMs (default);
// 1: split every tile; 0: never.  False when whole tiles are used.
bool gemm_streamk_plan(const GemmArgs& g, int mode, StreamKPlan* plan);
long long gemm_streamk_ws_elems(const StreamKPlan& plan);
int gemm_launch_streamk(const GemmArgs& g, const StreamKPlan& plan, float* ws, cudaStream_t stream);

// Host-side plan of a GEMM call (no launch): the kernel run_gemm would use
// (0 1-SM, 1 2-SM, 2 wide), operands swapped for a narrow N, wide-grid
// persistence and the stream-K tail.  For tests and diagnostics.
struct GemmPlanInfo {
  int kernel = 0, swapped = 0, persistent = 0;
  int sk_first = 0, sk_iters = 0, tail_tiles = 0, clusters = 0;
};
GemmPlanInfo gemm_plan_info(const GemmArgs& g, int streamk_mode);

// The wide kernel's work for a GEMM (host walk of the device schedule, for
// tests): per launch and cluster, each segment's pair tile, its CTA-0 tile
// origin and K-block range.
struct GemmSegment {
  int launch, cluster, pair_tile, m0, n0, kb0, kb1;
};
std::vector<GemmSegment> gemm_wide_schedule(const GemmArgs& g, int streamk_mode);

}  // namespace es
