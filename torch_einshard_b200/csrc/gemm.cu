// Launchers for the tcgen05 GEMM (plain store epilogue, optional SiLU).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gemm.h"
#include "gemm_tc.cuh"
#include "gemm_tc2.cuh"
#include "gemm_tc3.cuh"
#include "tma_desc.h"

#include <string.h>

namespace es {

static CUtensorMapDataType tma_dtype(int dtype) {
  return dtype == kDtypeBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// 0: 1-SM 128x256 kernel, 1: 2-SM 256x256, 2: wide 2-SM 256x512.
int pick_kernel(const GemmArgs& g) {
  if (g.pair >= 0) return g.pair;
  // Measured on B200 under the 1 kW cap (sustained, TP-MLP shapes): the wide
  // kernel beats the 1-SM kernel on every operand layout once there are enough
  // 256x512 pair tiles to give every SM pair work.  With fewer, the 256x256
  // pair kernel still fills the GPU when it has at least half as many pair
  // tiles as SM pairs (2048 x 2048 x 65536 weight gradient: 0.43 ms against
  // 0.49 ms on the 1-SM kernel); small problems keep the 1-SM kernel.
  const long long wide_tiles = static_cast<long long>((g.M + 255) / 256) * ((g.N + 511) / 512) * g.batch;
  const long long pair_tiles = static_cast<long long>((g.M + 255) / 256) * ((g.N + 255) / 256) * g.batch;
  if (wide_tiles >= g.num_sms / 2) return 2;
  if (2 * pair_tiles >= g.num_sms / 2 && g.M >= 256 && g.N >= 256 && g.K >= 16 * kBK) return 1;
  return 0;
}

bool use_pair_kernel(const GemmArgs& g) { return pick_kernel(g) >= 1; }

void make_operand_maps(const GemmArgs& g, CUtensorMap* ma, CUtensorMap* mb, bool pair) {
  const CUtensorMapDataType dt = tma_dtype(g.dtype);
  const uint64_t a_d0 = g.a_mn ? g.M : g.K;
  const uint64_t a_d1 = g.a_mn ? g.K : g.M;
  const uint64_t a_bs = g.batch > 1 ? g.a_batch_stride : g.lda * a_d1;
  *ma = make_tmap_3d(g.A, dt, 2, a_d0, a_d1, g.batch, g.lda, a_bs, 64, g.a_mn ? 64 : kBM);
  const uint64_t b_d0 = g.b_mn ? g.N : g.K;
  const uint64_t b_d1 = g.b_mn ? g.K : g.N;
  const uint64_t b_bs = g.batch > 1 ? g.b_batch_stride : g.ldb * b_d1;
  *mb = make_tmap_3d(g.B, dt, 2, b_d0, b_d1, g.batch, g.ldb, b_bs, 64, g.b_mn ? 64 : (pair ? kBN / 2 : kBN));
}

GemmShape make_shape(const GemmArgs& g) {
  GemmShape s;
  s.M = g.M;
  s.N = g.N;
  s.K = g.K;
  s.batch = g.batch;
  s.num_m = (g.M + kBM - 1) / kBM;
  s.num_n = (g.N + kBN - 1) / kBN;
  s.num_kb = (g.K + kBK - 1) / kBK;
  s.a_mn = g.a_mn;
  s.b_mn = g.b_mn;
  s.in_bf16 = g.dtype == kDtypeBF16 ? 1 : 0;
  s.group_m = g.group_m > 0 ? g.group_m : 16;
  s.pair = 0;
  s.split = 0;
  s.err = g.err;
  s.prof = g.prof;
  s.sleep_ns = g.sleep_ns;
  return s;
}

const char* check_gemm_args(const GemmArgs& g) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0 || g.batch <= 0) return "empty GEMM";
  if ((reinterpret_cast<uintptr_t>(g.A) & 15) || (reinterpret_cast<uintptr_t>(g.B) & 15))
    return "operand base not 16-byte aligned";
  if ((g.lda * 2) % 16 || (g.ldb * 2) % 16) return "operand row stride not a multiple of 16 bytes";
  if (g.batch > 1 && (((g.a_batch_stride * 2) % 16) || ((g.b_batch_stride * 2) % 16)))
    return "operand batch stride not a multiple of 16 bytes";
  return nullptr;
}

GemmShape make_shape_pair(const GemmArgs& g) {
  GemmShape s = make_shape(g);
  s.num_m = (g.M + 2 * kBM - 1) / (2 * kBM);
  s.group_m = g.group_m > 0 ? g.group_m : 8;
  s.pair = 1;
  return s;
}

// Launch a 2-SM kernel instantiation on clusters of two CTAs.
template <class Epi>
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const GemmShape& s,
                const Epi& epi, int num_sms, cudaStream_t stream) {
  auto kernel = gemm_tc2_kernel<Epi>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1ull)) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem2Bytes);
    cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    attr_set |= 1ull << dev;
  }
  const int pairs = s.num_m * s.num_n * s.batch;
  int clusters = num_sms / 2;
  if (pairs < clusters) clusters = pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem2Bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, ma, mb, mc, s, epi));
}

// C = A B computed as C^T = B^T A^T: operand roles and majorness swap, the
// epilogue stores transposed.  Used when N is narrower than a tile and M is
// larger, so the 256-wide N tile is not half empty.
static GemmArgs swapped(const GemmArgs& g) {
  GemmArgs t = g;
  t.A = g.B;
  t.B = g.A;
  t.M = g.N;
  t.N = g.M;
  t.a_mn = g.b_mn;  // B [N][K] K-major -> A' K-major; B [K][N] -> A' MN-major
  t.lda = g.ldb;
  t.a_batch_stride = g.b_batch_stride;
  t.b_mn = g.a_mn;
  t.ldb = g.lda;
  t.b_batch_stride = g.a_batch_stride;
  return t;
}

static bool want_swap(const GemmArgs& g) { return g.N < kBN && g.M > g.N; }

// Launch the wide 2-SM kernel (256 x 512 pair tiles) on clusters of two CTAs.
// Output map of the TMA-store epilogue (16-bit C, 16-byte aligned rows): 32 x 64
// boxes with 128-byte swizzle.  Returns false (map zeroed) when C does not qualify.
bool make_output_map(const GemmArgs& g, bool trans, CUtensorMap* mc) {
  memset(mc, 0, sizeof(*mc));
  const int out_bytes = g.out_dtype == kDtypeF32 ? 4 : 2;
  const bool ok = out_bytes == 2 && !trans && (reinterpret_cast<uintptr_t>(g.C) & 15) == 0 && (g.ldc * 2) % 16 == 0 &&
                  (g.batch == 1 || (g.c_batch_stride * 2) % 16 == 0);
  if (!ok) return false;
  const uint64_t dims[3] = {static_cast<uint64_t>(g.N), static_cast<uint64_t>(g.M), static_cast<uint64_t>(g.batch)};
  const uint64_t strides[2] = {static_cast<uint64_t>(g.ldc) * 2,
                               static_cast<uint64_t>(g.batch > 1 ? g.c_batch_stride : g.ldc * g.M) * 2};
  const uint32_t box[3] = {64, 32, 1};
  *mc = make_tmap_nd(g.C, g.out_dtype == kDtypeBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                     3, dims, strides, box);
  return true;
}

// Tile schedule of the wide kernel: 256 x 512 pair tiles, raster groups of 16.
static GemmShape wide_shape(const GemmArgs& g) {
  GemmShape s = make_shape(g);
  s.num_m = (g.M + 2 * kBM - 1) / (2 * kBM);
  s.num_n = (g.N + kBN3 - 1) / kBN3;
  s.group_m = g.group_m > 0 ? g.group_m : 16;
  s.pair = 1;
  s.split = g.split;
  return s;
}

// One pair tile per cluster (K > 2048 by default) or persistent clusters.
static bool wide_persistent(const GemmArgs& g) {
  return g.persistent > 0 || (g.persistent < 0 && (g.K + kBK - 1) / kBK <= 32);
}

// tile_limit > 0: only pair tiles [0, tile_limit) (the whole tiles before a stream-K tail).
// second: the map handed to the kernel in the stream-K workspace slot (the
// pre-activation output of the dual SiLU epilogue); zeroed when null.
template <class Epi>
int launch_wide(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, Epi epi, cudaStream_t stream,
                int tile_limit = 0, const CUtensorMap* second = nullptr) {
  CUtensorMap mc;
  epi.tma = make_output_map(g, epi.trans != 0, &mc) ? 1 : 0;
  GemmShape s = wide_shape(g);
  if (tile_limit > 0) s.split = 0;
  s.sk_first = tile_limit;
  auto kernel = gemm_tc3_kernel<Epi>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1ull)) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem3Bytes);
    attr_set |= 1ull << dev;
  }
  const int pairs = tile_limit > 0 ? tile_limit : s.num_m * s.num_n * s.batch;
  int clusters = g.num_sms / 2;
  // One pair tile per cluster held higher clocks under the power cap for long K;
  // with K <= 2048 the per-CTA setup and the unhidden pipeline fill dominate and
  // persistent clusters win (65536 x 2048 x 2048: 0.37 against 0.40 ms).
  if (pairs < clusters || !wide_persistent(g)) clusters = pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(kThreads3);
  cfg.dynamicSmemBytes = kSmem3Bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CUtensorMap mw;  // no stream-K workspace
  if (second != nullptr)
    mw = *second;
  else
    memset(&mw, 0, sizeof(mw));
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, ma, mb, mc, mw, s, epi, NoGather{}));
}

// C = silu(A @ B) and pre = A @ B from one pass over the accumulator (wide
// kernel, TMA-store epilogue).  cudaErrorNotSupported when the GEMM would not
// run on the wide kernel or an output does not qualify for TMA stores; the
// caller then runs the GEMM and the activation separately.
template <typename OutT>
static int launch_silu_dual(const GemmArgs& g, void* pre, long long ld_pre, long long pre_batch_stride,
                            cudaStream_t stream) {
  if (want_swap(g) || !use_pair_kernel(g) || pick_kernel(g) != 2) return static_cast<int>(cudaErrorNotSupported);
  GemmArgs gp = g;
  gp.C = pre;
  gp.ldc = ld_pre;
  gp.c_batch_stride = pre_batch_stride;
  CUtensorMap mpre, mc;
  if (!make_output_map(gp, false, &mpre) || !make_output_map(g, false, &mc))
    return static_cast<int>(cudaErrorNotSupported);
  CUtensorMap ma, mb;
  make_operand_maps(g, &ma, &mb, true);
  StoreEpilogue<OutT> epi;
  epi.C = reinterpret_cast<OutT*>(g.C);
  epi.ldc = g.ldc;
  epi.batch_stride = g.c_batch_stride;
  epi.act = kActSiluDual;
  epi.trans = 0;
  epi.tma = 1;
  epi.vec_ok = 1;
  return launch_wide(ma, mb, g, epi, stream, 0, &mpre);
}

int gemm_launch_silu_dual(const GemmArgs& g, void* pre, long long ld_pre, long long pre_batch_stride,
                          cudaStream_t stream) {
  if (g.out_dtype == kDtypeBF16) return launch_silu_dual<__nv_bfloat16>(g, pre, ld_pre, pre_batch_stride, stream);
  if (g.out_dtype == kDtypeF16) return launch_silu_dual<__half>(g, pre, ld_pre, pre_batch_stride, stream);
  return static_cast<int>(cudaErrorNotSupported);
}

template <typename OutT>
static int launch_store(const GemmArgs& g0, cudaStream_t stream) {
  const bool trans = want_swap(g0);
  const GemmArgs g = trans ? swapped(g0) : g0;
  const bool pair = use_pair_kernel(g);
  CUtensorMap ma, mb;
  make_operand_maps(g, &ma, &mb, pair);
  GemmShape s = pair ? make_shape_pair(g) : make_shape(g);
  StoreEpilogue<OutT> epi;
  epi.C = reinterpret_cast<OutT*>(g.C);
  epi.ldc = g.ldc;
  epi.batch_stride = g.c_batch_stride;
  epi.act = g.act;
  epi.trans = trans ? 1 : 0;
  epi.tma = 0;
  const int esz = sizeof(OutT);
  epi.vec_ok = ((reinterpret_cast<uintptr_t>(g.C) & 15) == 0) && ((g.ldc * esz) % 16 == 0) &&
               (g.batch == 1 || (g.c_batch_stride * esz) % 16 == 0);
  if (pair && pick_kernel(g) == 2) return launch_wide(ma, mb, g, epi, stream);
  if (pair) {
    CUtensorMap mc;
    epi.tma = make_output_map(g, trans, &mc) ? 1 : 0;
    return launch_pair(ma, mb, mc, s, epi, g.num_sms, stream);
  }
  auto kernel = gemm_tc_kernel<StoreEpilogue<OutT>>;
  static unsigned long long attr_set = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1ull)) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    attr_set |= 1ull << dev;
  }
  const int tiles = s.num_m * s.num_n * s.batch;
  const int grid = (tiles < g.num_sms || g.small_persistent == 0) ? tiles : g.num_sms;
  CUtensorMap mc;
  epi.tma = make_output_map(g, trans, &mc) ? 1 : 0;
  kernel<<<grid, kThreads, kSmemBytes, stream>>>(ma, mb, mc, s, epi, GemmLoads{});
  return static_cast<int>(cudaGetLastError());
}

// ------------------------------------------------------------------ stream-K tail

// Whole tiles (pair tile < sk_first) store through the plain TMA-store
// epilogue; tail segments add their fp32 partial into the workspace
// [tail tile][256][512]: the warp's 32 rows x 256 columns as eight 32 x 32
// boxes (128-byte rows, 128-byte swizzle), one TMA reduce-add each (the sum
// happens at L2, so segments of one tile from different clusters need no
// ordering).
template <typename OutT>
struct StreamKEpilogue {
  StoreEpilogue<OutT> store;
  int sk_first;
  __device__ __forceinline__ void setup(int*, const GemmShape&) {}
  __device__ __forceinline__ void finish(const GemmShape&, volatile int*) {}
  __device__ __forceinline__ bool tile(const EpiTile& et, const GemmShape& s, volatile int* abort_flag) {
    const int p = et.t >> 1;
    if (p < sk_first) return store.tile(et, s, abort_flag);
    const int x0 = et.c.n0 & (kBN3 - 1);          // column inside the 512-wide pair tile
    const int y0 = (et.c.m0 & (2 * kBM - 1)) + et.q * 32;  // row inside the 256-row pair tile
    uint4* stage = reinterpret_cast<uint4*>(et.stage);
#pragma unroll 1
    for (int sub = 0; sub < kBN / 32; ++sub) {
      uint32_t r[32];
      tmem_ld32(et.tmem + sub * 32, r);
      tmem_ld_wait();
      if (et.lane == 0) bulk_wait_group_read<0>();  // the previous box has left the staging buffer
      __syncwarp();
      const int sw = et.lane & 7;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        stage[et.lane * 8 + (j ^ sw)] = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (et.lane == 0) {
        tma_reduce_add_3d(et.tmw, et.stage, x0 + sub * 32, y0, p - sk_first);
        bulk_commit_group();
      }
    }
    return true;
  }
};

// C[tail tile] = act(workspace tile), converted to the output type.  Block
// (q, r): tail tile q, rows 16 r .. 16 r + 15; one thread per 4 columns.
template <typename OutT>
__global__ void streamk_finish_kernel(const float* __restrict__ ws, OutT* __restrict__ C, long long ldc,
                                      const GemmShape s, int act) {
  const int q = blockIdx.x;
  const TileCoord c = tile_coord3(s, s.sk_first + q, 0);
  const float* tile = ws + static_cast<long long>(q) * (2 * kBM) * kBN3;
  for (int i = threadIdx.x; i < 16 * (kBN3 / 4); i += blockDim.x) {
    const int r = blockIdx.y * 16 + i / (kBN3 / 4);
    const int col = (i % (kBN3 / 4)) * 4;
    const int row = c.m0 + r;
    if (row >= s.M || c.n0 + col >= s.N) continue;
    const float4 v = *reinterpret_cast<const float4*>(tile + r * kBN3 + col);
    const float f[4] = {v.x, v.y, v.z, v.w};
    OutT* dst = C + row * ldc + c.n0 + col;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (c.n0 + col + j >= s.N) break;
      StoreOut<OutT>::store1(dst + j, act == kActSilu ? silu_f(f[j]) : f[j]);
    }
  }
}

bool gemm_streamk_plan(const GemmArgs& g, int mode, StreamKPlan* plan) {
  // On request (mode 1) every tile is split; by default (mode -1) only the
  // partial last wave of a long-K GEMM, when the SM pairs it leaves idle cost
  // more than the tail's fp32 round trip.  Measured on B200: splitting all
  // tiles of 8192 x 2048 x 65536 took 1.91 ms against 1.43 ms in whole tiles
  // (each segment's fp32 reduce-adds, about 3.3 TB/s over the GPU, are not
  // hidden behind MMAs with the single-buffered wide accumulator), so the full
  // waves stay whole tiles.
  if (mode == 0 || g.batch != 1 || g.M < 2 * kBM || g.N < kBN3 || g.num_sms < 2) return false;
  const long long pair_tiles = static_cast<long long>((g.M + 2 * kBM - 1) / (2 * kBM)) * ((g.N + kBN3 - 1) / kBN3);
  const long long nkb = (g.K + kBK - 1) / kBK;
  const long long clusters = g.num_sms / 2;
  long long whole = 0;
  if (mode < 0) {
    const long long tail = pair_tiles % clusters;
    // whole waves first; an idle SM pair in the last wave loses a tile's worth of
    // K blocks, a tail segment costs about 60 blocks of reduce-add and finish
    // Worth it only for a small remainder: 224 tiles at tp = 8, 2 left over:
    // 1.17-1.19 ms against 1.41 ms whole; 1792 tiles, 16 left over: 11.2-12.2
    // against 11.0-11.2 ms; 128 tiles, 54 left over: 1.58 against 1.40 ms (the
    // tail segments read K ranges no other running cluster shares).
    if (pair_tiles < clusters || tail == 0 || nkb <= 32 || 9 * tail > clusters) return false;
    if (static_cast<double>(clusters - tail) / clusters * nkb < 60.0) return false;
    whole = pair_tiles - tail;
  }
  if ((pair_tiles - whole) * (2 * kBM) * kBN3 * 4 > (1LL << 30)) return false;  // workspace above 1 GiB
  const long long work = (pair_tiles - whole) * nkb;
  const long long per = (work + clusters - 1) / clusters;
  if (per <= 0 || per > 0x7fffffffLL) return false;
  plan->sk_first = static_cast<int>(whole);
  plan->sk_iters = static_cast<int>(per);
  plan->tail_tiles = static_cast<int>(pair_tiles - whole);
  plan->clusters = static_cast<int>(whole + (work + per - 1) / per);
  return true;
}

long long gemm_streamk_ws_elems(const StreamKPlan& plan) {
  return static_cast<long long>(plan.tail_tiles) * (2 * kBM) * kBN3;
}

template <typename OutT>
static int launch_streamk(const GemmArgs& g, const StreamKPlan& plan, float* ws, cudaStream_t stream) {
  CUtensorMap ma, mb, mc, mw;
  make_operand_maps(g, &ma, &mb, true);
  GemmShape s = wide_shape(g);
  s.split = 0;
  s.sk_iters = plan.sk_iters;
  s.sk_first = plan.sk_first;
  StreamKEpilogue<OutT> epi;
  epi.sk_first = plan.sk_first;
  epi.store.C = reinterpret_cast<OutT*>(g.C);
  epi.store.ldc = g.ldc;
  epi.store.batch_stride = g.c_batch_stride;
  epi.store.act = g.act;
  epi.store.trans = 0;
  const int esz = sizeof(OutT);
  epi.store.vec_ok = ((reinterpret_cast<uintptr_t>(g.C) & 15) == 0) && ((g.ldc * esz) % 16 == 0);
  epi.store.tma = make_output_map(g, false, &mc) ? 1 : 0;
  const uint64_t wdims[3] = {static_cast<uint64_t>(kBN3), static_cast<uint64_t>(2 * kBM),
                             static_cast<uint64_t>(plan.tail_tiles)};
  const uint64_t wstrides[2] = {static_cast<uint64_t>(kBN3) * 4, static_cast<uint64_t>(2 * kBM) * kBN3 * 4};
  const uint32_t wbox[3] = {32, 32, 1};
  mw = make_tmap_nd(ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, wdims, wstrides, wbox);
  cudaError_t e = cudaMemsetAsync(ws, 0, static_cast<size_t>(gemm_streamk_ws_elems(plan)) * sizeof(float), stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  auto kernel = gemm_tc3_kernel<StreamKEpilogue<OutT>>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1ull)) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem3Bytes);
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * plan.clusters);
  cfg.blockDim = dim3(kThreads3);
  cfg.dynamicSmemBytes = kSmem3Bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (plan.sk_first > 0) {
    // the full waves: the plain wide kernel on the first sk_first tiles
    const int rc = launch_wide(ma, mb, g, epi.store, stream, plan.sk_first);
    if (rc != 0) return rc;
  }
  s.sk_cluster0 = plan.sk_first;
  cfg.gridDim = dim3(2 * (plan.clusters - plan.sk_first));
  e = cudaLaunchKernelEx(&cfg, kernel, ma, mb, mc, mw, s, epi, NoGather{});
  if (e != cudaSuccess) return static_cast<int>(e);
  streamk_finish_kernel<OutT><<<dim3(plan.tail_tiles, (2 * kBM) / 16), 256, 0, stream>>>(
      ws, reinterpret_cast<OutT*>(g.C), g.ldc, s, g.act);
  return static_cast<int>(cudaGetLastError());
}

int gemm_launch_streamk(const GemmArgs& g, const StreamKPlan& plan, float* ws, cudaStream_t stream) {
  if (check_gemm_args(g) || plan.sk_iters <= 0 || plan.tail_tiles <= 0 || g.batch != 1) return -1;
  if ((reinterpret_cast<uintptr_t>(ws) & 15) != 0) return -2;
  if (plan.clusters - plan.sk_first > g.num_sms / 2) return -3;
  switch (g.out_dtype) {
    case kDtypeBF16:
      return launch_streamk<__nv_bfloat16>(g, plan, ws, stream);
    case kDtypeF16:
      return launch_streamk<__half>(g, plan, ws, stream);
    default:
      return launch_streamk<float>(g, plan, ws, stream);
  }
}

GemmPlanInfo gemm_plan_info(const GemmArgs& g0, int streamk_mode) {
  GemmPlanInfo info;
  info.swapped = want_swap(g0) ? 1 : 0;
  const GemmArgs g = info.swapped ? swapped(g0) : g0;
  StreamKPlan plan;
  if ((g0.pair < 0 || streamk_mode > 0) && gemm_streamk_plan(g0, streamk_mode, &plan)) {
    info.kernel = 2;
    info.swapped = 0;
    info.sk_first = plan.sk_first;
    info.sk_iters = plan.sk_iters;
    info.tail_tiles = plan.tail_tiles;
    info.clusters = plan.clusters;
    return info;
  }
  info.kernel = pick_kernel(g);
  if (info.kernel == 2) info.persistent = wide_persistent(g) ? 1 : 0;
  return info;
}

std::vector<GemmSegment> gemm_wide_schedule(const GemmArgs& g, int streamk_mode) {
  std::vector<GemmSegment> out;
  StreamKPlan plan;
  const bool sk = g.pair < 0 && gemm_streamk_plan(g, streamk_mode, &plan);
  GemmShape s = wide_shape(g);
  const int pairs = s.num_m * s.num_n * s.batch;
  auto walk = [&](const GemmShape& sh, int launch, int clusters) {
    for (int cl = 0; cl < clusters; ++cl) {
      SegIter it = seg_begin(sh, cl);
      TileCoord c;
      int p, k0, k1;
      while (seg_next(sh, cl, clusters, 0, it, &c, &p, &k0, &k1)) out.push_back({launch, cl, p, c.m0, c.n0, k0, k1});
    }
  };
  if (sk) {
    GemmShape whole = s;
    whole.split = 0;
    whole.sk_first = plan.sk_first;
    if (plan.sk_first > 0) walk(whole, 0, plan.sk_first);  // the plain launch, one tile per cluster
    GemmShape tail = s;
    tail.split = 0;
    tail.sk_iters = plan.sk_iters;
    tail.sk_first = plan.sk_first;
    tail.sk_cluster0 = plan.sk_first;
    walk(tail, 1, plan.clusters - plan.sk_first);
  } else {
    int clusters = g.num_sms / 2;
    if (pairs < clusters || !wide_persistent(g)) clusters = pairs;
    walk(s, 0, clusters);
  }
  return out;
}

int gemm_launch(const GemmArgs& g, cudaStream_t stream) {
  if (check_gemm_args(g)) return -1;
  switch (g.out_dtype) {
    case kDtypeBF16:
      return launch_store<__nv_bfloat16>(g, stream);
    case kDtypeF16:
      return launch_store<__half>(g, stream);
    case kDtypeF32:
      return launch_store<float>(g, stream);
    default:
      return -1;
  }
}

}  // namespace es
