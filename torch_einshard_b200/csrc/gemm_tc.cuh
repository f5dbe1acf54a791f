// Persistent warp-specialised tcgen05 GEMM mainloop for sm_100a.
//
//   C[b, m, n] = sum_k A[b, m, k] * B[b, k, n]      (bf16/fp16 in, fp32 accumulate)
//
// Tile 128 x 256 x 64, 4-stage TMA -> shared-memory pipeline, one UMMA
// (tcgen05.mma.cta_group::1, M=128 N=256 K=16) stream issued by a single
// thread, two TMEM accumulators (2 x 256 columns = all 512) so the epilogue of
// tile i overlaps the MMAs of tile i+1.  Either operand may be K-major or
// MN-major in global memory; the TMA boxes and the UMMA descriptors follow
// the 128-byte-swizzle canonical layouts:
//   K-major : rows of 64 elements (128 B), 8-row groups 1024 B apart (SBO)
//   MN-major: 64-element MN chunks 8 KB apart (LBO), 8-row K groups 1024 B apart (SBO)
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = MMA issuer and
// TMEM owner, warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31).
// The epilogue is a policy class so that fused variants (peer-memory
// all-reduce, activation) reuse the same mainloop.
//
// All waits are bounded (see ptx.cuh); on timeout the kernel records an error
// code, drains its own outstanding TMA loads and MMAs (bounded), frees TMEM and
// returns.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "gemm.h"
#include "ptx.cuh"

namespace es {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kUmmaK = 16;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kBBytes = kBN * kBK * 2;  // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kTmemCols = 512;
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kStageOut = 4096;  // per epilogue warp: staging buffer of the TMA-store epilogues
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*barriers*/ + 4 * kStageOut + 1024 /*alignment slack*/;

struct GemmShape {
  int M, N, K, batch;
  int num_m, num_n, num_kb;
  int a_mn, b_mn;  // operand majorness in global memory
  int in_bf16;
  int group_m;     // raster group height (M tiles) for L2 reuse
  int pair;        // 1: 2-SM kernel; tile t is half (t & 1) of 256-row pair tile t >> 1
  int split;       // wide kernel: 0 one tile sequence; 1/2 the clusters split in two sets (first/second
                   // half of the cluster ids, or even/odd ids), each walking one half of the M tiles
  int* err;
  unsigned long long* prof;  // optional: per-CTA wait-cycle counters (see gemm_tc3.cuh), null when off
  int sleep_ns;              // wide kernel: epilogue back-off between accumulator polls (0: spin)
  int sk_iters = 0;          // wide kernel: > 0 stream-K tail, K blocks per tail cluster (0: whole tiles only)
  int sk_first = 0;          // wide kernel: pair tiles [0, sk_first) whole, the rest split (with sk_iters);
                             // without sk_iters a nonzero sk_first limits the launch to those whole tiles
  int sk_cluster0 = 0;       // wide kernel, stream-K: cluster id of this launch's first cluster
};

struct TileCoord {
  int b, m0, n0;
};

template <typename T>
__host__ __device__ __forceinline__ T es_min(T a, T b) {
  return a < b ? a : b;
}

// Host-callable too: the host tests walk the same tile schedule.
__host__ __device__ __forceinline__ TileCoord tile_coord(const GemmShape& s, int t) {
  int half = 0;
  if (s.pair) {
    half = t & 1;
    t >>= 1;
  }
  const int per_batch = s.num_m * s.num_n;
  const int b = t / per_batch;
  const int r = t - b * per_batch;
  const int per_group = s.group_m * s.num_n;
  const int g = r / per_group;
  const int first_m = g * s.group_m;
  const int gm = es_min(s.num_m - first_m, s.group_m);
  const int in_group = r - g * per_group;
  const int mb = first_m + in_group % gm;
  const int nb = in_group / gm;
  return {b, mb * (s.pair ? 2 * kBM : kBM) + half * kBM, nb * kBN};
}

struct SharedState {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int consumed;  // k-iterations consumed by the MMA warp (for the producer's drain)
  int epi[32];   // scratch for the epilogue policy (its own queues and flags)
};

// Context handed to the epilogue policy for one tile.
struct EpiTile {
  TileCoord c;
  int t;          // linear tile index
  uint32_t tmem;  // TMEM address of this thread's lane quadrant and accumulator buffer
  int row;        // this thread's tile row (0..127)
  int q;          // lane quadrant of this warp
  int lane;
  const CUtensorMap* tmc = nullptr;  // output map for TMA stores (kernels that provide one)
  uint8_t* stage = nullptr;          // this warp's 4 KB staging buffer (1024-byte aligned)
  const CUtensorMap* tmw = nullptr;  // fp32 workspace map of stream-K partial tiles (wide kernel)
};

// Operand loads of one K block for the plain GEMM: A and B tiles by TMA from
// 3-D maps over [batch, rows, cols] (K-major: one box; MN-major: 64-wide boxes).
struct GemmLoads {
  __device__ __forceinline__ void load(const GemmShape& shp, const TileCoord& c, int kb, uint8_t* a, uint8_t* b,
                                       uint64_t* bar, const CUtensorMap* tmA, const CUtensorMap* tmB) const {
    const int k0 = kb * kBK;
    if (!shp.a_mn) {
      tma_load_3d(a, tmA, bar, k0, c.m0, c.b);
    } else {
      tma_load_3d(a, tmA, bar, c.m0, k0, c.b);
      tma_load_3d(a + 8192, tmA, bar, c.m0 + 64, k0, c.b);
    }
    if (!shp.b_mn) {
      tma_load_3d(b, tmB, bar, k0, c.n0, c.b);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) tma_load_3d(b + j * 8192, tmB, bar, c.n0 + 64 * j, k0, c.b);
    }
  }
};

template <class Epi, class Loads = GemmLoads>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const GemmShape shp, Epi epi, const Loads loads) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kABytes;
  SharedState* st = reinterpret_cast<SharedState*>(smem + kStages * kStageBytes);
  uint8_t* out_stage = smem + kStages * kStageBytes + 1024;  // 1024-byte aligned (TMA swizzle atom)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_tiles = shp.num_m * shp.num_n * shp.batch;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&st->full[s], 1);
      mbar_init(&st->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&st->tfull[a], 1);
      mbar_init(&st->tempty[a], kEpiThreads / 32);
    }
    mbar_init(&st->drain, 1);
    st->abort_flag = 0;
    st->consumed = 0;
    for (int i = 0; i < 32; ++i) st->epi[i] = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(&st->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = st->tmem_base;
  volatile int* abort_flag = &st->abort_flag;
  epi.setup(st->epi, shp);  // the policy's scratch words in shared memory

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    uint32_t it = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      const TileCoord c = tile_coord(shp, t);
      for (int kb = 0; kb < shp.num_kb; ++kb, ++it) {
        const int s = it % kStages;
        const uint32_t ph = (it / kStages) & 1u;
        if (!mbar_wait_lane0(&st->empty[s], ph ^ 1u, abort_flag, shp.err, kErrWaitEmpty)) goto producer_done;
        if (lane == 0) {
          mbar_arrive_expect_tx(&st->full[s], kStageBytes);
          loads.load(shp, c, kb, sA + s * kABytes, sB + s * kBBytes, &st->full[s], &tmA, &tmB);
        }
        __syncwarp();
      }
    }
  producer_done:
    __syncwarp();
    if (*abort_flag && lane == 0) {
      // drain: wait (bounded) for loads issued but never consumed
      const uint32_t consumed = static_cast<uint32_t>(*reinterpret_cast<volatile int*>(&st->consumed));
      for (uint32_t j = consumed; j < it; ++j) {
        int dummy_abort = 0;
        mbar_wait(&st->full[j % kStages], (j / kStages) & 1u, &dummy_abort, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = umma_idesc_f16(kBM, kBN, shp.in_bf16, shp.a_mn, shp.b_mn);
    // descriptor offsets: K-major advances 32 B per UMMA_K, MN-major 16 rows x 128 B
    const uint32_t a_lbo = shp.a_mn ? 8192u : 16u;
    const uint32_t b_lbo = shp.b_mn ? 8192u : 16u;
    const uint32_t a_kstep = shp.a_mn ? 2048u : 32u;
    const uint32_t b_kstep = shp.b_mn ? 2048u : 32u;
    uint32_t it = 0, tc = 0;
    bool issued_any = false;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++tc) {
      const uint32_t acc = tc & 1u;
      const uint32_t aph = (tc >> 1) & 1u;
      if (!mbar_wait_lane0(&st->tempty[acc], aph ^ 1u, abort_flag, shp.err, kErrWaitTmemEmpty)) goto mma_done;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * kBN;
      for (int kb = 0; kb < shp.num_kb; ++kb, ++it) {
        const int s = it % kStages;
        const uint32_t ph = (it / kStages) & 1u;
        if (!mbar_wait_lane0(&st->full[s], ph, abort_flag, shp.err, kErrWaitFull)) goto mma_done;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(sA + s * kABytes);
          const uint32_t b_addr = smem_u32(sB + s * kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            const uint64_t ad = umma_desc_sw128(a_addr + k * a_kstep, a_lbo, 1024u);
            const uint64_t bd = umma_desc_sw128(b_addr + k * b_kstep, b_lbo, 1024u);
            umma_f16(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&st->empty[s]);
          *reinterpret_cast<volatile int*>(&st->consumed) = static_cast<int>(it + 1);
        }
        issued_any = true;
        __syncwarp();
      }
      if (lane == 0) umma_commit(&st->tfull[acc]);
      __syncwarp();
    }
  mma_done:
    __syncwarp();
    if (*abort_flag && issued_any && lane == 0) {
      // make sure no MMA still writes TMEM before it is freed
      umma_commit(&st->drain);
      int dummy_abort = 0;
      mbar_wait(&st->drain, 0, &dummy_abort, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    uint32_t tc = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++tc) {
      const uint32_t acc = tc & 1u;
      const uint32_t ph = (tc >> 1) & 1u;
      if (!mbar_wait(&st->tfull[acc], ph, abort_flag, shp.err, kErrWaitTmemFull)) break;
      tc_fence_after();
      EpiTile et;
      et.c = tile_coord(shp, t);
      et.t = t;
      et.tmem = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kBN;
      et.row = q * 32 + lane;
      et.q = q;
      et.lane = lane;
      et.tmc = &tmC;
      et.stage = out_stage + q * kStageOut;
      const bool ok = epi.tile(et, shp, abort_flag);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&st->tempty[acc]);
      if (!ok) {
        *abort_flag = 1;
        break;
      }
    }
    epi.finish(shp, abort_flag);
    if (lane == 0) bulk_wait_group<0>();  // every TMA store of this warp has landed
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------- plain store epilogue
template <typename OutT>
struct StoreOut;
template <>
struct StoreOut<float> {
  static __device__ __forceinline__ void store32(float* p, const uint32_t (&r)[32], int base) {
    float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      q[i] = make_float4(__uint_as_float(r[base + 4 * i]), __uint_as_float(r[base + 4 * i + 1]),
                         __uint_as_float(r[base + 4 * i + 2]), __uint_as_float(r[base + 4 * i + 3]));
  }
  static __device__ __forceinline__ void store1(float* p, float v) { *p = v; }
  static __device__ __forceinline__ float cvt(float v) { return v; }
};
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
struct StoreOut<__nv_bfloat16> {
  static __device__ __forceinline__ void store32(__nv_bfloat16* p, const uint32_t (&r)[32], int) {
    uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      q[i] = make_uint4(pack_bf16(__uint_as_float(r[8 * i + 0]), __uint_as_float(r[8 * i + 1])),
                        pack_bf16(__uint_as_float(r[8 * i + 2]), __uint_as_float(r[8 * i + 3])),
                        pack_bf16(__uint_as_float(r[8 * i + 4]), __uint_as_float(r[8 * i + 5])),
                        pack_bf16(__uint_as_float(r[8 * i + 6]), __uint_as_float(r[8 * i + 7])));
  }
  static __device__ __forceinline__ void store1(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
  static __device__ __forceinline__ __nv_bfloat16 cvt(float v) { return __float2bfloat16_rn(v); }
};
template <>
struct StoreOut<__half> {
  static __device__ __forceinline__ void store32(__half* p, const uint32_t (&r)[32], int) {
    uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      q[i] = make_uint4(pack_f16(__uint_as_float(r[8 * i + 0]), __uint_as_float(r[8 * i + 1])),
                        pack_f16(__uint_as_float(r[8 * i + 2]), __uint_as_float(r[8 * i + 3])),
                        pack_f16(__uint_as_float(r[8 * i + 4]), __uint_as_float(r[8 * i + 5])),
                        pack_f16(__uint_as_float(r[8 * i + 6]), __uint_as_float(r[8 * i + 7])));
  }
  static __device__ __forceinline__ void store1(__half* p, float v) { *p = __float2half_rn(v); }
  static __device__ __forceinline__ __half cvt(float v) { return __float2half_rn(v); }
};

// Activation applied in the epilogue before the store: EpiAct (gemm.h).

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

template <typename OutT>
struct StoreEpilogue {
  OutT* C;
  long long ldc;
  long long batch_stride;
  int vec_ok;
  int act;
  int trans;  // 1: the kernel computes C^T (operands swapped); tile rows are columns of C
  int tma;    // 1: 16-bit output written by TMA stores through the warp's staging buffer

  __device__ __forceinline__ void setup(int*, const GemmShape&) {}
  __device__ __forceinline__ void finish(const GemmShape&, volatile int*) {}

  // 32 rows x 256 columns of this warp, as four 32 x 64 boxes: TMEM -> registers
  // (bf16/fp16) -> 128-byte-swizzled staging buffer -> one TMA store per box.
  // The stores are coalesced by the TMA engine and clipped at the tensor edges.
  __device__ __forceinline__ bool tile_tma(const EpiTile& et, const GemmShape& s) {
    const int row0 = et.c.m0 + et.q * 32;
#pragma unroll 1
    for (int sub = 0; sub < kBN / 64; ++sub) {
      const int col0 = et.c.n0 + sub * 64;
      if (col0 >= s.N) break;  // uniform across the warp
      uint32_t r0[32], r1[32];
      tmem_ld32(et.tmem + sub * 64, r0);
      tmem_ld32(et.tmem + sub * 64 + 32, r1);
      tmem_ld_wait();
      if (act == kActSiluDual) stage_box(et, r0, r1, et.tmw, col0, row0);  // the pre-activation
      if (act == kActSilu || act == kActSiluDual) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          r0[i] = __float_as_uint(silu_f(__uint_as_float(r0[i])));
          r1[i] = __float_as_uint(silu_f(__uint_as_float(r1[i])));
        }
      }
      stage_box(et, r0, r1, et.tmc, col0, row0);
    }
    return true;
  }

  // One 32 x 64 box of this warp (registers r0: columns 0-31, r1: 32-63) ->
  // 128-byte-swizzled staging buffer -> TMA store through `map`.
  __device__ __forceinline__ void stage_box(const EpiTile& et, const uint32_t (&r0)[32], const uint32_t (&r1)[32],
                                            const CUtensorMap* map, int col0, int row0) {
    uint4* stage = reinterpret_cast<uint4*>(et.stage);
    if (et.lane == 0) bulk_wait_group_read<0>();  // the previous box has left the staging buffer
    __syncwarp();
    const int sw = et.lane & 7;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t* src = j < 4 ? &r0[8 * j] : &r1[8 * (j - 4)];
      uint4 v;
      if (sizeof(OutT) == 2 && std::is_same<OutT, __half>::value) {
        v = make_uint4(pack_f16(__uint_as_float(src[0]), __uint_as_float(src[1])),
                       pack_f16(__uint_as_float(src[2]), __uint_as_float(src[3])),
                       pack_f16(__uint_as_float(src[4]), __uint_as_float(src[5])),
                       pack_f16(__uint_as_float(src[6]), __uint_as_float(src[7])));
      } else {
        v = make_uint4(pack_bf16(__uint_as_float(src[0]), __uint_as_float(src[1])),
                       pack_bf16(__uint_as_float(src[2]), __uint_as_float(src[3])),
                       pack_bf16(__uint_as_float(src[4]), __uint_as_float(src[5])),
                       pack_bf16(__uint_as_float(src[6]), __uint_as_float(src[7])));
      }
      stage[et.lane * 8 + (j ^ sw)] = v;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (et.lane == 0) {
      tma_store_3d(map, et.stage, col0, row0, et.c.b);
      bulk_commit_group();
    }
  }

  __device__ __forceinline__ bool tile(const EpiTile& et, const GemmShape& s, volatile int*) {
    if (tma && !trans && et.tmc != nullptr) return tile_tma(et, s);
    const int row = et.c.m0 + et.row;
    const bool row_ok = row < s.M;
    if (trans) {
      // lanes hold neighbouring columns of C: every store is 32 consecutive elements of one C row
      OutT* ccol = C + static_cast<long long>(et.c.b) * batch_stride + row;
#pragma unroll 1
      for (int chunk = 0; chunk < kBN / 32; ++chunk) {
        const int col0 = et.c.n0 + chunk * 32;
        if (col0 >= s.N) break;
        uint32_t r[32];
        tmem_ld32(et.tmem + chunk * 32, r);
        tmem_ld_wait();
        if (!row_ok) continue;
        const int valid = s.N - col0 < 32 ? s.N - col0 : 32;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float v = __uint_as_float(r[i]);
          if (act == kActSilu) v = silu_f(v);
          if (i < valid) StoreOut<OutT>::store1(ccol + static_cast<long long>(col0 + i) * ldc, v);
        }
      }
      return true;
    }
    OutT* crow = C + static_cast<long long>(et.c.b) * batch_stride + static_cast<long long>(row) * ldc;
#pragma unroll 1
    for (int chunk = 0; chunk < kBN / 32; ++chunk) {
      const int col0 = et.c.n0 + chunk * 32;
      if (col0 >= s.N) break;  // uniform across the warp
      uint32_t r[32];
      tmem_ld32(et.tmem + chunk * 32, r);
      tmem_ld_wait();
      if (act == kActSilu) {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(silu_f(__uint_as_float(r[i])));
      }
      if (!row_ok) continue;
      if (vec_ok && col0 + 32 <= s.N) {
        StoreOut<OutT>::store32(crow + col0, r, 0);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (col0 + i < s.N) StoreOut<OutT>::store1(crow + col0 + i, __uint_as_float(r[i]));
      }
    }
    return true;
  }
};

}  // namespace es
