// All-gather -> GEMM in one kernel (the wide 2-SM tcgen05 GEMM with a copy warp).
//
//   C = gather_rows(A_0, ..., A_{P-1}) @ B      (Megatron sequence parallelism)
//
// Rows of A form `segments` segments of P * shard rows; rank p holds rows
// [p * shard, (p + 1) * shard) of every segment in its symmetric data region
// ([segments][shard][K], staged by the caller).  Every CTA of the persistent
// GEMM has one extra warp that pulls 128-row chunks of A from their owner's
// region over NVLink into a local buffer (`xfull`, the gathered A, which the
// backward pass reuses) and then releases a per-chunk flag.  The TMA producer
// waits (bounded) for a chunk's flag before it loads those rows, so the
// transfer of later chunks overlaps the MMAs of earlier tiles.  M tiles and
// chunks are both visited local-rows-first, then rank+1, rank+2, ...: the first
// tiles never wait and the copy order matches the order tiles need their rows.
//
// Flags: peers' `staged` >= epoch before a chunk of theirs is read; per-chunk
// flags in this rank's flag region; `done` = epoch once every CTA finished (so
// peers may overwrite their regions).  All waits are bounded.
#include <cuda_bf16.h>
#include <string.h>

#include "comm.h"
#include "gemm.h"
#include "gemm_tc3.cuh"
#include "tma_desc.h"

namespace es {

constexpr int kFlagAg0 = kFlagTile0 + 2 * kMaxTiles;  // per-chunk flags of the gathered A
constexpr int kAgMaxChunks = static_cast<int>(kFlagBytes / 4) - kFlagAg0;

struct AgGather {
  static constexpr int kCopyWarps = 1;
  CommDev c;
  uint8_t* xfull;      // local gathered A [segments * P * shard][K] (bf16)
  long long row_bytes; // K * 2
  int segments;
  int shard_blocks;    // shard / 256 (pair blocks per shard)
  int nchunks;         // rows / 128

  __device__ __forceinline__ int* flag(int rank, int slot) const { return reinterpret_cast<int*>(c.flags[rank]) + slot; }

  // virtual pair block vb -> physical pair block: local shard first, then rank + 1, ...
  __host__ __device__ __forceinline__ int map_block(int vb, int blocks_per_shard) const {
    const int per_offset = segments * blocks_per_shard;
    const int o = vb / per_offset;
    const int r = vb - o * per_offset;
    const int g = r / blocks_per_shard;
    const int j = r - g * blocks_per_shard;
    const int q = (c.rank + o) % c.size;
    return (g * c.size + q) * blocks_per_shard + j;
  }
  __host__ __device__ __forceinline__ int map_m0(int m0) const {
    const int vb = m0 >> 8;
    return (map_block(vb, shard_blocks) << 8) + (m0 & 255);
  }
  __device__ __forceinline__ bool wait_rows(int m0, volatile int* abort_flag) const {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
      ok = wait_flag_geq_for(flag(c.rank, kFlagAg0 + (m0 >> 7)), c.epoch, c.err, kErrWaitPeerFlag, c.timeout_ns) ? 1 : 0;
      fence_proxy_async_global();  // the TMA (async proxy) reads rows written by the copy warps
      if (!ok) *abort_flag = 1;
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
  }
  // CTA 0: this rank's shard is staged (the copy before the kernel has finished)
  __device__ __forceinline__ void start() const {
    fence_acq_rel_sys();
    st_release_sys(flag(c.rank, kFlagStaged), c.epoch);
  }

  __device__ void copy(int cta, int ncta, volatile int* abort_flag) const {
    const int lane = threadIdx.x & 31;
    const int chunks_per_shard = shard_blocks * 2;
    const int per_offset = segments * chunks_per_shard;
    uint32_t staged_peers = 0;  // bit p: peer p's staged flag already seen
    for (int v = cta; v < nchunks; v += ncta) {
      if (*abort_flag) return;
      const int o = v / per_offset;
      const int r = v - o * per_offset;
      const int g = r / chunks_per_shard;
      const int j = r - g * chunks_per_shard;
      const int q = (c.rank + o) % c.size;
      if (!(staged_peers >> q & 1u)) {
        int ok = 1;
        if (lane == 0) ok = wait_flag_geq_for(flag(q, kFlagStaged), c.epoch, c.err, kErrWaitPeerFlag, c.timeout_ns) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, ok, 0)) {
          *abort_flag = 1;
          return;
        }
        staged_peers |= 1u << q;
      }
      const long long src_row = static_cast<long long>(g) * (chunks_per_shard * 128) + static_cast<long long>(j) * 128;
      const long long dst_chunk = (static_cast<long long>(g) * c.size + q) * chunks_per_shard + j;
      const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(c.data[q]) + src_row * row_bytes);
      uint4* dst = reinterpret_cast<uint4*>(xfull + dst_chunk * 128 * row_bytes);
      const long long n16 = 128 * row_bytes / 16;
      constexpr int kUnroll = 16;
      long long i = lane;
      for (; i + (kUnroll - 1) * 32 < n16; i += kUnroll * 32) {
        uint4 t[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) t[u] = src[i + u * 32];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) dst[i + u * 32] = t[u];
      }
      for (; i < n16; i += 32) dst[i] = src[i];
      fence_proxy_async_global();
      __syncwarp();
      if (lane == 0) {
        __threadfence();
        st_release_gpu(flag(c.rank, kFlagAg0 + static_cast<int>(dst_chunk)), c.epoch);
      }
    }
  }

  // thread 0 of every CTA: the last CTA of this rank publishes done
  __device__ void finish(bool ok) const {
    fence_acq_rel_sys();
    const int prev = atomicAdd(flag(c.rank, kFlagArrive), 1);
    if (static_cast<uint32_t>(prev + 1) - c.arrive_base == gridDim.x && ok) {
      fence_acq_rel_sys();
      st_release_sys(flag(c.rank, kFlagDone), c.epoch);
    }
  }
};

std::vector<int> gemm_allgather_row_order(int rank, int size, int segments, long long shard) {
  AgGather ag;
  memset(&ag, 0, sizeof(ag));
  ag.c.rank = rank;
  ag.c.size = size;
  ag.segments = segments;
  ag.shard_blocks = static_cast<int>(shard / 256);
  std::vector<int> out;
  const long long rows = static_cast<long long>(segments) * size * shard;
  for (long long m0 = 0; m0 < rows; m0 += 256) out.push_back(ag.map_m0(static_cast<int>(m0)));
  return out;
}

int gemm_allgather_grid(const GemmArgs& g) {
  const long long pair_tiles = static_cast<long long>((g.M + 255) / 256) * ((g.N + 511) / 512);
  const int clusters = pair_tiles < g.num_sms / 2 ? static_cast<int>(pair_tiles) : g.num_sms / 2;
  return 2 * clusters;
}

// g: the GEMM over the gathered rows (A = xfull, M = all rows).  Requires
// shard % 256 == 0, K * 2 % 16 == 0, bf16 in and out, batch 1.
int gemm_allgather_launch(const GemmArgs& g, const CommDev& comm, void* xfull, int segments, long long shard,
                          cudaStream_t stream) {
  if (check_gemm_args(g)) return -1;
  if (g.batch != 1 || g.a_mn || shard % 256 || (g.K * 2) % 16 || segments <= 0) return -2;
  if (static_cast<long long>(segments) * comm.size * shard != g.M) return -3;
  const int nchunks = g.M / 128;
  if (nchunks > kAgMaxChunks) return -4;
  CUtensorMap ma, mb, mc;
  make_operand_maps(g, &ma, &mb, true);
  GemmShape s = make_shape(g);
  s.num_m = (g.M + 2 * kBM - 1) / (2 * kBM);
  s.num_n = (g.N + kBN3 - 1) / kBN3;
  s.group_m = g.group_m > 0 ? g.group_m : 16;
  s.pair = 1;
  s.split = 0;
  StoreEpilogue<__nv_bfloat16> epi;
  epi.C = reinterpret_cast<__nv_bfloat16*>(g.C);
  epi.ldc = g.ldc;
  epi.batch_stride = g.c_batch_stride;
  epi.act = g.act;
  epi.trans = 0;
  epi.vec_ok = ((reinterpret_cast<uintptr_t>(g.C) & 15) == 0) && ((g.ldc * 2) % 16 == 0);
  epi.tma = make_output_map(g, false, &mc) ? 1 : 0;
  AgGather ag;
  ag.c = comm;
  ag.xfull = static_cast<uint8_t*>(xfull);
  ag.row_bytes = static_cast<long long>(g.K) * 2;
  ag.segments = segments;
  ag.shard_blocks = static_cast<int>(shard / 256);
  ag.nchunks = nchunks;
  auto kernel = gemm_tc3_kernel<StoreEpilogue<__nv_bfloat16>, AgGather>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1ull)) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem3Bytes);
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gemm_allgather_grid(g));
  cfg.blockDim = dim3(kThreads3 + 32 * AgGather::kCopyWarps);
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
  memset(&mw, 0, sizeof(mw));
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, ma, mb, mc, mw, s, epi, ag));
}

}  // namespace es
