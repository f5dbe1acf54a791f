// GEMM fused with an all-reduce of its output over NVLink (one cooperative kernel).
//
//   C = sum over ranks of (A_r @ B_r)      every rank gets the full C
//
// The tcgen05 mainloop of gemm_tc.cuh computes this rank's partial tile into
// TMEM.  Tile t is owned by rank t % P:
//   * non-owners store their bf16 partial tile into their own symmetric buffer
//     (chunk-interleaved so that a warp's NVLink reads are contiguous) and set
//     partial[t] = epoch in their flag region;
//   * the owner waits for partial[t] of every peer, sums the peers' partials with
//     its own fp32 accumulator read straight from TMEM, writes C's tile locally
//     and a reduced copy into its buffer, then sets reduced[t] = epoch;
//   * non-owners keep tile t in a small queue and, between later tiles (and at
//     the end), copy the owner's reduced tile into their own C.
// Only reads cross NVLink; every rank writes only its own memory.  The epoch
// protocol of comm.h makes buffer reuse across calls safe; every wait is bounded.
#include <cuda_bf16.h>
#include <string.h>

#include "comm.h"
#include "gemm.h"
#include "gemm_tc.cuh"
#include "gemm_ar.h"

namespace es {


constexpr int kTileBytes = kBM * kBN * 2;  // bf16 partial / reduced tile
constexpr int kQueue = 8;                  // pending pulls per CTA
// epilogue scratch slots in SharedState::epi
constexpr int kQHead = 0, kQTail = 1, kDecision = 2, kAbortEpi = 3, kQBase = 8;

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// element k (0..7) of eight packed bf16 values, without taking the vector's address
__device__ __forceinline__ __nv_bfloat16 bf16_at(const uint4& v, int k) {
  const uint32_t w = (k >> 1) == 0 ? v.x : (k >> 1) == 1 ? v.y : (k >> 1) == 2 ? v.z : v.w;
  return __ushort_as_bfloat16(static_cast<unsigned short>((k & 1) ? (w >> 16) : (w & 0xffffu)));
}

struct ArEpilogue {
  CommDev c;
  __nv_bfloat16* C;
  long long ldc;
  int vec_ok;  // C rows 16-byte aligned
  int* sm;     // SharedState::epi
  // Reduce-scatter mode (rs = 1): rows form segments of `seg` rows, each split
  // into size blocks of `shard` rows; rank p owns block p of every segment and
  // C is its local [segments * shard, N] output.  Tile t's owner is the owner
  // of its rows; nobody pulls reduced tiles back.
  int rs;
  long long seg, shard;

  __device__ __forceinline__ int owner_of(int t, const GemmShape& s) const {
    if (!rs) return t % c.size;
    const long long m0 = tile_coord(s, t).m0;
    return static_cast<int>((m0 % seg) / shard);
  }
  // row of this rank's C that holds global row `row`
  __device__ __forceinline__ long long out_row(long long row) const {
    if (!rs) return row;
    return (row / seg) * shard + (row % seg) - static_cast<long long>(c.rank) * shard;
  }

  __device__ __forceinline__ int* flag(int rank, int slot) const { return reinterpret_cast<int*>(c.flags[rank]) + slot; }
  __device__ __forceinline__ uint8_t* tile_buf(int rank, int t) const {
    return reinterpret_cast<uint8_t*>(c.data[rank]) + static_cast<size_t>(t) * kTileBytes;
  }

  __device__ void setup(int* scratch, const GemmShape&) {
    sm = scratch;
    // peers must be done reading our buffer from the previous operation
    if (threadIdx.x == 64) {
      for (int p = 0; p < c.size; ++p) {
        if (p == c.rank) continue;
        if (!wait_flag_geq_for(flag(p, kFlagDone), c.epoch - 1, c.err, kErrWaitPeerFlag, c.timeout_ns)) {
          sm[kAbortEpi] = 1;
          break;
        }
      }
    }
  }

  // copy the reduced tile t (owner o) into this rank's C.  The 16 loads of a
  // batch are issued before any store (the tile buffer is always whole, only the
  // stores are guarded), so a thread keeps 16 NVLink reads in flight.
  __device__ void pull_tile(int t, const GemmShape& s, int row_in_tile) {
    const TileCoord tc = tile_coord(s, t);
    const int row = tc.m0 + row_in_tile;
    const uint8_t* src = tile_buf(t % c.size, t);
    const bool row_ok = row < s.M;
    __nv_bfloat16* crow = C + static_cast<long long>(row_ok ? row : 0) * ldc;
    constexpr int kBatch = 16;
#pragma unroll 1
    for (int j0 = 0; j0 < kBN / 8; j0 += kBatch) {
      if (tc.n0 + j0 * 8 >= s.N) break;  // uniform across the epilogue threads
      uint4 v[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        v[u] = *reinterpret_cast<const uint4*>(src + (static_cast<size_t>(j0 + u) * kBM + row_in_tile) * 16);
      if (!row_ok) continue;
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int col = tc.n0 + (j0 + u) * 8;
        if (col >= s.N) break;
        if (col + 8 <= s.N && vec_ok) {
          *reinterpret_cast<uint4*>(crow + col) = v[u];
        } else {
          for (int k = 0; k < 8 && col + k < s.N; ++k) crow[col + k] = bf16_at(v[u], k);
        }
      }
    }
  }

  // Service the pull queue.  blocking: wait (bounded) for the oldest entry.
  // Returns false when the kernel must abort.
  __device__ bool service(const GemmShape& s, int e, bool blocking, int max_items) {
    for (int done = 0; done < max_items; ++done) {
      if (e == 0) {
        int decision = -1;
        if (sm[kQHead] != sm[kQTail]) {
          const int t = sm[kQBase + (sm[kQHead] % kQueue)];
          const int* f = flag(t % c.size, kFlagTile0 + kMaxTiles + t);
          bool ready = ld_acquire_sys(f) >= c.epoch;
          if (!ready && blocking) {
            ready = wait_flag_geq_for(f, c.epoch, c.err, kErrWaitPeerFlag, c.timeout_ns);
            if (!ready) sm[kAbortEpi] = 1;
          }
          if (ready) decision = t;
        }
        sm[kDecision] = decision;
      }
      epi_bar();
      const int t = sm[kDecision];
      if (sm[kAbortEpi]) return false;
      if (t < 0) return true;
      pull_tile(t, s, e);
      epi_bar();
      if (e == 0) ++sm[kQHead];
    }
    return true;
  }

  __device__ bool tile(const EpiTile& et, const GemmShape& s, volatile int* abort_flag) {
    const int e = et.row;  // epilogue thread index == tile row
    const int t = et.t;
    if (sm[kAbortEpi]) return false;
    const int owner = owner_of(t, s);
    const bool mine = owner == c.rank;
    uint8_t* my_buf = tile_buf(c.rank, t);
    if (!mine) {
#pragma unroll 1
      for (int chunk = 0; chunk < kBN / 32; ++chunk) {
        uint32_t r[32];
        tmem_ld32(et.tmem + chunk * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint4 v = make_uint4(pack_bf16(__uint_as_float(r[8 * k + 0]), __uint_as_float(r[8 * k + 1])),
                                     pack_bf16(__uint_as_float(r[8 * k + 2]), __uint_as_float(r[8 * k + 3])),
                                     pack_bf16(__uint_as_float(r[8 * k + 4]), __uint_as_float(r[8 * k + 5])),
                                     pack_bf16(__uint_as_float(r[8 * k + 6]), __uint_as_float(r[8 * k + 7])));
          *reinterpret_cast<uint4*>(my_buf + (static_cast<size_t>(chunk * 4 + k) * kBM + e) * 16) = v;
        }
      }
      epi_bar();
      if (e == 0) {
        fence_acq_rel_sys();
        st_release_sys(flag(c.rank, kFlagTile0 + t), c.epoch);
        if (!rs) {
          // queue the pull of the reduced tile; make room first if the queue is full
          sm[kQBase + (sm[kQTail] % kQueue)] = t;
          ++sm[kQTail];
        }
      }
      epi_bar();
      const bool full = (sm[kQTail] - sm[kQHead]) >= kQueue;
      return service(s, e, full, full ? 1 : 2);
    }
    // owner: gather every peer's partial of tile t
    if (e == 0) {
      for (int p = 0; p < c.size; ++p) {
        if (p == c.rank) continue;
        if (!wait_flag_geq_for(flag(p, kFlagTile0 + t), c.epoch, c.err, kErrWaitPeerFlag, c.timeout_ns)) {
          sm[kAbortEpi] = 1;
          *abort_flag = 1;
          break;
        }
      }
    }
    epi_bar();
    if (sm[kAbortEpi]) return false;
    const int row = et.c.m0 + e;
    __nv_bfloat16* crow = C + out_row(row) * ldc;
#pragma unroll 1
    for (int chunk = 0; chunk < kBN / 32; ++chunk) {
      uint32_t r[32];
      tmem_ld32(et.tmem + chunk * 32, r);
      tmem_ld_wait();
      float acc[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(r[i]);
      // all peers' 4 x 16-byte pieces of this 32-column chunk are loaded before the sums
      uint4 v[4][kMaxRanks - 1];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const size_t off = (static_cast<size_t>(chunk * 4 + q) * kBM + e) * 16;
#pragma unroll
        for (int k = 1; k < kMaxRanks; ++k)
          if (k < c.size) v[q][k - 1] = *reinterpret_cast<const uint4*>(tile_buf((c.rank + k) % c.size, t) + off);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int k = 1; k < kMaxRanks; ++k) {
          if (k >= c.size) break;
          const uint32_t w[4] = {v[q][k - 1].x, v[q][k - 1].y, v[q][k - 1].z, v[q][k - 1].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // a bf16 pair widened exactly: each half is the upper 16 bits of an fp32
            acc[8 * q + 2 * j] += __uint_as_float(w[j] << 16);
            acc[8 * q + 2 * j + 1] += __uint_as_float(w[j] & 0xffff0000u);
          }
        }
      }
      uint4 o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        o[q] = make_uint4(pack_bf16(acc[8 * q + 0], acc[8 * q + 1]), pack_bf16(acc[8 * q + 2], acc[8 * q + 3]),
                          pack_bf16(acc[8 * q + 4], acc[8 * q + 5]), pack_bf16(acc[8 * q + 6], acc[8 * q + 7]));
        if (!rs) *reinterpret_cast<uint4*>(my_buf + (static_cast<size_t>(chunk * 4 + q) * kBM + e) * 16) = o[q];
      }
      const int col0 = et.c.n0 + chunk * 32;
      if (row < s.M && col0 < s.N) {
        if (col0 + 32 <= s.N && vec_ok) {
#pragma unroll
          for (int q = 0; q < 4; ++q) *reinterpret_cast<uint4*>(crow + col0 + 8 * q) = o[q];
        } else {
          for (int q = 0; q < 4; ++q)
            for (int k = 0; k < 8 && col0 + 8 * q + k < s.N; ++k) crow[col0 + 8 * q + k] = bf16_at(o[q], k);
        }
      }
    }
    epi_bar();
    if (e == 0 && !rs) {
      fence_acq_rel_sys();
      st_release_sys(flag(c.rank, kFlagTile0 + kMaxTiles + t), c.epoch);
    }
    return service(s, e, false, 2);
  }

  __device__ void finish(const GemmShape& s, volatile int* abort_flag) {
    const int e = threadIdx.x - 64;
    bool ok = !sm[kAbortEpi] && !*abort_flag;
    if (ok) {
      while (true) {
        epi_bar();
        if (sm[kQHead] == sm[kQTail]) break;
        if (!service(s, e, true, 1)) {
          ok = false;
          break;
        }
      }
    }
    epi_bar();
    if (e == 0) {
      // the last CTA of this rank to finish publishes done = epoch
      int* arrive = flag(c.rank, kFlagArrive);
      fence_acq_rel_sys();
      const int prev = atomicAdd(arrive, 1);
      if (prev + 1 - static_cast<int>(c.arrive_base) == static_cast<int>(gridDim.x) && ok) {
        fence_acq_rel_sys();
        st_release_sys(flag(c.rank, kFlagDone), c.epoch);
      }
    }
  }
};

int gemm_allreduce_launch(const GemmArgs& g, const CommDev& comm, cudaStream_t stream, long long rs_seg,
                          long long rs_shard) {
  if (check_gemm_args(g)) return -1;
  if (rs_seg > 0 && (rs_seg % kBM || rs_shard % kBM || rs_shard * comm.size != rs_seg || g.M % rs_seg)) return -4;
  if (g.out_dtype != kDtypeBF16 || g.batch != 1) return -2;
  CUtensorMap ma, mb;
  make_operand_maps(g, &ma, &mb);
  GemmShape s = make_shape(g);
  const int tiles = s.num_m * s.num_n;
  if (tiles > kMaxTiles) return -3;
  ArEpilogue epi;
  epi.c = comm;
  epi.C = reinterpret_cast<__nv_bfloat16*>(g.C);
  epi.ldc = g.ldc;
  epi.vec_ok = ((reinterpret_cast<uintptr_t>(g.C) & 15) == 0) && (g.ldc % 8 == 0);
  epi.sm = nullptr;
  epi.rs = rs_seg > 0 ? 1 : 0;
  epi.seg = rs_seg > 0 ? rs_seg : 1;
  epi.shard = rs_shard > 0 ? rs_shard : 1;
  auto kernel = gemm_tc_kernel<ArEpilogue>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1ull)) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    attr_set |= 1ull << dev;
  }
  const int grid = tiles < g.num_sms ? tiles : g.num_sms;
  GemmLoads loads{};
  CUtensorMap mc;
  memset(&mc, 0, sizeof(mc));  // the all-reduce epilogue stores without TMA
  void* args[] = {&ma, &mb, &mc, &s, &epi, &loads};
  return static_cast<int>(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kernel), dim3(grid),
                                                      dim3(kThreads), args, kSmemBytes, stream));
}

}  // namespace es
