// GEMM fused with an all-reduce of its output, push model, on the 2-SM
// (256 x 256 pair tile) tcgen05 kernel with its double-buffered accumulators,
// so a tile's NVLink pushes overlap the next tile's MMAs.
//
//   C = sum over ranks of (A_r @ B_r)        every rank gets the full C
//
// Sub-tile t (128 rows x 256 columns: one CTA's half of a pair tile, handled by
// a 4-warp epilogue group) is owned by rank t % P.  In the epilogue:
//   * a non-owner converts its fp32 accumulator to bf16 and STORES it straight
//     into its slot of the owner's symmetric region (NVLink writes do not wait
//     for a round trip), then releases a flag in the owner's flag region;
//   * the owner waits for the P-1 flags in its OWN flag region, sums the
//     partials from its own HBM with the accumulator read from TMEM, writes its
//     C and pushes the reduced bf16 tile into every peer's region + flag;
//   * a non-owner later copies reduced tiles from its own region into C
//     (between tiles, and the rest at the end).
// So the only NVLink traffic is stores, and every wait polls local memory
// (except the start-of-op check that peers finished the previous op).
// Slots use a row-interleaved layout (16-byte piece j of row r at (j*128 + r)*16)
// so a warp's stores are 512 contiguous bytes.  Waits are bounded.
#include <cuda_bf16.h>
#include <string.h>

#include "comm.h"
#include "gemm.h"
#include "gemm_ar.h"
#include "gemm_tc2.cuh"
#include "tma_desc.h"

namespace es {

namespace {

constexpr int kSubBytes = kBM * kBN * 2;  // bf16 128 x 256 sub-tile
// per-group scratch in SharedState::epi: group g uses epi[16 g ... 16 g + 15]
constexpr int kPQHead = 0, kPQTail = 1, kPDecision = 2, kPAbort = 3, kPQBase = 4, kPQueue = 8;

__device__ __forceinline__ void group_bar(int g) {
  asm volatile("bar.sync %0, 128;" ::"r"(1 + g) : "memory");
}
__device__ __forceinline__ void epi_all_bar() { asm volatile("bar.sync 3, 256;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

struct PushArEpilogue {
  CommDev c;
  __nv_bfloat16* C;
  long long ldc;
  int vec_ok;
  int n256;             // sub-tiles per row of sub-tiles
  long long red_base;   // byte offset of the reduced slots in a data region
  int groups;           // 4-warp epilogue groups per CTA (1: 2-SM kernel, 2: wide kernel)
  int* sm;

  __device__ __forceinline__ int* flag(int rank, int slot) const { return reinterpret_cast<int*>(c.flags[rank]) + slot; }
  __device__ __forceinline__ int src_index(int src, int owner) const { return src < owner ? src : src - 1; }
  __device__ __forceinline__ int part_slot(int t, int src, int owner) const {
    return (t / c.size) * (c.size - 1) + src_index(src, owner);
  }
  __device__ __forceinline__ uint8_t* part_buf(int owner, int slot) const {
    return reinterpret_cast<uint8_t*>(c.data[owner]) + static_cast<size_t>(slot) * kSubBytes;
  }
  __device__ __forceinline__ uint8_t* red_buf(int rank, int t) const {
    return reinterpret_cast<uint8_t*>(c.data[rank]) + red_base + static_cast<size_t>(t) * kSubBytes;
  }
  __device__ __forceinline__ int pf_flag(int slot) const { return kFlagTile0 + slot; }
  __device__ __forceinline__ int rf_flag(int t) const { return kFlagTile0 + kMaxTiles + t; }

  // every rank must have finished the previous op (reading its region) before
  // anyone writes into it: all threads wait for the check
  __device__ void setup(int* scratch, const GemmShape&) {
    sm = scratch;
    if (threadIdx.x == 0) {
      int ok = 1;
      for (int p = 0; p < c.size && ok; ++p) {
        if (p == c.rank) continue;
        ok = wait_flag_geq_for(flag(p, kFlagDone), c.epoch - 1, c.err, kErrWaitPeerFlag, c.timeout_ns) ? 1 : 0;
      }
      if (!ok) sm[kPAbort] = sm[16 + kPAbort] = 1;
    }
    __syncthreads();
  }

  __device__ void copy_reduced(int t, int g_m0, int g_n0, const GemmShape& s, int e) {
    const int row = g_m0 + e;
    if (row >= s.M) return;
    const uint8_t* src = red_buf(c.rank, t);
    __nv_bfloat16* crow = C + static_cast<long long>(row) * ldc;
#pragma unroll 4
    for (int j = 0; j < kBN / 8; ++j) {
      const int col = g_n0 + j * 8;
      if (col >= s.N) break;
      const uint4 v = *reinterpret_cast<const uint4*>(src + (static_cast<size_t>(j) * kBM + e) * 16);
      if (col + 8 <= s.N && vec_ok) {
        *reinterpret_cast<uint4*>(crow + col) = v;
      } else {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        for (int k = 0; k < 8 && col + k < s.N; ++k) {
          const uint32_t bits = (w[k >> 1] >> ((k & 1) * 16)) & 0xffffu;
          crow[col + k] = __ushort_as_bfloat16(static_cast<unsigned short>(bits));
        }
      }
    }
  }

  // Copy ready reduced tiles of this group's queue into C.  blocking: wait
  // (bounded) for the oldest.  Returns false on abort.
  __device__ bool service(int g, const GemmShape& s, int e, bool blocking, int max_items) {
    int* q = sm + 16 * g;
    for (int done = 0; done < max_items; ++done) {
      if (e == 0) {
        int decision = -1;
        if (q[kPQHead] != q[kPQTail]) {
          const int t = q[kPQBase + (q[kPQHead] % kPQueue)];
          const int* f = flag(c.rank, rf_flag(t));
          bool ready = ld_acquire_sys(f) >= c.epoch;
          if (!ready && blocking) {
            ready = wait_flag_geq_for(f, c.epoch, c.err, kErrWaitPeerFlag, c.timeout_ns);
            if (!ready) q[kPAbort] = 1;
          }
          if (ready) decision = t;
        }
        q[kPDecision] = decision;
      }
      group_bar(g);
      const int t = q[kPDecision];
      if (q[kPAbort]) return false;
      if (t < 0) return true;
      const int mi = t / n256;
      copy_reduced(t, mi * kBM, (t - mi * n256) * kBN, s, e);
      group_bar(g);
      if (e == 0) ++q[kPQHead];
    }
    return true;
  }

  __device__ bool tile(const EpiTile& et, const GemmShape& s, volatile int* abort_flag) {
    const int warp = threadIdx.x >> 5;
    const int g = (warp - 2) >> 2;  // column half of the wide tile = epilogue group
    const int e = et.row;           // 0..127: this thread's row of the sub-tile
    int* q = sm + 16 * g;
    if (q[kPAbort]) return false;
    // the second half of the last pair tile can lie entirely below M: every rank
    // skips it, so no sub-tile index beyond the buffers is ever formed
    if (et.c.m0 >= s.M || et.c.n0 >= s.N) return true;
    const int t = (et.c.m0 / kBM) * n256 + et.c.n0 / kBN;
    const int owner = t % c.size;
    if (owner != c.rank) {
      // ---- push this rank's partial into the owner's slot
      const int slot = part_slot(t, c.rank, owner);
      uint8_t* dst = part_buf(owner, slot);
#pragma unroll 1
      for (int chunk = 0; chunk < kBN / 32; ++chunk) {
        uint32_t r[32];
        tmem_ld32(et.tmem + chunk * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint4 v = make_uint4(pack2(__uint_as_float(r[8 * k + 0]), __uint_as_float(r[8 * k + 1])),
                                     pack2(__uint_as_float(r[8 * k + 2]), __uint_as_float(r[8 * k + 3])),
                                     pack2(__uint_as_float(r[8 * k + 4]), __uint_as_float(r[8 * k + 5])),
                                     pack2(__uint_as_float(r[8 * k + 6]), __uint_as_float(r[8 * k + 7])));
          *reinterpret_cast<uint4*>(dst + (static_cast<size_t>(chunk * 4 + k) * kBM + e) * 16) = v;
        }
      }
      __threadfence_system();
      group_bar(g);
      if (e == 0) {
        st_release_sys(flag(owner, pf_flag(slot)), c.epoch);
        q[kPQBase + (q[kPQTail] % kPQueue)] = t;
        ++q[kPQTail];
      }
      group_bar(g);
      const bool full = (q[kPQTail] - q[kPQHead]) >= kPQueue;
      return service(g, s, e, full, full ? 1 : 2);
    }
    // ---- owner: every peer's partial is in this rank's own region
    if (e == 0) {
      for (int p = 0; p < c.size; ++p) {
        if (p == c.rank) continue;
        if (!wait_flag_geq_for(flag(c.rank, pf_flag(part_slot(t, p, owner))), c.epoch, c.err, kErrWaitPeerFlag, c.timeout_ns)) {
          q[kPAbort] = 1;
          *abort_flag = 1;
          break;
        }
      }
    }
    group_bar(g);
    if (q[kPAbort]) return false;
    const int row = et.c.m0 + e;
    __nv_bfloat16* crow = C + static_cast<long long>(row < s.M ? row : 0) * ldc;
    const int slot0 = (t / c.size) * (c.size - 1);
#pragma unroll 1
    for (int chunk = 0; chunk < kBN / 32; ++chunk) {
      uint32_t r[32];
      tmem_ld32(et.tmem + chunk * 32, r);
      tmem_ld_wait();
      float acc[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(r[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const size_t off = (static_cast<size_t>(chunk * 4 + k) * kBM + e) * 16;
        uint4 v[kMaxRanks - 1];
#pragma unroll
        for (int j = 0; j < kMaxRanks - 1; ++j)
          if (j < c.size - 1) v[j] = *reinterpret_cast<const uint4*>(part_buf(c.rank, slot0 + j) + off);
#pragma unroll
        for (int j = 0; j < kMaxRanks - 1; ++j) {
          if (j >= c.size - 1) break;
          const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            acc[8 * k + 2 * h] += __uint_as_float(w[h] << 16);
            acc[8 * k + 2 * h + 1] += __uint_as_float(w[h] & 0xffff0000u);
          }
        }
      }
      uint4 o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        o[k] = make_uint4(pack2(acc[8 * k + 0], acc[8 * k + 1]), pack2(acc[8 * k + 2], acc[8 * k + 3]),
                          pack2(acc[8 * k + 4], acc[8 * k + 5]), pack2(acc[8 * k + 6], acc[8 * k + 7]));
      // push the reduced piece to every peer
      for (int p = 0; p < c.size; ++p) {
        if (p == c.rank) continue;
        uint8_t* rb = red_buf(p, t);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *reinterpret_cast<uint4*>(rb + (static_cast<size_t>(chunk * 4 + k) * kBM + e) * 16) = o[k];
      }
      const int col0 = et.c.n0 + chunk * 32;
      if (row < s.M && col0 < s.N) {
        if (col0 + 32 <= s.N && vec_ok) {
#pragma unroll
          for (int k = 0; k < 4; ++k) *reinterpret_cast<uint4*>(crow + col0 + 8 * k) = o[k];
        } else {
          for (int k = 0; k < 4; ++k) {
            const uint32_t w[4] = {o[k].x, o[k].y, o[k].z, o[k].w};
            for (int x = 0; x < 8 && col0 + 8 * k + x < s.N; ++x) {
              const uint32_t bits = (w[x >> 1] >> ((x & 1) * 16)) & 0xffffu;
              crow[col0 + 8 * k + x] = __ushort_as_bfloat16(static_cast<unsigned short>(bits));
            }
          }
        }
      }
    }
    __threadfence_system();
    group_bar(g);
    if (e == 0) {
      for (int p = 0; p < c.size; ++p)
        if (p != c.rank) st_release_sys(flag(p, rf_flag(t)), c.epoch);
    }
    return service(g, s, e, false, 2);
  }

  __device__ void finish(const GemmShape& s, volatile int* abort_flag) {
    const int warp = threadIdx.x >> 5;
    const int g = (warp - 2) >> 2;
    const int e = (threadIdx.x - 64) - 128 * g;
    int* q = sm + 16 * g;
    bool ok = !q[kPAbort] && !*abort_flag;
    if (ok) {
      while (true) {
        group_bar(g);
        if (q[kPQHead] == q[kPQTail]) break;
        if (!service(g, s, e, true, 1)) {
          ok = false;
          break;
        }
      }
    }
    if (!ok) q[kPAbort] = 1;
    if (groups == 2) {
      epi_all_bar();  // both groups of this CTA are done
    } else {
      group_bar(0);
    }
    if (threadIdx.x == 64) {
      const bool all_ok = !sm[kPAbort] && (groups == 1 || !sm[16 + kPAbort]) && !*abort_flag;
      fence_acq_rel_sys();
      const int prev = atomicAdd(flag(c.rank, kFlagArrive), 1);
      if (static_cast<uint32_t>(prev + 1) - c.arrive_base == gridDim.x && all_ok) {
        fence_acq_rel_sys();
        st_release_sys(flag(c.rank, kFlagDone), c.epoch);
      }
    }
  }
};

}  // namespace

long long gemm_push_region_bytes(const GemmArgs& g, int size) {
  const long long tiles = static_cast<long long>((g.M + kBM - 1) / kBM) * ((g.N + kBN - 1) / kBN);
  const long long owned = (tiles + size - 1) / size;
  return (owned * (size - 1) + tiles) * kSubBytes;
}

int gemm_push_grid(const GemmArgs& g) {
  const long long pair_tiles = static_cast<long long>((g.M + 255) / 256) * ((g.N + 255) / 256);
  const int clusters = pair_tiles < g.num_sms / 2 ? static_cast<int>(pair_tiles) : g.num_sms / 2;
  return 2 * clusters;
}

int gemm_push_allreduce_launch(const GemmArgs& g, const CommDev& comm, cudaStream_t stream) {
  if (check_gemm_args(g)) return -1;
  if (g.out_dtype != kDtypeBF16 || g.batch != 1) return -2;
  const long long tiles = static_cast<long long>((g.M + kBM - 1) / kBM) * ((g.N + kBN - 1) / kBN);
  if (tiles + comm.size > kMaxTiles) return -3;  // partial-slot flags stay below the reduced-tile flags
  CUtensorMap ma, mb;
  make_operand_maps(g, &ma, &mb, true);
  GemmShape s = make_shape_pair(g);
  s.split = 0;
  PushArEpilogue epi;
  epi.c = comm;
  epi.C = reinterpret_cast<__nv_bfloat16*>(g.C);
  epi.ldc = g.ldc;
  epi.vec_ok = ((reinterpret_cast<uintptr_t>(g.C) & 15) == 0) && (g.ldc % 8 == 0);
  epi.n256 = (g.N + kBN - 1) / kBN;
  const long long owned = (tiles + comm.size - 1) / comm.size;
  epi.red_base = owned * (comm.size - 1) * kSubBytes;
  epi.groups = 1;
  epi.sm = nullptr;
  CUtensorMap mc;  // the push epilogue stores with plain NVLink writes: no output map
  memset(&mc, 0, sizeof(mc));
  auto kernel = gemm_tc2_kernel<PushArEpilogue>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1ull)) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem2Bytes);
    cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gemm_push_grid(g));
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

}  // namespace es
