// Fused GEMM + all-reduce through the NVSwitch: C = sum over ranks of A_r @ B_r,
// on every rank, in one launch.
//
// The launch holds two kinds of clusters (CTA pairs):
//  * GEMM clusters run the wide 2-SM tcgen05 GEMM (gemm_tc3.cuh) unchanged,
//    except that each epilogue warp stores its 32 x 256 unit of the bf16
//    partial product into this rank's symmetric heap (TMA store) and then
//    tells the unit's owner rank (u mod P) that the partial is there: a
//    release store of the call's epoch into the owner's ready[u][rank] word
//    over NVLink.  The accumulator is released to the next tile as soon as it
//    is read, as in the plain GEMM; the transfer never holds TMEM.
//  * The first R clusters reduce and copy out.  Their reduce warps take the
//    units this rank owns, in tile order: once ready[u][q] carries the epoch
//    for every rank q, one multimem.ld_reduce per 16 bytes sums the unit over
//    all ranks inside the switch (fp32 accumulation) and one multimem.st
//    writes the sum back into every rank's heap; a multicast release store
//    sets reduced[u] = epoch on every rank.  Their copy warps walk all units
//    in tile order and copy each reduced unit from the heap into the output
//    tensor.
// GEMM clusters never wait on anything but their own pipeline; reducers wait
// (bounded) for partials that GEMM clusters of every rank produce, so the
// launch cannot deadlock.  When a rank's launch ends it has seen reduced[u]
// for every unit, so every peer's access to its heap for this call (loads of
// its partials, stores of the sums) is over: the call needs no closing
// barrier, and the next call may overwrite the heap at once.  Flags carry
// epochs (one writer per word), so calls of different shapes can alternate.
//
// Per rank and output byte the links carry about 9/8 of the bytes each way at
// P = 8 (see nvls.cu); the GEMM runs on the SMs left after the R reducer
// pairs.  Replaces the reference's einsum followed by a separate all-reduce
// (src/torch_einshard/einsum.py:132 then mappings.py:4-13, helpers.py:27-32).
#include <cuda_bf16.h>

#include "gemm.h"
#include "gemm_nvls.h"
#include "gemm_tc3.cuh"
#include "nvls.h"
#include "tma_desc.h"

#include <string.h>

namespace es {
namespace {

__device__ __forceinline__ uint4 ld_reduce_bf16x8(const uint8_t* p) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ void mc_st16(uint8_t* p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void mc_st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("multimem.st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait of one thread until *p >= target (epochs, wrap-safe).
// Polls back off with __nanosleep (doubling up to 1 us) so waiting reducer
// warps issue few instructions and draw little power next to the GEMM.
__device__ __forceinline__ bool wait_epoch(const uint32_t* p, uint32_t target, uint64_t timeout_ns) {
  if (static_cast<int>(ld_acquire_sys_u32(p) - target) >= 0) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t nap = 32;
  while (static_cast<int>(ld_acquire_sys_u32(p) - target) < 0) {
    __nanosleep(nap);
    if (nap < 1024) nap <<= 1;
    if (global_timer_ns() - t0 > timeout_ns) return false;
  }
  return true;
}

// Unit u -> its first output row and column (unit = 32 rows x 256 columns of
// one CTA's half of a pair tile: u = (2 pair + cta) * 8 + half * 4 + quadrant).
__device__ __forceinline__ void unit_origin(const GemmShape& s, long long u, int* row0, int* col0) {
  const int tcta = static_cast<int>(u >> 3);
  const int half = static_cast<int>((u >> 2) & 1);
  const int q = static_cast<int>(u & 3);
  const TileCoord c = tile_coord3(s, tcta >> 1, tcta & 1);
  *row0 = c.m0 + q * 32;
  *col0 = c.n0 + half * kBN;
}

// Owner of a unit: all-reduce (seg == 0): u mod P; reduce-scatter: the rank
// whose rows the unit holds (rows [seg i + p shard, seg i + (p + 1) shard) are
// rank p's; shard is a multiple of the 32-row unit height).
__device__ __forceinline__ int unit_owner(long long u, int row0, int size, int seg, int shard) {
  return seg ? (row0 % seg) / shard : static_cast<int>(u % size);
}

struct ReduceJob {
  uint8_t* uc;         // this rank's partial / reduced C in the heap, bf16 [M][ldh]
  uint8_t* mc;         // multicast view of the same
  uint32_t* ready;     // this rank's ready[0][0]
  uint32_t* reduced;   // this rank's reduced[0]
  uint32_t* reduced_mc;
  uint8_t* out;        // output tensor, bf16 [M][ldo]
  long long ldh, ldo;
  long long units;
  int rank, size;
  uint32_t epoch;
  int clusters;        // reducer clusters at the front of the grid
  int seg, shard;      // reduce-scatter (seg > 0): out holds this rank's rows only, [M / P][ldo]
  int* err;
  uint64_t timeout_ns;
};

constexpr int kRowsInFlight = 32;  // reducer warps: a whole unit (16 KB per warp) in flight

// One unit owned by this rank: wait until every rank's partial is in its heap,
// sum it in the switch, then either multicast the sum back into every rank's
// heap (all-reduce) or store it into this rank's rows of the output
// (reduce-scatter), and multicast reduced[u] = epoch.  False on a timeout.
template <int kRows = kRowsInFlight>
__device__ __forceinline__ bool reduce_unit(const ReduceJob& j, const GemmShape& s, long long u, int row0, int col0,
                                            int lane) {
  bool ok = true;
  if (lane < j.size) ok = wait_epoch(j.ready + u * j.size + lane, j.epoch, j.timeout_ns);
  if (!__all_sync(0xffffffffu, ok)) {
    if (lane == 0) atomicCAS(j.err, 0, kErrWaitPeerFlag);
    return false;
  }
  const int col = col0 + lane * 8;
  const int rows = es_min(32, s.M - row0);
  if (col < s.N) {
    // the unit's rows: heap row pitch ldh; in reduce-scatter mode a 32-row unit
    // lies inside one owner's shard, so its output rows are consecutive too
    const long long pitch = j.ldh * 2;
    const uint8_t* src = j.mc + (static_cast<long long>(row0) * j.ldh + col) * 2;
    uint8_t* dst;
    long long dpitch;
    if (j.seg) {
      const long long local = (row0 / j.seg) * j.shard + (row0 % j.seg) - static_cast<long long>(j.rank) * j.shard;
      dst = j.out + (local * j.ldo + col) * 2;
      dpitch = j.ldo * 2;
    } else {
      dst = j.mc + (static_cast<long long>(row0) * j.ldh + col) * 2;
      dpitch = pitch;
    }
    for (int r0 = 0; r0 < rows; r0 += kRows) {
      uint4 v[kRows];
#pragma unroll
      for (int i = 0; i < kRows; ++i)
        if (r0 + i < rows) v[i] = ld_reduce_bf16x8(src + (r0 + i) * pitch);
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        if (r0 + i >= rows) continue;
        if (j.seg)
          *reinterpret_cast<uint4*>(dst + (r0 + i) * dpitch) = v[i];
        else
          mc_st16(dst + (r0 + i) * dpitch, v[i]);
      }
    }
  }
  __syncwarp();
  if (lane == 0) {
    fence_acq_rel_sys();
    mc_st_release_u32(j.reduced_mc + u, j.epoch);
  }
  return true;
}

constexpr int kCopyRowsInFlight = 16;

// Copy-out of one reduced unit by one warp through registers: wait until the
// unit's owner stored the sum into this rank's heap (reduced[u] = epoch), then
// move it to the output (all-reduce) or only wait (reduce-scatter: the owner
// stored its rows itself).  Loads bypass L1 (the sums arrived from the switch).
__device__ __forceinline__ bool copy_unit(const ReduceJob& j, const GemmShape& s, long long u, int lane) {
  int row0, col0;
  unit_origin(s, u, &row0, &col0);
  if (row0 >= s.M || col0 >= s.N) return true;
  bool ok = true;
  if (lane == 0) ok = wait_epoch(j.reduced + u, j.epoch, j.timeout_ns);
  if (!__shfl_sync(0xffffffffu, ok, 0)) {
    if (lane == 0) atomicCAS(j.err, 0, kErrWaitPeerFlag);
    return false;
  }
  if (j.seg) return true;
  const int col = col0 + lane * 8;
  if (col >= s.N) return true;
  const int rows = es_min(32, s.M - row0);
  const uint4* src = reinterpret_cast<const uint4*>(j.uc + (static_cast<long long>(row0) * j.ldh + col) * 2);
  uint4* dst = reinterpret_cast<uint4*>(j.out + (static_cast<long long>(row0) * j.ldo + col) * 2);
  const long long sp = j.ldh / 8, dp = j.ldo / 8;  // row pitches in uint4
  for (int r0 = 0; r0 < rows; r0 += kCopyRowsInFlight) {
    uint4 v[kCopyRowsInFlight];
#pragma unroll
    for (int i = 0; i < kCopyRowsInFlight; ++i)
      if (r0 + i < rows) v[i] = __ldcg(src + (r0 + i) * sp);
#pragma unroll
    for (int i = 0; i < kCopyRowsInFlight; ++i)
      if (r0 + i < rows) dst[(r0 + i) * dp] = v[i];
  }
  return true;
}

// Epilogue of the GEMM clusters: the plain TMA-store epilogue into the heap,
// then the unit's ready word on its owner.
struct PartialEpilogue {
  StoreEpilogue<__nv_bfloat16> store;
  ReduceJob job;              // overlap mode: what the epilogue warps reduce and copy out
  int lag;                    // overlap mode: slot p reduces tile p - lag, copies out tile p - 2 lag (0: off)
  int tiles;                  // pair tiles of the product
  uint64_t ready[kMaxRanks];  // each rank's ready[0][0] (peer-mapped)
  int rank, size;
  uint32_t epoch;
  int seg, shard;             // reduce-scatter row segments (seg == 0: all-reduce)

  __device__ __forceinline__ void setup(int*, const GemmShape&) {}
  __device__ __forceinline__ void finish(const GemmShape&, volatile int*) {}
  __device__ __forceinline__ bool tile(const EpiTile& et, const GemmShape& s, volatile int* abort_flag) {
    store.tile(et, s, abort_flag);
    const int half = (et.c.n0 / kBN) & 1;
    const long long u = static_cast<long long>(et.t) * 8 + half * 4 + et.q;
    if (et.lane == 0) {
      bulk_wait_group<0>();        // the unit's TMA stores have completed
      fence_proxy_async_global();  // ... and are ordered before generic-proxy accesses
      fence_acq_rel_sys();
      const int owner = unit_owner(u, et.c.m0 + et.q * 32, size, seg, shard);
      st_release_sys_u32(reinterpret_cast<uint32_t*>(ready[owner]) + u * size + rank, epoch);
    }
    __syncwarp();
    return true;
  }

  // Overlap mode (one tile per cluster, lag > 0): before waiting for its own
  // accumulator, the pair's 16 epilogue warps reduce the units of tile
  // slot - lag that this rank owns (warp w: the w-th of them) and copy out
  // unit w of tile slot - 2 lag.  Both tiles belong to clusters that started
  // earlier, so the waits point backwards in launch order; the last 2 lag
  // slots are clusters without a tile.
  __device__ __forceinline__ void overlap(int slot, int cta, int ewarp, int lane, const GemmShape& s) {
    if (lag != 0) overlap_slot(slot, cta, ewarp, lane, s);
  }
  // out of line: the epilogue loop's registers are saved once per tile rather
  // than squeezed under the 168-register cap of 10-warp blocks
  __device__ __noinline__ void overlap_slot(int slot, int cta, int ewarp, int lane, const GemmShape& s) const {
    if (*reinterpret_cast<volatile int*>(job.err) != 0) return;  // a wait of this call already gave up
    const int w = cta * kEpiWarps3 + ewarp;
    const int t = slot - lag;
    if (t >= 0 && t < tiles) {
      int k = 0;
      for (int i = 0; i < 16; ++i) {
        const long long u = static_cast<long long>(t) * 16 + i;
        int row0, col0;
        unit_origin(s, u, &row0, &col0);
        if (row0 >= s.M || col0 >= s.N || unit_owner(u, row0, size, seg, shard) != rank) continue;
        if (k++ == w) {
          // 16 rows in flight: the epilogue warps keep their tile state live
          if (!reduce_unit<16>(job, s, u, row0, col0, lane)) return;
          break;
        }
      }
    }
    const int t2 = slot - 2 * lag;
    if (t2 >= 0 && t2 < tiles) copy_unit(job, s, static_cast<long long>(t2) * 16 + w, lane);
  }
};

constexpr int kCopySlots = 8;            // 16 KB units in flight per reducer CTA's copy warp
constexpr int kUnitBytes = 32 * kBN * 2;  // 32 rows x 256 columns of bf16

// Copy warp of a reducer CTA (lane 0 drives the TMA engine): for the units
// u = cta, cta + ncta, ... it waits until the unit's owner reduced it, then
// (all-reduce) moves it from the heap to the output through shared memory with
// TMA bulk tensor copies, up to kCopySlots units in flight; in reduce-scatter
// mode it only waits.  When it returns, every peer's access to this rank's
// heap for the call is over.
__device__ void copy_role(const ReduceJob& j, const GemmShape& s, const CUtensorMap* tm_heap,
                          const CUtensorMap* tm_out, int cta, int ncta) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kCopySlots * kUnitBytes);
  if ((threadIdx.x & 31) != 0) return;
  for (int i = 0; i < kCopySlots; ++i) mbar_init(&bars[i], 1);
  fence_mbar_init();
  const bool copy = j.seg == 0;
  long long issued = 0, stored = 0;  // unit counts along u = cta + k ncta (in-range units only)
  int pending_row[kCopySlots], pending_col[kCopySlots];
  long long next = cta;
  int dummy_abort = 0;
  for (;;) {
    // issue loads while slots are free
    while (copy ? issued - stored < kCopySlots : true) {
      int row0 = 0, col0 = 0;
      while (next < j.units) {
        unit_origin(s, next, &row0, &col0);
        if (row0 < s.M && col0 < s.N) break;
        next += ncta;
      }
      if (next >= j.units) break;
      if (!wait_epoch(j.reduced + next, j.epoch, j.timeout_ns)) {
        atomicCAS(j.err, 0, kErrWaitPeerFlag);
        bulk_wait_group<0>();
        return;
      }
      next += ncta;
      if (!copy) continue;
      fence_proxy_async_global();  // the sums arrived as generic stores; the TMA load is an async-proxy read
      const int slot = static_cast<int>(issued % kCopySlots);
      if (issued >= kCopySlots) bulk_wait_group_read<0>();  // the slot's last store has read its bytes
      uint8_t* buf = ring + slot * kUnitBytes;
      mbar_arrive_expect_tx(&bars[slot], kUnitBytes);
#pragma unroll
      for (int b = 0; b < kBN / 64; ++b) tma_load_3d(buf + b * 4096, tm_heap, &bars[slot], col0 + 64 * b, row0, 0);
      pending_row[slot] = row0;
      pending_col[slot] = col0;
      ++issued;
    }
    if (!copy || stored == issued) break;
    // store the oldest loaded unit
    const int slot = static_cast<int>(stored % kCopySlots);
    const uint32_t parity = static_cast<uint32_t>((stored / kCopySlots) & 1);
    if (!mbar_wait(&bars[slot], parity, &dummy_abort, j.err, kErrWaitFull)) {
      bulk_wait_group<0>();
      return;
    }
    uint8_t* buf = ring + slot * kUnitBytes;
#pragma unroll
    for (int b = 0; b < kBN / 64; ++b)
      tma_store_3d(tm_out, buf + b * 4096, pending_col[slot] + 64 * b, pending_row[slot], 0);
    bulk_commit_group();
    ++stored;
  }
  bulk_wait_group<0>();
}

// Reduce and copy-out roles of the first job.clusters clusters: warp 0 copies
// out (copy_role), the other warps reduce the units this rank owns.
__device__ void reducer_role(const ReduceJob& j, const GemmShape& s, const CUtensorMap* tm_heap,
                             const CUtensorMap* tm_out, int cta, int ncta) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  if (warp == 0) {
    copy_role(j, s, tm_heap, tm_out, cta, ncta);
    return;
  }
  const int red_warps = nwarps - 1;
  const long long gw = static_cast<long long>(cta) * red_warps + (warp - 1);
  const long long W = static_cast<long long>(ncta) * red_warps;
  if (!j.seg) {
    for (long long k = gw;; k += W) {
      const long long u = j.rank + k * j.size;
      if (u >= j.units) break;
      int row0, col0;
      unit_origin(s, u, &row0, &col0);
      if (row0 >= s.M || col0 >= s.N) continue;
      if (!reduce_unit(j, s, u, row0, col0, lane)) return;
    }
    return;
  }
  // reduce-scatter: the units whose rows this rank owns, in unit order, found 32 at a time
  long long k = 0;
  for (long long base = 0; base < j.units; base += 32) {
    const long long u = base + lane;
    int row0 = 0, col0 = 0;
    bool mine = false;
    if (u < j.units) {
      unit_origin(s, u, &row0, &col0);
      mine = row0 < s.M && col0 < s.N && unit_owner(u, row0, j.size, j.seg, j.shard) == j.rank;
    }
    unsigned m = __ballot_sync(0xffffffffu, mine);
    while (m) {
      const int bit = __ffs(m) - 1;
      m &= m - 1;
      if (k % W == gw) {
        int r0, c0;
        unit_origin(s, base + bit, &r0, &c0);
        if (!reduce_unit(j, s, base + bit, r0, c0, lane)) return;
      }
      ++k;
    }
  }
}

__global__ void __launch_bounds__(kThreads3, 1)
    gemm_nvls_ar_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmW,
                        const GemmShape shp, PartialEpilogue epi, const ReduceJob job) {
  const int cluster = static_cast<int>(cluster_id_x());
  if (cluster < job.clusters) {
    reducer_role(job, shp, &tmC, &tmW, cluster * 2 + static_cast<int>(cluster_ctarank()), job.clusters * 2);
    return;
  }
  gemm_tc3_body(tmA, tmB, tmC, tmW, shp, epi, NoGather{}, cluster - job.clusters,
                static_cast<int>(nclusters_x()) - job.clusters);
}

}  // namespace

long long gemm_nvls_units(int M, int N) {
  const long long pairs = static_cast<long long>((M + 2 * kBM - 1) / (2 * kBM)) * ((N + kBN3 - 1) / kBN3);
  return pairs * 16;
}

int gemm_nvls_allreduce_launch(const GemmArgs& g, const NvlsGemmJob& nj, cudaStream_t stream) {
  if (g.batch != 1 || g.out_dtype != kDtypeBF16 || g.dtype != kDtypeBF16 || g.N % 8 != 0 || g.act != 0)
    return static_cast<int>(cudaErrorInvalidValue);
  const long long units = gemm_nvls_units(g.M, g.N);
  if (units > kNvlsMaxUnits || nj.reducer_clusters < 0 || nj.lag < 0)
    return static_cast<int>(cudaErrorInvalidValue);
  // overlap mode (no reducer clusters): register copy-out, 16-byte rows
  if (nj.reducer_clusters == 0 && (reinterpret_cast<uintptr_t>(g.C) % 16 != 0 || g.ldc % 8 != 0))
    return static_cast<int>(cudaErrorInvalidValue);
  if (nj.seg && (nj.shard % 32 != 0 || nj.shard * nj.size != nj.seg || g.M % nj.seg != 0))
    return static_cast<int>(cudaErrorInvalidValue);
  CUtensorMap ma, mb, mc, mw;
  make_operand_maps(g, &ma, &mb, true);
  // the partial product goes to the heap (row pitch N), not to the output tensor
  GemmArgs gh = g;
  gh.C = nj.heap_uc;
  gh.ldc = g.N;
  gh.c_batch_stride = 0;
  if (!make_output_map(gh, false, &mc)) return static_cast<int>(cudaErrorInvalidValue);
  // the output map (all-reduce copy-out target) travels in the stream-K workspace slot
  memset(&mw, 0, sizeof(mw));
  if (nj.seg == 0 && !make_output_map(g, false, &mw)) return static_cast<int>(cudaErrorInvalidValue);
  GemmShape s = make_shape(g);
  s.num_m = (g.M + 2 * kBM - 1) / (2 * kBM);
  s.num_n = (g.N + kBN3 - 1) / kBN3;
  s.group_m = g.group_m > 0 ? g.group_m : 16;
  s.pair = 1;
  s.split = 0;
  PartialEpilogue epi;
  epi.store.C = static_cast<__nv_bfloat16*>(nj.heap_uc);
  epi.store.ldc = g.N;
  epi.store.batch_stride = 0;
  epi.store.vec_ok = 1;
  epi.store.act = 0;
  epi.store.trans = 0;
  epi.store.tma = 1;
  for (int p = 0; p < kMaxRanks; ++p) epi.ready[p] = p < nj.size ? nj.ready_base[p] : 0;
  epi.rank = nj.rank;
  epi.size = nj.size;
  epi.epoch = nj.epoch;
  epi.seg = nj.seg;
  epi.shard = nj.shard;
  ReduceJob job;
  job.uc = static_cast<uint8_t*>(nj.heap_uc);
  job.mc = static_cast<uint8_t*>(nj.heap_mc);
  job.ready = reinterpret_cast<uint32_t*>(nj.ready_base[nj.rank]);
  job.reduced = nj.reduced;
  job.reduced_mc = nj.reduced_mc;
  job.out = static_cast<uint8_t*>(g.C);
  job.ldh = g.N;
  job.ldo = g.ldc;
  job.units = units;
  job.rank = nj.rank;
  job.size = nj.size;
  job.epoch = nj.epoch;
  job.clusters = nj.reducer_clusters;
  job.seg = nj.seg;
  job.shard = nj.shard;
  job.err = g.err;
  job.timeout_ns = nj.timeout_ns;
  const int pairs = s.num_m * s.num_n;
  epi.job = job;
  epi.tiles = pairs;
  epi.lag = 0;
  if (nj.reducer_clusters == 0) {
    // one tile per cluster; slot p reduces tile p - lag.  Two waves of
    // resident pairs: tile p - lag finished a wave before cluster p started on
    // this rank, which leaves a wave of slack for ranks running behind (2 GPUs:
    // 6.58 ms at lag 148 against 6.74 at 74, 6.27 at 37 and 9.30 at 16)
    epi.lag = es_min(pairs, nj.lag > 0 ? nj.lag : g.num_sms);
  }

  auto kernel = gemm_nvls_ar_kernel;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1ull)) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem3Bytes);
    attr_set |= 1ull << dev;
  }
  const bool persistent = g.persistent > 0 || (g.persistent < 0 && s.num_kb <= 32);
  int gemm_clusters = g.num_sms / 2 - nj.reducer_clusters;
  if (gemm_clusters < 1) return static_cast<int>(cudaErrorInvalidValue);
  if (pairs < gemm_clusters || !persistent) gemm_clusters = pairs;
  if (epi.lag > 0) gemm_clusters = pairs + 2 * epi.lag;  // the last 2 lag slots hold no tile
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (gemm_clusters + nj.reducer_clusters));
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
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, ma, mb, mc, mw, s, epi, job));
}

}  // namespace es
