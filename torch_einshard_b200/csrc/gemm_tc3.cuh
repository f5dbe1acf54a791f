// Wide 2-SM (CTA pair) persistent tcgen05 GEMM: 256 x 512 output tile per pair.
//
// Each CTA of the pair owns 128 rows x 512 columns of the tile, i.e. all 512
// TMEM columns as one fp32 accumulator; each K=16 step issues two
// tcgen05.mma.cta_group::2 (M=256, N=256), one per 256-column half.  Per 64-deep
// K block every SM stages 16 KB of A (its 128 rows) and 32 KB of B (its two
// 128-column quarters), so the L2->SM traffic per MMA cycle is 3/4 of the
// 256 x 256 pair kernel's and 1/2 of the 1-SM 128 x 256 kernel's; no TMA
// multicast is used (every CTA loads its own boxes).
//
// With the whole TMEM in one accumulator there is no second buffer: the MMA
// warp waits for the epilogue to drain the previous tile before the first MMA
// of the next one.  Eight epilogue warps per CTA (two per TMEM lane quadrant,
// one per 256-column half) keep that drain short, and the producer keeps
// filling the shared-memory stages meanwhile.
//
// Warps (320 threads): 0 TMA producer, 1 MMA issuer (leader CTA) + TMEM owner,
// 2..9 epilogue.  Barriers as in gemm_tc2.cuh; tempty counts the 16 epilogue
// warps of the pair.
//
// Stream-K tail (shp.sk_iters > 0): pair tiles [0, sk_first) are whole tiles,
// one per cluster (the full waves); the K blocks of the remaining tiles (the
// partial last wave) form one tile-major sequence that clusters sk_first,
// sk_first + 1, ... take in equal slices of sk_iters blocks, so the last wave
// keeps every SM pair busy.  A tail segment accumulates in TMEM from zero and
// its epilogue adds the fp32 partial into a zero-initialised workspace
// [tail tile][256][512] (TMA reduce-add through tmW); a finishing pass converts
// the tail tiles.  sk_first = 0 splits every tile.  A launch may hold only the
// tail clusters (sk_cluster0 = sk_first), the whole tiles running before it in
// a plain launch limited to sk_first tiles.
#pragma once

#include <type_traits>
#include <utility>

#include "gemm_tc.cuh"

namespace es {

constexpr int kBN3 = 512;                          // pair tile width
constexpr int kStages3 = 4;
constexpr int kA3Bytes = kBM * kBK * 2;            // 16 KB: this CTA's 128 A rows
constexpr int kB3Bytes = (kBN3 / 2) * kBK * 2;     // 32 KB: this CTA's two 128-column B quarters
constexpr int kStage3Bytes = kA3Bytes + kB3Bytes;
constexpr int kThreads3 = 320;
constexpr int kEpiWarps3 = 8;
constexpr int kStage3Out = 4096;                    // per epilogue warp: 32 rows x 64 cols x 2 B
constexpr int kSmem3Bytes = kStages3 * kStage3Bytes + 1024 + kEpiWarps3 * kStage3Out + 1024;

// Pipeline barriers of the wide kernel (only tfull_[0] / tempty_[0] are used:
// one accumulator) and the epilogue policy's scratch words.
struct SharedState3 {
  uint64_t full[kStages3];
  uint64_t empty[kStages3];
  uint64_t tfull_[2];
  uint64_t tempty_[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int consumed;
  int epi[32];
};
static_assert(kStages3 == kStages, "SharedState3 must mirror SharedState");

// Pair tile p -> this CTA's 128-row half; columns n0 .. n0 + 511.
__host__ __device__ __forceinline__ TileCoord tile_coord3(const GemmShape& s, int p, int rank) {
  const int per_batch = s.num_m * s.num_n;
  const int b = p / per_batch;
  const int r = p - b * per_batch;
  const int per_group = s.group_m * s.num_n;
  const int g = r / per_group;
  const int first_m = g * s.group_m;
  const int gm = es_min(s.num_m - first_m, s.group_m);
  const int in_group = r - g * per_group;
  const int mb = first_m + in_group % gm;
  const int nb = in_group / gm;
  return {b, mb * 2 * kBM + rank * kBM, nb * kBN3};
}

// The i-th pair tile of this cluster, or false when it has no more.  With a
// split, the two cluster sets walk disjoint halves of the M tiles (each set
// keeps its own A panels in L2 and the sets share B).
__host__ __device__ __forceinline__ bool pair_tile_at(const GemmShape& s, int cluster, int nclusters, int i, int rank,
                                             TileCoord* out) {
  if (s.split == 0 || (nclusters & 1) || s.num_m < 2) {
    const int p = cluster + i * nclusters;
    if (p >= (s.sk_first > 0 ? s.sk_first : s.num_m * s.num_n * s.batch)) return false;
    *out = tile_coord3(s, p, rank);
    return true;
  }
  const int per = nclusters >> 1;
  const int half = s.split == 1 ? (cluster >= per ? 1 : 0) : (cluster & 1);
  const int idx = s.split == 1 ? cluster - half * per : (cluster >> 1);
  const int m_lo = (s.num_m + 1) >> 1;
  GemmShape h = s;
  h.num_m = half ? s.num_m - m_lo : m_lo;
  const int p = idx + i * per;
  if (p >= h.num_m * h.num_n * h.batch) return false;
  TileCoord c = tile_coord3(h, p, rank);
  c.m0 += half * m_lo * 2 * kBM;
  *out = c;
  return true;
}

// The work of one cluster as a sequence of segments: a pair tile and a K-block
// range [kb0, kb1).  Tile mode: whole tiles from pair_tile_at; stream-K: the
// cluster's share of the tile-major K-block sequence.
struct SegIter {
  long long g = 0, end = 0;  // stream-K cursor and end (K blocks)
  int i = 0;                 // tile mode: tiles taken so far
};

__host__ __device__ __forceinline__ SegIter seg_begin(const GemmShape& s, int cluster) {
  SegIter it;
  if (s.sk_iters > 0) {
    const long long nkb = s.num_kb;
    const long long total = static_cast<long long>(s.num_m) * s.num_n * s.batch * nkb;
    const int cl = cluster + s.sk_cluster0;
    if (cl < s.sk_first) {
      it.g = static_cast<long long>(cl) * nkb;
      it.end = it.g + nkb;
    } else {
      it.g = es_min(total, static_cast<long long>(s.sk_first) * nkb +
                               static_cast<long long>(cl - s.sk_first) * s.sk_iters);
      it.end = es_min(total, it.g + s.sk_iters);
    }
  }
  return it;
}

// Next segment: tile coordinates (this CTA's half), linear pair tile index and
// K-block range; false when the cluster has no more work.
__host__ __device__ __forceinline__ bool seg_next(const GemmShape& s, int cluster, int nclusters, int rank, SegIter& it,
                                         TileCoord* c, int* pair_index, int* kb0, int* kb1) {
  if (s.sk_iters > 0) {
    if (it.g >= it.end) return false;
    const long long p = it.g / s.num_kb;
    const int k0 = static_cast<int>(it.g - p * s.num_kb);
    const long long left = it.end - it.g;
    const int k1 = left < s.num_kb - k0 ? k0 + static_cast<int>(left) : s.num_kb;
    *c = tile_coord3(s, static_cast<int>(p), rank);
    *pair_index = static_cast<int>(p);
    *kb0 = k0;
    *kb1 = k1;
    it.g += k1 - k0;
    return true;
  }
  if (!pair_tile_at(s, cluster, nclusters, it.i, rank, c)) return false;
  *pair_index = cluster + it.i * nclusters;
  *kb0 = 0;
  *kb1 = s.num_kb;
  ++it.i;
  return true;
}

// Gather policy of the wide kernel.  The plain GEMM has none; the fused
// all-gather -> GEMM (gemm_ag.cu) adds a copy warp that pulls peers' rows of A
// into a local buffer, orders the M tiles local-rows-first and makes the
// producer wait for a chunk's flag before its TMA loads read those rows.
struct NoGather {
  static constexpr int kCopyWarps = 0;
  __device__ __forceinline__ int map_m0(int m0) const { return m0; }
  __device__ __forceinline__ bool wait_rows(int, volatile int*) const { return true; }
  __device__ __forceinline__ void start() const {}
  __device__ __forceinline__ void copy(int, int, volatile int*) const {}
  __device__ __forceinline__ void finish(bool) const {}
};

// Optional epilogue-policy hook `overlap(slot, cta, ewarp, lane, shape)`:
// work the epilogue warps do for schedule slot `slot` (the cluster index)
// before they wait for the accumulator, i.e. overlapped with the slot's
// mainloop; clusters with no tile call it once.  Policies without it do nothing.
template <class E, class = void>
struct HasOverlap : std::false_type {};
template <class E>
struct HasOverlap<E, std::void_t<decltype(std::declval<E&>().overlap(0, 0, 0, 0, std::declval<const GemmShape&>()))>>
    : std::true_type {};

template <class Epi>
__device__ __forceinline__ void epilogue_overlap(Epi& epi, int slot, int cta, int ewarp, int lane, const GemmShape& s) {
  if constexpr (HasOverlap<Epi>::value) epi.overlap(slot, cta, ewarp, lane, s);
}

// The kernel body, for `nclusters` clusters of which this is number `cluster`
// (kernels that give some clusters another role run it with offset indices).
template <class Epi, class Gather>
__device__ __forceinline__ void gemm_tc3_body(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC,
                                              const CUtensorMap& tmW, const GemmShape& shp, Epi& epi,
                                              const Gather& gather, const int cluster, const int nclusters) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages3 * kA3Bytes;
  SharedState3* st = reinterpret_cast<SharedState3*>(smem + kStages3 * kStage3Bytes);
  uint8_t* out_stage = smem + kStages3 * kStage3Bytes + 1024;  // 1024-byte aligned (TMA swizzle atom)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages3; ++s) {
      mbar_init(&st->full[s], 1);
      mbar_init(&st->empty[s], 1);
    }
    mbar_init(&st->tfull_[0], 1);
    mbar_init(&st->tempty_[0], 2 * kEpiWarps3);
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
    tmem_alloc_pair(&st->tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = st->tmem_base;
  volatile int* abort_flag = &st->abort_flag;
  epi.setup(st->epi, shp);

  const uint32_t full_leader0 = map_to_cta(&st->full[0], 0);
  const uint32_t tempty_leader = map_to_cta(&st->tempty_[0], 0);
  if (threadIdx.x == 0 && cluster == 0 && rank == 0) gather.start();

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    uint32_t it = 0;
    TileCoord c;
    int pidx, kb0, kb1;
    SegIter seg = seg_begin(shp, cluster);
    while (seg_next(shp, cluster, nclusters, static_cast<int>(rank), seg, &c, &pidx, &kb0, &kb1)) {
      c.m0 = gather.map_m0(c.m0);
      if (!gather.wait_rows(c.m0, abort_flag)) goto producer_done;  // rows of A gathered from their owner
      const int nq0 = c.n0 + static_cast<int>(rank) * (kBN / 2);  // this CTA's quarter in each 256-col half
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % kStages3;
        const uint32_t ph = (it / kStages3) & 1u;
        if (!mbar_wait_lane0(&st->empty[s], ph ^ 1u, abort_flag, shp.err, kErrWaitEmpty)) goto producer_done;
        if (lane == 0) {
          uint8_t* a = sA + s * kA3Bytes;
          uint8_t* b = sB + s * kB3Bytes;
          const uint32_t fbar = full_leader0 + s * 8;
          if (leader) mbar_arrive_expect_tx(&st->full[s], 2 * kStage3Bytes);
          const int k0 = kb * kBK;
          if (!shp.a_mn) {
            tma_load_3d_pair(a, &tmA, fbar, k0, c.m0, c.b);
          } else {
            tma_load_3d_pair(a, &tmA, fbar, c.m0, k0, c.b);
            tma_load_3d_pair(a + 8192, &tmA, fbar, c.m0 + 64, k0, c.b);
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint8_t* bh = b + h * (kB3Bytes / 2);
            const int n = nq0 + h * kBN;
            if (!shp.b_mn) {
              tma_load_3d_pair(bh, &tmB, fbar, k0, n, c.b);
            } else {
              tma_load_3d_pair(bh, &tmB, fbar, n, k0, c.b);
              tma_load_3d_pair(bh + 8192, &tmB, fbar, n + 64, k0, c.b);
            }
          }
        }
        __syncwarp();
      }
    }
  producer_done:
    __syncwarp();
    if (*abort_flag && leader && lane == 0) {
      const uint32_t consumed = static_cast<uint32_t>(*reinterpret_cast<volatile int*>(&st->consumed));
      for (uint32_t j = consumed; j < it; ++j) {
        int dummy_abort = 0;
        mbar_wait(&st->full[j % kStages3], (j / kStages3) & 1u, &dummy_abort, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (leader) {
      const uint32_t idesc = umma_idesc_f16(2 * kBM, kBN, shp.in_bf16, shp.a_mn, shp.b_mn);
      const uint32_t a_lbo = shp.a_mn ? 8192u : 16u;
      const uint32_t b_lbo = shp.b_mn ? 8192u : 16u;
      const uint32_t a_kstep = shp.a_mn ? 2048u : 32u;
      const uint32_t b_kstep = shp.b_mn ? 2048u : 32u;
      uint32_t it = 0, tc = 0;
      bool issued_any = false;
      long long wait_full = 0, wait_tempty = 0;
      const long long t_start = clock64();
      TileCoord cm;
      int pidx, kb0, kb1;
      SegIter seg = seg_begin(shp, cluster);
      for (; seg_next(shp, cluster, nclusters, 0, seg, &cm, &pidx, &kb0, &kb1); ++tc) {
        const long long t_e0 = shp.prof ? clock64() : 0;
        if (!mbar_wait_lane0(&st->tempty_[0], (tc & 1u) ^ 1u, abort_flag, shp.err, kErrWaitTmemEmpty)) goto mma_done;
        if (shp.prof) wait_tempty += clock64() - t_e0;
        tc_fence_after();
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kStages3;
          const uint32_t ph = (it / kStages3) & 1u;
          const long long t_f0 = shp.prof ? clock64() : 0;
          if (!mbar_wait_lane0(&st->full[s], ph, abort_flag, shp.err, kErrWaitFull)) goto mma_done;
          if (shp.prof) wait_full += clock64() - t_f0;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_addr = smem_u32(sA + s * kA3Bytes);
            const uint32_t b_addr = smem_u32(sB + s * kB3Bytes);
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
              const uint64_t ad = umma_desc_sw128(a_addr + k * a_kstep, a_lbo, 1024u);
              const uint32_t acc = (kb != kb0 || k != 0) ? 1u : 0u;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint64_t bd = umma_desc_sw128(b_addr + h * (kB3Bytes / 2) + k * b_kstep, b_lbo, 1024u);
                umma_f16_pair(tmem_base + h * kBN, ad, bd, idesc, acc);
              }
            }
            umma_commit_pair_mc(&st->empty[s], 0x3);
            *reinterpret_cast<volatile int*>(&st->consumed) = static_cast<int>(it + 1);
          }
          issued_any = true;
          __syncwarp();
        }
        if (lane == 0) umma_commit_pair_mc(&st->tfull_[0], 0x3);
        __syncwarp();
      }
    mma_done:
      __syncwarp();
      if (shp.prof && lane == 0) {
        // counters: [0] MMA-warp cycles, [1] waiting for a filled stage, [2] waiting for the epilogue
        atomicAdd(&shp.prof[0], static_cast<unsigned long long>(clock64() - t_start));
        atomicAdd(&shp.prof[1], static_cast<unsigned long long>(wait_full));
        atomicAdd(&shp.prof[2], static_cast<unsigned long long>(wait_tempty));
      }
      if (*abort_flag && issued_any && lane == 0) {
        umma_commit_pair_mc(&st->drain, 0x1);
        int dummy_abort = 0;
        mbar_wait(&st->drain, 0, &dummy_abort, nullptr, 0);
      }
    }
  } else if (warp >= 2 + kEpiWarps3) {
    // ------------------------------------------------------------ copy warp (gather policies only)
    gather.copy(cluster * 2 + static_cast<int>(rank), nclusters * 2, abort_flag);
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs, 8 warps)
    const int q = warp & 3;           // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;  // 256-column half of the tile
    uint32_t tc = 0;
    bool any_tile = false;
    TileCoord ce;
    int pidx, kb0, kb1;
    SegIter seg = seg_begin(shp, cluster);
    for (; seg_next(shp, cluster, nclusters, static_cast<int>(rank), seg, &ce, &pidx, &kb0, &kb1); ++tc) {
      any_tile = true;
      ce.m0 = gather.map_m0(ce.m0);
      // work the policy overlaps with this tile's mainloop (while the accumulator fills)
      epilogue_overlap(epi, cluster, static_cast<int>(rank), warp - 2, lane, shp);
      if (!mbar_wait_sleepy(&st->tfull_[0], tc & 1u, abort_flag, shp.err, kErrWaitTmemFull, shp.sleep_ns)) break;
      tc_fence_after();
      EpiTile et;
      et.t = 2 * pidx + static_cast<int>(rank);
      et.c = ce;
      et.c.n0 += half * kBN;
      et.tmem = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + half * kBN;
      et.row = q * 32 + lane;
      et.q = q;
      et.lane = lane;
      et.tmc = &tmC;
      et.tmw = &tmW;
      et.stage = out_stage + (warp - 2) * kStage3Out;
      const bool ok = et.c.n0 < shp.N ? epi.tile(et, shp, abort_flag) : true;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader);
      if (!ok) {
        *abort_flag = 1;
        break;
      }
    }
    if (!any_tile) epilogue_overlap(epi, cluster, static_cast<int>(rank), warp - 2, lane, shp);  // clusters without a tile
    epi.finish(shp, abort_flag);
    if (lane == 0) bulk_wait_group<0>();  // every TMA store of this warp has landed
  }

  __syncthreads();
  if (threadIdx.x == 0) gather.finish(*abort_flag == 0);
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <class Epi, class Gather = NoGather>
__global__ void __launch_bounds__(kThreads3 + 32 * Gather::kCopyWarps, 1)
    gemm_tc3_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmW,
                    const GemmShape shp, Epi epi, const Gather gather = Gather()) {
  gemm_tc3_body(tmA, tmB, tmC, tmW, shp, epi, gather, static_cast<int>(cluster_id_x()),
                static_cast<int>(nclusters_x()));
}

}  // namespace es
