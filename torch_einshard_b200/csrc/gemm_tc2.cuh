// 2-SM (CTA pair) persistent tcgen05 GEMM mainloop for sm_100a.
//
// A cluster of two CTAs on neighbouring SMs computes one 256 x 256 output tile
// with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16): CTA r of the pair
// loads rows [128 r, 128 r + 128) of the A tile and columns [128 r, 128 r + 128)
// of the B tile into its own shared memory, so every SM stages only 32 KB per
// 64-deep K step (6 stages fit in 192 KB).  The leader CTA (rank 0) issues the
// MMAs; its instruction reads both CTAs' operand tiles and writes each CTA's
// 128 accumulator rows into that CTA's TMEM.
//
// Synchronisation (mbarriers):
//   full[s]   leader only; both CTAs' TMA loads signal it (cta_group::2 loads,
//             no multicast); the leader producer expects the pair's bytes.
//   empty[s]  in both CTAs; the leader's tcgen05.commit multicasts to both.
//   tfull[a]  in both CTAs; multicast commit after the last K step of a tile.
//   tempty[a] leader only; all 8 epilogue warps of the pair arrive on it.
// Tiles are handed to the epilogue policy as 128-row halves (EpiTile.t =
// 2 * pair_tile + rank), so the policies of gemm_tc.cuh work unchanged; each
// epilogue warp has a 4 KB staging buffer for TMA-store epilogues (tmC).
#pragma once

#include "gemm_tc.cuh"

namespace es {

constexpr int kStages2 = 6;
constexpr int kA2Bytes = kBM * kBK * 2;          // 16 KB: this CTA's 128 A rows
constexpr int kB2Bytes = (kBN / 2) * kBK * 2;    // 16 KB: this CTA's 128 B columns
constexpr int kStage2Bytes = kA2Bytes + kB2Bytes;
constexpr int kStage2Out = 4096;  // per epilogue warp: staging of one 32 x 64 16-bit output box
constexpr int kSmem2Bytes = kStages2 * kStage2Bytes + 1024 + 4 * kStage2Out + 1024;

struct SharedState2 {
  uint64_t full[kStages2];
  uint64_t empty[kStages2];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int consumed;
  int epi[32];
};

template <class Epi>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const GemmShape shp, Epi epi) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages2 * kA2Bytes;
  SharedState2* st = reinterpret_cast<SharedState2*>(smem + kStages2 * kStage2Bytes);
  uint8_t* out_stage = smem + kStages2 * kStage2Bytes + 1024;  // 1024-byte aligned (TMA swizzle atom)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pairs = shp.num_m * shp.num_n * shp.batch;  // num_m counts 256-row pair tiles
  const int cluster = static_cast<int>(cluster_id_x());
  const int nclusters = static_cast<int>(nclusters_x());

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&st->full[s], 1);
      mbar_init(&st->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&st->tfull[a], 1);
      mbar_init(&st->tempty[a], 2 * (kEpiThreads / 32));
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
    tmem_alloc_pair(&st->tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = st->tmem_base;
  volatile int* abort_flag = &st->abort_flag;
  epi.setup(st->epi, shp);

  const uint32_t full_leader0 = map_to_cta(&st->full[0], 0);
  const uint32_t tempty_leader0 = map_to_cta(&st->tempty[0], 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    uint32_t it = 0;
    for (int p = cluster; p < pairs; p += nclusters) {
      const TileCoord c = tile_coord(shp, 2 * p + static_cast<int>(rank));  // this CTA's 128-row half
      const int n_half = c.n0 + static_cast<int>(rank) * (kBN / 2);
      for (int kb = 0; kb < shp.num_kb; ++kb, ++it) {
        const int s = it % kStages2;
        const uint32_t ph = (it / kStages2) & 1u;
        if (!mbar_wait_lane0(&st->empty[s], ph ^ 1u, abort_flag, shp.err, kErrWaitEmpty)) goto producer_done;
        if (lane == 0) {
          uint8_t* a = sA + s * kA2Bytes;
          uint8_t* b = sB + s * kB2Bytes;
          const uint32_t fbar = full_leader0 + s * 8;
          if (leader) mbar_arrive_expect_tx(&st->full[s], 2 * kStage2Bytes);
          const int k0 = kb * kBK;
          if (!shp.a_mn) {
            tma_load_3d_pair(a, &tmA, fbar, k0, c.m0, c.b);
          } else {
            tma_load_3d_pair(a, &tmA, fbar, c.m0, k0, c.b);
            tma_load_3d_pair(a + 8192, &tmA, fbar, c.m0 + 64, k0, c.b);
          }
          if (!shp.b_mn) {
            tma_load_3d_pair(b, &tmB, fbar, k0, n_half, c.b);
          } else {
            tma_load_3d_pair(b, &tmB, fbar, n_half, k0, c.b);
            tma_load_3d_pair(b + 8192, &tmB, fbar, n_half + 64, k0, c.b);
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
        mbar_wait(&st->full[j % kStages2], (j / kStages2) & 1u, &dummy_abort, nullptr, 0);
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
      for (int p = cluster; p < pairs; p += nclusters, ++tc) {
        const uint32_t acc = tc & 1u;
        const uint32_t aph = (tc >> 1) & 1u;
        if (!mbar_wait_lane0(&st->tempty[acc], aph ^ 1u, abort_flag, shp.err, kErrWaitTmemEmpty)) goto mma_done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        for (int kb = 0; kb < shp.num_kb; ++kb, ++it) {
          const int s = it % kStages2;
          const uint32_t ph = (it / kStages2) & 1u;
          if (!mbar_wait_lane0(&st->full[s], ph, abort_flag, shp.err, kErrWaitFull)) goto mma_done;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_addr = smem_u32(sA + s * kA2Bytes);
            const uint32_t b_addr = smem_u32(sB + s * kB2Bytes);
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
              const uint64_t ad = umma_desc_sw128(a_addr + k * a_kstep, a_lbo, 1024u);
              const uint64_t bd = umma_desc_sw128(b_addr + k * b_kstep, b_lbo, 1024u);
              umma_f16_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            }
            umma_commit_pair_mc(&st->empty[s], 0x3);
            *reinterpret_cast<volatile int*>(&st->consumed) = static_cast<int>(it + 1);
          }
          issued_any = true;
          __syncwarp();
        }
        if (lane == 0) umma_commit_pair_mc(&st->tfull[acc], 0x3);
        __syncwarp();
      }
    mma_done:
      __syncwarp();
      if (*abort_flag && issued_any && lane == 0) {
        umma_commit_pair_mc(&st->drain, 0x1);
        int dummy_abort = 0;
        mbar_wait(&st->drain, 0, &dummy_abort, nullptr, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    uint32_t tc = 0;
    for (int p = cluster; p < pairs; p += nclusters, ++tc) {
      const uint32_t acc = tc & 1u;
      const uint32_t ph = (tc >> 1) & 1u;
      if (!mbar_wait(&st->tfull[acc], ph, abort_flag, shp.err, kErrWaitTmemFull)) break;
      tc_fence_after();
      EpiTile et;
      et.t = 2 * p + static_cast<int>(rank);
      et.c = tile_coord(shp, et.t);
      et.tmem = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kBN;
      et.row = q * 32 + lane;
      et.q = q;
      et.lane = lane;
      et.tmc = &tmC;
      et.stage = out_stage + q * kStage2Out;
      const bool ok = epi.tile(et, shp, abort_flag);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + acc * 8);
      if (!ok) {
        *abort_flag = 1;
        break;
      }
    }
    epi.finish(shp, abort_flag);
    if (lane == 0) bulk_wait_group<0>();  // every TMA store of this warp has landed
  }

  __syncthreads();
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still touch its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace es
