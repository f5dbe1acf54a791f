// Implicit-GEMM 2-D convolution on CTA pairs with the weights resident in
// shared memory (NHWC, bf16/fp16, stride 1, dilation 1).
//
//   out[b, h, w, o] = sum_{kh, kw, c} X[b, h + kh - ph, w + kw - pw, c] * W[o, kh, kw, c]
//
// GEMM view: M = output pixels, N = output channels, K = (kh, kw, c).  A pair
// tile is 256 consecutive output pixels of one output row (128 per CTA, the
// M = 256 tcgen05.mma.cta_group::2 layout: CTA r's TMEM lanes hold its 128
// pixels) times `otile` output channels (N; every CTA holds otile / 2 rows of
// the weights, the pair MMA's B split).  The pair loads its slice of the
// weights ONCE, as KH * KW * C / 64 swizzled [otile / 2 x 64] sub-tiles
// (147 KB per CTA for 3 x 3 x 128 -> 128), and keeps them for every tile it
// computes, so the mainloop streams only the input.
//
// Input reuse across the horizontal taps: for one (kh, 64-channel block) the
// producer loads ONE box of 128 + KW - 1 pixels (rounded up to 8 rows) at
// (c0, w0 - pw, h + kh - ph, b); the KW taps read it through descriptors whose
// start moves down by kw rows (kw x 128 B).  The 128-byte swizzle is a
// function of the shared-memory address and rows are 128 B apart inside the
// 1024-byte atoms, so row i of the shifted operand is row i + kw of the box.
// Per (kh, c block) a CTA stages 17 KB for KW x 4 MMAs of 256 x otile x 16:
// at otile = 128 that is 22 bytes of shared-memory fill per tensor-core clock,
// against 96 for the weights-streaming 128 x 256 conv of conv.cu.
//
// Zero padding, and the pixels past the end of a row in the last tile, read
// zeros through TMA out-of-bounds fill; pads may differ per side (the caller
// gives the offset and the output extent).
//
// Ghost rows (the halo of an image axis sharded over ranks): the input rows
// may continue above and below the caller's tensor in a second, small tensor
// G [B][gtop + gbot][W][C] (the neighbours' rows, exchanged beforehand).  A
// tap row r < 0 reads G row r + gtop, a row r >= H reads G row gtop + r - H,
// all others read the input itself, so the haloed input is never assembled in
// memory.
//
// Warps (192 threads): 0 TMA producer, 1 MMA issuer (leader CTA) + TMEM owner,
// 2..5 epilogue (TMEM lane quadrant warp % 4: one pixel per thread, its otile
// channels as contiguous 32-byte stores).  Two TMEM accumulators of otile
// columns: the epilogue of tile i overlaps the MMAs of tile i + 1.  Every wait
// is bounded (ptx.cuh); a timed-out kernel records a code, drains its own
// copies, frees TMEM and returns.
//
// Replaces the reference's halo-padded F.conv2d (src/torch_einshard/conv.py:46-53,
// cuDNN) on the einconv path.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <string.h>

#include "conv.h"
#include "gemm_tc.cuh"
#include "tma_desc.h"

namespace es {

namespace {

constexpr int kPairPx = 256;                 // output pixels per pair tile
constexpr int kCtaPx = 128;                  // ... per CTA
constexpr int kARows = kCtaPx + 8;           // A box rows: room for KW - 1 <= 8 extra pixels
constexpr int kAStage = kARows * 128;        // 17 KB per stage (64 channels = 128 B per pixel)
constexpr int kPStages = 4;
constexpr int kPThreads = 192;
constexpr int kSmemMax = 232448;             // opt-in dynamic shared memory per block
constexpr int kStateBytes = 256;
constexpr int kWeightBudget = kSmemMax - 1024 - kPStages * kAStage - kStateBytes;

struct PairState {
  uint64_t full[kPStages];
  uint64_t empty[kPStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t wfull;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int consumed;
};
static_assert(sizeof(PairState) <= kStateBytes, "PairState");

struct PairShape {
  int B, C, O, KH, KW;
  int ph, pw;         // input offset of output pixel (0, 0) is (-ph, -pw)
  int Hout, Wout;
  int out_wpitch, out_w0;  // output rows hold out_wpitch pixels; computed column w goes to w + out_w0
  int otile;          // output channels per tile (MMA N), multiple of 16
  int n_otiles;       // O / otile
  int wtiles;         // pair tiles per output row
  int ptiles;         // pixel tiles: B * Hout * wtiles
  int cblocks;        // C / 64
  int arows;          // rows of each A box (128 + KW - 1 rounded up to 8)
  int rows_x;         // input rows per image in the input tensor
  int gtop, gbot;     // ghost rows above and below it, in G (0: none)
  int tmem_cols;
  int in_bf16;
  int v8;             // output 32-byte aligned: 256-bit stores
  int* err;
  // optional wait-cycle counters: [0] MMA-warp cycles, [1] of them waiting for a
  // filled stage, [2] waiting for a free accumulator, [3] producer cycles,
  // [4] of them waiting for a free stage, [5] epilogue cycles waiting for a
  // full accumulator (warp 2 of each CTA), [6] epilogue cycles in all
  unsigned long long* prof;
};

__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int c0,
                                                 int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar_cluster_addr)
      : "memory");
}

// The KW x 4 MMAs of one (kh, channel block) stage.  `ad`: descriptor of the
// stage's input box; `bd`: descriptor of tap (kh, 0)'s weight sub-tile; `bstep`:
// descriptor units (16 B) between the taps' sub-tiles.  Descriptors advance by
// plain adds of the start-address field (kw rows = kw x 8 units, a K16 step = 2
// units), so the single issuing thread spends a few instructions per MMA: at
// N = 128 an M = 256 MMA keeps the tensor pipe busy for only 64 cycles.
template <int KWc>
__device__ __forceinline__ void issue_stage(uint32_t d_tmem, uint64_t ad, uint64_t bd, uint32_t bstep, int kw_n,
                                            uint32_t idesc, uint32_t& accum) {
#pragma unroll
  for (int kw = 0; kw < (KWc > 0 ? KWc : 9); ++kw) {
    if (KWc == 0 && kw >= kw_n) break;
#pragma unroll
    for (int k = 0; k < kBK / kUmmaK; ++k) {
      umma_f16_pair(d_tmem, ad + static_cast<uint64_t>(kw * 8 + k * 2),
                    bd + static_cast<uint64_t>(kw * bstep + k * 2), idesc, accum);
      accum = 1u;
    }
  }
}

// 32 fp32 values -> 32 bf16/fp16 at p (32-byte aligned) as two 256-bit stores:
// every store writes whole 32-byte sectors.
template <typename OutT>
__device__ __forceinline__ void store32_v8(OutT* p, const uint32_t (&r)[32]) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float a = __uint_as_float(r[2 * i]), b = __uint_as_float(r[2 * i + 1]);
    w[i] = std::is_same<OutT, __nv_bfloat16>::value ? pack_bf16(a, b) : pack_f16(a, b);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h)
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p + 16 * h), "r"(w[8 * h]),
                 "r"(w[8 * h + 1]), "r"(w[8 * h + 2]), "r"(w[8 * h + 3]), "r"(w[8 * h + 4]), "r"(w[8 * h + 5]),
                 "r"(w[8 * h + 6]), "r"(w[8 * h + 7])
                 : "memory");
}

// Pixel tile p of output-channel tile `ot` -> image, output row, first column of this CTA.
struct PixTile {
  int b, h, w0;
};
__device__ __forceinline__ PixTile pix_tile(const PairShape& s, int p, int rank) {
  const int wt = p % s.wtiles;
  const int r = p / s.wtiles;
  return {r / s.Hout, r % s.Hout, wt * kPairPx + rank * kCtaPx};
}

template <typename OutT>
__global__ void __launch_bounds__(kPThreads, 1)
    conv_pair_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmG,
                     const PairShape s, OutT* __restrict__ out, const float* __restrict__ bias) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                                  // kPStages x 17 KB
  uint8_t* sW = smem + kPStages * kAStage;             // resident weights, 1024-byte aligned sub-tiles
  const int wsub = (s.otile / 2) * 128;                // one [otile / 2 x 64] sub-tile
  const int nsub = s.KH * s.KW * s.cblocks;
  PairState* st = reinterpret_cast<PairState*>(sW + nsub * wsub);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = static_cast<int>(cluster_id_x());
  const int nclusters = static_cast<int>(nclusters_x());
  const int per_ot = nclusters / s.n_otiles;          // clusters per output-channel tile
  const int ot = cluster % s.n_otiles;
  const int first = cluster / s.n_otiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(&st->full[i], 1);
      mbar_init(&st->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&st->tfull[i], 1);
      mbar_init(&st->tempty[i], 8);  // 4 epilogue warps per CTA
    }
    mbar_init(&st->wfull, 1);
    mbar_init(&st->drain, 1);
    st->abort_flag = 0;
    st->consumed = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc_pair(&st->tmem_base, s.tmem_cols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = st->tmem_base;
  volatile int* abort_flag = &st->abort_flag;
  const uint32_t full_leader0 = map_to_cta(&st->full[0], 0);
  const uint32_t tempty_leader0 = map_to_cta(&st->tempty[0], 0);
  const int abytes = s.arows * 128;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    uint32_t it = 0;
    long long p_wait = 0;
    const long long p_start = clock64();
    if (lane == 0) {
      const uint32_t wbar = map_to_cta(&st->wfull, 0);
      if (leader) mbar_arrive_expect_tx(&st->wfull, 2u * static_cast<uint32_t>(nsub * wsub));
      const int o0 = ot * s.otile + static_cast<int>(rank) * (s.otile / 2);
      for (int t = 0; t < s.KH * s.KW; ++t)
        for (int cb = 0; cb < s.cblocks; ++cb)
          tma_load_3d_pair(sW + (t * s.cblocks + cb) * wsub, &tmW, wbar, t * s.C + cb * kBK, o0, 0);
    }
    __syncwarp();
    for (int p = first; p < s.ptiles; p += per_ot) {
      const PixTile pt = pix_tile(s, p, static_cast<int>(rank));
      for (int kh = 0; kh < s.KH; ++kh) {
        for (int cb = 0; cb < s.cblocks; ++cb, ++it) {
          const int stg = it % kPStages;
          const uint32_t ph = (it / kPStages) & 1u;
          const long long t_w = s.prof ? clock64() : 0;
          if (!mbar_wait_lane0(&st->empty[stg], ph ^ 1u, abort_flag, s.err, kErrWaitEmpty)) goto producer_done;
          if (s.prof) p_wait += clock64() - t_w;
          if (lane == 0) {
            if (leader) mbar_arrive_expect_tx(&st->full[stg], 2u * static_cast<uint32_t>(abytes));
            // input row of this tap: the tensor itself, a ghost row, or zero fill
            const int r = pt.h + kh - s.ph;
            const CUtensorMap* map = &tmX;
            int row = r;
            if (r < 0 && r >= -s.gtop) {
              map = &tmG;
              row = r + s.gtop;
            } else if (r >= s.rows_x && r < s.rows_x + s.gbot) {
              map = &tmG;
              row = s.gtop + r - s.rows_x;
            }
            tma_load_4d_pair(sA + stg * kAStage, map, full_leader0 + stg * 8, cb * kBK, pt.w0 - s.pw, row, pt.b);
          }
          __syncwarp();
        }
      }
    }
  producer_done:
    __syncwarp();
    if (s.prof && lane == 0) {
      atomicAdd(&s.prof[3], static_cast<unsigned long long>(clock64() - p_start));
      atomicAdd(&s.prof[4], static_cast<unsigned long long>(p_wait));
    }
    if (*abort_flag && leader && lane == 0) {
      // loads in flight must land before the CTA exits (bounded waits)
      int dummy_abort = 0;
      mbar_wait(&st->wfull, 0, &dummy_abort, nullptr, 0);
      const uint32_t consumed = static_cast<uint32_t>(*reinterpret_cast<volatile int*>(&st->consumed));
      for (uint32_t j = consumed; j < it; ++j) {
        dummy_abort = 0;
        mbar_wait(&st->full[j % kPStages], (j / kPStages) & 1u, &dummy_abort, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    // one thread runs the whole loop: no warp-wide votes between stages
    if (leader && lane == 0) {
      const uint32_t idesc = umma_idesc_f16(2 * kCtaPx, s.otile, s.in_bf16, 0, 0);
      const uint64_t adesc0 = umma_desc_sw128(smem_u32(sA), 16u, 1024u);
      const uint64_t wdesc0 = umma_desc_sw128(smem_u32(sW), 16u, 1024u);
      const uint32_t bstep = static_cast<uint32_t>(s.cblocks * wsub) >> 4;
      uint32_t it = 0, tc = 0;
      bool issued_any = false;
      long long w_full = 0, w_empty = 0;
      const long long m_start = clock64();
      if (!mbar_wait(&st->wfull, 0, abort_flag, s.err, kErrWaitFull)) goto mma_done;
      for (int p = first; p < s.ptiles; p += per_ot, ++tc) {
        const uint32_t acc = tc & 1u;
        const uint32_t aph = (tc >> 1) & 1u;
        const long long t_e = s.prof ? clock64() : 0;
        if (!mbar_wait(&st->tempty[acc], aph ^ 1u, abort_flag, s.err, kErrWaitTmemEmpty)) goto mma_done;
        if (s.prof) w_empty += clock64() - t_e;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * s.otile;
        uint32_t accum = 0u;  // the tile's first MMA overwrites the accumulator
        for (int kh = 0; kh < s.KH; ++kh) {
          for (int cb = 0; cb < s.cblocks; ++cb, ++it) {
            const int stg = it % kPStages;
            const uint32_t ph = (it / kPStages) & 1u;
            const long long t_f = s.prof ? clock64() : 0;
            if (!mbar_wait(&st->full[stg], ph, abort_flag, s.err, kErrWaitFull)) goto mma_done;
            if (s.prof) w_full += clock64() - t_f;
            tc_fence_after();
            // tap kw's operand starts kw pixel rows into the box
            const uint64_t ad = adesc0 + static_cast<uint64_t>((stg * kAStage) >> 4);
            const uint64_t bd = wdesc0 + static_cast<uint64_t>(((kh * s.KW * s.cblocks + cb) * wsub) >> 4);
            if (s.KW == 3)
              issue_stage<3>(d_tmem, ad, bd, bstep, 3, idesc, accum);
            else
              issue_stage<0>(d_tmem, ad, bd, bstep, s.KW, idesc, accum);
            umma_commit_pair_mc(&st->empty[stg], 0x3);
            *reinterpret_cast<volatile int*>(&st->consumed) = static_cast<int>(it + 1);
            issued_any = true;
          }
        }
        umma_commit_pair_mc(&st->tfull[acc], 0x3);
      }
    mma_done:
      if (s.prof) {
        atomicAdd(&s.prof[0], static_cast<unsigned long long>(clock64() - m_start));
        atomicAdd(&s.prof[1], static_cast<unsigned long long>(w_full));
        atomicAdd(&s.prof[2], static_cast<unsigned long long>(w_empty));
      }
      if (*abort_flag && issued_any) {
        umma_commit_pair_mc(&st->drain, 0x1);
        int dummy_abort = 0;
        mbar_wait(&st->drain, 0, &dummy_abort, nullptr, 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs, 4 warps)
    const int q = warp & 3;
    uint32_t tc = 0;
    long long e_wait = 0;
    const long long e_start = clock64();
    for (int p = first; p < s.ptiles; p += per_ot, ++tc) {
      const uint32_t acc = tc & 1u;
      const uint32_t aph = (tc >> 1) & 1u;
      const long long t_t = s.prof ? clock64() : 0;
      if (!mbar_wait_sleepy(&st->tfull[acc], aph, abort_flag, s.err, kErrWaitTmemFull, 64)) break;
      if (s.prof) e_wait += clock64() - t_t;
      tc_fence_after();
      const PixTile pt = pix_tile(s, p, static_cast<int>(rank));
      const int w = pt.w0 + q * 32 + lane;
      const bool valid = w < s.Wout;
      OutT* dst = out + ((static_cast<long long>(pt.b) * s.Hout + pt.h) * s.out_wpitch + w + s.out_w0) * s.O +
                  ot * s.otile;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * s.otile;
      for (int ch = 0; ch < s.otile; ch += 32) {
        uint32_t v[32];
        tmem_ld32(taddr + ch, v);
        tmem_ld_wait();
        if (bias != nullptr) {
          const float* bsrc = bias + ot * s.otile + ch;
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) + __ldg(bsrc + i));
        }
        if (valid) {
          if (s.v8)
            store32_v8(dst + ch, v);
          else
            StoreOut<OutT>::store32(dst + ch, v, 0);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + acc * 8);
    }
    if (s.prof && warp == 2 && lane == 0) {
      atomicAdd(&s.prof[5], static_cast<unsigned long long>(e_wait));
      atomicAdd(&s.prof[6], static_cast<unsigned long long>(clock64() - e_start));
    }
  }

  __syncthreads();
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, s.tmem_cols);
  }
}

// Largest output-channel tile whose weight slice fits the budget (0: none).
int pick_otile(const ConvArgs& a) {
  for (int ot : {128, 64, 32, 16}) {
    if (ot > a.O || a.O % ot) continue;
    const long long bytes = static_cast<long long>(a.KH) * a.KW * (a.C / kBK) * (ot / 2) * 128;
    if (bytes <= kWeightBudget) return ot;
  }
  return 0;
}

template <typename OutT>
int launch_pair(const ConvArgs& a, int otile, cudaStream_t stream) {
  const CUtensorMapDataType dt = a.dtype == kDtypeBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int K = a.KH * a.KW * a.C;
  PairShape s;
  s.B = a.B;
  s.C = a.C;
  s.O = a.O;
  s.KH = a.KH;
  s.KW = a.KW;
  s.ph = a.ph + a.gtop;  // tap rows in the input tensor's coordinates
  s.rows_x = a.Hin;
  s.gtop = a.gtop;
  s.gbot = a.gbot;
  s.pw = a.pw;
  s.Hout = conv_hout(a);
  s.Wout = conv_wout(a);
  s.out_wpitch = a.out_wpitch > 0 ? a.out_wpitch : s.Wout;
  s.out_w0 = a.out_w0;
  s.otile = otile;
  s.n_otiles = a.O / otile;
  s.wtiles = (s.Wout + kPairPx - 1) / kPairPx;
  s.ptiles = a.B * s.Hout * s.wtiles;
  s.cblocks = a.C / kBK;
  s.arows = kCtaPx + ((a.KW - 1 + 7) / 8) * 8;
  s.tmem_cols = 2 * otile < 32 ? 32 : 2 * otile;
  s.in_bf16 = a.dtype == kDtypeBF16 ? 1 : 0;
  s.err = a.err;
  s.prof = a.prof;
  s.v8 = (reinterpret_cast<uintptr_t>(a.out) & 31) == 0 ? 1 : 0;
  // X: NHWC input, dims (C, Win, Hin, B), box 64 channels x arows pixels
  const uint64_t dims[4] = {static_cast<uint64_t>(a.C), static_cast<uint64_t>(a.Win), static_cast<uint64_t>(a.Hin),
                            static_cast<uint64_t>(a.B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(a.C) * 2, static_cast<uint64_t>(a.Win) * a.C * 2,
                               static_cast<uint64_t>(a.Hin) * a.Win * a.C * 2};
  const uint32_t box[4] = {static_cast<uint32_t>(kBK), static_cast<uint32_t>(s.arows), 1, 1};
  const CUtensorMap mx = make_tmap_nd(a.x, dt, 4, dims, strides, box);
  CUtensorMap mg = mx;
  if (a.gtop + a.gbot > 0) {
    // the ghost rows may be wider than x (ghost_wpitch pixels per row); x's
    // columns start at pixel ghost_w0 of each ghost row
    const int gp = a.ghost_wpitch > 0 ? a.ghost_wpitch : a.Win;
    const uint64_t gdims[4] = {static_cast<uint64_t>(a.C), static_cast<uint64_t>(a.Win),
                               static_cast<uint64_t>(a.gtop + a.gbot), static_cast<uint64_t>(a.B)};
    const uint64_t gstrides[3] = {static_cast<uint64_t>(a.C) * 2, static_cast<uint64_t>(gp) * a.C * 2,
                                  static_cast<uint64_t>(a.gtop + a.gbot) * gp * a.C * 2};
    const void* gbase = static_cast<const uint8_t*>(a.ghosts) + static_cast<size_t>(a.ghost_w0) * a.C * 2;
    mg = make_tmap_nd(gbase, dt, 4, gdims, gstrides, box);
  }
  // W: [O][K] (K-major), box 64 x otile / 2
  const CUtensorMap mw = make_tmap_3d(a.w, dt, 2, K, a.O, 1, K, static_cast<uint64_t>(K) * a.O, kBK,
                                      static_cast<uint32_t>(otile / 2));
  const int nsub = a.KH * a.KW * s.cblocks;
  const int smem = 1024 + kPStages * kAStage + nsub * (otile / 2) * 128 + kStateBytes;
  auto kernel = conv_pair_kernel<OutT>;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int pairs = a.num_sms / 2;
  int per_ot = pairs / s.n_otiles;
  if (per_ot < 1) return -1;
  if (per_ot > s.ptiles) per_ot = s.ptiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * per_ot * s.n_otiles);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(
      cudaLaunchKernelEx(&cfg, kernel, mx, mw, mg, s, reinterpret_cast<OutT*>(a.out), a.bias));
}

}  // namespace

int conv_pair_otile(int C, int O, int KH, int KW) {
  if (C <= 0 || O <= 0 || KH <= 0 || KW < 1 || KW > 9 || C % kBK || O % 16) return 0;
  ConvArgs a;
  a.C = C;
  a.O = O;
  a.KH = KH;
  a.KW = KW;
  return pick_otile(a);
}

bool conv_pair_eligible(const ConvArgs& a) {
  if (a.gtop + a.gbot > 0 && (a.ghosts == nullptr || (reinterpret_cast<uintptr_t>(a.ghosts) & 15) != 0)) return false;
  if (a.out_wpitch > 0 && a.out_w0 + conv_wout(a) > a.out_wpitch) return false;
  return a.C % kBK == 0 && a.KW >= 1 && a.KW <= 9 && a.O % 16 == 0 && a.num_sms >= 2 && pick_otile(a) > 0 &&
         (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && static_cast<long long>(a.C) * a.Win * 2 % 16 == 0;
}

int conv_pair_launch(const ConvArgs& a, cudaStream_t stream) {
  if (check_conv_args(a) || !conv_pair_eligible(a)) return -1;
  const int otile = pick_otile(a);
  return a.dtype == kDtypeBF16 ? launch_pair<__nv_bfloat16>(a, otile, stream) : launch_pair<__half>(a, otile, stream);
}

}  // namespace es
