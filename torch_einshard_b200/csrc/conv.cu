// Implicit-GEMM 2-D convolution on the tcgen05 GEMM mainloop (NHWC, bf16/fp16,
// stride 1, dilation 1), with no im2col tensor in memory.
//
// The convolution is computed transposed, as one GEMM per launch:
//   out^T[o, p] = sum_{kh, kw, c} Wt[o, (kh, kw, c)] * X[b, h + kh - ph, w + kw - pw, c]
// with p = (b, h, w) an output pixel.  GEMM M = output channels (weights are the
// K-major A operand [O][KH*KW*C]), N = output pixels, K = KH*KW*C.  An N tile is
// 256 consecutive output columns w of one output row (b, h); the K loop walks
// (kh, kw, 64-channel block), and for every step the producer issues one 4-D
// TMA load of a [256 w x 64 c] box of the NHWC input at the shifted coordinates
// (c0, w0 + kw - pw, h + kh - ph, b).  Coordinates left of / above / beyond
// the tensor read zeros (TMA fill), which is the zero padding; the channel
// coordinate is always a multiple of 64, so the 16-byte rule holds.  The
// epilogue reads the accumulator tile (channels on TMEM lanes, pixels on
// columns), adds the bias and writes NHWC, one coalesced 2-byte store per lane
// per pixel (lanes are neighbouring channels).
//
// The same kernel computes the input gradient: dX = conv(dY, W') with
// W'[c, kh', kw', o] = W[o, KH-1-kh', KW-1-kw', c] and padding (KH-1, KW-1).
//
// Weight gradient (conv_wgrad_launch): dW[o, (kh, kw, c)] = sum_p dY[p, o] *
// X[p shifted by (kh - ph, kw - pw), c], a GEMM with M = O, N = KH*KW*C and
// K = output pixels (millions), both operands MN-major straight from the NHWC
// tensors.  A K block is 64 consecutive output columns of one output row: one
// [64 o x 64 w] box of dY (4-D map; columns past the row end read zeros, which
// zeroes the whole product there) and, for each 64-wide chunk of the N tile,
// one [64 c x 64 w] box of X at the tap's shifted coordinates (zero fill is the
// padding again).  K is split over the CTAs (split-K): virtual N tile
// vt = split * ntiles + n_tile, so CTAs that run at the same time share the
// rows of dY and X in L2, and each adds its fp32 partial tile into a
// zero-initialised dW with 16-byte vector atomics.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <string.h>

#include "conv.h"
#include "gemm_tc.cuh"
#include "tma_desc.h"

namespace es {

namespace {

struct ConvLoads {
  int C;        // input channels (multiple of 64)
  int KW;       // kernel width
  int Hout;     // output rows per image
  int Wv;       // virtual output width: column tiles per row * 256
  int ph, pw;   // input offset of output pixel (0, 0) is (-ph, -pw)
  __device__ __forceinline__ void load(const GemmShape&, const TileCoord& c, int kb, uint8_t* a, uint8_t* b,
                                       uint64_t* bar, const CUtensorMap* tmA, const CUtensorMap* tmB) const {
    const int k0 = kb * kBK;
    const int tap = k0 / C;
    const int c0 = k0 - tap * C;
    const int kh = tap / KW;
    const int kw = tap - kh * KW;
    tma_load_3d(a, tmA, bar, k0, c.m0, 0);
    const int r = c.n0 / Wv;
    const int w0 = c.n0 - r * Wv;
    const int img = r / Hout;
    const int h = r - img * Hout;
    tma_load_4d(b, tmB, bar, c0, w0 + kw - pw, h + kh - ph, img);
  }
};

template <typename OutT>
struct ConvStoreEpilogue {
  OutT* out;
  const float* bias;  // may be null
  int O, Wout, Wv;
  int tma;            // 1: TMA stores of [64 pixels x 32 channels] boxes through the warp's staging buffer

  __device__ __forceinline__ void setup(int*, const GemmShape&) {}
  __device__ __forceinline__ void finish(const GemmShape&, volatile int*) {}

  // Channels are on TMEM lanes, pixels on columns: each thread holds one channel
  // of 64 consecutive pixels.  The warp's 32 channels x 64 pixels are written
  // into the staging buffer in NHWC order ([pixel][32 channels], 2-byte stores
  // that are conflict-free across the warp), then one TMA store writes the box;
  // the map is (O, Wout, rows), so boxes clip at the end of an output row.
  __device__ __forceinline__ void tile_tma(const EpiTile& et) {
    const int c0 = et.c.m0 + et.q * 32;
    if (c0 >= O) return;  // this warp's channels are all beyond O (no box may start out of range)
    const int o = c0 + et.lane;
    const int r = et.c.n0 / Wv;
    const int w0 = et.c.n0 - r * Wv;
    const float bv = (o < O && bias != nullptr) ? bias[o] : 0.0f;
    OutT* stage = reinterpret_cast<OutT*>(et.stage);
#pragma unroll 1
    for (int sub = 0; sub < kBN / 64; ++sub) {
      const int col0 = w0 + sub * 64;
      if (col0 >= Wout) break;  // uniform across the warp
      uint32_t v0[32], v1[32];
      tmem_ld32(et.tmem + sub * 64, v0);
      tmem_ld32(et.tmem + sub * 64 + 32, v1);
      tmem_ld_wait();
      if (et.lane == 0) bulk_wait_group_read<0>();
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        stage[i * 32 + et.lane] = StoreOut<OutT>::cvt(__uint_as_float(v0[i]) + bv);
        stage[(32 + i) * 32 + et.lane] = StoreOut<OutT>::cvt(__uint_as_float(v1[i]) + bv);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (et.lane == 0) {
        tma_store_3d(et.tmc, et.stage, c0, col0, r);
        bulk_commit_group();
      }
    }
  }

  __device__ __forceinline__ bool tile(const EpiTile& et, const GemmShape&, volatile int*) {
    if (tma && et.tmc != nullptr) {
      tile_tma(et);
      return true;
    }
    const int o = et.c.m0 + et.row;
    const bool ok = o < O;
    const int r = et.c.n0 / Wv;
    const int w0 = et.c.n0 - r * Wv;
    const long long pix0 = static_cast<long long>(r) * Wout + w0;
    const float bv = (ok && bias != nullptr) ? bias[o] : 0.0f;
#pragma unroll 1
    for (int chunk = 0; chunk < kBN / 32; ++chunk) {
      const int col0 = w0 + chunk * 32;
      if (col0 >= Wout) break;  // uniform across the warp
      uint32_t v[32];
      tmem_ld32(et.tmem + chunk * 32, v);
      tmem_ld_wait();
      if (!ok) continue;
      OutT* dst = out + (pix0 + chunk * 32) * O + o;
      const int valid = Wout - col0 < 32 ? Wout - col0 : 32;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < valid) StoreOut<OutT>::store1(dst + static_cast<long long>(i) * O, __uint_as_float(v[i]) + bv);
    }
    return true;
  }
};

template <typename OutT>
int launch(const ConvArgs& a, cudaStream_t stream) {
  const CUtensorMapDataType dt = a.dtype == kDtypeBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int K = a.KH * a.KW * a.C;
  // A: weights [O][K] (K-major), as a 3-D map with one batch
  const CUtensorMap ma = make_tmap_3d(a.w, dt, 2, K, a.O, 1, K, static_cast<uint64_t>(K) * a.O, kBK, kBM);
  // B: NHWC input, dims (C, Win, Hin, B), box 64 channels x 256 columns
  const uint64_t dims[4] = {static_cast<uint64_t>(a.C), static_cast<uint64_t>(a.Win), static_cast<uint64_t>(a.Hin),
                            static_cast<uint64_t>(a.B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(a.C) * 2, static_cast<uint64_t>(a.Win) * a.C * 2,
                               static_cast<uint64_t>(a.Hin) * a.Win * a.C * 2};
  const uint32_t box[4] = {static_cast<uint32_t>(kBK), static_cast<uint32_t>(kBN), 1, 1};
  const CUtensorMap mb = make_tmap_nd(a.x, dt, 4, dims, strides, box);

  const int Hout = conv_hout(a);
  const int Wout = conv_wout(a);
  const int Wv = (Wout + kBN - 1) / kBN * kBN;
  GemmShape s;
  s.M = a.O;
  s.N = a.B * Hout * Wv;
  s.K = K;
  s.batch = 1;
  s.num_m = (a.O + kBM - 1) / kBM;
  s.num_n = s.N / kBN;
  s.num_kb = K / kBK;
  s.a_mn = 0;
  s.b_mn = 0;
  s.in_bf16 = a.dtype == kDtypeBF16 ? 1 : 0;
  s.group_m = 16;
  s.pair = 0;
  s.split = 0;
  s.err = a.err;
  s.prof = nullptr;
  s.sleep_ns = 0;

  ConvLoads loads{a.C, a.KW, Hout, Wv, a.ph, a.pw};
  ConvStoreEpilogue<OutT> epi{reinterpret_cast<OutT*>(a.out), a.bias, a.O, Wout, Wv, 0};
  // output map (O, Wout, B*Hout), box 32 channels x 64 pixels, no swizzle (64-byte rows)
  CUtensorMap mc;
  memset(&mc, 0, sizeof(mc));
  if ((reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && (a.O * 2) % 16 == 0) {
    const uint64_t odims[3] = {static_cast<uint64_t>(a.O), static_cast<uint64_t>(Wout),
                               static_cast<uint64_t>(a.B) * Hout};
    const uint64_t ostrides[2] = {static_cast<uint64_t>(a.O) * 2, static_cast<uint64_t>(Wout) * a.O * 2};
    const uint32_t obox[3] = {32, 64, 1};
    mc = make_tmap_nd(a.out, dt, 3, odims, ostrides, obox, CU_TENSOR_MAP_SWIZZLE_NONE);
    epi.tma = 1;
  }
  auto kernel = gemm_tc_kernel<ConvStoreEpilogue<OutT>, ConvLoads>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1ull)) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    attr_set |= 1ull << dev;
  }
  const long long tiles = static_cast<long long>(s.num_m) * s.num_n;
  const long long grid = (tiles < a.num_sms || a.persistent == 0) ? tiles : a.num_sms;
  kernel<<<static_cast<unsigned>(grid), kThreads, kSmemBytes, stream>>>(ma, mb, mc, s, epi, loads);
  return static_cast<int>(cudaGetLastError());
}

struct WgradLoads {
  int C, KW, taps;   // input channels, kernel width, KH * KW
  int Hout, Hin;     // output rows per image, input rows per image
  int wblocks;       // 64-column blocks per output row
  int ntiles;        // real N tiles
  int kb_per_split;  // K blocks per split
  int ph, pw;
  __device__ __forceinline__ void load(const GemmShape&, const TileCoord& c, int kb, uint8_t* a, uint8_t* b,
                                       uint64_t* bar, const CUtensorMap* tmA, const CUtensorMap* tmB) const {
    const int vt = c.n0 / kBN;
    const int sp = vt / ntiles;
    const int nt = vt - sp * ntiles;
    const long long kbg = static_cast<long long>(sp) * kb_per_split + kb;
    const long long r = kbg / wblocks;
    const int w0 = static_cast<int>(kbg - r * wblocks) * 64;
    const int img = static_cast<int>(r / Hout);  // past the last image: out of range, zero fill
    const int h = static_cast<int>(r - static_cast<long long>(img) * Hout);
    tma_load_4d(a, tmA, bar, c.m0, w0, h, img);
    tma_load_4d(a + 8192, tmA, bar, c.m0 + 64, w0, h, img);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = nt * kBN + 64 * j;
      const int tap = n / C;
      int c0 = n - tap * C, hh = Hin, ww = 0;  // columns past N: a row beyond the input (zeros)
      if (tap < taps) {
        const int kh = tap / KW;
        hh = h + kh - ph;
        ww = w0 + (tap - kh * KW) - pw;
      } else {
        c0 = 0;
      }
      tma_load_4d(b + j * 8192, tmB, bar, c0, ww, hh, img);
    }
  }
};

struct WgradEpilogue {
  float* dw;   // [O][N] fp32, zero-initialised; partial tiles are added atomically
  int O, N, ntiles;

  __device__ __forceinline__ void setup(int*, const GemmShape&) {}
  __device__ __forceinline__ void finish(const GemmShape&, volatile int*) {}

  __device__ __forceinline__ bool tile(const EpiTile& et, const GemmShape&, volatile int*) {
    const int nt = (et.c.n0 / kBN) % ntiles;
    const int n0 = nt * kBN;
    const int o = et.c.m0 + et.row;
    float* drow = dw + static_cast<long long>(o) * N;
#pragma unroll 1
    for (int chunk = 0; chunk < kBN / 32; ++chunk) {
      const int col0 = n0 + chunk * 32;
      if (col0 >= N) break;  // uniform across the warp
      uint32_t v[32];
      tmem_ld32(et.tmem + chunk * 32, v);
      tmem_ld_wait();
      if (o >= O) continue;
      if (col0 + 32 <= N) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          atomicAdd(reinterpret_cast<float4*>(drow + col0 + 4 * i),
                    make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (col0 + i < N) atomicAdd(drow + col0 + i, __uint_as_float(v[i]));
      }
    }
    return true;
  }
};

}  // namespace

const char* check_conv_wgrad_args(const ConvWgradArgs& a) {
  if (a.B <= 0 || a.Hin <= 0 || a.Win <= 0 || a.C <= 0 || a.O <= 0 || a.KH <= 0 || a.KW <= 0)
    return "empty convolution";
  if (a.C % 64 || a.O % 64) return "input and output channels must be multiples of 64";
  if (a.ph < 0 || a.pw < 0 || a.ph_hi < -1 || a.pw_hi < -1) return "negative padding";
  const int Hout = conv_hout(a);
  const int Wout = conv_wout(a);
  if (Hout <= 0 || Wout <= 0) return "empty output";
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.dy) | reinterpret_cast<uintptr_t>(a.dw)) & 15)
    return "operands not 16-byte aligned";
  const long long total_kb = static_cast<long long>(a.B) * Hout * ((Wout + 63) / 64);
  if (total_kb > 0x3fffffffLL) return "too many output pixels";
  return nullptr;
}

int conv_wgrad_launch(const ConvWgradArgs& a, cudaStream_t stream) {
  if (check_conv_wgrad_args(a)) return -1;
  const CUtensorMapDataType dt = a.dtype == kDtypeBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int Hout = conv_hout(a);
  const int Wout = conv_wout(a);
  const int N = a.KH * a.KW * a.C;
  // A: dY (O, Wout, Hout, B), box 64 channels x 64 columns (MN-major: channels contiguous)
  const uint64_t ady[4] = {static_cast<uint64_t>(a.O), static_cast<uint64_t>(Wout), static_cast<uint64_t>(Hout),
                           static_cast<uint64_t>(a.B)};
  const uint64_t asd[3] = {static_cast<uint64_t>(a.O) * 2, static_cast<uint64_t>(Wout) * a.O * 2,
                           static_cast<uint64_t>(Hout) * Wout * a.O * 2};
  const uint32_t box[4] = {64, 64, 1, 1};
  const CUtensorMap ma = make_tmap_nd(a.dy, dt, 4, ady, asd, box);
  // B: X (C, Win, Hin, B), same box
  const uint64_t bx[4] = {static_cast<uint64_t>(a.C), static_cast<uint64_t>(a.Win), static_cast<uint64_t>(a.Hin),
                          static_cast<uint64_t>(a.B)};
  const uint64_t bsd[3] = {static_cast<uint64_t>(a.C) * 2, static_cast<uint64_t>(a.Win) * a.C * 2,
                           static_cast<uint64_t>(a.Hin) * a.Win * a.C * 2};
  const CUtensorMap mb = make_tmap_nd(a.x, dt, 4, bx, bsd, box);
  CUtensorMap mc;
  memset(&mc, 0, sizeof(mc));

  const int wblocks = (Wout + 63) / 64;
  const long long total_kb = static_cast<long long>(a.B) * Hout * wblocks;
  const int num_m = (a.O + kBM - 1) / kBM;
  const int ntiles = (N + kBN - 1) / kBN;
  const int tiles = num_m * ntiles;
  // about two work items per SM, each with at least 16 K blocks
  long long splits = (2LL * a.num_sms) / tiles;
  if (splits < 1) splits = 1;
  if (splits > total_kb / 16) splits = total_kb / 16 > 0 ? total_kb / 16 : 1;
  const long long kb_per_split = (total_kb + splits - 1) / splits;

  GemmShape s;
  s.M = a.O;
  s.N = static_cast<int>(ntiles * splits) * kBN;
  s.K = static_cast<int>(kb_per_split) * kBK;
  s.batch = 1;
  s.num_m = num_m;
  s.num_n = static_cast<int>(ntiles * splits);
  s.num_kb = static_cast<int>(kb_per_split);
  s.a_mn = 1;
  s.b_mn = 1;
  s.in_bf16 = a.dtype == kDtypeBF16 ? 1 : 0;
  s.group_m = num_m;
  s.pair = 0;
  s.split = 0;
  s.err = a.err;
  s.prof = nullptr;
  s.sleep_ns = 0;
  WgradLoads loads{a.C, a.KW, a.KH * a.KW, Hout, a.Hin, wblocks, ntiles, static_cast<int>(kb_per_split), a.ph, a.pw};
  WgradEpilogue epi{a.dw, a.O, N, ntiles};
  auto kernel = gemm_tc_kernel<WgradEpilogue, WgradLoads>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1ull)) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    attr_set |= 1ull << dev;
  }
  const long long items = static_cast<long long>(tiles) * splits;
  const long long grid = items < a.num_sms ? items : a.num_sms;
  kernel<<<static_cast<unsigned>(grid), kThreads, kSmemBytes, stream>>>(ma, mb, mc, s, epi, loads);
  return static_cast<int>(cudaGetLastError());
}

const char* check_conv_args(const ConvArgs& a) {
  if (a.B <= 0 || a.Hin <= 0 || a.Win <= 0 || a.C <= 0 || a.O <= 0 || a.KH <= 0 || a.KW <= 0)
    return "empty convolution";
  if (a.C % kBK) return "input channels must be a multiple of 64";
  if (a.ph < 0 || a.pw < 0 || a.ph_hi < -1 || a.pw_hi < -1) return "negative padding";
  const int Hout = conv_hout(a);
  const int Wout = conv_wout(a);
  if (Hout <= 0 || Wout <= 0) return "empty output";
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.w)) & 15) return "operands not 16-byte aligned";
  const long long n = static_cast<long long>(a.B) * Hout * ((Wout + kBN - 1) / kBN) * kBN;
  if (n / kBN > 0x7fffffffLL / 2) return "too many output tiles";
  return nullptr;
}

int conv_launch(const ConvArgs& a, cudaStream_t stream) {
  if (check_conv_args(a)) return -1;
  if (a.gtop + a.gbot > 0 || a.out_wpitch > 0)  // ghosts and column ranges: pair kernel only
    return conv_pair_eligible(a) ? conv_pair_launch(a, stream) : -1;
  if (a.kernel == 0 && conv_pair_eligible(a)) return conv_pair_launch(a, stream);
  return a.dtype == kDtypeBF16 ? launch<__nv_bfloat16>(a, stream) : launch<__half>(a, stream);
}

}  // namespace es
