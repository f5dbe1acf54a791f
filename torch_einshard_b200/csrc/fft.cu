// Complex64 FFT kernels for sm_100a: power-of-two lengths 2..1024 along one
// axis of a tensor viewed as [outer, n, inner], and the slab-transpose variant
// whose loads pull the transposed data straight from peer GPUs' memory.
//
// Algorithm: n = N1 * N2 (N1 = 2^ceil(log n / 2)).  One CTA owns LPC lines.
//   pass 1  thread t of a line loads x[N2*n1 + t] (n1 < N1) from global memory
//           into registers, runs an N1-point radix-2 DIT FFT in registers,
//           multiplies by the twiddle W_n^(t*k1) and writes row k1 of a padded
//           shared-memory tile;
//   pass 2  thread t loads row t of the tile (N2 values), runs an N2-point
//           FFT in registers and stores X[t + N1*k2] (scaled) to global memory.
// So every element crosses HBM once in and once out, and shared memory holds
// only the transpose between the two register FFTs.  Thread-to-line mapping
// keeps global accesses coalesced: along contiguous lines the lanes walk the
// points, along strided lines they walk neighbouring lines.
//
// Twiddles are a table exp(-+2 pi i j / n), j < n, computed on the host in
// double precision and staged in shared memory per CTA.
//
// Slab variant: the global post-transpose tensor is distributed over the
// communicator's ranks (rank p holds points [p*Sl, (p+1)*Sl) of the FFT axis
// in its symmetric data region, with the other exchanged axis at full
// length).  Each CTA first waits (bounded) until every peer published that
// its data is staged for this epoch, then loads straight from the peers'
// regions over NVLink; the last CTA to finish publishes "done" so that peers
// may overwrite their regions.
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.h"
#include "fft.h"
#include "ptx.cuh"

namespace es {

namespace {

constexpr int kFftThreads = 256;

// Bit reversal of the low BITS bits; folds to a constant for constant x, so
// register arrays indexed with it stay in registers.
template <int BITS>
__device__ __forceinline__ int fft_bitrev(int x) {
  if constexpr (BITS == 0) {
    return 0;
  } else {
    return static_cast<int>(__brev(static_cast<unsigned>(x)) >> (32 - BITS));
  }
}

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// Radix-2 DIT FFT of 2^LOG points in registers; v[i] holds x[bitrev(i)] on
// entry and X[i] on exit.  tw[j] = W_(2^LOGN)^j.  One template instance per
// stage so that every loop bound and register index is a compile-time constant.
template <int S, int LOG, int LOGN, bool INV>
__device__ __forceinline__ void reg_stage(float2 (&v)[1 << LOG], const float2* tw) {
  if constexpr (S <= LOG) {
    constexpr int R = 1 << LOG;
    constexpr int len = 1 << S;
    constexpr int half = len >> 1;
#pragma unroll
    for (int i = 0; i < R; i += len) {
#pragma unroll
      for (int j = 0; j < half; ++j) {
        const float2 a = v[i + j];
        const float2 b = v[i + j + half];
        float2 t;
        if (j == 0) {
          t = b;
        } else if (4 * j == len) {  // W_len^(len/4) = -i (forward) or +i (inverse)
          t = INV ? make_float2(-b.y, b.x) : make_float2(b.y, -b.x);
        } else {
          t = cmul(tw[j << (LOGN - S)], b);
        }
        v[i + j] = make_float2(a.x + t.x, a.y + t.y);
        v[i + j + half] = make_float2(a.x - t.x, a.y - t.y);
      }
    }
    reg_stage<S + 1, LOG, LOGN, INV>(v, tw);
  }
}

template <int LOG, int LOGN, bool INV>
__device__ __forceinline__ void reg_fft(float2 (&v)[1 << LOG], const float2* tw) {
  reg_stage<1, LOG, LOGN, INV>(v, tw);
}

struct PlainLoader {
  const float2* in;
  long long os, ps, is;
  __device__ __forceinline__ long long base(long long o, long long i) const { return o * os + i * is; }
  __device__ __forceinline__ const float2* peer_ptr(int) const { return nullptr; }
  __device__ __forceinline__ float2 load(long long b, int p, const float2* const*) const {
    return __ldg(in + b + p * ps);
  }
};

// Post-transpose tensor spread over ranks; see the file comment.
struct SlabLoader {
  const float2* peer[kMaxRanks];
  int mode;  // 0: peer layout [A, Sl, B, D, C], output [A, S, B, Dl, C]; 1: [A, D, B, Sl, C] -> [A, Dl, B, S, C]
  int log_sl;
  long long B, C, D, Dl, doff, ps;
  __host__ __device__ __forceinline__ long long base(long long o, long long i) const {
    if (mode == 0) {
      const long long dlc = Dl * C;
      const long long b = i / dlc;
      const long long r = i - b * dlc;
      const long long dl = r / C;
      const long long c = r - dl * C;
      return (o << log_sl) * B * D * C + b * D * C + (dl + doff) * C + c;
    }
    const long long dlb = Dl * B;
    const long long a = o / dlb;
    const long long r = o - a * dlb;
    const long long dl = r / B;
    const long long b = r - dl * B;
    return ((((a * D + dl + doff) * B + b)) << log_sl) * C + i;
  }
  __device__ __forceinline__ const float2* peer_ptr(int p) const { return peer[p]; }
  // sp: the peer pointers staged in shared memory (a dynamic index into the
  // kernel parameter array would go through local memory)
  __device__ __forceinline__ float2 load(long long b, int p, const float2* const* sp) const {
    const int r = p >> log_sl;
    const int q = p & ((1 << log_sl) - 1);
    return sp[r][b + q * ps];
  }
};

struct SlabSync {
  int enabled;
  int size;
  int epoch;
  uint32_t arrive_base;
  int* peer_flags[kMaxRanks];
  int* local_flags;  // this rank's flag block (arrive counter, done flag)
  int* err;
  uint64_t timeout_ns;
};

template <int LOG1, int LOG2, bool INV, class Loader>
__global__ void __launch_bounds__(kFftThreads) fft2_kernel(Loader ld, float2* __restrict__ out, long long lines,
                                                           long long inner, long long out_os, long long out_ps,
                                                           long long out_is, const float2* __restrict__ tw_g,
                                                           float scale, int strided, SlabSync sync) {
  constexpr int N1 = 1 << LOG1;
  constexpr int N2 = 1 << LOG2;
  constexpr int LOGN = LOG1 + LOG2;
  constexpr int N = 1 << LOGN;
  constexpr int T = N1 > N2 ? N1 : N2;
  constexpr int LPC = kFftThreads / T;
  constexpr int RP = N2 + 1;                                // row pitch: rows k1 of one line
  constexpr int LP0 = N1 * RP;
  constexpr int LP = LP0 + ((2 - LP0 % 16) + 16) % 16;      // line pitch = 2 (mod 16) complex values
  extern __shared__ float2 fft_smem[];
  float2* tw = fft_smem;
  float2* buf = fft_smem + N;
  __shared__ int s_ok;
  __shared__ const float2* s_peer[kMaxRanks];

  for (int j = threadIdx.x; j < N; j += blockDim.x) tw[j] = tw_g[j];
#pragma unroll
  for (int p = 0; p < kMaxRanks; ++p)  // constant indices: no local-memory copy of the parameters
    if (threadIdx.x == p) s_peer[p] = ld.peer_ptr(p);
  if (threadIdx.x == 0) {
    int ok = 1;
    if (sync.enabled) {
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < sync.size && ok)
          ok = wait_flag_geq_for(sync.peer_flags[p] + kFlagStaged, sync.epoch, sync.err, kErrWaitPeerFlag, sync.timeout_ns) ? 1 : 0;
    }
    s_ok = ok;
  }
  __syncthreads();
  const bool ok = s_ok != 0;

  const int tid = threadIdx.x;
  const int line = strided ? tid % LPC : tid / T;
  const int t = strided ? tid / LPC : tid % T;
  const long long gl = static_cast<long long>(blockIdx.x) * LPC + line;
  const bool active = ok && gl < lines;
  const long long o = active ? gl / inner : 0;
  const long long i = active ? gl - o * inner : 0;
  float2* lb = buf + line * LP;

  if (active && t < N2) {
    const long long b = ld.base(o, i);
    float2 v[N1];
#pragma unroll
    for (int n1 = 0; n1 < N1; ++n1) v[fft_bitrev<LOG1>(n1)] = ld.load(b, n1 * N2 + t, s_peer);
    reg_fft<LOG1, LOGN, INV>(v, tw);
#pragma unroll
    for (int k1 = 0; k1 < N1; ++k1) lb[k1 * RP + t] = k1 == 0 ? v[0] : cmul(v[k1], tw[t * k1]);
  }
  __syncthreads();
  if (active && t < N1) {
    float2 v[N2];
#pragma unroll
    for (int n2 = 0; n2 < N2; ++n2) v[fft_bitrev<LOG2>(n2)] = lb[t * RP + n2];
    reg_fft<LOG2, LOGN, INV>(v, tw);
    float2* ob = out + o * out_os + i * out_is;
#pragma unroll
    for (int k2 = 0; k2 < N2; ++k2)
      ob[static_cast<long long>(t + k2 * N1) * out_ps] = make_float2(v[k2].x * scale, v[k2].y * scale);
  }

  if (sync.enabled) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const int prev = atomicAdd(sync.local_flags + kFlagArrive, 1);
      if (static_cast<uint32_t>(prev + 1) - sync.arrive_base == gridDim.x) {
        fence_acq_rel_sys();
        st_release_sys(sync.local_flags + kFlagDone, sync.epoch);
      }
    }
  }
}

template <int LOG1, int LOG2, bool INV, class Loader>
int launch_fft(const Loader& ld, float2* out, long long lines, long long inner, long long out_os, long long out_ps,
               long long out_is, const float2* tw, float scale, const SlabSync& sync, cudaStream_t stream) {
  constexpr int N1 = 1 << LOG1, N2 = 1 << LOG2, N = N1 * N2;
  constexpr int T = N1 > N2 ? N1 : N2;
  constexpr int LPC = kFftThreads / T;
  constexpr int RP = N2 + 1;
  constexpr int LP0 = N1 * RP;
  constexpr int LP = LP0 + ((2 - LP0 % 16) + 16) % 16;
  const size_t smem = static_cast<size_t>(N + LPC * LP) * sizeof(float2);
  auto kern = fft2_kernel<LOG1, LOG2, INV, Loader>;
  static int attr_set[64] = {0};  // per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && dev >= 0 && dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set[dev] = 1;
  }
  const long long blocks = (lines + LPC - 1) / LPC;
  if (blocks <= 0) return 0;
  if (blocks > 0x7fffffffLL) return static_cast<int>(cudaErrorInvalidValue);
  kern<<<static_cast<unsigned>(blocks), kFftThreads, smem, stream>>>(ld, out, lines, inner, out_os, out_ps, out_is, tw,
                                                                     scale, inner > 1 ? 1 : 0, sync);
  return static_cast<int>(cudaGetLastError());
}

template <bool INV, class Loader>
int dispatch(int logn, const Loader& ld, float2* out, long long lines, long long inner, long long out_os,
             long long out_ps, long long out_is, const float2* tw, float scale, const SlabSync& sync,
             cudaStream_t stream) {
  switch (logn) {
#define ES_FFT_CASE(L, A, B) \
  case L:                    \
    return launch_fft<A, B, INV>(ld, out, lines, inner, out_os, out_ps, out_is, tw, scale, sync, stream);
    ES_FFT_CASE(1, 1, 0)
    ES_FFT_CASE(2, 1, 1)
    ES_FFT_CASE(3, 2, 1)
    ES_FFT_CASE(4, 2, 2)
    ES_FFT_CASE(5, 3, 2)
    ES_FFT_CASE(6, 3, 3)
    ES_FFT_CASE(7, 4, 3)
    ES_FFT_CASE(8, 4, 4)
    ES_FFT_CASE(9, 5, 4)
    ES_FFT_CASE(10, 5, 5)
#undef ES_FFT_CASE
    default:
      return static_cast<int>(cudaErrorInvalidValue);
  }
}

int log2_exact(long long n) {
  int l = 0;
  while ((1LL << l) < n) ++l;
  return (1LL << l) == n ? l : -1;
}


// Persistent, software-pipelined variant for local transforms: each CTA walks
// tiles of LPC lines; while it transforms tile i out of shared memory, the
// cp.async copies of tile i + 1 are in flight, so HBM reads overlap the
// register FFTs and the (direct, coalesced) stores of the previous tile.
// Requires whole tiles: contiguous lines (inner == 1), or LPC neighbouring
// lines (inner % LPC == 0) so a tile is one 8*LPC-byte run per point.
template <int LOG1, int LOG2, bool INV>
__global__ void __launch_bounds__(kFftThreads) fft2_pipelined_kernel(const float2* __restrict__ in,
                                                                     float2* __restrict__ out, long long tiles,
                                                                     long long inner, long long os, long long ps,
                                                                     const float2* __restrict__ tw_g, float scale,
                                                                     int strided) {
  constexpr int N1 = 1 << LOG1;
  constexpr int N2 = 1 << LOG2;
  constexpr int LOGN = LOG1 + LOG2;
  constexpr int N = 1 << LOGN;
  constexpr int T = N1 > N2 ? N1 : N2;
  constexpr int LPC = kFftThreads / T;
  constexpr int RP = N2 + 1;
  constexpr int LP0 = N1 * RP;
  constexpr int LP = LP0 + ((2 - LP0 % 16) + 16) % 16;
  constexpr int TILE = N * LPC;              // complex values per tile
  constexpr int CHUNKS = TILE / 2;           // 16-byte pieces per tile
  extern __shared__ float2 fft_smem[];
  float2* tw = fft_smem;
  float2* buf = tw + N;                      // transpose tile (LPC * LP)
  float2* inb = buf + LPC * LP;              // two input tiles, 16-byte aligned
  for (int j = threadIdx.x; j < N; j += blockDim.x) tw[j] = tw_g[j];

  const int tid = threadIdx.x;
  const int line = strided ? tid % LPC : tid / T;
  const int t = strided ? tid / LPC : tid % T;

  // tile k: lines [k*LPC, (k+1)*LPC) = outer o, inner [i0, i0 + LPC) (strided) or outer k*LPC.. (contiguous)
  auto issue = [&](long long k, int slot) {
    float2* dst = inb + slot * TILE;
    if (strided) {
      const long long l0 = k * LPC;
      const long long o = l0 / inner;
      const long long i0 = l0 - o * inner;
      const float2* src = in + o * os + i0;
      // point p, pair q (two neighbouring lines): global src + p*ps + 2q, smem p*LPC + 2q
      for (int c = tid; c < CHUNKS; c += kFftThreads) {
        const int p = c / (LPC / 2);
        const int q = c - p * (LPC / 2);
        cp_async16(dst + p * LPC + 2 * q, src + p * ps + 2 * q);
      }
    } else {
      const float2* src = in + k * LPC * os;  // os = N for contiguous lines
      for (int c = tid; c < CHUNKS; c += kFftThreads) cp_async16(dst + 2 * c, src + 2 * c);
    }
    cp_async_commit();
  };

  long long k = blockIdx.x;
  if (k < tiles) issue(k, 0);
  int slot = 0;
  for (; k < tiles; k += gridDim.x, slot ^= 1) {
    const long long next = k + gridDim.x;
    if (next < tiles) {
      issue(next, slot ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // tile k (and the twiddles) visible to every thread
    const float2* tin = inb + slot * TILE;
    float2* lb = buf + line * LP;
    if (t < N2) {
      float2 v[N1];
#pragma unroll
      for (int n1 = 0; n1 < N1; ++n1) {
        const int p = n1 * N2 + t;
        v[fft_bitrev<LOG1>(n1)] = strided ? tin[p * LPC + line] : tin[line * N + p];
      }
      reg_fft<LOG1, LOGN, INV>(v, tw);
#pragma unroll
      for (int k1 = 0; k1 < N1; ++k1) lb[k1 * RP + t] = k1 == 0 ? v[0] : cmul(v[k1], tw[t * k1]);
    }
    __syncthreads();
    if (t < N1) {
      float2 v[N2];
#pragma unroll
      for (int n2 = 0; n2 < N2; ++n2) v[fft_bitrev<LOG2>(n2)] = lb[t * RP + n2];
      reg_fft<LOG2, LOGN, INV>(v, tw);
      const long long gl = k * LPC + line;
      const long long o = gl / inner;
      const long long i = gl - o * inner;
      float2* ob = out + o * os + i;
#pragma unroll
      for (int k2 = 0; k2 < N2; ++k2)
        ob[static_cast<long long>(t + k2 * N1) * ps] = make_float2(v[k2].x * scale, v[k2].y * scale);
    }
    __syncthreads();  // the transpose tile and input slot are reused two tiles later
  }
}

template <int LOG1, int LOG2, bool INV>
int launch_fft_pipelined(const FftLines& f, long long lines, cudaStream_t stream) {
  constexpr int N1 = 1 << LOG1, N2 = 1 << LOG2, N = N1 * N2;
  constexpr int T = N1 > N2 ? N1 : N2;
  constexpr int LPC = kFftThreads / T;
  constexpr int RP = N2 + 1;
  constexpr int LP0 = N1 * RP;
  constexpr int LP = LP0 + ((2 - LP0 % 16) + 16) % 16;
  const size_t smem = static_cast<size_t>(N + LPC * LP + 2 * N * LPC) * sizeof(float2);
  auto kern = fft2_pipelined_kernel<LOG1, LOG2, INV>;
  static int attr_set[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set[dev] = 1;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long tiles = lines / LPC;
  const long long grid = tiles < sms ? tiles : sms;
  kern<<<static_cast<unsigned>(grid), kFftThreads, smem, stream>>>(f.in, f.out, tiles, f.inner, f.in_os, f.in_ps, f.tw,
                                                                   f.scale, f.inner > 1 ? 1 : 0);
  return static_cast<int>(cudaGetLastError());
}

// The pipelined kernel covers 1024-point lines (the shape that dominates the
// 3-D transforms); out-of-place or in-place, whole tiles only.
bool pipelined_ok(const FftLines& f) {
  if (log2_exact(f.n) != 10) return false;
  constexpr int kLpc = kFftThreads / 32;
  if (f.in_is != 1 || f.out_is != 1 || f.in_os != f.out_os || f.in_ps != f.out_ps) return false;
  if (f.inner == 1) return f.in_ps == 1 && f.in_os == f.n && (f.outer % kLpc) == 0 &&
                           ((reinterpret_cast<uintptr_t>(f.in) & 15) == 0);
  return (f.inner % kLpc) == 0 && ((reinterpret_cast<uintptr_t>(f.in) & 15) == 0) && (f.in_ps % 2) == 0 &&
         (f.in_os % 2) == 0;
}

}  // namespace

bool fft_supported(long long n) {
  const int l = log2_exact(n);
  return l >= 1 && l <= kFftMaxLog;
}

long long fft_grid(long long n, long long lines) {
  const int logn = log2_exact(n);
  const int t = 1 << ((logn + 1) / 2);
  const int lpc = kFftThreads / t;
  return (lines + lpc - 1) / lpc;
}

int fft_lines(const FftLines& f, cudaStream_t stream) {
  const int logn = log2_exact(f.n);
  if (logn < 1 || logn > kFftMaxLog) return static_cast<int>(cudaErrorInvalidValue);
  const long long lines = f.outer * f.inner;
  if (f.pipelined && pipelined_ok(f) && f.in != f.out) {
    return f.inverse ? launch_fft_pipelined<5, 5, true>(f, lines, stream)
                     : launch_fft_pipelined<5, 5, false>(f, lines, stream);
  }
  PlainLoader ld{f.in, f.in_os, f.in_ps, f.in_is};
  SlabSync sync{};
  return f.inverse ? dispatch<true>(logn, ld, f.out, lines, f.inner, f.out_os, f.out_ps, f.out_is, f.tw, f.scale, sync,
                                    stream)
                   : dispatch<false>(logn, ld, f.out, lines, f.inner, f.out_os, f.out_ps, f.out_is, f.tw, f.scale,
                                     sync, stream);
}

__global__ void publish_kernel(int* flag, int value) {
  fence_acq_rel_sys();
  st_release_sys(flag, value);
}

__global__ void wait_peers_kernel(const CommDev c, int slot, int target) {
  if (threadIdx.x != 0) return;
  for (int p = 0; p < c.size; ++p) {
    if (p == c.rank) continue;
    if (!wait_flag_geq_for(reinterpret_cast<int*>(c.flags[p]) + slot, target, c.err, kErrWaitPeerFlag, c.timeout_ns)) return;
  }
}

int comm_wait_peers(const CommDev& c, int slot, int target, cudaStream_t stream) {
  wait_peers_kernel<<<1, 32, 0, stream>>>(c, slot, target);
  return static_cast<int>(cudaGetLastError());
}

namespace {

// Output line geometry of the slab exchange: lines of length n, `inner`
// neighbouring lines per outer index, output strides (outer, point, inner).
struct SlabLines {
  long long lines, inner, os, ps, is;
};

SlabLines slab_lines(const FftSlab& f) {
  if (f.mode == 0) {  // output [A, S, B, Dl, C]
    const long long inner = f.B * f.Dl * f.C;
    return {f.A * inner, inner, f.n * inner, inner, 1};
  }
  // output [A, Dl, B, S, C]
  return {f.A * f.Dl * f.B * f.C, f.C, f.n * f.C, f.C, 1};
}

SlabLoader slab_loader(const FftSlab& f, int log_sl) {
  SlabLoader ld{};
  ld.mode = f.mode;
  ld.log_sl = log_sl;
  ld.B = f.B;
  ld.C = f.C;
  ld.D = f.D;
  ld.Dl = f.Dl;
  ld.doff = f.doff;
  ld.ps = f.mode == 0 ? f.B * f.D * f.C : f.C;
  return ld;
}

}  // namespace

int fft_slab_sources(const FftSlab& f, int size, long long* out_off, int* src_rank, long long* src_off) {
  const int log_sl = log2_exact(f.n / size);
  if (log2_exact(f.n) < 1 || log_sl < 0 || f.n % size) return -1;
  const SlabLoader ld = slab_loader(f, log_sl);
  const SlabLines g = slab_lines(f);
  long long k = 0;
  for (long long l = 0; l < g.lines; ++l) {
    const long long o = l / g.inner, i = l - (l / g.inner) * g.inner;
    const long long b = ld.base(o, i);
    for (long long p = 0; p < f.n; ++p, ++k) {
      out_off[k] = o * g.os + i * g.is + p * g.ps;
      src_rank[k] = static_cast<int>(p >> log_sl);
      src_off[k] = b + (p & ((1LL << log_sl) - 1)) * ld.ps;
    }
  }
  return 0;
}

int fft_slab(const CommDev& c, const FftSlab& f, cudaStream_t stream) {
  const int logn = log2_exact(f.n);
  const int log_sl = log2_exact(f.n / c.size);
  if (logn < 1 || logn > kFftMaxLog || log_sl < 0 || f.n % c.size) return static_cast<int>(cudaErrorInvalidValue);
  // publish: this rank's region holds its staged input for this epoch
  publish_kernel<<<1, 1, 0, stream>>>(reinterpret_cast<int*>(c.flags[c.rank]) + kFlagStaged, c.epoch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  SlabLoader ld = slab_loader(f, log_sl);
  for (int p = 0; p < c.size; ++p) ld.peer[p] = reinterpret_cast<const float2*>(c.data[p]);
  SlabSync sync{};
  sync.enabled = 1;
  sync.size = c.size;
  sync.epoch = c.epoch;
  sync.arrive_base = c.arrive_base;
  sync.err = c.err;
  sync.timeout_ns = c.timeout_ns;
  for (int p = 0; p < c.size; ++p) sync.peer_flags[p] = reinterpret_cast<int*>(c.flags[p]);
  sync.local_flags = reinterpret_cast<int*>(c.flags[c.rank]);
  const SlabLines g = slab_lines(f);
  const long long lines = g.lines, inner = g.inner, os = g.os, ps = g.ps, is = g.is;
  return f.inverse ? dispatch<true>(logn, ld, f.out, lines, inner, os, ps, is, f.tw, f.scale, sync, stream)
                   : dispatch<false>(logn, ld, f.out, lines, inner, os, ps, is, f.tw, f.scale, sync, stream);
}

}  // namespace es
