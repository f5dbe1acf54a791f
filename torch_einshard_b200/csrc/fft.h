// Complex64 FFT kernels (fft.cu): one axis of a [outer, n, inner] view, and the
// slab-transpose FFT that reads its input from peer GPUs.
#pragma once

#include <cuda_runtime.h>

#include "comm.h"

namespace es {

constexpr int kFftMaxLog = 10;  // lengths 2 .. 1024

struct FftLines {
  const float2* in;
  float2* out;
  long long n, outer, inner;
  long long in_os, in_ps, in_is;     // element strides of outer, point and inner index
  long long out_os, out_ps, out_is;
  const float2* tw;                  // n entries exp(-+2 pi i j / n) for the direction
  float scale;
  int inverse;
  int pipelined = 1;                 // use the persistent cp.async-pipelined kernel where it applies
};

// Slab transpose + FFT along the exchanged axis S (length n, Sl = n / size per
// rank).  Every rank's symmetric data region holds its block with S local:
//   mode 0: [A, Sl, B, D, C] -> output [A, S, B, Dl, C]
//   mode 1: [A, D, B, Sl, C] -> output [A, Dl, B, S, C]
// where this rank's output keeps rows [doff, doff + Dl) of the other axis D.
struct FftSlab {
  float2* out;
  long long n, A, B, C, D, Dl, doff;
  int mode;
  const float2* tw;
  float scale;
  int inverse;
};

bool fft_supported(long long n);
// CTAs of a launch over `lines` lines of length n.
long long fft_grid(long long n, long long lines);
int fft_lines(const FftLines& f, cudaStream_t stream);
// Wait (bounded, one thread) until every peer's flag `slot` reaches `target`.
int comm_wait_peers(const CommDev& c, int slot, int target, cudaStream_t stream);
int fft_slab(const CommDev& c, const FftSlab& f, cudaStream_t stream);
// Host walk of the slab exchange's loads (for tests): for every output element
// in line order, its output offset and the (rank, element offset) it is read
// from in the peers' staged inputs.  Arrays hold lines * n entries.
int fft_slab_sources(const FftSlab& f, int size, long long* out_off, int* src_rank, long long* src_off);

}  // namespace es
