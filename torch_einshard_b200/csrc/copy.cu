// Strided gather: materialise an arbitrary strided view (rank <= 8) into a
// contiguous tensor with one memory-bound kernel.  The host merges dims that
// are contiguous in the source, so the innermost run is as long as possible;
// when that run and both pointers allow it, each thread moves 16-byte vectors,
// otherwise single elements.  Used for einwindow's window tensor (the run is
// the channel dim) and other permuted materialisations.
#include <cuda_runtime.h>
#include <stdint.h>

#include "copy.h"
#include "ptx.cuh"

namespace es {

namespace {

struct CopyGeom {
  int rank;                          // outer dims (rows), innermost last; the run dim is separate
  long long size[kCopyMaxRank];
  long long sstride[kCopyMaxRank];   // source strides in units
  long long run;                     // units per row (contiguous in source and destination)
  long long rows;
};

constexpr int kCopyThreads = 256;
constexpr int kRowsPerThread = 8;

// Each block walks kRowsPerThread groups of rpb rows; a thread owns one column
// (or a stride of columns when the run is longer than the block) of its row and
// advances the row's multi-index like an odometer, so the index arithmetic is
// paid once per thread, not once per element.
template <typename U>
__global__ void __launch_bounds__(kCopyThreads) gather_kernel(const U* __restrict__ src, U* __restrict__ dst,
                                                              CopyGeom g) {
  const long long run = g.run;
  const int rpb = run >= kCopyThreads ? 1 : static_cast<int>(kCopyThreads / run);
  const int r_local = run >= kCopyThreads ? 0 : static_cast<int>(threadIdx.x / run);
  const long long col0 = run >= kCopyThreads ? threadIdx.x : threadIdx.x - static_cast<long long>(r_local) * run;
  if (r_local >= rpb) return;
  long long row = (static_cast<long long>(blockIdx.x) * kRowsPerThread) * rpb + r_local;
  if (row >= g.rows) return;
  long long idx[kCopyMaxRank];
  long long off = 0;
  {
    long long rem = row;
#pragma unroll
    for (int d = kCopyMaxRank - 1; d >= 0; --d) {
      if (d < g.rank) {
        idx[d] = rem % g.size[d];
        rem /= g.size[d];
        off += idx[d] * g.sstride[d];
      }
    }
  }
  const int last = g.rank - 1;
  auto advance = [&]() {  // move this thread's row forward by rpb (odometer over the outer dims)
    row += rpb;
#pragma unroll
    for (int d = kCopyMaxRank - 1; d >= 0; --d) {  // constant indices only: idx stays in registers
      if (d == last) {
        idx[d] += rpb;
        off += rpb * g.sstride[d];
      }
      if (d > 0 && d <= last) {
        while (idx[d] >= g.size[d]) {
          idx[d] -= g.size[d];
          off -= g.size[d] * g.sstride[d];
          idx[d - 1] += 1;
          off += g.sstride[d - 1];
        }
      }
    }
  };
  if (run < kCopyThreads) {
    // one unit per row per thread: gather all rows' offsets, then issue every load
    // before the first store so kRowsPerThread loads are in flight per thread
    long long offs[kRowsPerThread], rows[kRowsPerThread];
#pragma unroll
    for (int j = 0; j < kRowsPerThread; ++j) {
      offs[j] = off;
      rows[j] = row;
      if (j + 1 < kRowsPerThread) advance();
    }
    U vals[kRowsPerThread];
#pragma unroll
    for (int j = 0; j < kRowsPerThread; ++j)
      if (rows[j] < g.rows) vals[j] = src[offs[j] + col0];
#pragma unroll
    for (int j = 0; j < kRowsPerThread; ++j)
      if (rows[j] < g.rows) dst[rows[j] * run + col0] = vals[j];
    return;
  }
  for (int j = 0; j < kRowsPerThread && row < g.rows; ++j) {
    const U* s = src + off;
    U* t = dst + row * run;
    long long c = col0;
    for (; c + 3 * kCopyThreads < run; c += 4 * kCopyThreads) {
      const U v0 = s[c], v1 = s[c + kCopyThreads], v2 = s[c + 2 * kCopyThreads], v3 = s[c + 3 * kCopyThreads];
      t[c] = v0;
      t[c + kCopyThreads] = v1;
      t[c + 2 * kCopyThreads] = v2;
      t[c + 3 * kCopyThreads] = v3;
    }
    for (; c < run; c += kCopyThreads) t[c] = s[c];
    advance();
  }
}

}  // namespace

int strided_gather(const void* src, void* dst, int esize, int rank, const long long* size, const long long* sstride,
                   int, cudaStream_t stream) {
  if (rank < 1 || rank > kCopyMaxRank) return -1;
  // merge dims d and d+1 when stride[d] == size[d+1] * stride[d+1] (contiguous in the source)
  long long sz[kCopyMaxRank], st[kCopyMaxRank];
  int r = 0;
  for (int d = 0; d < rank; ++d) {
    if (size[d] == 1) continue;
    if (r > 0 && st[r - 1] == size[d] * sstride[d]) {
      sz[r - 1] *= size[d];
      st[r - 1] = sstride[d];
    } else {
      sz[r] = size[d];
      st[r] = sstride[d];
      ++r;
    }
  }
  if (r == 0) {
    sz[0] = 1;
    st[0] = 1;
    r = 1;
  }
  const int vec = 16 / esize;
  bool vec_ok = esize <= 16 && 16 % esize == 0 && st[r - 1] == 1 && sz[r - 1] % vec == 0 &&
                ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
  for (int d = 0; d < r - 1; ++d) vec_ok = vec_ok && (st[d] % vec == 0);
  const int unit = vec_ok ? vec : 1;
  CopyGeom g;
  if (st[r - 1] == 1) {  // innermost dim is the contiguous run
    g.run = sz[r - 1] / unit;
    g.rank = r - 1;
  } else {
    g.run = 1;
    g.rank = r;
  }
  g.rows = 1;
  for (int d = 0; d < g.rank; ++d) {
    g.size[d] = sz[d];
    g.sstride[d] = st[d] / unit;
    g.rows *= sz[d];
  }
  const long long rpb = g.run >= 256 ? 1 : 256 / g.run;
  const long long blocks = (g.rows + rpb * 8 - 1) / (rpb * 8);
  if (blocks > 0x7fffffffLL) return -1;
  const unsigned nb = static_cast<unsigned>(blocks < 1 ? 1 : blocks);
  if (unit == vec && esize * unit == 16) {
    gather_kernel<uint4><<<nb, 256, 0, stream>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), g);
  } else if (esize == 1) {
    gather_kernel<uint8_t><<<nb, 256, 0, stream>>>(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), g);
  } else if (esize == 2) {
    gather_kernel<uint16_t><<<nb, 256, 0, stream>>>(static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), g);
  } else if (esize == 4) {
    gather_kernel<uint32_t><<<nb, 256, 0, stream>>>(static_cast<const uint32_t*>(src), static_cast<uint32_t*>(dst), g);
  } else if (esize == 8) {
    gather_kernel<uint2><<<nb, 256, 0, stream>>>(static_cast<const uint2*>(src), static_cast<uint2*>(dst), g);
  } else if (esize == 16) {
    gather_kernel<uint4><<<nb, 256, 0, stream>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), g);
  } else {
    return -1;
  }
  return static_cast<int>(cudaGetLastError());
}

// ------------------------------------------------------------------ cyclic roll

namespace {

// dst = src rolled along several dims at once.  The tensor is viewed as
// [lead dims ..., n, tail]: every rolled dim is a lead dim or n (the last
// rolled dim), tail is the product of the dims after it, moved as one block of
// `tail` units.  Output position (lead index i, c, t) reads source position
// ((i_d - shift_d) mod size_d, (c - shift_n) mod n, t).
struct RollGeom {
  int rank;                       // lead dims, outermost first
  long long size[kCopyMaxRank];
  long long shift[kCopyMaxRank];  // in [0, size)
  long long n, shift_n;           // the last rolled dim
  long long tail;                 // units per block
  long long total;                // units of the tensor
};

template <typename U>
__global__ void __launch_bounds__(256) roll_kernel(const U* __restrict__ src, U* __restrict__ dst, RollGeom g) {
  const long long nth = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < g.total; i += nth) {
    const long long t = i % g.tail;
    long long q = i / g.tail;
    const long long c = q % g.n;
    q /= g.n;
    long long sc = c - g.shift_n;
    if (sc < 0) sc += g.n;
    long long srow = 0, mult = 1;
#pragma unroll
    for (int d = kCopyMaxRank - 1; d >= 0; --d) {
      if (d < g.rank) {
        const long long id = q % g.size[d];
        q /= g.size[d];
        long long sd = id - g.shift[d];
        if (sd < 0) sd += g.size[d];
        srow += sd * mult;
        mult *= g.size[d];
      }
    }
    dst[i] = src[(srow * g.n + sc) * g.tail + t];
  }
}

}  // namespace

int roll_copy(const void* src, void* dst, int esize, int rank, const long long* size, const long long* shift,
              int num_sms, cudaStream_t stream) {
  if (rank < 1 || rank > kCopyMaxRank + 1) return -1;
  int last = -1;
  for (int d = 0; d < rank; ++d)
    if (shift[d] % size[d] != 0) last = d;
  long long total_elems = 1;
  for (int d = 0; d < rank; ++d) total_elems *= size[d];
  if (total_elems == 0) return 0;
  if (last < 0) {  // nothing moves
    return static_cast<int>(cudaMemcpyAsync(dst, src, total_elems * esize, cudaMemcpyDeviceToDevice, stream));
  }
  RollGeom g;
  long long tail = 1;
  for (int d = last + 1; d < rank; ++d) tail *= size[d];
  g.rank = last;
  for (int d = 0; d < last; ++d) {
    g.size[d] = size[d];
    g.shift[d] = ((shift[d] % size[d]) + size[d]) % size[d];
  }
  g.n = size[last];
  g.shift_n = ((shift[last] % size[last]) + size[last]) % size[last];
  const bool aligned = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
  int unit_bytes = esize;
  for (int u : {16, 8, 4}) {
    if (u > esize && (tail * esize) % u == 0 && aligned) {
      unit_bytes = u;
      break;
    }
  }
  g.tail = tail * esize / unit_bytes;
  g.total = total_elems * esize / unit_bytes;
  const long long want = (g.total + 255) / 256;
  const long long cap = static_cast<long long>(num_sms > 0 ? num_sms : 148) * 16;
  const unsigned nb = static_cast<unsigned>(want < 1 ? 1 : (want > cap ? cap : want));
  switch (unit_bytes) {
    case 16: roll_kernel<uint4><<<nb, 256, 0, stream>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), g); break;
    case 8: roll_kernel<uint2><<<nb, 256, 0, stream>>>(static_cast<const uint2*>(src), static_cast<uint2*>(dst), g); break;
    case 4: roll_kernel<uint32_t><<<nb, 256, 0, stream>>>(static_cast<const uint32_t*>(src), static_cast<uint32_t*>(dst), g); break;
    case 2: roll_kernel<uint16_t><<<nb, 256, 0, stream>>>(static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), g); break;
    case 1: roll_kernel<uint8_t><<<nb, 256, 0, stream>>>(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), g); break;
    default: return -1;
  }
  return static_cast<int>(cudaGetLastError());
}

// ------------------------------------------------------------------ bounded-wait probe

namespace {
__global__ void wait_probe_kernel(const int* flag, int target, int* err, long long timeout_ns, int* result) {
  if (threadIdx.x != 0) return;
  result[0] = wait_flag_geq_for(flag, target, err, kErrWaitPeerFlag, static_cast<uint64_t>(timeout_ns)) ? 1 : 0;
}
}  // namespace

int wait_probe(const int* flag, int target, int* err, long long timeout_ns, int* result, cudaStream_t stream) {
  wait_probe_kernel<<<1, 32, 0, stream>>>(flag, target, err, timeout_ns, result);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace es
