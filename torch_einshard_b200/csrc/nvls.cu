// NVLS (NVLink SHARP) collectives over the symmetric heap: see nvls.h for the
// per-block flag protocol.  The sums happen in the NVSwitch (multimem.ld_reduce,
// fp32 accumulation for 16-bit types); results reach every rank with one
// multimem.st.  Per rank and per byte of an all-reduce of N bytes, the links
// carry N/P reduced-load replies and N/P multicast stores out of this GPU, and
// (P-1)/P N of peers' reduced-load requests plus (P-1)/P N of their stores into
// it: about 9/8 N each way at P = 8, against 2 (P-1)/P N for a ring.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "nvls.h"
#include "ptx.cuh"

namespace es {
namespace {

constexpr int kNvlsThreads = 512;
constexpr int kUnroll = 8;  // 16-byte units in flight per thread

// ---------------------------------------------------------------- multimem wrappers

template <int DT>
__device__ __forceinline__ uint4 mm_ld_reduce(const uint8_t* p);

template <>
__device__ __forceinline__ uint4 mm_ld_reduce<0>(const uint8_t* p) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
template <>
__device__ __forceinline__ uint4 mm_ld_reduce<1>(const uint8_t* p) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
template <>
__device__ __forceinline__ uint4 mm_ld_reduce<2>(const uint8_t* p) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ void mm_st(uint8_t* p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void mm_red_add_release(uint32_t* p, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---------------------------------------------------------------- scaling

template <int DT>
__device__ __forceinline__ uint4 scale16(uint4 v, float s);

template <>
__device__ __forceinline__ uint4 scale16<0>(uint4 v, float s) {
  uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&w[i]);
    float2 f = __bfloat1622float2(h);
    h = __floats2bfloat162_rn(f.x * s, f.y * s);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return v;
}
template <>
__device__ __forceinline__ uint4 scale16<1>(uint4 v, float s) {
  uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<__half2*>(&w[i]);
    float2 f = __half22float2(h);
    h = __floats2half2_rn(f.x * s, f.y * s);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return v;
}
template <>
__device__ __forceinline__ uint4 scale16<2>(uint4 v, float s) {
  v.x = __float_as_uint(__uint_as_float(v.x) * s);
  v.y = __float_as_uint(__uint_as_float(v.y) * s);
  v.z = __float_as_uint(__uint_as_float(v.z) * s);
  v.w = __float_as_uint(__uint_as_float(v.w) * s);
  return v;
}

// ---------------------------------------------------------------- block-level protocol

// Block-wide bounded wait until this rank's flag word reaches `target`.
__device__ __forceinline__ bool block_wait(const NvlsDev& d, int slot, uint32_t target) {
  bool ok = true;
  if (threadIdx.x == 0) {
    const uint32_t* f = d.flags + slot;
    if (static_cast<int>(ld_acquire_sys_u32(f) - target) < 0) {
      const uint64_t t0 = global_timer_ns();
      uint32_t nap = 32;
      while (static_cast<int>(ld_acquire_sys_u32(f) - target) < 0) {
        __nanosleep(nap);
        if (nap < 512) nap <<= 1;
        if (global_timer_ns() - t0 > d.timeout_ns) {
          atomicCAS(d.err, 0, kErrWaitPeerFlag);
          ok = false;
          break;
        }
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// Every thread's earlier accesses of this block, then +1 on `slot` of every rank.
__device__ __forceinline__ void block_signal(const NvlsDev& d, int slot) {
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    mm_red_add_release(d.mcflags + slot, 1u);
  }
}

// End of a collective on this rank: the last block to finish adds 1 to the
// done counter of every rank.  A collective starts only when done reaches
// P x (epoch - 1), i.e. every block of every rank finished the previous one:
// the per-block counters alone do not order two collectives whose bytes fall
// to different blocks (the block of a byte depends on the collective's size),
// so without this a late multicast store or reduction of the previous
// collective could meet the next one's staging.
__device__ __forceinline__ void block_done(const NvlsDev& d) {
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    const uint32_t n = atomicAdd(d.flags + kNvlsArrived, 1u) + 1u;
    if (n == static_cast<uint32_t>(d.nblocks) * static_cast<uint32_t>(d.epoch)) {
      fence_acq_rel_sys();
      mm_red_add_release(d.mcflags + kNvlsDone, 1u);
    }
  }
}

__device__ __forceinline__ void unit_range(long long units, long long* u0, long long* u1) {
  const long long per = (units + gridDim.x - 1) / gridDim.x;
  const long long a = static_cast<long long>(blockIdx.x) * per;
  *u0 = a < units ? a : units;
  *u1 = a + per < units ? a + per : units;
}

// 16-byte unit u of a dense byte range of length n: full units are vector
// copies, the last partial one is assembled byte-wise (bytes beyond n read as 0).
__device__ __forceinline__ uint4 load_unit(const uint8_t* src, long long u, long long n) {
  const long long o = u * 16;
  if (o + 16 <= n) return *reinterpret_cast<const uint4*>(src + o);
  uint4 v = make_uint4(0, 0, 0, 0);
  uint8_t* b = reinterpret_cast<uint8_t*>(&v);
  for (long long i = o; i < n; ++i) b[i - o] = src[i];
  return v;
}
__device__ __forceinline__ void store_unit(uint8_t* dst, long long u, long long n, uint4 v) {
  const long long o = u * 16;
  if (o + 16 <= n) {
    *reinterpret_cast<uint4*>(dst + o) = v;
    return;
  }
  const uint8_t* b = reinterpret_cast<const uint8_t*>(&v);
  for (long long i = o; i < n; ++i) dst[i] = b[i - o];
}

// Per-thread loop over units [u0, u1) of this block with kUnroll units in
// flight: each round loads kUnroll units (block-strided) through `ld`, then
// stores them through `st`.
template <class Ld, class St>
__device__ __forceinline__ void unit_loop(long long u0, long long u1, Ld ld, St st) {
  const long long step = blockDim.x;
  for (long long base = u0 + threadIdx.x; base < u1; base += step * kUnroll) {
    uint4 v[kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      const long long u = base + j * step;
      if (u < u1) v[j] = ld(u);
    }
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      const long long u = base + j * step;
      if (u < u1) st(u, v[j]);
    }
  }
}

// ---------------------------------------------------------------- all-reduce

template <int DT>
__global__ void __launch_bounds__(kNvlsThreads) k_nvls_all_reduce(NvlsDev d, const uint8_t* in, uint8_t* out,
                                                                   long long nbytes, float scale, int two_shot) {
  const int b = blockIdx.x;
  const uint32_t P = static_cast<uint32_t>(d.size);
  const long long units = (nbytes + 15) / 16;
  long long u0, u1;
  unit_range(units, &u0, &u1);
  if (!block_wait(d, kNvlsDone, P * static_cast<uint32_t>(d.epoch - 1))) return;
  uint8_t* uc = d.uc;
  const uint8_t* mc = d.mc;
  if (in != nullptr)
    unit_loop(u0, u1, [&](long long u) { return load_unit(in, u, nbytes); },
              [&](long long u, uint4 v) { *reinterpret_cast<uint4*>(uc + u * 16) = v; });
  block_signal(d, kNvlsReady + b);
  if (!block_wait(d, kNvlsReady + b, P * static_cast<uint32_t>(d.epoch))) return;
  const bool scaled = scale != 1.0f;
  if (two_shot) {
    const long long len = u1 - u0;
    const long long s0 = u0 + len * d.rank / d.size;
    const long long s1 = u0 + len * (d.rank + 1) / d.size;
    unit_loop(s0, s1, [&](long long u) { return mm_ld_reduce<DT>(mc + u * 16); },
              [&](long long u, uint4 v) { mm_st(d.mc + u * 16, scaled ? scale16<DT>(v, scale) : v); });
    block_signal(d, kNvlsSeq + b);
    if (!block_wait(d, kNvlsSeq + b, P * static_cast<uint32_t>(d.epoch))) return;
    if (out != nullptr)
      unit_loop(u0, u1, [&](long long u) { return *reinterpret_cast<const uint4*>(uc + u * 16); },
                [&](long long u, uint4 v) { store_unit(out, u, nbytes, v); });
  } else {
    unit_loop(u0, u1, [&](long long u) { return mm_ld_reduce<DT>(mc + u * 16); },
              [&](long long u, uint4 v) { store_unit(out, u, nbytes, scaled ? scale16<DT>(v, scale) : v); });
    block_signal(d, kNvlsSeq + b);
  }
  block_done(d);
}

// ---------------------------------------------------------------- all-gather / reduce-scatter

// Byte position `pos` of shard q's dense layout -> byte offset in the full tensor.
__device__ __forceinline__ long long full_offset(const ShardLayout& L, int q, long long pos) {
  const long long row_bytes = L.len[q] * L.inner_bytes;
  const long long a = pos / row_bytes;
  const long long r = pos - a * row_bytes;
  return a * L.total_rows * L.inner_bytes + L.off[q] * L.inner_bytes + r;
}

__device__ __forceinline__ bool strided_units_ok(const ShardLayout& L, int q, const uint8_t* full) {
  return ((L.len[q] * L.inner_bytes) % 16 == 0) && ((L.off[q] * L.inner_bytes) % 16 == 0) &&
         ((L.total_rows * L.inner_bytes) % 16 == 0) && ((reinterpret_cast<uintptr_t>(full) & 15) == 0);
}

__global__ void __launch_bounds__(kNvlsThreads) k_nvls_all_gather(NvlsDev d, const uint8_t* in, uint8_t* out,
                                                                   ShardLayout L) {
  const int b = blockIdx.x;
  const uint32_t P = static_cast<uint32_t>(d.size);
  if (!block_wait(d, kNvlsDone, P * static_cast<uint32_t>(d.epoch - 1))) return;
  {
    const long long n = L.outer * L.len[d.rank] * L.inner_bytes;
    long long u0, u1;
    unit_range((n + 15) / 16, &u0, &u1);
    uint8_t* dst = d.mc + L.region[d.rank];
    unit_loop(u0, u1, [&](long long u) { return load_unit(in, u, n); },
              [&](long long u, uint4 v) { mm_st(dst + u * 16, v); });
  }
  block_signal(d, kNvlsReady + b);
  if (!block_wait(d, kNvlsReady + b, P * static_cast<uint32_t>(d.epoch))) return;
  for (int q = 0; q < d.size; ++q) {
    const long long n = L.outer * L.len[q] * L.inner_bytes;
    long long u0, u1;
    unit_range((n + 15) / 16, &u0, &u1);
    const uint8_t* src = d.uc + L.region[q];
    if (strided_units_ok(L, q, out)) {
      unit_loop(u0, u1, [&](long long u) { return *reinterpret_cast<const uint4*>(src + u * 16); },
                [&](long long u, uint4 v) { *reinterpret_cast<uint4*>(out + full_offset(L, q, u * 16)) = v; });
    } else {
      const long long e = u1 * 16 < n ? u1 * 16 : n;
      for (long long i = u0 * 16 + threadIdx.x; i < e; i += blockDim.x) out[full_offset(L, q, i)] = src[i];
    }
  }
  block_signal(d, kNvlsSeq + b);
  block_done(d);
}

template <int DT>
__global__ void __launch_bounds__(kNvlsThreads) k_nvls_reduce_scatter(NvlsDev d, const uint8_t* in, uint8_t* out,
                                                                       ShardLayout L, float scale) {
  const int b = blockIdx.x;
  const uint32_t P = static_cast<uint32_t>(d.size);
  if (!block_wait(d, kNvlsDone, P * static_cast<uint32_t>(d.epoch - 1))) return;
  for (int q = 0; q < d.size; ++q) {
    const long long n = L.outer * L.len[q] * L.inner_bytes;
    long long u0, u1;
    unit_range((n + 15) / 16, &u0, &u1);
    uint8_t* dst = d.uc + L.region[q];
    if (strided_units_ok(L, q, in)) {
      unit_loop(u0, u1,
                [&](long long u) {
                  const long long o = u * 16;
                  return o + 16 <= n ? *reinterpret_cast<const uint4*>(in + full_offset(L, q, o)) : make_uint4(0, 0, 0, 0);
                },
                [&](long long u, uint4 v) { *reinterpret_cast<uint4*>(dst + u * 16) = v; });
    } else {
      for (long long u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
        uint4 v = make_uint4(0, 0, 0, 0);
        uint8_t* vb = reinterpret_cast<uint8_t*>(&v);
        for (long long i = u * 16; i < u * 16 + 16 && i < n; ++i) vb[i - u * 16] = in[full_offset(L, q, i)];
        *reinterpret_cast<uint4*>(dst + u * 16) = v;
      }
    }
  }
  block_signal(d, kNvlsReady + b);
  if (!block_wait(d, kNvlsReady + b, P * static_cast<uint32_t>(d.epoch))) return;
  {
    const long long n = L.outer * L.len[d.rank] * L.inner_bytes;
    long long u0, u1;
    unit_range((n + 15) / 16, &u0, &u1);
    const uint8_t* src = d.mc + L.region[d.rank];
    const bool scaled = scale != 1.0f;
    unit_loop(u0, u1, [&](long long u) { return mm_ld_reduce<DT>(src + u * 16); },
              [&](long long u, uint4 v) { store_unit(out, u, n, scaled ? scale16<DT>(v, scale) : v); });
  }
  block_signal(d, kNvlsSeq + b);
  block_done(d);
}

// Wait until every rank finished the NVLS collectives issued so far on this heap
// (the done counter at P * epoch), before other kernels reuse the data region.
__global__ void k_nvls_quiesce(NvlsDev d) {
  if (threadIdx.x != 0) return;
  const uint32_t target = static_cast<uint32_t>(d.size) * static_cast<uint32_t>(d.epoch);
  const uint32_t* f = d.flags + kNvlsDone;
  const uint64_t t0 = global_timer_ns();
  while (static_cast<int>(ld_acquire_sys_u32(f) - target) < 0) {
    if (global_timer_ns() - t0 > d.timeout_ns) {
      atomicCAS(d.err, 0, kErrWaitPeerFlag);
      return;
    }
  }
}

}  // namespace

int nvls_quiesce(const NvlsDev& d, cudaStream_t stream) {
  k_nvls_quiesce<<<1, kNvlsMaxBlocks, 0, stream>>>(d);
  return static_cast<int>(cudaGetLastError());
}

int nvls_all_reduce(const NvlsDev& d, const void* in, void* out, long long nbytes, int dtype, float scale,
                    int two_shot, cudaStream_t stream) {
  const uint8_t* i = static_cast<const uint8_t*>(in);
  uint8_t* o = static_cast<uint8_t*>(out);
  if (dtype == 0)
    k_nvls_all_reduce<0><<<d.nblocks, kNvlsThreads, 0, stream>>>(d, i, o, nbytes, scale, two_shot);
  else if (dtype == 1)
    k_nvls_all_reduce<1><<<d.nblocks, kNvlsThreads, 0, stream>>>(d, i, o, nbytes, scale, two_shot);
  else
    k_nvls_all_reduce<2><<<d.nblocks, kNvlsThreads, 0, stream>>>(d, i, o, nbytes, scale, two_shot);
  return static_cast<int>(cudaGetLastError());
}

int nvls_all_gather(const NvlsDev& d, const void* in, void* out, const ShardLayout& L, cudaStream_t stream) {
  k_nvls_all_gather<<<d.nblocks, kNvlsThreads, 0, stream>>>(d, static_cast<const uint8_t*>(in),
                                                            static_cast<uint8_t*>(out), L);
  return static_cast<int>(cudaGetLastError());
}

int nvls_reduce_scatter(const NvlsDev& d, const void* in, void* out, const ShardLayout& L, int dtype, float scale,
                        cudaStream_t stream) {
  const uint8_t* i = static_cast<const uint8_t*>(in);
  uint8_t* o = static_cast<uint8_t*>(out);
  if (dtype == 0)
    k_nvls_reduce_scatter<0><<<d.nblocks, kNvlsThreads, 0, stream>>>(d, i, o, L, scale);
  else if (dtype == 1)
    k_nvls_reduce_scatter<1><<<d.nblocks, kNvlsThreads, 0, stream>>>(d, i, o, L, scale);
  else
    k_nvls_reduce_scatter<2><<<d.nblocks, kNvlsThreads, 0, stream>>>(d, i, o, L, scale);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace es
