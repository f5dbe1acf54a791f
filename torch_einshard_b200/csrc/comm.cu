// Pull-based NVLink collectives over peer-mapped symmetric buffers.
// See comm.h for the buffer layout and the epoch-flag protocol.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "comm.h"
#include "ptx.cuh"

namespace es {

// ------------------------------------------------------------------ device helpers

__device__ __forceinline__ int* flag_at(const CommDev& c, int rank, int slot) {
  return reinterpret_cast<int*>(c.flags[rank]) + slot;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier on a monotonic local counter; target counts block arrivals.
__device__ bool grid_barrier(const CommDev& c, uint32_t target) {
  bool ok = true;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* ctr = reinterpret_cast<uint32_t*>(flag_at(c, c.rank, kFlagBarrier));
    fence_acq_rel_sys();
    atomicAdd(ctr, 1u);
    const uint64_t t0 = global_timer_ns();
    while (static_cast<int>(ld_acquire_gpu_u32(ctr) - target) < 0) {
      if (global_timer_ns() - t0 > c.timeout_ns) {
        atomicCAS(c.err, 0, kErrWaitPeerFlag);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// Block-level wait until every peer's flag slot reaches `target`.
__device__ bool wait_peers(const CommDev& c, int slot, int target) {
  bool ok = true;
  if (threadIdx.x == 0) {
    for (int p = 0; p < c.size && ok; ++p) {
      if (p == c.rank) continue;
      ok = wait_flag_geq_for(flag_at(c, p, slot), target, c.err, kErrWaitPeerFlag, c.timeout_ns);
    }
  }
  return __syncthreads_and(ok) != 0;
}

__device__ __forceinline__ void publish(const CommDev& c, int slot) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    fence_acq_rel_sys();
    st_release_sys(flag_at(c, c.rank, slot), c.epoch);
  }
}

// Plain contiguous copy, 16 B vectors when possible.
__device__ void copy_bytes(void* dst, const void* src, size_t n) {
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t nth = (size_t)gridDim.x * blockDim.x;
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0) {
    const size_t nv = n / 16;
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (size_t i = tid; i < nv; i += nth) d[i] = s[i];
    for (size_t i = nv * 16 + tid; i < n; i += nth)
      reinterpret_cast<uint8_t*>(dst)[i] = reinterpret_cast<const uint8_t*>(src)[i];
  } else {
    for (size_t i = tid; i < n; i += nth) reinterpret_cast<uint8_t*>(dst)[i] = reinterpret_cast<const uint8_t*>(src)[i];
  }
}

__device__ __forceinline__ int pick_unit(const CopyBox& b, int esize, uintptr_t sbase, uintptr_t dbase) {
  const long long run = (long long)b.dims[3] * esize;
  uintptr_t bits = sbase | dbase | (uintptr_t)b.src_off | (uintptr_t)b.dst_off | (uintptr_t)run;
  for (int i = 0; i < 3; ++i) bits |= (uintptr_t)b.sstr[i] | (uintptr_t)b.dstr[i];
  if ((bits & 15) == 0) return 16;
  if ((bits & 7) == 0) return 8;
  if ((bits & 3) == 0) return 4;
  if ((bits & 1) == 0) return 2;
  return 1;
}

template <int U>
struct UnitT;
template <> struct UnitT<16> { using T = uint4; };
template <> struct UnitT<8> { using T = uint2; };
template <> struct UnitT<4> { using T = uint32_t; };
template <> struct UnitT<2> { using T = uint16_t; };
template <> struct UnitT<1> { using T = uint8_t; };

// Work items of a box: (row, chunk of up to kChunkUnits units of the row).
// Offsets are derived once per item, so long rows cost no per-unit index
// arithmetic and rows shorter than a chunk are one item each.
constexpr long long kChunkUnits = 2048;

template <int U>
__device__ void copy_box_units(const uint8_t* sbase, uint8_t* dbase, const CopyBox& b, int esize) {
  using T = typename UnitT<U>::T;
  const long long nu = (long long)b.dims[3] * esize / U;
  const long long rows = (long long)b.dims[2] * b.dims[1] * b.dims[0];
  if (nu >= 64) {
    const long long nchunk = (nu + kChunkUnits - 1) / kChunkUnits;
    for (long long item = blockIdx.x; item < rows * nchunk; item += gridDim.x) {
      const long long r = item / nchunk;
      const long long c0 = (item - r * nchunk) * kChunkUnits;
      const long long c1 = c0 + kChunkUnits < nu ? c0 + kChunkUnits : nu;
      const long long i2 = r % b.dims[2];
      const long long q = r / b.dims[2];
      const long long i1 = q % b.dims[1];
      const long long i0 = q / b.dims[1];
      const T* s = reinterpret_cast<const T*>(sbase + b.src_off + i0 * b.sstr[0] + i1 * b.sstr[1] + i2 * b.sstr[2]);
      T* d = reinterpret_cast<T*>(dbase + b.dst_off + i0 * b.dstr[0] + i1 * b.dstr[1] + i2 * b.dstr[2]);
      const long long step = blockDim.x;
      for (long long u = c0 + threadIdx.x; u < c1; u += 4 * step) {
        T v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (u + k * step < c1) v[k] = s[u + k * step];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (u + k * step < c1) d[u + k * step] = v[k];
      }
    }
    return;
  }
  const long long total = nu * rows;
  const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long nth = (long long)gridDim.x * blockDim.x;
  for (long long i = tid; i < total; i += nth) {
    long long r = i / nu;
    const long long u = i - r * nu;
    const long long i2 = r % b.dims[2];
    r /= b.dims[2];
    const long long i1 = r % b.dims[1];
    const long long i0 = r / b.dims[1];
    const long long so = b.src_off + i0 * b.sstr[0] + i1 * b.sstr[1] + i2 * b.sstr[2] + u * U;
    const long long dof = b.dst_off + i0 * b.dstr[0] + i1 * b.dstr[1] + i2 * b.dstr[2] + u * U;
    *reinterpret_cast<T*>(dbase + dof) = *reinterpret_cast<const T*>(sbase + so);
  }
}

__device__ void copy_box(const uint8_t* sbase, uint8_t* dbase, const CopyBox& b, int esize) {
  switch (pick_unit(b, esize, reinterpret_cast<uintptr_t>(sbase), reinterpret_cast<uintptr_t>(dbase))) {
    case 16: copy_box_units<16>(sbase, dbase, b, esize); break;
    case 8: copy_box_units<8>(sbase, dbase, b, esize); break;
    case 4: copy_box_units<4>(sbase, dbase, b, esize); break;
    case 2: copy_box_units<2>(sbase, dbase, b, esize); break;
    default: copy_box_units<1>(sbase, dbase, b, esize); break;
  }
}

__device__ __forceinline__ float load_as_float(const uint8_t* p, int dtype) {
  if (dtype == 0) return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
  if (dtype == 1) return __half2float(*reinterpret_cast<const __half*>(p));
  return *reinterpret_cast<const float*>(p);
}
__device__ __forceinline__ void store_float(uint8_t* p, int dtype, float v) {
  if (dtype == 0) *reinterpret_cast<__nv_bfloat16*>(p) = __float2bfloat16_rn(v);
  else if (dtype == 1) *reinterpret_cast<__half*>(p) = __float2half_rn(v);
  else *reinterpret_cast<float*>(p) = v;
}

// dst = scale * sum_p box(peer p) (+ dst if accumulate); element-wise generic path.
__device__ void reduce_box(const CommDev& c, uint8_t* dbase, const CopyBox& b, const CopyPlan& plan) {
  const int es_ = plan.esize;
  const long long n3 = b.dims[3];
  const long long total = n3 * b.dims[2] * b.dims[1] * b.dims[0];
  const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long nth = (long long)gridDim.x * blockDim.x;
  for (long long i = tid; i < total; i += nth) {
    long long r = i / n3;
    const long long u = i - r * n3;
    const long long i2 = r % b.dims[2];
    r /= b.dims[2];
    const long long i1 = r % b.dims[1];
    const long long i0 = r / b.dims[1];
    const long long so = b.src_off + i0 * b.sstr[0] + i1 * b.sstr[1] + i2 * b.sstr[2] + u * es_;
    const long long dof = b.dst_off + i0 * b.dstr[0] + i1 * b.dstr[1] + i2 * b.dstr[2] + u * es_;
    float acc = 0.f;
    for (int p = 0; p < c.size; ++p) {
      const int src = (c.rank + p) % c.size;  // stagger peers to spread NVLink load
      acc += load_as_float(reinterpret_cast<const uint8_t*>(c.data[src]) + so, plan.dtype);
    }
    acc *= plan.scale;
    if (plan.accumulate) acc += load_as_float(dbase + dof, plan.dtype);
    store_float(dbase + dof, plan.dtype, acc);
  }
}

// dst += box(src), element-wise typed (halo gradient scatter-add).
__device__ void acc_copy_box(const uint8_t* sbase, uint8_t* dbase, const CopyBox& b, const CopyPlan& plan) {
  const int es_ = plan.esize;
  const long long n3 = b.dims[3];
  const long long rows = (long long)b.dims[2] * b.dims[1] * b.dims[0];
  const long long nchunk = (n3 + kChunkUnits - 1) / kChunkUnits;
  // items of (row, chunk) as in copy_box_units; short rows are spread over threads
  if (n3 >= 64) {
    for (long long item = blockIdx.x; item < rows * nchunk; item += gridDim.x) {
      const long long r = item / nchunk;
      const long long c0 = (item - r * nchunk) * kChunkUnits;
      const long long c1 = c0 + kChunkUnits < n3 ? c0 + kChunkUnits : n3;
      const long long i2 = r % b.dims[2];
      const long long q = r / b.dims[2];
      const long long i1 = q % b.dims[1];
      const long long i0 = q / b.dims[1];
      const uint8_t* s = sbase + b.src_off + i0 * b.sstr[0] + i1 * b.sstr[1] + i2 * b.sstr[2];
      uint8_t* d = dbase + b.dst_off + i0 * b.dstr[0] + i1 * b.dstr[1] + i2 * b.dstr[2];
      for (long long u = c0 + threadIdx.x; u < c1; u += blockDim.x) {
        const float v = load_as_float(s + u * es_, plan.dtype) * plan.scale + load_as_float(d + u * es_, plan.dtype);
        store_float(d + u * es_, plan.dtype, v);
      }
    }
    return;
  }
  const long long total = n3 * rows;
  const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long nth = (long long)gridDim.x * blockDim.x;
  for (long long i = tid; i < total; i += nth) {
    long long r = i / n3;
    const long long u = i - r * n3;
    const long long i2 = r % b.dims[2];
    r /= b.dims[2];
    const long long i1 = r % b.dims[1];
    const long long i0 = r / b.dims[1];
    const long long so = b.src_off + i0 * b.sstr[0] + i1 * b.sstr[1] + i2 * b.sstr[2] + u * es_;
    const long long dof = b.dst_off + i0 * b.dstr[0] + i1 * b.dstr[1] + i2 * b.dstr[2] + u * es_;
    const float v = load_as_float(sbase + so, plan.dtype) * plan.scale + load_as_float(dbase + dof, plan.dtype);
    store_float(dbase + dof, plan.dtype, v);
  }
}

// ------------------------------------------------------------------ kernels

// src: the bytes staged into this rank's region; local: what boxes with
// src_rank < 0 read (this rank's own data, which need not be staged).
__global__ void __launch_bounds__(512) k_stage_and_run(CommDev c, const void* src, size_t nbytes, size_t stage_off,
                                                       void* dst, CopyPlan plan, int reduce, const void* local) {
  uint32_t bars = 0;
  const uint32_t nb = gridDim.x;
  // peers must be done reading our data region from the previous op
  if (!wait_peers(c, kFlagDone, c.epoch - 1)) return;
  if (nbytes) copy_bytes(reinterpret_cast<uint8_t*>(c.data[c.rank]) + stage_off, src, nbytes);
  uint8_t* d = reinterpret_cast<uint8_t*>(dst);
  // boxes that read only this rank's own data need nothing from the peers: run
  // them before waiting for the peers' staged data (a skew between ranks then
  // overlaps the local copy)
  if (!reduce) {
    for (int i = 0; i < plan.nbox; ++i) {
      const CopyBox& b = plan.box[i];
      if (b.src_rank >= 0) continue;
      if (plan.accumulate)
        acc_copy_box(reinterpret_cast<const uint8_t*>(local), d, b, plan);
      else
        copy_box(reinterpret_cast<const uint8_t*>(local), d, b, plan.esize);
      if (plan.sequential && !grid_barrier(c, c.bar_base + nb * ++bars)) return;
    }
  }
  if (!grid_barrier(c, c.bar_base + nb * ++bars)) return;
  publish(c, kFlagStaged);
  if (!wait_peers(c, kFlagStaged, c.epoch)) return;
  for (int i = 0; i < plan.nbox; ++i) {
    const CopyBox& b = plan.box[i];
    if (!reduce && b.src_rank < 0) continue;  // done above
    if (reduce) {
      reduce_box(c, d, b, plan);
    } else {
      const uint8_t* s = b.src_rank < 0 ? reinterpret_cast<const uint8_t*>(local)
                                        : reinterpret_cast<const uint8_t*>(c.data[b.src_rank]);
      if (plan.accumulate)
        acc_copy_box(s, d, b, plan);
      else
        copy_box(s, d, b, plan.esize);
    }
    if (plan.sequential && !grid_barrier(c, c.bar_base + nb * ++bars)) return;
  }
  if (!grid_barrier(c, c.bar_base + nb * ++bars)) return;
  publish(c, kFlagDone);
}

// Vectorised sum of 8 bf16/f16 or 4 f32 values from every rank's staged copy.
template <int DT>
__device__ __forceinline__ void sum_vec(const CommDev& c, long long off_bytes, float (&acc)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  for (int p = 0; p < c.size; ++p) {
    const int src = (c.rank + p) % c.size;
    const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(c.data[src]) + off_bytes);
    if (DT == 2) {
      acc[0] += __uint_as_float(v.x);
      acc[1] += __uint_as_float(v.y);
      acc[2] += __uint_as_float(v.z);
      acc[3] += __uint_as_float(v.w);
    } else {
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (DT == 0) {
          const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[j]);
          const float2 f = __bfloat1622float2(h);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        } else {
          const __half2 h = *reinterpret_cast<const __half2*>(&w[j]);
          const float2 f = __half22float2(h);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        }
      }
    }
  }
}

template <int DT>
__device__ __forceinline__ uint4 pack_vec(const float (&acc)[8], float scale) {
  uint4 o;
  if (DT == 2) {
    o.x = __float_as_uint(acc[0] * scale);
    o.y = __float_as_uint(acc[1] * scale);
    o.z = __float_as_uint(acc[2] * scale);
    o.w = __float_as_uint(acc[3] * scale);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (DT == 0) {
        __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * j] * scale, acc[2 * j + 1] * scale);
        w[j] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(acc[2 * j] * scale, acc[2 * j + 1] * scale);
        w[j] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    o = make_uint4(w[0], w[1], w[2], w[3]);
  }
  return o;
}

// Two-shot all-reduce: stage -> each rank reduces its chunk (reads every peer) ->
// each rank pulls the other chunks.  n16 = number of 16-byte vectors (n*esize/16).
template <int DT>
__global__ void __launch_bounds__(512) k_all_reduce(CommDev c, uint4* buf, long long n16, float scale) {
  uint32_t bars = 0;
  const uint32_t nb = gridDim.x;
  const size_t bytes = (size_t)n16 * 16;
  if (!wait_peers(c, kFlagDone, c.epoch - 1)) return;
  copy_bytes(reinterpret_cast<uint8_t*>(c.data[c.rank]), buf, bytes);
  if (!grid_barrier(c, c.bar_base + nb * ++bars)) return;
  publish(c, kFlagStaged);
  if (!wait_peers(c, kFlagStaged, c.epoch)) return;
  const long long per = (n16 + c.size - 1) / c.size;
  const long long lo = min((long long)c.rank * per, n16);
  const long long hi = min(lo + per, n16);
  const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long nth = (long long)gridDim.x * blockDim.x;
  uint4* reduced = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(c.data[c.rank]) + bytes);
  for (long long i = lo + tid; i < hi; i += nth) {
    float acc[8];
    sum_vec<DT>(c, i * 16, acc);
    const uint4 o = pack_vec<DT>(acc, scale);
    buf[i] = o;
    reduced[i - lo] = o;
  }
  if (!grid_barrier(c, c.bar_base + nb * ++bars)) return;
  publish(c, kFlagReduced);
  if (!wait_peers(c, kFlagReduced, c.epoch)) return;
  for (int k = 1; k < c.size; ++k) {
    const int o = (c.rank + k) % c.size;
    const long long olo = min((long long)o * per, n16);
    const long long ohi = min(olo + per, n16);
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(c.data[o]) + bytes);
    for (long long i = olo + tid; i < ohi; i += nth) buf[i] = src[i - olo];
  }
  if (!grid_barrier(c, c.bar_base + nb * ++bars)) return;
  publish(c, kFlagDone);
}

// acc += v (8 bf16/fp16 or 4 fp32 values in one 16-byte vector)
template <int DT>
__device__ __forceinline__ void add_vec(float (&acc)[8], const uint4 v) {
  if (DT == 2) {
    acc[0] += __uint_as_float(v.x);
    acc[1] += __uint_as_float(v.y);
    acc[2] += __uint_as_float(v.z);
    acc[3] += __uint_as_float(v.w);
  } else {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f;
      if (DT == 0) {
        f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
      } else {
        f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      }
      acc[2 * j] += f.x;
      acc[2 * j + 1] += f.y;
    }
  }
}

// Push-model two-shot all-reduce: every transfer over NVLink is a store into a
// peer's symmetric region, never a load.  Region of rank q (16-byte vectors,
// per = ceil(n16 / size)): in[p] = [p * per, (p + 1) * per) receives chunk q of
// rank p's buffer; out[p] = [(size + p) * per, ...) receives rank p's reduced
// chunk p.
//   1. rank r stores chunk q of buf into rank q's in[r] (q = r is local), then
//      publishes `staged`;
//   2. after every peer's `staged`, rank r sums in[0..size) from its own HBM,
//      scales, writes buf chunk r and stores the result into every peer's
//      out[r], then publishes `reduced`;
//   3. after every peer's `reduced`, rank r copies out[q] (local) into buf
//      chunk q for q != r and publishes `done`.
// NVLink carries 2 (size - 1) / size of the buffer per rank, all as posted
// writes; no staging copy of the whole buffer.  All waits are bounded.
template <int DT>
__global__ void __launch_bounds__(512) k_all_reduce_push(CommDev c, uint4* buf, long long n16, float scale) {
  uint32_t bars = 0;
  const uint32_t nb = gridDim.x;
  const long long per = (n16 + c.size - 1) / c.size;
  const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long nth = (long long)gridDim.x * blockDim.x;
  // region pointers in shared memory: a dynamic index into the kernel parameter
  // array would go through local memory
  __shared__ uint4* s_data[kMaxRanks];
#pragma unroll
  for (int p = 0; p < kMaxRanks; ++p)
    if (threadIdx.x == p) s_data[p] = reinterpret_cast<uint4*>(c.data[p]);
  __syncthreads();
  if (!wait_peers(c, kFlagDone, c.epoch - 1)) return;  // peers no longer read our region
  for (int k = 0; k < c.size; ++k) {
    const int q = (c.rank + k) % c.size;  // every rank starts with a different target
    const long long lo = min((long long)q * per, n16);
    const long long hi = min(lo + per, n16);
    uint4* dst = s_data[q] + (long long)c.rank * per - lo;
    for (long long i = lo + tid; i < hi; i += nth) dst[i] = buf[i];
  }
  if (!grid_barrier(c, c.bar_base + nb * ++bars)) return;
  publish(c, kFlagStaged);
  if (!wait_peers(c, kFlagStaged, c.epoch)) return;
  {
    const long long lo = min((long long)c.rank * per, n16);
    const long long hi = min(lo + per, n16);
    const uint4* in = s_data[c.rank];
    for (long long i = lo + tid; i < hi; i += nth) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      for (int p = 0; p < c.size; ++p) add_vec<DT>(acc, in[(long long)p * per + (i - lo)]);
      const uint4 o = pack_vec<DT>(acc, scale);
      buf[i] = o;
      for (int k = 1; k < c.size; ++k) {
        const int q = (c.rank + k) % c.size;
        s_data[q][(long long)(c.size + c.rank) * per + (i - lo)] = o;
      }
    }
  }
  if (!grid_barrier(c, c.bar_base + nb * ++bars)) return;
  publish(c, kFlagReduced);
  if (!wait_peers(c, kFlagReduced, c.epoch)) return;
  const uint4* own = s_data[c.rank];
  for (int k = 1; k < c.size; ++k) {
    const int q = (c.rank + k) % c.size;
    const long long lo = min((long long)q * per, n16);
    const long long hi = min(lo + per, n16);
    const uint4* src = own + (long long)(c.size + q) * per - lo;
    for (long long i = lo + tid; i < hi; i += nth) buf[i] = src[i];
  }
  if (!grid_barrier(c, c.bar_base + nb * ++bars)) return;
  publish(c, kFlagDone);
}

// ------------------------------------------------------------------ host launchers

static int launch_coop(const void* fn, int nblocks, void** args, cudaStream_t stream) {
  cudaError_t e = cudaLaunchCooperativeKernel(fn, dim3(nblocks), dim3(512), args, 0, stream);
  return static_cast<int>(e);
}

int comm_stage_and_copy(const CommDev& c, const void* src, size_t nbytes, size_t stage_off, void* dst,
                        const CopyPlan& plan, int nblocks, cudaStream_t stream, const void* local) {
  CommDev cc = c;
  const void* s = src;
  size_t n = nbytes, off = stage_off;
  void* d = dst;
  CopyPlan p = plan;
  int reduce = 0;
  const void* l = local != nullptr ? local : src;
  void* args[] = {&cc, &s, &n, &off, &d, &p, &reduce, &l};
  return launch_coop(reinterpret_cast<const void*>(k_stage_and_run), nblocks, args, stream);
}

int comm_stage_and_reduce(const CommDev& c, const void* src, size_t nbytes, size_t stage_off, void* dst,
                          const CopyPlan& plan, int nblocks, cudaStream_t stream) {
  CommDev cc = c;
  const void* s = src;
  size_t n = nbytes, off = stage_off;
  void* d = dst;
  CopyPlan p = plan;
  int reduce = 1;
  const void* l = src;
  void* args[] = {&cc, &s, &n, &off, &d, &p, &reduce, &l};
  return launch_coop(reinterpret_cast<const void*>(k_stage_and_run), nblocks, args, stream);
}

int comm_all_reduce(const CommDev& c, void* buf, long long n, int dtype, float scale, int nblocks,
                    cudaStream_t stream) {
  const int esize = dtype == 2 ? 4 : 2;
  if ((n * esize) % 16 || (reinterpret_cast<uintptr_t>(buf) & 15)) return -1;
  CommDev cc = c;
  uint4* b = reinterpret_cast<uint4*>(buf);
  long long n16 = n * esize / 16;
  float sc = scale;
  void* args[] = {&cc, &b, &n16, &sc};
  const void* fn = dtype == 0 ? reinterpret_cast<const void*>(k_all_reduce<0>)
                   : dtype == 1 ? reinterpret_cast<const void*>(k_all_reduce<1>)
                                : reinterpret_cast<const void*>(k_all_reduce<2>);
  return launch_coop(fn, nblocks, args, stream);
}

// Region bytes the push all-reduce needs for n16 16-byte vectors on `size` ranks.
long long comm_all_reduce_push_bytes(long long n16, int size) {
  return 2LL * size * ((n16 + size - 1) / size) * 16;
}

int comm_all_reduce_push(const CommDev& c, void* buf, long long n, int dtype, float scale, int nblocks,
                         cudaStream_t stream) {
  const int esize = dtype == 2 ? 4 : 2;
  if ((n * esize) % 16 || (reinterpret_cast<uintptr_t>(buf) & 15)) return -1;
  CommDev cc = c;
  uint4* b = reinterpret_cast<uint4*>(buf);
  long long n16 = n * esize / 16;
  float sc = scale;
  void* args[] = {&cc, &b, &n16, &sc};
  const void* fn = dtype == 0 ? reinterpret_cast<const void*>(k_all_reduce_push<0>)
                   : dtype == 1 ? reinterpret_cast<const void*>(k_all_reduce_push<1>)
                                : reinterpret_cast<const void*>(k_all_reduce_push<2>);
  return launch_coop(fn, nblocks, args, stream);
}

}  // namespace es
