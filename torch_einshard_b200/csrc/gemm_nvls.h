// Fused GEMM + NVLS all-reduce (gemm_nvls.cu): host interface.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.h"
#include "gemm.h"

namespace es {

struct NvlsGemmJob {
  void* heap_uc = nullptr;       // this rank's heap data region (partial product, bf16 [M][N])
  void* heap_mc = nullptr;       // multicast view of the same region
  uint64_t ready_base[kMaxRanks] = {};  // each rank's ready[0][0] word (peer-mapped)
  uint32_t* reduced = nullptr;   // this rank's reduced[0] word
  uint32_t* reduced_mc = nullptr;
  int rank = 0, size = 1;
  uint32_t epoch = 1;            // this call's number on the heap (>= 1, same on every rank)
  int reducer_clusters = 4;      // CTA pairs that reduce and copy out (0: overlap mode, the GEMM's
                                 // epilogue warps reduce and copy out during later tiles' mainloops)
  int lag = 0;                   // overlap mode: tiles between a tile and its reduction (0: auto)
  int seg = 0, shard = 0;        // reduce-scatter: rows [seg i + p shard, + shard) go to rank p (seg 0: all-reduce)
  uint64_t timeout_ns = 4000000000ull;
};

// Units (32 x 256 output blocks) of an M x N product on the wide kernel's tiles.
long long gemm_nvls_units(int M, int N);
// g.C / g.ldc: the output tensor (all-reduce: every rank gets the whole sum;
// reduce-scatter: this rank's rows, [M / P][ldc]); g.err: error word.
int gemm_nvls_allreduce_launch(const GemmArgs& g, const NvlsGemmJob& job, cudaStream_t stream);

}  // namespace es
