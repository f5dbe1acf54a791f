// GEMM fused with an NVLink all-reduce of its output (see gemm_ar.cu).
#pragma once

#include <vector>

#include "comm.h"
#include "gemm.h"

namespace es {

// Number of CTAs the fused kernel launches for this problem (the completion
// counter of the communicator advances by this much).
inline int gemm_allreduce_grid(const GemmArgs& g) {
  const int tiles = ((g.M + 127) / 128) * ((g.N + 255) / 256);
  return tiles < g.num_sms ? tiles : g.num_sms;
}

// rs_seg > 0 selects reduce-scatter: rows form segments of rs_seg rows, rank p
// keeps rows [p * rs_shard, (p + 1) * rs_shard) of every segment in its C.
int gemm_allreduce_launch(const GemmArgs& g, const CommDev& comm, cudaStream_t stream, long long rs_seg = 0,
                          long long rs_shard = 0);

// All-gather -> GEMM (gemm_ag.cu): g describes the GEMM over the gathered rows
// (A = xfull, M = segments * P * shard); this rank's shard must already be in its
// symmetric region as [segments][shard][K].
int gemm_allgather_grid(const GemmArgs& g);
// Row origin (multiple of 256) of the gathered A that the i-th 256-row block of
// the schedule reads on `rank`: this rank's shard first, then rank + 1, ...
// (host walk of the kernel's mapping, for tests).
std::vector<int> gemm_allgather_row_order(int rank, int size, int segments, long long shard);
int gemm_allgather_launch(const GemmArgs& g, const CommDev& comm, void* xfull, int segments, long long shard,
                          cudaStream_t stream);

// Push-model fused GEMM + all-reduce on the wide kernel (gemm_push.cu).
long long gemm_push_region_bytes(const GemmArgs& g, int size);
int gemm_push_grid(const GemmArgs& g);
int gemm_push_allreduce_launch(const GemmArgs& g, const CommDev& comm, cudaStream_t stream);

}  // namespace es
