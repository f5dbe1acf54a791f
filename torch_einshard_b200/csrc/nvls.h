// NVLS collectives on a symmetric heap (symm.h): multimem.ld_reduce sums the
// same address of every rank's heap inside the NVSwitch, multimem.st writes
// one value to every rank's heap, multimem.red adds to every rank's copy of a
// flag.  One launch per collective, with no grid-wide barrier: block b of every
// rank owns chunk b of the data, and the blocks of the same index on all ranks
// synchronise only with each other through two per-block counters:
//   ready[b] - each rank adds 1 once its input for chunk b is in its heap
//   seq[b]   - each rank adds 1 once it stopped touching chunk b (reads and stores)
// For the e-th collective on a heap (every rank runs the same sequence, with
// the same block count), block b waits for seq[b] >= P (e - 1) before writing
// into its chunk and for ready[b] >= P e before reading peers' copies.  Every
// wait is bounded; on expiry the block records an error code and returns.
//
// Layout of a rank's heap: [flag words (kFlagBytes)][data].  The NVLS words
// live in the upper half of the flag area (comm.h keeps the lower half).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.h"

namespace es {

constexpr int kNvlsReady = 262144;                 // word index: per-block ready counters
constexpr int kNvlsSeq = kNvlsReady + 1024;        // per-block completion counters
constexpr int kNvlsMaxBlocks = 1024;
constexpr int kNvlsDone = kNvlsSeq + kNvlsMaxBlocks;  // collectives every rank has finished, x P (multicast adds)
constexpr int kNvlsArrived = kNvlsDone + 1;          // this rank's blocks that finished a collective (local)
// Fused GEMM + all-reduce (gemm_nvls.cu), per 32 x 256 output unit u:
//   reduced[u]       - the epoch of the last call whose unit u is reduced (written by its owner, multicast)
//   ready[u][q]      - on the owner of u: the epoch of rank q's last partial of unit u
constexpr int kNvlsMaxUnits = 120000;
constexpr int kTileReduced0 = 270336;                              // word index of reduced[0]
constexpr int kTileReady0 = 393216;                                // word index of ready[0][0]
static_assert(kNvlsArrived + 1 <= kTileReduced0, "NVLS counters overlap the unit flags");
static_assert(kTileReduced0 + kNvlsMaxUnits <= kTileReady0, "unit flags overlap");
static_assert(kTileReady0 + kNvlsMaxUnits * kMaxRanks <= static_cast<int>(kFlagBytes / 4),
              "NVLS flags exceed the flag area");

struct NvlsDev {
  uint8_t* uc;        // this rank's data region
  uint8_t* mc;        // multicast view of the data region (same offsets on every rank)
  uint32_t* flags;    // this rank's flag words
  uint32_t* mcflags;  // multicast view of the flag words
  int rank, size;
  int epoch;          // this collective's sequence number on the heap (>= 1)
  int nblocks;        // the heap's fixed block count (every collective launches exactly this many)
  int* err;
  uint64_t timeout_ns;
};

// A shard layout for all-gather / reduce-scatter along one dimension of a
// tensor viewed as [outer, S, inner] (bytes: inner_bytes = inner * esize).
// Shard q covers rows [off[q], off[q] + len[q]) of S; in the heap it is stored
// densely as [outer, len[q], inner] at byte offset region[q] (16-byte aligned).
struct ShardLayout {
  long long outer;
  long long inner_bytes;
  long long total_rows;            // S
  long long off[kMaxRanks + 1];
  long long len[kMaxRanks];
  long long region[kMaxRanks];
};

// dtype: 0 bf16, 1 f16, 2 f32.  Return 0 or a cudaError_t.
// All-reduce of nbytes (multiple of 16 after the heap's padding, see nvls.cu):
// `in` is copied into the heap (nullptr: the data is already at offset 0 of
// the heap), `out` receives the sum times `scale` (nullptr: two-shot leaves it
// in the heap at offset 0).  two_shot: each rank reduces 1/P and multicasts it;
// otherwise every rank reduces everything for itself.
int nvls_all_reduce(const NvlsDev& d, const void* in, void* out, long long nbytes, int dtype, float scale,
                    int two_shot, cudaStream_t stream);
// out (viewed [outer, S, inner]) <- every rank's shard; `in` is this rank's
// dense shard [outer, len[rank], inner].
int nvls_all_gather(const NvlsDev& d, const void* in, void* out, const ShardLayout& L, cudaStream_t stream);
// out (dense [outer, len[rank], inner]) <- scale * sum over ranks of rows
// [off[rank], off[rank] + len[rank]) of `in` (viewed [outer, S, inner]).
int nvls_reduce_scatter(const NvlsDev& d, const void* in, void* out, const ShardLayout& L, int dtype, float scale,
                        cudaStream_t stream);

// Stream-ordered wait until every rank completed the NVLS collectives issued so
// far on the heap (d.epoch = the last one's number).
int nvls_quiesce(const NvlsDev& d, cudaStream_t stream);

}  // namespace es
