// Native NVLink communicator: symmetric peer-mapped buffers and pull-based
// collectives for one node (up to 8 ranks, one process per GPU).
//
// Each rank owns one device allocation: [flags (kFlagBytes)][data (data_bytes)],
// a cuMem heap that peers map (symm.h).  Only *reads* cross NVLink in the collectives
// (every rank writes only its own memory), which keeps buffer reuse safe with
// three monotonic epoch flags per rank:
//   staged  - this rank's input for op e is in its data region
//   reduced - this rank's reduced chunk for op e is in its data region
//   done    - this rank finished every remote read of op e
// Before overwriting its data region for op e, a rank waits until every peer
// reports done >= e-1.  All waits are bounded (see ptx.cuh).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace es {

constexpr int kMaxRanks = 8;
constexpr size_t kFlagBytes = 8 << 20;  // 2M int32 flag slots; from word 262144 on: NVLS counters and unit flags (nvls.h)
// flag slot indices
constexpr int kFlagDone = 0;
constexpr int kFlagStaged = 1;
constexpr int kFlagReduced = 2;
constexpr int kFlagBarrier = 8;       // local grid-barrier counter
constexpr int kFlagArrive = 9;        // local completion counter
constexpr int kFlagTile0 = 1024;      // per-tile flags of fused kernels: [kFlagTile0, kFlagTile0 + 2*kMaxTiles)
constexpr int kMaxTiles = 120000;

struct CommDev {
  int rank;
  int size;
  uint64_t data[kMaxRanks];   // data region of each rank (peer-mapped)
  uint64_t flags[kMaxRanks];  // flag region of each rank (peer-mapped)
  int epoch;                  // this op's epoch (>= 1)
  uint32_t bar_base;          // value of the local barrier counter at kernel start
  uint32_t arrive_base;       // value of the local completion counter at kernel start
  int* err;
  uint64_t timeout_ns;        // bound of every wait on a peer (EINSHARD_WAIT_TIMEOUT_US)
};

// A strided box copy (or reduction) in bytes: dims[0..3] sizes (innermost last),
// strides in bytes.  src is a peer data region (src_rank >= 0) at src_off, or the
// local input pointer (src_rank == -1); dst is the local output pointer at dst_off.
struct CopyBox {
  int src_rank;
  int dims[4];
  long long src_off;
  long long dst_off;
  long long sstr[4];
  long long dstr[4];
};

constexpr int kMaxBoxes = 16;

struct CopyPlan {
  int nbox;
  int esize;          // element size in bytes
  int dtype;          // for reductions: 0 bf16, 1 f16, 2 f32
  int accumulate;     // reductions: add into dst instead of overwrite
  float scale;        // reductions: multiply the sum
  int sequential;     // run boxes one after another with a grid barrier between them
  CopyBox box[kMaxBoxes];
};

// host API (comm.cu); the buffers come from the symmetric heap (symm.h)
// Stage `nbytes` of `src` into this rank's data region at `stage_off`, publish
// it, then run `plan` (copies from peers' staged data into `dst`).  With
// nbytes == 0 nothing is staged (the plan may read regions staged earlier).
// Boxes with src_rank < 0 read from `local` (default: `src`), so a rank's own
// pieces need not pass through its region.
int comm_stage_and_copy(const CommDev& c, const void* src, size_t nbytes, size_t stage_off, void* dst,
                        const CopyPlan& plan, int nblocks, cudaStream_t stream, const void* local = nullptr);
// Same, but the plan's boxes are summed over all ranks (box src_rank ignored).
int comm_stage_and_reduce(const CommDev& c, const void* src, size_t nbytes, size_t stage_off, void* dst,
                          const CopyPlan& plan, int nblocks, cudaStream_t stream);
// Two-shot all-reduce of `n` elements in place in `buf` (dtype 0 bf16, 1 f16, 2 f32),
// result multiplied by `scale`.
// Push-model variant (every NVLink transfer a store into a peer's region);
// needs comm_all_reduce_push_bytes(n16, size) bytes of symmetric region.
long long comm_all_reduce_push_bytes(long long n16, int size);
int comm_all_reduce_push(const CommDev& c, void* buf, long long n, int dtype, float scale, int nblocks,
                         cudaStream_t stream);
int comm_all_reduce(const CommDev& c, void* buf, long long n, int dtype, float scale, int nblocks,
                    cudaStream_t stream);

}  // namespace es
